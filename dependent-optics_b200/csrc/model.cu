// model.cu — the whole-model lens of the crate: mixtral::forward_backward
// (src/mixtral.rs:245-261): embed -> L blocks -> final RMSNorm -> LM head ->
// mean next-token cross-entropy, and its adjoint of every parameter.
//
// The blocks are the block lenses of block.cu (one handle, hence one
// residual, per layer); the embedding, LM head and loss kernels are here.
// The embedding adjoint is a deterministic gather: one CTA per vocabulary row
// walks the tokens in order and sums the rows whose token is that id.
#include <memory>
#include <vector>

#include "block.cuh"

namespace dop {

namespace {

// x[t] = table[tokens[t]] (embed, src/mixtral.rs:600-606)
template <typename T>
__global__ void k_embed(const T* __restrict__ table, const int64_t* __restrict__ tokens, int D,
                        float* __restrict__ x) {
  const int64_t t = blockIdx.x;
  const int64_t id = tokens[t];
  for (int i = threadIdx.x; i < D; i += blockDim.x) x[t * D + i] = ld(&table[id * D + i]);
}

// dtable[v] += sum_{t: tokens[t] == v} dx[t], tokens in order
// (embed_bwd, src/mixtral.rs:608-614)
__global__ void k_embed_bwd(const int64_t* __restrict__ tokens, int64_t T, int D,
                            const float* __restrict__ dx, float* __restrict__ dtable) {
  const int64_t v = blockIdx.x;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float acc = dtable[v * D + i];
    for (int64_t t = 0; t < T; ++t)
      if (tokens[t] == v) acc += dx[t * D + i];
    dtable[v * D + i] = acc;
  }
}

// cross_entropy (src/mixtral.rs:966-991), one CTA per token row:
// row_loss[t] = lse - logit[target]; d = (softmax - onehot) / n.
__global__ void k_cross_entropy(const float* __restrict__ logits, const int64_t* __restrict__ tgt,
                                int64_t n, int V, float* __restrict__ row_loss,
                                float* __restrict__ dlogits) {
  const int64_t t = blockIdx.x;
  const float* row = logits + t * V;
  __shared__ float red[32];
  __shared__ float bc;
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) m = fmaxf(m, row[v]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = -INFINITY;
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) mm = fmaxf(mm, red[q]);
    bc = mm;
  }
  __syncthreads();
  m = bc;
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) s += expf(row[v] - m);
  s = warp_sum(s);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float ss = 0.f;
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) ss += red[q];
    bc = ss;
  }
  __syncthreads();
  const float sum = bc;
  const int64_t target = tgt[t];
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    float d = (expf(row[v] - m) / sum) / (float)n;
    if (v == target) d -= 1.0f / (float)n;
    dlogits[t * V + v] = d;
  }
  if (threadIdx.x == 0) row_loss[t] = m + logf(sum) - row[target];
}

// loss = sum_t row_loss[t] / n, in token order (one thread: deterministic).
__global__ void k_mean_loss(const float* __restrict__ row_loss, int64_t n, float* __restrict__ loss) {
  if (threadIdx.x != 0) return;
  float s = 0.f;
  for (int64_t t = 0; t < n; ++t) s += row_loss[t];
  *loss = s / (float)n;
}

}  // namespace

// One model: L block handles and the head's buffers.
struct Model {
  dop_mixtral_cfg cfg{};
  int64_t B, S, T;
  int prec;
  LayerOffsets off{};
  int64_t embed = 0, layer0 = 0, final_norm = 0, lm_head = 0, total = 0;
  std::vector<std::unique_ptr<Block>> blocks;
  float *x = nullptr, *h_inv = nullptr, *logits = nullptr, *dlogits = nullptr, *row_loss = nullptr;
  float *dh = nullptr, *part = nullptr;
  void *h_act = nullptr, *dlogits_act = nullptr;
  std::vector<float*> acts;  // inputs of each layer (acts[l]) and the final output
  int64_t part_cap = 0;
  int64_t launches = 0;
  std::vector<void*> owned;

  void* alloc(size_t bytes) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, std::max<size_t>(bytes, 16));
    if (e != cudaSuccess) throw Error(DOP_E_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
    owned.push_back(p);
    return p;
  }

  Model(const dop_mixtral_cfg& c, int64_t batch, int64_t seq, int precision)
      : cfg(c), B(batch), S(seq), T(batch * seq), prec(precision) {
    DOP_REQUIRE(c.layers >= 1 && c.vocab >= 1, "the model needs layers >= 1 and vocab >= 1");
    DOP_REQUIRE(precision == DOP_F32 || c.vocab % 8 == 0, "the bf16 model needs vocab % 8 == 0");
    off = layer_offsets(c);
    const int64_t D = c.dim, V = c.vocab;
    embed = 0;
    layer0 = V * D;
    final_norm = layer0 + c.layers * off.total;
    lm_head = final_norm + D;
    total = lm_head + D * V;
    for (int64_t l = 0; l < c.layers; ++l) blocks.emplace_back(new Block(c, batch, seq, precision));
    const size_t a = precision == DOP_F32 ? 4 : 2;
    for (int64_t l = 0; l <= c.layers; ++l) acts.push_back((float*)alloc(4 * T * D));
    h_inv = (float*)alloc(4 * T);
    h_act = alloc(a * T * D);
    logits = (float*)alloc(4 * T * V);
    dlogits = (float*)alloc(4 * T * V);
    dlogits_act = alloc(a * T * V);
    row_loss = (float*)alloc(4 * T);
    dh = (float*)alloc(4 * T * D);
    x = (float*)alloc(4 * T * D);
    part_cap = 64 * D;
    part = (float*)alloc(4 * part_cap);
  }
  ~Model() {
    for (void* p : owned) cudaFree(p);
  }

  template <typename Act>
  void run(const Act* P, const int64_t* tokens, const int64_t* targets, float* loss, float* dP,
           float* logits_out, cudaStream_t s) {
    const int64_t D = cfg.dim, V = cfg.vocab, L = cfg.layers;
    const bool f32 = std::is_same<Act, float>::value;
    DOP_CHECK_CUDA(cudaMemsetAsync(dP, 0, sizeof(float) * total, s));  // a fresh adjoint
    k_embed<Act><<<(unsigned)T, 256, 0, s>>>(P + embed, tokens, (int)D, acts[0]);
    DOP_LAUNCHED(launches);
    for (int64_t l = 0; l < L; ++l)
      blocks[l]->forward(P + layer0 + l * off.total, acts[l], acts[l + 1], s);
    // final norm and LM head (src/mixtral.rs:279-280)
    rmsnorm_fwd<Act>(acts[L], P + final_norm, T, (int)D, cfg.rms_eps, (Act*)h_act, h_inv, nullptr,
                     s, launches);
    Gemm gh; gh.M = T; gh.N = V; gh.K = D; gh.A = h_act; gh.lda = D; gh.B = P + lm_head;
    gh.ldb = V; gh.C = logits; gh.ldc = V;
    gemm(gh, s);
    k_cross_entropy<<<(unsigned)T, 256, 0, s>>>(logits, targets, T, (int)V, row_loss, dlogits);
    DOP_LAUNCHED(launches);
    k_mean_loss<<<1, 32, 0, s>>>(row_loss, T, loss);
    DOP_LAUNCHED(launches);
    if (logits_out)
      DOP_CHECK_CUDA(cudaMemcpyAsync(logits_out, logits, sizeof(float) * T * V,
                                     cudaMemcpyDeviceToDevice, s));
    // backward (src/mixtral.rs:382-432)
    const void* dl_op = dlogits;
    if (!f32) {
      convert<Act>(dlogits, (Act*)dlogits_act, T * V, s, launches);
      dl_op = dlogits_act;
    }
    Gemm gd; gd.M = T; gd.N = D; gd.K = V; gd.A = dl_op; gd.lda = V; gd.B = P + lm_head;
    gd.ldb = V; gd.b_t = true; gd.C = dh; gd.ldc = D;
    gemm(gd, s);
    Gemm gw; gw.M = D; gw.N = V; gw.K = T; gw.A = h_act; gw.lda = D; gw.a_t = true; gw.B = dl_op;
    gw.ldb = V; gw.C = dP + lm_head; gw.ldc = V; gw.epi = Epi::Accum;
    gemm(gw, s);
    rmsnorm_bwd<Act>(dh, acts[L], h_inv, P + final_norm, nullptr, T, (int)D, x, (Act*)nullptr,
                     dP + final_norm, part, part_cap, s, launches);
    float* cur = x;
    float* nxt = dh;
    for (int64_t l = L - 1; l >= 0; --l) {
      blocks[l]->backward(P + layer0 + l * off.total, cur, nxt, dP + layer0 + l * off.total, s);
      std::swap(cur, nxt);
    }
    k_embed_bwd<<<(unsigned)V, 256, 0, s>>>(tokens, T, (int)D, cur, dP + embed);
    DOP_LAUNCHED(launches);
  }

  void gemm(const Gemm& g, cudaStream_t s) {
    if (prec == DOP_BF16) gemm_tc(g, nullptr, 0, TcEpilogue{}, s, launches);
    else gemm_simt<float>(g, s, launches);
  }
};

}  // namespace dop

namespace dop {
int set_last_error(int code, const char* msg);
}

#define DOP_MODEL_GUARD(body)                                  \
  try {                                                        \
    body;                                                      \
    return DOP_OK;                                             \
  } catch (const dop::Error& e) {                              \
    return dop::set_last_error(e.code, e.what());              \
  } catch (const std::bad_alloc&) {                            \
    return dop::set_last_error(DOP_E_NOMEM, "host allocation failed"); \
  } catch (const std::exception& e) {                          \
    return dop::set_last_error(DOP_E_INVALID, e.what());       \
  }

extern "C" {

int dop_model_create(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq, int precision,
                     dop_model** out) {
  DOP_MODEL_GUARD({
    DOP_REQUIRE(cfg && out, "null pointer");
    *out = reinterpret_cast<dop_model*>(new dop::Model(*cfg, batch, seq, precision));
  })
}

int dop_model_destroy(dop_model* m) {
  DOP_MODEL_GUARD({ delete reinterpret_cast<dop::Model*>(m); })
}

int dop_model_forward_backward(dop_model* m_, const void* params, const int64_t* tokens,
                               const int64_t* targets, float* loss, float* dparams,
                               float* logits, void* stream) {
  DOP_MODEL_GUARD({
    DOP_REQUIRE(m_ && params && tokens && targets && loss && dparams, "null pointer");
    auto* m = reinterpret_cast<dop::Model*>(m_);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (m->prec == DOP_F32)
      m->run<float>((const float*)params, tokens, targets, loss, dparams, logits, s);
    else
      m->run<dop::bf16>((const dop::bf16*)params, tokens, targets, loss, dparams, logits, s);
  })
}

int64_t dop_model_parameter_count(const dop_model* m) {
  return m ? reinterpret_cast<const dop::Model*>(m)->total : -1;
}

}  // extern "C"
