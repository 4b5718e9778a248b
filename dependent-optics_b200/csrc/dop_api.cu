// dop_api.cu — the C ABI of libdop (include/dop.h): status codes, the block
// lens handles, lens composition, kernel.rs programs and utilities.
//
// No exception crosses the ABI: every entry point catches dop::Error (and any
// std::exception), records the message for dop_last_error() on the calling
// thread, and returns the status code.
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "block.cuh"

namespace {
thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return DOP_OK;
  } catch (const dop::Error& e) {
    g_last_error = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return DOP_E_NOMEM;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return DOP_E_INVALID;
  }
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
}  // namespace

namespace dop {
// Record the calling thread's error message (for entry points defined in
// other translation units) and return its status code.
int set_last_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

int sm_count() {
  static int cached[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}
}  // namespace dop

// ------------------------------------------------------------------- lenses
struct dop_lens {
  virtual ~dop_lens() = default;
  virtual void forward(const float* x, float* y, cudaStream_t s) = 0;
  virtual void backward(const float* dy, float* dx, cudaStream_t s) = 0;
  int64_t in_len = 0, out_len = 0;
};

namespace {
struct BlockLens : dop_lens {
  dop::Block* blk;
  const void* params;
  float* dparams;
  BlockLens(dop::Block* b, const void* p, float* dp) : blk(b), params(p), dparams(dp) {
    in_len = out_len = b->T * b->cfg.dim;
  }
  void forward(const float* x, float* y, cudaStream_t s) override { blk->forward(params, x, y, s); }
  void backward(const float* dy, float* dx, cudaStream_t s) override {
    blk->backward(params, dy, dx, dparams, s);
  }
};

// compose(g, f) = g after f (src/dlens.rs:74-113): get = get_g . get_f,
// put(x, z') = put_f(x, put_g(get_f x, z')).  The intermediate activation
// and its cotangent live in the composite.
struct ComposedLens : dop_lens {
  dop_lens* g;
  dop_lens* f;
  float* mid = nullptr;
  float* dmid = nullptr;
  ComposedLens(dop_lens* g_, dop_lens* f_) : g(g_), f(f_) {
    DOP_REQUIRE(g->in_len == f->out_len, "compose(g, f): g's input length != f's output length");
    in_len = f->in_len;
    out_len = g->out_len;
    DOP_CHECK_CUDA(cudaMalloc(&mid, sizeof(float) * f->out_len));
    DOP_CHECK_CUDA(cudaMalloc(&dmid, sizeof(float) * f->out_len));
  }
  ~ComposedLens() override {
    if (mid) cudaFree(mid);
    if (dmid) cudaFree(dmid);
  }
  void forward(const float* x, float* y, cudaStream_t s) override {
    f->forward(x, mid, s);
    g->forward(mid, y, s);
  }
  void backward(const float* dy, float* dx, cudaStream_t s) override {
    g->backward(dy, dmid, s);
    f->backward(dmid, dx, s);
  }
};
}  // namespace

// ------------------------------------------------------------- programs
// kernel.rs programs (src/kernel.rs:27-447) on the device.
struct dop_program {
  std::vector<dop_stage> stages;
  int64_t input_len, output_len, param_len, tape_f32, tape_u8;
  int64_t act_cap = 0;
  float* tape = nullptr;
  uint8_t* mask = nullptr;
  float* buf[4] = {nullptr, nullptr, nullptr, nullptr};
  float* dbuf[2] = {nullptr, nullptr};
  // per attention stage: its output and log-sum-exp (the device residual)
  std::vector<float*> attn_out, attn_lse;
  float *delta = nullptr, *dq = nullptr, *dk = nullptr, *dv = nullptr, *part = nullptr;
  int64_t part_cap = 0;
  int64_t launches = 0;
  bool have_tape = false;
  // per stage: the skip cotangent an Add stage carries back to its source
  // (nullptr for other stages), and dy = 1 for the sum loss; allocated at
  // creation so that forward and backward only enqueue work on the stream
  std::vector<float*> side_buf;
  float* ones = nullptr;
  float* split_ws = nullptr;  // split-contraction partials of the CUDA-core GEMM
  int64_t split_cap = 0;
  std::vector<float*> owned;

  float* alloc(int64_t n) {
    float* p = nullptr;
    DOP_CHECK_CUDA(cudaMalloc(&p, sizeof(float) * std::max<int64_t>(n, 1)));
    owned.push_back(p);
    return p;
  }
  ~dop_program() {
    for (float* p : owned) cudaFree(p);
    if (mask) cudaFree(mask);
  }
};

namespace {
using dop::ceil_div;

void program_forward(dop_program* p, const float* x, const float* params, float* y,
                     cudaStream_t s) {
  float* cur = p->buf[0];
  DOP_CHECK_CUDA(cudaMemcpyAsync(cur, x, sizeof(float) * p->input_len, cudaMemcpyDeviceToDevice, s));
  int which = 0, ai = 0;
  for (const dop_stage& st : p->stages) {
    float* nxt = p->buf[(which + 1) % 2];
    if (st.kind == DOP_STAGE_GEMM) {
      DOP_CHECK_CUDA(cudaMemcpyAsync(p->tape + st.save_at, cur, sizeof(float) * st.batch * st.din,
                                     cudaMemcpyDeviceToDevice, s));
      dop::Gemm g;
      g.M = st.batch; g.N = st.dout; g.K = st.din;
      g.A = cur; g.lda = st.din;
      g.B = params + st.param_at; g.ldb = st.dout;
      g.C = nxt; g.ldc = st.dout;
      g.epi = dop::Epi::BiasRelu;
      g.bias = params + st.param_at + st.din * st.dout;
      g.relu = st.relu != 0;
      g.mask = st.relu ? p->mask + st.mask_at : nullptr;
      g.ws = p->split_ws; g.ws_cap = p->split_cap;
      dop::gemm_simt<float>(g, s, p->launches);
      which = (which + 1) % 2;
      cur = nxt;
    } else if (st.kind == DOP_STAGE_ATTENTION) {
      int64_t n = st.batch * st.tokens * st.dim;
      DOP_CHECK_CUDA(cudaMemcpyAsync(p->tape + st.x_at, cur, sizeof(float) * n,
                                     cudaMemcpyDeviceToDevice, s));
      dop::Attn a;
      a.B = st.batch; a.S = st.tokens; a.H = 1; a.KV = 1; a.hd = (int)st.dim;
      a.window = st.tokens; a.causal = false; a.scale = 1.0f / sqrtf((float)st.dim);
      dop::attn_fwd_simt<float>(a, cur, cur, cur, p->attn_out[ai], p->attn_lse[ai], s,
                                p->launches);
      DOP_CHECK_CUDA(cudaMemcpyAsync(nxt, p->attn_out[ai], sizeof(float) * n,
                                     cudaMemcpyDeviceToDevice, s));
      ++ai;
      which = (which + 1) % 2;
      cur = nxt;
    } else {
      dop::add_inplace(cur, p->tape + st.from, st.len, s, p->launches);
    }
  }
  DOP_CHECK_CUDA(cudaMemcpyAsync(y, cur, sizeof(float) * p->output_len, cudaMemcpyDeviceToDevice, s));
  p->have_tape = true;
}

void program_backward(dop_program* p, const float* params, const float* dy, float* dx,
                      float* dparams, cudaStream_t s) {
  if (!p->have_tape) throw dop::Error(DOP_E_STATE, "backward called before forward");
  float* cur = p->dbuf[0];
  // sum loss when dy is null: dy = 1 (src/kernel.rs:237)
  DOP_CHECK_CUDA(cudaMemcpyAsync(cur, dy ? dy : p->ones, sizeof(float) * p->output_len,
                                 cudaMemcpyDeviceToDevice, s));
  struct Side { int64_t at; float* buf; int64_t len; };
  std::vector<Side> side;
  auto add_side = [&](int64_t at, float* d, int64_t len) {  // src/kernel.rs:376-388
    for (size_t i = 0; i < side.size();) {
      if (side[i].at == at) {
        dop::add_inplace(d, side[i].buf, std::min(len, side[i].len), s, p->launches);
        side.erase(side.begin() + i);
      } else {
        ++i;
      }
    }
  };
  int which = 0;
  int ai = (int)p->attn_out.size();
  for (size_t si = p->stages.size(); si-- > 0;) {
    const dop_stage& st = p->stages[si];
    float* nxt = p->dbuf[(which + 1) % 2];
    if (st.kind == DOP_STAGE_ADD) {
      float* b = p->side_buf[si];
      DOP_CHECK_CUDA(cudaMemcpyAsync(b, cur, sizeof(float) * st.len, cudaMemcpyDeviceToDevice, s));
      side.push_back({st.from, b, st.len});
    } else if (st.kind == DOP_STAGE_GEMM) {
      if (st.relu) dop::relu_mask_bwd(cur, p->mask + st.mask_at, st.batch * st.dout, s, p->launches);
      const float* xs = p->tape + st.save_at;
      dop::Gemm gx;  // dx = dy W^T
      gx.M = st.batch; gx.N = st.din; gx.K = st.dout;
      gx.A = cur; gx.lda = st.dout;
      gx.B = params + st.param_at; gx.ldb = st.dout; gx.b_t = true;
      gx.C = nxt; gx.ldc = st.din;
      gx.ws = p->split_ws; gx.ws_cap = p->split_cap;
      dop::gemm_simt<float>(gx, s, p->launches);
      dop::Gemm gw;  // dW = x^T dy (assigned, src/kernel.rs:342)
      gw.M = st.din; gw.N = st.dout; gw.K = st.batch;
      gw.A = xs; gw.lda = st.din; gw.a_t = true;
      gw.B = cur; gw.ldb = st.dout;
      gw.C = dparams + st.param_at; gw.ldc = st.dout;
      gw.ws = p->split_ws; gw.ws_cap = p->split_cap;
      dop::gemm_simt<float>(gw, s, p->launches);
      // db = sum_m dy (assigned, src/kernel.rs:345-351)
      dop::col_sum(cur, st.batch, st.dout, dparams + st.param_at + st.din * st.dout, p->part,
                   p->part_cap, false, s, p->launches);
      add_side(st.save_at, nxt, st.batch * st.din);
      which = (which + 1) % 2;
      cur = nxt;
    } else {
      --ai;
      int64_t n = st.batch * st.tokens * st.dim;
      const float* xs = p->tape + st.x_at;
      dop::Attn a;
      a.B = st.batch; a.S = st.tokens; a.H = 1; a.KV = 1; a.hd = (int)st.dim;
      a.window = st.tokens; a.causal = false; a.scale = 1.0f / sqrtf((float)st.dim);
      dop::attn_bwd_simt<float>(a, xs, xs, xs, p->attn_out[ai], cur, p->attn_lse[ai], p->delta,
                                p->dq, p->dk, p->dv, s, p->launches);
      // dx = dV + dQ + dK (src/kernel.rs:442-446)
      DOP_CHECK_CUDA(cudaMemcpyAsync(nxt, p->dv, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
      dop::add_inplace(nxt, p->dq, n, s, p->launches);
      dop::add_inplace(nxt, p->dk, n, s, p->launches);
      add_side(st.x_at, nxt, n);
      which = (which + 1) % 2;
      cur = nxt;
    }
  }
  if (!side.empty()) throw dop::Error(DOP_E_STATE, "skip cotangent had no saved activation");
  DOP_CHECK_CUDA(cudaMemcpyAsync(dx, cur, sizeof(float) * p->input_len, cudaMemcpyDeviceToDevice, s));
}
}  // namespace

// ------------------------------------------------------------------ C ABI
extern "C" {

const char* dop_last_error(void) { return g_last_error.c_str(); }
const char* dop_version(void) { return "dop-b200 0.1 (sm_100a)"; }

int dop_layer_layout_of(const dop_mixtral_cfg* cfg, dop_layer_layout* out) {
  return guarded([&] {
    DOP_REQUIRE(cfg && out, "null pointer");
    dop::LayerOffsets o = dop::layer_offsets(*cfg);
    out->attn_norm = o.attn_norm; out->q = o.q; out->k = o.k; out->v = o.v; out->o = o.o;
    out->ffn_norm = o.ffn_norm; out->router = o.router; out->gate0 = o.gate0; out->up0 = o.up0;
    out->down0 = o.down0; out->expert_stride = o.expert_stride; out->total = o.total;
  });
}

int64_t dop_parameter_count(const dop_mixtral_cfg* c) {
  if (!c) return -1;
  dop::LayerOffsets o = dop::layer_offsets(*c);
  return c->vocab * c->dim + c->layers * o.total + c->dim + c->dim * c->vocab;
}

int dop_block_create(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq, int precision,
                     dop_block** out) {
  return guarded([&] {
    DOP_REQUIRE(cfg && out, "null pointer");
    *out = reinterpret_cast<dop_block*>(new dop::Block(*cfg, batch, seq, precision));
  });
}

int dop_block_create_ep(const dop_mixtral_cfg* cfg, int64_t batch, int64_t seq, int precision,
                        int rank, int world, dop_block** out) {
  return guarded([&] {
    DOP_REQUIRE(cfg && out, "null pointer");
    DOP_REQUIRE(world >= 2, "an expert-parallel block needs world >= 2");
    *out = reinterpret_cast<dop_block*>(new dop::Block(*cfg, batch, seq, precision, rank, world));
  });
}

int dop_block_ep_handle(const dop_block* blk, void* handle) {
  return guarded([&] {
    DOP_REQUIRE(blk && handle, "null pointer");
    auto* b = reinterpret_cast<const dop::Block*>(blk);
    DOP_REQUIRE(b->ep_world > 1, "not an expert-parallel block");
    static_assert(sizeof(cudaIpcMemHandle_t) == DOP_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    DOP_CHECK_CUDA(cudaIpcGetMemHandle(&h, b->base));
    std::memcpy(handle, &h, sizeof(h));
  });
}

int dop_block_ep_connect(dop_block* blk, const void* handles) {
  return guarded([&] {
    DOP_REQUIRE(blk && handles, "null pointer");
    auto* b = reinterpret_cast<dop::Block*>(blk);
    DOP_REQUIRE(b->ep_world > 1, "not an expert-parallel block");
    std::vector<cudaIpcMemHandle_t> hs(b->ep_world);
    std::memcpy(hs.data(), handles, sizeof(cudaIpcMemHandle_t) * b->ep_world);
    b->ep_connect(hs.data());
  });
}

int dop_block_destroy(dop_block* blk) {
  return guarded([&] { delete reinterpret_cast<dop::Block*>(blk); });
}

int dop_block_set_router_bias(dop_block* blk, const float* bias) {
  return guarded([&] {
    DOP_REQUIRE(blk, "null block");
    reinterpret_cast<dop::Block*>(blk)->router_bias = bias;
  });
}

int dop_block_forward(dop_block* blk, const void* params, const float* x, float* y, void* s) {
  return guarded([&] {
    DOP_REQUIRE(blk, "null block");
    reinterpret_cast<dop::Block*>(blk)->forward(params, x, y, as_stream(s));
  });
}

int dop_block_backward(dop_block* blk, const void* params, const float* dy, float* dx,
                       float* dparams, void* s) {
  return guarded([&] {
    DOP_REQUIRE(blk, "null block");
    reinterpret_cast<dop::Block*>(blk)->backward(params, dy, dx, dparams, as_stream(s));
  });
}

int64_t dop_block_workspace_bytes(const dop_block* blk) {
  return blk ? (int64_t)reinterpret_cast<const dop::Block*>(blk)->bytes : -1;
}

int64_t dop_block_launches(const dop_block* blk) {
  return blk ? reinterpret_cast<const dop::Block*>(blk)->launches : -1;
}

int dop_block_set_adjoint_stream(dop_block* blk, void* stream) {
  return guarded([&] {
    DOP_REQUIRE(blk, "null block");
    reinterpret_cast<dop::Block*>(blk)->adjoint_stream = as_stream(stream);
  });
}

int dop_block_set_timing(dop_block* blk, int on) {
  return guarded([&] {
    DOP_REQUIRE(blk, "null block");
    reinterpret_cast<dop::Block*>(blk)->timing = on != 0;
  });
}

int dop_block_phase_count(const dop_block* blk) {
  return blk ? (int)reinterpret_cast<const dop::Block*>(blk)->n_phases : -1;
}

int dop_block_phase(const dop_block* blk_, int i, const char** name, float* ms) {
  return guarded([&] {
    DOP_REQUIRE(blk_ && name && ms, "null pointer");
    auto* b = reinterpret_cast<const dop::Block*>(blk_);
    DOP_REQUIRE(i >= 0 && (size_t)i < b->n_phases, "phase index out of range");
    const auto& p = b->phases[i];
    DOP_CHECK_CUDA(cudaEventSynchronize(p.b));
    DOP_CHECK_CUDA(cudaEventElapsedTime(ms, p.a, p.b));
    *name = p.name;
  });
}

int64_t dop_block_permuted_rows(const dop_block* blk) {
  return blk ? reinterpret_cast<const dop::Block*>(blk)->rows_cap : -1;
}

int dop_block_routing(const dop_block* blk_, int32_t* top_i, float* top_w, float* top_p,
                      float* router_probs, void* s) {
  return guarded([&] {
    DOP_REQUIRE(blk_, "null block");
    auto* b = reinterpret_cast<const dop::Block*>(blk_);
    if (!b->have_tape) throw dop::Error(DOP_E_STATE, "no forward has run");
    cudaStream_t st = as_stream(s);
    int64_t tk = b->T * b->cfg.top_k;
    if (top_i) DOP_CHECK_CUDA(cudaMemcpyAsync(top_i, b->top_i, 4 * tk, cudaMemcpyDeviceToDevice, st));
    if (top_w) DOP_CHECK_CUDA(cudaMemcpyAsync(top_w, b->top_w, 4 * tk, cudaMemcpyDeviceToDevice, st));
    if (top_p) DOP_CHECK_CUDA(cudaMemcpyAsync(top_p, b->top_p, 4 * tk, cudaMemcpyDeviceToDevice, st));
    if (router_probs)
      DOP_CHECK_CUDA(cudaMemcpyAsync(router_probs, b->probs, 4 * b->T * b->cfg.experts,
                                     cudaMemcpyDeviceToDevice, st));
  });
}

int dop_block_ffn_input(const dop_block* blk_, float* mid, void* s) {
  return guarded([&] {
    DOP_REQUIRE(blk_ && mid, "null block or buffer");
    auto* b = reinterpret_cast<const dop::Block*>(blk_);
    if (!b->have_tape) throw dop::Error(DOP_E_STATE, "no forward has run");
    DOP_CHECK_CUDA(cudaMemcpyAsync(mid, b->mid, 4 * b->T * b->cfg.dim, cudaMemcpyDeviceToDevice,
                                   as_stream(s)));
  });
}

int dop_block_permutation(const dop_block* blk_, int32_t* slot_row, int32_t* seg_off,
                          int32_t* row_token, void* s) {
  return guarded([&] {
    DOP_REQUIRE(blk_, "null block");
    auto* b = reinterpret_cast<const dop::Block*>(blk_);
    if (!b->have_tape) throw dop::Error(DOP_E_STATE, "no forward has run");
    cudaStream_t st = as_stream(s);
    if (slot_row)
      DOP_CHECK_CUDA(cudaMemcpyAsync(slot_row, b->slot_row, 4 * b->T * b->cfg.top_k,
                                     cudaMemcpyDeviceToDevice, st));
    if (seg_off)
      DOP_CHECK_CUDA(cudaMemcpyAsync(seg_off, b->seg_off, 4 * (b->cfg.experts + 1),
                                     cudaMemcpyDeviceToDevice, st));
    if (row_token)
      DOP_CHECK_CUDA(cudaMemcpyAsync(row_token, b->row_token, 4 * b->rows_cap,
                                     cudaMemcpyDeviceToDevice, st));
  });
}

int dop_lens_from_block(dop_block* blk, const void* params, float* dparams, dop_lens** out) {
  return guarded([&] {
    DOP_REQUIRE(blk && params && dparams && out, "null pointer");
    *out = new BlockLens(reinterpret_cast<dop::Block*>(blk), params, dparams);
  });
}

int dop_compose(dop_lens* g, dop_lens* f, dop_lens** out) {
  return guarded([&] {
    DOP_REQUIRE(g && f && out, "null pointer");
    *out = new ComposedLens(g, f);
  });
}

int dop_lens_forward(dop_lens* l, const float* x, float* y, void* s) {
  return guarded([&] {
    DOP_REQUIRE(l && x && y, "null pointer");
    l->forward(x, y, as_stream(s));
  });
}

int dop_lens_backward(dop_lens* l, const float* dy, float* dx, void* s) {
  return guarded([&] {
    DOP_REQUIRE(l && dy && dx, "null pointer");
    l->backward(dy, dx, as_stream(s));
  });
}

int dop_lens_destroy(dop_lens* l) {
  return guarded([&] { delete l; });
}

int dop_program_create(const dop_stage* stages, int64_t n_stages, int64_t input_len,
                       int64_t output_len, int64_t param_len, int64_t tape_f32, int64_t tape_u8,
                       dop_program** out) {
  return guarded([&] {
    DOP_REQUIRE(out && (stages || n_stages == 0) && n_stages >= 0, "bad program");
    auto p = std::make_unique<dop_program>();
    p->stages.assign(stages, stages + n_stages);
    p->input_len = input_len; p->output_len = output_len; p->param_len = param_len;
    p->tape_f32 = tape_f32; p->tape_u8 = tape_u8;
    int64_t cap = std::max(input_len, output_len);
    int64_t max_rows = 1, max_cols = 1;
    for (const dop_stage& st : p->stages) {
      if (st.kind == DOP_STAGE_GEMM) {
        DOP_REQUIRE(st.batch >= 1 && st.din >= 1 && st.dout >= 1, "bad Gemm stage");
        DOP_REQUIRE(st.save_at + st.batch * st.din <= tape_f32, "Gemm stage saves past the tape");
        DOP_REQUIRE(st.param_at + st.din * st.dout + st.dout <= param_len, "Gemm params out of range");
        DOP_REQUIRE(!st.relu || st.mask_at + st.batch * st.dout <= tape_u8, "mask out of range");
        cap = std::max({cap, st.batch * st.din, st.batch * st.dout});
        max_rows = std::max(max_rows, st.batch);
        max_cols = std::max(max_cols, st.dout);
      } else if (st.kind == DOP_STAGE_ATTENTION) {
        DOP_REQUIRE(st.batch >= 1 && st.tokens >= 1 && st.dim >= 2 && st.dim <= 128 && st.dim % 2 == 0,
                    "attention stages need an even dim <= 128");
        DOP_REQUIRE(st.x_at + st.batch * st.tokens * st.dim <= tape_f32, "attention x past the tape");
        cap = std::max(cap, st.batch * st.tokens * st.dim);
      } else if (st.kind == DOP_STAGE_ADD) {
        DOP_REQUIRE(st.from >= 0 && st.from + st.len <= tape_f32, "Add reads past the tape");
      } else {
        DOP_REQUIRE(false, "unknown stage kind");
      }
    }
    p->act_cap = cap;
    p->tape = p->alloc(tape_f32);
    DOP_CHECK_CUDA(cudaMalloc(&p->mask, std::max<int64_t>(tape_u8, 1)));
    for (int i = 0; i < 2; ++i) p->buf[i] = p->alloc(cap);
    for (int i = 0; i < 2; ++i) p->dbuf[i] = p->alloc(cap);
    for (const dop_stage& st : p->stages)
      if (st.kind == DOP_STAGE_ATTENTION) {
        p->attn_out.push_back(p->alloc(st.batch * st.tokens * st.dim));
        p->attn_lse.push_back(p->alloc(st.batch * st.tokens));
      }
    p->delta = p->alloc(cap);
    p->dq = p->alloc(cap);
    p->dk = p->alloc(cap);
    p->dv = p->alloc(cap);
    p->part_cap = 64 * max_cols;
    p->part = p->alloc(p->part_cap);
    for (const dop_stage& st : p->stages)
      p->side_buf.push_back(st.kind == DOP_STAGE_ADD ? p->alloc(st.len) : nullptr);
    p->ones = p->alloc(output_len);
    int64_t widest = 1;
    for (const dop_stage& st : p->stages)
      if (st.kind == DOP_STAGE_GEMM)
        widest = std::max({widest, st.din * st.dout, st.batch * st.din, st.batch * st.dout});
    p->split_cap = std::min<int64_t>(1 << 22, 16 * widest);
    p->split_ws = p->alloc(p->split_cap);
    {
      std::vector<float> h(std::max<int64_t>(output_len, 1), 1.0f);
      DOP_CHECK_CUDA(cudaMemcpy(p->ones, h.data(), sizeof(float) * h.size(),
                                cudaMemcpyHostToDevice));
    }
    (void)max_rows;
    *out = p.release();
  });
}

int dop_program_destroy(dop_program* p) {
  return guarded([&] { delete p; });
}

int64_t dop_program_launches(const dop_program* p) { return p ? p->launches : -1; }

int dop_program_forward(dop_program* p, const float* x, const float* params, float* y, void* s) {
  return guarded([&] {
    DOP_REQUIRE(p && x && params && y, "null pointer");
    program_forward(p, x, params, y, as_stream(s));
  });
}

int dop_program_backward(dop_program* p, const float* params, const float* dy, float* dx,
                         float* dparams, void* s) {
  return guarded([&] {
    DOP_REQUIRE(p && params && dx && dparams, "null pointer");
    program_backward(p, params, dy, dx, dparams, as_stream(s));
  });
}

int dop_program_forward_backward(dop_program* p, const float* x, const float* params,
                                 const float* dy, float* y, float* dx, float* dparams, void* s) {
  return guarded([&] {
    DOP_REQUIRE(p && x && params && y && dx && dparams, "null pointer");
    program_forward(p, x, params, y, as_stream(s));
    program_backward(p, params, dy, dx, dparams, as_stream(s));
  });
}

int dop_mse_loss_grad(const float* y, const float* t, int64_t n, float* loss, float* dy, void* s) {
  return guarded([&] {
    DOP_REQUIRE(y && t && loss && dy && n >= 1, "bad mse arguments");
    int64_t l = 0;
    dop::mse(y, t, n, loss, dy, as_stream(s), l);
  });
}

int dop_gemm_bf16(int64_t M, int64_t N, int64_t K, const uint16_t* A, int64_t lda, int a_t,
                  const uint16_t* B, int64_t ldb, int b_t, void* C, int64_t ldc, int c_f32,
                  int accumulate, void* s) {
  return guarded([&] {
    DOP_REQUIRE(A && B && C && M > 0 && N > 0 && K > 0, "bad GEMM arguments");
    DOP_REQUIRE(!accumulate || c_f32, "accumulation needs an fp32 C");
    dop::Gemm g;
    g.M = M; g.N = N; g.K = K;
    g.A = A; g.lda = lda; g.a_t = a_t != 0;
    g.B = B; g.ldb = ldb; g.b_t = b_t != 0;
    g.C = C; g.ldc = ldc; g.c_f32 = c_f32 != 0;
    g.epi = accumulate ? dop::Epi::Accum : dop::Epi::Store;
    int64_t l = 0;
    dop::gemm_tc(g, nullptr, 0, dop::TcEpilogue{}, as_stream(s), l);
  });
}

int dop_device_status(void) { return dop::tc_error_status(); }

namespace {
dop::Attn gqa_desc(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, int64_t hd,
                   int64_t window) {
  DOP_REQUIRE(batch >= 1 && seq >= 1 && heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0,
              "bad attention shape");
  DOP_REQUIRE(hd >= 2 && hd % 2 == 0 && window >= 1, "bad head_dim or window");
  dop::Attn a;
  a.B = batch; a.S = seq; a.H = (int)heads; a.KV = (int)kv_heads; a.hd = (int)hd;
  a.window = window; a.causal = true; a.scale = 1.0f / sqrtf((float)hd);
  return a;
}
}  // namespace

int dop_gqa_forward(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, int64_t hd,
                    int64_t window, int precision, const void* q, const void* k, const void* v,
                    void* o, float* lse, void* s) {
  return guarded([&] {
    DOP_REQUIRE(q && k && v && o && lse, "null pointer");
    dop::Attn a = gqa_desc(batch, seq, heads, kv_heads, hd, window);
    int64_t l = 0;
    if (precision == DOP_BF16 && hd == 128)
      dop::attn_fwd_tc(a, (const dop::bf16*)q, (const dop::bf16*)k, (const dop::bf16*)v,
                       (dop::bf16*)o, lse, as_stream(s), l);
    else if (precision == DOP_BF16)
      dop::attn_fwd_simt<dop::bf16>(a, (const dop::bf16*)q, (const dop::bf16*)k,
                                    (const dop::bf16*)v, (dop::bf16*)o, lse, as_stream(s), l);
    else
      dop::attn_fwd_simt<float>(a, (const float*)q, (const float*)k, (const float*)v, (float*)o,
                                lse, as_stream(s), l);
  });
}

int dop_gqa_backward(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, int64_t hd,
                     int64_t window, int precision, const void* q, const void* k, const void* v,
                     const void* o, const void* dout, const float* lse, float* delta_ws,
                     float* dq, float* dk, float* dv, void* s) {
  return guarded([&] {
    DOP_REQUIRE(q && k && v && o && dout && lse && delta_ws && dq && dk && dv, "null pointer");
    dop::Attn a = gqa_desc(batch, seq, heads, kv_heads, hd, window);
    int64_t l = 0;
    if (precision == DOP_BF16 && hd == 128)
      dop::attn_bwd_tc(a, (const dop::bf16*)q, (const dop::bf16*)k, (const dop::bf16*)v,
                       (const dop::bf16*)o, (const dop::bf16*)dout, lse, delta_ws, dq, dk, dv,
                       as_stream(s), l);
    else if (precision == DOP_BF16)
      dop::attn_bwd_simt<dop::bf16>(a, (const dop::bf16*)q, (const dop::bf16*)k,
                                    (const dop::bf16*)v, (const dop::bf16*)o,
                                    (const dop::bf16*)dout, lse, delta_ws, dq, dk, dv,
                                    as_stream(s), l);
    else
      dop::attn_bwd_simt<float>(a, (const float*)q, (const float*)k, (const float*)v,
                                (const float*)o, (const float*)dout, lse, delta_ws, dq, dk, dv,
                                as_stream(s), l);
  });
}

int dop_f32_to_bf16(const float* src, uint16_t* dst, int64_t n, void* s) {
  return guarded([&] {
    DOP_REQUIRE(src && dst && n >= 0, "bad conversion arguments");
    int64_t l = 0;
    dop::convert<dop::bf16>(src, reinterpret_cast<dop::bf16*>(dst), n, as_stream(s), l);
  });
}

int dop_exp2_poly(const float* x, float* y, int64_t n, void* s) {
  return guarded([&] {
    DOP_REQUIRE(x && y && n >= 0, "bad exp2 arguments");
    int64_t l = 0;
    dop::tc::exp2_poly(x, y, n, as_stream(s), l);
  });
}

int dop_sgd_step(float* params, const float* grad, int64_t n, float lr, void* s) {
  return guarded([&] {
    DOP_REQUIRE(params && grad && n >= 0, "bad sgd arguments");
    int64_t l = 0;
    dop::sgd(params, grad, n, lr, as_stream(s), l);
  });
}

}  // extern "C"
