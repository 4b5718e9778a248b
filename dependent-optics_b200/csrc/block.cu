// block.cu — the Mixtral block lens on the device.
//
// forward  = src/mixtral.rs:291-380 (forward_layer)
// backward = src/mixtral.rs:434-598 (backward_layer)
// with the crate's per-token expert loop replaced by the deterministic
// expert permutation and grouped GEMMs over the expert-sorted rows.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "block.cuh"

namespace dop {

LayerOffsets layer_offsets(const dop_mixtral_cfg& c) {
  LayerOffsets o{};
  const int64_t D = c.dim, qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
  int64_t at = 0;
  o.attn_norm = at; at += D;
  o.q = at; at += D * qd;
  o.k = at; at += D * kvd;
  o.v = at; at += D * kvd;
  o.o = at; at += qd * D;
  o.ffn_norm = at; at += D;
  o.router = at; at += D * c.experts;
  o.gate0 = at;
  o.up0 = at + D * c.intermediate;
  o.down0 = at + 2 * D * c.intermediate;
  o.expert_stride = 3 * D * c.intermediate;
  o.total = at + c.experts * o.expert_stride;
  return o;
}

namespace {
struct Carver {
  size_t at = 0;
  template <typename P>
  void take(P*& p, size_t bytes, char* base) {
    at = (at + 255) & ~size_t(255);
    p = base ? reinterpret_cast<P*>(base + at) : nullptr;
    at += bytes;
  }
};
}  // namespace

Block::Block(const dop_mixtral_cfg& c, int64_t batch, int64_t seq, int precision, int rank,
             int world, bool allocate)
    : cfg(c), B(batch), S(seq), T(batch * seq), prec(precision), ep_rank(rank), ep_world(world) {
  DOP_REQUIRE(batch >= 1 && seq >= 1, "batch and seq must be >= 1");
  DOP_REQUIRE(c.dim >= 1 && c.heads >= 1 && c.kv_heads >= 1 && c.head_dim >= 2,
              "bad model widths");
  DOP_REQUIRE(c.heads % c.kv_heads == 0, "heads must be a multiple of kv_heads");
  DOP_REQUIRE(c.head_dim % 2 == 0, "head_dim must be even");
  DOP_REQUIRE(c.experts >= 1 && c.experts <= kMaxExperts, "experts out of range");
  DOP_REQUIRE(c.top_k >= 1 && c.top_k <= kMaxTopK && c.top_k <= c.experts, "top_k out of range");
  DOP_REQUIRE(c.sliding_window >= 1, "sliding_window must be >= 1");
  DOP_REQUIRE(c.intermediate >= 1, "intermediate must be >= 1");
  DOP_REQUIRE(precision == DOP_F32 || precision == DOP_BF16, "precision must be DOP_F32 or DOP_BF16");
  DOP_REQUIRE(c.dim <= 1024 * 32, "dim too large");
  DOP_REQUIRE(T * c.top_k < (int64_t)1 << 30, "too many tokens");
  if (precision == DOP_BF16) {
    // tensor-core operands: 16-byte row strides (TMA) and 32-column SwiGLU tiles
    DOP_REQUIRE(c.dim % 8 == 0 && (c.heads * c.head_dim) % 8 == 0 &&
                    (c.kv_heads * c.head_dim) % 8 == 0,
                "the bf16 lens needs dim, heads*head_dim and kv_heads*head_dim multiples of 8");
    DOP_REQUIRE(c.intermediate % 32 == 0, "the bf16 lens needs intermediate % 32 == 0");
  }
  DOP_REQUIRE(world >= 1 && world <= kEpMaxWorld && rank >= 0 && rank < world,
              "expert-parallel rank/world out of range");
  if (world > 1) {
    DOP_REQUIRE(precision == DOP_BF16, "expert parallelism runs the bf16 lens");
    DOP_REQUIRE(c.experts % world == 0, "experts must be a multiple of the expert-parallel world");
  }
  off = layer_offsets(c);
  const int64_t D = c.dim, E = c.experts, K = c.top_k, I = c.intermediate;
  const int64_t qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
  rows_cap = round_up(T * K + E * (kSegAlign - 1), kSegAlign);
  max_tiles = (int)(rows_cap / kRowAlign);
  const bool ep = world > 1;
  ep_local = (int)(E / world);
  recv_cap = ep ? world * rows_cap : 0;
  const int recv_tiles = (int)(recv_cap / kRowAlign);
  const int64_t xe = ep ? 0 : 1;  // the local expert buffers exist without EP only
  const size_t a = prec == DOP_F32 ? 4 : 2;  // activation element size
  const int64_t chunks = ceil_div(T * K, kPermChunk);
  part_cap = std::max<int64_t>((int64_t)sm_count() * 4 * D, 64 * D * E);
  part_cap = std::max<int64_t>(part_cap, 64 * std::max(qd, D));
  split_cap = prec == DOP_F32 ? std::min<int64_t>(1 << 22, 16 * D * std::max(qd, D)) : 0;
  // fp32 lens: tf32 hi / lo operands of the largest contraction on the
  // tensor cores (3xTF32): experts (grouped over E), their weight adjoints
  // (contraction over every expert-sorted row), the attention projections
  if (prec == DOP_F32) {
    const int64_t W = std::max(D, qd);
    tf32_cap = 2 * std::max({rows_cap * D + E * I * D, rows_cap * I + E * D * I,
                             (I + D) * rows_cap, T * W + W * W, 2 * W * T});
  }

  auto carve = [&](char* base_) {
    Carver cv;
    cv.take(x_in, 4 * T * D, base_);
    cv.take(inv1, 4 * T, base_);
    cv.take(mid, 4 * T * D, base_);
    cv.take(inv2, 4 * T, base_);
    cv.take(lse, 4 * T * c.heads, base_);
    cv.take(probs, 4 * T * E, base_);
    cv.take(top_p, 4 * T * K, base_);
    cv.take(top_w, 4 * T * K, base_);
    cv.take(row_w, 4 * rows_cap, base_);
    cv.take(out, 4 * rows_cap * D, base_);
    cv.take(top_i, 4 * T * K, base_);
    cv.take(slot_row, 4 * T * K, base_);
    cv.take(seg_off, 4 * (E + 1), base_);
    cv.take(tile_expert, 4 * max_tiles, base_);
    cv.take(row_token, 4 * rows_cap, base_);
    cv.take(chunk_counts, 4 * chunks * E, base_);
    cv.take(xn, a * T * D, base_);
    cv.take(q, a * T * qd, base_);
    cv.take(k, a * T * kvd, base_);
    cv.take(v, a * T * kvd, base_);
    cv.take(mix, a * T * qd, base_);
    cv.take(xn2, a * T * D, base_);
    cv.take(xp, xe * a * rows_cap * D, base_);
    cv.take(g, xe * a * rows_cap * I, base_);
    cv.take(u, xe * a * rows_cap * I, base_);
    cv.take(h, xe * a * rows_cap * I, base_);
    cv.take(qpre, 4 * T * qd, base_);
    cv.take(kpre, 4 * T * kvd, base_);
    cv.take(rope_cos, 4 * S * (c.head_dim / 2), base_);
    cv.take(rope_sin, 4 * S * (c.head_dim / 2), base_);
    cv.take(dz, 4 * T * E, base_);
    cv.take(dh, prec == DOP_F32 ? 4 * rows_cap * I : 0, base_);
    cv.take(dxp, xe * 4 * rows_cap * D, base_);
    cv.take(dxn2, 4 * T * D, base_);
    cv.take(dmid, 4 * T * D, base_);
    cv.take(dxn, 4 * T * D, base_);
    cv.take(dq, 4 * T * qd, base_);
    cv.take(dk, 4 * T * kvd, base_);
    cv.take(dv, 4 * T * kvd, base_);
    cv.take(delta, 4 * T * c.heads, base_);
    cv.take(part, 4 * part_cap, base_);
    cv.take(split_ws, 4 * split_cap, base_);
    cv.take(tf32_ws, 4 * tf32_cap, base_);
    cv.take(dO, a * rows_cap * D, base_);
    cv.take(dg, xe * a * rows_cap * I, base_);
    cv.take(du, xe * a * rows_cap * I, base_);
    cv.take(dmid_a, a * T * D, base_);
    cv.take(dmix, a * T * qd, base_);
    cv.take(dq_a, a * T * qd, base_);
    cv.take(dk_a, a * T * kvd, base_);
    cv.take(dv_a, a * T * kvd, base_);
    if (ep) {
      cv.take(ep_flags, 4 * kEpBarriers * kEpMaxWorld, base_);
      cv.take(piece_pos, 4 * E, base_);
      cv.take(ep_bounds, 4 * (kEpMaxWorld + 1), base_);
      cv.take(recv_seg_off, 4 * (E + 1), base_);
      cv.take(own_end, 4 * E, base_);
      cv.take(help_end, 4 * E, base_);
      cv.take(helpers, 4 * E, base_);
      cv.take(recv_tile_expert, 4 * recv_tiles, base_);
      cv.take(recv_tile_src, 4 * recv_tiles, base_);
      cv.take(recv_tile_row0, 4 * recv_tiles, base_);
      cv.take(xr, 2 * recv_cap * D, base_);
      cv.take(gr, 2 * recv_cap * I, base_);
      cv.take(ur, 2 * recv_cap * I, base_);
      cv.take(hr, 2 * recv_cap * I, base_);
      cv.take(dOr, 2 * recv_cap * D, base_);
      cv.take(outr, 4 * recv_cap * D, base_);
      cv.take(dxpr, 4 * recv_cap * D, base_);
      cv.take(dw_help, 4 * E * off.expert_stride, base_);
    }
    return cv.at;
  };
  bytes = carve(nullptr);
  if (!allocate) return;  // size query only (no device work)
  cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) {
    base = nullptr;
    throw Error(DOP_E_NOMEM, "cudaMalloc of " + std::to_string(bytes) + " bytes for the block: " +
                                 cudaGetErrorString(e));
  }
  carve(base);
  if (ep) {
    DOP_CHECK_CUDA(cudaMemset(ep_flags, 0, 4 * kEpBarriers * kEpMaxWorld));
    ep_peer_base.assign(world, nullptr);
    ep_peer_base[rank] = base;
  }
  // RoPE table (positions 0..S-1) once per handle.
  rope_table((int)S, (int)c.head_dim, c.rope_theta, rope_cos, rope_sin, 0, launches);
  DOP_CHECK_CUDA(cudaStreamSynchronize(0));
}

Block::~Block() {
  for (int r = 0; r < (int)ep_peer_base.size(); ++r)
    if (r != ep_rank && ep_peer_base[r]) cudaIpcCloseMemHandle(ep_peer_base[r]);
  if (ep_peers_dev) cudaFree(ep_peers_dev);
  if (ep_stream) cudaStreamDestroy(ep_stream);
  if (ep_ev_dx) cudaEventDestroy(ep_ev_dx);
  if (ep_ev_combined) cudaEventDestroy(ep_ev_combined);
  if (ep_ev_dw) cudaEventDestroy(ep_ev_dw);
  if (ep_ev_reduced) cudaEventDestroy(ep_ev_reduced);
  if (expert_adjoint_done) cudaEventDestroy(expert_adjoint_done);
  for (auto& p : phases) {
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  if (base) cudaFree(base);
}

// ------------------------------------------------------ expert parallelism
EpView Block::ep_view() const {
  EpView v;
  v.rank = ep_rank; v.world = ep_world; v.local = ep_local; v.E = (int)cfg.experts;
  v.recv_tiles = (int)(recv_cap / kRowAlign);
  v.recv_cap = recv_cap;
  v.expert_stride = off.expert_stride;
  v.peers = ep_peers_dev; v.flags = ep_flags;
  v.seg_off = seg_off; v.row_token = row_token; v.piece_pos = piece_pos; v.bounds = ep_bounds;
  v.recv_seg_off = recv_seg_off; v.own_end = own_end; v.help_end = help_end; v.helpers = helpers;
  v.recv_tile_expert = recv_tile_expert;
  v.recv_tile_src = recv_tile_src; v.recv_tile_row0 = recv_tile_row0;
  v.xr = (bf16*)xr; v.outr = outr; v.dxpr = dxpr; v.dw_help = dw_help;
  return v;
}

void Block::ep_connect(const cudaIpcMemHandle_t* handles) {
  DOP_REQUIRE(ep_world > 1, "not an expert-parallel block");
  DOP_REQUIRE(!ep_peers_dev, "expert-parallel block already connected");
  for (int r = 0; r < ep_world; ++r) {
    if (r == ep_rank) continue;
    void* p = nullptr;
    DOP_CHECK_CUDA(cudaIpcOpenMemHandle(&p, handles[r], cudaIpcMemLazyEnablePeerAccess));
    ep_peer_base[r] = (char*)p;
  }
  DOP_CHECK_CUDA(cudaMalloc(&ep_peers_dev, sizeof(char*) * ep_world));
  DOP_CHECK_CUDA(cudaMemcpy(ep_peers_dev, ep_peer_base.data(), sizeof(char*) * ep_world,
                            cudaMemcpyHostToDevice));
}

void Block::ep_barrier_next(int k, cudaStream_t s) {
  DOP_REQUIRE(ep_peers_dev, "expert-parallel block is not connected (dop_block_ep_connect)");
  ep_barrier(ep_view(), k, ++ep_epoch, s, launches);
}

// Forward experts of an expert-parallel block, after the permutation:
// plan the step (which rank processes which rows), gather this rank's
// receive rows from the sources, gate/up (SwiGLU) and down over them, then
// combine the processing ranks' outputs into y.  The grouped GEMMs run over
// every expert (absolute expert indices; the experts this rank has no rows
// of are empty segments).
void Block::ep_fwd_experts(const bf16* P, float* y, cudaStream_t s) {
  const int64_t D = cfg.dim, I = cfg.intermediate, K = cfg.top_k;
  const int E = (int)cfg.experts;
  const EpView v = ep_view();
  ph_begin("ep_wait_rows", s);
  ep_barrier_next(0, s);  // every rank's xn2, row_token, seg_off are written
  ph_end(s);
  ph_begin("ep_dispatch", s);
  ep_layout(v, s, launches);
  ep_gather_tokens(v, (const bf16*)xn2, (int)D, s, launches);
  ph_end(s);
  ph_begin("expert_gate_up", s);
  {
    Gemm gg; gg.M = recv_cap; gg.N = I; gg.K = D; gg.A = xr; gg.lda = D;
    gg.B = P + off.gate0; gg.ldb = I; gg.C = gr; gg.ldc = I; gg.c_f32 = false;
    gg.group = 1; gg.seg_off = recv_seg_off; gg.tile_expert = recv_tile_expert; gg.G = E;
    gg.b_gs = off.expert_stride;
    TcEpilogue te; te.kind = kTcSwiGLU; te.up_B = P + off.up0;
    te.g_out = (bf16*)gr; te.u_out = (bf16*)ur; te.h_out = (bf16*)hr; te.ldg = I;
    gemm_tc(gg, nullptr, 0, te, s, launches);
  }
  ph_end(s);
  ph_begin("expert_down", s);
  {
    Gemm gd; gd.M = recv_cap; gd.N = D; gd.K = I; gd.A = hr; gd.lda = I;
    gd.B = P + off.down0; gd.ldb = D; gd.C = outr; gd.ldc = D;
    gd.group = 1; gd.seg_off = recv_seg_off; gd.tile_expert = recv_tile_expert; gd.G = E;
    gd.b_gs = off.expert_stride;
    gemm<bf16>(gd, s);
  }
  ph_end(s);
  ph_begin("ep_wait_outputs", s);
  ep_barrier_next(1, s);  // every rank's expert outputs are written
  ph_end(s);
  ph_begin("combine", s);
  ep_combine(v, mid, top_i, slot_row, top_w, T, (int)K, (int)D, out, y, s, launches);
  ph_end(s);
}

// Backward experts of an expert-parallel block, after the output cotangent
// rows dO are written: gather them for this rank's rows, dH with the SwiGLU
// adjoint, the weight adjoints of this rank's rows (into dparams for the
// experts it owns, into dw_help for the others), and dXp for the sources.
// After the last barrier the owner adds the helpers' partial adjoints.
void Block::ep_bwd_experts(const bf16* P, float* dP, cudaStream_t s) {
  const int64_t D = cfg.dim, I = cfg.intermediate;
  const int E = (int)cfg.experts;
  const EpView v = ep_view();
  const int64_t up_at = off.up0 - off.gate0, down_at = off.down0 - off.gate0;
  ph_begin("ep_wait_dO", s);
  ep_barrier_next(2, s);  // every rank's dO is written
  ph_end(s);
  ph_begin("ep_dispatch_bwd", s);
  ep_gather_rows(v, (const bf16*)dO, (bf16*)dOr, (int)D, s, launches);
  ph_end(s);
  ph_begin("expert_dh", s);
  {
    Gemm g1; g1.M = recv_cap; g1.N = I; g1.K = D; g1.A = dOr; g1.lda = D;
    g1.B = P + off.down0; g1.ldb = D; g1.b_t = true; g1.C = dh; g1.ldc = I;
    g1.group = 1; g1.seg_off = recv_seg_off; g1.tile_expert = recv_tile_expert; g1.G = E;
    g1.b_gs = off.expert_stride;
    // dg, du overwrite g, u in place (each element is read before it is written)
    TcEpilogue te; te.kind = kTcSwiGLUBwd; te.g_in = (const bf16*)gr; te.u_in = (const bf16*)ur;
    te.dg_out = (bf16*)gr; te.du_out = (bf16*)ur; te.ldg = I;
    gemm_tc(g1, nullptr, 0, te, s, launches);
  }
  ph_end(s);
  // a grouped weight adjoint over this rank's rows: the owned experts'
  // segments accumulate into dparams, the others' overwrite dw_help
  auto dw = [&](Gemm g, int64_t at) {
    Gemm own = g;
    own.C = dP + off.gate0 + at; own.epi = Epi::Accum; own.seg_end = own_end;
    gemm<bf16>(own, s);
    Gemm help = g;
    help.C = dw_help + at; help.epi = Epi::Store; help.seg_end = help_end;
    gemm<bf16>(help, s);
  };
  ph_begin("expert_dw_down", s);
  {
    Gemm g2; g2.M = I; g2.N = D; g2.K = recv_cap; g2.A = hr; g2.lda = I; g2.a_t = true;
    g2.B = dOr; g2.ldb = D; g2.ldc = D;
    g2.group = 2; g2.seg_off = recv_seg_off; g2.G = E; g2.c_gs = off.expert_stride;
    dw(g2, down_at);
  }
  ph_end(s);
  ph_begin("expert_dx", s);
  {
    Gemm g3; g3.M = recv_cap; g3.N = D; g3.K = I; g3.A = gr; g3.lda = I;
    g3.B = P + off.gate0; g3.ldb = I; g3.b_t = true; g3.C = dxpr; g3.ldc = D;
    g3.group = 1; g3.seg_off = recv_seg_off; g3.tile_expert = recv_tile_expert; g3.G = E;
    g3.b_gs = off.expert_stride;
    GemmPart up{ur, I, P + off.up0, I, I};
    gemm<bf16>(g3, s, &up, 1);
  }
  ph_end(s);
  // The sources' backward combine (wait for every rank's dXp, then read
  // this rank's pairs) runs on the exchange stream while this rank computes
  // its gate/up weight adjoints, which nothing there reads.
  if (!ep_stream) {
    DOP_CHECK_CUDA(cudaStreamCreateWithFlags(&ep_stream, cudaStreamNonBlocking));
    DOP_CHECK_CUDA(cudaEventCreateWithFlags(&ep_ev_dx, cudaEventDisableTiming));
    DOP_CHECK_CUDA(cudaEventCreateWithFlags(&ep_ev_combined, cudaEventDisableTiming));
    DOP_CHECK_CUDA(cudaEventCreateWithFlags(&ep_ev_dw, cudaEventDisableTiming));
    DOP_CHECK_CUDA(cudaEventCreateWithFlags(&ep_ev_reduced, cudaEventDisableTiming));
  }
  DOP_CHECK_CUDA(cudaEventRecord(ep_ev_dx, s));
  DOP_CHECK_CUDA(cudaStreamWaitEvent(ep_stream, ep_ev_dx, 0));
  ep_barrier_next(3, ep_stream);  // every rank's dXp is written
  ep_unpermute_router_dx<bf16>(v, top_i, slot_row, dz, P + off.router, T, E, (int)cfg.top_k,
                               (int)D, dxn2, ep_stream, launches);
  DOP_CHECK_CUDA(cudaEventRecord(ep_ev_combined, ep_stream));
  ph_begin("expert_dw_gate_up", s);
  {
    Gemm g5; g5.M = D; g5.N = I; g5.K = recv_cap; g5.A = xr; g5.lda = D; g5.a_t = true;
    g5.B = gr; g5.ldb = I; g5.ldc = I;
    g5.group = 2; g5.seg_off = recv_seg_off; g5.G = E; g5.c_gs = off.expert_stride;
    dw(g5, 0);
    Gemm g6 = g5; g6.B = ur;
    dw(g6, up_at);
  }
  ph_end(s);
  // every rank's partial adjoints are written: the owners add them (on the
  // exchange stream, beside the attention half of the backward)
  DOP_CHECK_CUDA(cudaEventRecord(ep_ev_dw, s));
  DOP_CHECK_CUDA(cudaStreamWaitEvent(ep_stream, ep_ev_dw, 0));
  ep_barrier_next(4, ep_stream);
  ep_reduce_adjoint(v, dP + off.gate0, ep_stream, launches);
  DOP_CHECK_CUDA(cudaEventRecord(ep_ev_reduced, ep_stream));
}

void Block::ph_begin(const char* name, cudaStream_t s) {
  cur_phase = name;
  if (!timing) return;
  if (n_phases == phases.size()) {
    Phase p{name, nullptr, nullptr};
    DOP_CHECK_CUDA(cudaEventCreate(&p.a));
    DOP_CHECK_CUDA(cudaEventCreate(&p.b));
    phases.push_back(p);
  }
  phases[n_phases].name = name;
  DOP_CHECK_CUDA(cudaEventRecord(phases[n_phases].a, s));
}

void Block::ph_end(cudaStream_t s) {
  // DOP_DEBUG_SYNC=1: synchronise after every phase and report it on stderr
  static const bool debug_sync = getenv("DOP_DEBUG_SYNC") != nullptr;
  if (debug_sync) {
    cudaError_t e = cudaStreamSynchronize(s);
    fprintf(stderr, "[dop] phase %s done: %s, tensor-core status %d\n", cur_phase,
            cudaGetErrorString(e), tc_error_status());
  }
  if (!timing) return;
  DOP_CHECK_CUDA(cudaEventRecord(phases[n_phases].b, s));
  ++n_phases;
}

// Contraction dispatch: the fp32 lens runs the CUDA-core GEMM (extra K
// parts as accumulating passes), the bf16 lens the tcgen05 GEMM (extra K
// parts summed in one TMEM accumulator).
template <typename Act>
void Block::gemm(const Gemm& g, cudaStream_t s, const GemmPart* extra, int n_extra) {
  if (std::is_same<Act, bf16>::value) {
    gemm_tc(g, extra, n_extra, TcEpilogue{}, s, launches);
    return;
  }
  // fp32 contractions on the tensor cores as three tf32 products when the
  // shape allows (fp32 C, 16-byte rows), on the CUDA cores otherwise
  auto tf32_part = [&](const Gemm& gp) {
    return gemm_tc_f32_ok(gp) && gemm_tc_f32_scratch(gp) <= tf32_cap;
  };
  bool tc = tf32_part(g);
  for (int i = 0; i < n_extra && tc; ++i) {
    Gemm gi = g;
    gi.A = extra[i].A; gi.lda = extra[i].lda; gi.B = extra[i].B; gi.ldb = extra[i].ldb;
    gi.K = extra[i].K; gi.epi = Epi::Accum;
    tc = tf32_part(gi);
  }
  if (tc) {
    gemm_tc_f32(g, tf32_ws, tf32_cap, s, launches);
    for (int i = 0; i < n_extra; ++i) {
      Gemm gi = g;
      gi.A = extra[i].A; gi.lda = extra[i].lda; gi.B = extra[i].B; gi.ldb = extra[i].ldb;
      gi.K = extra[i].K; gi.epi = Epi::Accum;
      gemm_tc_f32(gi, tf32_ws, tf32_cap, s, launches);
    }
    return;
  }
  Gemm gs = g;
  gs.ws = split_ws;
  gs.ws_cap = split_cap;
  gemm_simt<Act>(gs, s, launches);
  for (int i = 0; i < n_extra; ++i) {
    Gemm gi = gs;
    gi.A = extra[i].A; gi.lda = extra[i].lda; gi.B = extra[i].B; gi.ldb = extra[i].ldb;
    gi.K = extra[i].K; gi.epi = Epi::Accum;
    gemm_simt<Act>(gi, s, launches);
  }
}

void Block::forward(const void* params, const float* x, float* y, cudaStream_t s) {
  DOP_REQUIRE(params && x && y, "null pointer");
  n_phases = 0;
  if (prec == DOP_F32) fwd<float>((const float*)params, x, y, s);
  else fwd<bf16>((const bf16*)params, x, y, s);
  n_fwd_phases = n_phases;
  have_tape = true;
}

void Block::backward(const void* params, const float* dy, float* dx, float* dparams,
                     cudaStream_t s) {
  DOP_REQUIRE(params && dy && dx && dparams, "null pointer");
  if (!have_tape) throw Error(DOP_E_STATE, "backward called before forward");
  n_phases = n_fwd_phases;
  if (prec == DOP_F32) bwd<float>((const float*)params, dy, dx, dparams, s);
  else bwd<bf16>((const bf16*)params, dy, dx, dparams, s);
}

template <typename Act>
void Block::fwd(const Act* P, const float* x, float* y, cudaStream_t s) {
  const int64_t D = cfg.dim, E = cfg.experts, K = cfg.top_k, I = cfg.intermediate;
  const int H = (int)cfg.heads, KV = (int)cfg.kv_heads, hd = (int)cfg.head_dim;
  const int64_t qd = (int64_t)H * hd, kvd = (int64_t)KV * hd;
  Act* xn_ = (Act*)xn; Act* q_ = (Act*)q; Act* k_ = (Act*)k; Act* v_ = (Act*)v; Act* mix_ = (Act*)mix;
  Act* xn2_ = (Act*)xn2; Act* xp_ = (Act*)xp; Act* g_ = (Act*)g; Act* u_ = (Act*)u; Act* h_ = (Act*)h;

  // attention half: xn = rmsnorm(x); q,k,v = xn W; rope; gqa; mid = x + mix Wo
  ph_begin("attn_norm", s);
  rmsnorm_fwd<Act>(x, P + off.attn_norm, T, (int)D, cfg.rms_eps, xn_, inv1, x_in, s, launches);
  ph_end(s);
  // bf16 with 128-wide heads: RoPE is applied in the Q/K GEMMs' epilogue
  // on the fp32 accumulators, which round once into the bf16 q and k
  const bool rope_in_gemm = std::is_same<Act, bf16>::value && hd == 128;
  ph_begin("qkv_gemm", s);
  {
    Gemm gq; gq.M = T; gq.N = qd; gq.K = D; gq.A = xn_; gq.lda = D; gq.B = P + off.q; gq.ldb = qd;
    gq.C = qpre; gq.ldc = qd;
    Gemm gk = gq; gk.N = kvd; gk.B = P + off.k; gk.ldb = kvd; gk.C = kpre; gk.ldc = kvd;
    if (rope_in_gemm) {
      TcEpilogue te; te.kind = kTcRope;
      te.rope_cos = rope_cos; te.rope_sin = rope_sin; te.rope_seq = (int)S;
      gq.C = q_; gq.c_f32 = false;
      gk.C = k_; gk.c_f32 = false;
      gemm_tc(gq, nullptr, 0, te, s, launches);
      gemm_tc(gk, nullptr, 0, te, s, launches);
    } else {
      gemm<Act>(gq, s);
      gemm<Act>(gk, s);
    }
    Gemm gv = gk; gv.B = P + off.v; gv.C = v_; gv.c_f32 = std::is_same<Act, float>::value;
    gemm<Act>(gv, s);
  }
  ph_end(s);
  if (!rope_in_gemm) {
    ph_begin("rope", s);
    rope<float, Act>(qpre, q_, T, (int)S, H, hd, rope_cos, rope_sin, 1.f, s, launches);
    rope<float, Act>(kpre, k_, T, (int)S, KV, hd, rope_cos, rope_sin, 1.f, s, launches);
    ph_end(s);
  }
  Attn at; at.B = B; at.S = S; at.H = H; at.KV = KV; at.hd = hd; at.window = cfg.sliding_window;
  at.causal = true; at.scale = 1.0f / sqrtf((float)hd);
  ph_begin("attn_fwd", s);
  if (std::is_same<Act, bf16>::value && hd == 128)
    attn_fwd_tc(at, (const bf16*)q_, (const bf16*)k_, (const bf16*)v_, (bf16*)mix_, lse, s,
                launches);
  else
    attn_fwd_simt<Act>(at, q_, k_, v_, mix_, lse, s, launches);
  ph_end(s);
  ph_begin("o_gemm", s);
  {
    Gemm go; go.M = T; go.N = D; go.K = qd; go.A = mix_; go.lda = qd; go.B = P + off.o; go.ldb = D;
    go.C = mid; go.ldc = D; go.epi = Epi::AddRes; go.R = x; go.ldr = D;
    gemm<Act>(go, s);
  }
  ph_end(s);
  // mixture half: xn2 = rmsnorm(mid); router; permute; experts; y = mid + mixed
  ph_begin("ffn_norm_router", s);
  rmsnorm_router<Act>(mid, P + off.ffn_norm, P + off.router, router_bias, T, (int)D, (int)E,
                    (int)K, cfg.rms_eps, xn2_, inv2, probs, top_i, top_p, top_w, s, launches);
  ph_end(s);
  ph_begin("permute", s);
  permute(top_i, top_w, T, (int)E, (int)K, chunk_counts, seg_off, tile_expert, max_tiles,
          slot_row, row_token, row_w, rows_cap, s, launches);
  if constexpr (std::is_same<Act, bf16>::value) {
    if (ep_world > 1) {  // the owners gather the rows themselves
      ph_end(s);
      ep_fwd_experts(P, y, s);
      return;
    }
  }
  scatter_rows<Act>(xn2_, slot_row, T, (int)K, row_token, seg_off, (int)E, (int)D, rows_cap, xp_, s,
                    launches);
  ph_end(s);
  ph_begin("expert_gate_up", s);
  {
    Gemm gg; gg.M = rows_cap; gg.N = I; gg.K = D; gg.A = xp_; gg.lda = D;
    gg.B = P + off.gate0; gg.ldb = I; gg.C = g_; gg.ldc = I; gg.c_f32 = std::is_same<Act, float>::value;
    gg.group = 1; gg.seg_off = seg_off; gg.tile_expert = tile_expert; gg.G = (int)E;
    gg.b_gs = off.expert_stride;
    if (std::is_same<Act, bf16>::value) {
      // one tensor-core pass: B = [gate | up], epilogue writes g, u and
      // h = silu(g) * u (src/mixtral.rs:318-329)
      TcEpilogue te; te.kind = kTcSwiGLU; te.up_B = P + off.up0;
      te.g_out = (bf16*)g_; te.u_out = (bf16*)u_; te.h_out = (bf16*)h_; te.ldg = I;
      gemm_tc(gg, nullptr, 0, te, s, launches);
    } else {
      gemm<Act>(gg, s);
      Gemm gu = gg; gu.B = P + off.up0; gu.C = u_;
      gemm<Act>(gu, s);
      ph_end(s);
      ph_begin("swiglu", s);
      silu_mul<Act>(g_, u_, seg_off, (int)E, I, rows_cap, h_, s, launches);
    }
  }
  ph_end(s);
  ph_begin("expert_down", s);
  {
    Gemm gd; gd.M = rows_cap; gd.N = D; gd.K = I; gd.A = h_; gd.lda = I;
    gd.B = P + off.down0; gd.ldb = D; gd.C = out; gd.ldc = D;
    gd.group = 1; gd.seg_off = seg_off; gd.tile_expert = tile_expert; gd.G = (int)E;
    gd.b_gs = off.expert_stride;
    gemm<Act>(gd, s);
  }
  ph_end(s);
  ph_begin("combine", s);
  combine(mid, out, slot_row, top_w, T, (int)K, (int)D, y, s, launches);
  ph_end(s);
}

template <typename Act>
void Block::bwd(const Act* P, const float* dy, float* dx, float* dP, cudaStream_t s) {
  const int64_t D = cfg.dim, E = cfg.experts, K = cfg.top_k, I = cfg.intermediate;
  const int H = (int)cfg.heads, KV = (int)cfg.kv_heads, hd = (int)cfg.head_dim;
  const int64_t qd = (int64_t)H * hd, kvd = (int64_t)KV * hd;
  const bool f32 = std::is_same<Act, float>::value;
  Act* xn_ = (Act*)xn; Act* q_ = (Act*)q; Act* k_ = (Act*)k; Act* v_ = (Act*)v; Act* mix_ = (Act*)mix;
  Act* xp_ = (Act*)xp; Act* g_ = (Act*)g; Act* u_ = (Act*)u; Act* h_ = (Act*)h;
  Act* dO_ = (Act*)dO; Act* dg_ = (Act*)dg; Act* du_ = (Act*)du; Act* dmid_ = (Act*)dmid_a;
  Act* dmix_ = (Act*)dmix; Act* dq_ = (Act*)dq_a; Act* dk_ = (Act*)dk_a; Act* dv_ = (Act*)dv_a;

  // router Jacobian (src/mixtral.rs:456-541) and the down projection's output
  // cotangent d_out = w * dy, in expert-sorted rows
  ph_begin("router_bwd", s);
  router_bwd(dy, out, slot_row, top_i, top_p, top_w, probs, T, (int)E, (int)K, (int)D, dz, s,
             launches);
  scatter_scale_rows<Act>(dy, slot_row, top_w, T, (int)K, row_token, row_w, seg_off, (int)E, (int)D,
                          rows_cap, dO_, s, launches);
  ph_end(s);
  bool ep = false;
  if constexpr (std::is_same<Act, bf16>::value) {
    if (ep_world > 1) {
      ep_bwd_experts(P, dP, s);
      ep = true;
    }
  }
  if (!ep) {
    // dH = dO Wd^T (Wd_e is [I, D]) and the SwiGLU adjoint (src/mixtral.rs:478-486)
    ph_begin("expert_dh", s);
    {
      Gemm g1; g1.M = rows_cap; g1.N = I; g1.K = D; g1.A = dO_; g1.lda = D;
      g1.B = P + off.down0; g1.ldb = D; g1.b_t = true; g1.C = dh; g1.ldc = I;
      g1.group = 1; g1.seg_off = seg_off; g1.tile_expert = tile_expert; g1.G = (int)E;
      g1.b_gs = off.expert_stride;
      if (!f32) {
        TcEpilogue te; te.kind = kTcSwiGLUBwd; te.g_in = (const bf16*)g_; te.u_in = (const bf16*)u_;
        te.dg_out = (bf16*)dg_; te.du_out = (bf16*)du_; te.ldg = I;
        gemm_tc(g1, nullptr, 0, te, s, launches);
      } else {
        gemm<Act>(g1, s);
        ph_end(s);
        ph_begin("swiglu_bwd", s);
        silu_mul_bwd<Act>(dh, g_, u_, seg_off, (int)E, I, rows_cap, dg_, du_, s, launches);
      }
    }
    ph_end(s);
    // dWd_e += H^T dO over expert e's rows (src/mixtral.rs:478-480)
    ph_begin("expert_dw_down", s);
    {
      Gemm g2; g2.M = I; g2.N = D; g2.K = rows_cap; g2.A = h_; g2.lda = I; g2.a_t = true;
      g2.B = dO_; g2.ldb = D; g2.C = dP + off.down0; g2.ldc = D; g2.epi = Epi::Accum;
      g2.group = 2; g2.seg_off = seg_off; g2.G = (int)E; g2.c_gs = off.expert_stride;
      gemm<Act>(g2, s);
    }
    ph_end(s);
    // dXp = dG Wg^T + dU Wu^T (Wg_e, Wu_e are [D, I]; src/mixtral.rs:488-516)
    ph_begin("expert_dx", s);
    {
      Gemm g3; g3.M = rows_cap; g3.N = D; g3.K = I; g3.A = dg_; g3.lda = I;
      g3.B = P + off.gate0; g3.ldb = I; g3.b_t = true; g3.C = dxp; g3.ldc = D;
      g3.group = 1; g3.seg_off = seg_off; g3.tile_expert = tile_expert; g3.G = (int)E;
      g3.b_gs = off.expert_stride;
      GemmPart up{du_, I, P + off.up0, I, I};
      gemm<Act>(g3, s, &up, 1);
    }
    ph_end(s);
    // dWg_e += Xp^T dG, dWu_e += Xp^T dU
    ph_begin("expert_dw_gate_up", s);
    {
      Gemm g5; g5.M = D; g5.N = I; g5.K = rows_cap; g5.A = xp_; g5.lda = D; g5.a_t = true;
      g5.B = dg_; g5.ldb = I; g5.C = dP + off.gate0; g5.ldc = I; g5.epi = Epi::Accum;
      g5.group = 2; g5.seg_off = seg_off; g5.G = (int)E; g5.c_gs = off.expert_stride;
      gemm<Act>(g5, s);
      Gemm g6 = g5; g6.B = du_; g6.C = dP + off.up0;
      gemm<Act>(g6, s);
    }
    ph_end(s);
  }
  if (adjoint_stream) {  // the experts' adjoints are final from here on
    if (!expert_adjoint_done)
      DOP_CHECK_CUDA(cudaEventCreateWithFlags(&expert_adjoint_done, cudaEventDisableTiming));
    // expert parallel: final once the owners have added the helpers' partials
    DOP_CHECK_CUDA(cudaEventRecord(expert_adjoint_done, ep ? ep_stream : s));
    DOP_CHECK_CUDA(cudaStreamWaitEvent(adjoint_stream, expert_adjoint_done, 0));
  }
  // d_xn2 = sum_k dXp[row(t,k)] + dz Wr^T; router weight adjoint
  ph_begin("unpermute_router", s);
  if (ep) {  // computed on the exchange stream during the expert adjoints
    DOP_CHECK_CUDA(cudaStreamWaitEvent(s, ep_ev_combined, 0));
  } else {
    unpermute_router_dx<Act>(dxp, slot_row, dz, P + off.router, T, (int)E, (int)K, (int)D, dxn2, s,
                             launches);
  }
  router_dw<Act>(mid, inv2, P + off.ffn_norm, dz, T, (int)D, (int)E, dP + off.router, part,
                 part_cap, s, launches);
  ph_end(s);
  // d_mid = rmsnorm_bwd(d_xn2) + dy (src/mixtral.rs:543-557)
  ph_begin("ffn_norm_bwd", s);
  rmsnorm_bwd<Act>(dxn2, mid, inv2, P + off.ffn_norm, dy, T, (int)D, dmid, f32 ? nullptr : dmid_,
                   dP + off.ffn_norm, part, part_cap, s, launches);
  ph_end(s);
  const Act* dmid_op = f32 ? (const Act*)dmid : dmid_;
  // d_mix = d_mid Wo^T (Wo is [qd, D]); dWo += mix^T d_mid (src/mixtral.rs:560-561)
  ph_begin("o_grad", s);
  {
    Gemm g7; g7.M = T; g7.N = qd; g7.K = D; g7.A = dmid_op; g7.lda = D;
    g7.B = P + off.o; g7.ldb = D; g7.b_t = true; g7.C = dmix_; g7.ldc = qd; g7.c_f32 = f32;
    gemm<Act>(g7, s);
    Gemm g8; g8.M = qd; g8.N = D; g8.K = T; g8.A = mix_; g8.lda = qd; g8.a_t = true;
    g8.B = dmid_op; g8.ldb = D; g8.C = dP + off.o; g8.ldc = D; g8.epi = Epi::Accum;
    gemm<Act>(g8, s);
  }
  ph_end(s);
  ph_begin("attn_bwd", s);
  Attn at; at.B = B; at.S = S; at.H = H; at.KV = KV; at.hd = hd; at.window = cfg.sliding_window;
  at.causal = true; at.scale = 1.0f / sqrtf((float)hd);
  const Act* dv_op;
  if (!f32 && hd == 128) {
    // the attention backward writes bf16 dq, dk (rotated back by the RoPE
    // adjoint) and dv straight from its accumulators
    AttnBwdBf16 o16;
    o16.dq = (bf16*)dq_; o16.dk = (bf16*)dk_; o16.dv = (bf16*)dv_;
    o16.cs = rope_cos; o16.sn = rope_sin;
    attn_bwd_tc(at, (const bf16*)q_, (const bf16*)k_, (const bf16*)v_, (const bf16*)mix_,
                (const bf16*)dmix_, lse, delta, nullptr, nullptr, nullptr, s, launches, &o16);
    dv_op = dv_;
    ph_end(s);
  } else {
    attn_bwd_simt<Act>(at, q_, k_, v_, mix_, dmix_, lse, delta, dq, dk, dv, s, launches);
    ph_end(s);
    ph_begin("rope_bwd", s);
    rope<float, Act>(dq, dq_, T, (int)S, H, hd, rope_cos, rope_sin, -1.f, s, launches);
    rope<float, Act>(dk, dk_, T, (int)S, KV, hd, rope_cos, rope_sin, -1.f, s, launches);
    if (f32) dv_op = (const Act*)dv;
    else { convert<Act>(dv, dv_, T * kvd, s, launches); dv_op = dv_; }
    ph_end(s);
  }
  // d_xn = dq Wq^T + dk Wk^T + dv Wv^T (src/mixtral.rs:571-580)
  ph_begin("qkv_dgrad", s);
  {
    Gemm a1; a1.M = T; a1.N = D; a1.K = qd; a1.A = dq_; a1.lda = qd; a1.B = P + off.q;
    a1.ldb = qd; a1.b_t = true; a1.C = dxn; a1.ldc = D;
    GemmPart kv[2] = {{dk_, kvd, P + off.k, kvd, kvd}, {dv_op, kvd, P + off.v, kvd, kvd}};
    gemm<Act>(a1, s, kv, 2);
  }
  ph_end(s);
  // dWq += xn^T dq, dWk += xn^T dk, dWv += xn^T dv
  ph_begin("qkv_wgrad", s);
  {
    Gemm w1; w1.M = D; w1.N = qd; w1.K = T; w1.A = xn_; w1.lda = D; w1.a_t = true; w1.B = dq_;
    w1.ldb = qd; w1.C = dP + off.q; w1.ldc = qd; w1.epi = Epi::Accum;
    gemm<Act>(w1, s);
    Gemm w2 = w1; w2.N = kvd; w2.B = dk_; w2.ldb = kvd; w2.C = dP + off.k; w2.ldc = kvd;
    gemm<Act>(w2, s);
    Gemm w3 = w2; w3.B = dv_op; w3.C = dP + off.v;
    gemm<Act>(w3, s);
  }
  ph_end(s);
  // dx = rmsnorm_bwd(d_xn) + d_mid (src/mixtral.rs:581-597)
  ph_begin("attn_norm_bwd", s);
  rmsnorm_bwd<Act>(dxn, x_in, inv1, P + off.attn_norm, dmid, T, (int)D, dx, (Act*)nullptr,
                   dP + off.attn_norm, part, part_cap, s, launches);
  ph_end(s);
  // expert parallel: the call's stream also covers the owners' reduction of
  // the helpers' partial adjoints (and orders the next step after it)
  if (ep) DOP_CHECK_CUDA(cudaStreamWaitEvent(s, ep_ev_reduced, 0));
}

}  // namespace dop
