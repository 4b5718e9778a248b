// block.cuh — the Mixtral block lens (get = forward, put = backward) and its
// device residual.
#pragma once

#include "../../include/dop.h"
#include <vector>

#include "ep.cuh"
#include "kernels.cuh"

namespace dop {

// Offsets of one layer's parameters inside its slice (src/mixtral.rs:135-171).
struct LayerOffsets {
  int64_t attn_norm, q, k, v, o, ffn_norm, router, gate0, up0, down0, expert_stride, total;
};
LayerOffsets layer_offsets(const dop_mixtral_cfg& c);

// Device residual of one block.  Unlike the crate's LayerTape
// (src/mixtral.rs:212-228) it holds the attention log-sum-exp instead of the
// probabilities, the post-RoPE q/k instead of the pre-RoPE ones, and the
// expert activations in expert-sorted (permuted) order.
struct Block {
  dop_mixtral_cfg cfg{};
  int64_t B = 0, S = 0, T = 0;
  int prec = DOP_F32;
  LayerOffsets off{};
  int64_t rows_cap = 0;   // capacity of the expert-sorted buffers
  int max_tiles = 0;      // rows_cap / kRowAlign
  int64_t launches = 0;
  bool have_tape = false;
  const float* router_bias = nullptr;
  cudaStream_t adjoint_stream = nullptr;  // waits for the experts' adjoints
  cudaEvent_t expert_adjoint_done = nullptr;
  size_t bytes = 0;
  char* base = nullptr;   // one device allocation, carved below

  // residual (forward -> backward)
  float *x_in, *inv1, *mid, *inv2, *lse, *probs, *top_p, *top_w, *row_w, *out;
  int *top_i, *slot_row, *seg_off, *tile_expert, *row_token, *chunk_counts;
  void *xn, *q, *k, *v, *mix, *xn2, *xp, *g, *u, *h;
  // forward scratch
  float *qpre, *kpre, *rope_cos, *rope_sin;
  // backward scratch
  float *dz, *dh, *dxp, *dxn2, *dmid, *dxn, *dq, *dk, *dv, *delta, *part;
  int64_t part_cap;
  float* split_ws = nullptr;  // fp32 lens: split-contraction partials (gemm_simt)
  int64_t split_cap = 0;
  float* tf32_ws = nullptr;   // fp32 lens: tf32 hi / lo operands (gemm_tc_f32)
  int64_t tf32_cap = 0;
  void *dO, *dg, *du, *dmid_a, *dmix, *dq_a, *dk_a, *dv_a;

  // expert parallelism (ep_world > 1, bf16 only; ep.cu): this rank owns the
  // adjoint of experts [ep_rank * ep_local, (ep_rank + 1) * ep_local) and
  // processes the chunk of every rank's routed rows that the step's plan
  // gives it (capacity recv_cap = ep_world * rows_cap, the most any routing
  // can send).  The receive buffers of g and u are reused for dg and du (the
  // SwiGLU adjoint reads each element before it writes it).
  int ep_rank = 0, ep_world = 1, ep_local = 0;
  int64_t recv_cap = 0;
  unsigned ep_epoch = 0;
  std::vector<char*> ep_peer_base;  // workspace bases as mapped here, [ep_world]
  char** ep_peers_dev = nullptr;    // device copy of ep_peer_base
  unsigned* ep_flags = nullptr;
  cudaStream_t ep_stream = nullptr;  // the backward combine, beside the dW GEMMs
  cudaEvent_t ep_ev_dx = nullptr, ep_ev_combined = nullptr;
  cudaEvent_t ep_ev_dw = nullptr, ep_ev_reduced = nullptr;
  int *piece_pos = nullptr, *ep_bounds = nullptr, *recv_seg_off = nullptr;
  int *own_end = nullptr, *help_end = nullptr, *helpers = nullptr, *recv_tile_expert = nullptr;
  int *recv_tile_src = nullptr, *recv_tile_row0 = nullptr;
  void *xr = nullptr, *gr = nullptr, *ur = nullptr, *hr = nullptr, *dOr = nullptr;
  float *outr = nullptr, *dxpr = nullptr;
  float* dw_help = nullptr;  // [E][expert_stride] partial adjoints of experts owned elsewhere
  EpView ep_view() const;
  void ep_barrier_next(int k, cudaStream_t s);
  // Map the peers' workspaces (handles in rank order; own entry ignored).
  void ep_connect(const cudaIpcMemHandle_t* handles);

  // per-phase CUDA-event timing (dop_block_set_timing)
  struct Phase { const char* name; cudaEvent_t a, b; };
  bool timing = false;
  std::vector<Phase> phases;
  size_t n_phases = 0, n_fwd_phases = 0;
  const char* cur_phase = "";
  void ph_begin(const char* name, cudaStream_t s);
  void ph_end(cudaStream_t s);

  // allocate = false only computes `bytes` (the workspace a handle would
  // hold) without touching the device.
  Block(const dop_mixtral_cfg& c, int64_t batch, int64_t seq, int precision, int rank = 0,
        int world = 1, bool allocate = true);
  ~Block();
  void forward(const void* params, const float* x, float* y, cudaStream_t s);
  void backward(const void* params, const float* dy, float* dx, float* dparams, cudaStream_t s);

 private:
  template <typename Act> void fwd(const Act* P, const float* x, float* y, cudaStream_t s);
  template <typename Act> void bwd(const Act* P, const float* dy, float* dx, float* dP, cudaStream_t s);
  template <typename Act>
  void gemm(const Gemm& g, cudaStream_t s, const GemmPart* extra = nullptr, int n_extra = 0);
  void ep_fwd_experts(const bf16* P, float* y, cudaStream_t s);
  void ep_bwd_experts(const bf16* P, float* dP, cudaStream_t s);
};

}  // namespace dop
