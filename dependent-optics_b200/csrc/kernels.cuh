// kernels.cuh — launchers of every libdop kernel, grouped by file.
#pragma once

#include <cuda.h>

#include <algorithm>

#include "common.cuh"

namespace dop {

constexpr int kMaxExperts = 16;  // router kernels keep E logits in registers
constexpr int kMaxTopK = 4;
constexpr int kRowAlign = 128;   // row tiles of the expert-sorted buffers
constexpr int kSegAlign = 256;   // expert segments start at multiples of this (a
                                 // pair of row tiles: the 2-SM GEMM's 256-row tile)
constexpr int kPermChunk = 1024; // (token, slot) pairs per permutation CTA

// ----------------------------------------------------- elementwise.cu
template <typename T>
void rmsnorm_fwd(const float* x, const T* w, int64_t rows, int D, float eps, T* y, float* inv,
                 float* x_copy, cudaStream_t s, int64_t& launches);
template <typename T>
void rmsnorm_router(const float* x, const T* w, const T* wr, const float* bias, int64_t rows,
                    int D, int E, int K, float eps, T* y, float* inv, float* probs, int* top_i,
                    float* top_p, float* top_w, cudaStream_t s, int64_t& launches);
template <typename T>
void rmsnorm_bwd(const float* dy, const float* x, const float* inv, const T* w, const float* res,
                 int64_t rows, int D, float* dx, T* dx_act, float* dw_accum, float* part_buf,
                 int64_t part_cap, cudaStream_t s, int64_t& launches);
void rope_table(int S, int hd, float theta, float* cs, float* sn, cudaStream_t s,
                int64_t& launches);
template <typename TI, typename TO>
void rope(const TI* src, TO* dst, int64_t T, int S, int heads, int hd, const float* cs,
          const float* sn, float sign, cudaStream_t s, int64_t& launches);
void permute(const int* top_i, const float* top_w, int64_t T, int E, int K, int* chunk_counts,
             int* seg_off, int* tile_expert, int max_tiles, int* slot_row, int* row_token,
             float* row_w, int64_t rows_cap, cudaStream_t s, int64_t& launches);
template <typename T>
void gather_rows(const T* src, const int* row_token, const int* seg_off, int E, int D,
                 int64_t rows_cap, T* dst, cudaStream_t s, int64_t& launches);
// The same rows written token-major (each token row read once, written to its
// K expert rows slot_row[t K + k]; padding rows zeroed).
template <typename T>
void scatter_rows(const T* src, const int* slot_row, int64_t Tn, int K, const int* row_token,
                  const int* seg_off, int E, int D, int64_t rows_cap, T* dst, cudaStream_t s,
                  int64_t& launches);
template <typename T>
void gather_scale_rows(const float* src, const int* row_token, const float* row_w,
                       const int* seg_off, int E, int D, int64_t rows_cap, T* dst, cudaStream_t s,
                       int64_t& launches);
// dst[slot_row[t K + k]] = top_w[t K + k] dy[t] token-major (each dy row read
// once); padding rows zeroed.  Falls back to gather_scale_rows when the rows
// are not 16-byte aligned.
template <typename T>
void scatter_scale_rows(const float* src, const int* slot_row, const float* top_w, int64_t Tn,
                        int K, const int* row_token, const float* row_w, const int* seg_off, int E,
                        int D, int64_t rows_cap, T* dst, cudaStream_t s, int64_t& launches);
template <typename T>
void silu_mul(const T* g, const T* u, const int* seg_off, int E, int64_t I, int64_t rows_cap,
              T* h, cudaStream_t s, int64_t& launches);
template <typename T>
void silu_mul_bwd(const float* dh, const T* g, const T* u, const int* seg_off, int E, int64_t I,
                  int64_t rows_cap, T* dg, T* du, cudaStream_t s, int64_t& launches);
void combine(const float* mid, const float* out, const int* slot_row, const float* top_w,
             int64_t T, int K, int D, float* y, cudaStream_t s, int64_t& launches);
void router_bwd(const float* dy, const float* out, const int* slot_row, const int* top_i,
                const float* top_p, const float* top_w, const float* probs, int64_t Tn, int E,
                int K, int D, float* dz, cudaStream_t s, int64_t& launches);
template <typename T>
void unpermute_router_dx(const float* dxp, const int* slot_row, const float* dz, const T* wr,
                         int64_t Tn, int E, int K, int D, float* dxn, cudaStream_t s,
                         int64_t& launches);
template <typename T>
void router_dw(const float* mid, const float* inv, const T* w, const float* dz, int64_t rows,
               int D, int E, float* dwr_accum, float* part_buf, int64_t part_cap,
               cudaStream_t s, int64_t& launches);
template <typename T>
void convert(const float* src, T* dst, int64_t n, cudaStream_t s, int64_t& launches);
void col_sum(const float* x, int64_t rows, int64_t cols, float* out, float* part_buf,
             int64_t part_cap, bool accumulate, cudaStream_t s, int64_t& launches);
void sgd(float* p, const float* g, int64_t n, float lr, cudaStream_t s, int64_t& launches);
void add_inplace(float* dst, const float* src, int64_t n, cudaStream_t s, int64_t& launches);
void relu_mask_bwd(float* dy, const uint8_t* mask, int64_t n, cudaStream_t s,
                   int64_t& launches);
void mse(const float* y, const float* t, int64_t n, float* loss, float* dy, cudaStream_t s,
         int64_t& launches);

// ------------------------------------------------------------- GEMMs
// C[m, n] (epilogue) sum_k A(m, k) * B(k, n) over fp32 accumulators.
//   A(m, k) = A[m * lda + k]     (a_t = false, K-major)
//           = A[k * lda + m]     (a_t = true,  M-major)
//   B(k, n) = B[k * ldb + n]     (b_t = false, N-major: the crate's W[k*dout+n])
//           = B[n * ldb + k]     (b_t = true,  K-major: W^T)
// group = 1: rows are expert segments of kRowAlign-aligned length
//            (seg_off[G+1], tile_expert[]); B advances b_gs elements per expert.
// group = 2: the contraction runs over expert segment e = blockIdx.z
//            (rows seg_off[e] .. seg_off[e+1]); C advances c_gs per expert.
enum class Epi : int {
  Store = 0,     // C = acc
  Accum = 1,     // C += acc (fp32 C only)
  AddRes = 2,    // C = acc + R (fp32 C only)
  BiasRelu = 3,  // C = acc + bias[n]; if relu: mask = C > 0, C = max(C, 0)
};
struct Gemm {
  int64_t M = 0, N = 0, K = 0;
  const void* A = nullptr; int64_t lda = 0; bool a_t = false;
  const void* B = nullptr; int64_t ldb = 0; bool b_t = false;
  void* C = nullptr; int64_t ldc = 0; bool c_f32 = true;
  Epi epi = Epi::Store;
  const float* R = nullptr; int64_t ldr = 0;
  const float* bias = nullptr; uint8_t* mask = nullptr; bool relu = false;
  int group = 0; const int* seg_off = nullptr; const int* tile_expert = nullptr; int G = 0;
  // group == 2 (grouped contraction) on the tensor cores: group g contracts
  // over rows [seg_off[g], seg_end[g]) instead of [seg_off[g], seg_off[g + 1])
  const int* seg_end = nullptr;
  int64_t b_gs = 0, c_gs = 0;
  // CUDA-core path: fp32 scratch (ws_cap floats) for split-contraction
  // partials; without it a narrow problem runs unsplit
  float* ws = nullptr; int64_t ws_cap = 0;
};
template <typename T>
void gemm_simt(const Gemm& g, cudaStream_t s, int64_t& launches);

// Tensor-core (tcgen05) bf16 GEMM, gemm_tc.cu.  Extra K parts (A_i, B_i) are
// summed into the same accumulator (same majors and grouping as g).  The
// epilogue defaults to g.epi / g.c_f32; TcEpilogue selects the fused SwiGLU
// forward (B = [gate | up], writes g, u, h) or backward (acc = dH; reads g, u,
// writes dG, dU).
struct GemmPart {
  const void* A; int64_t lda; const void* B; int64_t ldb; int64_t K;
};
struct TcEpilogue {
  int kind = -1;  // -1 from Gemm; 4 SwiGLU forward; 5 SwiGLU backward; 6 RoPE
  const void* up_B = nullptr;
  bf16 *g_out = nullptr, *u_out = nullptr, *h_out = nullptr;
  const bf16 *g_in = nullptr, *u_in = nullptr;
  bf16 *dg_out = nullptr, *du_out = nullptr;
  int64_t ldg = 0;
  // kind 6: C (bf16) holds heads of 128 columns rotated by RoPE at position
  // row mod rope_seq, from the [rope_seq][64] cos/sin tables
  const float *rope_cos = nullptr, *rope_sin = nullptr;
  int rope_seq = 0;
};
constexpr int kTcSwiGLU = 4, kTcSwiGLUBwd = 5, kTcRope = 6;
void gemm_tc(const Gemm& g, const GemmPart* extra, int n_extra, const TcEpilogue& te,
             cudaStream_t s, int64_t& launches);
// The fp32 lens's contraction on the tensor cores as three tf32 products
// (3xTF32, gemm_tc.cu): g's fp32 operands are split into tf32 hi / lo parts
// in `ws` (gemm_tc_f32_scratch(g) floats).  gemm_tc_f32_ok: shapes and
// epilogues it takes (fp32 C; store, accumulate or residual add).
bool gemm_tc_f32_ok(const Gemm& g);
int64_t gemm_tc_f32_scratch(const Gemm& g);
void gemm_tc_f32(const Gemm& g, float* ws, int64_t ws_cap, cudaStream_t s, int64_t& launches);
// 3-D bf16 TMA descriptor, 128-byte swizzle: extents dims (dims[0]
// contiguous), strides of dims 1 and 2 in elements, box extents.
CUtensorMap make_map3(const void* base, const int64_t dims[3], const int64_t strides[2],
                      const int box[3]);
// First bounded-wait failure recorded by a tensor-core kernel (0 = none).
int tc_error_status();

// ------------------------------------------------------------ attention
// Sliding-window causal grouped-query attention (src/mixtral.rs:799-922),
// flash-style: the residual is the log-sum-exp per (b, h, query), not the
// probabilities.  q [T, H, hd], k/v [T, KV, hd]; causal = false drops the
// mask (kernel.rs Q=K=V=X attention, src/kernel.rs:256-291).
struct Attn {
  int64_t B = 0, S = 0; int H = 0, KV = 0, hd = 0; int64_t window = 0; bool causal = true;
  float scale = 1.f;
};
template <typename T>
void attn_fwd_simt(const Attn& a, const T* q, const T* k, const T* v, T* o, float* lse,
                   cudaStream_t s, int64_t& launches);
// Tensor-core (tcgen05) flash attention for bf16, head_dim 128 (attn_tc.cu).
void attn_fwd_tc(const Attn& a, const bf16* q, const bf16* k, const bf16* v, bf16* o, float* lse,
                 cudaStream_t s, int64_t& launches);
// Optional bf16 outputs of attn_bwd_tc: dq, dk, dv rounded once from the fp32
// accumulators, dq and dk rotated back by the RoPE adjoint (tables cs, sn of
// [S][hd/2], position = index within the sequence) when cs is set.  With
// them the fp32 dq, dk, dv are not written.
struct AttnBwdBf16 {
  bf16* dq = nullptr; bf16* dk = nullptr; bf16* dv = nullptr;
  const float* cs = nullptr; const float* sn = nullptr;
};
void attn_bwd_tc(const Attn& a, const bf16* q, const bf16* k, const bf16* v, const bf16* o,
                 const bf16* dout, const float* lse, float* delta, float* dq, float* dk, float* dv,
                 cudaStream_t s, int64_t& launches, const AttnBwdBf16* out16 = nullptr);
// y = 2^x by the polynomial the tensor-core softmax evaluates on the FMA
// pipe for part of its exponentials (attn_tc.cu); x < 128.
namespace tc {
void exp2_poly(const float* x, float* y, int64_t n, cudaStream_t s, int64_t& launches);
}
template <typename T>
void attn_bwd_simt(const Attn& a, const T* q, const T* k, const T* v, const T* o, const T* dout,
                   const float* lse, float* delta, float* dq, float* dk, float* dv,
                   cudaStream_t s, int64_t& launches);

}  // namespace dop
