// gemm_simt.cu — CUDA-core fp32-accumulate GEMM.
//
// This is the contraction of the fp32 lens (precision DOP_F32): the crate's
// `linear`/`linear_bwd`/`gemm` (src/mixtral.rs:616-659, src/kernel.rs:242-254,
// 320-352) at fp32 accuracy, which tf32/bf16 tensor cores cannot give.  It
// supports both operand majors, the bias/ReLU/residual/accumulate epilogues
// and the expert-grouped forms of kernels.cuh.
//
// Tile 128 x 128 x 16, 256 threads, 8 x 8 outputs per thread, double-buffered
// shared-memory stages.
#include "kernels.cuh"

namespace dop {

namespace {

constexpr int BM = 128, BN = 128, BK = 16, NT = 256;
static_assert(BM == kRowAlign, "grouped-M tiles must match the segment alignment");

struct Args {
  int64_t M, N, K;
  const void* A; int64_t lda;
  const void* B; int64_t ldb;
  void* C; int64_t ldc;
  int epi;
  const float* R; int64_t ldr;
  const float* bias; uint8_t* mask; int relu;
  int group; const int* seg_off; const int* tile_expert; int G;
  int64_t b_gs, c_gs;
};

template <typename T, bool AT, bool BT, typename TC>
__global__ __launch_bounds__(NT) void k_gemm_simt(Args g) {
  __shared__ float As[2][BK][BM + 4];
  __shared__ float Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const T* A = (const T*)g.A;
  const T* B = (const T*)g.B;
  TC* C = (TC*)g.C;
  int64_t M = g.M, kbeg = 0, kend = g.K;
  if (g.group == 1) {
    M = g.seg_off[g.G];
    if (m0 >= M) return;
    const int e = g.tile_expert[m0 / BM];
    if (e < 0) return;
    B += (int64_t)e * g.b_gs;
  } else if (g.group == 2) {
    const int e = blockIdx.z;
    kbeg = g.seg_off[e];
    kend = g.seg_off[e + 1];
    C += (int64_t)e * g.c_gs;
  }
  if (m0 >= M || n0 >= g.N) return;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[8], rb[8];
  auto load = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int mm, kk;
      if (!AT) { kk = tid % BK; mm = tid / BK + 16 * i; }
      else { mm = tid % BM; kk = tid / BM + 2 * i; }
      int64_t m = m0 + mm, k = k0 + kk;
      float v = 0.f;
      if (m < M && k < kend) v = ld(AT ? &A[k * g.lda + m] : &A[m * g.lda + k]);
      ra[i] = v;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int nn, kk;
      if (!BT) { nn = tid % BN; kk = tid / BN + 2 * i; }
      else { kk = tid % BK; nn = tid / BK + 16 * i; }
      int64_t n = n0 + nn, k = k0 + kk;
      float v = 0.f;
      if (n < g.N && k < kend) v = ld(BT ? &B[n * g.ldb + k] : &B[k * g.ldb + n]);
      rb[i] = v;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int mm, kk;
      if (!AT) { kk = tid % BK; mm = tid / BK + 16 * i; }
      else { mm = tid % BM; kk = tid / BM + 2 * i; }
      As[buf][kk][mm] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int nn, kk;
      if (!BT) { nn = tid % BN; kk = tid / BN + 2 * i; }
      else { kk = tid % BK; nn = tid / BK + 16 * i; }
      Bs[buf][kk][nn] = rb[i];
    }
  };

  int buf = 0;
  if (kbeg < kend) {
    load(kbeg);
    store(0);
  }
  __syncthreads();
  for (int64_t k0 = kbeg; k0 < kend; k0 += BK) {
    const bool more = k0 + BK < kend;
    if (more) load(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[buf][kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[buf][kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + tx + 16 * j;
      if (n >= g.N) continue;
      float v = acc[i][j];
      TC* c = &C[m * g.ldc + n];
      if (g.epi == (int)Epi::Accum) {
        v += ld(c);
      } else if (g.epi == (int)Epi::AddRes) {
        v += g.R[m * g.ldr + n];
      } else if (g.epi == (int)Epi::BiasRelu) {
        v += g.bias[n];
        if (g.relu) {
          bool on = v > 0.f;
          g.mask[m * g.N + n] = on ? 1 : 0;
          if (!on) v = 0.f;
        }
      }
      st(c, v);
    }
  }
}

template <typename T, bool AT, bool BT>
void launch_tc(const Gemm& g, const Args& a, dim3 grid, cudaStream_t s) {
  if (g.c_f32)
    k_gemm_simt<T, AT, BT, float><<<grid, NT, 0, s>>>(a);
  else
    k_gemm_simt<T, AT, BT, T><<<grid, NT, 0, s>>>(a);
}

}  // namespace

template <typename T>
void gemm_simt(const Gemm& g, cudaStream_t s, int64_t& launches) {
  DOP_REQUIRE(g.M >= 0 && g.N >= 0 && g.K >= 0, "negative GEMM extent");
  DOP_REQUIRE(g.epi == Epi::Store || g.c_f32, "accumulating epilogues need an fp32 C");
  if (g.M == 0 || g.N == 0) return;
  Args a{g.M, g.N, g.K, g.A, g.lda, g.B, g.ldb, g.C, g.ldc, (int)g.epi, g.R, g.ldr,
         g.bias, g.mask, g.relu ? 1 : 0, g.group, g.seg_off, g.tile_expert, g.G, g.b_gs, g.c_gs};
  dim3 grid((unsigned)ceil_div(g.N, BN), (unsigned)ceil_div(g.M, BM),
            g.group == 2 ? (unsigned)g.G : 1u);
  DOP_REQUIRE(grid.y < 65536, "GEMM M too large for the CUDA-core path");
  if (!g.a_t && !g.b_t) launch_tc<T, false, false>(g, a, grid, s);
  else if (!g.a_t && g.b_t) launch_tc<T, false, true>(g, a, grid, s);
  else if (g.a_t && !g.b_t) launch_tc<T, true, false>(g, a, grid, s);
  else launch_tc<T, true, true>(g, a, grid, s);
  DOP_LAUNCHED(launches);
}

template void gemm_simt<float>(const Gemm&, cudaStream_t, int64_t&);
template void gemm_simt<bf16>(const Gemm&, cudaStream_t, int64_t&);

}  // namespace dop
