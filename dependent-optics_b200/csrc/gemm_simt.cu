// gemm_simt.cu — CUDA-core fp32-accumulate GEMM.
//
// This is the contraction of the fp32 lens (precision DOP_F32): the crate's
// `linear`/`linear_bwd`/`gemm` (src/mixtral.rs:616-659, src/kernel.rs:242-254,
// 320-352) at fp32 accuracy, which tf32/bf16 tensor cores cannot give.  It
// supports both operand majors, the bias/ReLU/residual/accumulate epilogues
// and the expert-grouped forms of kernels.cuh.
//
// Tiles of 128 x 128 (8 x 8 outputs per thread) or 64 x 64 (4 x 4) by 16,
// 256 threads, double-buffered shared-memory stages, operands read from
// shared memory as float4.  Problems whose
// 128 x 128 tiles would leave most SMs idle (weight gradients of narrow
// layers, whose contraction runs over every token) take 64 x 64 tiles and,
// when the caller lends a workspace, a split of the contraction: each split
// writes its partial tile to the workspace and one pass sums the partials in
// split order and applies the epilogue, so results stay deterministic.
#include "kernels.cuh"

namespace dop {

namespace {

constexpr int BK = 16, NT = 256;
constexpr int kSplitGroup = 3;  // Args::group of a split-contraction launch

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
  int64_t kc;  // contraction length of one split (group kSplitGroup)
};

// C[m, n] = epilogue(v) for the fp32 sum v of output (m, n).
template <typename TC>
__device__ __forceinline__ void store_out(const Args& g, TC* C, int64_t m, int64_t n, float v) {
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

template <typename T, bool AT, bool BT, typename TC, int BM, int BN>
__global__ __launch_bounds__(NT) void k_gemm_simt(Args g) {
  // Thread (tx, ty) of the 16 x 16 grid owns TM rows in GM groups of four,
  // {q BM/GM + 4 ty + r}, and TN columns likewise, so that its operands are
  // float4 shared-memory reads and the 16 threads of a row read consecutive
  // 16-byte words (no bank conflicts).
  constexpr int TM = BM / 16, TN = BN / 16;      // outputs per thread
  constexpr int GM = TM / 4, GN = TN / 4;        // groups of four rows / columns
  constexpr int LA = BM * BK / NT, LB = BN * BK / NT;  // loads per thread
  static_assert(TM % 4 == 0 && TN % 4 == 0, "four-wide thread fragments");
  static_assert(NT % BM == 0 && NT % BN == 0 && NT % BK == 0, "tile and thread counts");
  static_assert(kRowAlign % BM == 0, "grouped-M tiles must not straddle a segment");
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];
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
    const int e = g.tile_expert[m0 / kRowAlign];
    if (e < 0) return;
    B += (int64_t)e * g.b_gs;
  } else if (g.group == 2) {
    const int e = blockIdx.z;
    kbeg = g.seg_off[e];
    kend = g.seg_off[e + 1];
    C += (int64_t)e * g.c_gs;
  } else if (g.group == kSplitGroup) {
    kbeg = (int64_t)blockIdx.z * g.kc;
    kend = kbeg + g.kc < g.K ? kbeg + g.kc : g.K;
    C += (int64_t)blockIdx.z * g.c_gs;
  }
  if (m0 >= M || n0 >= g.N) return;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  float ra[LA], rb[LB];
  auto load = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < LA; ++i) {
      int mm, kk;
      if (!AT) { kk = tid % BK; mm = tid / BK + (NT / BK) * i; }
      else { mm = tid % BM; kk = tid / BM + (NT / BM) * i; }
      int64_t m = m0 + mm, k = k0 + kk;
      float v = 0.f;
      if (m < M && k < kend) v = ld(AT ? &A[k * g.lda + m] : &A[m * g.lda + k]);
      ra[i] = v;
    }
#pragma unroll
    for (int i = 0; i < LB; ++i) {
      int nn, kk;
      if (!BT) { nn = tid % BN; kk = tid / BN + (NT / BN) * i; }
      else { kk = tid % BK; nn = tid / BK + (NT / BK) * i; }
      int64_t n = n0 + nn, k = k0 + kk;
      float v = 0.f;
      if (n < g.N && k < kend) v = ld(BT ? &B[n * g.ldb + k] : &B[k * g.ldb + n]);
      rb[i] = v;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < LA; ++i) {
      int mm, kk;
      if (!AT) { kk = tid % BK; mm = tid / BK + (NT / BK) * i; }
      else { mm = tid % BM; kk = tid / BM + (NT / BM) * i; }
      As[buf][kk][mm] = ra[i];
    }
#pragma unroll
    for (int i = 0; i < LB; ++i) {
      int nn, kk;
      if (!BT) { nn = tid % BN; kk = tid / BN + (NT / BN) * i; }
      else { kk = tid % BK; nn = tid / BK + (NT / BK) * i; }
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
      float a[TM], b[TN];
#pragma unroll
      for (int q = 0; q < TM / 4; ++q)
        *reinterpret_cast<float4*>(&a[4 * q]) =
            *reinterpret_cast<const float4*>(&As[buf][kk][q * (BM / GM) + 4 * ty]);
#pragma unroll
      for (int q = 0; q < TN / 4; ++q)
        *reinterpret_cast<float4*>(&b[4 * q]) =
            *reinterpret_cast<const float4*>(&Bs[buf][kk][q * (BN / GN) + 4 * tx]);
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = m0 + (i / 4) * (BM / GM) + 4 * ty + (i % 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t n = n0 + (j / 4) * (BN / GN) + 4 * tx + (j % 4);
      if (n >= g.N) continue;
      store_out(g, C, m, n, acc[i][j]);
    }
  }
}

// Sum of the splits' partial tiles (ws[z][M][N], z in increasing order), then
// the epilogue of the original launch.
template <typename TC>
__global__ void k_split_reduce(const float* __restrict__ ws, int splits, Args g) {
  const int64_t MN = g.M * g.N;
  TC* C = (TC*)g.C;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < MN;
       idx += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += ws[(int64_t)z * MN + idx];
    store_out(g, C, idx / g.N, idx % g.N, v);
  }
}

template <typename T, bool AT, bool BT, typename TC>
void launch_majors(const Args& a, dim3 grid, bool small, cudaStream_t s) {
  if (small)
    k_gemm_simt<T, AT, BT, TC, 64, 64><<<grid, NT, 0, s>>>(a);
  else
    k_gemm_simt<T, AT, BT, TC, 128, 128><<<grid, NT, 0, s>>>(a);
}

template <typename T, typename TC>
void launch(const Gemm& g, const Args& a, dim3 grid, bool small, cudaStream_t s) {
  if (!g.a_t && !g.b_t) launch_majors<T, false, false, TC>(a, grid, small, s);
  else if (!g.a_t && g.b_t) launch_majors<T, false, true, TC>(a, grid, small, s);
  else if (g.a_t && !g.b_t) launch_majors<T, true, false, TC>(a, grid, small, s);
  else launch_majors<T, true, true, TC>(a, grid, small, s);
}

}  // namespace

template <typename T>
void gemm_simt(const Gemm& g, cudaStream_t s, int64_t& launches) {
  DOP_REQUIRE(g.M >= 0 && g.N >= 0 && g.K >= 0, "negative GEMM extent");
  DOP_REQUIRE(g.epi == Epi::Store || g.c_f32, "accumulating epilogues need an fp32 C");
  if (g.M == 0 || g.N == 0) return;
  Args a{g.M, g.N, g.K, g.A, g.lda, g.B, g.ldb, g.C, g.ldc, (int)g.epi, g.R, g.ldr,
         g.bias, g.mask, g.relu ? 1 : 0, g.group, g.seg_off, g.tile_expert, g.G, g.b_gs, g.c_gs, 0};
  const int64_t z = g.group == 2 ? g.G : 1;
  const int64_t sms = sm_count();
  const bool small = ceil_div(g.M, 128) * ceil_div(g.N, 128) * z < sms;
  const int tile = small ? 64 : 128;
  dim3 grid((unsigned)ceil_div(g.N, tile), (unsigned)ceil_div(g.M, tile), (unsigned)z);
  DOP_REQUIRE(grid.y < 65536, "GEMM M too large for the CUDA-core path");
  // split the contraction when even the small tiles leave SMs idle: about
  // two CTAs per SM, at least 256 of K per split, partials within the workspace
  int splits = 1;
  const int64_t tiles = (int64_t)grid.x * grid.y;
  if (g.group == 0 && small && g.ws && tiles < sms) {
    int64_t sp = std::min<int64_t>({ceil_div(2 * sms, tiles), g.K / 256, 16,
                                    g.ws_cap / (g.M * g.N)});
    splits = (int)std::max<int64_t>(1, sp);
  }
  if (splits > 1) {
    Args p = a;
    p.group = kSplitGroup;
    p.kc = round_up(ceil_div(g.K, splits), BK);
    splits = (int)ceil_div(g.K, p.kc);
    p.C = g.ws; p.ldc = g.N; p.c_gs = g.M * g.N;
    p.epi = (int)Epi::Store;
    grid.z = (unsigned)splits;
    launch<T, float>(g, p, grid, true, s);
    DOP_LAUNCHED(launches);
    const unsigned rb = (unsigned)std::min<int64_t>(ceil_div(g.M * g.N, 256), 8 * sms);
    if (g.c_f32)
      k_split_reduce<float><<<rb, 256, 0, s>>>(g.ws, splits, a);
    else
      k_split_reduce<T><<<rb, 256, 0, s>>>(g.ws, splits, a);
    DOP_LAUNCHED(launches);
    return;
  }
  if (g.c_f32) launch<T, float>(g, a, grid, small, s);
  else launch<T, T>(g, a, grid, small, s);
  DOP_LAUNCHED(launches);
}

template void gemm_simt<float>(const Gemm&, cudaStream_t, int64_t&);
template void gemm_simt<bf16>(const Gemm&, cudaStream_t, int64_t&);

}  // namespace dop
