// attn_simt.cu — CUDA-core flash attention, forward and backward, fp32
// arithmetic on fp32 or bf16 storage.
//
// Computes the crate's sliding-window grouped-query attention (gqa_forward /
// gqa_backward, src/mixtral.rs:799-922; visible(q, k) = k <= q && q - k < W)
// and the unmasked Q=K=V=X attention of src/kernel.rs:256-447, without
// materialising probabilities: the forward keeps the row log-sum-exp, the
// backward recomputes P from it.
//
// Every contraction is a 64 x 64 register-tiled product out of shared memory:
// 256 threads, each owning a 4 x 4 block of the score tile (and 4 rows x 4*G
// columns of an output tile), with both operands of a product stored
// contraction-major so that one k step is two float4 loads and 16 FMAs.  Head
// dimensions are padded with zeros to HDP = 32, 64 or 128.
//
//   forward  grid (query tiles, H, B): S = Q K^T, online softmax, O += P V.
//   dQ       grid (query tiles, H, B): recompute S and dP = dO V^T per key
//            tile, dS = P (dP - delta), dQ += dS K.
//   dK, dV   grid (key tiles * C, KV, B) in clusters of C CTAs: the C CTAs of
//            a cluster take the query heads of one KV head's group in turn
//            (head rank, rank + C, ...), accumulate partial dK, dV in
//            registers and sum them through distributed shared memory in rank
//            order, so no atomics are needed and results are bitwise
//            reproducible.
//
// This is the fp32 lens's attention (DOP_F32) and supports head_dim <= 128.
#include <cooperative_groups.h>

#include <initializer_list>

#include "kernels.cuh"

namespace dop {

namespace {

namespace cg = cooperative_groups;

constexpr int TB = 64;      // queries or keys per tile
constexpr int TP = TB + 4;  // pitch of contraction-major tiles ([HDP][TP]) and of P / dS
constexpr int NTH = 256;

template <int HDP>
struct Dim {
  static constexpr int RP = HDP + 4;               // pitch of row-major tiles [TB][RP]
  static constexpr int NDG = HDP / 4;              // float4 groups of a row
  static constexpr int GPT = (NDG + 15) / 16;      // groups per thread of an output row
  static constexpr size_t fwd_smem = sizeof(float) * (2 * HDP * TP + TB * RP + TB * TP);
  static constexpr size_t dq_smem = sizeof(float) * (4 * HDP * TP + TB * RP + TB * TP);
  static constexpr size_t dkdv_smem = sizeof(float) * (4 * HDP * TP + 2 * TB * RP + TB * TP);
};

__device__ __forceinline__ bool vis(const Attn& a, int64_t q, int64_t k) {
  if (q >= a.S || k >= a.S) return false;
  if (!a.causal) return true;
  return k <= q && q - k < a.window;
}

// c[i][j] += a[i] * b[j]
__device__ __forceinline__ void outer(float (&c)[4][4], float4 a, float4 b) {
  const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = fmaf(av[i], bv[j], c[i][j]);
}
__device__ __forceinline__ float4 lds4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// Four elements (n of them valid, n may be <= 0) of a row as floats.
template <typename T>
__device__ __forceinline__ float4 load4(const T* p, int n, bool vec) {
  if (vec && n >= 4) return ld4(p);
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (n > 0) r.x = ld(p);
  if (n > 1) r.y = ld(p + 1);
  if (n > 2) r.z = ld(p + 2);
  if (n > 3) r.w = ld(p + 3);
  return r;
}

// Rows [row0, row0 + TB) of one head (base = row 0 of that head, row stride
// `stride` elements), zero past S and past hd, into a contraction-major tile
// t[d][r] (pitch TP) and / or a row-major tile rm[r][d] (pitch HDP + 4).  Lanes
// run over rows, so both shared-memory stores are conflict-free.
template <typename T, int HDP>
__device__ __forceinline__ void load_tile(const T* __restrict__ base, int64_t stride, int64_t row0,
                                          int64_t S, int hd, bool vec, float* t, float* rm) {
  for (int i = threadIdx.x; i < TB * Dim<HDP>::NDG; i += NTH) {
    const int r = i & (TB - 1), g = i / TB;
    const int64_t row = row0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < S) v = load4(base + row * stride + 4 * g, hd - 4 * g, vec);
    if (t) {
      t[(4 * g + 0) * TP + r] = v.x;
      t[(4 * g + 1) * TP + r] = v.y;
      t[(4 * g + 2) * TP + r] = v.z;
      t[(4 * g + 3) * TP + r] = v.w;
    }
    if (rm) *reinterpret_cast<float4*>(&rm[r * Dim<HDP>::RP + 4 * g]) = v;
  }
}

// acc[i][4*gi + e] += sum_k A[k][4*ty + i] * B[k][4*(tx + 16*gi) + e] over k < TB:
// A contraction-major with pitch TP, B row-major with pitch HDP + 4.
template <int HDP>
__device__ __forceinline__ void product_out(float (&acc)[4][4 * Dim<HDP>::GPT], const float* A,
                                            const float* B, int tx, int ty) {
  constexpr int GPT = Dim<HDP>::GPT, NDG = Dim<HDP>::NDG, RP = Dim<HDP>::RP;
#pragma unroll 4
  for (int k = 0; k < TB; ++k) {
    const float4 a = lds4(&A[k * TP + 4 * ty]);
#pragma unroll
    for (int gi = 0; gi < GPT; ++gi) {
      const int g = tx + 16 * gi;
      if (NDG % 16 == 0 || g < NDG) {
        const float4 b = lds4(&B[k * RP + 4 * g]);
        float c[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) c[i][e] = acc[i][4 * gi + e];
        outer(c, a, b);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][4 * gi + e] = c[i][e];
      }
    }
  }
}

// Rows 4*ty + i of an output tile (columns 4*(tx + 16*gi) + e < hd) to
// dst[row * stride + d] for rows < S, each value times mul[i].
template <typename T, int HDP>
__device__ __forceinline__ void store_out(T* __restrict__ base, int64_t stride, int64_t row0,
                                          int64_t S, int hd, bool vec,
                                          const float (&acc)[4][4 * Dim<HDP>::GPT],
                                          const float (&mul)[4], int tx, int ty) {
  constexpr int GPT = Dim<HDP>::GPT, NDG = Dim<HDP>::NDG;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = row0 + 4 * ty + i;
    if (row >= S) continue;
#pragma unroll
    for (int gi = 0; gi < GPT; ++gi) {
      const int g = tx + 16 * gi;
      if (g >= NDG || 4 * g >= hd) continue;
      T* p = base + row * stride + 4 * g;
      const float4 v = make_float4(acc[i][4 * gi] * mul[i], acc[i][4 * gi + 1] * mul[i],
                                   acc[i][4 * gi + 2] * mul[i], acc[i][4 * gi + 3] * mul[i]);
      if (vec && 4 * g + 4 <= hd) {
        st4(p, v);
      } else {
        if (4 * g + 0 < hd) st(p + 0, v.x);
        if (4 * g + 1 < hd) st(p + 1, v.y);
        if (4 * g + 2 < hd) st(p + 2, v.z);
        if (4 * g + 3 < hd) st(p + 3, v.w);
      }
    }
  }
}

// Key tiles a query tile starting at q0 sees: [kbeg, kend), kbeg tile-aligned.
__device__ __forceinline__ void key_range(const Attn& a, int64_t q0, int64_t& kbeg,
                                          int64_t& kend) {
  kbeg = 0;
  kend = a.S;
  if (a.causal) {
    kbeg = q0 - a.window + 1;
    if (kbeg < 0) kbeg = 0;
    kend = q0 + TB < a.S ? q0 + TB : a.S;
  }
  kbeg = kbeg / TB * TB;
}

// Forward.  grid (ceil(S/TB), H, B).
template <typename T, int HDP>
__global__ __launch_bounds__(NTH) void k_attn_fwd(Attn a, const T* __restrict__ q,
                                                  const T* __restrict__ k,
                                                  const T* __restrict__ v, T* __restrict__ o,
                                                  float* __restrict__ lse, bool vec) {
  constexpr int GPT = Dim<HDP>::GPT;
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;                 // [HDP][TP]
  float* Kt = Qt + HDP * TP;      // [HDP][TP]
  float* Vr = Kt + HDP * TP;      // [TB][RP]
  float* Pt = Vr + TB * Dim<HDP>::RP;  // [TB keys][TP]
  const int64_t b = blockIdx.z;
  const int h = blockIdx.y, kvh = h / (a.H / a.KV), hd = a.hd;
  const int64_t q0 = (int64_t)blockIdx.x * TB;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  const T* qb = q + b * a.S * qstride + (int64_t)h * hd;
  const T* kb = k + b * a.S * kstride + (int64_t)kvh * hd;
  const T* vb = v + b * a.S * kstride + (int64_t)kvh * hd;
  load_tile<T, HDP>(qb, qstride, q0, a.S, hd, vec, Qt, nullptr);
  float m_run[4], l_run[4], acc[4][4 * GPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4 * GPT; ++c) acc[i][c] = 0.f;
  }
  int64_t kbeg, kend;
  key_range(a, q0, kbeg, kend);
  for (int64_t k0 = kbeg; k0 < kend; k0 += TB) {
    __syncthreads();
    load_tile<T, HDP>(kb, kstride, k0, a.S, hd, vec, Kt, nullptr);
    load_tile<T, HDP>(vb, kstride, k0, a.S, hd, vec, nullptr, Vr);
    __syncthreads();
    float s[4][4] = {};
#pragma unroll 8
    for (int d = 0; d < HDP; ++d) outer(s, lds4(&Qt[d * TP + 4 * ty]), lds4(&Kt[d * TP + 4 * tx]));
    float p[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + 4 * ty + i;
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = vis(a, qi, k0 + 4 * tx + j) ? s[i][j] * a.scale : -INFINITY;
        mt = fmaxf(mt, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_run[i], mt);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p[i][j] = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - m_new);
        rs += p[i][j];
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      const float alpha = m_run[i] == -INFINITY ? (m_new == -INFINITY ? 1.f : 0.f)
                                                : expf(m_run[i] - m_new);
      l_run[i] = l_run[i] * alpha + rs;
      m_run[i] = m_new;
#pragma unroll
      for (int c = 0; c < 4 * GPT; ++c) acc[i][c] *= alpha;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(&Pt[(4 * tx + j) * TP + 4 * ty]) =
          make_float4(p[0][j], p[1][j], p[2][j], p[3][j]);
    __syncthreads();
    product_out<HDP>(acc, Pt, Vr, tx, ty);
  }
  float inv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) inv[i] = 1.0f / l_run[i];
  store_out<T, HDP>(o + b * a.S * qstride + (int64_t)h * hd, qstride, q0, a.S, hd, vec, acc,
                    inv, tx, ty);
  if (tx == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + 4 * ty + i;
      if (qi < a.S) lse[(b * a.H + h) * a.S + qi] = m_run[i] + logf(l_run[i]);
    }
  }
}

// delta[b,h,i] = sum_d dO[i,d] * O[i,d]  (= sum_j P_ij dA_ij of gqa_backward)
template <typename T>
__global__ void k_attn_delta(Attn a, const T* __restrict__ o, const T* __restrict__ dout,
                             float* __restrict__ delta) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t total = a.B * a.S * a.H;
  if (row >= total) return;
  const int64_t t = row / a.H;
  const int h = (int)(row % a.H);
  const int64_t base = t * a.H * a.hd + (int64_t)h * a.hd;
  float s = 0.f;
  for (int d = lane; d < a.hd; d += 32) s += ld(&dout[base + d]) * ld(&o[base + d]);
  s = warp_sum(s);
  const int64_t b = t / a.S, i = t % a.S;
  if (lane == 0) delta[(b * a.H + h) * a.S + i] = s;
}

// dQ.  grid (ceil(S/TB), H, B).  The score tile is held key-major (thread:
// keys 4*ty + i, queries 4*tx + j) so that dS lands in shared memory as the
// contraction-major operand of dQ += dS K.
template <typename T, int HDP>
__global__ __launch_bounds__(NTH) void k_attn_dq(Attn a, const T* __restrict__ q,
                                                 const T* __restrict__ k,
                                                 const T* __restrict__ v,
                                                 const T* __restrict__ dout,
                                                 const float* __restrict__ lse,
                                                 const float* __restrict__ delta,
                                                 float* __restrict__ dq, bool vec) {
  constexpr int GPT = Dim<HDP>::GPT;
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;                   // [HDP][TP]
  float* dOt = Qt + HDP * TP;       // [HDP][TP]
  float* Kt = dOt + HDP * TP;       // [HDP][TP]
  float* Vt = Kt + HDP * TP;        // [HDP][TP]
  float* Kr = Vt + HDP * TP;        // [TB][RP]
  float* dSt = Kr + TB * Dim<HDP>::RP;  // [TB keys][TP]
  const int64_t b = blockIdx.z;
  const int h = blockIdx.y, kvh = h / (a.H / a.KV), hd = a.hd;
  const int64_t q0 = (int64_t)blockIdx.x * TB;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  const int64_t qoff = b * a.S * qstride + (int64_t)h * hd;
  const int64_t koff = b * a.S * kstride + (int64_t)kvh * hd;
  load_tile<T, HDP>(q + qoff, qstride, q0, a.S, hd, vec, Qt, nullptr);
  load_tile<T, HDP>(dout + qoff, qstride, q0, a.S, hd, vec, dOt, nullptr);
  float lr[4], dr[4], acc[4][4 * GPT];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t qi = q0 + 4 * tx + j;
    lr[j] = qi < a.S ? lse[(b * a.H + h) * a.S + qi] : 0.f;
    dr[j] = qi < a.S ? delta[(b * a.H + h) * a.S + qi] : 0.f;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4 * GPT; ++c) acc[i][c] = 0.f;
  int64_t kbeg, kend;
  key_range(a, q0, kbeg, kend);
  for (int64_t k0 = kbeg; k0 < kend; k0 += TB) {
    __syncthreads();
    load_tile<T, HDP>(k + koff, kstride, k0, a.S, hd, vec, Kt, Kr);
    load_tile<T, HDP>(v + koff, kstride, k0, a.S, hd, vec, Vt, nullptr);
    __syncthreads();
    float s[4][4] = {}, dp[4][4] = {};
#pragma unroll 4
    for (int d = 0; d < HDP; ++d) {
      outer(s, lds4(&Kt[d * TP + 4 * ty]), lds4(&Qt[d * TP + 4 * tx]));
      outer(dp, lds4(&Vt[d * TP + 4 * ty]), lds4(&dOt[d * TP + 4 * tx]));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t kj = k0 + 4 * ty + i;
      float ds[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ds[j] = 0.f;
        if (vis(a, q0 + 4 * tx + j, kj)) {
          const float p = expf(s[i][j] * a.scale - lr[j]);
          ds[j] = p * (dp[i][j] - dr[j]) * a.scale;
        }
      }
      *reinterpret_cast<float4*>(&dSt[(4 * ty + i) * TP + 4 * tx]) =
          make_float4(ds[0], ds[1], ds[2], ds[3]);
    }
    __syncthreads();
    product_out<HDP>(acc, dSt, Kr, tx, ty);
  }
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_out<float, HDP>(dq + qoff, qstride, q0, a.S, hd, false, acc, one, tx, ty);
}

// dK, dV.  grid (ceil(S/TB) * C, KV, B), clusters of C CTAs along x.  The
// score tile is held query-major (thread: queries 4*ty + i, keys 4*tx + j),
// so P and dS land in shared memory as the contraction-major operands of
// dV += P^T dO and dK += dS^T Q.
template <typename T, int HDP>
__global__ __launch_bounds__(NTH) void k_attn_dkdv(Attn a, const T* __restrict__ q,
                                                   const T* __restrict__ k,
                                                   const T* __restrict__ v,
                                                   const T* __restrict__ dout,
                                                   const float* __restrict__ lse,
                                                   const float* __restrict__ delta,
                                                   float* __restrict__ dk,
                                                   float* __restrict__ dv, bool vec, int C) {
  constexpr int GPT = Dim<HDP>::GPT, RP = Dim<HDP>::RP;
  extern __shared__ __align__(16) float sm[];
  float* Kt = sm;                   // [HDP][TP]
  float* Vt = Kt + HDP * TP;        // [HDP][TP]
  float* Qt = Vt + HDP * TP;        // [HDP][TP]
  float* dOt = Qt + HDP * TP;       // [HDP][TP]
  float* Qr = dOt + HDP * TP;       // [TB][RP]
  float* dOr = Qr + TB * RP;        // [TB][RP]
  float* PS = dOr + TB * RP;        // [TB queries][TP]: P, then dS
  const int64_t b = blockIdx.z;
  const int kvh = blockIdx.y, hd = a.hd;
  const int group = a.H / a.KV;
  const int rank = (int)(blockIdx.x % C);
  const int64_t j0 = (int64_t)(blockIdx.x / C) * TB;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  const int64_t koff = b * a.S * kstride + (int64_t)kvh * hd;
  load_tile<T, HDP>(k + koff, kstride, j0, a.S, hd, vec, Kt, nullptr);
  load_tile<T, HDP>(v + koff, kstride, j0, a.S, hd, vec, Vt, nullptr);
  float adk[4][4 * GPT], adv[4][4 * GPT];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 4 * GPT; ++c) adk[i][c] = adv[i][c] = 0.f;
  int64_t qbeg = 0, qend = a.S;
  if (a.causal) {
    qbeg = j0;
    const int64_t last = j0 + TB - 1 + a.window - 1;
    qend = last + 1 < a.S ? last + 1 : a.S;
  }
  for (int hh = rank; hh < group; hh += C) {
    const int h = kvh * group + hh;
    const int64_t qoff = b * a.S * qstride + (int64_t)h * hd;
    for (int64_t i0 = qbeg; i0 < qend; i0 += TB) {
      __syncthreads();
      load_tile<T, HDP>(q + qoff, qstride, i0, a.S, hd, vec, Qt, Qr);
      load_tile<T, HDP>(dout + qoff, qstride, i0, a.S, hd, vec, dOt, dOr);
      float lq[4], dl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t qi = i0 + 4 * ty + i;
        lq[i] = qi < a.S ? lse[(b * a.H + h) * a.S + qi] : 0.f;
        dl[i] = qi < a.S ? delta[(b * a.H + h) * a.S + qi] : 0.f;
      }
      __syncthreads();
      float s[4][4] = {}, dp[4][4] = {};
#pragma unroll 4
      for (int d = 0; d < HDP; ++d) {
        outer(s, lds4(&Qt[d * TP + 4 * ty]), lds4(&Kt[d * TP + 4 * tx]));
        outer(dp, lds4(&dOt[d * TP + 4 * ty]), lds4(&Vt[d * TP + 4 * tx]));
      }
      float ds[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t qi = i0 + 4 * ty + i;
        float p[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          p[j] = vis(a, qi, j0 + 4 * tx + j) ? expf(s[i][j] * a.scale - lq[i]) : 0.f;
          ds[i][j] = p[j] * (dp[i][j] - dl[i]) * a.scale;
        }
        *reinterpret_cast<float4*>(&PS[(4 * ty + i) * TP + 4 * tx]) =
            make_float4(p[0], p[1], p[2], p[3]);
      }
      __syncthreads();
      product_out<HDP>(adv, PS, dOr, tx, ty);
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(&PS[(4 * ty + i) * TP + 4 * tx]) =
            make_float4(ds[i][0], ds[i][1], ds[i][2], ds[i][3]);
      __syncthreads();
      product_out<HDP>(adk, PS, Qr, tx, ty);
    }
  }
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  if (C == 1) {
    store_out<float, HDP>(dk + koff, kstride, j0, a.S, hd, false, adk, one, tx, ty);
    store_out<float, HDP>(dv + koff, kstride, j0, a.S, hd, false, adv, one, tx, ty);
    return;
  }
  // Sum the C partials through distributed shared memory: each CTA parks its
  // partial dK / dV (keys x HDP, row-major) in Qr / dOr, then rank r adds the
  // rows [r*TB/C, (r+1)*TB/C) of every CTA's partials in rank order.
  cg::cluster_group cluster = cg::this_cluster();
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int gi = 0; gi < GPT; ++gi) {
      const int g = tx + 16 * gi;
      if (g >= Dim<HDP>::NDG) continue;
      const int off = (4 * ty + i) * RP + 4 * g;
      *reinterpret_cast<float4*>(&Qr[off]) = make_float4(adk[i][4 * gi], adk[i][4 * gi + 1],
                                                         adk[i][4 * gi + 2], adk[i][4 * gi + 3]);
      *reinterpret_cast<float4*>(&dOr[off]) = make_float4(adv[i][4 * gi], adv[i][4 * gi + 1],
                                                          adv[i][4 * gi + 2], adv[i][4 * gi + 3]);
    }
  cluster.sync();
  const int r_lo = rank * TB / C, r_hi = (rank + 1) * TB / C;
  const int ng = (hd + 3) / 4;
  for (int e = threadIdx.x; e < (r_hi - r_lo) * ng; e += NTH) {
    const int r = r_lo + e / ng, g = e % ng;
    const int64_t kj = j0 + r;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
    for (int src = 0; src < C; ++src) {
      const float* pk = cluster.map_shared_rank(Qr, src);
      const float* pv = cluster.map_shared_rank(dOr, src);
      const float4 xk = lds4(&pk[r * RP + 4 * g]), xv = lds4(&pv[r * RP + 4 * g]);
      sk.x += xk.x; sk.y += xk.y; sk.z += xk.z; sk.w += xk.w;
      sv.x += xv.x; sv.y += xv.y; sv.z += xv.z; sv.w += xv.w;
    }
    if (kj >= a.S) continue;
    float* ok = dk + koff + kj * kstride + 4 * g;
    float* ov = dv + koff + kj * kstride + 4 * g;
    const float ak[4] = {sk.x, sk.y, sk.z, sk.w}, av[4] = {sv.x, sv.y, sv.z, sv.w};
    for (int c = 0; c < 4 && 4 * g + c < hd; ++c) {
      ok[c] = ak[c];
      ov[c] = av[c];
    }
  }
  // keep this CTA's partials alive until every rank has read them
  cluster.sync();
}

void check(const Attn& a) {
  DOP_REQUIRE(a.hd >= 2 && a.hd <= 128 && a.hd % 2 == 0, "head_dim must be even and <= 128");
  DOP_REQUIRE(a.KV >= 1 && a.H % a.KV == 0, "heads must be a multiple of kv_heads");
  DOP_REQUIRE(!a.causal || a.window >= 1, "sliding window must be >= 1");
}

// 16-byte (fp32) or 8-byte (bf16) accesses of four elements are possible when
// every row of every head starts on that boundary.
template <typename T>
bool vec_ok(const Attn& a, std::initializer_list<const void*> ptrs) {
  if (a.hd % 4 != 0) return false;
  for (const void* p : ptrs)
    if ((uintptr_t)p % (4 * sizeof(T)) != 0) return false;
  return true;
}

// Cluster size of the dK / dV kernel: the largest divisor of the head group
// that is at most 8 (the portable cluster limit).
int dkdv_cluster(const Attn& a) {
  const int group = a.H / a.KV;
  for (int c = 8; c > 1; --c)
    if (group % c == 0) return c;
  return 1;
}

template <typename T, int HDP>
void fwd_launch(const Attn& a, const T* q, const T* k, const T* v, T* o, float* lse,
                cudaStream_t s, int64_t& launches) {
  constexpr size_t smem = Dim<HDP>::fwd_smem;
  auto kern = k_attn_fwd<T, HDP>;
  static bool attr = false;
  if (!attr) {
    DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  dim3 grid((unsigned)ceil_div(a.S, TB), (unsigned)a.H, (unsigned)a.B);
  kern<<<grid, NTH, smem, s>>>(a, q, k, v, o, lse, vec_ok<T>(a, {q, k, v, o}));
  DOP_LAUNCHED(launches);
}

template <typename T, int HDP>
void bwd_launch(const Attn& a, const T* q, const T* k, const T* v, const T* dout,
                const float* lse, const float* delta, float* dq, float* dk, float* dv,
                cudaStream_t s, int64_t& launches) {
  const bool vec = vec_ok<T>(a, {q, k, v, dout});
  {
    constexpr size_t smem = Dim<HDP>::dq_smem;
    auto kern = k_attn_dq<T, HDP>;
    static bool attr = false;
    if (!attr) {
      DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr = true;
    }
    dim3 grid((unsigned)ceil_div(a.S, TB), (unsigned)a.H, (unsigned)a.B);
    kern<<<grid, NTH, smem, s>>>(a, q, k, v, dout, lse, delta, dq, vec);
    DOP_LAUNCHED(launches);
  }
  {
    constexpr size_t smem = Dim<HDP>::dkdv_smem;
    auto kern = k_attn_dkdv<T, HDP>;
    static bool attr = false;
    if (!attr) {
      DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attr = true;
    }
    const int C = dkdv_cluster(a);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(ceil_div(a.S, TB) * C), (unsigned)a.KV, (unsigned)a.B);
    cfg.blockDim = dim3(NTH, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    DOP_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, a, q, k, v, dout, lse, delta, dk, dv, vec, C));
    DOP_LAUNCHED(launches);
  }
}

}  // namespace

template <typename T>
void attn_fwd_simt(const Attn& a, const T* q, const T* k, const T* v, T* o, float* lse,
                   cudaStream_t s, int64_t& launches) {
  check(a);
  if (a.hd <= 32)
    fwd_launch<T, 32>(a, q, k, v, o, lse, s, launches);
  else if (a.hd <= 64)
    fwd_launch<T, 64>(a, q, k, v, o, lse, s, launches);
  else
    fwd_launch<T, 128>(a, q, k, v, o, lse, s, launches);
}

template <typename T>
void attn_bwd_simt(const Attn& a, const T* q, const T* k, const T* v, const T* o, const T* dout,
                   const float* lse, float* delta, float* dq, float* dk, float* dv,
                   cudaStream_t s, int64_t& launches) {
  check(a);
  const int64_t rows = a.B * a.S * a.H;
  k_attn_delta<T><<<(unsigned)ceil_div(rows, 8), 256, 0, s>>>(a, o, dout, delta);
  DOP_LAUNCHED(launches);
  if (a.hd <= 32)
    bwd_launch<T, 32>(a, q, k, v, dout, lse, delta, dq, dk, dv, s, launches);
  else if (a.hd <= 64)
    bwd_launch<T, 64>(a, q, k, v, dout, lse, delta, dq, dk, dv, s, launches);
  else
    bwd_launch<T, 128>(a, q, k, v, dout, lse, delta, dq, dk, dv, s, launches);
}

template void attn_fwd_simt<float>(const Attn&, const float*, const float*, const float*, float*,
                                   float*, cudaStream_t, int64_t&);
template void attn_fwd_simt<bf16>(const Attn&, const bf16*, const bf16*, const bf16*, bf16*,
                                  float*, cudaStream_t, int64_t&);
template void attn_bwd_simt<float>(const Attn&, const float*, const float*, const float*,
                                   const float*, const float*, const float*, float*, float*,
                                   float*, float*, cudaStream_t, int64_t&);
template void attn_bwd_simt<bf16>(const Attn&, const bf16*, const bf16*, const bf16*, const bf16*,
                                  const bf16*, const float*, float*, float*, float*, float*,
                                  cudaStream_t, int64_t&);

}  // namespace dop
