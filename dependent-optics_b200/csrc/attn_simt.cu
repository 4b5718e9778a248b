// attn_simt.cu — CUDA-core flash attention, forward and backward, fp32
// arithmetic on fp32 or bf16 storage.
//
// Computes the crate's sliding-window grouped-query attention (gqa_forward /
// gqa_backward, src/mixtral.rs:799-922; visible(q, k) = k <= q && q - k < W)
// and the unmasked Q=K=V=X attention of src/kernel.rs:256-447, without
// materialising probabilities: the forward keeps the row log-sum-exp, the
// backward recomputes P from it.  dK/dV are produced by a key-major kernel
// that loops over the query heads of its group, so no atomics are needed and
// the result is bitwise reproducible.
//
// This is the fp32 lens's attention (DOP_F32) and supports head_dim <= 128.
#include "kernels.cuh"

namespace dop {

namespace {

constexpr int QB = 32;  // queries per CTA (8 warps x 4 rows)
constexpr int KB = 64;  // keys per shared-memory tile
constexpr int NTH = 256;

__device__ __forceinline__ bool vis(const Attn& a, int64_t q, int64_t k) {
  if (!a.causal) return true;
  return k <= q && q - k < a.window;
}

// Forward.  grid (ceil(S/QB), H, B).  Dynamic smem: Qs[QB][hd], Ks[KB][hd+1],
// Vs[KB][hd].
template <typename T>
__global__ __launch_bounds__(NTH) void k_attn_fwd(Attn a, const T* __restrict__ q,
                                                  const T* __restrict__ k,
                                                  const T* __restrict__ v, T* __restrict__ o,
                                                  float* __restrict__ lse) {
  extern __shared__ float sm[];
  const int hd = a.hd, hp = hd + 1;
  float* Qs = sm;
  float* Ks = Qs + QB * hd;
  float* Vs = Ks + KB * hp;
  const int64_t b = blockIdx.z;
  const int h = blockIdx.y, kvh = h / (a.H / a.KV);
  const int64_t q0 = (int64_t)blockIdx.x * QB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  for (int i = threadIdx.x; i < QB * hd; i += NTH) {
    int r = i / hd, d = i % hd;
    int64_t qi = q0 + r;
    Qs[i] = qi < a.S ? ld(&q[(b * a.S + qi) * qstride + (int64_t)h * hd + d]) : 0.f;
  }
  float m_run[4], l_run[4], acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
  }
  int64_t kbeg = 0, kend = a.S;
  if (a.causal) {
    kbeg = q0 - a.window + 1;
    if (kbeg < 0) kbeg = 0;
    kend = q0 + QB < a.S ? q0 + QB : a.S;
  }
  kbeg = kbeg / KB * KB;
  for (int64_t k0 = kbeg; k0 < kend; k0 += KB) {
    __syncthreads();
    for (int i = threadIdx.x; i < KB * hd; i += NTH) {
      int r = i / hd, d = i % hd;
      int64_t kj = k0 + r;
      float kvv = 0.f, vv = 0.f;
      if (kj < a.S) {
        kvv = ld(&k[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]);
        vv = ld(&v[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]);
      }
      Ks[r * hp + d] = kvv;
      Vs[r * hd + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qr = warp * 4 + r;
      const int64_t qi = q0 + qr;
      if (qi >= a.S) continue;
      float s2[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int kr = lane + 32 * half;
        const int64_t kj = k0 + kr;
        float sc = -INFINITY;
        if (kj < a.S && vis(a, qi, kj)) {
          float dot = 0.f;
          for (int d = 0; d < hd; ++d) dot += Qs[qr * hd + d] * Ks[kr * hp + d];
          sc = dot * a.scale;
        }
        s2[half] = sc;
      }
      const float mt = warp_max(fmaxf(s2[0], s2[1]));
      if (mt == -INFINITY) continue;
      const float m_new = fmaxf(m_run[r], mt);
      const float alpha = expf(m_run[r] - m_new);
      const float p0 = s2[0] == -INFINITY ? 0.f : expf(s2[0] - m_new);
      const float p1 = s2[1] == -INFINITY ? 0.f : expf(s2[1] - m_new);
      l_run[r] = l_run[r] * alpha + warp_sum(p0 + p1);
      m_run[r] = m_new;
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[r][c] *= alpha;
      for (int j = 0; j < KB; ++j) {
        const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
        if (pj == 0.f) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int d = lane + 32 * c;
          if (d < hd) acc[r][c] += pj * Vs[j * hd + d];
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t qi = q0 + warp * 4 + r;
    if (qi >= a.S) continue;
    const float inv_l = 1.0f / l_run[r];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = lane + 32 * c;
      if (d < hd) st(&o[(b * a.S + qi) * qstride + (int64_t)h * hd + d], acc[r][c] * inv_l);
    }
    if (lane == 0) lse[(b * a.H + h) * a.S + qi] = m_run[r] + logf(l_run[r]);
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

// dQ.  grid (ceil(S/QB), H, B).  smem: Qs, dOs [QB][hd]; Ks, Vs [KB][hd+1].
template <typename T>
__global__ __launch_bounds__(NTH) void k_attn_dq(Attn a, const T* __restrict__ q,
                                                 const T* __restrict__ k,
                                                 const T* __restrict__ v,
                                                 const T* __restrict__ dout,
                                                 const float* __restrict__ lse,
                                                 const float* __restrict__ delta,
                                                 float* __restrict__ dq) {
  extern __shared__ float sm[];
  const int hd = a.hd, hp = hd + 1;
  float* Qs = sm;
  float* dOs = Qs + QB * hd;
  float* Ks = dOs + QB * hd;
  float* Vs = Ks + KB * hp;
  const int64_t b = blockIdx.z;
  const int h = blockIdx.y, kvh = h / (a.H / a.KV);
  const int64_t q0 = (int64_t)blockIdx.x * QB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  for (int i = threadIdx.x; i < QB * hd; i += NTH) {
    int r = i / hd, d = i % hd;
    int64_t qi = q0 + r;
    bool ok = qi < a.S;
    Qs[i] = ok ? ld(&q[(b * a.S + qi) * qstride + (int64_t)h * hd + d]) : 0.f;
    dOs[i] = ok ? ld(&dout[(b * a.S + qi) * qstride + (int64_t)h * hd + d]) : 0.f;
  }
  float acc[4][4];
  float lrow[4], drow[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t qi = q0 + warp * 4 + r;
    lrow[r] = qi < a.S ? lse[(b * a.H + h) * a.S + qi] : 0.f;
    drow[r] = qi < a.S ? delta[(b * a.H + h) * a.S + qi] : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
  }
  int64_t kbeg = 0, kend = a.S;
  if (a.causal) {
    kbeg = q0 - a.window + 1;
    if (kbeg < 0) kbeg = 0;
    kend = q0 + QB < a.S ? q0 + QB : a.S;
  }
  kbeg = kbeg / KB * KB;
  for (int64_t k0 = kbeg; k0 < kend; k0 += KB) {
    __syncthreads();
    for (int i = threadIdx.x; i < KB * hd; i += NTH) {
      int r = i / hd, d = i % hd;
      int64_t kj = k0 + r;
      float kvv = 0.f, vv = 0.f;
      if (kj < a.S) {
        kvv = ld(&k[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]);
        vv = ld(&v[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]);
      }
      Ks[r * hp + d] = kvv;
      Vs[r * hp + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qr = warp * 4 + r;
      const int64_t qi = q0 + qr;
      if (qi >= a.S) continue;
      float ds2[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int kr = lane + 32 * half;
        const int64_t kj = k0 + kr;
        float ds = 0.f;
        if (kj < a.S && vis(a, qi, kj)) {
          float dot = 0.f, dp = 0.f;
          for (int d = 0; d < hd; ++d) {
            dot += Qs[qr * hd + d] * Ks[kr * hp + d];
            dp += dOs[qr * hd + d] * Vs[kr * hp + d];
          }
          const float p = expf(dot * a.scale - lrow[r]);
          ds = p * (dp - drow[r]) * a.scale;
        }
        ds2[half] = ds;
      }
      for (int j = 0; j < KB; ++j) {
        const float dsj = __shfl_sync(0xffffffffu, j < 32 ? ds2[0] : ds2[1], j & 31);
        if (dsj == 0.f) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int d = lane + 32 * c;
          if (d < hd) acc[r][c] += dsj * Ks[j * hp + d];
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t qi = q0 + warp * 4 + r;
    if (qi >= a.S) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = lane + 32 * c;
      if (d < hd) dq[(b * a.S + qi) * qstride + (int64_t)h * hd + d] = acc[r][c];
    }
  }
}

// dK, dV.  grid (ceil(S/QB) key blocks, KV, B); each warp owns 4 keys and
// loops over every query head of its group and every visible query tile.
// smem: Kt, Vt [QB][hd]; Qs, dOs [KB][hd+1]; lse/delta [KB].
template <typename T>
__global__ __launch_bounds__(NTH) void k_attn_dkdv(Attn a, const T* __restrict__ q,
                                                   const T* __restrict__ k,
                                                   const T* __restrict__ v,
                                                   const T* __restrict__ dout,
                                                   const float* __restrict__ lse,
                                                   const float* __restrict__ delta,
                                                   float* __restrict__ dk, float* __restrict__ dv) {
  extern __shared__ float sm[];
  const int hd = a.hd, hp = hd + 1;
  float* Kt = sm;
  float* Vt = Kt + QB * hd;
  float* Qs = Vt + QB * hd;
  float* dOs = Qs + KB * hp;
  float* Ls = dOs + KB * hp;
  float* Ds = Ls + KB;
  const int64_t b = blockIdx.z;
  const int kvh = blockIdx.y;
  const int group = a.H / a.KV;
  const int64_t j0 = (int64_t)blockIdx.x * QB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t qstride = (int64_t)a.H * hd, kstride = (int64_t)a.KV * hd;
  for (int i = threadIdx.x; i < QB * hd; i += NTH) {
    int r = i / hd, d = i % hd;
    int64_t kj = j0 + r;
    bool ok = kj < a.S;
    Kt[i] = ok ? ld(&k[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]) : 0.f;
    Vt[i] = ok ? ld(&v[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d]) : 0.f;
  }
  float adk[4][4], adv[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) adk[r][c] = adv[r][c] = 0.f;
  int64_t qbeg = 0, qend = a.S;
  if (a.causal) {
    qbeg = j0;
    int64_t last = j0 + QB - 1 + a.window - 1;
    qend = last + 1 < a.S ? last + 1 : a.S;
  }
  qbeg = qbeg / KB * KB;
  for (int hh = 0; hh < group; ++hh) {
    const int h = kvh * group + hh;
    for (int64_t i0 = qbeg; i0 < qend; i0 += KB) {
      __syncthreads();
      for (int i = threadIdx.x; i < KB * hd; i += NTH) {
        int r = i / hd, d = i % hd;
        int64_t qi = i0 + r;
        bool ok = qi < a.S;
        Qs[r * hp + d] = ok ? ld(&q[(b * a.S + qi) * qstride + (int64_t)h * hd + d]) : 0.f;
        dOs[r * hp + d] = ok ? ld(&dout[(b * a.S + qi) * qstride + (int64_t)h * hd + d]) : 0.f;
      }
      for (int i = threadIdx.x; i < KB; i += NTH) {
        int64_t qi = i0 + i;
        Ls[i] = qi < a.S ? lse[(b * a.H + h) * a.S + qi] : 0.f;
        Ds[i] = qi < a.S ? delta[(b * a.H + h) * a.S + qi] : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int kr = warp * 4 + r;
        const int64_t kj = j0 + kr;
        if (kj >= a.S) continue;
        float p2[2], ds2[2];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int qr = lane + 32 * half;
          const int64_t qi = i0 + qr;
          float p = 0.f, ds = 0.f;
          if (qi < a.S && vis(a, qi, kj)) {
            float dot = 0.f, dp = 0.f;
            for (int d = 0; d < hd; ++d) {
              dot += Qs[qr * hp + d] * Kt[kr * hd + d];
              dp += dOs[qr * hp + d] * Vt[kr * hd + d];
            }
            p = expf(dot * a.scale - Ls[qr]);
            ds = p * (dp - Ds[qr]) * a.scale;
          }
          p2[half] = p;
          ds2[half] = ds;
        }
        for (int i = 0; i < KB; ++i) {
          const float pi = __shfl_sync(0xffffffffu, i < 32 ? p2[0] : p2[1], i & 31);
          const float dsi = __shfl_sync(0xffffffffu, i < 32 ? ds2[0] : ds2[1], i & 31);
          if (pi == 0.f && dsi == 0.f) continue;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int d = lane + 32 * c;
            if (d < hd) {
              adv[r][c] += pi * dOs[i * hp + d];
              adk[r][c] += dsi * Qs[i * hp + d];
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int64_t kj = j0 + warp * 4 + r;
    if (kj >= a.S) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = lane + 32 * c;
      if (d < hd) {
        dk[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d] = adk[r][c];
        dv[(b * a.S + kj) * kstride + (int64_t)kvh * hd + d] = adv[r][c];
      }
    }
  }
}

void check(const Attn& a) {
  DOP_REQUIRE(a.hd >= 2 && a.hd <= 128 && a.hd % 2 == 0, "head_dim must be even and <= 128");
  DOP_REQUIRE(a.KV >= 1 && a.H % a.KV == 0, "heads must be a multiple of kv_heads");
  DOP_REQUIRE(!a.causal || a.window >= 1, "sliding window must be >= 1");
}

}  // namespace

template <typename T>
void attn_fwd_simt(const Attn& a, const T* q, const T* k, const T* v, T* o, float* lse,
                   cudaStream_t s, int64_t& launches) {
  check(a);
  size_t smem = sizeof(float) * (QB * a.hd + KB * (a.hd + 1) + KB * a.hd);
  auto kern = k_attn_fwd<T>;
  DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)ceil_div(a.S, QB), (unsigned)a.H, (unsigned)a.B);
  kern<<<grid, NTH, smem, s>>>(a, q, k, v, o, lse);
  DOP_LAUNCHED(launches);
}

template <typename T>
void attn_bwd_simt(const Attn& a, const T* q, const T* k, const T* v, const T* o, const T* dout,
                   const float* lse, float* delta, float* dq, float* dk, float* dv,
                   cudaStream_t s, int64_t& launches) {
  check(a);
  const int64_t rows = a.B * a.S * a.H;
  k_attn_delta<T><<<(unsigned)ceil_div(rows, 8), 256, 0, s>>>(a, o, dout, delta);
  DOP_LAUNCHED(launches);
  {
    size_t smem = sizeof(float) * (2 * QB * a.hd + 2 * KB * (a.hd + 1));
    auto kern = k_attn_dq<T>;
    DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)ceil_div(a.S, QB), (unsigned)a.H, (unsigned)a.B);
    kern<<<grid, NTH, smem, s>>>(a, q, k, v, dout, lse, delta, dq);
    DOP_LAUNCHED(launches);
  }
  {
    size_t smem = sizeof(float) * (2 * QB * a.hd + 2 * KB * (a.hd + 1) + 2 * KB);
    auto kern = k_attn_dkdv<T>;
    DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)ceil_div(a.S, QB), (unsigned)a.KV, (unsigned)a.B);
    kern<<<grid, NTH, smem, s>>>(a, q, k, v, dout, lse, delta, dk, dv);
    DOP_LAUNCHED(launches);
  }
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
