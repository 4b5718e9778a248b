// elementwise.cu — the memory-bound kernels of the Mixtral block lens:
// RMSNorm forward (+ fused router softmax/top-k), RMSNorm backward with a
// deterministic weight reduction, rotary embedding and its adjoint, the
// deterministic expert permutation (count / scan / stable scatter), row
// gather/combine, SwiGLU forward/backward, and the router Jacobian.
//
// Every reduction that produces a parameter adjoint is two-stage (per-chunk
// partials in a fixed order, then a fixed-order sum): no floating-point
// atomics, so two runs give the same bits.
#include "kernels.cuh"

namespace dop {

// ---------------------------------------------------------------- RMSNorm
// rmsnorm (src/mixtral.rs:667-684): r = 1 / sqrt(sum(x^2)/D + eps),
// y = x * r * w.  One CTA per token row.
template <typename T>
__global__ void k_rmsnorm_fwd(const float* __restrict__ x, const T* __restrict__ w, int D,
                              float eps, T* __restrict__ y, float* __restrict__ inv,
                              float* __restrict__ x_copy) {
  const int64_t row = blockIdx.x;
  const float* xr = x + row * D;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = xr[i];
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = red[0] / (float)D + eps;
  const float r = 1.0f / sqrtf(mean);
  if (threadIdx.x == 0) inv[row] = r;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = xr[i];
    st(&y[row * D + i], v * r * ld(&w[i]));
    if (x_copy) x_copy[row * D + i] = v;
  }
}

// ------------------------------------------- vectorised row kernels
// The kernels below are the row kernels above with 4-wide accesses (float4
// for fp32, 8-byte bf16 quads) and the row held in registers between the
// reduction and the write.  The host launchers pick them when D % 4 == 0 and
// every pointer is aligned for the wide access; the per-element arithmetic is
// the same, only the order of the partial sums inside a row differs.

// Sum of v over the CTA (blockDim.x a multiple of 32); every thread gets it.
__device__ __forceinline__ float block_sum(float v, float* red /* [33] */) {
  v = warp_sum(v);
  __syncthreads();  // red may still be read from a previous call
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}


// RMSNorm forward, NV quads per thread (256 threads, D / 4 <= 256 NV).
template <typename T, int NV>
__global__ void __launch_bounds__(256) k_rmsnorm_fwd_v(const float* __restrict__ x,
                                                       const T* __restrict__ w, int D, float eps,
                                                       T* __restrict__ y, float* __restrict__ inv,
                                                       float* __restrict__ x_copy) {
  const int64_t row = blockIdx.x;
  const int D4 = D >> 2;
  const float* xr = x + row * D;
  __shared__ float red[33];
  float4 xv[NV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < D4) {
      xv[j] = ld4(xr + 4 * i);
      ss += xv[j].x * xv[j].x + xv[j].y * xv[j].y + xv[j].z * xv[j].z + xv[j].w * xv[j].w;
    }
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
  if (threadIdx.x == 0) inv[row] = r;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < D4) {
      const float4 wv = ld4(w + 4 * i);
      const float4 v = xv[j];
      st4(y + row * D + 4 * i, make_float4(v.x * r * wv.x, v.y * r * wv.y, v.z * r * wv.z,
                                           v.w * r * wv.w));
      if (x_copy) st4(x_copy + row * D + 4 * i, v);
    }
  }
}

// ------------------------------------------------------------- router stage
// RMSNorm of the feed-forward input and the router, in the crate's
// arithmetic (rmsnorm src/mixtral.rs:667-684, router logits `linear`
// :616-628 at :312, softmax :924-929, topk_renorm :931-939): every sum runs
// over the model dimension in index order from 0.0f, no multiply-add is
// fused (__fmul_rn / __fadd_rn; paired .f32x2 multiply-add sequences are
// not used because they do not keep the two roundings apart), division and
// square root are IEEE, and exp is evaluated in double precision and
// rounded once to float.  On the same input row the routing is therefore
// the crate's to the bit (an exp result can differ in its last bit only
// where the libm's own result is not the correctly rounded one).
//
// Sequential sums leave one dependent chain per row (the sum of squares)
// and per row and expert (the logits), and the norm's sum must finish before
// the first logit term, so the stage is two kernels over the rows:
//   k_router_rms     one lane per row: r = 1 / sqrt(sum x^2 / D + eps), the
//                    row read in 16-byte pieces (a lane's 64-column run of
//                    its row is 256 contiguous bytes, reused from L1);
//   k_router_logits  two lanes per row, each owning half of the expert
//                    chains; rows stream through a per-warp shared tile of 16
//                    rows x 64 columns (read coalesced, one tile ahead in
//                    registers), xn = (x r) w is written from the tile in its
//                    coalesced layout, and the lane that owns expert 0 runs
//                    softmax and top-k.
// Two IEEE round-to-nearest products in one instruction (PTX mul.rn.f32x2,
// sm_100): each lane of the pair is rounded exactly as __fmul_rn would.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint64_t d, ua, ub;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ua) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(ub) : "f"(b.x), "f"(b.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(ua), "l"(ub));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}

constexpr int kRtCols = 64;                // columns per tile
constexpr int kRtPitch = kRtCols + 4;      // floats per tile row in shared memory
constexpr int kRtRows = 16;                // rows per warp (two lanes a row)
constexpr int kRtWarps = 1;                // warps per CTA (one: the SMs' shares differ by a warp)

// Crate-rounded exp: double-precision exp of the float argument, rounded
// once to float.
__device__ __forceinline__ float exp_rounded(float z) { return __double2float_rn(exp((double)z)); }

template <bool VEC>
__global__ void __launch_bounds__(32) k_router_rms(const float* __restrict__ x, int64_t rows,
                                                    int D, float eps, float* __restrict__ inv) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* xr = x + row * D;
  float ss = 0.0f;
  if (VEC) {
    // 64-column runs, the next run's loads in flight while this one is summed
    constexpr int J = kRtCols / 4;
    auto fetch = [&](int c0, float4 (&v)[J]) {
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int c = c0 + 4 * j;
        v[j] = c < D ? __ldg(reinterpret_cast<const float4*>(xr + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    float4 a[J], b[J];
    fetch(0, a);
    for (int c0 = 0; c0 < D; c0 += 2 * kRtCols) {
      if (c0 + kRtCols < D) fetch(c0 + kRtCols, b);
      // zeros past D add nothing: ss + 0 * 0 = ss exactly
#pragma unroll
      for (int j = 0; j < J; ++j) {
        ss = __fadd_rn(ss, __fmul_rn(a[j].x, a[j].x));
        ss = __fadd_rn(ss, __fmul_rn(a[j].y, a[j].y));
        ss = __fadd_rn(ss, __fmul_rn(a[j].z, a[j].z));
        ss = __fadd_rn(ss, __fmul_rn(a[j].w, a[j].w));
      }
      if (c0 + kRtCols >= D) break;
      if (c0 + 2 * kRtCols < D) fetch(c0 + 2 * kRtCols, a);
#pragma unroll
      for (int j = 0; j < J; ++j) {
        ss = __fadd_rn(ss, __fmul_rn(b[j].x, b[j].x));
        ss = __fadd_rn(ss, __fmul_rn(b[j].y, b[j].y));
        ss = __fadd_rn(ss, __fmul_rn(b[j].z, b[j].z));
        ss = __fadd_rn(ss, __fmul_rn(b[j].w, b[j].w));
      }
    }
  } else {
    for (int c = 0; c < D; ++c) ss = __fadd_rn(ss, __fmul_rn(xr[c], xr[c]));
  }
  inv[row] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
}

// Columns [c0, c0 + 64) of the warp's 16 rows (zeros outside the matrix):
// lane l holds rows (l / 16) + 2 j, columns 4 (l % 16) .. + 3.
template <bool VEC>
struct RtTile {
  float v[32];
  __device__ __forceinline__ void load(const float* __restrict__ x, int64_t rows, int D,
                                       int64_t r0, int c0, int lane) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t row = r0 + (lane >> 4) + 2 * j;
      const int col = c0 + 4 * (lane & 15);
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < rows) {
        const float* p = x + row * D + col;
        if (VEC) {
          if (col < D) t = *reinterpret_cast<const float4*>(p);
        } else {
          if (col < D) t.x = p[0];
          if (col + 1 < D) t.y = p[1];
          if (col + 2 < D) t.z = p[2];
          if (col + 3 < D) t.w = p[3];
        }
      }
      v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
    }
  }
  __device__ __forceinline__ void store(float* tile, int lane) const {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(tile + ((lane >> 4) + 2 * j) * kRtPitch + 4 * (lane & 15)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
};

// The norm weights and router rows of one tile (64 model rows), in registers
// one tile ahead (lane l: model rows l and l + 32), stored to shared memory
// in fp32: ws[c] and wrs[c * NE + e] (zeros past D and past E).
template <typename T, int NE>
struct RtWeights {
  float wn[2];
  float wv[2][NE];
  __device__ __forceinline__ void load(const T* __restrict__ w, const T* __restrict__ wr, int E,
                                       int D, int c0, int lane) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + lane + 32 * h;
      const bool in = c < D;
      wn[h] = in ? ld(&w[c]) : 0.f;
      if (NE == 8 && E == 8 && in) {
        if (sizeof(T) == 2) {
          ld_row8(wr + (int64_t)c * 8, wv[h]);
        } else {
          const float4 a = *reinterpret_cast<const float4*>(wr + (int64_t)c * 8);
          const float4 b = *reinterpret_cast<const float4*>(wr + (int64_t)c * 8 + 4);
          wv[h][0] = a.x; wv[h][1] = a.y; wv[h][2] = a.z; wv[h][3] = a.w;
          wv[h][4] = b.x; wv[h][5] = b.y; wv[h][6] = b.z; wv[h][7] = b.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < NE; ++e) wv[h][e] = (in && e < E) ? ld(&wr[(int64_t)c * E + e]) : 0.f;
      }
    }
  }
  __device__ __forceinline__ void store(float* ws, float* wrs, int lane) const {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = lane + 32 * h;
      ws[c] = wn[h];
      if (NE % 4 == 0) {
#pragma unroll
        for (int e = 0; e < NE; e += 4)
          *reinterpret_cast<float4*>(wrs + c * NE + e) =
              make_float4(wv[h][e], wv[h][e + 1], wv[h][e + 2], wv[h][e + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < NE; ++e) wrs[c * NE + e] = wv[h][e];
      }
    }
  }
};

template <typename T, int NE, bool VEC>
__global__ void __launch_bounds__(32 * kRtWarps, 16 / kRtWarps) k_router_logits(
    const float* __restrict__ x, const T* __restrict__ w, const T* __restrict__ wr,
    const float* __restrict__ bias, int64_t rows, int D, int E, int K,
    const float* __restrict__ inv, T* __restrict__ y, float* __restrict__ probs,
    int* __restrict__ top_i, float* __restrict__ top_p, float* __restrict__ top_w) {
  constexpr int EPL = NE / 2;  // logit chains per lane (0 when E == 1)
  __shared__ __align__(16) float tile_all[kRtWarps][kRtRows * kRtPitch];
  __shared__ __align__(16) float wrs_all[kRtWarps][kRtCols * NE];
  __shared__ __align__(16) float ws_all[kRtWarps][kRtCols];
  __shared__ float r_all[kRtWarps][kRtRows];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int rr = lane >> 1, q = lane & 1;  // row in the warp, expert half
  const int64_t r0 = ((int64_t)blockIdx.x * kRtWarps + wid) * kRtRows;
  if (r0 >= rows) return;  // whole warp
  const int64_t row = r0 + rr;
  const bool live = row < rows;
  float* tile = tile_all[wid];
  float* wrs = wrs_all[wid];
  float* ws = ws_all[wid];
  float* rs = r_all[wid];
  const float r = live ? inv[row] : 0.f;
  if (q == 0) rs[rr] = r;

  float z[EPL > 0 ? EPL : 1];
#pragma unroll
  for (int k = 0; k < (EPL > 0 ? EPL : 1); ++k) z[k] = 0.0f;
  const int nt = (D + kRtCols - 1) / kRtCols;
  RtTile<VEC> cur, nxt;
  RtWeights<T, NE> wcur, wnxt;
  cur.load(x, rows, D, r0, 0, lane);
  wcur.load(w, wr, E, D, 0, lane);
  for (int t = 0; t < nt; ++t) {
    const int c0 = t * kRtCols, n = min(kRtCols, D - c0);
    __syncwarp();
    cur.store(tile, lane);
    wcur.store(ws, wrs, lane);
    if (t + 1 < nt) {
      nxt.load(x, rows, D, r0, c0 + kRtCols, lane);
      wnxt.load(w, wr, E, D, c0 + kRtCols, lane);
    }
    __syncwarp();
    // xn = (x r) w from the tile in its coalesced layout: rows (lane / 16) + 2 j
    {
      const int col = 4 * (lane & 15);
      if (col < n) {
        const float4 wv = *reinterpret_cast<const float4*>(ws + col);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int tr = (lane >> 4) + 2 * j;
          if (r0 + tr >= rows) continue;
          const float rj = rs[tr];
          const float4 xv = *reinterpret_cast<const float4*>(tile + tr * kRtPitch + col);
          const float2 r2 = make_float2(rj, rj);
          const float2 o01 = mul2_rn(mul2_rn(make_float2(xv.x, xv.y), r2), make_float2(wv.x, wv.y));
          const float2 o23 = mul2_rn(mul2_rn(make_float2(xv.z, xv.w), r2), make_float2(wv.z, wv.w));
          const float4 o = make_float4(o01.x, o01.y, o23.x, o23.y);
          T* dst = y + (r0 + tr) * D + c0 + col;
          if (VEC && col + 4 <= n) {
            st4(dst, o);
          } else {
            const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (col + e < n) st(dst + e, ov[e]);
          }
        }
      }
    }
    // this lane's logit chains over the tile's columns, in index order
    if (EPL > 0) {
      const float* mine = tile + rr * kRtPitch;
      const float* wq = wrs + q * EPL;
      const float2 r2 = make_float2(r, r);
      // products in pairs (exact), the sums one chain per expert in column
      // order; EPL is even
      auto step = [&](float xn, int c) {
        const float2 xx = make_float2(xn, xn);
#pragma unroll
        for (int k = 0; k < EPL; k += 2) {
          const float2 pr = mul2_rn(xx, *reinterpret_cast<const float2*>(wq + c * NE + k));
          z[k] = __fadd_rn(z[k], pr.x);
          z[k + 1] = __fadd_rn(z[k + 1], pr.y);
        }
      };
      if (n == kRtCols) {
#pragma unroll 4
        for (int c = 0; c < kRtCols; c += 4) {
          const float4 xv = *reinterpret_cast<const float4*>(mine + c);
          const float4 wv = *reinterpret_cast<const float4*>(ws + c);
          const float2 x01 = mul2_rn(mul2_rn(make_float2(xv.x, xv.y), r2), make_float2(wv.x, wv.y));
          const float2 x23 = mul2_rn(mul2_rn(make_float2(xv.z, xv.w), r2), make_float2(wv.z, wv.w));
          step(x01.x, c);
          step(x01.y, c + 1);
          step(x23.x, c + 2);
          step(x23.y, c + 3);
        }
      } else {
        for (int c = 0; c < n; ++c) step(__fmul_rn(__fmul_rn(mine[c], r), ws[c]), c);
      }
    }
    cur = nxt;
    wcur = wnxt;
  }
  // the row's E logits to the lane that owns expert 0
  float zf[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e)
    zf[e] = EPL > 0 ? __shfl_sync(0xffffffffu, z[EPL > 0 ? e % EPL : 0], 2 * rr + (EPL > 0 ? e / EPL : 0))
                    : 0.0f;
  if (!live || q != 0) return;

  // bias (skewed routing), softmax (src/mixtral.rs:924-929)
  float m = -INFINITY;
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    if (e < E) {
      if (bias) zf[e] = __fadd_rn(zf[e], bias[e]);
      m = fmaxf(m, zf[e]);
    }
  }
  float p[NE];
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    p[e] = e < E ? exp_rounded(__fsub_rn(zf[e], m)) : 0.f;
    if (e < E) s = __fadd_rn(s, p[e]);
  }
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    if (e < E) {
      p[e] = __fdiv_rn(p[e], s);
      probs[row * E + e] = p[e];
    }
  }
  // topk_renorm (src/mixtral.rs:931-939): probability desc, then index asc
  unsigned taken = 0;
  float pk[kMaxTopK];
  int ik[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    pk[k] = 0.f;
    ik[k] = 0;
    if (k < K) {
      int best = -1;
      float bp = 0.f;
#pragma unroll
      for (int e = 0; e < NE; ++e) {
        if (e < E && !((taken >> e) & 1u) && (best < 0 || p[e] > bp)) {
          best = e;
          bp = p[e];
        }
      }
      taken |= 1u << best;
      ik[k] = best;
      pk[k] = bp;
    }
  }
  float sk = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k)
    if (k < K) sk = __fadd_rn(sk, pk[k]);
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    if (k < K) {
      top_i[row * K + k] = ik[k];
      top_p[row * K + k] = pk[k];
      top_w[row * K + k] = __fdiv_rn(pk[k], sk);
    }
  }
}

// Xp[r] = xn[row_token[r]] in 16-byte words (zero rows for padding).
__global__ void k_gather_rows16(const uint4* __restrict__ src, const int* __restrict__ row_token,
                                const int* __restrict__ seg_off, int E, int n16,
                                uint4* __restrict__ dst) {
  const int64_t r = blockIdx.x;
  if (r >= seg_off[E]) return;
  const int t = row_token[r];
  for (int i = threadIdx.x; i < n16; i += blockDim.x)
    dst[r * n16 + i] = t >= 0 ? src[(int64_t)t * n16 + i] : make_uint4(0u, 0u, 0u, 0u);
}

// Token-major form of k_gather_rows16: CTA t reads token row t once and
// writes it to its K expert rows slot_row[t K + k] (16-byte words).
__global__ void k_scatter_rows16(const uint4* __restrict__ src, const int* __restrict__ slot_row,
                                 int K, int n16, uint4* __restrict__ dst) {
  const int64_t t = blockIdx.x;
  int64_t rows[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) rows[k] = k < K ? slot_row[t * K + k] : 0;
  for (int i = threadIdx.x; i < n16; i += blockDim.x) {
    const uint4 v = src[t * n16 + i];
#pragma unroll
    for (int k = 0; k < kMaxTopK; ++k)
      if (k < K) dst[rows[k] * n16 + i] = v;
  }
}
// The padding rows of the expert segments (row_token < 0) to zero, one warp
// a row.
__global__ void k_zero_pad_rows16(const int* __restrict__ row_token, const int* __restrict__ seg_off,
                                  int E, int64_t rows_cap, int n16, uint4* __restrict__ dst) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows_cap || r >= seg_off[E] || row_token[r] >= 0) return;
  for (int i = threadIdx.x & 31; i < n16; i += 32) dst[r * n16 + i] = make_uint4(0u, 0u, 0u, 0u);
}

// dO[r] = row_w[r] * dy[row_token[r]], 4 elements per access.
template <typename T>
__global__ void k_gather_scale_rows_v(const float* __restrict__ src,
                                      const int* __restrict__ row_token,
                                      const float* __restrict__ row_w,
                                      const int* __restrict__ seg_off, int E, int D,
                                      T* __restrict__ dst) {
  const int64_t r = blockIdx.x;
  if (r >= seg_off[E]) return;
  const int t = row_token[r];
  const float w = t >= 0 ? row_w[r] : 0.f;
  for (int i = threadIdx.x * 4; i < D; i += blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t >= 0) {
      const float4 a = ld4(src + (int64_t)t * D + i);
      v = make_float4(w * a.x, w * a.y, w * a.z, w * a.w);
    }
    st4(dst + r * D + i, v);
  }
}

// Token-major form of k_gather_scale_rows_v: CTA t reads dy row t once and
// writes top_w[t K + k] * dy[t] to its K expert rows slot_row[t K + k] (the
// same products as the row-major form, row_w[slot_row[p]] = top_w[p]).
template <typename T>
__global__ void __launch_bounds__(256) k_scatter_scale_rows_v(const float* __restrict__ src,
                                                              const int* __restrict__ slot_row,
                                                              const float* __restrict__ top_w,
                                                              int K, int D, T* __restrict__ dst) {
  const int64_t t = blockIdx.x;
  int64_t rows[kMaxTopK];
  float w[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    rows[k] = k < K ? slot_row[t * K + k] : 0;
    w[k] = k < K ? top_w[t * K + k] : 0.f;
  }
  constexpr int U = 4;  // float4 loads in flight per thread
  for (int i0 = threadIdx.x * 4; i0 < D; i0 += U * 1024) {
    float4 a[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * 1024;
      a[u] = i < D ? ld4(src + t * D + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * 1024;
      if (i >= D) break;
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K)
          st4(dst + rows[k] * D + i,
              make_float4(w[k] * a[u].x, w[k] * a[u].y, w[k] * a[u].z, w[k] * a[u].w));
    }
  }
}

// y[t] = mid[t] + sum_k w_k * out[row(t,k)], 4 elements per access; the slot
// sum is taken in slot order from zero, as in k_combine.
__global__ void k_combine_v(const float* __restrict__ mid, const float* __restrict__ out,
                            const int* __restrict__ slot_row, const float* __restrict__ top_w,
                            int K, int D, float* __restrict__ y) {
  const int64_t t = blockIdx.x;
  __shared__ int64_t rows[kMaxTopK];
  __shared__ float ws[kMaxTopK];
  if (threadIdx.x < K) {
    rows[threadIdx.x] = slot_row[t * K + threadIdx.x];
    ws[threadIdx.x] = top_w[t * K + threadIdx.x];
  }
  __syncthreads();
  for (int i = threadIdx.x * 4; i < D; i += blockDim.x * 4) {
    float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const float4 o = ld4(out + rows[k] * D + i);
      m.x += ws[k] * o.x; m.y += ws[k] * o.y; m.z += ws[k] * o.z; m.w += ws[k] * o.w;
    }
    const float4 a = ld4(mid + t * D + i);
    st4(y + t * D + i, make_float4(a.x + m.x, a.y + m.y, a.z + m.z, a.w + m.w));
  }
}

// rmsnorm_bwd (src/mixtral.rs:696-723), input cotangent: one warp per row,
// dx = r (dy*w - xhat * mean(dy*w*xhat)) (+ res), xhat = x r.  Rows are read
// twice (at large T the second pass misses L2), float4 when D % 128 == 0 and
// every pointer is 16-byte (fp32) or 8-byte (bf16) aligned.  The launcher
// prefers k_rmsnorm_bwd_v (one read) when D fits one CTA's registers.
template <typename T>
__global__ void k_rmsnorm_bwd_rows(const float* __restrict__ dy, const float* __restrict__ x,
                                   const float* __restrict__ inv, const T* __restrict__ w,
                                   const float* __restrict__ res, int64_t rows, int D,
                                   float* __restrict__ dx, T* __restrict__ dx_act, bool vec) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float r = inv[row];
  const float* xr = x + row * D;
  const float* gr = dy + row * D;
  float dot = 0.f;
  if (vec) {
    for (int i = lane * 4; i < D; i += 128) {
      const float4 xv = ld4(xr + i);
      const float4 gv = ld4(gr + i);
      const float4 wv = ld4(w + i);
      dot += (gv.x * wv.x) * (xv.x * r) + (gv.y * wv.y) * (xv.y * r) +
             (gv.z * wv.z) * (xv.z * r) + (gv.w * wv.w) * (xv.w * r);
    }
  } else {
    for (int i = lane; i < D; i += 32) dot += (gr[i] * ld(&w[i])) * (xr[i] * r);
  }
  dot = warp_sum(dot);
  const float mean = dot / (float)D;
  if (vec) {
    for (int i = lane * 4; i < D; i += 128) {
      const float4 xv = ld4(xr + i);
      const float4 gv = ld4(gr + i);
      const float4 wv = ld4(w + i);
      float4 o;
      o.x = r * (gv.x * wv.x - (xv.x * r) * mean);
      o.y = r * (gv.y * wv.y - (xv.y * r) * mean);
      o.z = r * (gv.z * wv.z - (xv.z * r) * mean);
      o.w = r * (gv.w * wv.w - (xv.w * r) * mean);
      if (res) {
        const float4 rv = ld4(res + row * D + i);
        o.x += rv.x; o.y += rv.y; o.z += rv.z; o.w += rv.w;
      }
      st4(dx + row * D + i, o);
      if (dx_act) st4(dx_act + row * D + i, o);
    }
  } else {
    for (int i = lane; i < D; i += 32) {
      float v = r * (gr[i] * ld(&w[i]) - (xr[i] * r) * mean);
      if (res) v += res[row * D + i];
      dx[row * D + i] = v;
      if (dx_act) st(&dx_act[row * D + i], v);
    }
  }
}

// The same adjoint with one CTA per row and the row's dy, x and residual
// cotangent loaded before the reduction and held in registers until the
// output pass (NV quads per thread), so each is read from DRAM once and no
// load waits behind the reduction.
template <typename T, int NV>
__global__ void __launch_bounds__(256) k_rmsnorm_bwd_v(const float* __restrict__ dy,
                                                       const float* __restrict__ x,
                                                       const float* __restrict__ inv,
                                                       const T* __restrict__ w,
                                                       const float* __restrict__ res, int D,
                                                       float* __restrict__ dx,
                                                       T* __restrict__ dx_act) {
  const int64_t row = blockIdx.x;
  const int D4 = D >> 2;
  const float r = inv[row];
  __shared__ float red[33];
  float4 xv[NV], gv[NV], rv[NV];
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < D4) {
      xv[j] = ld4(x + row * D + 4 * i);
      gv[j] = ld4(dy + row * D + 4 * i);
      if (res) rv[j] = ld4(res + row * D + 4 * i);
      const float4 wv = ld4(w + 4 * i);
      dot += (gv[j].x * wv.x) * (xv[j].x * r) + (gv[j].y * wv.y) * (xv[j].y * r) +
             (gv[j].z * wv.z) * (xv[j].z * r) + (gv[j].w * wv.w) * (xv[j].w * r);
    }
  }
  const float mean = block_sum(dot, red) / (float)D;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < D4) {
      const float4 wv = ld4(w + 4 * i);
      const float4 xq = xv[j], gq = gv[j];
      float4 o;
      o.x = r * (gq.x * wv.x - (xq.x * r) * mean);
      o.y = r * (gq.y * wv.y - (xq.y * r) * mean);
      o.z = r * (gq.z * wv.z - (xq.z * r) * mean);
      o.w = r * (gq.w * wv.w - (xq.w * r) * mean);
      if (res) {
        o.x += rv[j].x; o.y += rv[j].y; o.z += rv[j].z; o.w += rv[j].w;
      }
      st4(dx + row * D + 4 * i, o);
      if (dx_act) st4(dx_act + row * D + 4 * i, o);
    }
  }
}

// k_rmsnorm_bwd_v and the weight adjoint partials in one pass: CTA c walks
// the rows of chunk c (the same per-row arithmetic as k_rmsnorm_bwd_v, so dx
// is bit-identical to it) and accumulates part[c, i] = sum over its rows of
// dy[t,i] * (x[t,i] r[t]) in increasing row order, from the dy and x it
// already holds, so the weight adjoint costs no second read of either.
template <typename T, int NV>
__global__ void __launch_bounds__(256, 3) k_rmsnorm_bwd_dw_v(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ inv,
    const T* __restrict__ w, const float* __restrict__ res, int64_t rows, int D,
    int rows_per_chunk, float* __restrict__ dx, T* __restrict__ dx_act, float* __restrict__ part) {
  const int c = blockIdx.x;
  const int64_t t0 = (int64_t)c * rows_per_chunk;
  const int64_t t1 = ::min(rows, t0 + rows_per_chunk);
  const int D4 = D >> 2;
  __shared__ float red[33];
  float4 dw[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) dw[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t row = t0; row < t1; ++row) {
    const float r = inv[row];
    float4 xv[NV], gv[NV], rv[NV];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * 256;
      if (i < D4) {
        xv[j] = ld4(x + row * D + 4 * i);
        gv[j] = ld4(dy + row * D + 4 * i);
        if (res) rv[j] = ld4(res + row * D + 4 * i);
        const float4 wv = ld4(w + 4 * i);
        dot += (gv[j].x * wv.x) * (xv[j].x * r) + (gv[j].y * wv.y) * (xv[j].y * r) +
               (gv[j].z * wv.z) * (xv[j].z * r) + (gv[j].w * wv.w) * (xv[j].w * r);
      }
    }
    const float mean = block_sum(dot, red) / (float)D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * 256;
      if (i < D4) {
        const float4 wv = ld4(w + 4 * i);
        const float4 xq = xv[j], gq = gv[j];
        float4 o;
        o.x = r * (gq.x * wv.x - (xq.x * r) * mean);
        o.y = r * (gq.y * wv.y - (xq.y * r) * mean);
        o.z = r * (gq.z * wv.z - (xq.z * r) * mean);
        o.w = r * (gq.w * wv.w - (xq.w * r) * mean);
        if (res) {
          o.x += rv[j].x; o.y += rv[j].y; o.z += rv[j].z; o.w += rv[j].w;
        }
        st4(dx + row * D + 4 * i, o);
        if (dx_act) st4(dx_act + row * D + 4 * i, o);
        dw[j].x += gq.x * (xq.x * r);
        dw[j].y += gq.y * (xq.y * r);
        dw[j].z += gq.z * (xq.z * r);
        dw[j].w += gq.w * (xq.w * r);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < D4) *reinterpret_cast<float4*>(part + (int64_t)c * D + 4 * i) = dw[j];
  }
}

// out[i] += sum over c < chunks of part[c, i], for many chunks: warp w of a
// CTA sums the chunks [w L, (w + 1) L) of 32 columns in order, then warp 0
// adds the 32 slice sums in order (deterministic).
__global__ void __launch_bounds__(1024) k_reduce_chunks_wide(const float* __restrict__ part,
                                                             int chunks, int64_t n,
                                                             float* __restrict__ out) {
  __shared__ float sl[32][33];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 32 + l;
  const int L = (chunks + 31) / 32;
  float s = 0.f;
  if (i < n) {
    const int c1 = ::min(chunks, (w + 1) * L);
    for (int c = w * L; c < c1; ++c) s += part[(int64_t)c * n + i];
  }
  sl[w][l] = s;
  __syncthreads();
  if (w == 0 && i < n) {
    float t = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) t += sl[k][l];
    out[i] += t;
  }
}

// Weight adjoint partials: part[c, i] = sum_{t in chunk c} dy[t,i] * x[t,i] r[t],
// rows in increasing order (deterministic).
__global__ void k_rmsnorm_dw_part(const float* __restrict__ dy, const float* __restrict__ x,
                                  const float* __restrict__ inv, int64_t rows, int D,
                                  int rows_per_chunk, float* __restrict__ part) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int c = blockIdx.y;
  if (i >= D) return;
  const int64_t t0 = (int64_t)c * rows_per_chunk;
  const int64_t t1 = ::min((int64_t)rows, t0 + rows_per_chunk);
  float acc = 0.f;
#pragma unroll 8
  for (int64_t t = t0; t < t1; ++t) acc += dy[t * D + i] * (x[t * D + i] * inv[t]);
  part[(int64_t)c * D + i] = acc;
}

// out[i] += sum_{c < chunks} part[c, i] in chunk order (deterministic).
__global__ void k_reduce_chunks(const float* __restrict__ part, int chunks, int64_t n,
                                float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += part[(int64_t)c * n + i];
  out[i] += s;
}

// ------------------------------------------------------------------ RoPE
// rope_angles (src/mixtral.rs:725-739): freq_i = theta^(-(2i)/hd), angle =
// pos * freq_i, one table row per position.
__global__ void k_rope_table(int S, int half, int hd, float theta, float* __restrict__ cs,
                             float* __restrict__ sn) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)S * half) return;
  int s = (int)(idx / half), i = (int)(idx % half);
  float freq = powf(theta, -(2.0f * (float)i) / (float)hd);
  float ang = (float)s * freq;
  float sv, cv;
  sincosf(ang, &sv, &cv);
  cs[idx] = cv;
  sn[idx] = sv;
}

// rope_one (src/mixtral.rs:741-753) over [T, heads, hd]; sign -1 is the
// adjoint (rope_qkv_transpose, :777-797).  pos = t mod S.
template <typename TI, typename TO>
__global__ void k_rope(const TI* __restrict__ src, TO* __restrict__ dst, int64_t T, int S,
                       int heads, int hd, const float* __restrict__ cs,
                       const float* __restrict__ sn, float sign) {
  const int half = hd / 2;
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = T * heads * half;
  if (idx >= total) return;
  int i = (int)(idx % half);
  int64_t th = idx / half;  // t * heads + h
  int64_t t = th / heads;
  int pos = (int)(t % S);
  int64_t base = th * hd;
  float c = cs[(int64_t)pos * half + i], s = sign * sn[(int64_t)pos * half + i];
  float q1 = ld(&src[base + i]), q2 = ld(&src[base + half + i]);
  st(&dst[base + i], q1 * c - q2 * s);
  st(&dst[base + half + i], q2 * c + q1 * s);
}

// ------------------------------------------------- expert permutation (K7)
// The canonical order of the (token, slot) pairs routed to an expert is the
// token-major order (t, then slot): a stable counting sort by expert.  Each
// expert's segment starts at a multiple of kSegAlign rows, so a GEMM row tile
// (or the 2-SM GEMM's pair of tiles) never straddles two experts and padded
// rows can be zero; the row tile -> expert map has one entry per kRowAlign
// rows.
//
// Pass 1: per chunk of kPermChunk pairs, count pairs per expert.
__global__ void k_perm_count(const int* __restrict__ top_i, int64_t pairs, int E,
                             int* __restrict__ chunk_counts) {
  __shared__ int cnt[kMaxExperts];
  if (threadIdx.x < kMaxExperts) cnt[threadIdx.x] = 0;
  __syncthreads();
  int64_t p = (int64_t)blockIdx.x * kPermChunk + threadIdx.x;
  for (int q = 0; q < kPermChunk / (int)blockDim.x; ++q, p += blockDim.x)
    if (p < pairs) atomicAdd(&cnt[top_i[p]], 1);  // integer: order-free
  __syncthreads();
  if (threadIdx.x < E) chunk_counts[(int64_t)blockIdx.x * E + threadIdx.x] = cnt[threadIdx.x];
}

// Pass 2 (one CTA): exclusive scan over chunks per expert, padded segment
// offsets seg_off[E+1], and the row-tile -> expert map of the padded buffer.
__global__ void k_perm_scan(int* __restrict__ chunk_counts, int chunks, int E,
                            int* __restrict__ seg_off, int* __restrict__ tile_expert,
                            int max_tiles) {
  __shared__ int tot[kMaxExperts];
  int e = threadIdx.x;
  if (e < E) {
    int run = 0;
    for (int c = 0; c < chunks; ++c) {
      int v = chunk_counts[(int64_t)c * E + e];
      chunk_counts[(int64_t)c * E + e] = run;
      run += v;
    }
    tot[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int q = 0; q < E; ++q) {
      seg_off[q] = off;
      off += (tot[q] + kSegAlign - 1) / kSegAlign * kSegAlign;
    }
    seg_off[E] = off;
  }
  __syncthreads();
  for (int tile = threadIdx.x; tile < max_tiles; tile += blockDim.x) {
    int row = tile * kRowAlign, ex = -1;
    for (int q = 0; q < E; ++q)
      if (row >= seg_off[q] && row < seg_off[q + 1]) ex = q;
    tile_expert[tile] = ex;
  }
}

// Pass 3: stable scatter.  Pair p's row = seg_off[e] + (pairs of expert e in
// earlier chunks) + (pairs of expert e earlier in this chunk).  The in-chunk
// rank uses warp match masks and a per-warp count table, so the result is
// the same on every run.
__global__ void k_perm_scatter(const int* __restrict__ top_i, const float* __restrict__ top_w,
                               int64_t pairs, int E, int K, const int* __restrict__ chunk_base,
                               const int* __restrict__ seg_off, int* __restrict__ slot_row,
                               int* __restrict__ row_token, float* __restrict__ row_w) {
  __shared__ int wcnt[kPermChunk / 32][kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = kPermChunk / 32;
  for (int i = threadIdx.x; i < nwarps * kMaxExperts; i += blockDim.x)
    (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t p = (int64_t)blockIdx.x * kPermChunk + threadIdx.x;
  const bool valid = p < pairs;
  const int e = valid ? top_i[p] : -1;
  const unsigned same = __match_any_sync(0xffffffffu, e);
  const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
  if (valid && rank_in_warp == 0) wcnt[warp][e] = __popc(same);
  __syncthreads();
  if (valid) {
    int before = 0;
    for (int q = 0; q < warp; ++q) before += wcnt[q][e];
    int row = seg_off[e] + chunk_base[(int64_t)blockIdx.x * E + e] + before + rank_in_warp;
    slot_row[p] = row;
    row_token[row] = (int)(p / K);
    row_w[row] = top_w[p];
  }
}

// Xp[r] = xn[row_token[r]] (zero rows for padding).  One CTA per row.
template <typename T>
__global__ void k_gather_rows(const T* __restrict__ src, const int* __restrict__ row_token,
                              const int* __restrict__ seg_off, int E, int D, T* __restrict__ dst) {
  const int64_t r = blockIdx.x;
  if (r >= seg_off[E]) return;
  const int t = row_token[r];
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    dst[r * D + i] = t >= 0 ? src[(int64_t)t * D + i] : T(0.f);
}

// dO[r] = row_w[r] * dy[row_token[r]] (zero rows for padding): the down
// projection's output cotangent, d_out = w * d_mixed (src/mixtral.rs:474-477).
template <typename T>
__global__ void k_gather_scale_rows(const float* __restrict__ src, const int* __restrict__ row_token,
                                    const float* __restrict__ row_w,
                                    const int* __restrict__ seg_off, int E, int D,
                                    T* __restrict__ dst) {
  const int64_t r = blockIdx.x;
  if (r >= seg_off[E]) return;
  const int t = row_token[r];
  const float w = t >= 0 ? row_w[r] : 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x)
    st(&dst[r * D + i], t >= 0 ? w * src[(int64_t)t * D + i] : 0.f);
}

// ------------------------------------------------------------- SwiGLU
// silu_mul (src/mixtral.rs:941-951): h = g * sigmoid(g) * u.
template <typename T>
__global__ void k_silu_mul(const T* __restrict__ g, const T* __restrict__ u,
                           const int* __restrict__ seg_off, int E, int64_t I, T* __restrict__ h) {
  int64_t n = (int64_t)seg_off[E] * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float z = ld(&g[i]);
    float s = 1.0f / (1.0f + expf(-z));
    st(&h[i], z * s * ld(&u[i]));
  }
}

// silu_mul_bwd (src/mixtral.rs:953-964): dg = dh*u*s*(1+z(1-s)), du = dh*silu(z).
template <typename T>
__global__ void k_silu_mul_bwd(const float* __restrict__ dh, const T* __restrict__ g,
                               const T* __restrict__ u, const int* __restrict__ seg_off, int E,
                               int64_t I, T* __restrict__ dg, T* __restrict__ du) {
  int64_t n = (int64_t)seg_off[E] * I;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float z = ld(&g[i]);
    float s = 1.0f / (1.0f + expf(-z));
    float dsilu = s * (1.0f + z * (1.0f - s));
    float d = dh[i];
    st(&dg[i], d * ld(&u[i]) * dsilu);
    st(&du[i], d * (z * s));
  }
}

// ------------------------------------------------------ combine (K9 tail)
// y[t] = mid[t] + sum_k w_k * out[row(t,k)], the slot sum taken in slot
// order from zero as in src/mixtral.rs:330-359.
__global__ void k_combine(const float* __restrict__ mid, const float* __restrict__ out,
                          const int* __restrict__ slot_row, const float* __restrict__ top_w,
                          int K, int D, float* __restrict__ y) {
  const int64_t t = blockIdx.x;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float m = 0.f;
    for (int k = 0; k < K; ++k) {
      int64_t r = slot_row[t * K + k];
      m += top_w[t * K + k] * out[r * D + i];
    }
    y[t * D + i] = mid[t * D + i] + m;
  }
}

// ------------------------------------------- router Jacobian / mix bwd (K10)
// src/mixtral.rs:456-541 for one token: dvalue_k = <dy, out_k>,
// dvalues_k = (dvalue_k - sum_j w_j dvalue_j) / s with s = sum top_p,
// dz = p (dp - <p, dp>).
__global__ void k_router_bwd(const float* __restrict__ dy, const float* __restrict__ out,
                             const int* __restrict__ slot_row, const int* __restrict__ top_i,
                             const float* __restrict__ top_p, const float* __restrict__ top_w,
                             const float* __restrict__ probs, int E, int K, int D,
                             float* __restrict__ dz) {
  const int64_t t = blockIdx.x;
  __shared__ float red[kMaxTopK][32];
  __shared__ float dv[kMaxTopK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = 0; k < K; ++k) {
    const int64_t r = slot_row[t * K + k];
    float acc = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) acc += dy[t * D + i] * out[r * D + i];
    acc = warp_sum(acc);
    if (lane == 0) red[k][warp] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f, wdot = 0.f;
    for (int k = 0; k < K; ++k) s += top_p[t * K + k];
    for (int k = 0; k < K; ++k) {
      float v = 0.f;
      for (int q = 0; q < (int)(blockDim.x >> 5); ++q) v += red[k][q];
      dv[k] = v;
      wdot += v * top_w[t * K + k];
    }
    float dp[kMaxExperts];
    for (int e = 0; e < E; ++e) dp[e] = 0.f;
    for (int k = 0; k < K; ++k) dp[top_i[t * K + k]] = dv[k] / s - wdot / s;
    float dot = 0.f;
    for (int e = 0; e < E; ++e) dot += probs[t * E + e] * dp[e];
    for (int e = 0; e < E; ++e) dz[t * E + e] = probs[t * E + e] * (dp[e] - dot);
  }
}

// d_xn2[t] = sum_k dXp[row(t,k)] + sum_e dz[t,e] * Wr[i,e]  (src/mixtral.rs:
// 516, 535-540: expert input cotangents in slot order, then the router's).
template <typename T>
__global__ void k_unpermute_router_dx(const float* __restrict__ dxp,
                                      const int* __restrict__ slot_row,
                                      const float* __restrict__ dz, const T* __restrict__ wr,
                                      int E, int K, int D, float* __restrict__ dxn) {
  const int64_t t = blockIdx.x;
  __shared__ float dzs[kMaxExperts];
  if (threadIdx.x < E) dzs[threadIdx.x] = dz[t * E + threadIdx.x];
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float a = 0.f;
    for (int k = 0; k < K; ++k) a += dxp[(int64_t)slot_row[t * K + k] * D + i];
    float rr = 0.f;
    for (int e = 0; e < E; ++e) rr += dzs[e] * ld(&wr[(int64_t)i * E + e]);
    dxn[t * D + i] = a + rr;
  }
}

// k_router_bwd with 4-wide dot products (D % 4 == 0, aligned rows): a thread
// takes the NV quads threadIdx.x + 256 j of the row and issues all of their
// loads (dy and the KK <= kMaxTopK expert-output rows) before the first
// product, so that NV (1 + K) 16-byte loads are in flight.
template <int NV, int KK>
__global__ void __launch_bounds__(256) k_router_bwd_v(
    const float* __restrict__ dy, const float* __restrict__ out, const int* __restrict__ slot_row,
    const int* __restrict__ top_i, const float* __restrict__ top_p, const float* __restrict__ top_w,
    const float* __restrict__ probs, int E, int K, int D, float* __restrict__ dz) {
  const int64_t t = blockIdx.x;
  __shared__ float red[kMaxTopK][32];
  __shared__ float dv[kMaxTopK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D4 = D / 4;
  int64_t rows[KK];
#pragma unroll
  for (int k = 0; k < KK; ++k) rows[k] = k < K ? slot_row[t * K + k] : 0;
  float4 g[NV], o[NV][KK];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + 256 * j;
    g[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < D4) g[j] = ld4(dy + t * D + 4 * i);
#pragma unroll
    for (int k = 0; k < KK; ++k) {
      o[j][k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < K && i < D4) o[j][k] = ld4(out + rows[k] * D + 4 * i);
    }
  }
  float acc[KK];
#pragma unroll
  for (int k = 0; k < KK; ++k) {
    acc[k] = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
      acc[k] += g[j].x * o[j][k].x + g[j].y * o[j][k].y + g[j].z * o[j][k].z + g[j].w * o[j][k].w;
  }
#pragma unroll
  for (int k = 0; k < KK; ++k) {
    if (k < K) {
      const float v = warp_sum(acc[k]);
      if (lane == 0) red[k][warp] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f, wdot = 0.f;
    for (int k = 0; k < K; ++k) s += top_p[t * K + k];
    for (int k = 0; k < K; ++k) {
      float v = 0.f;
      for (int q = 0; q < (int)(blockDim.x >> 5); ++q) v += red[k][q];
      dv[k] = v;
      wdot += v * top_w[t * K + k];
    }
    float dp[kMaxExperts];
    for (int e = 0; e < E; ++e) dp[e] = 0.f;
    for (int k = 0; k < K; ++k) dp[top_i[t * K + k]] = dv[k] / s - wdot / s;
    float dot = 0.f;
    for (int e = 0; e < E; ++e) dot += probs[t * E + e] * dp[e];
    for (int e = 0; e < E; ++e) dz[t * E + e] = probs[t * E + e] * (dp[e] - dot);
  }
}

// k_unpermute_router_dx with 4-wide accesses: a thread takes the NV quads
// threadIdx.x + 256 j of the token's row and issues every expert-row load
// (KK >= K of them per quad) before the first sum, so that NV K 16-byte loads
// are in flight; the router rows (E8: 8 experts, 16 or 32 bytes a row) come
// from L1.  Per element the sums run in the same order as
// k_unpermute_router_dx's.
template <typename T, bool E8, int NV, int KK>
__global__ void __launch_bounds__(256) k_unpermute_router_dx_v(
    const float* __restrict__ dxp, const int* __restrict__ slot_row, const float* __restrict__ dz,
    const T* __restrict__ wr, int E, int K, int D, float* __restrict__ dxn) {
  const int64_t t = blockIdx.x;
  __shared__ float dzs[kMaxExperts];
  __shared__ int64_t rows[kMaxTopK];
  if (threadIdx.x < E) dzs[threadIdx.x] = dz[t * E + threadIdx.x];
  if (threadIdx.x < K) rows[threadIdx.x] = slot_row[t * K + threadIdx.x];
  __syncthreads();
  const int D4 = D / 4;
  float4 v[NV][KK];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + 256 * j;
#pragma unroll
    for (int k = 0; k < KK; ++k)
      v[j][k] = (i < D4 && k < K) ? ld4(dxp + rows[k] * D + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + 256 * j;
    if (i >= D4) continue;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < KK; ++k) {
      if (k < K) { a.x += v[j][k].x; a.y += v[j][k].y; a.z += v[j][k].z; a.w += v[j][k].w; }
    }
    float rr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const T* wrow = wr + (int64_t)(4 * i + u) * E;
      float acc = 0.f;
      if (E8) {
        float wv8[8];
        ld_row8(wrow, wv8);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc += dzs[e] * wv8[e];
      } else {
        for (int e = 0; e < E; ++e) acc += dzs[e] * ld(&wrow[e]);
      }
      rr[u] = acc;
    }
    st4(dxn + t * D + 4 * i, make_float4(a.x + rr[0], a.y + rr[1], a.z + rr[2], a.w + rr[3]));
  }
}

// k_unpermute_router_dx with the router rows held in registers: a thread
// owns four columns (one quad) of the model dimension, reads their router
// rows once, and runs over a chunk of kUdTok tokens (their dz and expert rows
// staged in shared memory), four tokens' loads in flight.  The weights are
// read once per chunk instead of once per token; per element the sums run in
// the same order as k_unpermute_router_dx's.
constexpr int kUdTok = 64;
template <typename T, int NE, int KK>
__global__ void __launch_bounds__(256) k_unpermute_router_dx_ws(
    const float* __restrict__ dxp, const int* __restrict__ slot_row, const float* __restrict__ dz,
    const T* __restrict__ wr, int64_t Tn, int E, int K, int D, float* __restrict__ dxn) {
  __shared__ float dzs[kUdTok][NE];
  __shared__ int64_t rows_s[kUdTok][kMaxTopK];
  const int64_t t0 = (int64_t)blockIdx.y * kUdTok;
  const int nt = (int)(Tn - t0 < kUdTok ? Tn - t0 : kUdTok);
  for (int k = threadIdx.x; k < kUdTok * NE; k += blockDim.x) {
    const int tt = k / NE, e = k % NE;
    dzs[tt][e] = (tt < nt && e < E) ? dz[(t0 + tt) * E + e] : 0.f;
  }
  for (int k = threadIdx.x; k < kUdTok * kMaxTopK; k += blockDim.x) {
    const int tt = k / kMaxTopK, j = k % kMaxTopK;
    rows_s[tt][j] = (tt < nt && j < K) ? slot_row[(t0 + tt) * K + j] : 0;
  }
  __syncthreads();
  const int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= D) return;
  float w[4][NE];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const T* wrow = wr + (int64_t)(i + u) * E;
    if (NE == 8 && E == 8) {
      ld_row8(wrow, w[u]);
    } else {
#pragma unroll
      for (int e = 0; e < NE; ++e) w[u][e] = e < E ? ld(&wrow[e]) : 0.f;
    }
  }
  for (int tt0 = 0; tt0 < nt; tt0 += 4) {
    float4 v[4][KK];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < KK; ++k)
        if (tt0 + q < nt && k < K) v[q][k] = ld4(dxp + rows_s[tt0 + q][k] * D + i);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int tt = tt0 + q;
      if (tt >= nt) break;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < KK; ++k) {
        if (k < K) { a.x += v[q][k].x; a.y += v[q][k].y; a.z += v[q][k].z; a.w += v[q][k].w; }
      }
      float rr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < NE; ++e)
          if (NE == 8 || e < E) acc += dzs[tt][e] * w[u][e];
        rr[u] = acc;
      }
      st4(dxn + (t0 + tt) * D + i, make_float4(a.x + rr[0], a.y + rr[1], a.z + rr[2], a.w + rr[3]));
    }
  }
}

// Router weight adjoint partials: part[c, i, e] = sum_{t in chunk c}
// xn2[t,i] * dz[t,e] with xn2 recomputed in fp32 from (mid, inv, w).
template <typename T>
__global__ void k_router_dw(const float* __restrict__ mid, const float* __restrict__ inv,
                            const T* __restrict__ w, const float* __restrict__ dz, int64_t rows,
                            int D, int E, int rows_per_chunk, float* __restrict__ part) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int c = blockIdx.y;
  if (i >= D) return;
  const int64_t t0 = (int64_t)c * rows_per_chunk;
  const int64_t t1 = ::min((int64_t)(rows), (int64_t)(t0 + rows_per_chunk));
  float acc[kMaxExperts];
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e) acc[e] = 0.f;
  const float wi = ld(&w[i]);
  for (int64_t t = t0; t < t1; ++t) {
    float xn = mid[t * D + i] * inv[t] * wi;
#pragma unroll
    for (int e = 0; e < kMaxExperts; ++e)
      if (e < E) acc[e] += xn * dz[t * E + e];
  }
#pragma unroll
  for (int e = 0; e < kMaxExperts; ++e)
    if (e < E) part[((int64_t)c * D + i) * E + e] = acc[e];
}

// k_router_dw for 8 experts with two columns a thread and sixteen rows'
// loads in flight (the scalar kernel has one 4-byte load in flight per
// thread and is latency-bound); the rows' dz and inv are staged in shared
// memory 256 rows at a time.  Same products summed in the same row order
// per element, so the partials are bit-identical to k_router_dw's.
constexpr int kRdwRows = 256;
template <typename T>
__global__ void __launch_bounds__(128, 5) k_router_dw_v(const float* __restrict__ mid,
                                                     const float* __restrict__ inv,
                                                     const T* __restrict__ w,
                                                     const float* __restrict__ dz, int64_t rows,
                                                     int D, int rows_per_chunk,
                                                     float* __restrict__ part) {
  constexpr int E = 8, U = 16;
  __shared__ __align__(16) float dzs[kRdwRows][E];
  __shared__ float ivs[kRdwRows];
  const int i2 = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  const bool col_ok = i2 < D;
  const int c = blockIdx.y;
  const int64_t t0 = (int64_t)c * rows_per_chunk;
  const int64_t t1 = ::min((int64_t)rows, t0 + rows_per_chunk);
  float acc[2][E];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[q][e] = 0.f;
  const float wq[2] = {col_ok ? ld(&w[i2]) : 0.f, col_ok ? ld(&w[i2 + 1]) : 0.f};
  for (int64_t p0 = t0; p0 < t1; p0 += kRdwRows) {
    const int np = (int)::min((int64_t)kRdwRows, t1 - p0);
    __syncthreads();
    for (int k = threadIdx.x; k < np * E; k += blockDim.x) dzs[k / E][k % E] = dz[p0 * E + k];
    for (int k = threadIdx.x; k < np; k += blockDim.x) ivs[k] = inv[p0 + k];
    __syncthreads();
    if (!col_ok) continue;
    for (int r = 0; r < np; r += U) {
      float2 mv[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (r + u < np) mv[u] = *reinterpret_cast<const float2*>(mid + (p0 + r + u) * D + i2);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (r + u < np) {
          const float4 d0 = *reinterpret_cast<const float4*>(&dzs[r + u][0]);
          const float4 d1 = *reinterpret_cast<const float4*>(&dzs[r + u][4]);
          const float dv[E] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
          const float mq[2] = {mv[u].x, mv[u].y};
          const float iv = ivs[r + u];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const float xn = mq[q] * iv * wq[q];
#pragma unroll
            for (int e = 0; e < E; ++e) acc[q][e] += xn * dv[e];
          }
        }
      }
    }
  }
  if (!col_ok) return;
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int e = 0; e < E; ++e) part[((int64_t)c * D + i2 + q) * E + e] = acc[q][e];
}

// --------------------------------------------------------------- misc
template <typename T>
__global__ void k_convert(const float* __restrict__ s, T* __restrict__ d, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    st(&d[i], s[i]);
}

// Column sums of x[rows, cols]: part[c, j] = sum over row chunk c.
__global__ void k_col_part(const float* __restrict__ x, int64_t rows, int64_t cols,
                           int rows_per_chunk, float* __restrict__ part) {
  int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int c = blockIdx.y;
  if (j >= cols) return;
  int64_t r0 = (int64_t)c * rows_per_chunk, r1 = ::min((int64_t)(rows), (int64_t)(r0 + rows_per_chunk));
  float s = 0.f;
  for (int64_t r = r0; r < r1; ++r) s += x[r * cols + j];
  part[(int64_t)c * cols + j] = s;
}

__global__ void k_set_chunks(const float* __restrict__ part, int chunks, int64_t n,
                             float* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += part[(int64_t)c * n + i];
  out[i] = s;
}

__global__ void k_add(float* __restrict__ d, const float* __restrict__ s, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    d[i] += s[i];
}

__global__ void k_relu_mask_bwd(float* __restrict__ dy, const uint8_t* __restrict__ m, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    if (m[i] == 0) dy[i] = 0.f;
}

// Mean-squared error, one CTA: loss = sum (y-t)^2 / n, dy = 2 (y-t) / n.
__global__ void k_mse(const float* __restrict__ y, const float* __restrict__ t, int64_t n,
                      float* __restrict__ loss, float* __restrict__ dy) {
  __shared__ float red[32];
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float d = y[i] - t[i];
    acc += d * d;
    dy[i] = 2.0f * d / (float)n;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) s += red[q];
    *loss = s / (float)n;
  }
}

__global__ void k_sgd(float* __restrict__ p, const float* __restrict__ g, int64_t n, float lr) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] -= lr * g[i];
}

__global__ void k_fill_i32(int* __restrict__ p, int64_t n, int v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ----------------------------------------------------------- launchers
static int grid_for(int64_t n, int block) {
  int64_t g = ceil_div(n, block);
  int64_t cap = (int64_t)sm_count() * 16;
  return (int)(g < cap ? (g > 0 ? g : 1) : cap);
}

// Quads per thread of the vectorised row kernels (256 threads): 1, 2, 4 or 8,
// or 0 when D is not a multiple of 4 or too wide for registers.
static int row_quads(int D) {
  if (D % 4 != 0 || D > 4 * 256 * 8) return 0;
  const int need = (int)ceil_div(D / 4, 256);
  return need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : 8;
}

template <typename T>
void rmsnorm_fwd(const float* x, const T* w, int64_t rows, int D, float eps, T* y, float* inv,
                 float* x_copy, cudaStream_t s, int64_t& launches) {
  const int nv = row_quads(D);
  if (nv && aligned4(x) && aligned4(w) && aligned4(y) && (!x_copy || aligned4(x_copy))) {
    auto k = nv == 1 ? k_rmsnorm_fwd_v<T, 1> : nv == 2 ? k_rmsnorm_fwd_v<T, 2>
           : nv == 4 ? k_rmsnorm_fwd_v<T, 4> : k_rmsnorm_fwd_v<T, 8>;
    k<<<(unsigned)rows, 256, 0, s>>>(x, w, D, eps, y, inv, x_copy);
  } else {
    k_rmsnorm_fwd<T><<<(unsigned)rows, 256, 0, s>>>(x, w, D, eps, y, inv, x_copy);
  }
  DOP_LAUNCHED(launches);
}

template <typename T>
void rmsnorm_router(const float* x, const T* w, const T* wr, const float* bias, int64_t rows,
                    int D, int E, int K, float eps, T* y, float* inv, float* probs, int* top_i,
                    float* top_p, float* top_w, cudaStream_t s, int64_t& launches) {
  DOP_REQUIRE(E <= kMaxExperts && K <= kMaxTopK && K <= E, "experts/top_k out of range");
  const bool vec = D % 4 == 0 && aligned4(x) && aligned4(y);
  // one row a thread, one-warp CTAs so that the SMs' shares differ by at most a warp
  if (vec) k_router_rms<true><<<(unsigned)ceil_div(rows, 32), 32, 0, s>>>(x, rows, D, eps, inv);
  else k_router_rms<false><<<(unsigned)ceil_div(rows, 32), 32, 0, s>>>(x, rows, D, eps, inv);
  DOP_LAUNCHED(launches);
  const unsigned grid = (unsigned)ceil_div(rows, kRtRows * kRtWarps);
  const dim3 block(32 * kRtWarps);
#define DOP_ROUTER(NE)                                                                        \
  (vec ? k_router_logits<T, NE, true> : k_router_logits<T, NE, false>)<<<grid, block, 0, s>>>( \
      x, w, wr, bias, rows, D, E, K, inv, y, probs, top_i, top_p, top_w)
  if (E == 1) DOP_ROUTER(1);
  else if (E <= 4) DOP_ROUTER(4);
  else if (E <= 8) DOP_ROUTER(8);
  else DOP_ROUTER(16);
#undef DOP_ROUTER
  DOP_LAUNCHED(launches);
}

template <typename T>
void rmsnorm_bwd(const float* dy, const float* x, const float* inv, const T* w,
                 const float* res, int64_t rows, int D, float* dx, T* dx_act, float* dw_accum,
                 float* part_buf, int64_t part_cap, cudaStream_t s, int64_t& launches) {
  if (rows <= 0 || D <= 0) return;  // nothing to do (and no empty grid)
  const bool vec = D % 128 == 0 && aligned4(dy) && aligned4(x) && aligned4(w) &&
                   (!res || aligned4(res)) && aligned4(dx) && (!dx_act || aligned4(dx_act));
  const int nv = row_quads(D);
  if (vec && nv && nv <= 4 && aligned4(part_buf)) {
    // the input adjoint and the weight adjoint's partials in one pass over
    // dy and x, three CTAs per SM, each walking a chunk of rows
    int64_t chunks = std::min<int64_t>({rows, part_cap / D, 3 * (int64_t)sm_count()});
    chunks = std::max<int64_t>(1, chunks);
    const int rows_per_chunk = (int)ceil_div(rows, chunks);
    chunks = ceil_div(rows, rows_per_chunk);
    auto k = nv == 1 ? k_rmsnorm_bwd_dw_v<T, 1> : nv == 2 ? k_rmsnorm_bwd_dw_v<T, 2>
                                                          : k_rmsnorm_bwd_dw_v<T, 4>;
    k<<<(unsigned)chunks, 256, 0, s>>>(dy, x, inv, w, res, rows, D, rows_per_chunk, dx, dx_act,
                                       part_buf);
    DOP_LAUNCHED(launches);
    k_reduce_chunks_wide<<<(unsigned)ceil_div(D, 32), 1024, 0, s>>>(part_buf, (int)chunks, D,
                                                                    dw_accum);
    DOP_LAUNCHED(launches);
    return;
  }
  if (vec && nv) {
    auto k = nv == 1 ? k_rmsnorm_bwd_v<T, 1> : nv == 2 ? k_rmsnorm_bwd_v<T, 2>
           : nv == 4 ? k_rmsnorm_bwd_v<T, 4> : k_rmsnorm_bwd_v<T, 8>;
    k<<<(unsigned)rows, 256, 0, s>>>(dy, x, inv, w, res, D, dx, dx_act);
  } else {
    k_rmsnorm_bwd_rows<T><<<(unsigned)ceil_div(rows, 8), 256, 0, s>>>(dy, x, inv, w, res, rows,
                                                                       D, dx, dx_act, vec);
  }
  DOP_LAUNCHED(launches);
  int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(rows, 64));
  int rows_per_chunk = (int)ceil_div(rows, chunks);
  chunks = ceil_div(rows, rows_per_chunk);
  DOP_REQUIRE(chunks * D <= part_cap, "partial buffer too small");
  dim3 grid((unsigned)ceil_div(D, 128), (unsigned)chunks);
  k_rmsnorm_dw_part<<<grid, 128, 0, s>>>(dy, x, inv, rows, D, rows_per_chunk, part_buf);
  DOP_LAUNCHED(launches);
  k_reduce_chunks<<<(unsigned)ceil_div(D, 256), 256, 0, s>>>(part_buf, (int)chunks, D, dw_accum);
  DOP_LAUNCHED(launches);
}

void rope_table(int S, int hd, float theta, float* cs, float* sn, cudaStream_t s,
                int64_t& launches) {
  int half = hd / 2;
  int64_t n = (int64_t)S * half;
  k_rope_table<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(S, half, hd, theta, cs, sn);
  DOP_LAUNCHED(launches);
}

template <typename TI, typename TO>
void rope(const TI* src, TO* dst, int64_t T, int S, int heads, int hd, const float* cs,
          const float* sn, float sign, cudaStream_t s, int64_t& launches) {
  int64_t n = T * heads * (hd / 2);
  k_rope<TI, TO><<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(src, dst, T, S, heads, hd, cs, sn,
                                                            sign);
  DOP_LAUNCHED(launches);
}

void permute(const int* top_i, const float* top_w, int64_t T, int E, int K, int* chunk_counts,
             int* seg_off, int* tile_expert, int max_tiles, int* slot_row, int* row_token,
             float* row_w, int64_t rows_cap, cudaStream_t s, int64_t& launches) {
  int64_t pairs = T * K;
  int chunks = (int)ceil_div(pairs, kPermChunk);
  k_fill_i32<<<grid_for(rows_cap, 256), 256, 0, s>>>(row_token, rows_cap, -1);
  DOP_LAUNCHED(launches);
  k_perm_count<<<chunks, 256, 0, s>>>(top_i, pairs, E, chunk_counts);
  DOP_LAUNCHED(launches);
  k_perm_scan<<<1, 256, 0, s>>>(chunk_counts, chunks, E, seg_off, tile_expert, max_tiles);
  DOP_LAUNCHED(launches);
  k_perm_scatter<<<chunks, kPermChunk, 0, s>>>(top_i, top_w, pairs, E, K, chunk_counts, seg_off,
                                               slot_row, row_token, row_w);
  DOP_LAUNCHED(launches);
}

template <typename T>
void gather_rows(const T* src, const int* row_token, const int* seg_off, int E, int D,
                 int64_t rows_cap, T* dst, cudaStream_t s, int64_t& launches) {
  const int64_t bytes = (int64_t)D * sizeof(T);
  if (bytes % 16 == 0 && (uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0)
    k_gather_rows16<<<(unsigned)rows_cap, 128, 0, s>>>((const uint4*)src, row_token, seg_off, E,
                                                        (int)(bytes / 16), (uint4*)dst);
  else
    k_gather_rows<T><<<(unsigned)rows_cap, 256, 0, s>>>(src, row_token, seg_off, E, D, dst);
  DOP_LAUNCHED(launches);
}

template <typename T>
void scatter_rows(const T* src, const int* slot_row, int64_t Tn, int K, const int* row_token,
                  const int* seg_off, int E, int D, int64_t rows_cap, T* dst, cudaStream_t s,
                  int64_t& launches) {
  const int64_t bytes = (int64_t)D * sizeof(T);
  if (bytes % 16 != 0 || (uintptr_t)src % 16 != 0 || (uintptr_t)dst % 16 != 0 || K > kMaxTopK) {
    gather_rows<T>(src, row_token, seg_off, E, D, rows_cap, dst, s, launches);
    return;
  }
  const int n16 = (int)(bytes / 16);
  k_scatter_rows16<<<(unsigned)Tn, 128, 0, s>>>((const uint4*)src, slot_row, K, n16, (uint4*)dst);
  DOP_LAUNCHED(launches);
  k_zero_pad_rows16<<<(unsigned)ceil_div(rows_cap, 8), 256, 0, s>>>(row_token, seg_off, E, rows_cap,
                                                                     n16, (uint4*)dst);
  DOP_LAUNCHED(launches);
}

template <typename T>
void scatter_scale_rows(const float* src, const int* slot_row, const float* top_w, int64_t Tn,
                        int K, const int* row_token, const float* row_w, const int* seg_off, int E,
                        int D, int64_t rows_cap, T* dst, cudaStream_t s, int64_t& launches) {
  const int64_t bytes = (int64_t)D * sizeof(T);
  if (D % 4 != 0 || bytes % 16 != 0 || !aligned4(src) || (uintptr_t)dst % 16 != 0 ||
      K > kMaxTopK) {
    gather_scale_rows<T>(src, row_token, row_w, seg_off, E, D, rows_cap, dst, s, launches);
    return;
  }
  k_scatter_scale_rows_v<T><<<(unsigned)Tn, 256, 0, s>>>(src, slot_row, top_w, K, D, dst);
  DOP_LAUNCHED(launches);
  k_zero_pad_rows16<<<(unsigned)ceil_div(rows_cap, 8), 256, 0, s>>>(row_token, seg_off, E, rows_cap,
                                                                     (int)(bytes / 16), (uint4*)dst);
  DOP_LAUNCHED(launches);
}

template <typename T>
void gather_scale_rows(const float* src, const int* row_token, const float* row_w,
                       const int* seg_off, int E, int D, int64_t rows_cap, T* dst, cudaStream_t s,
                       int64_t& launches) {
  if (D % 4 == 0 && aligned4(src) && aligned4(dst))
    k_gather_scale_rows_v<T><<<(unsigned)rows_cap, 256, 0, s>>>(src, row_token, row_w, seg_off, E,
                                                                D, dst);
  else
    k_gather_scale_rows<T><<<(unsigned)rows_cap, 256, 0, s>>>(src, row_token, row_w, seg_off, E,
                                                              D, dst);
  DOP_LAUNCHED(launches);
}

template <typename T>
void silu_mul(const T* g, const T* u, const int* seg_off, int E, int64_t I, int64_t rows_cap,
              T* h, cudaStream_t s, int64_t& launches) {
  k_silu_mul<T><<<grid_for(rows_cap * I, 256), 256, 0, s>>>(g, u, seg_off, E, I, h);
  DOP_LAUNCHED(launches);
}

template <typename T>
void silu_mul_bwd(const float* dh, const T* g, const T* u, const int* seg_off, int E, int64_t I,
                  int64_t rows_cap, T* dg, T* du, cudaStream_t s, int64_t& launches) {
  k_silu_mul_bwd<T><<<grid_for(rows_cap * I, 256), 256, 0, s>>>(dh, g, u, seg_off, E, I, dg, du);
  DOP_LAUNCHED(launches);
}

void combine(const float* mid, const float* out, const int* slot_row, const float* top_w,
             int64_t T, int K, int D, float* y, cudaStream_t s, int64_t& launches) {
  if (D % 4 == 0 && aligned4(mid) && aligned4(out) && aligned4(y))
    k_combine_v<<<(unsigned)T, 256, 0, s>>>(mid, out, slot_row, top_w, K, D, y);
  else
    k_combine<<<(unsigned)T, 256, 0, s>>>(mid, out, slot_row, top_w, K, D, y);
  DOP_LAUNCHED(launches);
}

void router_bwd(const float* dy, const float* out, const int* slot_row, const int* top_i,
                const float* top_p, const float* top_w, const float* probs, int64_t Tn, int E,
                int K, int D, float* dz, cudaStream_t s, int64_t& launches) {
  const int nv = row_quads(D);
  if (nv && aligned4(dy) && aligned4(out)) {
#define DOP_RBWD(NV, KK) k_router_bwd_v<NV, KK><<<(unsigned)Tn, 256, 0, s>>>( \
    dy, out, slot_row, top_i, top_p, top_w, probs, E, K, D, dz)
    if (K <= 2) {
      if (nv == 1) DOP_RBWD(1, 2); else if (nv == 2) DOP_RBWD(2, 2);
      else if (nv == 4) DOP_RBWD(4, 2); else DOP_RBWD(8, 2);
    } else {
      if (nv == 1) DOP_RBWD(1, 4); else if (nv == 2) DOP_RBWD(2, 4);
      else if (nv == 4) DOP_RBWD(4, 4); else DOP_RBWD(8, 4);
    }
#undef DOP_RBWD
  } else
    k_router_bwd<<<(unsigned)Tn, 256, 0, s>>>(dy, out, slot_row, top_i, top_p, top_w, probs, E, K,
                                              D, dz);
  DOP_LAUNCHED(launches);
}

template <typename T>
void unpermute_router_dx(const float* dxp, const int* slot_row, const float* dz, const T* wr,
                         int64_t Tn, int E, int K, int D, float* dxn, cudaStream_t s,
                         int64_t& launches) {
  if (D % 4 == 0 && aligned4(dxp) && aligned4(dxn) && K <= kMaxTopK) {
    const dim3 grid((unsigned)ceil_div(D / 4, 256), (unsigned)ceil_div(Tn, kUdTok));
    const bool e8 = E == 8 && (uintptr_t)wr % 16 == 0;
#define DOP_UDWS(NE, KK) k_unpermute_router_dx_ws<T, NE, KK><<<grid, 256, 0, s>>>( \
    dxp, slot_row, dz, wr, Tn, E, K, D, dxn)
    if (e8 && K <= 2) DOP_UDWS(8, 2);
    else if (e8) DOP_UDWS(8, 4);
    else if (K <= 2) DOP_UDWS(kMaxExperts, 2);
    else DOP_UDWS(kMaxExperts, 4);
#undef DOP_UDWS
    DOP_LAUNCHED(launches);
    return;
  }
  const int nv = row_quads(D);
  if (nv && aligned4(dxp) && aligned4(dxn)) {
    const bool e8 = E == 8 && (uintptr_t)wr % 16 == 0;
#define DOP_UPDX(E8, NV, KK) k_unpermute_router_dx_v<T, E8, NV, KK><<<(unsigned)Tn, 256, 0, s>>>( \
    dxp, slot_row, dz, wr, E, K, D, dxn)
#define DOP_UPDX_NV(E8, KK)                          \
  if (nv == 1) DOP_UPDX(E8, 1, KK);                  \
  else if (nv == 2) DOP_UPDX(E8, 2, KK);             \
  else if (nv == 4) DOP_UPDX(E8, 4, KK);             \
  else DOP_UPDX(E8, 8, KK)
    if (e8 && K <= 2) { DOP_UPDX_NV(true, 2); }
    else if (e8) { DOP_UPDX_NV(true, 4); }
    else if (K <= 2) { DOP_UPDX_NV(false, 2); }
    else { DOP_UPDX_NV(false, 4); }
#undef DOP_UPDX_NV
#undef DOP_UPDX
  } else {
    k_unpermute_router_dx<T><<<(unsigned)Tn, 256, 0, s>>>(dxp, slot_row, dz, wr, E, K, D, dxn);
  }
  DOP_LAUNCHED(launches);
}

template <typename T>
void router_dw(const float* mid, const float* inv, const T* w, const float* dz, int64_t rows,
               int D, int E, float* dwr_accum, float* part_buf, int64_t part_cap,
               cudaStream_t s, int64_t& launches) {
  const bool vec = E == 8 && D % 4 == 0 && aligned4(mid) && aligned4(w) && aligned4(dz);
  // the 4-wide kernel: as many row chunks as fill one wave of resident CTAs
  // (five per SM) over the column blocks, at most 64
  const int64_t col_blocks = ceil_div(D / 2, 128);
  int64_t chunks = vec ? std::max<int64_t>(1, std::min<int64_t>(64, 5 * sm_count() / col_blocks)) : 64;
  chunks = std::min<int64_t>(rows, chunks);
  int rows_per_chunk = (int)ceil_div(rows, chunks);
  chunks = ceil_div(rows, rows_per_chunk);
  DOP_REQUIRE(chunks * D * E <= part_cap, "partial buffer too small");
  if (vec) {
    dim3 grid((unsigned)col_blocks, (unsigned)chunks);
    k_router_dw_v<T><<<grid, 128, 0, s>>>(mid, inv, w, dz, rows, D, rows_per_chunk, part_buf);
  } else {
    dim3 grid((unsigned)ceil_div(D, 128), (unsigned)chunks);
    k_router_dw<T><<<grid, 128, 0, s>>>(mid, inv, w, dz, rows, D, E, rows_per_chunk, part_buf);
  }
  DOP_LAUNCHED(launches);
  k_reduce_chunks<<<(unsigned)ceil_div((int64_t)D * E, 256), 256, 0, s>>>(part_buf, (int)chunks,
                                                                           (int64_t)D * E, dwr_accum);
  DOP_LAUNCHED(launches);
}

template <typename T>
void convert(const float* src, T* dst, int64_t n, cudaStream_t s, int64_t& launches) {
  k_convert<T><<<grid_for(n, 256), 256, 0, s>>>(src, dst, n);
  DOP_LAUNCHED(launches);
}

void col_sum(const float* x, int64_t rows, int64_t cols, float* out, float* part_buf,
             int64_t part_cap, bool accumulate, cudaStream_t s, int64_t& launches) {
  int64_t chunks = std::max<int64_t>(1, std::min<int64_t>(rows, 64));
  int rows_per_chunk = (int)ceil_div(rows, chunks);
  chunks = std::max<int64_t>(1, ceil_div(rows, rows_per_chunk));
  DOP_REQUIRE(chunks * cols <= part_cap, "partial buffer too small");
  dim3 grid((unsigned)ceil_div(cols, 128), (unsigned)chunks);
  k_col_part<<<grid, 128, 0, s>>>(x, rows, cols, rows_per_chunk, part_buf);
  DOP_LAUNCHED(launches);
  if (accumulate)
    k_reduce_chunks<<<(unsigned)ceil_div(cols, 256), 256, 0, s>>>(part_buf, (int)chunks, cols, out);
  else
    k_set_chunks<<<(unsigned)ceil_div(cols, 256), 256, 0, s>>>(part_buf, (int)chunks, cols, out);
  DOP_LAUNCHED(launches);
}

void add_inplace(float* dst, const float* src, int64_t n, cudaStream_t s, int64_t& launches) {
  k_add<<<grid_for(n, 256), 256, 0, s>>>(dst, src, n);
  DOP_LAUNCHED(launches);
}

void relu_mask_bwd(float* dy, const uint8_t* mask, int64_t n, cudaStream_t s, int64_t& launches) {
  k_relu_mask_bwd<<<grid_for(n, 256), 256, 0, s>>>(dy, mask, n);
  DOP_LAUNCHED(launches);
}

void mse(const float* y, const float* t, int64_t n, float* loss, float* dy, cudaStream_t s,
         int64_t& launches) {
  k_mse<<<1, 1024, 0, s>>>(y, t, n, loss, dy);
  DOP_LAUNCHED(launches);
}

void sgd(float* p, const float* g, int64_t n, float lr, cudaStream_t s, int64_t& launches) {
  k_sgd<<<grid_for(n, 256), 256, 0, s>>>(p, g, n, lr);
  DOP_LAUNCHED(launches);
}

// explicit instantiations for the two activation types
#define DOP_INST(T)                                                                             \
  template void rmsnorm_fwd<T>(const float*, const T*, int64_t, int, float, T*, float*, float*, \
                               cudaStream_t, int64_t&);                                         \
  template void rmsnorm_router<T>(const float*, const T*, const T*, const float*, int64_t, int, \
                                  int, int, float, T*, float*, float*, int*, float*, float*,    \
                                  cudaStream_t, int64_t&);                                      \
  template void rmsnorm_bwd<T>(const float*, const float*, const float*, const T*,             \
                               const float*, int64_t, int, float*, T*, float*, float*, int64_t, \
                               cudaStream_t, int64_t&);                                         \
  template void gather_scale_rows<T>(const float*, const int*, const float*, const int*, int,  \
                                     int, int64_t, T*, cudaStream_t, int64_t&);                 \
  template void scatter_scale_rows<T>(const float*, const int*, const float*, int64_t, int,    \
                                      const int*, const float*, const int*, int, int, int64_t, \
                                      T*, cudaStream_t, int64_t&);                              \
  template void convert<T>(const float*, T*, int64_t, cudaStream_t, int64_t&);                  \
  template void rope<float, T>(const float*, T*, int64_t, int, int, int, const float*,         \
                               const float*, float, cudaStream_t, int64_t&);                    \
  template void gather_rows<T>(const T*, const int*, const int*, int, int, int64_t, T*,        \
                               cudaStream_t, int64_t&);                                         \
  template void scatter_rows<T>(const T*, const int*, int64_t, int, const int*, const int*, int, \
                                int, int64_t, T*, cudaStream_t, int64_t&);                       \
  template void silu_mul<T>(const T*, const T*, const int*, int, int64_t, int64_t, T*,         \
                            cudaStream_t, int64_t&);                                            \
  template void silu_mul_bwd<T>(const float*, const T*, const T*, const int*, int, int64_t,    \
                                int64_t, T*, T*, cudaStream_t, int64_t&);                       \
  template void unpermute_router_dx<T>(const float*, const int*, const float*, const T*,       \
                                       int64_t, int, int, int, float*, cudaStream_t, int64_t&); \
  template void router_dw<T>(const float*, const float*, const T*, const float*, int64_t, int,  \
                             int, float*, float*, int64_t, cudaStream_t, int64_t&);

DOP_INST(float)
DOP_INST(bf16)

}  // namespace dop
