// attn_tc.cu — flash attention on the 5th-generation tensor cores (bf16,
// head_dim 128), the bf16 lens's gqa_forward / gqa_backward
// (src/mixtral.rs:799-922): causal sliding-window grouped-query attention,
// visible(q, k) = k <= q && q - k < W.
//
// Forward, one CTA per (pair of 128-query tiles, head, sequence):
//   warp 0      TMA: the two Q tiles once, then K and V tiles of 128 keys,
//               each into its own 2-stage ring (128B-swizzled, bf16)
//   warp 1      TMEM owner; one thread issues S_g = Q_g K^T into S_g and
//               O_g += P_g V (P_g read from TMEM) for both query tiles g
//   warps 2..9  softmax, one query row per thread, warps 2-5 for tile A and
//               6-9 for tile B: online max / sum in the log2 domain, P_g
//               written back over S_g in TMEM as packed bf16, O_g rescaled
//               in TMEM only when the row max grows by more than 2^8, and
//               the log-sum-exp kept for the backward pass.
// The tensor core alternates between the tiles: while one tile's softmax
// runs, the other tile's P V and next S run.
#include "kernels.cuh"
#include "tc_ptx.cuh"

namespace dop {
namespace tc {

constexpr int AT = 128;             // queries per CTA and keys per tile
constexpr int HD = 128;             // head dim
constexpr uint32_t HALF = 16384;    // [128 rows][64 cols] bf16 box
constexpr uint32_t TILE = 2 * HALF; // [128 rows][128 cols] bf16 as two 64-col boxes
constexpr float kLog2e = 1.4426950408889634f;

struct FwdParams {
  int S, H, KV, group, window, n_qt;
  float sl2;  // softmax scale * log2(e)
  bf16* o;
  float* lse;
};

// Write 32 bf16 values (row `r`, columns c0..c0+31 of a [128][128] K-major
// tile stored as two 128B-swizzled 64-column boxes) to shared memory.
__device__ __forceinline__ void st_tile_row32(uint8_t* tile, int r, int c0, const float* v) {
  const int atom = c0 >> 6;
  uint8_t* rowp = tile + atom * HALF + r * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int chunk = ((c0 & 63) >> 3) + q;
    const int swz = chunk ^ (r & 7);
    uint4 val = make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7]));
    *reinterpret_cast<uint4*>(rowp + swz * 16) = val;
  }
}

// Forward, one CTA per (256-query pair of tiles, head, sequence), 320
// threads: warp 0 TMA, warp 1 MMA, warps 2-5 softmax of query tile A
// (rows q0..q0+127), warps 6-9 softmax of tile B (q0+128..q0+255).
// TMEM columns: S_A 0-127 (P_A packed bf16 in 0-63), S_B 128-255, O_A 256-383,
// O_B 384-511.  O accumulates in TMEM (P V with accumulate); a row's running
// max is only raised when the new max exceeds it by more than kRescale (log2
// units), so O is rescaled in TMEM rarely.  The tensor core alternates
// between the tiles: PV_A, S_A(next) run while B's softmax works and back.
constexpr float kRescale = 8.0f;
// kPolyPairs of every 16 exponential pairs of the forward softmax (spread
// evenly) are evaluated by exp2_poly2 on the FMA pipe instead of the MUFU.
constexpr int kPolyPairs = 2;
__device__ __forceinline__ constexpr bool poly_pair(int i) { return (i * kPolyPairs) % 16 < kPolyPairs; }

__global__ void __launch_bounds__(320, 1)
    k_attn_fwd_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                  const __grid_constant__ CUtensorMap mv, const FwdParams p) {
  if (tc_failed()) return;  // an earlier wait failed: do nothing (sticky error)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;                // tiles A and B
  uint8_t* sK = smem + 2 * TILE;     // 2 stages
  uint8_t* sV = smem + 4 * TILE;     // 2 stages
  uint64_t* bars = (uint64_t*)(smem + 6 * TILE);
  uint32_t* tmem_slot = (uint32_t*)(bars + 16);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0, drain = b0 + 8;
  // K and V stages are released separately: K(t) once both S MMAs of tile t
  // are issued, V(t) once both P V MMAs are, so K(t+2) streams in while
  // tile t+1 is still on the tensor core.
  auto k_full = [&](int st) { return b0 + 16 + 8u * st; };
  auto k_empty = [&](int st) { return b0 + 32 + 8u * st; };
  auto s_full = [&](int g) { return b0 + 48 + 8u * g; };
  auto p_full = [&](int g) { return b0 + 64 + 8u * g; };
  auto o_done = [&](int g) { return b0 + 80 + 8u * g; };
  auto v_full = [&](int st) { return b0 + 96 + 8u * st; };
  auto v_empty = [&](int st) { return b0 + 112 + 8u * st; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pt = p.n_qt - 1 - (int)blockIdx.x;  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.group;
  const int q0 = pt * 2 * AT;
  const int row0 = b * p.S;
  // key-tile ranges of the two query tiles (empty when the tile is past S)
  int g_lo[2], g_hi[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int r0 = q0 + g * AT;
    if (r0 >= p.S) { g_lo[g] = 1; g_hi[g] = 0; continue; }
    g_lo[g] = max(0, r0 - p.window + 1) / AT;
    g_hi[g] = min(p.S - 1, r0 + AT - 1) / AT;
  }
  const int u0 = g_lo[0];
  const int u1 = max(g_hi[0], g_hi[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full(i), 1);
      mbar_init(k_empty(i), 1);
      mbar_init(v_full(i), 1);
      mbar_init(v_empty(i), 1);
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i), 4);
      mbar_init(o_done(i), 1);
    }
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_map(&mq);
      prefetch_map(&mk);
      prefetch_map(&mv);
      const uint32_t q_s = smem_u32(sQ);
      mbar_expect_tx(q_full, 2 * TILE);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        tma_load_3d(q_s + g * TILE, &mq, q_full, 0, h, row0 + q0 + g * AT);
        tma_load_3d(q_s + g * TILE + HALF, &mq, q_full, 64, h, row0 + q0 + g * AT);
      }
      int nk = 0, nv = 0;  // K and V tiles issued
      bool ok = true;
      for (int t = u0; t <= u1; ++t) {
        const int j = t - u0, st = j & 1, ph = ((j >> 1) & 1) ^ 1;
        const int k0 = t * AT;
        if (!mbar_wait(k_empty(st), ph, abort_flag, 11)) { ok = false; break; }
        const uint32_t ks = smem_u32(sK + st * TILE), vs = smem_u32(sV + st * TILE);
        mbar_expect_tx(k_full(st), TILE);
        tma_load_3d(ks, &mk, k_full(st), 0, kvh, row0 + k0);
        tma_load_3d(ks + HALF, &mk, k_full(st), 64, kvh, row0 + k0);
        ++nk;
        if (!mbar_wait(v_empty(st), ph, abort_flag, 10)) { ok = false; break; }
        mbar_expect_tx(v_full(st), TILE);
        tma_load_3d(vs, &mv, v_full(st), 0, kvh, row0 + k0);
        tma_load_3d(vs + HALF, &mv, v_full(st), 64, kvh, row0 + k0);
        ++nv;
      }
      if (!ok) {
        mbar_wait_drain(q_full, 0);
        for (int j = nk - 1; j >= 0 && j >= nk - 2; --j) mbar_wait_drain(k_full(j & 1), (j >> 1) & 1);
        for (int j = nv - 1; j >= 0 && j >= nv - 2; --j) mbar_wait_drain(v_full(j & 1), (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, 128, false, false);  // Q K^T
      constexpr uint32_t ID_PV = idesc_bf16(128, 128, false, true);  // P V (V N-major)
      const uint32_t q_s = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, 12);
      int nd0 = 0, nd1 = 0;     // tiles whose S was issued, per query tile
      int pd0 = -1, pd1 = -1;   // tile whose P V is still to issue, per query tile
      // P_g(tile) V(tile) into O_g; it must precede S_g(next), which
      // overwrites P_g in TMEM (tcgen05 MMAs of one thread run in order)
      auto issue_pv = [&](const int g, int& pend, const int nd, const int lo, const int hi) -> bool {
        const int t = pend;
        const int j = t - u0;
        if (!mbar_wait(p_full(g), (nd - 1) & 1, abort_flag, 13 + g)) return false;
        tc_fence_after();
        const uint32_t vs = smem_u32(sV + (j & 1) * TILE);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + 256 + g * 128, tmem + g * 128 + k * 8,
                      mnmajor_desc(vs + k * 2048, HALF), ID_PV, (t > lo || k > 0) ? 1u : 0u);
        pend = -1;
        if (t == hi) mma_commit(o_done(g));
        return true;
      };
      auto issue_s = [&](const int g, const uint32_t ks) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * HALF + (k & 3) * 32;
          mma_bf16(tmem + g * 128, kmajor_desc(q_s + g * TILE + off), kmajor_desc(ks + off), ID_S,
                   k > 0);
        }
        mma_commit(s_full(g));
      };
      const int lo0 = g_lo[0], hi0 = g_hi[0], lo1 = g_lo[1], hi1 = g_hi[1];
      for (int t = u0; t <= u1 && ok; ++t) {
        const int j = t - u0, st = j & 1;
        // P V of tile t-1 needs V(t-1)
        if ((pd0 >= 0 || pd1 >= 0) &&
            !mbar_wait(v_full((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag, 16)) { ok = false; break; }
        tc_fence_after();
        if (pd0 >= 0 && !issue_pv(0, pd0, nd0, lo0, hi0)) { ok = false; break; }
        if (!mbar_wait(k_full(st), (j >> 1) & 1, abort_flag, 15)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ks = smem_u32(sK + st * TILE);
        if (t >= lo0 && t <= hi0) { issue_s(0, ks); ++nd0; pd0 = t; }
        if (pd1 >= 0 && !issue_pv(1, pd1, nd1, lo1, hi1)) { ok = false; break; }
        // every P V that reads V(t-1) has been issued: release its stage
        if (j >= 1) mma_commit(v_empty((j - 1) & 1));
        if (t >= lo1 && t <= hi1) { issue_s(1, ks); ++nd1; pd1 = t; }
        mma_commit(k_empty(st));  // both S MMAs that read K(t) are issued
      }
      if (ok && (pd0 >= 0 || pd1 >= 0)) {
        const int j = u1 - u0;
        ok = mbar_wait(v_full(j & 1), (j >> 1) & 1, abort_flag, 16);
        tc_fence_after();
      }
      if (ok && pd0 >= 0 && !issue_pv(0, pd0, nd0, lo0, hi0)) ok = false;
      if (ok && pd1 >= 0 && !issue_pv(1, pd1, nd1, lo1, hi1)) ok = false;
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    // One query row per thread.  S is read from TMEM once (128 columns);
    // masks are applied only on tiles that cross the diagonal or the
    // window edge; the row max and sum use independent accumulators and
    // paired fp32 instructions so that a single warp per SM sub-partition
    // keeps its pipelines busy.
    const int g = (warp - 2) >> 2;          // query tile of this warp group
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int r0 = q0 + g * AT;
    const int qi = r0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t ts = tmem + g * 128 + lane_off;        // S_g, then P_g
    const uint32_t to = tmem + 256 + g * 128 + lane_off;  // O_g
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    const int my_lo = g ? g_lo[1] : g_lo[0];
    const int n = (g ? g_hi[1] : g_hi[0]) - my_lo + 1;
    const float2 sl2v = make_float2(p.sl2, p.sl2);
    for (int it = 0; it < n; ++it) {
      if (!mbar_wait(s_full(g), it & 1, abort_flag, 17 + g)) { ok = false; break; }
      tc_fence_after();
      const int k0 = (my_lo + it) * AT;
      // every (query, key) pair of the tile is visible: no masks
      const bool full = (k0 + AT - 1 <= r0) && (r0 + AT - 1 - k0 < p.window);
      float sv[128];
      tmem_ld128(ts, sv);
      if (!full) {
#pragma unroll
        for (int i = 0; i < 128; ++i) {
          const int key = k0 + i;
          if (!(key <= qi && qi - key < p.window)) sv[i] = -INFINITY;
        }
      }
      // row max of the raw scores (scaling by sl2 > 0 after the max gives
      // the same value as the max of the scaled scores)
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = fmax3(sv[u], sv[8 + u], sv[16 + u]);
#pragma unroll
      for (int i = 24; i < 120; i += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) a[u] = fmax3(a[u], sv[i + u], sv[i + 8 + u]);
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = fmaxf(a[u], sv[120 + u]);
      const float mx = fmaxf(fmax3(a[0], a[1], a[2]), fmax3(fmax3(a[3], a[4], a[5]), a[6], a[7])) *
                       p.sl2;
      // Raise the reference max when it grew by more than kRescale.  The
      // decision is per row, but the TMEM loads/stores that rescale O are
      // warp-collective, so the warp rescales when any of its rows needs it
      // (rows that do not keep alpha = 1).
      const bool raise = mx > m + kRescale || (m == -INFINITY && mx > -INFINITY);
      const float m_new = raise ? mx : m;
      const float alpha = raise ? (m == -INFINITY ? 0.f : fast_exp2(m - m_new)) : 1.f;
      const bool rescale = it > 0 && __any_sync(0xffffffffu, raise && m != -INFINITY);
      m = m_new;
      // P = 2^(s sl2 - m); a row with nothing visible yet (m = -inf) has
      // every score masked to -inf, and 2^(-inf) = 0
      const float nm = m == -INFINITY ? 0.f : -m;
      const float2 nmv = make_float2(nm, nm);
      if (rescale) {
        // O is complete (S_g(it) was issued after P V of the previous tile)
        // and stays so until p_full is signalled below; 16 columns at a
        // time, while the scores are held in registers
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          float ov[16];
          uint32_t ou[16];
          tmem_ld16(to + c * 16, ov);
#pragma unroll
          for (int i = 0; i < 16; ++i) ou[i] = __float_as_uint(ov[i] * alpha);
          tmem_st16u(to + c * 16, ou);
        }
      }
      float2 acc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] = make_float2(0.f, 0.f);
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(sv[qq * 32 + 2 * i], sv[qq * 32 + 2 * i + 1]), sl2v, nmv);
          // kPolyPairs of the 16 pairs on the FMA pipe, the rest on the MUFU
          const float2 e = poly_pair(i)
                               ? exp2_poly2(x)
                               : make_float2(fast_exp2(x.x), fast_exp2(x.y));
          acc[i & 3] = fadd2(acc[i & 3], e);
          pk[i] = pack_bf16(e.x, e.y);
        }
        tmem_st16u(ts + qq * 16, pk);
      }
      const float2 s01 = fadd2(acc[0], acc[1]), s23 = fadd2(acc[2], acc[3]);
      const float2 s4 = fadd2(s01, s23);
      l = l * alpha + (s4.x + s4.y);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(g));
    }
    if (n > 0 && ok && mbar_wait(o_done(g), 0, abort_flag, 19)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(to + c * 32, ov);
        if (qi < p.S) {
          uint4* dst = reinterpret_cast<uint4*>(p.o + ((int64_t)(row0 + qi) * p.H + h) * HD + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16(ov[8 * q] * inv_l, ov[8 * q + 1] * inv_l),
                                pack_bf16(ov[8 * q + 2] * inv_l, ov[8 * q + 3] * inv_l),
                                pack_bf16(ov[8 * q + 4] * inv_l, ov[8 * q + 5] * inv_l),
                                pack_bf16(ov[8 * q + 6] * inv_l, ov[8 * q + 7] * inv_l));
        }
      }
      // natural-log LSE of the scaled scores (m is in log2 units)
      if (qi < p.S) p.lse[((int64_t)b * p.H + h) * p.S + qi] = m / kLog2e + logf(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

constexpr size_t kFwdSmem = 6 * TILE + 1024 + 256;  // Q x2, K x2, V x2

// ------------------------------------------------------------------ backward
struct BwdParams {
  int S, H, KV, group, window, n_tiles;
  float sl2, scale;
  const float* lse;
  const float* delta;
  float* delta_out;  // written by the dQ kernel
  float* dq;
  float* dk;
  float* dv;
  AttnBwdBf16 o16;  // bf16 outputs (o16.dq set) instead of dq, dk, dv
};

// Row `pos` of a head's gradient, columns d and d + 64 (d in c0..c0+31) in
// a[] and b[]: rotate back by the RoPE adjoint (rope_qkv_transpose,
// src/mixtral.rs:777-797) when cs is set, round to bf16 and store.
__device__ __forceinline__ void store_grad_bf16(bf16* dst, int c0, const float* a, const float* b,
                                                const float* cs, const float* sn, int pos) {
  float o1[32], o2[32];
  if (cs) {
    const float4* c4 = reinterpret_cast<const float4*>(cs + (int64_t)pos * (HD / 2) + c0);
    const float4* s4 = reinterpret_cast<const float4*>(sn + (int64_t)pos * (HD / 2) + c0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 cv = c4[q], sv = s4[q];
      const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = 4 * q + u;
        o1[i] = a[i] * cc[u] + b[i] * ss[u];
        o2[i] = b[i] * cc[u] - a[i] * ss[u];
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) { o1[i] = a[i]; o2[i] = b[i]; }
  }
  uint4* d1 = reinterpret_cast<uint4*>(dst + c0);
  uint4* d2 = reinterpret_cast<uint4*>(dst + c0 + HD / 2);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    d1[q] = make_uint4(pack_bf16(o1[8 * q], o1[8 * q + 1]), pack_bf16(o1[8 * q + 2], o1[8 * q + 3]),
                       pack_bf16(o1[8 * q + 4], o1[8 * q + 5]), pack_bf16(o1[8 * q + 6], o1[8 * q + 7]));
    d2[q] = make_uint4(pack_bf16(o2[8 * q], o2[8 * q + 1]), pack_bf16(o2[8 * q + 2], o2[8 * q + 3]),
                       pack_bf16(o2[8 * q + 4], o2[8 * q + 5]), pack_bf16(o2[8 * q + 6], o2[8 * q + 7]));
  }
}

// Backward kernels.  Both use 320 threads: warp 0 TMA, warp 1 MMA, warps
// 2-5 and 6-9 two elementwise groups that take alternate tiles, so one
// group's exp/shuffle work overlaps the other group's MMAs.  The bf16
// operands the elementwise groups produce (dS, P^T, dS^T) are written back
// into the TMEM columns they were computed from and read from there as the
// A operand of the next MMA.
constexpr int QB = 64;               // queries per dK/dV tile, keys per dQ tile
constexpr uint32_t QHALF = 8192;     // [64 rows][64 cols] bf16 box
constexpr uint32_t QTILE = 2 * QHALF;
constexpr int BSTAGES = 4;

// dQ: one CTA per (128-query tile, head, sequence), 64-key tiles, 448
// threads: warp 0 TMA, warp 1 MMA, warps 2-13 three elementwise groups of
// four warps taking key tiles in turn (tile j to group j mod 3).
// TMEM: dQ 0-127; group g: S_g 128+128g (dS_g packed in its first 32
// columns), dP_g 192+128g.  Per key tile j: S = Q K_j^T, dP = dO V_j^T,
// dS = P (dP - delta) scale, dQ += dS K_j.  The MMA thread issues dQ_j after
// S_{j+2} and dP_{j+2}, so a group has two tiles of tensor-core work to turn
// S_j into dS_j.  The prologue also computes delta = rowsum(dO o O) from the
// dO and O tiles in shared memory (O loaded with Q and dO) and writes it for
// the dK/dV kernel, which runs next.
constexpr int DQ_GROUPS = 3;
constexpr int DQ_THREADS = 64 + DQ_GROUPS * 128 + 64;  // + the dQ (warp 14) and dP (warp 15) MMA issuers
__global__ void __launch_bounds__(DQ_THREADS, 1)
    k_attn_dq_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                 const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                 const __grid_constant__ CUtensorMap mo, const BwdParams p) {
  if (tc_failed()) return;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sQ = smem;
  uint8_t* sDO = smem + TILE;
  uint8_t* sO = smem + 2 * TILE;
  uint8_t* sK = smem + 3 * TILE;              // BSTAGES x [64 keys][128 d]
  uint8_t* sV = sK + BSTAGES * QTILE;
  uint64_t* bars = (uint64_t*)(sV + BSTAGES * QTILE);
  uint32_t* tmem_slot = (uint32_t*)(bars + 24);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t q_full = b0, dq_done = b0 + 8, drain = b0 + 16;
  auto kv_full = [&](int st) { return b0 + 24 + 8u * st; };
  auto kv_empty = [&](int st) { return b0 + 56 + 8u * st; };
  auto sd_full = [&](int g) { return b0 + 88 + 8u * g; };
  auto ds_full = [&](int g) { return b0 + 112 + 8u * g; };
  // group g's dS columns have been read by the dQ MMAs
  auto dq_free = [&](int g) { return b0 + 136 + 8u * g; };
  const uint32_t drain2 = b0 + 160, drain3 = b0 + 168;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_tiles - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.group;
  const int q0 = qt * AT;
  const int lo = max(0, q0 - p.window + 1) / QB;
  const int hi = min(p.S - 1, q0 + AT - 1) / QB;
  const int nt = hi - lo + 1;
  const int row0 = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(dq_done, 1);
    mbar_init(drain, 1);
    for (int st = 0; st < BSTAGES; ++st) {
      mbar_init(kv_full(st), 1);
      mbar_init(kv_empty(st), 1);
    }
    for (int g = 0; g < DQ_GROUPS; ++g) {
      mbar_init(sd_full(g), 2);  // the S and the dP issuer
      mbar_init(ds_full(g), 4);
      mbar_init(dq_free(g), 1);
    }
    mbar_init(drain2, 1);
    mbar_init(drain3, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qs = smem_u32(sQ), dos = smem_u32(sDO), os = smem_u32(sO);
      mbar_expect_tx(q_full, 3 * TILE);
      tma_load_3d(qs, &mq, q_full, 0, h, row0 + q0);
      tma_load_3d(qs + HALF, &mq, q_full, 64, h, row0 + q0);
      tma_load_3d(dos, &mdo, q_full, 0, h, row0 + q0);
      tma_load_3d(dos + HALF, &mdo, q_full, 64, h, row0 + q0);
      tma_load_3d(os, &mo, q_full, 0, h, row0 + q0);
      tma_load_3d(os + HALF, &mo, q_full, 64, h, row0 + q0);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nt; ++j) {
        const int st = j % BSTAGES;
        if (!mbar_wait(kv_empty(st), ((j / BSTAGES) & 1) ^ 1, abort_flag, 21)) { ok = false; break; }
        const int k0 = (lo + j) * QB;
        const uint32_t ks = smem_u32(sK + st * QTILE), vs = smem_u32(sV + st * QTILE);
        mbar_expect_tx(kv_full(st), 2 * QTILE);
        tma_load_3d(ks, &mk, kv_full(st), 0, kvh, row0 + k0);
        tma_load_3d(ks + QHALF, &mk, kv_full(st), 64, kvh, row0 + k0);
        tma_load_3d(vs, &mv, kv_full(st), 0, kvh, row0 + k0);
        tma_load_3d(vs + QHALF, &mv, kv_full(st), 64, kvh, row0 + k0);
        ++issued;
      }
      if (!ok) {
        mbar_wait_drain(q_full, 0);
        for (int j = issued - 1; j >= 0 && j >= issued - BSTAGES; --j)
          mbar_wait_drain(kv_full(j % BSTAGES), (j / BSTAGES) & 1);
      }
    }
  } else if (warp == 1 || warp == 15) {
    // S (warp 1) and dP (warp 15) are issued by two threads and dQ += dS K
    // by warp 14, so that three instruction streams are issued in parallel;
    // S and dP of tile j wait until the dQ MMAs of tile j - 3 (same group
    // columns) have run.
    if (lane == 0) {
      constexpr uint32_t ID_SD = idesc_bf16(128, 64, false, false);   // Q K^T, dO V^T
      const bool is_s = warp == 1;
      const uint32_t as = smem_u32(is_s ? sQ : sDO);
      uint8_t* const bstage = is_s ? sK : sV;
      const uint32_t dcol = is_s ? 128u : 192u;
      bool ok = mbar_wait(q_full, 0, abort_flag, 22);
      for (int j = 0; j < nt && ok; ++j) {
        const int g = j % DQ_GROUPS, st = j % BSTAGES;
        if (!mbar_wait(kv_full(st), (j / BSTAGES) & 1, abort_flag, 24)) { ok = false; break; }
        if (j >= DQ_GROUPS &&
            !mbar_wait(dq_free(g), ((j - DQ_GROUPS) / DQ_GROUPS) & 1, abort_flag, 27)) { ok = false; break; }
        tc_fence_after();
        const uint32_t bs = smem_u32(bstage + st * QTILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t oa = (k >> 2) * HALF + (k & 3) * 32;
          const uint32_t ob = (k >> 2) * QHALF + (k & 3) * 32;
          mma_bf16(tmem + dcol + g * 128, kmajor_desc(as + oa), kmajor_desc(bs + ob), ID_SD, k > 0);
        }
        mma_commit(sd_full(g));
      }
      const uint32_t dr = is_s ? drain : drain3;
      mma_commit(dr);
      mbar_wait_drain(dr, 0);
    }
  } else if (warp == 14) {
    if (lane == 0) {
      constexpr uint32_t ID_DQ = idesc_bf16(128, 128, false, true);   // dS K (K N-major)
      bool ok = true;
      for (int i = 0; i < nt && ok; ++i) {
        const int gi = i % DQ_GROUPS;
        if (!mbar_wait(ds_full(gi), (i / DQ_GROUPS) & 1, abort_flag, 23)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ks = smem_u32(sK + (i % BSTAGES) * QTILE);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem, tmem + 128 + gi * 128 + k * 8, mnmajor_desc(ks + k * 2048, QHALF),
                      ID_DQ, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(kv_empty(i % BSTAGES));
        mma_commit(dq_free(gi));
      }
      if (ok && nt > 0) mma_commit(dq_done);
      mma_commit(drain2);
      mbar_wait_drain(drain2, 0);
    }
  } else {
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t ts = tmem + 128 + g * 128 + lane_off;  // S_g, then dS_g
    const uint32_t td = tmem + 192 + g * 128 + lane_off;  // dP_g
    const bool row_ok = qi < p.S;
    const float lse2 = row_ok ? p.lse[((int64_t)b * p.H + h) * p.S + qi] * kLog2e : 0.f;
    bool ok = mbar_wait(q_full, 0, abort_flag, 25);
    // delta = sum_d dO[r, d] O[r, d] (= sum_j P_rj dA_rj of gqa_backward),
    // columns in order; both tiles are 128B-swizzled alike (16-byte chunk c
    // of row r at chunk c ^ (r & 7)), so the lanes of a phase read distinct
    // banks.
    float dlt = 0.f;
    if (ok) {
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t off = (c >> 3) * HALF + r * 128 + (((c & 7) ^ (r & 7)) << 4);
        const uint4 ov = *reinterpret_cast<const uint4*>(sO + off);
        const uint4 gv = *reinterpret_cast<const uint4*>(sDO + off);
        const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
        const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 x = __bfloat1622float2(o2[u]), y = __bfloat1622float2(g2[u]);
          dlt += x.x * y.x;
          dlt += x.y * y.y;
        }
      }
      if (g == 0 && row_ok) p.delta_out[((int64_t)b * p.H + h) * p.S + qi] = dlt;
    }
    // P = 2^(s sl2 - lse2), dS = P (dP scale - delta scale), as paired FMAs
    const float2 sl2v = make_float2(p.sl2, p.sl2), scv = make_float2(p.scale, p.scale);
    const float2 nl2 = make_float2(-lse2, -lse2);
    const float2 nd2 = make_float2(-dlt * p.scale, -dlt * p.scale);
    int cnt = 0;
    for (int j = g; j < nt && ok; j += DQ_GROUPS, ++cnt) {
      if (!mbar_wait(sd_full(g), cnt & 1, abort_flag, 26)) { ok = false; break; }
      tc_fence_after();
      const int k0 = (lo + j) * QB;
      // every (query, key) pair of the 128 x 64 tile is visible: no masks
      const bool full = (k0 + QB - 1 <= q0) && (q0 + AT - 1 - k0 < p.window) && (q0 + AT <= p.S);
      uint32_t pk[32];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float sv[32], dp[32];
        tmem_ld32x2(ts + hh * 32, td + hh * 32, sv, dp);
        if (!full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = k0 + hh * 32 + i;
            if (!(row_ok && key <= qi && qi - key < p.window)) sv[i] = -INFINITY;
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(sv[2 * i], sv[2 * i + 1]), sl2v, nl2);
          const float2 pr = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          const float2 d = ffma2(make_float2(dp[2 * i], dp[2 * i + 1]), scv, nd2);
          const float2 ds = fmul2(pr, d);
          pk[hh * 16 + i] = pack_bf16(ds.x, ds.y);
        }
      }
      tmem_st32u(ts, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full(g));
    }
    const bool done = g == 0 && ok && mbar_wait(dq_done, 0, abort_flag, 28);
    if (done) tc_fence_after();
    if (done && p.o16.dq) {
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float a[32], bb[32];
        tmem_ld32x2(tmem + lane_off + c * 32, tmem + lane_off + (c + 2) * 32, a, bb);
        if (row_ok)
          store_grad_bf16(p.o16.dq + ((int64_t)(row0 + qi) * p.H + h) * HD, c * 32, a, bb,
                          p.o16.cs, p.o16.sn, qi);
      }
    } else if (done) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_off + c * 32, v);
        if (row_ok) {
          float4* dst = reinterpret_cast<float4*>(p.dq + ((int64_t)(row0 + qi) * p.H + h) * HD + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

constexpr size_t kDqSmem = 3 * TILE + 2 * BSTAGES * QTILE + 1024 + 256;
static_assert(kDqSmem <= 232448, "dQ kernel shared memory above the per-CTA limit");

// dK, dV: one CTA per (128-key tile, kv head, sequence), looping over the
// query heads of the group and the 64-query tiles that see the keys (tile i
// to group i & 1).  TMEM: dV 0-127, dK 128-255; group g: S^T_g 256+128g
// (P^T packed in its first 32 columns), dP^T_g 320+128g (dS^T packed).
// S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q.
constexpr int DKDV_THREADS = 384;  // TMA, S^T issuer, 2 x 4 elementwise, accumulate issuer, dP^T issuer
__global__ void __launch_bounds__(DKDV_THREADS, 1)
    k_attn_dkdv_tc(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                   const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                   const BwdParams p) {
  if (tc_failed()) return;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sK = smem;
  uint8_t* sV = smem + TILE;
  uint8_t* sQ = smem + 2 * TILE;                // BSTAGES x [64 q][128 d]
  uint8_t* sDO = sQ + BSTAGES * QTILE;
  float* sLD = (float*)(sDO + BSTAGES * QTILE); // [8 warps][-lse2 64 | -delta scale 64]
  uint64_t* bars = (uint64_t*)(sLD + 8 * 128);
  uint32_t* tmem_slot = (uint32_t*)(bars + 16);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  const uint32_t b0 = smem_u32(bars);
  const uint32_t kv_full = b0, acc_done = b0 + 8, drain = b0 + 16;
  auto q_full = [&](int st) { return b0 + 24 + 8u * st; };
  auto q_empty = [&](int st) { return b0 + 56 + 8u * st; };
  auto sd_full = [&](int g) { return b0 + 88 + 8u * g; };
  auto pd_full = [&](int g) { return b0 + 104 + 8u * g; };
  // group g's P^T / dS^T columns have been read by the accumulating MMAs
  auto acc_free = [&](int g) { return b0 + 136 + 8u * g; };
  const uint32_t drain2 = b0 + 152, drain3 = b0 + 160;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = (int)blockIdx.x;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int k0 = kt * AT;
  const int qhi = min(p.S - 1, k0 + AT - 1 + p.window - 1);
  const int qt0 = k0 / QB, nq = qhi / QB - qt0 + 1;
  const int total = nq * p.group;  // (head, query tile) pairs, head-major
  const int row0 = b * p.S;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    for (int st = 0; st < BSTAGES; ++st) {
      mbar_init(q_full(st), 1);
      mbar_init(q_empty(st), 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(sd_full(g), 2);  // the S^T and the dP^T issuer
      mbar_init(pd_full(g), 4);
      mbar_init(acc_free(g), 1);
    }
    mbar_init(drain2, 1);
    mbar_init(drain3, 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t ks = smem_u32(sK), vs = smem_u32(sV);
      mbar_expect_tx(kv_full, 2 * TILE);
      tma_load_3d(ks, &mk, kv_full, 0, kvh, row0 + k0);
      tma_load_3d(ks + HALF, &mk, kv_full, 64, kvh, row0 + k0);
      tma_load_3d(vs, &mv, kv_full, 0, kvh, row0 + k0);
      tma_load_3d(vs + HALF, &mv, kv_full, 64, kvh, row0 + k0);
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < total; ++i) {
        const int st = i % BSTAGES;
        const int h = kvh * p.group + i / nq;
        const int qq0 = (qt0 + i % nq) * QB;
        if (!mbar_wait(q_empty(st), ((i / BSTAGES) & 1) ^ 1, abort_flag, 31)) { ok = false; break; }
        const uint32_t qs = smem_u32(sQ + st * QTILE), dos = smem_u32(sDO + st * QTILE);
        mbar_expect_tx(q_full(st), 2 * QTILE);
        tma_load_3d(qs, &mq, q_full(st), 0, h, row0 + qq0);
        tma_load_3d(qs + QHALF, &mq, q_full(st), 64, h, row0 + qq0);
        tma_load_3d(dos, &mdo, q_full(st), 0, h, row0 + qq0);
        tma_load_3d(dos + QHALF, &mdo, q_full(st), 64, h, row0 + qq0);
        ++issued;
      }
      if (!ok) {
        mbar_wait_drain(kv_full, 0);
        for (int i = issued - 1; i >= 0 && i >= issued - BSTAGES; --i)
          mbar_wait_drain(q_full(i % BSTAGES), (i / BSTAGES) & 1);
      }
    }
  } else if (warp == 1 || warp == 11) {
    // S^T (warp 1) and dP^T (warp 11) are issued by two threads and the
    // accumulating MMAs (dV += P^T dO, dK += dS^T Q) by warp 10, so that
    // three instruction streams are issued in parallel; S^T and dP^T of
    // pair i wait until the accumulating MMAs of pair i - 2 (same group
    // columns) have run.
    if (lane == 0) {
      constexpr uint32_t ID_ST = idesc_bf16(128, 64, false, false);   // K Q^T, V dO^T
      const bool is_s = warp == 1;
      const uint32_t as = smem_u32(is_s ? sK : sV);
      uint8_t* const bstage = is_s ? sQ : sDO;
      const uint32_t dcol = is_s ? 256u : 320u;
      bool ok = mbar_wait(kv_full, 0, abort_flag, 32);
      for (int i = 0; i < total && ok; ++i) {
        const int g = i & 1, st = i % BSTAGES;
        if (!mbar_wait(q_full(st), (i / BSTAGES) & 1, abort_flag, 34)) { ok = false; break; }
        if (i >= 2 && !mbar_wait(acc_free(g), ((i - 2) >> 1) & 1, abort_flag, 35)) { ok = false; break; }
        tc_fence_after();
        const uint32_t bs = smem_u32(bstage + st * QTILE);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ka = (k >> 2) * HALF + (k & 3) * 32;   // K/V: two 16 KB d-boxes
          const uint32_t kb = (k >> 2) * QHALF + (k & 3) * 32;  // Q/dO: two 8 KB d-boxes
          mma_bf16(tmem + dcol + g * 128, kmajor_desc(as + ka), kmajor_desc(bs + kb), ID_ST, k > 0);
        }
        mma_commit(sd_full(g));
      }
      const uint32_t dr = is_s ? drain : drain3;
      mma_commit(dr);
      mbar_wait_drain(dr, 0);
    }
  } else if (warp == 10) {
    if (lane == 0) {
      constexpr uint32_t ID_ACC = idesc_bf16(128, 128, false, true);  // P^T dO, dS^T Q
      bool ok = true;
      int i = 0;
      for (; i < total && ok; ++i) {
        const int gi = i & 1, st = i % BSTAGES;
        if (!mbar_wait(pd_full(gi), (i >> 1) & 1, abort_flag, 33)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qs = smem_u32(sQ + st * QTILE), dos = smem_u32(sDO + st * QTILE);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          mma_bf16_ts(tmem, tmem + 256 + gi * 128 + k * 8, mnmajor_desc(dos + k * 2048, QHALF),
                      ID_ACC, acc);
          mma_bf16_ts(tmem + 128, tmem + 320 + gi * 128 + k * 8, mnmajor_desc(qs + k * 2048, QHALF),
                      ID_ACC, acc);
        }
        mma_commit(q_empty(st));
        mma_commit(acc_free(gi));
      }
      if (ok && total > 0) mma_commit(acc_done);
      mma_commit(drain2);
      mbar_wait_drain(drain2, 0);
    }
  } else {
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;   // key row of this thread
    const int kj = k0 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tsv = tmem + 256 + g * 128 + lane_off;  // S^T_g, then P^T_g
    const uint32_t tdp = tmem + 320 + g * 128 + lane_off;  // dP^T_g, then dS^T_g
    float* ld = sLD + (warp - 2) * 128;                    // this warp's -lse2 | -delta scale
    const bool key_ok = kj < p.S;
    const float2 sl2v = make_float2(p.sl2, p.sl2), scv = make_float2(p.scale, p.scale);
    bool ok = true;
    int cnt = 0;
    // -lse2 and -delta scale of the 64 queries of pair i (lane: queries lane
    // and lane + 32), fetched one group tile ahead so that the global load
    // latency overlaps the previous tile's work
    float nl_pre[2], nd_pre[2];
    auto fetch = [&](int i) {
      const int hf = kvh * p.group + i / nq;
      const int qf = (qt0 + i % nq) * QB;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int qi = qf + lane + 32 * u;
        const bool in = qi < p.S;
        const int64_t at = ((int64_t)b * p.H + hf) * p.S + qi;
        nl_pre[u] = in ? -p.lse[at] * kLog2e : 0.f;
        nd_pre[u] = in ? -p.delta[at] * p.scale : 0.f;
      }
    };
    if (g < total) fetch(g);
    for (int i = g; i < total; i += 2, ++cnt) {
      const int qq0 = (qt0 + i % nq) * QB;
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        ld[lane + 32 * u] = nl_pre[u];       // -lse2
        ld[QB + lane + 32 * u] = nd_pre[u];  // -delta scale
      }
      __syncwarp();
      if (i + 2 < total) fetch(i + 2);
      if (!mbar_wait(sd_full(g), cnt & 1, abort_flag, 36)) { ok = false; break; }
      tc_fence_after();
      // every (key, query) pair of the 128 x 64 tile is visible: no masks
      const bool full = (k0 + AT <= p.S) && (qq0 + QB <= p.S) && (k0 + AT - 1 <= qq0) &&
                        (qq0 + QB - 1 - k0 < p.window);
      // two halves of 32 queries: read S^T / dP^T columns 32*hh.. and write
      // the packed P^T / dS^T to columns 16*hh.. (already-read columns)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float sv[32], dp[32];
        tmem_ld32x2(tsv + hh * 32, tdp + hh * 32, sv, dp);
        if (!full) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int qi = qq0 + hh * 32 + e;
            if (!(key_ok && qi < p.S && kj <= qi && qi - kj < p.window)) sv[e] = -INFINITY;
          }
        }
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int e4 = 0; e4 < 8; ++e4) {
          const int c = hh * 32 + 4 * e4;
          const float4 nl = *reinterpret_cast<const float4*>(ld + c);
          const float4 nd = *reinterpret_cast<const float4*>(ld + QB + c);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int e = 2 * e4 + u;
            const float2 nlu = u ? make_float2(nl.z, nl.w) : make_float2(nl.x, nl.y);
            const float2 ndu = u ? make_float2(nd.z, nd.w) : make_float2(nd.x, nd.y);
            const float2 x = ffma2(make_float2(sv[2 * e], sv[2 * e + 1]), sl2v, nlu);
            const float2 pr = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            const float2 d = ffma2(make_float2(dp[2 * e], dp[2 * e + 1]), scv, ndu);
            const float2 ds = fmul2(pr, d);
            pp[e] = pack_bf16(pr.x, pr.y);
            pd[e] = pack_bf16(ds.x, ds.y);
          }
        }
        tmem_st16u(tsv + hh * 16, pp);
        tmem_st16u(tdp + hh * 16, pd);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pd_full(g));
    }
    const bool done = g == 0 && ok && mbar_wait(acc_done, 0, abort_flag, 38);
    if (done) tc_fence_after();
    if (done && p.o16.dq) {
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float a[32], bb[32];
        const int64_t base = ((int64_t)(row0 + kj) * p.KV + kvh) * HD;
        tmem_ld32x2(tmem + lane_off + c * 32, tmem + lane_off + (c + 2) * 32, a, bb);
        if (key_ok) store_grad_bf16(p.o16.dv + base, c * 32, a, bb, nullptr, nullptr, kj);
        tmem_ld32x2(tmem + 128 + lane_off + c * 32, tmem + 128 + lane_off + (c + 2) * 32, a, bb);
        if (key_ok) store_grad_bf16(p.o16.dk + base, c * 32, a, bb, p.o16.cs, p.o16.sn, kj);
      }
    } else if (done) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32], k[32];
        tmem_ld32(tmem + lane_off + c * 32, v);
        tmem_ld32(tmem + 128 + lane_off + c * 32, k);
        if (key_ok) {
          const int64_t base = ((int64_t)(row0 + kj) * p.KV + kvh) * HD + c * 32;
          float4* dv4 = reinterpret_cast<float4*>(p.dv + base);
          float4* dk4 = reinterpret_cast<float4*>(p.dk + base);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            dv4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            dk4[q] = make_float4(k[4 * q], k[4 * q + 1], k[4 * q + 2], k[4 * q + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

constexpr size_t kDkdvSmem = 2 * TILE + 2 * BSTAGES * QTILE + 8 * 128 * 4 + 1024 + 256;


// y = exp2_poly2(x) elementwise: the softmax's FMA-pipe exponential, for
// checking its error bound against exp2.
__global__ void k_exp2_poly(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  for (int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x); i < n;
       i += 2 * (int64_t)gridDim.x * blockDim.x) {
    const float2 r = exp2_poly2(make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f));
    y[i] = r.x;
    if (i + 1 < n) y[i + 1] = r.y;
  }
}

void exp2_poly(const float* x, float* y, int64_t n, cudaStream_t s, int64_t& launches) {
  if (n <= 0) return;
  const int grid = (int)std::min<int64_t>(ceil_div(ceil_div(n, 2), 256), 1024);
  k_exp2_poly<<<grid, 256, 0, s>>>(x, y, n);
  DOP_LAUNCHED(launches);
}

}  // namespace tc

static void check_tc(const Attn& a) {
  DOP_REQUIRE(a.hd == 128, "the tensor-core attention needs head_dim 128");
  DOP_REQUIRE(a.causal && a.window >= 1, "the tensor-core attention is causal");
  DOP_REQUIRE(a.H % a.KV == 0, "heads must be a multiple of kv_heads");
  DOP_REQUIRE(a.B * a.S < (int64_t)1 << 31, "too many tokens");
}

void attn_fwd_tc(const Attn& a, const bf16* q, const bf16* k, const bf16* v, bf16* o, float* lse,
                 cudaStream_t s, int64_t& launches) {
  using namespace tc;
  check_tc(a);
  bind_error_word();
  const int64_t T = a.B * a.S;
  const int64_t dq[3] = {HD, a.H, T}, sq[2] = {HD, (int64_t)a.H * HD};
  const int64_t dk[3] = {HD, a.KV, T}, sk[2] = {HD, (int64_t)a.KV * HD};
  const int box[3] = {64, 1, AT};
  CUtensorMap mq = make_map3(q, dq, sq, box), mk = make_map3(k, dk, sk, box),
              mv = make_map3(v, dk, sk, box);
  FwdParams p;
  p.S = (int)a.S; p.H = a.H; p.KV = a.KV; p.group = a.H / a.KV;
  p.window = (int)std::min<int64_t>(a.window, a.S + 1);
  p.n_qt = (int)ceil_div(a.S, 2 * AT);  // pairs of query tiles
  p.sl2 = a.scale * kLog2e;
  p.o = o;
  p.lse = lse;
  static bool attr = false;
  if (!attr) {
    DOP_CHECK_CUDA(cudaFuncSetAttribute(k_attn_fwd_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kFwdSmem));
    attr = true;
  }
  dim3 grid((unsigned)p.n_qt, (unsigned)a.H, (unsigned)a.B);
  k_attn_fwd_tc<<<grid, 320, kFwdSmem, s>>>(mq, mk, mv, p);
  DOP_LAUNCHED(launches);
}

void attn_bwd_tc(const Attn& a, const bf16* q, const bf16* k, const bf16* v, const bf16* o,
                 const bf16* dout, const float* lse, float* delta, float* dq, float* dk, float* dv,
                 cudaStream_t s, int64_t& launches, const AttnBwdBf16* out16) {
  using namespace tc;
  check_tc(a);
  bind_error_word();
  const int64_t T = a.B * a.S;
  const int64_t dq_[3] = {HD, a.H, T}, sq[2] = {HD, (int64_t)a.H * HD};
  const int64_t dk_[3] = {HD, a.KV, T}, sk[2] = {HD, (int64_t)a.KV * HD};
  const int box128[3] = {64, 1, AT}, box64[3] = {64, 1, QB};
  BwdParams p;
  p.S = (int)a.S; p.H = a.H; p.KV = a.KV; p.group = a.H / a.KV;
  p.window = (int)std::min<int64_t>(a.window, a.S + 1);
  p.sl2 = a.scale * kLog2e;
  p.scale = a.scale;
  p.lse = lse; p.delta = delta; p.delta_out = delta; p.dq = dq; p.dk = dk; p.dv = dv;
  if (out16) {
    DOP_REQUIRE(out16->dq && out16->dk && out16->dv, "bf16 gradient outputs need dq, dk and dv");
    DOP_REQUIRE(!out16->cs || out16->sn, "RoPE adjoint needs both tables");
    p.o16 = *out16;
  } else {
    DOP_REQUIRE(dq && dk && dv, "null gradient output");
  }
  {
    CUtensorMap mq = make_map3(q, dq_, sq, box128), mdo = make_map3(dout, dq_, sq, box128);
    CUtensorMap mo = make_map3(o, dq_, sq, box128);
    CUtensorMap mk = make_map3(k, dk_, sk, box64), mv = make_map3(v, dk_, sk, box64);
    p.n_tiles = (int)ceil_div(a.S, AT);
    static bool attr = false;
    if (!attr) {
      DOP_CHECK_CUDA(cudaFuncSetAttribute(k_attn_dq_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kDqSmem));
      attr = true;
    }
    dim3 grid((unsigned)p.n_tiles, (unsigned)a.H, (unsigned)a.B);
    k_attn_dq_tc<<<grid, DQ_THREADS, kDqSmem, s>>>(mq, mk, mv, mdo, mo, p);
    DOP_LAUNCHED(launches);
  }
  {
    CUtensorMap mq = make_map3(q, dq_, sq, box64), mdo = make_map3(dout, dq_, sq, box64);
    CUtensorMap mk = make_map3(k, dk_, sk, box128), mv = make_map3(v, dk_, sk, box128);
    p.n_tiles = (int)ceil_div(a.S, AT);
    static bool attr = false;
    if (!attr) {
      DOP_CHECK_CUDA(cudaFuncSetAttribute(k_attn_dkdv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)kDkdvSmem));
      attr = true;
    }
    dim3 grid((unsigned)p.n_tiles, (unsigned)a.KV, (unsigned)a.B);
    k_attn_dkdv_tc<<<grid, DKDV_THREADS, kDkdvSmem, s>>>(mq, mk, mv, mdo, p);
    DOP_LAUNCHED(launches);
  }
}



}  // namespace dop
