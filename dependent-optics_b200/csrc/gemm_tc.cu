// gemm_tc.cu — bf16 x bf16 -> fp32 GEMM on the 5th-generation tensor cores.
//
// One persistent, warp-specialised kernel serves every contraction of the
// bf16 block lens (dense Q/K/V/O projections and their gradients, the expert
// SwiGLU projections grouped over expert-sorted row segments, and their
// weight / input gradients):
//
//   warp 0        TMA producer: 128B-swizzled tiles of A and B into a
//                 STAGES-deep shared-memory ring (cp.async.bulk.tensor)
//   warp 1        allocates 512 TMEM columns; one thread issues
//                 tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit
//   warps 2..9    epilogue: tcgen05.ld of the fp32 accumulator (two warps
//                 per 32-lane TMEM quadrant, each owning half the columns),
//                 fused epilogue math, global stores
//
// The accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of tile i overlaps the main loop of tile i+1.  Either operand may be
// K-major or M/N-major (the instruction descriptor's transpose bits), which
// covers Y = X W, dX = dY W^T and dW = X^T dY on the crate's [din, dout]
// weights without a transpose.  Outputs that a tile writes once (everything
// but the accumulated weight gradients) are stored with the streaming
// (evict-first) hint, so the output stream does not push the operand tiles
// that later tiles re-read out of L2.  Every mbarrier wait is bounded; a wait that
// runs out records an error code, stops the tile loop and drains what is in
// flight before TMEM is freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <type_traits>

#include "kernels.cuh"

#include "tc_ptx.cuh"

namespace dop {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int STAGES = 4;       // one CTA per tile: 48 KB stages
// A pair of CTAs per tile: 32 KB stages per CTA, seven of them (224 KB plus
// the barriers and ~1 KB of static shared memory, inside the 227 KB a CTA
// may hold).  Measured against six: the 16384 x 14336 x 4096 GEMM 1.318 ->
// 1.295 ms, the Mixtral-8x7B block step 75.3-76.0 -> 74.4-74.8 ms.
constexpr int PAIR_STAGES = 7;
constexpr int THREADS = 320;  // TMA warp, MMA warp, 8 epilogue warps

enum EpiKind : int {
  kStoreF32 = 0,
  kStoreBF16 = 1,
  kAccumF32 = 2,
  kAddResF32 = 3,
  kSwiGLU = 4,     // dual-B forward: cols [0,BN/2) = gate, [BN/2,BN) = up -> g, u, h
  kSwiGLUBwd = 5,  // acc = dH; with g, u in global -> dG, dU
  kRopeBF16 = 6,   // bf16 store of 128-wide heads rotated by RoPE (rotate_half)
};

struct Params {
  int M, N;         // output extent (rows, cols); grouped-K: per expert
  int mode;         // 0 plain, 1 grouped rows (expert segments), 2 grouped contraction
  int nparts;       // K segments (A_i, B_i) summed into one accumulator
  int kb[3];        // k-blocks of each part (plain / grouped rows)
  const int* seg_off;
  const int* seg_end;  // grouped contraction: group g runs over [seg_off[g], seg_end[g])
                       // (null: [seg_off[g], seg_off[g + 1])); empty groups are skipped
  const int* tile_expert;
  int G;
  int m_tiles, n_tiles;  // n_tiles counts BN-wide (dual: BN/2-wide output) tiles
  int gm;               // row tiles walked before the next column tile
  int* tile_ctr;         // non-null: tiles are taken in order from this counter (zeroed
                         // before the launch); null: CTA (pair) u takes u, u + units, ...
  int epi;
  void* C;
  int64_t ldc, c_gs;
  const float* R;
  int64_t ldr;
  bf16 *g_out, *u_out, *h_out;   // SwiGLU forward outputs [rows, ldg]
  const bf16 *g_in, *u_in;       // SwiGLU backward inputs
  bf16 *dg_out, *du_out;
  int64_t ldg;
  const float *rope_cos, *rope_sin;  // [seq][64] tables of kRopeBF16
  int rope_seq;
  // mode 2 with kchunk > 0: split contraction of a plain product, group g
  // contracting over [g kchunk, min(ktot, (g + 1) kchunk)) into C + g c_gs
  int kchunk, ktot;
};

// Tile id -> (group, m tile, n tile).  Consecutive ids walk GM row tiles
// before moving to the next column tile, so a wave of CTAs shares A and B
// tiles in L2.
struct Tile { int g, m, n; };
__device__ __forceinline__ Tile tile_of(int t, int m_tiles, int n_tiles, int GM) {
  Tile r;
  const int per_g = m_tiles * n_tiles;
  r.g = t / per_g;
  t -= r.g * per_g;
  const int band = t / (GM * n_tiles);
  const int rows = min(GM, m_tiles - band * GM);
  const int in = t - band * GM * n_tiles;
  r.m = band * GM + in % rows;
  r.n = in / rows;
  return r;
}

// PAIR: a cluster of two CTAs on two SMs computes one 256-row tile with
// cta_group::2 MMAs (M = 256): each CTA loads its 128 rows of A and half of
// B's columns (for the SwiGLU pass: CTA 0 the gate tile, CTA 1 the up tile),
// CTA 0's MMA thread issues for both, and each CTA's epilogue drains the 128
// accumulator rows in its own TMEM.  Per FLOP this reads a third less
// operand data from L2 and shared memory than one CTA per 128-row tile.
// TF: tf32 operands (fp32 bit patterns, 32 per 128-byte K-major row, both
// operands K-major): the 3xTF32 products of the fp32 lens (gemm_tc_f32).
template <bool A_MN, bool B_MN, int BN, bool DUAL, bool PAIR, bool TF = false>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
              const __grid_constant__ CUtensorMap mA2, const __grid_constant__ CUtensorMap mB0,
              const __grid_constant__ CUtensorMap mB1, const __grid_constant__ CUtensorMap mB2,
              const Params p) {
  constexpr int STG = PAIR ? PAIR_STAGES : STAGES;
  constexpr int BNL = PAIR ? BN / 2 : BN;  // B columns this CTA loads
  constexpr int TM = PAIR ? 2 * BM : BM;   // rows of a tile
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BNL * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static_assert(!TF || (!A_MN && !B_MN && !DUAL), "tf32 operands are K-major, no SwiGLU");
  constexpr int BKE = TF ? 32 : BK;             // elements of a 128-byte k-block row
  constexpr uint32_t FMT = TF ? 2u : 1u;        // operand format: BF16 1, TF32 2
  constexpr uint32_t IDESC = (1u << 4) | (FMT << 7) | (FMT << 10) | ((A_MN ? 1u : 0u) << 15) |
                             ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(TM >> 4) << 24);
  // An earlier wait failed (sticky error): do no work.  A CTA of a pair
  // still takes part in the pair's cluster barriers below.
  const bool failed = tc_failed();
  if (!PAIR && failed) return;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;   // tile walker
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + STG * STAGE_BYTES);
  // bars: full[STG], empty[STG], acc_full[2], acc_empty[2], drain
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STG + 5);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
  // grouped contraction: the groups with a non-empty contraction, in order
  __shared__ int s_groups[kMaxExperts];
  __shared__ int s_ngroups;
  // Dynamic tile order (p.tile_ctr): the first CTA's producer takes the next
  // tile id from the counter and publishes it in a ring in both CTAs' shared
  // memory (tid_full); every role reads the ids in ring order and releases
  // the slot on the first CTA's tid_empty.  Tiles in flight therefore stay
  // consecutive in tile order however the CTAs drift, so tiles that share
  // an operand run close together and share it in L2.
  constexpr int TR = 4;
  __shared__ int s_tid[TR];
  __shared__ __align__(8) uint64_t s_tbar[2 * TR];
  const bool dyn = p.tile_ctr != nullptr;
  const uint32_t smem0 = smem_u32(smem);
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STG + s); };
  auto accf_bar = [&](int a) { return bar0 + 8u * (2 * STG + a); };
  auto acce_bar = [&](int a) { return bar0 + 8u * (2 * STG + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STG + 4);
  auto tid_full = [&](int r) { return smem_u32(&s_tbar[r]); };
  auto tid_empty = [&](int r) { return smem_u32(&s_tbar[TR + r]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      // every epilogue warp of the tile (both CTAs of a pair) frees it
      mbar_init(acce_bar(a), PAIR ? 16 : 8);
    }
    mbar_init(drain_bar, 1);
    for (int r = 0; r < TR; ++r) {
      mbar_init(tid_full(r), 1);
      // readers of a slot: the MMA thread and 8 epilogue warps of the first
      // CTA, the producer and 8 epilogue warps of the second
      mbar_init(tid_empty(r), PAIR ? 18 : 9);
    }
    *abort_flag = failed ? 1 : 0;
    int ng = 0;
    if (p.mode == 2) {
      for (int g = 0; g < p.G && g < kMaxExperts; ++g) {
        const int lo = p.kchunk ? g * p.kchunk : p.seg_off[g];
        const int hi = p.kchunk ? min(p.ktot, lo + p.kchunk)
                                : (p.seg_end ? p.seg_end[g] : p.seg_off[g + 1]);
        if (hi > lo) s_groups[ng++] = g;
      }
    }
    s_ngroups = ng;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(512));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs' barriers exist before either is signalled
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // work description shared by all roles
  int rows_total = p.M;
  if (p.mode == 1) rows_total = p.seg_off[p.G];
  const int m_tiles = p.mode == 1 ? (rows_total + TM - 1) / TM : p.m_tiles;
  const int groups = p.mode == 2 ? s_ngroups : 1;
  const int total = groups * m_tiles * p.n_tiles;
  // tile id -> tile, with the group index of a grouped contraction mapped
  // to the non-empty groups
  auto tile_at = [&](int t) {
    Tile r = tile_of(t, m_tiles, p.n_tiles, p.gm);
    if (p.mode == 2) r.g = s_groups[r.g];
    return r;
  };
  // Next tile id of a reader of the ring (dynamic order) or of the static
  // walk: >= 0 a tile, -1 no more tiles, -2 a bounded wait ran out.  A
  // whole warp (warp_wide: every lane reads, lane 0 releases the slot) or a
  // single thread (the producer of the second CTA, the MMA thread) reads.
  auto next_tile = [&](int& it, int& rs, uint32_t& rph, int code, bool warp_wide) -> int {
    if (!dyn) {
      const int t = unit + (it++) * units;
      return t < total ? t : -1;
    }
    const bool got = leader ? mbar_wait(tid_full(rs), rph, abort_flag, code)
                            : mbar_wait_cluster(tid_full(rs), rph, abort_flag, code);
    if (warp_wide) {
      // the same answer on every lane: the slot is released once
      if (!__all_sync(0xffffffffu, got)) return -2;
    } else if (!got) {
      return -2;
    }
    const int t = *(volatile int*)&s_tid[rs];
    if (warp_wide) __syncwarp();
    if (!warp_wide || (threadIdx.x & 31) == 0) {
      if (leader) mbar_arrive(tid_empty(rs));
      else mbar_arrive_cluster(mapa_shared(tid_empty(rs), 0));
    }
    if (++rs == TR) { rs = 0; rph ^= 1u; }
    return t;
  };
  // The first CTA's producer: take the next id and publish it to both CTAs.
  auto take_tile = [&](int& rs, uint32_t& rph) -> int {
    if (!mbar_wait(tid_empty(rs), rph ^ 1u, abort_flag, 5)) return -2;
    int t = atomicAdd(p.tile_ctr, 1);
    if (t >= total) t = -1;
    s_tid[rs] = t;
    if (PAIR) {
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(smem_u32(&s_tid[rs]), 1)),
                   "r"(t)
                   : "memory");
      mbar_arrive_cluster(mapa_shared(tid_full(rs), 1));
    }
    mbar_arrive(tid_full(rs));
    if (++rs == TR) { rs = 0; rph ^= 1u; }
    return t;
  };
  auto k_blocks = [&](const Tile& t, int part, int& k0) -> int {
    if (p.mode == 2 && p.kchunk) {
      k0 = t.g * p.kchunk;
      return (min(p.ktot, k0 + p.kchunk) - k0 + BKE - 1) / BKE;
    }
    if (p.mode == 2) {
      k0 = p.seg_off[t.g];
      return ((p.seg_end ? p.seg_end[t.g] : p.seg_off[t.g + 1]) - k0) / BKE;
    }
    k0 = 0;
    return p.kb[part];
  };

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_map(&mA0);
      prefetch_map(&mB0);
      int s = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = !*abort_flag;
      // a pair counts both CTAs' bytes on the first CTA's full barriers
      auto fullb = [&](int st) { return PAIR ? mapa_shared(full_bar(st), 0) : full_bar(st); };
      auto load = [&](uint32_t dst, const CUtensorMap* map, int st, int c0, int c1, int c2) {
        if (PAIR) tma_load_3d_pair(dst, map, fullb(st), c0, c1, c2);
        else tma_load_3d(dst, map, full_bar(st), c0, c1, c2);
      };
      int it = 0, rs = 0;
      uint32_t rph = 0;
      while (ok) {
        const int t = (dyn && leader) ? take_tile(rs, rph) : next_tile(it, rs, rph, 6, false);
        if (t == -2) ok = false;
        if (t < 0 || !ok) break;
        const Tile tl = tile_at(t);
        const int m0 = tl.m * TM + (int)rank * BM;  // this CTA's rows
        // expert of the tile (segments are kSegAlign-aligned: one expert per tile)
        const int z = p.mode == 1 ? max(p.tile_expert[tl.m * (TM / BM)], 0) : 0;
        for (int part = 0; part < p.nparts && ok; ++part) {
          const CUtensorMap* ma = part == 0 ? &mA0 : (part == 1 ? &mA1 : &mA2);
          const CUtensorMap* mb = part == 0 ? &mB0 : (part == 1 ? &mB1 : &mB2);
          int kbase;
          const int nk = k_blocks(tl, part, kbase);
          for (int kb = 0; kb < nk; ++kb) {
            if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, 1)) { ok = false; break; }
            const uint32_t sa = smem0 + s * STAGE_BYTES, sb = sa + A_BYTES;
            if (leader) mbar_expect_tx(full_bar(s), PAIR ? 2 * STAGE_BYTES : STAGE_BYTES);
            const int k0 = kbase + kb * BKE;
            if (!A_MN) {
              load(sa, ma, s, k0, m0, 0);
            } else {
              load(sa, ma, s, m0, k0, 0);
              load(sa + A_BYTES / 2, ma, s, m0 + 64, k0, 0);
            }
            if (!DUAL) {
              const int n0 = tl.n * BN + (int)rank * BNL;  // this CTA's columns
              if (!B_MN) {
                load(sb, mb, s, k0, n0, z);
              } else {
#pragma unroll
                for (int j = 0; j < BNL / 64; ++j) load(sb + j * 8192, mb, s, n0 + 64 * j, k0, z);
              }
            } else if (PAIR) {
              // B = [gate tile | up tile]: the first CTA loads the gate
              // columns, the second the up columns
              const int n0 = tl.n * (BN / 2);
              const CUtensorMap* mgu = rank == 0 ? &mB0 : &mB1;
              if (!B_MN) {
                load(sb, mgu, s, k0, n0, z);
              } else {
#pragma unroll
                for (int j = 0; j < BNL / 64; ++j) load(sb + j * 8192, mgu, s, n0 + 64 * j, k0, z);
              }
            } else {
              // B = [gate tile | up tile], each BN/2 columns of the output
              const int n0 = tl.n * (BN / 2);
              const CUtensorMap* mg = &mB0;
              const CUtensorMap* mu = &mB1;
              if (!B_MN) {
                load(sb, mg, s, k0, n0, z);
                load(sb + B_BYTES / 2, mu, s, k0, n0, z);
              } else {
#pragma unroll
                for (int j = 0; j < BN / 128; ++j) {
                  load(sb + j * 8192, mg, s, n0 + 64 * j, k0, z);
                  load(sb + B_BYTES / 2 + j * 8192, mu, s, n0 + 64 * j, k0, z);
                }
              }
            }
            ++issued;
            if (++s == STG) { s = 0; ph ^= 1u; }
          }
        }
        if (!ok) break;
      }
      if (!ok && leader) {
        // drain: wait (bounded) for the copies of the stages still in flight
        // (a pair's copies all complete on the first CTA's barriers)
        for (int q = 0; q < STG && q < issued; ++q) {
          if (--s < 0) { s = STG - 1; ph ^= 1u; }
          mbar_wait_drain(full_bar(s), ph);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // (a pair's second CTA issues nothing: its tensor core is driven by the
    // first CTA's cta_group::2 MMAs)
    if (lane == 0 && leader) {
      int s = 0, a = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = !*abort_flag;
      // arrive on a barrier in both CTAs of the pair (or this CTA alone)
      auto commit_both = [&](uint32_t bar) {
        if (PAIR) {
          mma_commit_pair(bar);
          mma_commit_pair(mapa_shared(bar, 1));
        } else {
          mma_commit(bar);
        }
      };
      int it = 0, rs = 0;
      uint32_t rph = 0;
      while (ok) {
        const int t = next_tile(it, rs, rph, 7, false);
        if (t == -2) ok = false;
        if (t < 0 || !ok) break;
        const Tile tl = tile_at(t);
        const bool freed = PAIR ? mbar_wait_cluster(acce_bar(a), aph ^ 1u, abort_flag, 2)
                                : mbar_wait(acce_bar(a), aph ^ 1u, abort_flag, 2);
        if (!freed) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(a * BN);
        uint32_t accum = 0;
        for (int part = 0; part < p.nparts && ok; ++part) {
          int kbase;
          const int nk = k_blocks(tl, part, kbase);
          for (int kb = 0; kb < nk; ++kb) {
            if (!mbar_wait(full_bar(s), ph, abort_flag, 3)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem0 + s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
            for (int ks = 0; ks < BK / 16; ++ks) {
              const uint64_t ad = A_MN ? sdesc(sa + ks * 2048, 8192, 1024)
                                       : sdesc(sa + ks * 32, 16, 1024);
              const uint64_t bd = B_MN ? sdesc(sb + ks * 2048, 8192, 1024)
                                       : sdesc(sb + ks * 32, 16, 1024);
              if (TF) {
                if (PAIR) mma_tf32_pair(d, ad, bd, IDESC, accum);
                else mma_tf32(d, ad, bd, IDESC, accum);
              } else {
                if (PAIR) mma_bf16_pair(d, ad, bd, IDESC, accum);
                else mma_bf16(d, ad, bd, IDESC, accum);
              }
              accum = 1;
            }
            commit_both(empty_bar(s));
            if (++s == STG) { s = 0; ph ^= 1u; }
          }
        }
        if (!ok) break;
        commit_both(accf_bar(a));
        if (++a == 2) { a = 0; aph ^= 1u; }
      }
      // make sure every issued MMA has finished before TMEM can be freed
      if (PAIR) mma_commit_pair(drain_bar);
      else mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // two warps per TMEM lane quadrant (warp & 3), each owning half of the
    // tile's columns
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int chalf = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    int a = 0;
    uint32_t aph = 0;
    // the first CTA's barrier that frees accumulator a (a pair frees it from both CTAs)
    auto acce_leader = [&](int ab) { return PAIR ? mapa_shared(acce_bar(ab), 0) : acce_bar(ab); };
    int it = 0, rs = 0;
    uint32_t rph = 0;
    for (;;) {
      if (*abort_flag) break;
      const int t = next_tile(it, rs, rph, 8, true);
      if (t < 0) break;
      const Tile tl = tile_at(t);
      if (!mbar_wait(accf_bar(a), aph, abort_flag, 4)) break;
      tc_fence_after();
      int kbase;
      bool empty_k = false;
      if (p.mode == 2) empty_k = k_blocks(tl, 0, kbase) == 0;
      const int64_t m = (int64_t)tl.m * TM + (int64_t)rank * BM + row_in_tile;
      const bool row_ok = m < rows_total;
      const uint32_t tbase = tmem + (uint32_t)(a * BN) + ((uint32_t)(quad * 32) << 16);
      if (p.epi == kSwiGLU) {
        const int64_t nb = (int64_t)tl.n * (BN / 2);
#pragma unroll 1
        for (int c = chalf * (BN / 128); c < (chalf + 1) * (BN / 128); ++c) {
          float g[32], u[32];
          tmem_ld32(tbase + c * 32, g);
          tmem_ld32(tbase + BN / 2 + c * 32, u);
          const int64_t n = nb + c * 32;
          if (row_ok && n < p.N) {
            uint32_t pg[16], pu[16], ph2[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              // g and u are rounded to bf16 first: h is computed from the
              // stored residual, as the backward pass will see it
              float g0 = __bfloat162float(__float2bfloat16_rn(g[2 * j]));
              float g1 = __bfloat162float(__float2bfloat16_rn(g[2 * j + 1]));
              float u0 = __bfloat162float(__float2bfloat16_rn(u[2 * j]));
              float u1 = __bfloat162float(__float2bfloat16_rn(u[2 * j + 1]));
              pg[j] = pack_bf16(g0, g1);
              pu[j] = pack_bf16(u0, u1);
              // silu(g) u with the fast exponential and division (h is
              // rounded to bf16 next; for g -> -inf the quotient is 0)
              float h0 = __fdividef(g0, 1.0f + __expf(-g0)) * u0;
              float h1 = __fdividef(g1, 1.0f + __expf(-g1)) * u1;
              ph2[j] = pack_bf16(h0, h1);
            }
            uint4* og = (uint4*)(p.g_out + m * p.ldg + n);
            uint4* ou = (uint4*)(p.u_out + m * p.ldg + n);
            uint4* oh = (uint4*)(p.h_out + m * p.ldg + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              __stcs(og + q, make_uint4(pg[4 * q], pg[4 * q + 1], pg[4 * q + 2], pg[4 * q + 3]));
              __stcs(ou + q, make_uint4(pu[4 * q], pu[4 * q + 1], pu[4 * q + 2], pu[4 * q + 3]));
              __stcs(oh + q, make_uint4(ph2[4 * q], ph2[4 * q + 1], ph2[4 * q + 2], ph2[4 * q + 3]));
            }
          }
        }
      } else if (p.epi == kRopeBF16) {
        // this warp's 128 columns are one head: column d pairs with d + 64
        const int64_t nb = (int64_t)tl.n * BN + chalf * (BN / 2);
        const int pos = (int)(m % p.rope_seq);
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float a[32], b[32];
          tmem_ld32(tbase + chalf * (BN / 2) + c * 32, a);
          tmem_ld32(tbase + chalf * (BN / 2) + (c + 2) * 32, b);
          if (!row_ok || nb >= p.N) continue;
          const float4* c4 = (const float4*)(p.rope_cos + (int64_t)pos * 64 + c * 32);
          const float4* s4 = (const float4*)(p.rope_sin + (int64_t)pos * 64 + c * 32);
          uint32_t o1[16], o2[16];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 cv = c4[q], sv = s4[q];
            const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
            float r1[4], r2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = 4 * q + e;
              r1[e] = a[i] * cc[e] - b[i] * ss[e];
              r2[e] = b[i] * cc[e] + a[i] * ss[e];
            }
            o1[2 * q] = pack_bf16(r1[0], r1[1]);
            o1[2 * q + 1] = pack_bf16(r1[2], r1[3]);
            o2[2 * q] = pack_bf16(r2[0], r2[1]);
            o2[2 * q + 1] = pack_bf16(r2[2], r2[3]);
          }
          uint4* d1 = (uint4*)((bf16*)p.C + m * p.ldc + nb + c * 32);
          uint4* d2 = (uint4*)((bf16*)p.C + m * p.ldc + nb + 64 + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __stcs(d1 + q, make_uint4(o1[4 * q], o1[4 * q + 1], o1[4 * q + 2], o1[4 * q + 3]));
            __stcs(d2 + q, make_uint4(o2[4 * q], o2[4 * q + 1], o2[4 * q + 2], o2[4 * q + 3]));
          }
        }
      } else {
        const int64_t nb = (int64_t)tl.n * BN;
        char* Cb = (char*)p.C;
        if (p.mode == 2) Cb += (int64_t)tl.g * p.c_gs * (p.epi == kStoreBF16 ? 2 : 4);
#pragma unroll 1
        for (int c = chalf * (BN / 64); c < (chalf + 1) * (BN / 64); ++c) {
          float v[32];
          // the SwiGLU adjoint's g and u: loaded before the accumulator so
          // that the two latencies overlap
          uint4 g4p[4], u4p[4];
          if (p.epi == kSwiGLUBwd && row_ok && nb + c * 32 < p.N) {
            const uint4* gi = (const uint4*)(p.g_in + m * p.ldg + nb + c * 32);
            const uint4* ui = (const uint4*)(p.u_in + m * p.ldg + nb + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              g4p[q] = gi[q];
              u4p[q] = ui[q];
            }
          }

          if (!empty_k) tmem_ld32(tbase + c * 32, v);
          else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          const int64_t n = nb + c * 32;
          if (!row_ok || n >= p.N) continue;
          const bool full = n + 32 <= p.N;
          if (p.epi == kStoreBF16) {
            bf16* out = (bf16*)Cb + m * p.ldc + n;
            if (full) {
              uint4* o4 = (uint4*)out;
#pragma unroll
              for (int q = 0; q < 4; ++q)
                __stcs(o4 + q, make_uint4(pack_bf16(v[8 * q], v[8 * q + 1]), pack_bf16(v[8 * q + 2], v[8 * q + 3]),
                                          pack_bf16(v[8 * q + 4], v[8 * q + 5]), pack_bf16(v[8 * q + 6], v[8 * q + 7])));
            } else {
              for (int j = 0; j < 32 && n + j < p.N; ++j) out[j] = __float2bfloat16_rn(v[j]);
            }
          } else if (p.epi == kSwiGLUBwd) {
            // v = dH; dG = dH * u * s (1 + g (1 - s)), dU = dH * g * s
            // (N and ldg are multiples of 32 and 8: whole 16-byte vectors)
            uint4* dgo = (uint4*)(p.dg_out + m * p.ldg + n);
            uint4* duo = (uint4*)(p.du_out + m * p.ldg + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 g4 = g4p[q], u4 = u4p[q];
              const __nv_bfloat162* g2 = (const __nv_bfloat162*)&g4;
              const __nv_bfloat162* u2 = (const __nv_bfloat162*)&u4;
              uint32_t rg[4], ru[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 z = __bfloat1622float2(g2[e]), uu = __bfloat1622float2(u2[e]);
                const float s0 = __fdividef(1.0f, 1.0f + __expf(-z.x));
                const float s1 = __fdividef(1.0f, 1.0f + __expf(-z.y));
                const float d0 = v[8 * q + 2 * e], d1 = v[8 * q + 2 * e + 1];
                rg[e] = pack_bf16(d0 * uu.x * (s0 * (1.0f + z.x * (1.0f - s0))),
                                  d1 * uu.y * (s1 * (1.0f + z.y * (1.0f - s1))));
                ru[e] = pack_bf16(d0 * (z.x * s0), d1 * (z.y * s1));
              }
              __stcs(dgo + q, make_uint4(rg[0], rg[1], rg[2], rg[3]));
              __stcs(duo + q, make_uint4(ru[0], ru[1], ru[2], ru[3]));
            }
          } else {
            float* out = (float*)Cb + m * p.ldc + n;
            if (p.epi == kAccumF32) {
              if (empty_k) continue;
              if (full) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  float4 o = ((float4*)out)[q];
                  o.x += v[4 * q]; o.y += v[4 * q + 1]; o.z += v[4 * q + 2]; o.w += v[4 * q + 3];
                  ((float4*)out)[q] = o;
                }
              } else {
                for (int j = 0; j < 32 && n + j < p.N; ++j) out[j] += v[j];
              }
            } else {
              if (p.epi == kAddResF32) {
                // the residual in 16-byte loads when the 32 columns are whole
                // and aligned
                const float* rp = p.R + m * p.ldr + n;
                if (full && ((uintptr_t)rp & 15) == 0) {
#pragma unroll
                  for (int q = 0; q < 8; ++q) {
                    const float4 r4 = ((const float4*)rp)[q];
                    v[4 * q] += r4.x;
                    v[4 * q + 1] += r4.y;
                    v[4 * q + 2] += r4.z;
                    v[4 * q + 3] += r4.w;
                  }
                } else {
                  const float* r = p.R + m * p.ldr + n;
                  for (int j = 0; j < 32; ++j)
                    if (n + j < p.N) v[j] += r[j];
                }
              }
              if (full) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  __stcs((float4*)out + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
              } else {
                for (int j = 0; j < 32 && n + j < p.N; ++j) out[j] = v[j];
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && !leader) mbar_arrive_cluster(acce_leader(a));
        else mbar_arrive(acce_bar(a));
      }
      if (++a == 2) { a = 0; aph ^= 1u; }
    }
  }
  tc_fence_before();
  __syncthreads();
  // a pair: neither CTA frees its TMEM or leaves while the other may still
  // signal its barriers (the first CTA's MMAs have drained by now)
  if (PAIR) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
  });
  if (!fn) throw Error(-2, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

}  // namespace tc

// 3-D bf16 tensor map with 128-byte swizzle: extents dims[0..2] (dims[0]
// contiguous), strides of dims 1 and 2 in elements, box box[0..2].
CUtensorMap make_map3(const void* base, const int64_t dims[3], const int64_t strides[2],
                      const int box[3]) {
  DOP_REQUIRE(((uintptr_t)base & 15) == 0, "TMA base address must be 16-byte aligned");
  DOP_REQUIRE(strides[0] % 8 == 0 && strides[1] % 8 == 0,
              "TMA strides must be multiples of 16 bytes (8 bf16)");
  CUtensorMap m;
  cuuint64_t gd[3] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2]};
  cuuint64_t gs[2] = {(cuuint64_t)strides[0] * 2, (cuuint64_t)strides[1] * 2};
  cuuint32_t bx[3] = {(cuuint32_t)box[0], (cuuint32_t)box[1], (cuuint32_t)box[2]};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = tc::encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gd,
                               gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(-2, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

namespace tc {
// 3-D map {inner, outer, depth} with box {64, box_outer, 1}.
CUtensorMap make_map(const void* base, int64_t inner, int64_t outer, int64_t depth,
                     int64_t row_stride, int64_t depth_stride, int box_outer) {
  const int64_t dims[3] = {inner, outer, depth};
  const int64_t strides[2] = {row_stride, depth_stride};
  const int box[3] = {64, box_outer, 1};
  return make_map3(base, dims, strides, box);
}

template <bool A_MN, bool B_MN, int BN, bool DUAL, bool PAIR, bool TF = false>
void launch(const CUtensorMap* ma, const CUtensorMap* mb, const Params& p, int grid,
            cudaStream_t s) {
  constexpr int STG = PAIR ? PAIR_STAGES : STAGES;
  constexpr int BNL = PAIR ? BN / 2 : BN;
  constexpr size_t smem = (size_t)STG * (BM * BK * 2 + BNL * BK * 2) + 1024 + 256;
  static_assert(smem + 1024 <= 232448, "stages beyond the per-CTA shared memory");
  auto kern = k_gemm_tc<A_MN, B_MN, BN, DUAL, PAIR, TF>;
  bind_error_word();
  static bool attr = false;
  if (!attr) {
    DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  if (!PAIR) {
    kern<<<grid, THREADS, smem, s>>>(ma[0], ma[1], ma[2], mb[0], mb[1], mb[2], p);
    return;
  }
  // pairs of CTAs: clusters of two
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  DOP_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, ma[0], ma[1], ma[2], mb[0], mb[1], mb[2], p));
}

// Pairs of CTAs of this kernel that can be resident at once on the current
// device (cudaOccupancyMaxActiveClusters, clusters of two), cached.
template <bool A_MN, bool B_MN, int BN, bool DUAL, bool TF = false>
int pair_slots() {
  static int slots[16] = {0};
  int dev = 0;
  DOP_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) dev = 0;
  if (!slots[dev]) {
    constexpr size_t smem = (size_t)PAIR_STAGES * (BM * BK * 2 + (BN / 2) * BK * 2) + 1024 + 256;
    auto kern = k_gemm_tc<A_MN, B_MN, BN, DUAL, true, TF>;
    DOP_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)sm_count(), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    DOP_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    slots[dev] = n > 0 ? n : 1;
  }
  return slots[dev];
}

// Tile counter of the dynamic tile order for launches on stream `s`: one int
// per (device, stream) from a per-device pool; launches on one stream are
// serialised, so they can share it (each zeroes it first).  Null (static
// order) when the pool is used up, or when the stream is being captured and
// has no counter yet (the pool is allocated outside captures).
int* tile_counter(cudaStream_t s) {
  constexpr int kPool = 1024;
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, int*> ctr;
  static int* pool[16] = {nullptr};
  static int used[16] = {0};
  int dev = 0;
  DOP_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 16) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  auto it = ctr.find({dev, s});
  if (it != ctr.end()) return it->second;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  DOP_CHECK_CUDA(cudaStreamIsCapturing(s, &cap));
  if (cap != cudaStreamCaptureStatusNone) return nullptr;
  if (!pool[dev]) DOP_CHECK_CUDA(cudaMalloc(&pool[dev], sizeof(int) * kPool));
  if (used[dev] == kPool) return nullptr;
  int* c = pool[dev] + used[dev]++;
  ctr[{dev, s}] = c;
  return c;
}

}  // namespace tc

// One tensor-core GEMM.  `parts` are (A, lda, B, ldb, K) triples summed into
// one accumulator; all share the majors of g (a_t, b_t).
void gemm_tc(const Gemm& g, const GemmPart* extra, int n_extra, const TcEpilogue& te,
             cudaStream_t s, int64_t& launches) {
  using namespace tc;
  constexpr int BN = 256;
  DOP_REQUIRE(g.M > 0 && g.N > 0, "empty GEMM");
  DOP_REQUIRE(g.K > 0, "GEMM contraction extent (the row extent for grouped contractions) must be > 0");
  const bool dual = te.kind == kSwiGLU;
  Params p{};
  p.M = (int)g.M;
  p.N = (int)g.N;
  p.mode = g.group;
  p.seg_off = g.seg_off;
  p.seg_end = g.seg_end;
  p.tile_expert = g.tile_expert;
  p.G = g.G;
  DOP_REQUIRE(g.group != 2 || g.G <= kMaxExperts, "grouped contraction: at most kMaxExperts groups");
  if (te.kind >= 0) {
    p.epi = te.kind;
  } else if (g.epi == Epi::Store) {
    p.epi = g.c_f32 ? kStoreF32 : kStoreBF16;
  } else if (g.epi == Epi::Accum) {
    DOP_REQUIRE(g.c_f32, "accumulation needs an fp32 C");
    p.epi = kAccumF32;
  } else if (g.epi == Epi::AddRes) {
    DOP_REQUIRE(g.c_f32, "residual add needs an fp32 C");
    p.epi = kAddResF32;
  } else {
    throw Error(-4, "epilogue not implemented on the tensor-core path");
  }
  DOP_REQUIRE(g.ldc % 8 == 0 || te.kind >= 0, "ldc must be a multiple of 8");
  DOP_REQUIRE(te.kind < 0 || (g.N % 32 == 0 && te.ldg % 8 == 0),
              "SwiGLU epilogues need N and ldg multiples of 32 and 8");
  p.C = g.C;
  p.ldc = g.ldc;
  p.c_gs = g.c_gs;
  p.R = g.R;
  p.ldr = g.ldr;
  p.g_out = te.g_out; p.u_out = te.u_out; p.h_out = te.h_out;
  p.g_in = te.g_in; p.u_in = te.u_in; p.dg_out = te.dg_out; p.du_out = te.du_out;
  p.ldg = te.ldg;
  p.rope_cos = te.rope_cos;
  p.rope_sin = te.rope_sin;
  p.rope_seq = te.rope_seq;
  if (te.kind == kRopeBF16) {
    DOP_REQUIRE(g.group == 0 && g.N % 128 == 0 && g.ldc % 8 == 0 && te.rope_cos && te.rope_sin &&
                    te.rope_seq > 0,
                "the RoPE epilogue needs a plain GEMM, 128-wide heads and the tables");
  }
  const int out_tile = dual ? BN / 2 : BN;
  p.n_tiles = (int)ceil_div(g.N, out_tile);
  // pairs of CTAs (256-row tiles) whenever there are at least 256 rows
  const bool pair = g.M >= 2 * BM;
  p.m_tiles = (int)ceil_div(g.M, pair ? 2 * BM : BM);
  // parts
  GemmPart parts[3];
  parts[0] = GemmPart{g.A, g.lda, g.B, g.ldb, g.K};
  DOP_REQUIRE(n_extra >= 0 && n_extra <= 2, "at most three K parts");
  for (int i = 0; i < n_extra; ++i) parts[i + 1] = extra[i];
  p.nparts = 1 + n_extra;
  DOP_REQUIRE(g.group != 2 || p.nparts == 1, "grouped contraction takes one part");
  CUtensorMap ma[3], mb[3];
  const int64_t Gd = g.group == 1 ? g.G : 1;  // expert depth of B maps
  for (int i = 0; i < p.nparts; ++i) {
    const GemmPart& q = parts[i];
    const int64_t Kext = g.group == 2 ? q.K : q.K;  // rows of the contraction
    p.kb[i] = (int)ceil_div(q.K, BK);
    // A: (M x K); K-major [M][K] or M-major [K][M]
    if (!g.a_t) ma[i] = make_map(q.A, Kext, g.M, 1, q.lda, q.lda * g.M, BM);
    else ma[i] = make_map(q.A, g.M, Kext, 1, q.lda, q.lda * Kext, 64);
    // B: (K x N); N-major [K][N] (b_t = false) or K-major [N][K]
    const int64_t Nb = dual ? g.N : g.N;
    const int box_n = (dual || pair) ? BN / 2 : BN;
    if (!g.b_t) mb[i] = make_map(q.B, Nb, Kext, Gd, q.ldb, Gd > 1 ? g.b_gs : q.ldb * Kext, 64);
    else mb[i] = make_map(q.B, Kext, Nb, Gd, q.ldb, Gd > 1 ? g.b_gs : q.ldb * Nb, box_n);
  }
  if (dual) {
    DOP_REQUIRE(te.up_B != nullptr, "SwiGLU needs the up-projection weights");
    if (!g.b_t) mb[1] = make_map(te.up_B, g.N, g.K, Gd, g.ldb, Gd > 1 ? g.b_gs : g.ldb * g.K, 64);
    else mb[1] = make_map(te.up_B, g.K, g.N, Gd, g.ldb, Gd > 1 ? g.b_gs : g.ldb * g.N, BN / 2);
    DOP_REQUIRE(p.nparts == 1, "SwiGLU GEMM takes one part");
  }
  for (int i = p.nparts; i < 3; ++i) ma[i] = ma[0];
  for (int i = (dual ? 2 : p.nparts); i < 3; ++i) mb[i] = mb[0];
  const int64_t tiles = (int64_t)(g.group == 2 ? g.G : 1) * p.m_tiles * p.n_tiles;
  // Row tiles walked before the next column tile: 8 for long contractions
  // (>= 8192; an operand tile there is >= 4 MB and must be reused by tiles
  // that run close together), else 16.  Measured on the Mixtral-8x7B step:
  // 57.6 ms of GEMMs against 59.4 (16 everywhere), 58.1 (4) and 59.0 (2).
  p.gm = (int64_t)(n_extra + 1) * g.K >= 8192 ? 8 : 16;
  // dynamic tile order: the stream's counter, zeroed before the launch
  p.tile_ctr = tile_counter(s);
  if (p.tile_ctr) DOP_CHECK_CUDA(cudaMemsetAsync(p.tile_ctr, 0, sizeof(int), s));
  const bool A = g.a_t, B = !g.b_t;  // MN-major flags
  if (dual && A) throw Error(-4, "SwiGLU GEMM needs a K-major A");
  auto go = [&](auto a_mn, auto b_mn, auto du, auto pr) {
    constexpr bool AM = decltype(a_mn)::value, BMN = decltype(b_mn)::value;
    constexpr bool DU = decltype(du)::value, PR = decltype(pr)::value;
    // persistent grid: one CTA (pair) per SM (pair of SMs) that can be resident
    int units = PR ? pair_slots<AM, BMN, BN, DU>() : sm_count();
    int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, units));
    launch<AM, BMN, BN, DU, PR>(ma, mb, p, PR ? 2 * grid : grid, s);
  };
  using T_ = std::true_type;
  using F_ = std::false_type;
  if (pair) {
    if (dual) {
      if (B) go(F_{}, T_{}, T_{}, T_{});
      else go(F_{}, F_{}, T_{}, T_{});
    } else if (!A && B) go(F_{}, T_{}, F_{}, T_{});
    else if (!A && !B) go(F_{}, F_{}, F_{}, T_{});
    else if (A && B) go(T_{}, T_{}, F_{}, T_{});
    else go(T_{}, F_{}, F_{}, T_{});
  } else {
    if (dual) {
      if (B) go(F_{}, T_{}, T_{}, F_{});
      else go(F_{}, F_{}, T_{}, F_{});
    } else if (!A && B) go(F_{}, T_{}, F_{}, F_{});
    else if (!A && !B) go(F_{}, F_{}, F_{}, F_{});
    else if (A && B) go(T_{}, T_{}, F_{}, F_{});
    else go(T_{}, F_{}, F_{}, F_{});
  }
  DOP_LAUNCHED(launches);
}

// ------------------------------------------------------ 3xTF32 (fp32 lens)
// The fp32 lens's contractions on the tensor cores: each fp32 operand x is
// split into hi = x rounded to tf32 and lo = x - hi (exact in fp32), and
// C = A_hi B_hi + A_hi B_lo + A_lo B_hi is accumulated in fp32 TMEM as the
// three K parts of one tf32 GEMM (the dropped lo x lo term is ~2^-22 of the
// product; the tensor core reads lo to tf32 precision, ~2^-11 of lo).  The
// split also lays both operands out K-major, which the tf32 path requires.

namespace {
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// out[z][o][i] = split(src(z, o, i)) with src(z, o, i) = src[z zs + o ld + i]:
// an elementwise map, four elements (16-byte loads, two 16-byte stores) a
// thread when the rows allow it.
template <bool VEC>
__global__ void k_split_tf32_rows(const float* __restrict__ src, int64_t Z, int64_t O, int64_t Ki,
                                  int64_t ld, int64_t zs, float* __restrict__ hi,
                                  float* __restrict__ lo) {
  constexpr int W = VEC ? 4 : 1;
  const int64_t per_row = Ki / W, total = Z * O * per_row;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / per_row, i = (e % per_row) * W;
    const int64_t z = row / O, o = row % O;
    const float* sp = src + z * zs + o * ld + i;
    const int64_t at = row * Ki + i;
    if (VEC) {
      const float4 x = *reinterpret_cast<const float4*>(sp);
      const float4 h = make_float4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
      *reinterpret_cast<float4*>(hi + at) = h;
      *reinterpret_cast<float4*>(lo + at) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    } else {
      const float x = sp[0], h = tf32_rna(x);
      hi[at] = h;
      lo[at] = x - h;
    }
  }
}

// out[z][o][i] = split(src[z zs + i ld + o]): a transposition through a
// 32 x 32 shared tile per CTA of 32 x 8 threads, read along o and written
// along i, both coalesced.
__global__ void k_split_tf32_tr(const float* __restrict__ src, int64_t O, int64_t Ki, int64_t ld,
                                int64_t zs, float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int64_t z = blockIdx.z;
  const int64_t o0 = (int64_t)blockIdx.y * 32, i0 = (int64_t)blockIdx.x * 32;
  const float* sz = src + z * zs;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int r = ty; r < 32; r += 8) {  // rows i, columns o (contiguous in src)
    const int64_t i = i0 + r, o = o0 + tx;
    tile[r][tx] = (i < Ki && o < O) ? sz[i * ld + o] : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {  // rows o, columns i
    const int64_t o = o0 + r, i = i0 + tx;
    if (o >= O || i >= Ki) continue;
    const float x = tile[tx][r];
    const float h = tf32_rna(x);
    const int64_t at = (z * O + o) * Ki + i;
    hi[at] = h;
    lo[at] = x - h;
  }
}

void split_tf32(const float* src, int64_t Z, int64_t O, int64_t Ki, int64_t ld, int64_t zs, bool tr,
                float* hi, float* lo, cudaStream_t s, int64_t& launches) {
  if (tr) {
    const dim3 grid((unsigned)ceil_div(Ki, 32), (unsigned)ceil_div(O, 32), (unsigned)Z);
    k_split_tf32_tr<<<grid, dim3(32, 8), 0, s>>>(src, O, Ki, ld, zs, hi, lo);
  } else {
    const bool vec = Ki % 4 == 0 && ld % 4 == 0 && zs % 4 == 0 && (uintptr_t)src % 16 == 0;
    const int64_t items = Z * O * (vec ? Ki / 4 : Ki);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, 256), 16 * sm_count()));
    if (vec) k_split_tf32_rows<true><<<grid, 256, 0, s>>>(src, Z, O, Ki, ld, zs, hi, lo);
    else k_split_tf32_rows<false><<<grid, 256, 0, s>>>(src, Z, O, Ki, ld, zs, hi, lo);
  }
  DOP_LAUNCHED(launches);
}

// C (epi) = sum over s < S of part[s] (M x N, row-major), summed in s order:
// the split contraction's partial products.  VEC: 4 columns a thread.
template <bool VEC>
__global__ void k_sum_chunks_f32(const float* __restrict__ part, int S, int64_t M, int64_t N,
                                 float* __restrict__ C, int64_t ldc, int epi,
                                 const float* __restrict__ R, int64_t ldr) {
  constexpr int W = VEC ? 4 : 1;
  const int64_t cols = N / W, total = M * cols, MN = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / cols, n = (i % cols) * W;
    float v[W];
#pragma unroll
    for (int e = 0; e < W; ++e) v[e] = 0.f;
    for (int c = 0; c < S; ++c) {
      const float* src = part + c * MN + m * N + n;
      if constexpr (VEC) {
        const float4 x = *(const float4*)src;
        v[0] += x.x;
        v[1] += x.y;
        v[2] += x.z;
        v[3] += x.w;
      } else {
        v[0] += src[0];
      }
    }
    float* out = C + m * ldc + n;
    const float* r = R ? R + m * ldr + n : nullptr;
#pragma unroll
    for (int e = 0; e < W; ++e) {
      if (epi == tc::kAccumF32) out[e] += v[e];
      else if (epi == tc::kAddResF32) out[e] = v[e] + r[e];
      else out[e] = v[e];
    }
  }
}

// 3-D fp32 (tf32) tensor map with 128-byte swizzle, box {32, box_outer, 1}.
CUtensorMap make_map3_f32(const float* base, int64_t inner, int64_t outer, int64_t depth,
                          int64_t row_stride, int64_t depth_stride, int box_outer) {
  DOP_REQUIRE((uintptr_t)base % 16 == 0, "TMA base must be 16-byte aligned");
  DOP_REQUIRE(row_stride % 4 == 0 && depth_stride % 4 == 0,
              "TMA strides must be multiples of 16 bytes (4 floats)");
  CUtensorMap m;
  cuuint64_t gd[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)depth};
  cuuint64_t gs[2] = {(cuuint64_t)row_stride * 4, (cuuint64_t)depth_stride * 4};
  cuuint32_t bx[3] = {32, (cuuint32_t)box_outer, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = tc::encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), gd,
                               gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw Error(-2, "cuTensorMapEncodeTiled (fp32) failed (" + std::to_string((int)r) + ")");
  return m;
}
}  // namespace

int64_t gemm_tc_f32_scratch(const Gemm& g) {
  const int64_t Gb = g.group == 1 ? g.G : 1;
  return 2 * (g.M * g.K + Gb * g.N * g.K);
}

bool gemm_tc_f32_ok(const Gemm& g) {
  return g.M >= 128 && g.N >= 64 && g.K >= 32 && g.K % 4 == 0 && g.c_f32 &&
         (g.epi == Epi::Store || g.epi == Epi::Accum || g.epi == Epi::AddRes) && !g.relu &&
         !g.bias && !g.mask && g.ldc % 4 == 0 && (uintptr_t)g.C % 16 == 0;
}

void gemm_tc_f32(const Gemm& g, float* ws, int64_t ws_cap, cudaStream_t s, int64_t& launches) {
  using namespace tc;
  constexpr int BN = 256;
  DOP_REQUIRE(gemm_tc_f32_ok(g), "shape or epilogue outside the 3xTF32 path");
  DOP_REQUIRE(ws && gemm_tc_f32_scratch(g) <= ws_cap, "3xTF32 scratch too small");
  const int64_t M = g.M, N = g.N, K = g.K;
  const int64_t Gb = g.group == 1 ? g.G : 1;
  float* a_hi = ws;
  float* a_lo = a_hi + M * K;
  float* b_hi = a_lo + M * K;
  float* b_lo = b_hi + Gb * N * K;
  // A(m, k) = A[m lda + k] or A[k lda + m] (a_t) -> [M][K]
  split_tf32((const float*)g.A, 1, M, K, g.lda, 0, g.a_t, a_hi, a_lo, s, launches);
  // B(k, n) = B[k ldb + n] or B[n ldb + k] (b_t), per expert z -> [Gb][N][K]
  split_tf32((const float*)g.B, Gb, N, K, g.ldb, Gb > 1 ? g.b_gs : 0, !g.b_t, b_hi, b_lo, s,
             launches);
  Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.mode = g.group;
  p.seg_off = g.seg_off;
  p.seg_end = g.seg_end;
  p.tile_expert = g.tile_expert;
  p.G = g.G;
  p.epi = g.epi == Epi::Store ? kStoreF32 : (g.epi == Epi::Accum ? kAccumF32 : kAddResF32);
  p.C = g.C;
  p.ldc = g.ldc;
  p.c_gs = g.c_gs;
  p.R = g.R;
  p.ldr = g.ldr;
  p.n_tiles = (int)ceil_div(N, BN);
  const bool pair = M >= 2 * BM;
  p.m_tiles = (int)ceil_div(M, pair ? 2 * BM : BM);
  p.nparts = 3;
  for (int i = 0; i < 3; ++i) p.kb[i] = (int)ceil_div(K, 32);
  p.gm = 3 * K >= 8192 ? 8 : 16;
  // A plain product with too few output tiles to fill the GPU splits its
  // contraction: chunk g of S (a multiple of 4 k-blocks) runs as group g of
  // a grouped contraction into partials after the operands in `ws`, summed
  // in chunk order by k_sum_chunks_f32 (deterministic).
  int S = 1;
  float* part = b_lo + Gb * N * K;
  if (g.group == 0) {
    const int64_t tiles0 = (int64_t)p.m_tiles * p.n_tiles;
    const int64_t units = pair ? pair_slots<false, false, BN, false, true>() : sm_count();
    const int64_t kb = ceil_div(K, 32);
    const int64_t room = (ws_cap - gemm_tc_f32_scratch(g)) / (M * N);
    const int64_t want = std::min<int64_t>({units / std::max<int64_t>(tiles0, 1), kb / 4,
                                            (int64_t)kMaxExperts, room});
    if (want >= 2) S = (int)want;
  }
  if (S > 1) {
    const int64_t kb = ceil_div(K, 32);
    p.mode = 2;
    p.G = S;
    p.kchunk = (int)(ceil_div(kb, S) * 32);
    p.ktot = (int)K;
    S = (int)ceil_div(K, p.kchunk);  // every chunk non-empty
    p.G = S;
    p.C = part;
    p.ldc = N;
    p.c_gs = M * N;
    p.epi = kStoreF32;
  }
  const int box_n = pair ? BN / 2 : BN;
  CUtensorMap ma[3], mb[3];
  ma[0] = ma[1] = make_map3_f32(a_hi, K, M, 1, K, K * M, BM);
  ma[2] = make_map3_f32(a_lo, K, M, 1, K, K * M, BM);
  mb[0] = mb[2] = make_map3_f32(b_hi, K, N, Gb, K, N * K, box_n);
  mb[1] = make_map3_f32(b_lo, K, N, Gb, K, N * K, box_n);
  const int64_t tiles = (int64_t)(p.mode == 2 ? p.G : 1) * p.m_tiles * p.n_tiles;
  p.tile_ctr = tile_counter(s);
  if (p.tile_ctr) DOP_CHECK_CUDA(cudaMemsetAsync(p.tile_ctr, 0, sizeof(int), s));
  if (pair) {
    const int units = pair_slots<false, false, BN, false, true>();
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, units));
    launch<false, false, BN, false, true, true>(ma, mb, p, 2 * grid, s);
  } else {
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, sm_count()));
    launch<false, false, BN, false, false, true>(ma, mb, p, grid, s);
  }
  DOP_LAUNCHED(launches);
  if (S > 1) {
    const int epi = g.epi == Epi::Store ? kStoreF32 : (g.epi == Epi::Accum ? kAccumF32 : kAddResF32);
    const bool vec = N % 4 == 0 && g.ldc % 4 == 0 && (uintptr_t)g.C % 16 == 0 &&
                     (g.epi != Epi::AddRes || (g.ldr % 4 == 0 && (uintptr_t)g.R % 16 == 0));
    const int64_t items = M * N / (vec ? 4 : 1);
    const int grid = (int)std::min<int64_t>(ceil_div(items, 256), 8 * sm_count());
    if (vec)
      k_sum_chunks_f32<true><<<grid, 256, 0, s>>>(part, S, M, N, (float*)g.C, g.ldc, epi, g.R, g.ldr);
    else
      k_sum_chunks_f32<false><<<grid, 256, 0, s>>>(part, S, M, N, (float*)g.C, g.ldc, epi, g.R, g.ldr);
    DOP_LAUNCHED(launches);
  }
}

int* tc_error_word() {
  static int* words[16] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  DOP_CHECK_CUDA(cudaGetDevice(&dev));
  DOP_REQUIRE(dev >= 0 && dev < 16, "device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev]) {
    DOP_CHECK_CUDA(cudaMalloc(&words[dev], kErrWords * sizeof(int)));
    DOP_CHECK_CUDA(cudaMemset(words[dev], 0, kErrWords * sizeof(int)));
  }
  return words[dev];
}

int tc_error_status() {
  int v = 0;
  int* w = tc_error_word();
  if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return v;
}

}  // namespace dop
