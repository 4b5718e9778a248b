// ep.cu — expert parallelism for the Mixtral block lens: each rank owns
// experts [rank * Ed, (rank + 1) * Ed) (Ed = E / world) and runs their
// grouped GEMMs over the expert-sorted rows that every rank routed to them.
//
// The exchange is fused with the permutation and the combine: there is no
// separate all-to-all and no send buffer.  Every rank's block workspace is
// one cudaMalloc shared with the other ranks through CUDA IPC, so a rank
// reads a peer's buffer at (peer base + the same offset as its own):
//   dispatch (fwd)   the owner gathers its receive rows straight from the
//                    sources' normalised activations xn2, through the
//                    sources' row -> token maps (k_ep_gather_tokens);
//   combine (fwd)    each source reads the expert outputs of its (token,
//                    slot) pairs from the owners and sums them into y
//                    (k_ep_combine), keeping a local copy for the backward;
//   dispatch (bwd)   the owner copies the sources' output cotangent rows
//                    (k_ep_gather_rows);
//   combine (bwd)    each source sums the expert-input cotangents of its
//                    pairs from the owners (k_ep_unpermute_router_dx).
// Receive buffers are expert-major: local expert j's rows from source 0, 1,
// ...; each (expert, source) piece keeps the source's segment padding (a
// multiple of 256 rows, the pair GEMM's tile), so a GEMM row tile belongs to
// one expert and the weight-gradient contraction of expert j runs over one
// contiguous range.
//
// Which rank processes which rows is decided every step by a plan that every
// rank computes from the same routing counts (k_ep_layout): the expert-major
// sequence of (expert, source) pieces is cut into `world` near-equal chunks,
// snapping a cut to an expert boundary when one lies within a tenth of a
// chunk.  Balanced routing thus keeps each expert whole on one rank; under
// skewed routing a hot expert's rows are split over several ranks (its
// weights are on every rank: the block reads the whole layer slice).  A rank
// that processes rows of an expert it does not own writes that expert's
// partial weight adjoint to dw_help; after the last barrier the owner adds
// the helpers' partials, in rank order, into its dparams.  The split is
// invisible in y and dx: a row's GEMMs do not depend on where the row runs.
//
// Ordering between ranks uses five flag barriers per step (k_ep_barrier):
// after the permutation (sources' rows readable), after the down projection
// (expert outputs readable), after the output-cotangent gather source is
// written (dO readable), after the expert-input cotangent GEMM (dXp
// readable), after the weight-adjoint GEMMs (partial adjoints readable).
// Every buffer a peer reads is next overwritten only after a later barrier,
// which the reader can only pass after its reads.  Waits are bounded; a wait
// that runs out records a code in the device error word and the kernels that
// follow skip their work.
#include <climits>

#include "ep.cuh"
#include "tc_ptx.cuh"

namespace dop {
namespace ep {

using tc::g_err;
using tc::gtime_ns;

constexpr uint64_t kBarrierNs = 20000000000ull;  // default: 20 s per barrier

__device__ __forceinline__ uint64_t barrier_limit_ns() {
  const uint64_t v = *(volatile const uint64_t*)(g_err + 4);
  return v ? v : kBarrierNs;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Peer copy of a workspace pointer: same offset from the peer's base.
template <typename P>
__device__ __forceinline__ P* peer(const EpView& v, int s, P* mine) {
  return reinterpret_cast<P*>(v.peers[s] + (reinterpret_cast<const char*>(mine) - v.peers[v.rank]));
}

// Barrier `k` of epoch `epoch`: thread s tells rank s that this rank
// arrived (flags[k][rank] on rank s), then waits until rank s arrived here.
__global__ void k_ep_barrier(EpView v, int k, unsigned epoch) {
  const int s = threadIdx.x;
  if (s < v.world) {
    __threadfence_system();
    st_release_sys(peer(v, s, v.flags) + k * kEpMaxWorld + v.rank, epoch);
    const unsigned* mine = v.flags + k * kEpMaxWorld + s;
    const uint64_t t0 = gtime_ns();
    // bounded: gives up when another wait already failed or after the limit
    for (uint32_t i = 0;; ++i) {
      if ((int)(ld_acquire_sys(mine) - epoch) >= 0) break;
      if ((i & 255u) == 255u) {
        if (*(volatile int*)g_err) break;
        if (gtime_ns() - t0 > barrier_limit_ns()) {
          atomicCAS(g_err, 0, 60 + k);
          break;
        }
      }
    }
    __threadfence_system();
  }
}

// The plan and this rank's receive layout (one CTA): reads every rank's
// padded segment offsets, cuts the expert-major piece sequence into the
// ranks' chunks, and writes this rank's receive segments per expert, its
// tile -> (expert, source, source row) map, where this rank's own pieces sit
// in the global sequence, and which ranks help with each expert.
__global__ void k_ep_layout(EpView v) {
  if (tc::tc_failed()) return;  // an earlier wait gave up: skip (sticky error)
  __shared__ int so[kEpMaxWorld][kMaxExperts + 1];
  __shared__ int pstart[kMaxExperts][kEpMaxWorld];  // global start of piece (e, s)
  __shared__ int estart[kMaxExperts + 1];
  __shared__ int bnd[kEpMaxWorld + 1];
  const int W = v.world, E = v.E;
  for (int i = threadIdx.x; i < W * (E + 1); i += blockDim.x) {
    const int s = i / (E + 1), e = i % (E + 1);
    so[s][e] = __ldcv(peer(v, s, v.seg_off) + e);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int at = 0;
    for (int e = 0; e < E; ++e) {
      estart[e] = at;
      for (int s = 0; s < W; ++s) {
        pstart[e][s] = at;
        at += so[s][e + 1] - so[s][e];
      }
    }
    estart[E] = at;
    const int N = at;  // a multiple of kSegAlign: every piece is
    bnd[0] = 0;
    bnd[W] = N;
    for (int d = 1; d < W; ++d) {
      int cut = (int)((int64_t)N * d / W / kSegAlign * kSegAlign);
      int best = cut, dist = INT_MAX;
      for (int e = 0; e <= E; ++e) {
        const int dd = abs(estart[e] - cut);
        if (dd < dist) { dist = dd; best = estart[e]; }
      }
      if ((int64_t)dist * 10 * W <= N) cut = best;  // within a tenth of a chunk
      bnd[d] = min(max(cut, bnd[d - 1]), N);
    }
    for (int d = 0; d <= W; ++d) v.bounds[d] = bnd[d];
    const int lo = bnd[v.rank], hi = bnd[v.rank + 1];
    for (int e = 0; e < E; ++e) v.piece_pos[e] = pstart[e][v.rank];
    for (int e = 0; e <= E; ++e) v.recv_seg_off[e] = min(max(estart[e], lo), hi) - lo;
    for (int e = 0; e < E; ++e) {
      const int owner = e / v.local;
      const bool mine = owner == v.rank;
      v.own_end[e] = mine ? v.recv_seg_off[e + 1] : v.recv_seg_off[e];
      v.help_end[e] = mine ? v.recv_seg_off[e] : v.recv_seg_off[e + 1];
      int mask = 0;
      for (int d = 0; d < W; ++d)
        if (d != owner && bnd[d] < estart[e + 1] && bnd[d + 1] > estart[e]) mask |= 1 << d;
      v.helpers[e] = mask;
    }
  }
  __syncthreads();
  // tile map of this rank's receive buffer
  const int lo = bnd[v.rank], rows = bnd[v.rank + 1] - lo;
  for (int t = threadIdx.x; t < v.recv_tiles; t += blockDim.x) {
    int ex = -1, src = -1, srow = 0;
    if (t * kRowAlign < rows) {
      const int g = lo + t * kRowAlign;
      for (int e = 0; e < E && ex < 0; ++e)
        for (int s = 0; s < W; ++s) {
          const int n = so[s][e + 1] - so[s][e];
          if (g >= pstart[e][s] && g < pstart[e][s] + n) {
            ex = e; src = s; srow = so[s][e] + (g - pstart[e][s]);
            break;
          }
        }
    }
    v.recv_tile_expert[t] = ex;
    v.recv_tile_src[t] = src;
    v.recv_tile_row0[t] = srow;
  }
}

// One warp copies a row of n16 16-byte words from a peer: each lane issues
// eight loads before it stores any, so eight NVLink round trips overlap.
__device__ __forceinline__ void copy_row16(uint4* dst, const uint4* src, int n16, int lane) {
  for (int i0 = lane; i0 < n16; i0 += 8 * 32) {
    uint4 w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * 32 < n16) w[u] = __ldcv(src + i0 + u * 32);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i0 + u * 32 < n16) dst[i0 + u * 32] = w[u];
  }
}

// Owner side of the forward dispatch: receive row r (a row of source s's
// expert-sorted buffer) = xn2_s[row_token_s[row]], or zeros for padding.
// One warp per row, 16-byte words.
__global__ void k_ep_gather_tokens(EpView v, const bf16* xn2, int D) {
  if (tc::tc_failed()) return;
  const int n16 = D * 2 / 16;
  const int rows = v.recv_seg_off[v.E];
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int tile = (int)(r / kRowAlign);
    const int s = v.recv_tile_src[tile];
    if (s < 0 || s >= v.world) continue;
    const int srow = v.recv_tile_row0[tile] + (int)(r % kRowAlign);
    const int tok = __ldcv(peer(v, s, v.row_token) + srow);
    uint4* dst = reinterpret_cast<uint4*>(v.xr) + r * n16;
    if (tok >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(peer(v, s, xn2)) + (int64_t)tok * n16;
      copy_row16(dst, src, n16, lane);
    } else {
      for (int i = lane; i < n16; i += 32) dst[i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// Owner side of the backward dispatch: receive row r = row srow of source
// s's expert-sorted output cotangent dO.
__global__ void k_ep_gather_rows(EpView v, const bf16* dO, bf16* dst_rows, int D) {
  if (tc::tc_failed()) return;
  const int n16 = D * 2 / 16;
  const int rows = v.recv_seg_off[v.E];
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int tile = (int)(r / kRowAlign);
    const int s = v.recv_tile_src[tile];
    if (s < 0 || s >= v.world) continue;
    const int srow = v.recv_tile_row0[tile] + (int)(r % kRowAlign);
    const uint4* src = reinterpret_cast<const uint4*>(peer(v, s, dO)) + (int64_t)srow * n16;
    uint4* dst = reinterpret_cast<uint4*>(dst_rows) + r * n16;
    copy_row16(dst, src, n16, lane);
  }
}

// The rank that processed the row of this rank's expert-sorted row
// `slot_row` (expert e) and where it sits in that rank's receive buffer,
// clamped into the buffer (it is inside whenever the barriers held).
__device__ __forceinline__ int64_t processed_at(const EpView& v, int e, int slot_row, int& d) {
  const int pos = v.piece_pos[e] + (slot_row - v.seg_off[e]);
  d = 0;
  while (d + 1 < v.world && v.bounds[d + 1] <= pos) ++d;
  const int64_t r = (int64_t)pos - v.bounds[d];
  return r < 0 ? 0 : (r >= v.recv_cap ? v.recv_cap - 1 : r);
}

// Source side of the forward combine: y[t] = mid[t] + sum_k w_k out_k, with
// out_k read from the owner of expert top_i[t, k] (slot order, from zero, as
// src/mixtral.rs:330-359) and copied to this rank's `out` at slot_row for
// the router Jacobian of the backward.
__global__ void k_ep_combine(EpView v, const float* __restrict__ mid, const int* __restrict__ top_i,
                             const int* __restrict__ slot_row, const float* __restrict__ top_w,
                             int K, int D, float* __restrict__ out, float* __restrict__ y) {
  if (tc::tc_failed()) return;
  const int64_t t = blockIdx.x;
  __shared__ const float4* src[kMaxTopK];
  __shared__ float4* stash[kMaxTopK];
  __shared__ float ws[kMaxTopK];
  if (threadIdx.x < K) {
    const int k = threadIdx.x;
    const int e = top_i[t * K + k], sr = slot_row[t * K + k];
    int d;
    const int64_t row = processed_at(v, e, sr, d);
    src[k] = reinterpret_cast<const float4*>(peer(v, d, v.outr) + row * D);
    stash[k] = reinterpret_cast<float4*>(out + (int64_t)sr * D);
    ws[k] = top_w[t * K + k];
  }
  __syncthreads();
  const int D4 = D / 4;
  // every peer load of a thread's four columns is issued before any is used
  for (int i0 = threadIdx.x; i0 < D4; i0 += 4 * blockDim.x) {
    float4 o[4][kMaxTopK];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K && i0 + u * (int)blockDim.x < D4) o[u][k] = __ldcv(src[k] + i0 + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= D4) break;
      float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k) {
        if (k >= K) break;
        stash[k][i] = o[u][k];
        m.x += ws[k] * o[u][k].x; m.y += ws[k] * o[u][k].y;
        m.z += ws[k] * o[u][k].z; m.w += ws[k] * o[u][k].w;
      }
      const float4 a = reinterpret_cast<const float4*>(mid + t * D)[i];
      reinterpret_cast<float4*>(y + t * D)[i] =
          make_float4(a.x + m.x, a.y + m.y, a.z + m.z, a.w + m.w);
    }
  }
}

// Source side of the backward combine: d_xn2[t] = sum_k dXp_k + dz[t] Wr^T,
// dXp_k read from the owners (src/mixtral.rs:516, 535-540).
template <typename T, bool E8>
__global__ void k_ep_unpermute_router_dx(EpView v, const int* __restrict__ top_i,
                                         const int* __restrict__ slot_row,
                                         const float* __restrict__ dz, const T* __restrict__ wr,
                                         int E, int K, int D, float* __restrict__ dxn) {
  if (tc::tc_failed()) return;
  const int64_t t = blockIdx.x;
  __shared__ float dzs[kMaxExperts];
  __shared__ const float4* src[kMaxTopK];
  if (threadIdx.x < E) dzs[threadIdx.x] = dz[t * E + threadIdx.x];
  if (threadIdx.x < K) {
    const int k = threadIdx.x;
    const int e = top_i[t * K + k], sr = slot_row[t * K + k];
    int d;
    const int64_t row = processed_at(v, e, sr, d);
    src[k] = reinterpret_cast<const float4*>(peer(v, d, v.dxpr) + row * D);
  }
  __syncthreads();
  const int D4 = D / 4;
  for (int i0 = threadIdx.x; i0 < D4; i0 += 4 * blockDim.x) {
    float4 o[4][kMaxTopK];
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K && i0 + u * (int)blockDim.x < D4) o[u][k] = __ldcv(src[k] + i0 + u * blockDim.x);
#pragma unroll
    for (int u4 = 0; u4 < 4; ++u4) {
    const int i = i0 + u4 * blockDim.x;
    if (i >= D4) break;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < kMaxTopK; ++k) {
      if (k >= K) break;
      a.x += o[u4][k].x; a.y += o[u4][k].y; a.z += o[u4][k].z; a.w += o[u4][k].w;
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
    reinterpret_cast<float4*>(dxn + t * D)[i] =
        make_float4(a.x + rr[0], a.y + rr[1], a.z + rr[2], a.w + rr[3]);
    }
  }
}

// Owner side of the adjoint of the experts it owns: dP[e] += the partial
// adjoints the helper ranks wrote for e, in rank order (VT = float4 when the
// slices are 16-byte aligned, else float; every helper's load is issued
// before the sum).
template <typename VT>
__global__ void k_ep_reduce_adjoint(EpView v, float* __restrict__ dP) {
  if (tc::tc_failed()) return;
  constexpr int W4 = sizeof(VT) / 4;
  const int64_t nv = v.expert_stride / W4;
  for (int j = 0; j < v.local; ++j) {
    const int e = v.rank * v.local + j;
    const int mask = v.helpers[e];
    if (!mask) continue;
    const VT* hp[kEpMaxWorld];
    int nh = 0;
    for (int d = 0; d < v.world; ++d)
      if ((mask >> d) & 1)
        hp[nh++] = reinterpret_cast<const VT*>(peer(v, d, v.dw_help) + e * v.expert_stride);
    VT* out = reinterpret_cast<VT*>(dP + e * v.expert_stride);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv;
         i += (int64_t)gridDim.x * blockDim.x) {
      VT h[kEpMaxWorld];
#pragma unroll
      for (int q = 0; q < kEpMaxWorld; ++q)
        if (q < nh) h[q] = __ldcv(hp[q] + i);
      VT a = out[i];
      float* af = reinterpret_cast<float*>(&a);
#pragma unroll
      for (int q = 0; q < kEpMaxWorld; ++q) {
        if (q >= nh) break;
        const float* hf = reinterpret_cast<const float*>(&h[q]);
#pragma unroll
        for (int c = 0; c < W4; ++c) af[c] += hf[c];
      }
      out[i] = a;
    }
  }
}

}  // namespace ep

using namespace ep;

void ep_barrier(const EpView& v, int k, unsigned epoch, cudaStream_t s, int64_t& launches) {
  tc::bind_error_word();
  k_ep_barrier<<<1, 32, 0, s>>>(v, k, epoch);
  DOP_LAUNCHED(launches);
}

void ep_layout(const EpView& v, cudaStream_t s, int64_t& launches) {
  tc::bind_error_word();
  DOP_REQUIRE(v.E <= kMaxExperts && v.world <= kEpMaxWorld && v.E % v.world == 0,
              "expert-parallel plan out of range");
  k_ep_layout<<<1, 256, 0, s>>>(v);
  DOP_LAUNCHED(launches);
}

void ep_reduce_adjoint(const EpView& v, float* dP_experts, cudaStream_t s, int64_t& launches) {
  tc::bind_error_word();
  const bool vec = v.expert_stride % 4 == 0 && (uintptr_t)dP_experts % 16 == 0 &&
                   (uintptr_t)v.dw_help % 16 == 0;
  if (vec) k_ep_reduce_adjoint<float4><<<sm_count() * 4, 256, 0, s>>>(v, dP_experts);
  else k_ep_reduce_adjoint<float><<<sm_count() * 4, 256, 0, s>>>(v, dP_experts);
  DOP_LAUNCHED(launches);
}

void ep_gather_tokens(const EpView& v, const bf16* xn2, int D, cudaStream_t s, int64_t& launches) {
  tc::bind_error_word();
  k_ep_gather_tokens<<<sm_count() * 8, 256, 0, s>>>(v, xn2, D);
  DOP_LAUNCHED(launches);
}

void ep_gather_rows(const EpView& v, const bf16* dO, bf16* dst, int D, cudaStream_t s,
                    int64_t& launches) {
  tc::bind_error_word();
  k_ep_gather_rows<<<sm_count() * 8, 256, 0, s>>>(v, dO, dst, D);
  DOP_LAUNCHED(launches);
}

void ep_combine(const EpView& v, const float* mid, const int* top_i, const int* slot_row,
                const float* top_w, int64_t T, int K, int D, float* out, float* y, cudaStream_t s,
                int64_t& launches) {
  tc::bind_error_word();
  k_ep_combine<<<(unsigned)T, 256, 0, s>>>(v, mid, top_i, slot_row, top_w, K, D, out, y);
  DOP_LAUNCHED(launches);
}

template <typename T>
void ep_unpermute_router_dx(const EpView& v, const int* top_i, const int* slot_row,
                            const float* dz, const T* wr, int64_t Tn, int E, int K, int D,
                            float* dxn, cudaStream_t s, int64_t& launches) {
  tc::bind_error_word();
  if (E == 8 && (uintptr_t)wr % 16 == 0)
    k_ep_unpermute_router_dx<T, true><<<(unsigned)Tn, 256, 0, s>>>(v, top_i, slot_row, dz, wr, E, K,
                                                                   D, dxn);
  else
    k_ep_unpermute_router_dx<T, false><<<(unsigned)Tn, 256, 0, s>>>(v, top_i, slot_row, dz, wr, E,
                                                                    K, D, dxn);
  DOP_LAUNCHED(launches);
}
template void ep_unpermute_router_dx<bf16>(const EpView&, const int*, const int*, const float*,
                                           const bf16*, int64_t, int, int, int, float*,
                                           cudaStream_t, int64_t&);

}  // namespace dop
