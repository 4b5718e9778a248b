// ep.cuh — expert-parallel exchange of the Mixtral block lens (ep.cu).
#pragma once

#include "kernels.cuh"

namespace dop {

constexpr int kEpMaxWorld = 8;   // ranks of one expert-parallel group
constexpr int kEpBarriers = 5;   // flag barriers per step

// What the exchange kernels need to know about this rank's workspace and
// its peers' (passed by value).  Every pointer is into this rank's block
// workspace; peers[s] is rank s's workspace base as mapped here (peers[rank]
// is this rank's own base), so rank s's copy of a buffer is at the same
// offset from peers[s].
//
// Rows are placed by a plan that every rank computes from the same inputs
// (ep_layout): the expert-major sequence of every (expert, source) piece of
// routed rows is cut into `world` near-equal chunks, rank d processing global
// rows [bounds[d], bounds[d + 1]).  A cut snaps to an expert boundary when
// one is near, so balanced routing keeps each expert on one rank; a hot
// expert is split over several.  Rank r still owns the adjoint of experts
// [r * local, (r + 1) * local): the partial weight adjoints that other ranks
// computed for them (dw_help) are added into the owner's dparams.
struct EpView {
  int rank = 0, world = 1, local = 0;  // local = experts whose adjoint this rank owns
  int E = 0;                           // experts
  int recv_tiles = 0;                  // receive capacity / kRowAlign
  int64_t recv_cap = 0;                // receive capacity in rows
  int64_t expert_stride = 0;           // floats of one expert's gate, up and down
  char* const* peers = nullptr;        // device array [world]
  unsigned* flags = nullptr;           // [kEpBarriers][kEpMaxWorld]
  const int* seg_off = nullptr;        // this rank's padded expert segments [E+1]
  const int* row_token = nullptr;      // this rank's sorted row -> token
  int* piece_pos = nullptr;            // [E] global position of (expert e, this rank as source)
  int* bounds = nullptr;               // [world+1] global rows of each rank's chunk
  int* recv_seg_off = nullptr;         // [E+1] receive segment of each expert on this rank
  int* own_end = nullptr;              // [E] end of expert e's segment if this rank owns e, else its start
  int* help_end = nullptr;             // [E] the same for the experts this rank does not own
  int* helpers = nullptr;              // [E] bit d: rank d != owner processed rows of e
  int* recv_tile_expert = nullptr;     // [recv_tiles] expert of a receive tile, -1 past the end
  int* recv_tile_src = nullptr;        // [recv_tiles] source rank of the tile
  int* recv_tile_row0 = nullptr;       // [recv_tiles] source row of the tile's first row
  bf16* xr = nullptr;                  // receive rows of the forward dispatch
  float* outr = nullptr;               // expert outputs of the receive rows
  float* dxpr = nullptr;               // expert-input cotangents of the receive rows
  float* dw_help = nullptr;            // [E][expert_stride] partial adjoints of other ranks' experts
};

void ep_barrier(const EpView& v, int k, unsigned epoch, cudaStream_t s, int64_t& launches);
void ep_layout(const EpView& v, cudaStream_t s, int64_t& launches);
void ep_gather_tokens(const EpView& v, const bf16* xn2, int D, cudaStream_t s, int64_t& launches);
void ep_gather_rows(const EpView& v, const bf16* dO, bf16* dst, int D, cudaStream_t s,
                    int64_t& launches);
void ep_combine(const EpView& v, const float* mid, const int* top_i, const int* slot_row,
                const float* top_w, int64_t T, int K, int D, float* out, float* y, cudaStream_t s,
                int64_t& launches);
template <typename T>
void ep_unpermute_router_dx(const EpView& v, const int* top_i, const int* slot_row,
                            const float* dz, const T* wr, int64_t Tn, int E, int K, int D,
                            float* dxn, cudaStream_t s, int64_t& launches);
// Owner side of the adjoint: dP_experts[e] += the helpers' dw_help[e] (rank
// order) for each expert e this rank owns.  dP_experts = dparams + gate0.
void ep_reduce_adjoint(const EpView& v, float* dP_experts, cudaStream_t s, int64_t& launches);

}  // namespace dop
