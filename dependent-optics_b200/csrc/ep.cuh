// ep.cuh — expert-parallel exchange of the Mixtral block lens (ep.cu).
#pragma once

#include "kernels.cuh"

namespace dop {

constexpr int kEpMaxWorld = 8;   // ranks of one expert-parallel group
constexpr int kEpBarriers = 4;   // flag barriers per step

// What the exchange kernels need to know about this rank's workspace and
// its peers' (passed by value).  Every pointer is into this rank's block
// workspace; peers[s] is rank s's workspace base as mapped here (peers[rank]
// is this rank's own base), so rank s's copy of a buffer is at the same
// offset from peers[s].
struct EpView {
  int rank = 0, world = 1, local = 0;  // local = experts per rank
  int recv_tiles = 0;                  // receive capacity / kRowAlign
  int64_t recv_cap = 0;                // receive capacity in rows
  char* const* peers = nullptr;        // device array [world]
  unsigned* flags = nullptr;           // [kEpBarriers][kEpMaxWorld]
  const int* seg_off = nullptr;        // this rank's padded expert segments [E+1]
  const int* row_token = nullptr;      // this rank's sorted row -> token
  int* send_off = nullptr;             // [E] start of (expert, this rank) at the owner
  int* recv_seg_off = nullptr;         // [local+1] receive segments per local expert
  int* recv_tile_expert = nullptr;     // [recv_tiles] local expert of a receive tile, -1 past the end
  int* recv_tile_src = nullptr;        // [recv_tiles] source rank of the tile
  int* recv_tile_row0 = nullptr;       // [recv_tiles] source row of the tile's first row
  bf16* xr = nullptr;                  // receive rows of the forward dispatch
  float* outr = nullptr;               // expert outputs of the receive rows
  float* dxpr = nullptr;               // expert-input cotangents of the receive rows
};

void ep_barrier(const EpView& v, int k, unsigned epoch, cudaStream_t s, int64_t& launches);
void ep_layout(const EpView& v, int E, cudaStream_t s, int64_t& launches);
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

}  // namespace dop
