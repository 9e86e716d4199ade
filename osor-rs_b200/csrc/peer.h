// Exchanges of a row-band group over peer memory (peer.cu).
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace osor {

constexpr int kMaxPeerRanks = 64;
constexpr int kPeerHandleBytes = 64;

// Byte offsets of one rank's arena: halo slots [2] from the rank above and
// [2] from the rank below, all-gather slots [2][kMaxPeerRanks], bulk slots
// [ranks], arrival flags per kind and source rank, the kernels' counters.
struct ArenaLayout {
  size_t halo_bytes, gather_bytes, bulk_bytes;
  size_t from_up, from_down, gather, bulk, flags_halo, flags_gather, flags_bulk, counters, total;
};
ArenaLayout layout_of(size_t halo_bytes, size_t gather_bytes, size_t bulk_bytes, int ranks);

struct PeerGroup {
  int device = 0, ranks = 0, rank = 0;
  ArenaLayout l{};
  uint8_t* arena = nullptr;
  uint8_t* peers[kMaxPeerRanks] = {};
  bool opened[kMaxPeerRanks] = {};
};

// Allocates and clears this rank's arena on `device` and writes its IPC
// handle (kPeerHandleBytes) to `handle`; null on success, else the reason.
// bulk_bytes: the largest per-rank part of a bulk all-gather (0: none).
const char* peer_group_create(int device, int ranks, int rank, size_t halo_bytes,
                              size_t gather_bytes, size_t bulk_bytes, PeerGroup** out,
                              void* handle);
// Maps rank `peer`'s arena from its handle.
const char* peer_group_open(PeerGroup* g, int peer, const void* handle);
// Waits for the device, unmaps the peers' arenas and frees this rank's.
void peer_group_destroy(PeerGroup* g);

// Halo rows of an extended band x [rows + 2][row_bytes]: row 1 goes to the
// rank above (its row rows + 1), row `rows` to the rank below (its row 0);
// rows 0 and rows + 1 are filled from the neighbours, zeros at the image's
// top and bottom.
const char* band_halo_check(const PeerGroup* g, long long row_bytes, int rows);
cudaError_t band_halo_launch(PeerGroup* g, void* x, long long row_bytes, int rows,
                             cudaStream_t s);

// band_halo and band_gather of one layer in one launch (one rendezvous of the
// ranks instead of two); the checks of both apply.
cudaError_t band_halo_gather_launch(PeerGroup* g, void* x, long long row_bytes, int rows,
                                    const void* src, size_t bytes, void* dst, cudaStream_t s);

// dst[r] = rank r's src (bytes each), for every rank of the group.
const char* band_gather_check(const PeerGroup* g, size_t bytes);
cudaError_t band_gather_launch(PeerGroup* g, const void* src, size_t bytes, void* dst,
                               cudaStream_t s);

// Bulk all-gather into this rank's arena: afterwards bulk_slots(g) +
// r * g->l.bulk_bytes holds rank r's src for every rank (contiguous parts when
// bytes equals the slot size, a multiple of 256). The slots are single buffered: between
// two bulk gathers every rank must have passed an exchange that waits on every
// other rank (a band_gather), so that no rank still reads the previous one.
const char* band_bulk_check(const PeerGroup* g, size_t bytes);
cudaError_t band_bulk_launch(PeerGroup* g, const void* src, size_t bytes, cudaStream_t s);
inline uint8_t* bulk_slots(const PeerGroup* g) { return g->arena + g->l.bulk; }

}  // namespace osor
