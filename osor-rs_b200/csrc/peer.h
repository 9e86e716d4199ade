// Exchanges of a row-band group over peer memory (peer.cu).
#pragma once
#include <cstddef>

#include <cuda_runtime.h>

namespace osor {

constexpr int kMaxPeerRanks = 64;
constexpr int kPeerHandleBytes = 64;

struct PeerGroup;

// Allocates and clears this rank's arena on `device` and writes its IPC
// handle (kPeerHandleBytes) to `handle`; null on success, else the reason.
const char* peer_group_create(int device, int ranks, int rank, size_t halo_bytes,
                              size_t gather_bytes, PeerGroup** out, void* handle);
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

// dst[r] = rank r's src (bytes each), for every rank of the group.
const char* band_gather_check(const PeerGroup* g, size_t bytes);
cudaError_t band_gather_launch(PeerGroup* g, const void* src, size_t bytes, void* dst,
                               cudaStream_t s);

}  // namespace osor
