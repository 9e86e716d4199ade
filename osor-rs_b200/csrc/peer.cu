// Exchanges of a row-band group over peer memory (NVLink), replacing the
// NCCL send / receive and all-gather calls of the band split between layers.
//
// Every rank of a group owns one arena (cudaMalloc) that its neighbours write
// into: two halo-row slots from the rank above, two from the rank below, two
// all-gather slots per rank, one arrival flag per (kind, source rank) and the
// kernels' own counters. The arenas are shared through CUDA IPC handles, so a
// kernel writes a neighbour's slot with plain stores through the mapped
// pointer and then publishes the exchange's epoch in the neighbour's flag
// (system-scope release); the neighbour's kernel spins on its own flag
// (acquire, bounded) and copies the slot into place.
//
// Epochs live on the device (one counter per kind in the arena, advanced by
// the kernel that completes an exchange), so the kernels take the same
// arguments every time and a decode made of them can be captured once in a
// CUDA graph and replayed. Slots alternate by epoch parity: a rank writes a
// slot of epoch e + 2 only after it has seen the owner's flag of epoch e + 1,
// which the owner publishes after it has copied out epoch e.
//
// Reference counterpart: the band geometry of the column convolution
// (src/native/conv.rs:96-108, src/native/columns.rs:335-362); the exchange
// itself has no counterpart there (the reference runs its bands one after
// another on one device).
#include <cstdint>
#include <cstring>

#include <cuda_runtime.h>

#include "common.cuh"
#include "device_guard.h"
#include "peer.h"

namespace osor {
namespace {

constexpr int kHaloCtas = 16;  // per direction
constexpr int kHaloThreads = 256;
constexpr uint64_t kPeerWaitNs = 2000000000ull;

}  // namespace

ArenaLayout layout_of(size_t halo_bytes, size_t gather_bytes, size_t bulk_bytes, int ranks) {
  ArenaLayout l;
  l.halo_bytes = (halo_bytes + 255) / 256 * 256;
  l.gather_bytes = (gather_bytes + 255) / 256 * 256;
  l.bulk_bytes = (bulk_bytes + 255) / 256 * 256;
  l.from_up = 0;
  l.from_down = l.from_up + 2 * l.halo_bytes;
  l.gather = l.from_down + 2 * l.halo_bytes;
  l.bulk = l.gather + 2 * (size_t)kMaxPeerRanks * l.gather_bytes;
  l.flags_halo = l.bulk + (size_t)ranks * l.bulk_bytes;
  l.flags_gather = l.flags_halo + kMaxPeerRanks * sizeof(unsigned int);
  l.flags_bulk = l.flags_gather + kMaxPeerRanks * sizeof(unsigned int);
  l.counters = l.flags_bulk + kMaxPeerRanks * sizeof(unsigned int);
  // counters: halo epoch, gather epoch, halo phase-1 count, halo phase-3
  // count, bulk epoch, bulk phase-1 count, bulk phase-3 count
  l.total = l.counters + 8 * sizeof(unsigned long long);
  return l;
}

namespace {

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin until *flag >= epoch (wrapping compare), at most kPeerWaitNs.
__device__ bool wait_flag(const unsigned int* flag, unsigned int epoch) {
  const uint64_t t0 = global_timer_ns();
  while ((int)(ld_acquire_sys(flag) - epoch) < 0) {
    if (global_timer_ns() - t0 > kPeerWaitNs) {
      record_device_error(kDevWaitTimeout);
      return false;
    }
  }
  return true;
}

__device__ void copy16(uint4* dst, const uint4* src, long long n, long long first, long long step) {
  for (long long i = first; i < n; i += step) dst[i] = src[i];
}
__device__ void zero16(uint4* dst, long long n, long long first, long long step) {
  for (long long i = first; i < n; i += step) dst[i] = make_uint4(0, 0, 0, 0);
}

struct HaloArgs {
  uint8_t* x;             // extended band [rows + 2][row_bytes]
  long long row_bytes;
  int rows;
  uint8_t* local;         // this rank's arena
  uint8_t* up_arena;      // the rank above's arena (null at the image top)
  uint8_t* down_arena;    // the rank below's arena (null at the image bottom)
  int rank, up, down;     // group ranks (-1: none)
  ArenaLayout l;
};

// Grid: 2 x kHaloCtas CTAs. Phase 1: CTAs [0, kHaloCtas) copy row 1 into the
// rank above's from_down slot, the others row `rows` into the rank below's
// from_up slot. Phase 2: the last CTA to finish publishes the epoch in both
// neighbours' flags. Phase 3: every CTA waits for this rank's flags from its
// neighbours and copies its share of the received rows into rows 0 and
// rows + 1 (zeros at the image's top and bottom). The last CTA to finish
// advances the epoch.
__device__ __forceinline__ void halo_body(const HaloArgs& a, int nctas, int cta) {
  unsigned long long* counters = reinterpret_cast<unsigned long long*>(a.local + a.l.counters);
  unsigned int* flags = reinterpret_cast<unsigned int*>(a.local + a.l.flags_halo);
  const unsigned int epoch = (unsigned int)(*reinterpret_cast<volatile unsigned long long*>(&counters[0])) + 1u;
  const int parity = (int)(epoch & 1u);
  const long long n16 = a.row_bytes / 16;
  const bool to_up = cta < kHaloCtas;
  const int part = to_up ? cta : cta - kHaloCtas;
  const long long first = (long long)part * blockDim.x + threadIdx.x;
  const long long step = (long long)kHaloCtas * blockDim.x;
  // Phase 1.
  if (to_up && a.up_arena) {
    copy16(reinterpret_cast<uint4*>(a.up_arena + a.l.from_down + parity * a.l.halo_bytes),
           reinterpret_cast<const uint4*>(a.x + a.row_bytes), n16, first, step);
  } else if (!to_up && a.down_arena) {
    copy16(reinterpret_cast<uint4*>(a.down_arena + a.l.from_up + parity * a.l.halo_bytes),
           reinterpret_cast<const uint4*>(a.x + (long long)a.rows * a.row_bytes), n16, first,
           step);
  }
  // One system-scope fence per CTA after the barrier: it is cumulative over
  // the stores the barrier ordered before it.
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned long long target = (unsigned long long)epoch * nctas;
    last = atomicAdd(&counters[2], 1ull) + 1ull == target;
  }
  __syncthreads();
  // Phase 2.
  if (last && threadIdx.x == 0) {
    __threadfence_system();
    if (a.up_arena)
      st_release_sys(reinterpret_cast<unsigned int*>(a.up_arena + a.l.flags_halo) + a.rank, epoch);
    if (a.down_arena)
      st_release_sys(reinterpret_cast<unsigned int*>(a.down_arena + a.l.flags_halo) + a.rank,
                     epoch);
  }
  // Phase 3: this CTA's share of the row it receives from its direction's
  // neighbour (the rank above fills row 0, the rank below row rows + 1).
  __shared__ bool ok;
  if (threadIdx.x == 0) {
    const int src = to_up ? a.up : a.down;
    ok = src < 0 || wait_flag(flags + src, epoch);
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(a.x + (to_up ? 0 : (long long)(a.rows + 1) * a.row_bytes));
  if (ok) {
    if (to_up ? a.up < 0 : a.down < 0) {
      zero16(dst, n16, first, step);
    } else {
      const uint8_t* slot = a.local + (to_up ? a.l.from_up : a.l.from_down) + parity * a.l.halo_bytes;
      copy16(dst, reinterpret_cast<const uint4*>(slot), n16, first, step);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long target = (unsigned long long)epoch * nctas;
    if (atomicAdd(&counters[3], 1ull) + 1ull == target) {
      __threadfence();
      atomicAdd(&counters[0], 1ull);
    }
  }
}

__global__ void __launch_bounds__(kHaloThreads) band_halo_kernel(const HaloArgs a) {
  halo_body(a, gridDim.x, blockIdx.x);
}

struct GatherArgs {
  const uint8_t* src;
  long long bytes;
  uint8_t* dst;  // [ranks][bytes]
  uint8_t* local;
  uint8_t* peers[kMaxPeerRanks];
  int rank, ranks;
  ArenaLayout l;
};

// One CTA: write src into every peer's gather slot [parity][rank], publish
// the epoch, wait for every peer's, copy the slots into dst in rank order.
__device__ __forceinline__ void gather_body(const GatherArgs& a) {
  unsigned long long* counters = reinterpret_cast<unsigned long long*>(a.local + a.l.counters);
  unsigned int* flags = reinterpret_cast<unsigned int*>(a.local + a.l.flags_gather);
  const unsigned int epoch = (unsigned int)(*reinterpret_cast<volatile unsigned long long*>(&counters[1])) + 1u;
  const int parity = (int)(epoch & 1u);
  const long long n16 = a.bytes / 16;
  const size_t slot0 = a.l.gather + (size_t)parity * kMaxPeerRanks * a.l.gather_bytes;
  for (int r = 0; r < a.ranks; ++r) {
    if (r == a.rank) continue;
    copy16(reinterpret_cast<uint4*>(a.peers[r] + slot0 + (size_t)a.rank * a.l.gather_bytes),
           reinterpret_cast<const uint4*>(a.src), n16, threadIdx.x, blockDim.x);
  }
  copy16(reinterpret_cast<uint4*>(a.dst + (size_t)a.rank * a.bytes),
         reinterpret_cast<const uint4*>(a.src), n16, threadIdx.x, blockDim.x);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < a.ranks; ++r)
      if (r != a.rank)
        st_release_sys(reinterpret_cast<unsigned int*>(a.peers[r] + a.l.flags_gather) + a.rank,
                       epoch);
  }
  __shared__ bool ok;
  if (threadIdx.x == 0) {
    bool good = true;
    for (int r = 0; r < a.ranks && good; ++r)
      if (r != a.rank) good = wait_flag(flags + r, epoch);
    ok = good;
  }
  __syncthreads();
  if (ok) {
    for (int r = 0; r < a.ranks; ++r) {
      if (r == a.rank) continue;
      copy16(reinterpret_cast<uint4*>(a.dst + (size_t)r * a.bytes),
             reinterpret_cast<const uint4*>(a.local + slot0 + (size_t)r * a.l.gather_bytes), n16,
             threadIdx.x, blockDim.x);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(&counters[1], 1ull);
  }
}

__global__ void __launch_bounds__(256) band_gather_kernel(const GatherArgs a) { gather_body(a); }

// The halo exchange (CTAs [0, 2 kHaloCtas)) and the all-gather (the last CTA)
// of one layer in one launch, so the ranks meet once.
__global__ void __launch_bounds__(kHaloThreads) band_halo_gather_kernel(const HaloArgs h,
                                                                        const GatherArgs g) {
  if (blockIdx.x < 2 * kHaloCtas)
    halo_body(h, 2 * kHaloCtas, blockIdx.x);
  else
    gather_body(g);
}

constexpr int kBulkCtas = 64;

struct BulkArgs {
  const uint8_t* src;
  long long bytes;
  uint8_t* local;
  uint8_t* peers[kMaxPeerRanks];
  int rank, ranks;
  ArenaLayout l;
};

// Grid: kBulkCtas CTAs. Every CTA stores its share of src into slot [rank] of
// every rank's arena (this rank's included); the last CTA to finish
// publishes the epoch in every peer's flag; every CTA then waits for all
// peers' flags; the last CTA to finish advances the epoch.
__global__ void __launch_bounds__(256) band_bulk_kernel(const BulkArgs a) {
  unsigned long long* counters = reinterpret_cast<unsigned long long*>(a.local + a.l.counters);
  unsigned int* flags = reinterpret_cast<unsigned int*>(a.local + a.l.flags_bulk);
  const unsigned int epoch = (unsigned int)(*reinterpret_cast<volatile unsigned long long*>(&counters[4])) + 1u;
  const long long n16 = a.bytes / 16;
  const long long first = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (int r = 0; r < a.ranks; ++r)
    copy16(reinterpret_cast<uint4*>(a.peers[r] + a.l.bulk + (size_t)a.rank * a.l.bulk_bytes),
           reinterpret_cast<const uint4*>(a.src), n16, first, step);
  // One system-scope fence per CTA after the barrier: it is cumulative over
  // the stores the barrier ordered before it.
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned long long target = (unsigned long long)epoch * gridDim.x;
    last = atomicAdd(&counters[5], 1ull) + 1ull == target;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < a.ranks; ++r)
      if (r != a.rank)
        st_release_sys(reinterpret_cast<unsigned int*>(a.peers[r] + a.l.flags_bulk) + a.rank,
                       epoch);
  }
  if (threadIdx.x == 0) {
    for (int r = 0; r < a.ranks; ++r)
      if (r != a.rank && !wait_flag(flags + r, epoch)) break;
    const unsigned long long target = (unsigned long long)epoch * gridDim.x;
    if (atomicAdd(&counters[6], 1ull) + 1ull == target) {
      __threadfence();
      atomicAdd(&counters[4], 1ull);
    }
  }
}

}  // namespace

const char* peer_group_create(int device, int ranks, int rank, size_t halo_bytes,
                              size_t gather_bytes, size_t bulk_bytes, PeerGroup** out,
                              void* handle) {
  *out = nullptr;
  if (ranks < 1 || ranks > kMaxPeerRanks || rank < 0 || rank >= ranks)
    return "peer group: 1..64 ranks and a rank inside the group";
  if (halo_bytes == 0 || gather_bytes == 0 || halo_bytes > (1ull << 30) ||
      gather_bytes > (1ull << 20) || bulk_bytes > (1ull << 34))
    return "peer group: halo slots up to 1 GiB, gather slots up to 1 MiB, bulk parts up to 16 GiB";
  PeerGroup* g = new PeerGroup;
  g->device = device;
  g->ranks = ranks;
  g->rank = rank;
  g->l = layout_of(halo_bytes, gather_bytes, bulk_bytes, ranks);
  int prev = 0;
  cudaGetDevice(&prev);
  const char* err = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) {
    err = "peer group: cannot select the device";
  } else if (cudaMalloc(&g->arena, g->l.total) != cudaSuccess) {
    g->arena = nullptr;
    err = "peer group: cannot allocate the arena";
  } else if (cudaMemset(g->arena, 0, g->l.total) != cudaSuccess ||
             cudaDeviceSynchronize() != cudaSuccess) {
    err = "peer group: cannot clear the arena";
  } else {
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, g->arena) != cudaSuccess) {
      err = "peer group: cannot export the arena";
    } else {
      static_assert(sizeof(h) <= kPeerHandleBytes, "IPC handle size");
      std::memset(handle, 0, kPeerHandleBytes);
      std::memcpy(handle, &h, sizeof(h));
      g->peers[rank] = g->arena;
    }
  }
  if (err) {
    if (g->arena) cudaFree(g->arena);
    delete g;
    cudaSetDevice(prev);
    return err;
  }
  cudaSetDevice(prev);
  *out = g;
  return nullptr;
}

const char* peer_group_open(PeerGroup* g, int peer, const void* handle) {
  if (peer < 0 || peer >= g->ranks) return "peer group: rank outside the group";
  if (peer == g->rank) return nullptr;
  if (g->opened[peer]) return "peer group: rank already opened";
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return "peer group: cannot map the peer's arena";
  g->peers[peer] = static_cast<uint8_t*>(p);
  g->opened[peer] = true;
  return nullptr;
}

void peer_group_destroy(PeerGroup* g) {
  if (!g) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < g->ranks; ++r)
    if (g->opened[r]) cudaIpcCloseMemHandle(g->peers[r]);
  if (g->arena) cudaFree(g->arena);
  cudaSetDevice(prev);
  delete g;
}

const char* band_halo_check(const PeerGroup* g, long long row_bytes, int rows) {
  if (rows < 1) return "band halo: at least one band row";
  if (row_bytes <= 0 || row_bytes % 16 != 0) return "band halo: rows of a multiple of 16 bytes";
  if ((size_t)row_bytes > g->l.halo_bytes) return "band halo: rows wider than the halo slots";
  const int up = g->rank - 1, down = g->rank + 1 < g->ranks ? g->rank + 1 : -1;
  if ((up >= 0 && !g->peers[up]) || (down >= 0 && !g->peers[down]))
    return "band halo: a neighbour's arena is not mapped";
  return nullptr;
}

namespace {
HaloArgs halo_args(PeerGroup* g, void* x, long long row_bytes, int rows) {
  HaloArgs a;
  a.x = static_cast<uint8_t*>(x);
  a.row_bytes = row_bytes;
  a.rows = rows;
  a.local = g->arena;
  a.rank = g->rank;
  a.up = g->rank - 1;
  a.down = g->rank + 1 < g->ranks ? g->rank + 1 : -1;
  a.up_arena = a.up >= 0 ? g->peers[a.up] : nullptr;
  a.down_arena = a.down >= 0 ? g->peers[a.down] : nullptr;
  a.l = g->l;
  return a;
}
GatherArgs gather_args(PeerGroup* g, const void* src, size_t bytes, void* dst) {
  GatherArgs a;
  a.src = static_cast<const uint8_t*>(src);
  a.bytes = (long long)bytes;
  a.dst = static_cast<uint8_t*>(dst);
  a.local = g->arena;
  for (int r = 0; r < kMaxPeerRanks; ++r) a.peers[r] = r < g->ranks ? g->peers[r] : nullptr;
  a.rank = g->rank;
  a.ranks = g->ranks;
  a.l = g->l;
  return a;
}
}  // namespace

cudaError_t band_halo_launch(PeerGroup* g, void* x, long long row_bytes, int rows,
                             cudaStream_t s) {
  band_halo_kernel<<<2 * kHaloCtas, kHaloThreads, 0, s>>>(halo_args(g, x, row_bytes, rows));
  return cudaGetLastError();
}

cudaError_t band_halo_gather_launch(PeerGroup* g, void* x, long long row_bytes, int rows,
                                    const void* src, size_t bytes, void* dst, cudaStream_t s) {
  band_halo_gather_kernel<<<2 * kHaloCtas + 1, kHaloThreads, 0, s>>>(
      halo_args(g, x, row_bytes, rows), gather_args(g, src, bytes, dst));
  return cudaGetLastError();
}

const char* band_gather_check(const PeerGroup* g, size_t bytes) {
  if (bytes == 0 || bytes % 16 != 0) return "band gather: a multiple of 16 bytes";
  if (bytes > g->l.gather_bytes) return "band gather: larger than the gather slots";
  for (int r = 0; r < g->ranks; ++r)
    if (!g->peers[r]) return "band gather: a rank's arena is not mapped";
  return nullptr;
}

const char* band_bulk_check(const PeerGroup* g, size_t bytes) {
  if (bytes == 0 || bytes % 16 != 0) return "band bulk gather: a multiple of 16 bytes";
  if (bytes > g->l.bulk_bytes) return "band bulk gather: larger than the bulk slots";
  for (int r = 0; r < g->ranks; ++r)
    if (!g->peers[r]) return "band bulk gather: a rank's arena is not mapped";
  return nullptr;
}

cudaError_t band_bulk_launch(PeerGroup* g, const void* src, size_t bytes, cudaStream_t s) {
  BulkArgs a;
  a.src = static_cast<const uint8_t*>(src);
  a.bytes = (long long)bytes;
  a.local = g->arena;
  for (int r = 0; r < kMaxPeerRanks; ++r) a.peers[r] = r < g->ranks ? g->peers[r] : nullptr;
  a.rank = g->rank;
  a.ranks = g->ranks;
  a.l = g->l;
  band_bulk_kernel<<<kBulkCtas, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t band_gather_launch(PeerGroup* g, const void* src, size_t bytes, void* dst,
                               cudaStream_t s) {
  band_gather_kernel<<<1, 256, 0, s>>>(gather_args(g, src, bytes, dst));
  return cudaGetLastError();
}

}  // namespace osor
