// Fused single-head attention softmax(Q K^T) V for the VAE mid-block at width
// D = 512 on CTA pairs (clusters of two), with no N^2 buffer and no repeated
// Q K^T.
//
// One task = one image and 128 query rows, taken by both CTAs of a cluster.
// Keys go in tiles of 256; CTA r computes the scores of keys r*128 .. r*128+127
// of every tile, S_r = Q K_r^T (M = 128, N = 128, K = 512), into one of two
// TMEM score buffers, and accumulates output columns r*256 .. r*256+255,
// O_r += P V[:, r*256 ..] (M = 128, N = 256, K = 256 keys), in TMEM. Per tile:
//   * each CTA's four softmax warps (one query row per thread) take their
//     128 scores' row maximum and send it to the other CTA (distributed shared
//     memory); both then hold the tile maximum and take identical running-
//     maximum decisions (the maximum moves, and O is rescaled, only when it
//     grows by more than 2^8, so P <= 256);
//   * each CTA writes its half of P = 2^(S log2 e - m) as 16-bit K-major tiles
//     into its own and the other CTA's shared memory; the PV MMAs read the
//     whole 128 x 256 P from local shared memory;
//   * each CTA keeps the fp32 row sum of its own P half; the halves are added
//     once per task before the output is normalised and stored.
// The two score buffers are filled together: each shared-memory stage carries
// one 64-wide chunk of Q and the matching K chunks of two tiles, so Q crosses
// from L2 once per two tiles (the stages' load latency, not the tensor core,
// bounds this kernel). The scores of tiles j + 2 and j + 3 are computed while
// the softmax warps work on tiles j and j + 1, and P V of each tile follows
// its softmax.
//
// Roles (224 threads per CTA): warp 0 TMA producer of the Q and K chunks,
// warp 6 TMA producer of the V^T chunks of this CTA's output half (two
// producers, so that neither stream waits behind the other's ring), warp 1
// TMEM allocator and MMA issuer, which issues each score chunk and each P V
// chunk as soon as its operands have arrived, warps 2..5 softmax and output
// epilogue. All waits are bounded; a CTA that
// gives up sets its abort flag, and the cluster barrier at the end keeps
// either CTA from leaving while the other may still write into it.
//
// Reference counterpart: Attention::forward_checked / attend_with
// (src/native/vae_encoder.rs:237-340, src/native/attention.rs:27-84).
#include <atomic>

#include "attn_fa.h"
#include "common.cuh"
#include "device_guard.h"

namespace osor {
namespace {

constexpr int kRows = 128;                  // query rows per task
constexpr int kTileKeys = 256;              // keys per tile (both CTAs)
constexpr int kOwnKeys = 128;               // keys per tile and CTA
constexpr int kDim = 512;
constexpr int kDHalf = 256;                 // output columns per CTA
constexpr int kDChunk = 64;
constexpr int kDChunks = kDim / kDChunk;    // 8
constexpr int kQBytes = kRows * kDChunk * 2;        // 16 KB
constexpr int kKBytes = kOwnKeys * kDChunk * 2;     // 16 KB
constexpr int kAStage = kQBytes + 2 * kKBytes;      // 48 KB: a Q chunk and the K chunks of two tiles
constexpr int kVStage = kDHalf * 64 * 2;            // V^T chunk: 256 rows x 64 keys (32 KB)
constexpr int kPBlock = kRows * 64 * 2;             // P: 128 rows x 64 keys (16 KB)
constexpr int kAStages = 2;
constexpr int kVStages = 2;
constexpr int kThreads = 224;
// Exchange area: the peer's row maxima [2][128], the peer's row sums [128],
// and this CTA's row maxima staged for the copy to the peer [2][128].
constexpr int kExBytes = (2 * kRows + kRows + 2 * kRows) * 4;
// No alignment slack: the dynamic window of a kernel without static shared
// memory starts 1024-byte aligned (checked in the kernel).
constexpr int kSmem = kAStages * kAStage + kVStages * kVStage + 4 * kPBlock + kExBytes + 256;
static_assert(kSmem <= 227 * 1024, "shared memory");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;
constexpr uint32_t kTmemO = 256;                    // O half at columns 256..511

struct PairParams {
  int n_q, n_kv, batch;
  int tiles;  // n_kv / 256 (even)
  int tasks;  // batch * n_q / 128
  void* out;
  long long ld_out;
};

__device__ void pair_drain(uint64_t* bars, int n, int stage, uint32_t phase) {
  for (int s = 0; s < n; ++s) {
    int st = stage - 1 - s;
    uint32_t ph = phase;
    if (st < 0) {
      st += n;
      ph ^= 1;
    }
    const uint32_t addr = smem_u32(&bars[st]);
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(addr, ph) && global_timer_ns() - t0 < kWaitLimitNs) {
    }
  }
}

template <int D>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_vt, const PairParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The 128-byte swizzled tiles need 1024-byte aligned addresses.
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0) record_device_error(kDevBadShape);
    return;
  }
  uint8_t* ring_a = smem_raw;
  uint8_t* ring_v = ring_a + kAStages * kAStage;
  uint8_t* pbuf = ring_v + kVStages * kVStage;
  float* mx = reinterpret_cast<float*>(pbuf + 4 * kPBlock);  // [2][128], written by the peer
  float* lx = mx + 2 * kRows;                                 // [128], written by the peer
  float* mstage = lx + kRows;                                 // [2][128], copied to the peer
  uint64_t* a_full = reinterpret_cast<uint64_t*>(mstage + 2 * kRows);
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* v_full = a_empty + kAStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_full = v_empty + kVStages;  // [2]
  uint64_t* s_free = s_full + 2;          // [2]
  uint64_t* mx_ready = s_free + 2;        // [2]
  uint64_t* p_ready = mx_ready + 2;
  uint64_t* p_free = p_ready + 1;
  uint64_t* o_free = p_free + 1;
  uint64_t* l_ready = o_free + 1;
  uint64_t* drain = l_ready + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);    // the four softmax warps
      // Four local arrivals (one per softmax warp, each expecting the 128
      // bytes of row maxima that the peer's warp of the same rows copies in).
      mbar_init(&mx_ready[b], 4);
    }
    // Four local arrivals (each softmax warp after writing its P rows, each
    // expecting the 8 KB of P rows that the peer's warp copies in).
    mbar_init(p_ready, 4);
    mbar_init(p_free, 2);   // this CTA's and the peer's PV commit
    mbar_init(o_free, 4);
    mbar_init(l_ready, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_vt);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int qtiles = p.n_q / kRows;
  const int cluster_id = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int as = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int t = cluster_id; t < p.tasks && ok; t += clusters) {
        const int qt = t % qtiles;
        const int b = t / qtiles;
        const int qrow = b * p.n_q + qt * kRows;
        for (int j = 0; j < p.tiles && ok; j += 2) {
          // One Q chunk serves the scores of two tiles, j and j + 1.
          const int krow = b * p.n_kv + j * kTileKeys + (int)rank * kOwnKeys;
          for (int dc = 0; dc < kDChunks; ++dc) {
            if (!mbar_wait(&a_empty[as], aph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&a_full[as], kAStage);
            uint8_t* st = ring_a + as * kAStage;
            tma_load_2d(st, &tmap_q, &a_full[as], dc * kDChunk, qrow);
            tma_load_2d(st + kQBytes, &tmap_k, &a_full[as], dc * kDChunk, krow);
            tma_load_2d(st + kQBytes + kKBytes, &tmap_k, &a_full[as], dc * kDChunk,
                        krow + kTileKeys);
            if (++as == kAStages) {
              as = 0;
              aph ^= 1;
            }
          }
        }
      }
      if (!ok) pair_drain(a_full, kAStages, as, aph);
    }
  } else if (warp == 6) {
    if (lane == 0) {
      // ---------------------------------------------------------- V^T producer
      int vs = 0;
      uint32_t vph = 0;
      bool ok = true;
      for (int t = cluster_id; t < p.tasks && ok; t += clusters) {
        const int b = t / qtiles;
        for (int j = 0; j < p.tiles && ok; ++j) {
          for (int c = 0; c < kTileKeys / 64; ++c) {
            if (!mbar_wait(&v_empty[vs], vph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&v_full[vs], kVStage);
            tma_load_3d(ring_v + vs * kVStage, &tmap_vt, &v_full[vs], j * kTileKeys + c * 64,
                        (int)rank * kDHalf, b);
            if (++vs == kVStages) {
              vs = 0;
              vph ^= 1;
            }
          }
        }
      }
      if (!ok) pair_drain(v_full, kVStages, vs, vph);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f32acc(kRows, kOwnKeys, Elem<D>::kUmmaFormat);
      constexpr uint32_t idesc_o = umma_idesc_f32acc(kRows, kDHalf, Elem<D>::kUmmaFormat);
      const uint32_t tmem_o = tmem_base + kTmemO;
      int as = 0, vs = 0;
      uint32_t aph = 0, vph = 0;
      long long u = 0;   // global score-tile counter (this CTA)
      long long pv = 0;  // global PV counter
      int task_idx = 0;
      bool ok = true, issued = false;
      // Iteration i of a task issues the scores of tiles 2i and 2i + 1 into
      // the two score buffers (kDChunks A stages, each a Q chunk with both
      // tiles' K chunks) and O += P V of tiles 2i - 2 and 2i - 1 (four V^T
      // chunks each), each chunk as soon as its operands have arrived, P V
      // first when both can go: the two rings' loads overlap instead of one
      // waiting behind the other. The barriers are polled with test_wait
      // (which never suspends the thread); a poll that finds nothing ready
      // for kWaitLimitNs gives up like the other waits.
      uint64_t t_idle = 0;
      const int pairs = p.tiles / 2;
      for (int t = cluster_id; t < p.tasks && ok; t += clusters, ++task_idx) {
        for (int i = 0; i <= pairs && ok; ++i) {
          int sc = i < pairs ? 0 : kDChunks;  // A stages issued
          int pc = i > 0 ? 0 : 8;             // P V chunks issued (two tiles)
          bool s_gate = false, p_gate = false;
          const uint32_t s_par = (uint32_t)(((u >> 1) & 1) ^ 1);
          while (sc < kDChunks || pc < 8) {
            bool progress = false;
            if (pc < 8) {
              if (!p_gate) {
                // The first P V of a task overwrites O: the previous task's
                // epilogue must have read it. P of the tile must be complete
                // in this CTA (its rows and the peer's).
                const bool o_ok = !(i == 1 && pc == 0 && task_idx > 0) ||
                                  mbar_test_wait(smem_u32(o_free), (uint32_t)((task_idx - 1) & 1));
                if (o_ok && mbar_test_wait_cluster(smem_u32(p_ready), (uint32_t)(pv & 1))) {
                  p_gate = true;
                  tc_fence_after();
                }
              }
              if (p_gate && mbar_test_wait(smem_u32(&v_full[vs]), vph)) {
                tc_fence_after();
                const int c = pc & 3;
                const uint32_t a_addr = smem_u32(pbuf + c * kPBlock);
                const uint32_t b_addr = smem_u32(ring_v + vs * kVStage);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  umma_bf16(tmem_o, sw128_kmajor_desc(a_addr + k * 32),
                            sw128_kmajor_desc(b_addr + k * 32), idesc_o,
                            !(i == 1 && pc == 0 && k == 0));
                issued = true;
                umma_commit(&v_empty[vs]);
                if (++vs == kVStages) {
                  vs = 0;
                  vph ^= 1;
                }
                if ((++pc & 3) == 0) {
                  // P and O are free once these MMAs complete, here and in the peer.
                  umma_commit_multicast(p_free, 0x3);
                  ++pv;
                  p_gate = false;
                }
                progress = true;
              }
            }
            if (sc < kDChunks) {
              // The softmax warps have read both buffers' previous scores.
              if (!s_gate && mbar_test_wait(smem_u32(&s_free[0]), s_par) &&
                  mbar_test_wait(smem_u32(&s_free[1]), s_par)) {
                s_gate = true;
                tc_fence_after();
              }
              if (s_gate && mbar_test_wait(smem_u32(&a_full[as]), aph)) {
                tc_fence_after();
                const uint32_t q_addr = smem_u32(ring_a + as * kAStage);
#pragma unroll
                for (int tb = 0; tb < 2; ++tb) {
                  const uint32_t k_addr = q_addr + kQBytes + tb * kKBytes;
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    umma_bf16(tmem_base + tb * kOwnKeys, sw128_kmajor_desc(q_addr + k * 32),
                              sw128_kmajor_desc(k_addr + k * 32), idesc_s, (sc | k) != 0);
                  if (sc == kDChunks - 1) umma_commit(&s_full[tb]);
                }
                issued = true;
                umma_commit(&a_empty[as]);
                if (++as == kAStages) {
                  as = 0;
                  aph ^= 1;
                }
                ++sc;
                progress = true;
              }
            }
            if (progress) {
              t_idle = 0;
            } else if (*abort_flag) {
              ok = false;
            } else if (t_idle == 0) {
              t_idle = global_timer_ns();
            } else if (global_timer_ns() - t_idle > kWaitLimitNs) {
              record_device_error(kDevWaitTimeout);
              *abort_flag = 1;
              ok = false;
            }
            if (!ok) break;
          }
          if (i < pairs) u += 2;
        }
      }
      if (!ok && issued) {
        umma_commit(drain);
        const uint32_t addr = smem_u32(drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(addr, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------- softmax + epilogue
    const int quad = warp & 3;          // warps 2..5 read TMEM lane quadrants 2, 3, 0, 1
    const int row = quad * 32 + lane;   // query row within the task
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tmem_o = tmem_base + kTmemO;
    const uint32_t peer_mx = map_to_rank(smem_u32(mx), peer);
    const uint32_t peer_lx = map_to_rank(smem_u32(lx), peer);
    const uint32_t peer_pbuf = map_to_rank(smem_u32(pbuf), peer);
    const uint32_t peer_mx_ready[2] = {map_to_rank(smem_u32(&mx_ready[0]), peer),
                                       map_to_rank(smem_u32(&mx_ready[1]), peer)};
    const uint32_t peer_p_ready = map_to_rank(smem_u32(p_ready), peer);
    const uint32_t peer_l_ready = map_to_rank(smem_u32(l_ready), peer);
    long long u = 0;
    int task_idx = 0;
    bool ok = true;
    for (int t = cluster_id; t < p.tasks && ok; t += clusters, ++task_idx) {
      const int qt = t % qtiles;
      const int b = t / qtiles;
      float m = 0.0f, l = 0.0f;
      for (int j = 0; j < p.tiles; ++j, ++u) {
        const int buf = (int)(u & 1);
        const uint32_t par = (uint32_t)((u >> 1) & 1);
        // Waits are agreed per warp (a lane that gave up takes its warp
        // along), so the warp-collective tcgen05.ld / st below always run
        // with all 32 lanes.
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[buf], par, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // This row's 128 scores stay in registers for both passes.
        const uint32_t s_tmem = tmem_base + buf * kOwnKeys + lane_off;
        float sv[kOwnKeys];
        {
          uint32_t r[kOwnKeys];
#pragma unroll
          for (int c = 0; c < kOwnKeys / 32; ++c)
            tmem_load_32x32b_x32(s_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < kOwnKeys; ++k) sv[k] = __uint_as_float(r[k]);
        }
        // The scores have been read: the buffer takes tile u + 2.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[buf]);
        // Row maximum as a tree of eight chains (one chain of 128 dependent
        // max operations would put its latency on every tile's critical path).
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = sv[i];
#pragma unroll
        for (int k = 8; k < kOwnKeys; ++k) acc[k & 7] = fmaxf(acc[k & 7], sv[k]);
#pragma unroll
        for (int w = 4; w > 0; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) acc[i] = fmaxf(acc[i], acc[i + w]);
        const float mloc = acc[0] * kLog2e;
        // Row maxima to the peer: staged, then one bulk copy per warp that
        // completes its 128 bytes on the peer's mx_ready.
        mstage[buf * kRows + row] = mloc;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&mx_ready[buf], 128);
          bulk_copy_to_cluster(peer_mx + (uint32_t)((buf * kRows + quad * 32) * 4),
                               mstage + buf * kRows + quad * 32, 128, peer_mx_ready[buf]);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&mx_ready[buf], par, abort_flag))) {
          ok = false;
          break;
        }
        const float mt = fmaxf(mloc, mx[buf * kRows + row]);
        // The running-maximum decision and this tile's probabilities need
        // only the scores: they are computed while the previous tile's PV
        // still runs, and only the stores into P (and a rescale of O) wait
        // for it.
        float f = 1.0f;
        bool rescale = false;
        if (j == 0) {
          m = mt;
          l = 0.0f;
        } else {
          const bool grow = mt > m + kRescaleLog2;
          // tcgen05.ld / st are warp-collective (.sync.aligned): the warp
          // rescales together when any of its rows needs it, each row with
          // its own factor (1 for rows whose maximum stays).
          rescale = __any_sync(0xffffffffu, grow);
          if (grow) {
            f = ex2_approx(m - mt);
            m = mt;
          }
          l *= f;
        }
        // P = 2^(S log2 e - m) for this CTA's keys, packed 16-bit.
        float lsum = 0.0f;
        uint32_t pk[kOwnKeys / 2];
#pragma unroll
        for (int k = 0; k < kOwnKeys / 2; ++k) {
          const float p0 = ex2_approx(fmaf(sv[2 * k], kLog2e, -m));
          const float p1 = ex2_approx(fmaf(sv[2 * k + 1], kLog2e, -m));
          lsum += p0 + p1;
          pk[k] = Elem<D>::pack(p0, p1);
        }
        l += lsum;
        // P (and, for a rescale, O) may be written once both CTAs' PV of the
        // previous tile have completed.
        if (u > 0 &&
            !__all_sync(0xffffffffu,
                        mbar_wait_cluster(p_free, (uint32_t)((u - 1) & 1), abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (rescale) {
#pragma unroll 1
          for (int c = 0; c < kDHalf / 32; ++c) {
            uint32_t r[32];
            tmem_load_32x32b_x32(tmem_o + lane_off + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * f);
            tmem_store_32x32b_x32(tmem_o + lane_off + c * 32, r);
          }
          tmem_wait_st();
        }
        // P as 16-bit K-major tiles of 64 keys (blocks 2r, 2r + 1 of the
        // tile's four).
#pragma unroll
        for (int c = 0; c < kOwnKeys / 32; ++c) {
          const int blk = 2 * (int)rank + (c >> 1);
          uint8_t* rowp = pbuf + blk * kPBlock + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (c & 1) * 4 + q;
            const int k0 = c * 16 + 4 * q;
            *reinterpret_cast<uint4*>(rowp + ((chunk ^ (row & 7)) << 4)) =
                make_uint4(pk[k0], pk[k0 + 1], pk[k0 + 2], pk[k0 + 3]);
          }
        }
        // The warp's 32 rows of both blocks to the peer (two 4 KB bulk copies
        // completing on the peer's p_ready), then ready here: P (and a
        // rescaled O) visible to this CTA's tensor core.
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t off = (uint32_t)((2 * (int)rank + h) * kPBlock + quad * 32 * 128);
            bulk_copy_to_cluster(peer_pbuf + off, pbuf + off, 32 * 128, peer_p_ready);
          }
          mbar_arrive_expect_tx(p_ready, 2 * 32 * 128);
        }
      }
      if (!ok) break;
      // O is final once both CTAs' last PV completed; add the peer's row sum.
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(p_free, (uint32_t)((u - 1) & 1), abort_flag)))
        break;
      tc_fence_after();
      st_cluster_f32(peer_lx + (uint32_t)(row * 4), l);
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_release(peer_l_ready);
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(l_ready, (uint32_t)(task_idx & 1), abort_flag)))
        break;
      const float inv = 1.0f / (l + lx[row]);
      uint4* dst = reinterpret_cast<uint4*>(
          static_cast<uint16_t*>(p.out) +
          ((long long)b * p.n_q + qt * kRows + row) * p.ld_out + (int)rank * kDHalf);
#pragma unroll 1
      for (int c = 0; c < kDHalf / 32; ++c) {
        uint32_t r[32];
        tmem_load_32x32b_x32(tmem_o + lane_off + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int k = 0; k < 16; ++k)
          pk[k] = Elem<D>::pack(__uint_as_float(r[2 * k]) * inv, __uint_as_float(r[2 * k + 1]) * inv);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[c * 4 + q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still write into it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

typedef CUresult (*EncodeTiledFnP)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnP encode_fn_p() {
  static EncodeTiledFnP fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnP>(ptr);
    return static_cast<EncodeTiledFnP>(nullptr);
  }();
  return fn;
}

PerDeviceOnce g_pair_smem[2];
std::atomic<int> g_pair_clusters[2][kMaxDevices];

template <int D>
cudaError_t pair_launch_typed(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                              const PairParams& p, cudaStream_t stream) {
  const int di = D == kF16 ? 1 : 0;
  cudaError_t e = g_pair_smem[di].run([] {
    return cudaFuncSetAttribute(attn_pair_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kSmem);
  });
  if (e != cudaSuccess) return e;
  int device = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  int clusters = g_pair_clusters[di][device].load();
  if (clusters == 0) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, attn_pair_kernel<D>, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorNotSupported;
    clusters = n < sms / 2 ? n : sms / 2;
    g_pair_clusters[di][device].store(clusters);
  }
  if (clusters > p.tasks) clusters = p.tasks;
  attn_pair_kernel<D><<<2 * clusters, kThreads, kSmem, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace

bool attn_pair_ok(int n_q, int n_kv, int dim, long long ld_q, long long ld_kv, long long ld_out,
                  const void* q, const void* k, const void* vt, const void* out) {
  if (n_q <= 0 || n_q % kRows != 0 || n_kv <= 0 || n_kv % (2 * kTileKeys) != 0 || dim != kDim)
    return false;
  if (ld_q % 8 != 0 || ld_kv % 8 != 0 || ld_out % 8 != 0) return false;
  return ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
           reinterpret_cast<uintptr_t>(vt) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
}

cudaError_t attn_pair_launch(int dtype, const void* q, long long ld_q, const void* k,
                             long long ld_kv, const void* vt, void* out, long long ld_out,
                             int batch, int n_q, int n_kv, cudaStream_t stream) {
  if (!attn_pair_ok(n_q, n_kv, kDim, ld_q, ld_kv, ld_out, q, k, vt, out) || batch <= 0)
    return cudaErrorInvalidValue;
  EncodeTiledFnP encode = encode_fn_p();
  if (!encode) return cudaErrorNotSupported;
  const CUtensorMapDataType tdt =
      dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv;
  cuuint32_t estr[3] = {1, 1, 1};
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDim, (cuuint64_t)batch * n_q};
    cuuint64_t strides[1] = {(cuuint64_t)ld_q * 2};
    cuuint32_t box[2] = {(cuuint32_t)kDChunk, (cuuint32_t)kRows};
    if (encode(&tq, tdt, 2, const_cast<void*>(q), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    dims[1] = (cuuint64_t)batch * n_kv;
    strides[0] = (cuuint64_t)ld_kv * 2;
    box[1] = kOwnKeys;
    if (encode(&tk, tdt, 2, const_cast<void*>(k), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    // V^T per image: [dim][n_kv], images contiguous.
    cuuint64_t dims[3] = {(cuuint64_t)n_kv, (cuuint64_t)kDim, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)n_kv * 2, (cuuint64_t)n_kv * kDim * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)kDHalf, 1};
    if (encode(&tv, tdt, 3, const_cast<void*>(vt), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  PairParams p;
  p.n_q = n_q;
  p.n_kv = n_kv;
  p.batch = batch;
  p.tiles = n_kv / kTileKeys;
  p.tasks = batch * (n_q / kRows);
  p.out = out;
  p.ld_out = ld_out;
  return dtype == kF16 ? pair_launch_typed<kF16>(tq, tk, tv, p, stream)
                       : pair_launch_typed<kBf16>(tq, tk, tv, p, stream);
}

}  // namespace osor
