// Multi-head attention of head width 64 on the sm_100a tensor cores (the SDXL
// UNet's self and cross attention: 10 heads over 4096 tokens, 20 over 1024,
// cross attention over the 77 prompt tokens).
//
// One CTA (one per SM) takes a task of one batch entry, one head and 256
// query rows as two 128-row groups A and B that share every key / value tile:
//   S_g = Q_g K^T      M = 128, N = 128 keys, K = 64    -> TMEM (one buffer per group)
//   O_g += P_g V       M = 128, N = 64, K = 128 keys    -> TMEM (per group), with P_g
//                      itself in TMEM (written by the softmax threads with
//                      tcgen05.st, read as the MMA's A operand)
// Two softmax warp groups (four warps each, one query row per thread) work on
// A and B in turn, so one group's exponentials overlap the other group's
// MMAs: the MMA issuer runs S_A(0), S_B(0), then per tile S_A(j+1), PV_A(j),
// S_B(j+1), PV_B(j): a group's softmax takes its scores into registers and
// frees the TMEM buffer at once, so the next tile's scores are computed while
// it evaluates the exponentials. The running maximum moves, and O is rescaled, only when
// it grows by more than 2^8 (so P <= 256); keys past the last valid one of a
// ragged tile are masked.
//
// Both products keep their shared-memory traffic small: P never goes through
// shared memory (the softmax threads store it into TMEM with tcgen05.st and
// the P V MMA reads its A operand from TMEM), and V is read as loaded (rows =
// keys of 64 head columns) as the MMA's MN-major B operand, so q, k and v come
// straight from the fused q|k|v product with no transpose.
//
// Roles (352 threads): warp 0 TMA producer, warp 1 TMEM allocator and MMA
// issuer, warp 2 idle, warps 3..6 softmax group A, warps 7..10 group B (warp
// w reads TMEM lanes 32 (w % 4) ..). TMEM: S_A 0..127, S_B 128..255, O_A
// 256..319, O_B 320..383, P_A 384..447, P_B 448..511. All waits are bounded.
//
// Reference counterpart: SelfAttention / FixedCrossAttention's attend
// (src/native/spatial.rs:29-46, 83-158).
#include <atomic>

#include "common.cuh"
#include "device_guard.h"
#include "unet.h"

namespace osor {
namespace {

constexpr int kHd = 64;                       // head width
constexpr int kGRows = 128;                   // query rows per group
constexpr int kKeys = 128;                    // keys per tile
constexpr int kTileBytes = kKeys * kHd * 2;   // 16 KB: Q group, K tile, V tile, V^T tile
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kThreadsH = 352;
constexpr int kSmemH = 2 * kTileBytes            // Q groups
                       + kKStages * kTileBytes   // K ring
                       + kVStages * kTileBytes   // V ring
                       + 256 + 1024;
constexpr uint32_t kTmemP = 384;  // P_g (16-bit, two keys per column) at 384 + 64 g
constexpr float kLog2eH = 1.4426950408889634f;
constexpr float kRescaleLog2H = 8.0f;

struct HeadsParams {
  int batch, heads, n_q, n_kv;
  int qtiles;      // n_q / 256
  int tiles;       // ceil(n_kv / 128)
  int tasks;       // batch * heads * qtiles
  int kv_shared;   // 1: one key / value set for every batch entry
  void* out;
  long long ld_out, out_bs;
};

__device__ void heads_drain(uint64_t* bars, int n, int stage, uint32_t phase) {
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
__global__ void __launch_bounds__(kThreadsH, 1)
    attn_heads64_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                           const __grid_constant__ CUtensorMap tmap_k,
                           const __grid_constant__ CUtensorMap tmap_v, const HeadsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* qbuf = smem;                                  // [2 groups][16 KB]
  uint8_t* kring = qbuf + 2 * kTileBytes;
  uint8_t* vring = kring + kKStages * kTileBytes;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(vring + kVStages * kTileBytes);
  uint64_t* q_free = q_full + 1;
  uint64_t* k_full = q_free + 1;
  uint64_t* k_empty = k_full + kKStages;
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + kVStages;
  uint64_t* s_full = v_empty + kVStages;    // [group]
  uint64_t* s_free = s_full + 2;            // [group]
  uint64_t* p_ready = s_free + 2;           // [group]
  uint64_t* p_free = p_ready + 2;           // [group]
  uint64_t* o_free = p_free + 2;            // [group]
  uint64_t* drain = o_free + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_free, 2);  // one MMA commit per group's last S of the task
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
      mbar_init(&p_ready[b], 4);
      mbar_init(&p_free[b], 1);
      mbar_init(&o_free[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // TMEM: S_A 0..127, S_B 128..255, O_A 256..319, O_B 320..383.
  const int per_b = p.heads * p.qtiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int ks = 0, vs = 0;
      uint32_t kph = 0, vph = 0;
      int task_idx = 0, q_loads = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x, ++task_idx) {
        const int b = t / per_b;
        const int rem = t - b * per_b;
        const int h = rem / p.qtiles;
        const int qt = rem - h * p.qtiles;
        const int bkv = p.kv_shared ? 0 : b;
        // Both groups' Q rows, once the previous task's last S products read them.
        if (task_idx > 0 && !mbar_wait(q_free, (uint32_t)((task_idx - 1) & 1), abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
        tma_load_3d(qbuf, &tmap_q, q_full, h * kHd, qt * 2 * kGRows, b);
        tma_load_3d(qbuf + kTileBytes, &tmap_q, q_full, h * kHd, qt * 2 * kGRows + kGRows, b);
        ++q_loads;
        for (int j = 0; j < p.tiles && ok; ++j) {
          if (!mbar_wait(&k_empty[ks], kph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[ks], kTileBytes);
          tma_load_3d(kring + ks * kTileBytes, &tmap_k, &k_full[ks], h * kHd, j * kKeys, bkv);
          if (++ks == kKStages) {
            ks = 0;
            kph ^= 1;
          }
          if (!mbar_wait(&v_empty[vs], vph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[vs], kTileBytes);
          tma_load_3d(vring + vs * kTileBytes, &tmap_v, &v_full[vs], h * kHd, j * kKeys, bkv);
          if (++vs == kVStages) {
            vs = 0;
            vph ^= 1;
          }
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits.
        heads_drain(k_full, kKStages, ks, kph);
        heads_drain(v_full, kVStages, vs, vph);
        if (q_loads > 0) {
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(smem_u32(q_full), (uint32_t)((q_loads - 1) & 1)) &&
                 global_timer_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_f32acc(kGRows, kKeys, Elem<D>::kUmmaFormat);
      // B (V) is MN-major: bit 16 of the instruction descriptor transposes it.
      constexpr uint32_t idesc_o =
          umma_idesc_f32acc(kGRows, kHd, Elem<D>::kUmmaFormat) | (1u << 16);
      int ks = 0, vs = 0;
      uint32_t kph = 0, vph = 0;
      long long tile_u = 0;   // global tile counter
      long long s_use = 0;    // S products issued per group (same for both)
      int task_idx = 0;
      bool ok = true, issued = false;
      auto s_product = [&](int g, bool last_for_task) -> bool {
        // S_g = Q_g K^T into the group's buffer, after its softmax read the
        // previous one.
        if (!mbar_wait(&s_free[g], (uint32_t)((s_use & 1) ^ 1), abort_flag)) return false;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(qbuf + g * kTileBytes);
        const uint32_t b_addr = smem_u32(kring + ks * kTileBytes);
#pragma unroll
        for (int k = 0; k < kHd / 16; ++k)
          umma_bf16(tmem_base + g * kKeys, sw128_kmajor_desc(a_addr + k * 32),
                    sw128_kmajor_desc(b_addr + k * 32), idesc_s, k != 0);
        issued = true;
        umma_commit(&s_full[g]);
        if (last_for_task) umma_commit(q_free);
        return true;
      };
      auto pv_product = [&](int g, bool first) -> bool {
        if (!mbar_wait(&p_ready[g], (uint32_t)(tile_u & 1), abort_flag)) return false;
        tc_fence_after();
        const uint32_t o_tmem = tmem_base + 256 + g * kHd;
        // A = P_g from TMEM (keys 16 kb .. + 15 in columns 8 kb .. + 7); B =
        // the V tile as loaded, rows = keys of 64 head columns (128 bytes):
        // the MN-major operand, 16 keys = two 8-row swizzle atoms per step.
        const uint32_t p_tmem = tmem_base + kTmemP + g * 64;
        const uint32_t v_addr = smem_u32(vring + vs * kTileBytes);
#pragma unroll
        for (int kb = 0; kb < kKeys / 16; ++kb)
          umma_bf16_tmem_a(o_tmem, p_tmem + kb * 8, sw128_kmajor_desc(v_addr + kb * 2048), idesc_o,
                           !(first && kb == 0));
        issued = true;
        umma_commit(&p_free[g]);
        return true;
      };
      for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x, ++task_idx) {
        if (!mbar_wait(q_full, (uint32_t)(task_idx & 1), abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // K tile 0, both groups' first scores.
        if (!mbar_wait(&k_full[ks], kph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!(ok = s_product(0, p.tiles == 1))) break;
        if (!(ok = s_product(1, p.tiles == 1))) break;
        ++s_use;
        umma_commit(&k_empty[ks]);
        if (++ks == kKStages) {
          ks = 0;
          kph ^= 1;
        }
        for (int j = 0; j < p.tiles && ok; ++j, ++tile_u) {
          // Per group: the next tile's scores as soon as the softmax has
          // taken this tile's into registers (they run while it computes
          // P), then this tile's P V once P is in shared memory.
          const bool more = j + 1 < p.tiles;
          if (more) {
            if (!mbar_wait(&k_full[ks], kph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          for (int g = 0; g < 2 && ok; ++g) {
            if (more) {
              if (!(ok = s_product(g, j + 2 == p.tiles))) break;
              if (g == 1) umma_commit(&k_empty[ks]);
            }
            if (g == 0) {
              if (!mbar_wait(&v_full[vs], vph, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            if (j == 0 && task_idx > 0) {
              // The previous task's epilogue of this group has read O_g.
              if (!mbar_wait(&o_free[g], (uint32_t)((task_idx - 1) & 1), abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            if (!(ok = pv_product(g, j == 0))) break;
          }
          if (!ok) break;
          umma_commit(&v_empty[vs]);
          if (++vs == kVStages) {
            vs = 0;
            vph ^= 1;
          }
          if (more) {
            ++s_use;
            if (++ks == kKStages) {
              ks = 0;
              kph ^= 1;
            }
          }
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
  } else if (warp >= 3) {
    // ---------------------------------------------------------- softmax + epilogue
    const int g = (warp - 3) >> 2;     // group
    const int quad = warp & 3;         // TMEM lane quadrant
    const int row = quad * 32 + lane;  // row within the group
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_tmem = tmem_base + g * kKeys + lane_off;
    const uint32_t o_tmem = tmem_base + 256 + g * kHd + lane_off;
    long long tile_u = 0;
    long long s_use = 0;
    int task_idx = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x, ++task_idx) {
      const int b = t / per_b;
      const int rem = t - b * per_b;
      const int h = rem / p.qtiles;
      const int qt = rem - h * p.qtiles;
      float m = 0.0f, l = 0.0f;
      for (int j = 0; j < p.tiles; ++j, ++tile_u, ++s_use) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g], (uint32_t)(s_use & 1), abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // The row's 128 scores into registers; the buffer then takes the
        // next tile's scores while P is computed.
        float sv[kKeys];
        {
          uint32_t r[kKeys];
#pragma unroll
          for (int c = 0; c < kKeys / 32; ++c)
            tmem_load_32x32b_x32(s_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < kKeys; ++k) sv[k] = __uint_as_float(r[k]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[g]);
        // Keys past the last one of a ragged tile do not take part (their
        // probability underflows to zero).
        const int valid = p.n_kv - j * kKeys;
        if (valid < kKeys) {
#pragma unroll
          for (int k = 0; k < kKeys; ++k)
            if (k >= valid) sv[k] = -3.0e38f;
        }
        // Row maximum as a tree of eight chains (one chain of 128 dependent
        // max operations would sit on every tile's critical path).
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = sv[i];
#pragma unroll
        for (int k = 8; k < kKeys; ++k) acc[k & 7] = fmaxf(acc[k & 7], sv[k]);
#pragma unroll
        for (int w = 4; w > 0; w >>= 1)
#pragma unroll
          for (int i = 0; i < w; ++i) acc[i] = fmaxf(acc[i], acc[i + w]);
        const float mt = acc[0] * kLog2eH;
        float f = 1.0f;
        bool rescale = false;
        if (j == 0) {
          m = mt;
          l = 0.0f;
        } else {
          const bool grow = mt > m + kRescaleLog2H;
          rescale = __any_sync(0xffffffffu, grow);  // tcgen05.ld / st below are warp-wide
          if (grow) {
            f = ex2_approx(m - mt);
            m = mt;
          }
          l *= f;
        }
        float lsum = 0.0f;
        uint32_t pk[kKeys / 2];
#pragma unroll
        for (int k = 0; k < kKeys / 2; ++k) {
          const float p0 = ex2_approx(fmaf(sv[2 * k], kLog2eH, -m));
          const float p1 = ex2_approx(fmaf(sv[2 * k + 1], kLog2eH, -m));
          lsum += p0 + p1;
          pk[k] = Elem<D>::pack(p0, p1);
        }
        l += lsum;
        // P and O may be written once this group's previous PV completed.
        if (j > 0 || task_idx > 0) {
          if (!__all_sync(0xffffffffu,
                          mbar_wait(&p_free[g], (uint32_t)((tile_u - 1) & 1), abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (rescale) {
#pragma unroll 1
          for (int c = 0; c < kHd / 32; ++c) {
            uint32_t r[32];
            tmem_load_32x32b_x32(o_tmem + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 32; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * f);
            tmem_store_32x32b_x32(o_tmem + c * 32, r);
          }
          tmem_wait_st();
        }
        // P into TMEM (this row's lane, two keys per column), the A operand
        // of the group's P V product: no shared-memory round trip.
        const uint32_t p_tmem = tmem_base + kTmemP + g * 64 + lane_off;
        tmem_store_32x32b_x32(p_tmem, *reinterpret_cast<const uint32_t(*)[32]>(pk));
        tmem_store_32x32b_x32(p_tmem + 32, *reinterpret_cast<const uint32_t(*)[32]>(pk + 32));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[g]);
      }
      if (!ok) break;
      // O_g is final after this group's last PV.
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&p_free[g], (uint32_t)((tile_u - 1) & 1), abort_flag)))
        break;
      tc_fence_after();
      const float inv = 1.0f / l;
      uint32_t r[kHd];
#pragma unroll
      for (int c = 0; c < kHd / 32; ++c)
        tmem_load_32x32b_x32(o_tmem + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[g]);
      const int qrow = qt * 2 * kGRows + g * kGRows + row;
      if (qrow < p.n_q) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + b * p.out_bs +
                                              (long long)qrow * p.ld_out + h * kHd);
#pragma unroll
        for (int q = 0; q < kHd / 8; ++q)
          dst[q] = make_uint4(Elem<D>::pack(__uint_as_float(r[8 * q]) * inv,
                                            __uint_as_float(r[8 * q + 1]) * inv),
                              Elem<D>::pack(__uint_as_float(r[8 * q + 2]) * inv,
                                            __uint_as_float(r[8 * q + 3]) * inv),
                              Elem<D>::pack(__uint_as_float(r[8 * q + 4]) * inv,
                                            __uint_as_float(r[8 * q + 5]) * inv),
                              Elem<D>::pack(__uint_as_float(r[8 * q + 6]) * inv,
                                            __uint_as_float(r[8 * q + 7]) * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

typedef CUresult (*EncodeTiledFnH)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnH encode_fn_h() {
  static EncodeTiledFnH fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnH>(ptr);
    return static_cast<EncodeTiledFnH>(nullptr);
  }();
  return fn;
}

PerDeviceOnce g_heads_smem[2];
std::atomic<int> g_heads_sms[kMaxDevices];

// 3-D map over [batch][rows][cols] 16-bit rows of stride ld, batch stride bs
// (batch 1 when bs == 0), box of 64 columns x 128 rows.
bool rows_map(EncodeTiledFnH encode, CUtensorMapDataType tdt, CUtensorMap* map, const void* base,
              int cols, int rows, int batch, long long ld, long long bs) {
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)(bs ? batch : 1)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(bs ? bs : (long long)rows * ld) * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, tdt, 3, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

}  // namespace

bool attn_heads64_tc_ok(const void* q, long long ld_q, long long q_bs, const void* k,
                        const void* v, long long ld_kv, long long kv_bs, const void* out,
                        long long ld_out, long long out_bs, int n_q, int n_kv) {
  if (n_q <= 0 || n_q % (2 * kGRows) != 0 || n_kv <= 0) return false;
  if (ld_q % 8 || ld_kv % 8 || ld_out % 8 || q_bs % 8 || kv_bs % 8 || out_bs % 8) return false;
  if (q_bs != 0 && q_bs < (long long)n_q * ld_q) return false;
  if (kv_bs != 0 && kv_bs < (long long)n_kv * ld_kv) return false;
  return ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
           reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
}

cudaError_t attn_heads64_tc_launch(int dtype, const void* q, long long ld_q, long long q_bs,
                                   const void* k, const void* v, long long ld_kv, long long kv_bs,
                                   void* out, long long ld_out, long long out_bs, int batch,
                                   int heads, int n_q, int n_kv, cudaStream_t s) {
  if (!attn_heads64_tc_ok(q, ld_q, q_bs, k, v, ld_kv, kv_bs, out, ld_out, out_bs, n_q, n_kv) ||
      batch <= 0 || heads <= 0)
    return cudaErrorInvalidValue;
  EncodeTiledFnH encode = encode_fn_h();
  if (!encode) return cudaErrorNotSupported;
  const CUtensorMapDataType tdt =
      dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv;
  const int cols = heads * kHd;
  if (!rows_map(encode, tdt, &tq, q, cols, n_q, batch, ld_q, q_bs) ||
      !rows_map(encode, tdt, &tk, k, cols, n_kv, batch, ld_kv, kv_bs) ||
      !rows_map(encode, tdt, &tv, v, cols, n_kv, batch, ld_kv, kv_bs))
    return cudaErrorInvalidValue;
  HeadsParams p;
  p.batch = batch;
  p.heads = heads;
  p.n_q = n_q;
  p.n_kv = n_kv;
  p.qtiles = n_q / (2 * kGRows);
  p.tiles = (n_kv + kKeys - 1) / kKeys;
  p.tasks = batch * heads * p.qtiles;
  p.kv_shared = kv_bs == 0 ? 1 : 0;
  p.out = out;
  p.ld_out = ld_out;
  p.out_bs = out_bs;
  const int di = dtype == kF16 ? 1 : 0;
  cudaError_t e = g_heads_smem[di].run([&] {
    return dtype == kF16 ? cudaFuncSetAttribute(attn_heads64_tc_kernel<kF16>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmemH)
                         : cudaFuncSetAttribute(attn_heads64_tc_kernel<kBf16>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmemH);
  });
  if (e != cudaSuccess) return e;
  int device = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  int sms = g_heads_sms[device].load();
  if (sms == 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (sms <= 0) sms = 148;
    g_heads_sms[device].store(sms);
  }
  const int grid = p.tasks < sms ? p.tasks : sms;
  if (dtype == kF16)
    attn_heads64_tc_kernel<kF16><<<grid, kThreadsH, kSmemH, s>>>(tq, tk, tv, p);
  else
    attn_heads64_tc_kernel<kBf16><<<grid, kThreadsH, kSmemH, s>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace osor
