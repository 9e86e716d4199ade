// Fused single-head attention softmax(Q K^T) V for the VAE mid-block
// (N = h*w tokens, D = 256 or 512 channels, q and k already scaled by D^-1/4).
//
// One CTA task = one image, 128 query rows and one 256-column half of D.
// Per key tile of 256 keys:
//   S = Q K^T (M = 128, N = 256, K = D) accumulates in TMEM columns 0..255
//   from (Q chunk, K chunk) stages of 64 channels;
//   four softmax warps (one TMEM lane quadrant each, one query row per
//   thread) take the row maximum, rescale O when the maximum grew by more
//   than 2^8 (otherwise the stale maximum stays and P stays <= 256), write
//   P = 2^(S log2 e - m) as 16-bit K-major tiles to shared memory and keep
//   the fp32 row sum;
//   O += P V_half (M = 128, N = 256, K = 256 keys) accumulates in TMEM
//   columns 256..511 from V^T chunks [256 channels x 64 keys].
// The next tile's S MMAs run while the softmax warps work on this one; the
// P buffer is single, so P(j) is written only after PV(j-1) has consumed
// P(j-1). Scores never leave the SM: HBM traffic is Q, K, V^T (from L2) and
// the output. The D split costs one redundant Q K^T per half; TMEM (512
// columns) holds one 256-key S tile and one 128 x 256 O half, not a full
// 128 x 512 O.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM allocator and MMA
// issuer, warps 2..5 softmax and output epilogue.
//
// Reference counterpart: Attention::forward_checked / attend_with
// (src/native/vae_encoder.rs:237-340, src/native/attention.rs:27-84).
#include <atomic>
#include "attn_fa.h"
#include "common.cuh"

namespace osor {
namespace {

constexpr int kQRows = 128;
constexpr int kKeys = 256;  // keys per tile
constexpr int kDChunk = 64;
constexpr int kDHalf = 256;
constexpr int kQChunkBytes = kQRows * kDChunk * 2;  // 16 KB
constexpr int kKChunkBytes = kKeys * kDChunk * 2;   // 32 KB
constexpr int kAStage = kQChunkBytes + kKChunkBytes;
constexpr int kBStage = kDHalf * 64 * 2;            // V^T chunk: 256 channels x 64 keys
constexpr int kPBlock = kQRows * 64 * 2;            // P: 128 rows x 64 keys
constexpr int kAStages = 2;
constexpr int kBStages = 2;
constexpr int kFaThreads = 192;
constexpr int kFaSmem = kAStages * kAStage + kBStages * kBStage + 4 * kPBlock + 1024 + 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;

struct FaParams {
  int tokens, dim, batch;
  int halves;  // dim / 256
  int tiles;   // tokens / 256
  int tasks;   // batch * tokens / 128 * halves
  void* out;
  long long ld_out;
};

__device__ void fa_drain(uint64_t* bars, int n, int stage, uint32_t phase) {
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
__global__ void __launch_bounds__(kFaThreads, 1)
    attn_fa_kernel(const __grid_constant__ CUtensorMap tmap_q,
                   const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_vt, const FaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring_a = smem;
  uint8_t* ring_b = ring_a + kAStages * kAStage;
  uint8_t* pbuf = ring_b + kBStages * kBStage;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(pbuf + 4 * kPBlock);
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* b_full = a_empty + kAStages;
  uint64_t* b_empty = b_full + kBStages;
  uint64_t* s_full = b_empty + kBStages;
  uint64_t* pv_done = s_full + 1;
  uint64_t* p_ready = pv_done + 1;
  uint64_t* o_free = p_ready + 1;
  uint64_t* drain = o_free + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(pv_done, 1);
    mbar_init(p_ready, 4);
    mbar_init(o_free, 4);
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
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t tmem_s = tmem_base;
  const uint32_t tmem_o = tmem_base + 256;
  const int qtiles = p.tokens / kQRows;
  const int d_chunks = p.dim / kDChunk;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ producer
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      bool ok = true;
      auto load_v = [&](int b, int dh, int tile) -> bool {
        for (int c = 0; c < kKeys / 64; ++c) {
          if (!mbar_wait(&b_empty[bs], bph ^ 1, abort_flag)) return false;
          mbar_arrive_expect_tx(&b_full[bs], kBStage);
          tma_load_3d(ring_b + bs * kBStage, &tmap_vt, &b_full[bs], tile * kKeys + c * 64,
                      dh * kDHalf, b);
          if (++bs == kBStages) {
            bs = 0;
            bph ^= 1;
          }
        }
        return true;
      };
      for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x) {
        const int dh = t % p.halves;
        const int qt = (t / p.halves) % qtiles;
        const int b = t / (p.halves * qtiles);
        const int qrow = b * p.tokens + qt * kQRows;
        for (int j = 0; j < p.tiles && ok; ++j) {
          for (int dc = 0; dc < d_chunks; ++dc) {
            if (!mbar_wait(&a_empty[as], aph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&a_full[as], kAStage);
            uint8_t* st = ring_a + as * kAStage;
            tma_load_2d(st, &tmap_q, &a_full[as], dc * kDChunk, qrow);
            tma_load_2d(st + kQChunkBytes, &tmap_k, &a_full[as], dc * kDChunk,
                        b * p.tokens + j * kKeys);
            if (++as == kAStages) {
              as = 0;
              aph ^= 1;
            }
          }
          if (ok && j > 0) ok = load_v(b, dh, j - 1);
        }
        if (ok) ok = load_v(b, dh, p.tiles - 1);
      }
      if (!ok) {
        fa_drain(a_full, kAStages, as, aph);
        fa_drain(b_full, kBStages, bs, bph);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = umma_idesc_f32acc(kQRows, 256, Elem<D>::kUmmaFormat);
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0, pr_par = 0, of_par = 0;
      bool ok = true, issued = false, first_task = true;
      auto pv = [&](bool first_tile) -> bool {
        // O += P V^T-chunks: P block c holds keys 64c .. 64c+63.
        for (int c = 0; c < kKeys / 64; ++c) {
          if (!mbar_wait(&b_full[bs], bph, abort_flag)) return false;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(pbuf + c * kPBlock);
          const uint32_t b_addr = smem_u32(ring_b + bs * kBStage);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem_o, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32),
                      idesc, !(first_tile && c == 0 && k == 0));
          issued = true;
          umma_commit(&b_empty[bs]);
          if (++bs == kBStages) {
            bs = 0;
            bph ^= 1;
          }
        }
        umma_commit(pv_done);
        return true;
      };
      for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x) {
        for (int j = 0; j < p.tiles && ok; ++j) {
          if (j > 0) {
            // softmax(j - 1) is done: S is free, P(j - 1) written, O rescaled.
            if (!mbar_wait(p_ready, pr_par, abort_flag)) {
              ok = false;
              break;
            }
            pr_par ^= 1;
            tc_fence_after();
          }
          for (int dc = 0; dc < d_chunks; ++dc) {
            if (!mbar_wait(&a_full[as], aph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t q_addr = smem_u32(ring_a + as * kAStage);
            const uint32_t k_addr = q_addr + kQChunkBytes;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_bf16(tmem_s, sw128_kmajor_desc(q_addr + k * 32),
                        sw128_kmajor_desc(k_addr + k * 32), idesc, (dc | k) != 0);
            issued = true;
            umma_commit(&a_empty[as]);
            if (++as == kAStages) {
              as = 0;
              aph ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(s_full);
          if (j > 0) {
            if (j == 1 && !first_task) {
              // The previous task's epilogue has read O.
              if (!mbar_wait(o_free, of_par, abort_flag)) {
                ok = false;
                break;
              }
              of_par ^= 1;
              tc_fence_after();
            }
            if (!(ok = pv(j == 1))) break;
          }
        }
        if (!ok) break;
        if (!mbar_wait(p_ready, pr_par, abort_flag)) {
          ok = false;
          break;
        }
        pr_par ^= 1;
        tc_fence_after();
        if (p.tiles == 1 && !first_task) {
          if (!mbar_wait(o_free, of_par, abort_flag)) {
            ok = false;
            break;
          }
          of_par ^= 1;
          tc_fence_after();
        }
        if (!(ok = pv(p.tiles == 1))) break;
        first_task = false;
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
    // ------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // query row within the task
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    uint32_t sf_par = 0, pv_par = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tasks && ok; t += gridDim.x) {
      const int dh = t % p.halves;
      const int qt = (t / p.halves) % qtiles;
      const int b = t / (p.halves * qtiles);
      float m = 0.0f, l = 0.0f;
      for (int j = 0; j < p.tiles; ++j) {
        if (!mbar_wait(s_full, sf_par, abort_flag)) {
          ok = false;
          break;
        }
        sf_par ^= 1;
        tc_fence_after();
        // Row maximum of this tile (log2 units).
        float mt = -3.0e38f;
#pragma unroll 1
        for (int c = 0; c < kKeys / 32; ++c) {
          uint32_t r[32];
          tmem_load_32x32b_x32(tmem_s + lane_off + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; ++k) mt = fmaxf(mt, __uint_as_float(r[k]));
        }
        mt *= kLog2e;
        if (j > 0) {
          // PV(j - 1) has consumed P(j - 1) and O is final for keys < 256 j.
          if (!mbar_wait(pv_done, pv_par, abort_flag)) {
            ok = false;
            break;
          }
          pv_par ^= 1;
          tc_fence_after();
          // tcgen05.ld / st are warp-collective (.sync.aligned): the warp
          // rescales together when any of its rows needs it, each row with
          // its own factor (1 for rows whose maximum stays).
          const bool grow = mt > m + kRescaleLog2;
          if (__any_sync(0xffffffffu, grow)) {
            const float f = grow ? ex2_approx(m - mt) : 1.0f;
            l *= f;
            if (grow) m = mt;
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
        } else {
          m = mt;
        }
        // P = 2^(S log2 e - m), 16-bit, K-major 128-byte-swizzled tiles of
        // 64 keys; row sum in fp32.
#pragma unroll 1
        for (int c = 0; c < kKeys / 32; ++c) {
          uint32_t r[32];
          tmem_load_32x32b_x32(tmem_s + lane_off + c * 32, r);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(r[2 * k]), kLog2e, -m));
            const float p1 = ex2_approx(fmaf(__uint_as_float(r[2 * k + 1]), kLog2e, -m));
            l += p0 + p1;
            pk[k] = Elem<D>::pack(p0, p1);
          }
          uint8_t* blk = pbuf + (c >> 1) * kPBlock + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (c & 1) * 4 + q;
            *reinterpret_cast<uint4*>(blk + ((chunk ^ (row & 7)) << 4)) =
                make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_ready);
      }
      if (!ok) break;
      // O is final after the last PV.
      if (!mbar_wait(pv_done, pv_par, abort_flag)) break;
      pv_par ^= 1;
      tc_fence_after();
      const float inv = 1.0f / l;
      uint4* dst = reinterpret_cast<uint4*>(
          static_cast<uint16_t*>(p.out) +
          ((long long)b * p.tokens + qt * kQRows + row) * p.ld_out + dh * kDHalf);
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

typedef CUresult (*EncodeTiledFnA)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnA encode_fn_a() {
  static EncodeTiledFnA fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnA>(ptr);
    return static_cast<EncodeTiledFnA>(nullptr);
  }();
  return fn;
}

template <int D>
cudaError_t fa_launch_typed(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const FaParams& p, cudaStream_t stream) {
  static std::atomic<int> sms[64];  // zero-initialized; atomic for concurrent callers
  int device = 0;
  cudaGetDevice(&device);
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (sms[device] == 0) {
    cudaError_t e = cudaFuncSetAttribute(attn_fa_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem);
    if (e != cudaSuccess) return e;
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    sms[device] = n > 0 ? n : 148;
  }
  const int resident = sms[device].load();
  const int grid = p.tasks < resident ? p.tasks : resident;
  attn_fa_kernel<D><<<grid, kFaThreads, kFaSmem, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace

bool attn_fused_ok(int tokens, int dim, long long ld, long long ld_out, const void* q,
                   const void* k, const void* vt, const void* out) {
  if (tokens <= 0 || tokens % kKeys != 0 || (dim != 256 && dim != 512)) return false;
  if (ld % 8 != 0 || ld_out % 8 != 0) return false;
  return ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
           reinterpret_cast<uintptr_t>(vt) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
}

cudaError_t attn_fused_launch(int dtype, const void* q, const void* k, long long ld,
                              const void* vt, void* out, long long ld_out, int batch, int tokens,
                              int dim, cudaStream_t stream) {
  EncodeTiledFnA encode = encode_fn_a();
  if (!encode) return cudaErrorNotSupported;
  const CUtensorMapDataType tdt =
      dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq, tk, tv;
  cuuint32_t estr[3] = {1, 1, 1};
  {
    cuuint64_t dims[2] = {(cuuint64_t)dim, (cuuint64_t)batch * tokens};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kDChunk, (cuuint32_t)kQRows};
    if (encode(&tq, tdt, 2, const_cast<void*>(q), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    box[1] = kKeys;
    if (encode(&tk, tdt, 2, const_cast<void*>(k), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    // V^T per image: [dim][tokens], images contiguous.
    cuuint64_t dims[3] = {(cuuint64_t)tokens, (cuuint64_t)dim, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)tokens * 2, (cuuint64_t)tokens * dim * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)kDHalf, 1};
    if (encode(&tv, tdt, 3, const_cast<void*>(vt), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  FaParams p;
  p.tokens = tokens;
  p.dim = dim;
  p.batch = batch;
  p.halves = dim / kDHalf;
  p.tiles = tokens / kKeys;
  p.tasks = batch * (tokens / kQRows) * p.halves;
  p.out = out;
  p.ld_out = ld_out;
  return dtype == kF16 ? fa_launch_typed<kF16>(tq, tk, tv, p, stream)
                       : fa_launch_typed<kBf16>(tq, tk, tv, p, stream);
}

}  // namespace osor
