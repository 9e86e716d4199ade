// Implicit-GEMM 3x3 (or 1x1) convolution with the pixels on the MMA's N side.
//
// For Cout <= 128 this kernel swaps the GEMM operands so that every
// tcgen05.mma is a full M = 128, N = 256 instruction:
// D[cout][pixel] = W[cout][K] x X[pixel][K]^T, M = 128 output channels
// (weight rows past Cout read as zeros), N = 256 pixels of one output row.
//
// Pixel stages use the row-shift layout: one stage holds input pixels
// x0 - 1 .. x0 + 270 of one input row (two TMA boxes of 136 pixels) and one
// 64-channel block, and serves the three horizontal taps as N = 256 views
// starting one 128-byte swizzle row apart. Weight stages (one tap and
// channel block, 16 KB) stream through their own ring.
//
// Epilogue: TMEM row = output channel, so each thread holds one channel of
// 32 consecutive pixels. 16-bit NHWC results go to a 128-byte-swizzled
// shared tile (32 pixels x 128 channels per half-tile, double buffered) and
// leave through TMA bulk stores, and residuals are read one pixel per
// instruction across the warp's 32 channels (64 contiguous bytes): both keep
// the L1 traffic per instruction to whole lines, where one pixel per lane
// would touch 32 lines per instruction and slow the tensor core's
// shared-memory reads. The thin NCHW f32 output (conv_out) is written
// directly, 32 consecutive pixels per thread.
//
// Roles (384 threads): warp 0 pixel TMA producer, warp 1 TMEM allocator and
// MMA issuer, warp 2 weight TMA producer, warps 4..11 epilogue (two per TMEM
// lane quadrant, 128 pixels each).
//
// Fused input GroupNorm (FUSE = 1): the input is the raw activation; warps
// 8..11 normalise (+SiLU) each pixel stage in place (gn_stage.cuh) and the
// MMAs wait for their `pready` arrival instead of the TMA's. The epilogue
// then runs on warps 4..7 (one per lane quadrant, both 128-pixel halves).
//
// Reference counterpart: BandedConv2d::forward_checked
// (src/native/conv.rs:54-145).
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "conv_epilogue.cuh"
#include "conv_tc.h"
#include "gn_stage.cuh"

namespace osor {
namespace {

constexpr int kNM = 128;                       // MMA M: output channels
constexpr int kNN = 256;                       // MMA N: pixels per tile
constexpr int kNK = 64;                        // K block: 64 channels of one tap
constexpr int kBoxRows = 136;                  // pixels per TMA box (17 swizzle atoms)
constexpr int kPixStage = 2 * kBoxRows * 128;  // 272 pixel rows of 128 bytes
constexpr int kWStage = kNM * kNK * 2;         // 16 KB
constexpr int kFirstEpiWarp = 4;
constexpr int kThreadsN = 32 * (kFirstEpiWarp + 8);
// Epilogue warps: 8 (two per lane quadrant), or 4 when warps 8..11 transform.
template <int FUSE>
__host__ __device__ constexpr int epi_warps_n() {
  return FUSE ? 4 : 8;
}
constexpr int kXfWarp0 = kFirstEpiWarp + 4;
// Output staging: per half-tile and buffer, 32 pixels x 128 channels as two
// 64-channel TMA boxes of 32 x 128 bytes (4 KB each, 128-byte swizzle).
constexpr int kOutBox = 32 * 128;
constexpr int kOutTile = 2 * kOutBox;
// Ring depths and output buffers per variant. FUSE = 1 (the transform sits
// between a pixel stage's load and its MMAs) takes a fourth pixel stage, from
// one weight stage and the second warp set's output buffers.
template <int FUSE>
struct TcnShape {
  static constexpr int kPix = FUSE ? 4 : 3;
  static constexpr int kW = FUSE ? 4 : 5;
  static constexpr int kOutBufs = FUSE ? 2 : 4;  // [half][buffer], or FUSE: [buffer]
  static constexpr int kSmem = kPix * kPixStage + kW * kWStage + kOutBufs * kOutTile + 1024 + 256;
};

struct TcnParams {
  int tiles;       // batch * height * row_tiles
  int row_tiles;   // width / 256
  int height, width;
  int ksize, pad;  // 3 / 1
  int c_blocks;
  int units;       // pixel stages per tile: ksize * c_blocks, (ky, cb)
  const float* bias;
  const void* residual;
  long long ld_res;
  void* out;       // thin output only (16-bit output leaves through tmap_out)
  int cout;
  int out_nchw;    // f32 planes out[b][c][y][x] (cout <= 16)
  float* gn_part;  // per 128-pixel tile and group (mean, M2), CPG > 0
  int gn_groups;
  // FUSE = 1: GroupNorm(+SiLU) of the input from coef[img][c][4]; input rows
  // outside [in_y0, in_y1) are zero padding.
  const float* in_coef;
  int in_c, in_silu, in_y0, in_y1;
};

// Wait for the phases armed on `bars` (ring of n, next stage `stage` with
// parity `phase`) so no TMA write lands after the CTA has left.
__device__ void drain_ring(uint64_t* bars, int n, int stage, uint32_t phase) {
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

// Named barrier of the four epilogue warps of one half-tile (ids 2, 3).
__device__ __forceinline__ void half_sync(int bar) {
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
}

template <int D, int CPG, int FUSE>
__global__ void __launch_bounds__(kThreadsN, 1)
    conv_tcn_kernel(const __grid_constant__ CUtensorMap tmap_x,
                    const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_out, const TcnParams p) {
  using T = typename Elem<D>::T;
  constexpr int kEpiWarpsN = epi_warps_n<FUSE>();
  constexpr int kPixStages = TcnShape<FUSE>::kPix;
  constexpr int kWStages = TcnShape<FUSE>::kW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* pix = smem;
  uint8_t* wst = smem + kPixStages * kPixStage;
  uint8_t* out_tiles = wst + kWStages * kWStage;  // [half][buffer] (FUSE: [buffer]) kOutTile each
  uint64_t* pfull = reinterpret_cast<uint64_t*>(out_tiles + TcnShape<FUSE>::kOutBufs * kOutTile);
  uint64_t* pempty = pfull + kPixStages;
  uint64_t* wfull = pempty + kPixStages;
  uint64_t* wempty = wfull + kWStages;
  uint64_t* tfull = wempty + kWStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* pready = drain + 1;  // FUSE: pixel stage normalised
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pready + kPixStages);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPixStages; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 1);
      mbar_init(&pready[s], kXfThreads / 32);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarpsN);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
    if (!p.out_nchw) tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 2 * kNN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int per_image = p.height * p.row_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ pixel producer
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int img = t / per_image;
        const int r = t - img * per_image;
        const int y = r / p.row_tiles;
        const int x0 = (r - y * p.row_tiles) * kNN;
        for (int u = 0; u < p.units; ++u) {
          const int ky = u / p.c_blocks;
          const int cb = u - ky * p.c_blocks;
          if (!mbar_wait(&pempty[st], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&pfull[st], kPixStage);
          uint8_t* dst = pix + st * kPixStage;
          const int xs = x0 - p.pad, ys = y + ky - p.pad;
          tma_load_4d(dst, &tmap_x, &pfull[st], cb * kNK, xs, ys, img);
          tma_load_4d(dst + kBoxRows * 128, &tmap_x, &pfull[st], cb * kNK, xs + kBoxRows, ys,
                      img);
          if (++st == kPixStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) drain_ring(pfull, kPixStages, st, ph);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------------ weight producer
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        for (int u = 0; u < p.units && ok; ++u) {
          const int ky = u / p.c_blocks;
          const int cb = u - ky * p.c_blocks;
          for (int kx = 0; kx < p.ksize; ++kx) {
            if (!mbar_wait(&wempty[st], ph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&wfull[st], kWStage);
            const int kb = (ky * p.ksize + kx) * p.c_blocks + cb;
            tma_load_2d(wst + st * kWStage, &tmap_w, &wfull[st], kb * kNK, 0);
            if (++st == kWStages) {
              st = 0;
              ph ^= 1;
            }
          }
        }
      }
      if (!ok) drain_ring(wfull, kWStages, st, ph);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = umma_idesc_f32acc(kNM, kNN, Elem<D>::kUmmaFormat);
      int ps = 0, ws = 0, acc = 0;
      uint32_t pph = 0, wph = 0, aph = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kNN;
        for (int u = 0; u < p.units && ok; ++u) {
          if (!mbar_wait(FUSE ? &pready[ps] : &pfull[ps], pph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_base = smem_u32(pix + ps * kPixStage);
          for (int kx = 0; kx < p.ksize; ++kx) {
            if (!mbar_wait(&wfull[ws], wph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(wst + ws * kWStage);
            // Tap kx reads the pixel stage from row kx on: the 128-byte
            // swizzle follows the address bits, so a view may start on any
            // row of a swizzle atom.
#pragma unroll
            for (int k = 0; k < kNK / 16; ++k)
              umma_bf16(d_tmem, sw128_kmajor_desc(a_base + k * 32),
                        sw128_kmajor_desc(b_base + kx * 128 + k * 32), idesc, (u | kx | k) != 0);
            issued = true;
            umma_commit(&wempty[ws]);
            if (++ws == kWStages) {
              ws = 0;
              wph ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(&pempty[ps]);
          if (++ps == kPixStages) {
            ps = 0;
            pph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1;
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
  } else if (warp >= kFirstEpiWarp && warp < kFirstEpiWarp + kEpiWarpsN) {
    // ------------------------------------------------------ epilogue
    const int quad = warp & 3;                     // TMEM lanes = channels quad*32 ..
    // Pixels half*128 .. +127 of the tile; FUSE: both halves in turn.
    const int half0 = FUSE ? 0 : (warp - kFirstEpiWarp) >> 2;
    constexpr int kHalves = FUSE ? 2 : 1;
    const bool issuer = quad == 0 && lane == 0;    // TMA stores of this warp set
    const int c = quad * 32 + lane;
    const bool valid = c < p.cout;
    const float bias = (p.bias && valid) ? __ldg(p.bias + c) : 0.0f;
    // This thread's byte offset inside a staged 32 x 128 output tile for
    // pixel row 0: box c / 64, 16-byte chunk (c % 64) / 8 (XOR row & 7 per
    // row), element c % 8.
    const int obox = (c >> 6) * kOutBox;
    const int ochunk = (c & 63) >> 3;
    const int oelem = (c & 7) * 2;
    uint32_t stores = 0;  // chunks staged by this half so far (buffer = stores & 1)
    int acc = 0;
    uint32_t aph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
      const int img = t / per_image;
      const int r = t - img * per_image;
      const int y = r / p.row_tiles;
      const bool nhwc = !p.out_nchw;
      for (int hh = 0; hh < kHalves; ++hh) {
        const int half = half0 + hh;
        const int hbar = 2 + half;
        const int xh = (r - y * p.row_tiles) * kNN + half * 128;  // first pixel of this half
        const long long pix0 = ((long long)img * p.height + y) * p.width + xh;
        // Residuals of chunk 0 (later chunks are fetched one chunk ahead):
        // pixel k of the chunk, this thread's channel.
        T res[32];
        if (nhwc && p.residual && valid) {
          const T* rs = static_cast<const T*>(p.residual) + pix0 * p.ld_res + c;
#pragma unroll
          for (int k = 0; k < 32; ++k) res[k] = rs[(long long)k * p.ld_res];
        }
        // All four warps of a half wait on the same tfull phase with the same
        // abort flag, so a failed wait is seen by all of them and the named
        // barriers below stay matched.
        if (hh == 0) {
          if (!mbar_wait(&tfull[acc], aph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        float prev_m = 0.0f, prev_q = 0.0f, run_m = 0.0f, run_q = 0.0f;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t rv[32];
          tmem_load_32x32b_x32(
              tmem_base + ((uint32_t)(quad * 32) << 16) + acc * kNN + half * 128 + ch * 32, rv);
          tmem_wait_ld();
          if (ch == 3 && hh == kHalves - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
          float v[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(rv[k]) + bias;
          if (!nhwc) {
            if (valid) {
              float4* o = reinterpret_cast<float4*>(
                  static_cast<float*>(p.out) +
                  (((long long)img * p.cout + c) * p.height + y) * p.width + xh + ch * 32);
#pragma unroll
              for (int k = 0; k < 8; ++k)
                o[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
            }
            continue;
          }
          if (p.residual && valid) {
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] += Elem<D>::to_f(res[k]);
            if (ch < 3) {
              const T* rs =
                  static_cast<const T*>(p.residual) + (pix0 + (ch + 1) * 32) * p.ld_res + c;
#pragma unroll
              for (int k = 0; k < 32; ++k) res[k] = rs[(long long)k * p.ld_res];
            }
          }
          // Stage the 16-bit chunk: pixel k, channel c.
          const int obuf = FUSE ? (int)(stores & 1) : half * 2 + (int)(stores & 1);
          uint8_t* tile = out_tiles + obuf * kOutTile + obox + oelem;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const T h = Elem<D>::from_f(v[k]);
            *reinterpret_cast<T*>(tile + k * 128 + ((ochunk ^ (k & 7)) << 4)) = h;
            v[k] = Elem<D>::to_f(h);  // statistics of the stored value
          }
          fence_proxy_async_smem();
          // Before the barrier the issuer makes sure its previous store has
          // finished reading the other buffer, which the next chunk writes.
          if (issuer) bulk_wait_group_read<0>();
          half_sync(hbar);
          if (issuer) {
            const uint8_t* src = out_tiles + obuf * kOutTile;
            const int prow = (int)(pix0 + ch * 32);
            tma_store_2d(&tmap_out, src, 0, prow);
            if (p.cout > 64) tma_store_2d(&tmap_out, src + kOutBox, 64, prow);
            bulk_commit_group();
          }
          ++stores;
          if constexpr (CPG > 0) {
            // This channel's 32 pixels, then the group's CPG channels (lanes).
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; ++k) s += v[k];
            float mean = s * (1.0f / 32.0f);
            float m2 = 0.0f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float d = v[k] - mean;
              m2 += d * d;
            }
            float n = 32.0f;
#pragma unroll
            for (int o = 1; o < CPG; o <<= 1) {
              const float mo = __shfl_xor_sync(0xffffffffu, mean, o);
              const float qo = __shfl_xor_sync(0xffffffffu, m2, o);
              merge_equal_counts(mean, m2, mo, qo, n);
              n *= 2.0f;
            }
            // Chunks merge as a pairwise tree: (0, 1), (2, 3), then both.
            const float nc = 32.0f * CPG;
            if ((ch & 1) == 0) {
              prev_m = mean;
              prev_q = m2;
            } else {
              merge_equal_counts(prev_m, prev_q, mean, m2, nc);
              if (ch == 1) {
                run_m = prev_m;
                run_q = prev_q;
              } else {
                merge_equal_counts(run_m, run_q, prev_m, prev_q, 2.0f * nc);
              }
            }
          }
        }
        if constexpr (CPG > 0) {
          if (nhwc && valid && (lane & (CPG - 1)) == 0) {
            float* dst = p.gn_part + ((pix0 >> 7) * p.gn_groups + c / CPG) * 2;
            dst[0] = run_m;
            dst[1] = run_q;
          }
        }
      }
      if (!ok) break;
      if (++acc == 2) {
        acc = 0;
        aph ^= 1;
      }
    }
    if (issuer) bulk_wait_group<0>();
  } else if (FUSE && warp >= kXfWarp0) {
    // ------------------------------------------------------ transform
    // Same tile / unit order as the pixel producer: wait for the stage,
    // normalise its 256 + ksize - 1 pixel rows, release it to the MMAs.
    const int tid = threadIdx.x - 32 * kXfWarp0;
    int st = 0;
    uint32_t ph = 0;
    bool ok = true;
    float4 raw[8];  // coefficients of the next unit, fetched one unit ahead
    if ((int)blockIdx.x < p.tiles)
      gn_stage_coef_fetch(p.in_coef, (int)blockIdx.x / per_image, p.in_c, 0, tid, raw);
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
      const int img = t / per_image;
      const int r = t - img * per_image;
      const int y = r / p.row_tiles;
      const int x0 = (r - y * p.row_tiles) * kNN;
      for (int u = 0; u < p.units; ++u) {
        const int ky = u / p.c_blocks;
        const int cb = u - ky * p.c_blocks;
        const int ys = y + ky - p.pad;
        StageCoef<D> k;
        gn_stage_coef_prepare<D>(raw, p.in_silu != 0, k);
        {
          const int nt = u + 1 < p.units ? t : t + (int)gridDim.x;
          gn_stage_coef_fetch(p.in_coef, nt < p.tiles ? nt / per_image : img, p.in_c,
                              u + 1 < p.units ? (cb + 1) % p.c_blocks : 0, tid, raw);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&pfull[st], ph, abort_flag))) {
          ok = false;
          break;
        }
        gn_stage_apply<D>(pix + st * kPixStage, kNN + p.ksize - 1, x0 - p.pad, p.width,
                          ys >= p.in_y0 && ys < p.in_y1, k, p.in_silu != 0, tid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pready[st]);
        if (++st == kPixStages) {
          st = 0;
          ph ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kNN);
  }
}

typedef CUresult (*EncodeTiledFnN)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnN encode_fn_n() {
  static EncodeTiledFnN fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnN>(ptr);
    return static_cast<EncodeTiledFnN>(nullptr);
  }();
  return fn;
}

template <int D, int CPG, int FUSE>
cudaError_t launch_n(const CUtensorMap& tx, const CUtensorMap& tw, const CUtensorMap& to,
                     const TcnParams& p, cudaStream_t stream) {
  static std::atomic<int> sms[64];  // zero-initialized; atomic for concurrent callers
  int device = 0;
  cudaGetDevice(&device);
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (sms[device] == 0) {
    cudaError_t e = cudaFuncSetAttribute(conv_tcn_kernel<D, CPG, FUSE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         TcnShape<FUSE>::kSmem);
    if (e != cudaSuccess) return e;
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    sms[device] = n > 0 ? n : 148;
  }
  const int resident = sms[device].load();
  const int grid = p.tiles < resident ? p.tiles : resident;
  conv_tcn_kernel<D, CPG, FUSE><<<grid, kThreadsN, TcnShape<FUSE>::kSmem, stream>>>(tx, tw, to, p);
  return cudaGetLastError();
}

template <int FUSE>
cudaError_t launch_cpg_n(int dtype, int cpg, const CUtensorMap& tx, const CUtensorMap& tw,
                         const CUtensorMap& to, const TcnParams& p, cudaStream_t stream) {
  if (dtype == kF16) {
    switch (cpg) {
      case 4: return launch_n<kF16, 4, FUSE>(tx, tw, to, p, stream);
      case 8: return launch_n<kF16, 8, FUSE>(tx, tw, to, p, stream);
      case 16: return launch_n<kF16, 16, FUSE>(tx, tw, to, p, stream);
      default: return launch_n<kF16, 0, FUSE>(tx, tw, to, p, stream);
    }
  }
  switch (cpg) {
    case 4: return launch_n<kBf16, 4, FUSE>(tx, tw, to, p, stream);
    case 8: return launch_n<kBf16, 8, FUSE>(tx, tw, to, p, stream);
    case 16: return launch_n<kBf16, 16, FUSE>(tx, tw, to, p, stream);
    default: return launch_n<kBf16, 0, FUSE>(tx, tw, to, p, stream);
  }
}

}  // namespace

const char* conv_tcn_check(const ConvTcArgs& a) {
  if (a.upsample || a.row_scale || a.softmax_stats || a.softmax_max || a.geglu)
    return "pixel-N kernel: plain convolution only";
  if (!((a.ksize == 3 && a.pad == 1) || (a.ksize == 1 && a.pad == 0)) || a.stride != 1)
    return "pixel-N kernel: 3x3 pad 1 or 1x1, stride 1";
  if (a.out_h != a.in_h || a.out_w != a.in_w) return "pixel-N kernel: same-size output";
  if (a.out_w <= 0 || a.out_h <= 0 || a.batch <= 0) return "empty convolution";
  if (a.out_w % kNN != 0) return "pixel-N kernel: width must be a multiple of 256";
  if (a.cin <= 0 || a.cin % kNK != 0) return "pixel-N kernel: Cin % 64";
  if (a.out_nchw) {
    if (a.cout <= 0 || a.cout > 16 || !a.out_f32 || a.residual || a.gn_part)
      return "pixel-N kernel: thin NCHW output needs 1..16 f32 channels";
    if (reinterpret_cast<uintptr_t>(a.out) & 15) return "output alignment";
  } else {
    if (a.out_f32 || (a.cout != 64 && a.cout != kNM))
      return "pixel-N kernel: 16-bit output with Cout 64 or 128";
    if (a.ld_out % 8 != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15)) return "output alignment";
    if (a.residual && (a.ld_res <= 0 || (reinterpret_cast<uintptr_t>(a.residual) & 1)))
      return "residual alignment";
    if (a.gn_part && (a.cout != kNM || (a.gn_cpg != 4 && a.gn_cpg != 8 && a.gn_cpg != 16)))
      return "pixel-N kernel: statistics need Cout 128 and 4, 8 or 16 channels per group";
  }
  if (a.pixel_stride % 8 != 0 || a.ldw % 8 != 0) return "strides";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w)) & 15)
    return "alignment";
  if (a.dtype != kBf16 && a.dtype != kF16) return "dtype";
  if ((long long)a.batch * a.out_h * a.out_w > 0x7fffffffLL) return "problem too large";
  if (a.in_coef) {
    if (a.out_nchw) return "pixel-N kernel: fused input GroupNorm with a 16-bit output only";
    if (reinterpret_cast<uintptr_t>(a.in_coef) & 15) return "pixel-N kernel: coefficient alignment";
    if (a.in_y0 < 0 || (a.in_y1 >= 0 && (a.in_y1 < a.in_y0 || a.in_y1 > a.in_h)))
      return "pixel-N kernel: input row range";
  }
  return nullptr;
}

cudaError_t conv_tcn_launch(const ConvTcArgs& a, cudaStream_t stream) {
  EncodeTiledFnN encode = encode_fn_n();
  if (!encode) return cudaErrorNotSupported;
  const CUtensorMapDataType tdt =
      a.dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tx, tw, to;
  {
    const cuuint64_t ps = (cuuint64_t)a.pixel_stride * 2;
    cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in_w, (cuuint64_t)a.in_h,
                          (cuuint64_t)a.batch};
    cuuint64_t strides[3] = {ps, ps * a.in_w, ps * a.in_w * a.in_h};
    cuuint32_t box[4] = {(cuuint32_t)kNK, (cuuint32_t)kBoxRows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    if (encode(&tx, tdt, 4, const_cast<void*>(a.x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    // Weight rows past Cout: the caller's zero padding when it allocated 128
    // rows, else outside the tensor (the box reads them as zeros).
    const int k_total = a.ksize * a.ksize * a.cin;
    const int rows = a.w_rows >= kNM ? kNM : a.cout;
    cuuint64_t dims[2] = {(cuuint64_t)k_total, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldw * 2};
    cuuint32_t box[2] = {(cuuint32_t)kNK, (cuuint32_t)kNM};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&tw, tdt, 2, const_cast<void*>(a.w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (!a.out_nchw) {
    // Output rows (pixels) of ld_out elements; boxes of 64 channels x 32 pixels.
    cuuint64_t dims[2] = {(cuuint64_t)a.cout, (cuuint64_t)a.batch * a.out_h * a.out_w};
    cuuint64_t strides[1] = {(cuuint64_t)a.ld_out * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&to, tdt, 2, a.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    to = tx;  // unused by the thin output
  }
  TcnParams p;
  p.row_tiles = a.out_w / kNN;
  p.height = a.out_h;
  p.width = a.out_w;
  p.tiles = a.batch * a.out_h * p.row_tiles;
  p.ksize = a.ksize;
  p.pad = a.pad;
  p.c_blocks = a.cin / kNK;
  p.units = a.ksize * p.c_blocks;
  p.bias = a.bias;
  p.residual = a.residual;
  p.ld_res = a.ld_res;
  p.out = a.out;
  p.cout = a.cout;
  p.out_nchw = a.out_nchw;
  const int cpg = a.gn_part ? a.gn_cpg : 0;
  p.gn_part = a.gn_part;
  p.gn_groups = cpg ? a.cout / cpg : 0;
  p.in_coef = a.in_coef;
  p.in_c = a.cin;
  p.in_silu = a.in_silu;
  p.in_y0 = a.in_y0;
  p.in_y1 = a.in_y1 < 0 ? a.in_h : a.in_y1;
  if (a.in_coef) return launch_cpg_n<1>(a.dtype, cpg, tx, tw, to, p, stream);
  return launch_cpg_n<0>(a.dtype, cpg, tx, tw, to, p, stream);
}

}  // namespace osor
