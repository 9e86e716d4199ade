// The decoder's last two layers in one pass: GroupNorm(+SiLU) apply of the
// final 128-channel activation and the 3x3 convolution to RGB
// (conv_norm_out + SiLU + conv_out, src/native/vae_decoder.rs:112-113).
//
// A 3x3 convolution with 3 output channels is thin: as an implicit GEMM with
// the pixels on M every tcgen05.mma would produce 3 useful columns of 16, and
// the pixels-on-N form pads the weight side from 3 to 128 rows. Here the GEMM
// runs per input pixel instead: Z[p][n] = S[p][:] . W'[n][:] with
// n = (ky * 3 + kx) * 3 + co (27 of N = 32 columns used, K = 128 channels), so
// one M = 128, N = 32, K = 16 instruction covers 128 pixels' contributions to
// all nine taps. The 3x3 neighbourhood sum is done in the epilogue:
// out[y][x][co] = bias[co] + sum over (ky, kx) of Z[(y + ky - 1, x + kx - 1)][(ky, kx, co)].
// Horizontal taps come from the neighbouring TMEM lanes (warp shuffles; the
// two edge lanes of each warp through shared memory), vertical taps from
// three rolling row accumulators in registers: input row yi adds its ky = 2
// terms to output row yi - 1 (then complete and stored), ky = 1 to row yi and
// ky = 0 to row yi + 1.
//
// S = silu(GroupNorm(x)) is applied once per element in shared memory between
// the TMA load and the MMA (the convolution's zero padding applies to S:
// pixels past the image's right edge are zeroed, rows outside it skipped), so
// the normalized activation never goes to HBM: one read of x, one write of
// the f32 image.
//
// Each CTA (one per SM) owns a band of whole rows of one image (two segments
// when its band crosses an image boundary) and reads the band plus one halo
// row above and below. Roles (576 threads): warp 0 TMA producer, warp 1 TMEM
// allocator and MMA issuer, warps 2..9 the GroupNorm transform (the
// elementwise work dominates: eight warps keep the schedulers issuing), warps
// 10..17 the epilogue (warp w reads TMEM lane quadrant w % 4; warps 10..13 own
// tiles 0..3 of the row and warps 14..17 tiles 4..7, one pixel per thread and
// tile). Two TMEM row buffers of 8 tiles x 32 columns let the MMAs of row
// yi + 1 run under the epilogue of row yi.
#include <atomic>

#include "common.cuh"
#include "conv_out.h"
#include "device_guard.h"

namespace osor {
namespace {

constexpr int kTilePx = 128;                     // MMA M: pixels per tile
constexpr int kCin = 128;                        // input channels: two 64-channel boxes
constexpr int kBoxBytes = kTilePx * 128;         // 128 pixels x 64 channels (16 KB)
constexpr int kStageBytes = 2 * kBoxBytes;       // one tile of one row, all channels
constexpr int kStages = 6;
constexpr int kN = 32;                           // MMA N: (ky, kx, co), 27 used
constexpr int kCout = 3;
constexpr int kMaxTiles = 8;                     // width <= 1024
constexpr int kRowCols = kMaxTiles * kN;         // TMEM columns per row buffer
constexpr int kWBoxBytes = kN * 128;             // 32 weight rows x 64 channels (4 KB)
constexpr int kFirstTransformWarp = 2;
constexpr int kTransformWarps = 8;
constexpr int kFirstEpiWarp = 10;
constexpr int kEpiWarps = 8;                     // two per TMEM lane quadrant
constexpr int kEpiTiles = kMaxTiles / 2;         // tiles per epilogue warp
constexpr int kThreads = 32 * (kFirstEpiWarp + kEpiWarps);
// Edge exchange: [row parity][side][tile][quadrant][ky * 3 + co].
constexpr int kEdgeFloats = 2 * 2 * kMaxTiles * 4 * 9;
constexpr int kSmem = kStages * kStageBytes + 2 * kWBoxBytes + kEdgeFloats * 4 + 256 + 1024;

struct OutParams {
  int batch, height, width, tiles;
  const float* coef;  // [batch][kCin][4]: (mean, rstd * gamma, beta, -)
  int silu;
  int normalize;      // 0: S = x (a plain 3x3 convolution; coef unused)
  int w_conv;         // 1: weights in the convolution layout [cout][3][3][cin] at wconv
  const uint16_t* wconv;
  const float* bias;  // [kCout]
  float* out;         // [batch][kCout][height][width]
};

// Wait for the phases armed on the last n stages of a ring so that no TMA
// write lands after the CTA has left (bounded).
__device__ void drain_stages(uint64_t* bars, int n, int stage, uint32_t phase) {
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

// Named barrier 1 over the eight epilogue warps (256 threads), returning the
// OR of `v` over them: every epilogue thread takes the same branch after it.
__device__ __forceinline__ bool epi_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "barrier.red.or.pred p, 1, 256, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

// The CTA's rows: [r_begin, r_end) of the (image, row) sequence, split at
// image boundaries into segments; each segment reads rows y0 - 1 .. y1.
struct Rows {
  long long begin, end;
  __device__ Rows(int batch, int height) {
    const long long total = (long long)batch * height;
    begin = (long long)blockIdx.x * total / gridDim.x;
    end = (long long)(blockIdx.x + 1) * total / gridDim.x;
  }
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    gn_conv_out_kernel(const __grid_constant__ CUtensorMap tmap_x,
                       const __grid_constant__ CUtensorMap tmap_w, const OutParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* wz = stages + kStages * kStageBytes;
  float* edges = reinterpret_cast<float*>(wz + 2 * kWBoxBytes);
  uint64_t* pfull = reinterpret_cast<uint64_t*>(edges + kEdgeFloats);
  uint64_t* pempty = pfull + kStages;
  uint64_t* xready = pempty + kStages;
  uint64_t* tfull = xready + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* wfull = tempty + 2;
  uint64_t* drain = wfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 1);
      mbar_init(&xready[s], kTransformWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(wfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 2 * kRowCols);
    tmem_relinquish();
  }
  if (p.w_conv && threadIdx.x < 2 * kN * 8) {
    // Convolution-layout weights [co][ky][kx][ci] into the operand's
    // tap-major rows (ky * 3 + kx) * 3 + co, 16 bytes per thread, in the
    // 128-byte swizzled layout (chunk j of row r at j ^ (r % 8)); rows 27..31
    // of the N = 32 operand are zero.
    const int box = threadIdx.x / (kN * 8), rem = threadIdx.x % (kN * 8);
    const int r = rem >> 3, j = rem & 7;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < 9 * kCout) {
      const int tap = r / kCout, co = r % kCout;
      v = __ldg(reinterpret_cast<const uint4*>(p.wconv + ((long long)co * 9 + tap) * kCin +
                                               box * 64 + j * 8));
    }
    *reinterpret_cast<uint4*>(wz + box * kWBoxBytes + r * 128 + ((j ^ (r & 7)) << 4)) = v;
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const Rows rows(p.batch, p.height);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      if (p.w_conv) {
        mbar_arrive(wfull);  // the weights were stored before the setup barrier
      } else {
        mbar_arrive_expect_tx(wfull, 2 * kWBoxBytes);
        tma_load_2d(wz, &tmap_w, wfull, 0, 0);
        tma_load_2d(wz + kWBoxBytes, &tmap_w, wfull, 64, 0);
      }
      int st = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (long long r = rows.begin; r < rows.end && ok;) {
        const int img = (int)(r / p.height);
        const int y0 = (int)(r - (long long)img * p.height);
        const int y1 = (int)min((long long)p.height, y0 + (rows.end - r));
        r += y1 - y0;
        for (int yi = max(y0 - 1, 0); yi <= min(y1, p.height - 1) && ok; ++yi) {
          for (int t = 0; t < p.tiles; ++t) {
            if (!mbar_wait(&pempty[st], ph ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&pfull[st], kStageBytes);
            uint8_t* dst = stages + st * kStageBytes;
            tma_load_4d(dst, &tmap_x, &pfull[st], 0, t * kTilePx, yi, img);
            tma_load_4d(dst + kBoxBytes, &tmap_x, &pfull[st], 64, t * kTilePx, yi, img);
            if (++st == kStages) {
              st = 0;
              ph ^= 1;
            }
          }
        }
      }
      if (!ok) drain_stages(pfull, kStages, st, ph);
      // The weight load completes before the MMA issuer starts; wait for it
      // here as well in case the issuer gave up first.
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(smem_u32(wfull), 0) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = umma_idesc_f32acc(kTilePx, kN, Elem<D>::kUmmaFormat);
      bool ok = mbar_wait(wfull, 0, abort_flag);
      tc_fence_after();
      const uint32_t b_base = smem_u32(wz);
      int st = 0, rb = 0;
      uint32_t ph = 0, rph = 0;
      bool issued = false;
      for (long long r = rows.begin; r < rows.end && ok;) {
        const int img = (int)(r / p.height);
        const int y0 = (int)(r - (long long)img * p.height);
        const int y1 = (int)min((long long)p.height, y0 + (rows.end - r));
        r += y1 - y0;
        for (int yi = max(y0 - 1, 0); yi <= min(y1, p.height - 1) && ok; ++yi) {
          if (!mbar_wait(&tempty[rb], rph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int t = 0; t < p.tiles; ++t) {
            if (!mbar_wait(&xready[st], ph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(stages + st * kStageBytes);
            const uint32_t d_tmem = tmem_base + rb * kRowCols + t * kN;
#pragma unroll
            for (int cb = 0; cb < 2; ++cb)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_bf16(d_tmem, sw128_kmajor_desc(a_base + cb * kBoxBytes + k * 32),
                          sw128_kmajor_desc(b_base + cb * kWBoxBytes + k * 32), idesc,
                          (cb | k) != 0);
            issued = true;
            umma_commit(&pempty[st]);
            if (++st == kStages) {
              st = 0;
              ph ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(&tfull[rb]);
          if (++rb == 2) {
            rb = 0;
            rph ^= 1;
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
  } else if (warp >= kFirstTransformWarp && warp < kFirstTransformWarp + kTransformWarps) {
    // ------------------------------------------------------ GroupNorm transform
    // Thread k handles 16-byte chunk position q = k % 8 of rows k / 8 + 32 m of
    // both boxes; with the 128-byte swizzle (chunk j of row r at position
    // j ^ (r % 8)) that position always holds logical chunk j, i.e. channels
    // box * 64 + j * 8 .. + 7, so the thread keeps 16 coefficient pairs.
    const int k = threadIdx.x - 32 * kFirstTransformWarp;
    const int q = k & 7, row0 = k >> 3;
    const int j = q ^ (row0 & 7);
    const bool silu = p.silu != 0;
    float ca[2][8], cb[2][8];
    int cur_img = -1;
    int st = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (long long r = rows.begin; r < rows.end && ok;) {
      const int img = (int)(r / p.height);
      const int y0 = (int)(r - (long long)img * p.height);
      const int y1 = (int)min((long long)p.height, y0 + (rows.end - r));
      r += y1 - y0;
      if (img != cur_img && p.normalize) {
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 c = __ldg(reinterpret_cast<const float4*>(p.coef) +
                                   (long long)img * kCin + b * 64 + j * 8 + e);
            gn_coef_prepare(c.x, c.y, c.z, silu, ca[b][e], cb[b][e]);
          }
        cur_img = img;
      }
      for (int yi = max(y0 - 1, 0); yi <= min(y1, p.height - 1) && ok; ++yi) {
        for (int t = 0; t < p.tiles; ++t) {
          if (!mbar_wait(&pfull[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sbuf = stages + st * kStageBytes;
          const int valid_px = min(kTilePx, p.width - t * kTilePx);
          // Without the normalisation the stage is the convolution's input
          // as loaded (the TMA zero fill covers the pixels past the edge).
#pragma unroll
          for (int b = 0; b < (p.normalize ? 2 : 0); ++b) {
#pragma unroll 4
            for (int m = 0; m < kTilePx / 32; ++m) {
              const int row = row0 + 32 * m;
              uint4* ptr = reinterpret_cast<uint4*>(sbuf + b * kBoxBytes + row * 128 + q * 16);
              if (row < valid_px) {
                float f[8];
                unpack8<D>(*ptr, f);
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = gn_apply_prepared(f[e], ca[b][e], cb[b][e], silu);
                *ptr = pack8<D>(f);
              } else {
                *ptr = make_uint4(0u, 0u, 0u, 0u);  // past the right edge: zero padding
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&xready[st]);
          if (++st == kStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp >= kFirstEpiWarp) {
    // ------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lanes quad * 32 ..: warps 10..13 take quadrants 2, 3, 0, 1
    const int t0 = ((warp - kFirstEpiWarp) >> 2) * kEpiTiles;  // this warp's first tile
    const float bias0 = __ldg(p.bias), bias1 = __ldg(p.bias + 1), bias2 = __ldg(p.bias + 2);
    // Output rows yi - 1, yi, yi + 1 for this thread's pixel of each tile.
    float acc_a[kEpiTiles][kCout], acc_b[kEpiTiles][kCout], acc_c[kEpiTiles][kCout];
    int rb = 0;
    uint32_t rph = 0;
    int step = 0;
    bool stop = false;
    for (long long r = rows.begin; r < rows.end && !stop;) {
      const int img = (int)(r / p.height);
      const int y0 = (int)(r - (long long)img * p.height);
      const int y1 = (int)min((long long)p.height, y0 + (rows.end - r));
      r += y1 - y0;
#pragma unroll
      for (int i = 0; i < kEpiTiles; ++i)
#pragma unroll
        for (int c = 0; c < kCout; ++c) {
          acc_a[i][c] = 0.0f;
          acc_b[i][c] = 0.0f;
        }
      for (int yi = y0 - 1; yi <= y1; ++yi, ++step) {
        const bool valid = yi >= 0 && yi < p.height;
        bool bad = false;
        if (valid) bad = !mbar_wait(&tfull[rb], rph, abort_flag);
        if (epi_any(bad)) {
          stop = true;
          break;
        }
        tc_fence_after();
        float* edge_out = edges + (step & 1) * (2 * kMaxTiles * 4 * 9);
#pragma unroll
        for (int i = 0; i < kEpiTiles; ++i) {
          const int t = t0 + i;
          if (t >= p.tiles) break;
          // One tap row (ky) of this pixel: z9[kx * 3 + co].
          float* e_right = edge_out + ((0 * kMaxTiles + t) * 4 + quad) * 9;
          float* e_left = edge_out + ((1 * kMaxTiles + t) * 4 + quad) * 9;
          auto tap_row = [&](const float (&z9)[9], int ky) {
#pragma unroll
            for (int c = 0; c < kCout; ++c) {
              // Output x reads input x + kx - 1: kx = 1 from its own pixel,
              // kx = 0 from x - 1 and kx = 2 from x + 1 (the lanes beside it;
              // the warp's edge lanes get the other warp's value after the
              // barrier below).
              const float left = __shfl_up_sync(0xffffffffu, z9[0 * kCout + c], 1);
              const float right = __shfl_down_sync(0xffffffffu, z9[2 * kCout + c], 1);
              float h = z9[1 * kCout + c];
              if (lane > 0) h += left;
              if (lane < 31) h += right;
              if (ky == 2) acc_a[i][c] += h;
              if (ky == 1) acc_b[i][c] += h;
              if (ky == 0) acc_c[i][c] = h;
              // For the pixel to the right (lane 31): this pixel's kx = 0
              // term; for the pixel to the left (lane 0): its kx = 2 term.
              if (lane == 31) e_right[ky * 3 + c] = z9[0 * kCout + c];
              if (lane == 0) e_left[ky * 3 + c] = z9[2 * kCout + c];
            }
          };
          // Columns 0..15 hold tap row 0 and most of row 1, columns 16..31
          // the rest of row 1 and row 2: two 16-column loads keep fewer
          // registers live than one of 32.
          float z0[9], z1[9], z2[9];
          uint32_t rv[16];
          const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + rb * kRowCols + t * kN;
          if (valid) {
            tmem_load_32x32b_x16(taddr, rv);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int n = 0; n < 16; ++n) rv[n] = 0u;
          }
#pragma unroll
          for (int n = 0; n < 9; ++n) z0[n] = __uint_as_float(rv[n]);
#pragma unroll
          for (int n = 0; n < 7; ++n) z1[n] = __uint_as_float(rv[9 + n]);
          tap_row(z0, 0);
          if (valid) {
            tmem_load_32x32b_x16(taddr + 16, rv);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int n = 0; n < 16; ++n) rv[n] = 0u;
          }
          z1[7] = __uint_as_float(rv[0]);
          z1[8] = __uint_as_float(rv[1]);
#pragma unroll
          for (int n = 0; n < 9; ++n) z2[n] = __uint_as_float(rv[2 + n]);
          tap_row(z1, 1);
          tap_row(z2, 2);
        }
        if (valid) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[rb]);
          if (++rb == 2) {
            rb = 0;
            rph ^= 1;
          }
        }
        epi_sync();  // edges of this row visible to every epilogue warp
#pragma unroll
        for (int i = 0; i < kEpiTiles; ++i) {
          const int t = t0 + i;
          if (t >= p.tiles) break;
          const float* e = nullptr;
          if (lane == 0) {  // left neighbour: lane 31 of the previous quadrant / tile
            if (quad > 0)
              e = edge_out + ((0 * kMaxTiles + t) * 4 + quad - 1) * 9;
            else if (t > 0)
              e = edge_out + ((0 * kMaxTiles + t - 1) * 4 + 3) * 9;
          } else if (lane == 31) {  // right neighbour: lane 0 of the next quadrant / tile
            if (quad < 3)
              e = edge_out + ((1 * kMaxTiles + t) * 4 + quad + 1) * 9;
            else if (t + 1 < p.tiles)
              e = edge_out + ((1 * kMaxTiles + t + 1) * 4 + 0) * 9;
          }
          if (e) {
#pragma unroll
            for (int c = 0; c < kCout; ++c) {
              acc_a[i][c] += e[2 * 3 + c];
              acc_b[i][c] += e[1 * 3 + c];
              acc_c[i][c] += e[0 * 3 + c];
            }
          }
        }
        // Output row yi - 1 is complete.
        const int yo = yi - 1;
        if (yo >= y0 && yo < y1) {
#pragma unroll
          for (int i = 0; i < kEpiTiles; ++i) {
            const int t = t0 + i;
            if (t >= p.tiles) break;
            const int x = t * kTilePx + quad * 32 + lane;
            if (x < p.width) {
              float* o = p.out + (((long long)img * kCout) * p.height + yo) * p.width + x;
              const long long plane = (long long)p.height * p.width;
              o[0] = acc_a[i][0] + bias0;
              o[plane] = acc_a[i][1] + bias1;
              o[2 * plane] = acc_a[i][2] + bias2;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kEpiTiles; ++i)
#pragma unroll
          for (int c = 0; c < kCout; ++c) {
            acc_a[i][c] = acc_b[i][c];
            acc_b[i][c] = acc_c[i][c];
          }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kRowCols);
  }
}

typedef CUresult (*EncodeTiledFnO)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFnO encode_fn_o() {
  static EncodeTiledFnO fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFnO>(ptr);
    return static_cast<EncodeTiledFnO>(nullptr);
  }();
  return fn;
}

PerDeviceOnce g_smem_set[2];
std::atomic<int> g_sms[kMaxDevices];

}  // namespace

const char* gn_conv_out_check(const GnConvOutArgs& a) {
  if (a.dtype != kBf16 && a.dtype != kF16) return "dtype";
  if (a.cin != kCin) return "fused conv_out: 128 input channels";
  if (a.cout != kCout) return "fused conv_out: 3 output channels";
  if (a.batch <= 0 || a.height <= 0 || a.width <= 0) return "empty convolution";
  if (a.width > kMaxTiles * kTilePx) return "fused conv_out: width <= 1024";
  if (!a.x || !a.wz || (a.normalize && !a.coef) || !a.bias || !a.out) return "null argument";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.wz) |
       reinterpret_cast<uintptr_t>(a.coef)) & 15)
    return "alignment";
  return nullptr;
}

cudaError_t gn_conv_out_launch(const GnConvOutArgs& a, cudaStream_t stream) {
  if (gn_conv_out_check(a) != nullptr) return cudaErrorInvalidValue;
  EncodeTiledFnO encode = encode_fn_o();
  if (!encode) return cudaErrorNotSupported;
  const CUtensorMapDataType tdt =
      a.dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tx, tw;
  {
    cuuint64_t dims[4] = {(cuuint64_t)kCin, (cuuint64_t)a.width, (cuuint64_t)a.height,
                          (cuuint64_t)a.batch};
    const cuuint64_t ps = (cuuint64_t)kCin * 2;
    cuuint64_t strides[3] = {ps, ps * a.width, ps * a.width * a.height};
    cuuint32_t box[4] = {64, (cuuint32_t)kTilePx, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    if (encode(&tx, tdt, 4, const_cast<void*>(a.x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (a.w_conv) {
    // The kernel stores the convolution-layout weights itself; the weight
    // map is unused (a copy of the input's keeps the parameter valid).
    tw = tx;
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)kCin, (cuuint64_t)kN};
    cuuint64_t strides[1] = {(cuuint64_t)kCin * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kN};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&tw, tdt, 2, const_cast<void*>(a.wz), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  OutParams p;
  p.batch = a.batch;
  p.height = a.height;
  p.width = a.width;
  p.tiles = (a.width + kTilePx - 1) / kTilePx;
  p.coef = a.coef;
  p.silu = a.silu;
  p.normalize = a.normalize;
  p.w_conv = a.w_conv;
  p.wconv = static_cast<const uint16_t*>(a.wz);
  p.bias = a.bias;
  p.out = a.out;
  const int di = a.dtype == kF16 ? 1 : 0;
  cudaError_t e = g_smem_set[di].run([&] {
    return a.dtype == kF16 ? cudaFuncSetAttribute(gn_conv_out_kernel<kF16>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  kSmem)
                           : cudaFuncSetAttribute(gn_conv_out_kernel<kBf16>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  kSmem);
  });
  if (e != cudaSuccess) return e;
  int device = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  int sms = g_sms[device].load();
  if (sms == 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (sms <= 0) sms = 148;
    g_sms[device].store(sms);
  }
  const long long rows = (long long)a.batch * a.height;
  const int grid = rows < sms ? (int)rows : sms;
  if (a.dtype == kF16)
    gn_conv_out_kernel<kF16><<<grid, kThreads, kSmem, stream>>>(tx, tw, p);
  else
    gn_conv_out_kernel<kBf16><<<grid, kThreads, kSmem, stream>>>(tx, tw, p);
  return cudaGetLastError();
}

}  // namespace osor
