// Implicit-GEMM convolution / GEMM on the sm_100a tensor cores.
//
// One kernel covers every tensor-core contraction of the VAE:
//   * 3x3 stride-1 pad-1 and 1x1 convolutions over NHWC bf16 activations,
//   * 3x3 stride-2 convolutions with the encoder's right/bottom zero pad,
//   * plain row-major GEMMs (attention scores Q K^T and P V^T^T), expressed as
//     a 1x1 "convolution" over a [1, 1, M, K] activation.
// GEMM view: M = output pixels, N = output channels, K = taps * Cin. No im2col
// buffer exists: for K block (tap, channel block) the producer warp issues one
// TMA load of the shifted NHWC halo box (zero fill outside the image supplies
// the padding) and one TMA load of the matching weight tile. tcgen05.mma
// accumulates 128 x BLOCK_N fp32 tiles in TMEM (double buffered so the
// epilogue of one tile overlaps the MMAs of the next); four epilogue warps read
// TMEM, add bias / residual / per-row scale and store bf16 or fp32.
//
// Warp roles (192 threads, one persistent CTA per SM):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  epilogue, TMEM lane quadrant = warp % 4
//
// Reference counterpart: the convolution of BandedConv2d::forward_checked
// (src/native/conv.rs:54-112) with its bias add (:116-145) and the residual
// add of Resnet::forward_checked (src/native/vae_encoder.rs:150), and the
// score / value matmuls of attend (src/native/attention.rs:23).
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "conv_epilogue.cuh"
#include "conv_tc.h"

#include <cstdio>
#include <mutex>

namespace osor {

__device__ int g_device_status = 0;

namespace {

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kABytes = kBlockM * kBlockK * 2;

struct TcParams {
  int num_m_tiles, num_n_tiles;
  int k_blocks, c_blocks;  // k_blocks = taps * c_blocks
  int ksize, stride, pad;
  int tiles_x, tiles_y;    // output tile grid per image
  int tile_w, tile_h;      // output pixels per tile along W / H (tile_w*tile_h = 128)
  int n_out;               // valid output columns (N)
  const float* bias;       // [N] or nullptr
  const void* residual;    // 16-bit [M, ld_res] or nullptr
  long long ld_res;
  void* out;               // [M, ld_out]
  long long ld_out;
  const float* row_scale;  // [M] or nullptr
  int out_f32;
  // GroupNorm partial statistics of the (rounded) output, written when the
  // kernel is instantiated with CPG > 0: gn_part[m_tile][group] = (mean, M2)
  // over the tile's 128 pixels x CPG channels of that group.
  float* gn_part;
  int gn_groups;  // groups per pixel row (Cout / CPG)
  // Thin-output mode (BLOCK_N 16): n_valid NCHW f32 planes of out_hw pixels.
  int n_valid;
  long long out_hw;
  // Fused nearest-2x upsample (phases == 4): the tile grid runs over the
  // low_h x low_w input, each tile is computed for the four output phases
  // with weight rows [phase * cout_total, ...), and results land on the
  // 2*low_h x 2*low_w output. phases == 1: plain convolution.
  int phases;
  int low_h, low_w;
  int cout_total;  // weight rows per phase (0 when phases == 1)
  // 16-bit outputs leave through TMA stores of 32 consecutive tile pixels,
  // except for an upsampled output with low_w % 32 != 0 (direct stores).
  int direct_store;
  // Two-pass row softmax (ConvTcArgs::softmax_*).
  float* softmax_stats;
  int softmax_stats_ld;
  const float* softmax_max;
};

template <int BLOCK_N>
struct TcConfig {
  static constexpr int kBBytes = BLOCK_N * kBlockK * 2;
  static constexpr int kStages = BLOCK_N == 256 ? 4 : (BLOCK_N == 128 ? 6 : 8);
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BLOCK_N;
  // Epilogue warps: four (one per TMEM lane quadrant) for the thin output;
  // otherwise sixteen, four per quadrant, each owning BLOCK_N / 128
  // 32-column chunks.
  static constexpr int kEpiWarps = BLOCK_N == 16 ? 4 : 16;
  static constexpr int kChunksPerWarp = BLOCK_N == 16 ? 1 : BLOCK_N / 128;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  // GroupNorm tile statistics, one half per accumulator: [quad][group][mean, M2].
  static constexpr int kStatBytes = 2 * 4 * 64 * 2 * 4;
  // Output staging for the TMA stores: 1 KB per epilogue warp (32 pixels x
  // 32 bytes: 16 channels of a 16-bit output or 8 of an f32 one).
  static constexpr int kOutStageBytes = BLOCK_N == 16 ? 0 : kEpiWarps * 1024;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ +
                                    kStatBytes + kOutStageBytes;
};

// The four epilogue warps of one column slot (one per TMEM lane quadrant)
// synchronise on named barrier 2 + slot, 128 threads; id 0 is __syncthreads.
__device__ __forceinline__ void slot_sync(int bar) {
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
}
// AND of `ok` over the slot's four warps, so that they take the same branch.
__device__ __forceinline__ bool slot_all(int bar, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %2, 0;\n\t"
      "bar.red.and.pred q, %1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(bar), "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

template <int BLOCK_N, int D, int CPG>
__global__ void __launch_bounds__(TcConfig<BLOCK_N>::kThreads, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_out, const TcParams p) {
  using Cfg = TcConfig<BLOCK_N>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* stat_smem = reinterpret_cast<float*>(smem + S * Cfg::kStageBytes + 256);
  uint8_t* out_stage = smem + S * Cfg::kStageBytes + 256 + Cfg::kStatBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Cfg::kEpiWarps);  // lane 0 of every epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // Tile order: m_tile (outer), upsample phase, n_tile (inner), so CTAs that
  // run together share input rows in L2.
  const int tiles_per_m = p.phases * p.num_n_tiles;
  const int num_tiles = p.num_m_tiles * tiles_per_m;
  const int tiles_per_image = p.tiles_x * p.tiles_y;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_tile = tile / tiles_per_m;
        const int mrem = tile - m_tile * tiles_per_m;
        const int ph = mrem / p.num_n_tiles;
        const int n_tile = mrem - ph * p.num_n_tiles;
        const int img = m_tile / tiles_per_image;
        const int rem = m_tile - img * tiles_per_image;
        const int ty = rem / p.tiles_x;
        const int tx = rem - ty * p.tiles_x;
        // Upsample phase (a, b) = (ph >> 1, ph & 1): a 2x2 conv on the
        // low-res input starting one row / column up-left for a / b = 0.
        const int pad_y = p.phases == 4 ? 1 - (ph >> 1) : p.pad;
        const int pad_x = p.phases == 4 ? 1 - (ph & 1) : p.pad;
        const int ox = tx * p.tile_w * p.stride - pad_x;
        const int oy = ty * p.tile_h * p.stride - pad_y;
        const int b_row = ph * p.cout_total + n_tile * BLOCK_N;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          const int tap = kb / p.c_blocks;
          const int cb = kb - tap * p.c_blocks;
          const int ky = tap / p.ksize;
          const int kx = tap - ky * p.ksize;
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_4d(smem_a + stage * kABytes, &tmap_a, &full[stage], cb * kBlockK, ox + kx,
                      oy + ky, img);
          tma_load_2d(smem_b + stage * Cfg::kBBytes, &tmap_b, &full[stage], kb * kBlockK, b_row);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let every armed load land before the CTA leaves.
        for (int s = 0; s < S; ++s) {
          int st = stage - 1 - s;
          uint32_t ph = phase;
          if (st < 0) {
            st += S;
            ph ^= 1;
          }
          const uint32_t addr = smem_u32(&full[st]);
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(addr, ph) && global_timer_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_f32acc(kBlockM, BLOCK_N, Elem<D>::kUmmaFormat);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BLOCK_N;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * kABytes);
          const uint32_t b_addr = smem_u32(smem_b + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {
            umma_bf16(d_tmem, sw128_kmajor_desc(a_addr + k * 32),
                      sw128_kmajor_desc(b_addr + k * 32), idesc, (kb | k) != 0);
          }
          issued = true;
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok && issued) {
        // Drain outstanding MMAs before TMEM is released.
        umma_commit(drain);
        const uint32_t addr = smem_u32(drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(addr, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;           // TMEM lanes quad*32 .. quad*32+31
    const int slot = (warp - 2) >> 2;    // column slot (0 for the thin output)
    const int sbar = 2 + slot;
    const int row = quad * 32 + lane;
    constexpr int CPW = Cfg::kChunksPerWarp;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_tile = tile / tiles_per_m;
      const int mrem = tile - m_tile * tiles_per_m;
      const int ph = mrem / p.num_n_tiles;
      const int n_tile = mrem - ph * p.num_n_tiles;
      const long long m = (long long)m_tile * kBlockM + row;
      // Output row of pixel m: itself, or for an upsample phase (a, b) the
      // high-res pixel (img, 2i + a, 2j + b) of low-res pixel (img, i, j).
      long long orow = m;
      // GroupNorm partial slot: tiles of one image stay contiguous (phase-major
      // within the image for the upsampled output).
      int stat_slot = m_tile;
      int up_j = 0, up_row = 0;  // upsample: first low-res column of this warp's pixels, image row
      if (p.phases == 4) {
        const long long low_hw = (long long)p.low_h * p.low_w;
        const long long img = m / low_hw;
        const long long rem = m - img * low_hw;
        const long long i = rem / p.low_w, j = rem - (rem / p.low_w) * p.low_w;
        orow = (img * 2 * p.low_h + 2 * i + (ph >> 1)) * (2LL * p.low_w) + 2 * j + (ph & 1);
        const int mt_img = m_tile / tiles_per_image;
        stat_slot = (mt_img * 4 + ph) * tiles_per_image + (m_tile - mt_img * tiles_per_image);
        // The warp's 32 pixels are consecutive columns of one low-res row.
        const long long m_first = m - lane;
        const long long rem0 = m_first - img * low_hw;
        up_j = (int)(rem0 % p.low_w);
        up_row = (int)(img * p.low_h + rem0 / p.low_w);
      }
      // The residual does not depend on the accumulator: start its loads
      // before waiting for the MMAs.
      uint4 res[CPW][4];
      if (BLOCK_N != 16 && p.residual) {
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const uint4* r4 = reinterpret_cast<const uint4*>(
              static_cast<const uint16_t*>(p.residual) + orow * p.ld_res + n_tile * BLOCK_N +
              (slot * CPW + c) * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) res[c][j] = __ldg(r4 + j);
        }
      }
      // The slot's four warps leave together: the statistics below use a
      // named barrier that all of them must reach.
      if (!slot_all(sbar, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const float scale = p.row_scale ? __ldg(p.row_scale + m) : 1.0f;
      if constexpr (BLOCK_N == 16) {
        // Thin output (Cout <= 16, weights zero-padded to 16 rows): the first
        // n_valid channels as NCHW f32 planes; a warp writes 32 consecutive
        // pixels of each plane.
        uint32_t r[16];
        tmem_load_32x32b_x16(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * 16, r);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        const long long img = m / p.out_hw;
        const long long pix = m - img * p.out_hw;
        float* o = static_cast<float*>(p.out) + img * p.n_valid * p.out_hw + pix;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < p.n_valid)
            o[(long long)j * p.out_hw] =
                __uint_as_float(r[j]) * scale + (p.bias ? __ldg(p.bias + j) : 0.0f);
      } else {
        float* st = stat_smem + acc * (4 * 64 * 2);
        float sm_max = 0.0f, sm_sum = 0.0f;  // softmax statistics pass
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const int chunk = slot * CPW + c;
          uint32_t r[32];
          tmem_load_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BLOCK_N +
                                   chunk * 32,
                               r);
          tmem_wait_ld();
          if (c == CPW - 1) {
            // This warp's columns are all in registers: release the
            // accumulator so the next tile's MMAs can start.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
          const int n0 = n_tile * BLOCK_N + chunk * 32;
          float v[32];
          if (p.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 b = __ldg(b4 + j);
              v[4 * j + 0] = fmaf(__uint_as_float(r[4 * j + 0]), scale, b.x);
              v[4 * j + 1] = fmaf(__uint_as_float(r[4 * j + 1]), scale, b.y);
              v[4 * j + 2] = fmaf(__uint_as_float(r[4 * j + 2]), scale, b.z);
              v[4 * j + 3] = fmaf(__uint_as_float(r[4 * j + 3]), scale, b.w);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * scale;
          }
          if (p.residual) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float f[8];
              unpack8<D>(res[c][j], f);
#pragma unroll
              for (int t = 0; t < 8; ++t) v[8 * j + t] += f[t];
            }
          }
          if (p.softmax_stats) {
            // Row softmax statistics of this warp's CPW x 32 columns, merged
            // across its chunks online; nothing is stored.
            constexpr float kLog2e = 1.4426950408889634f;
            float mx = v[0];
#pragma unroll
            for (int j = 1; j < 32; ++j) mx = fmaxf(mx, v[j]);
            if (c > 0) mx = fmaxf(mx, sm_max);
            float sum = c > 0 ? sm_sum * ex2_approx((sm_max - mx) * kLog2e) : 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) sum += ex2_approx((v[j] - mx) * kLog2e);
            sm_max = mx;
            sm_sum = sum;
            if (c == CPW - 1) {
              const int block = (n_tile * BLOCK_N + slot * CPW * 32) / (CPW * 32);
              reinterpret_cast<float2*>(p.softmax_stats)[m * p.softmax_stats_ld + block] =
                  make_float2(sm_max, sm_sum);
            }
            continue;
          }
          if (p.softmax_max) {
            constexpr float kLog2e = 1.4426950408889634f;
            const float mrow = __ldg(p.softmax_max + m) * kLog2e;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = ex2_approx(fmaf(v[j], kLog2e, -mrow));
          }
          // Stores leave through TMA from a 1 KB staging tile per warp
          // (pixel row = lane, 32 bytes each): one lane per pixel would make
          // every store instruction touch 32 cache lines.
          uint8_t* sb = out_stage + (warp - 2) * 1024;
          uint4* sdst = reinterpret_cast<uint4*>(sb + lane * 32);
          if (p.out_f32) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              if (lane == 0) bulk_wait_group_read<0>();
              __syncwarp();
              sdst[0] = make_uint4(__float_as_uint(v[8 * q4]), __float_as_uint(v[8 * q4 + 1]),
                                   __float_as_uint(v[8 * q4 + 2]), __float_as_uint(v[8 * q4 + 3]));
              sdst[1] = make_uint4(__float_as_uint(v[8 * q4 + 4]), __float_as_uint(v[8 * q4 + 5]),
                                   __float_as_uint(v[8 * q4 + 6]), __float_as_uint(v[8 * q4 + 7]));
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmap_out, sb, n0 + 8 * q4, (int)(m - lane));
                bulk_commit_group();
              }
            }
          } else {
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] = Elem<D>::pack(v[2 * j], v[2 * j + 1]);
            if (p.direct_store) {
              // Upsampled output narrower than 32 low-res columns: a warp's
              // pixels span several output rows, store them lane by lane.
              uint4* o4 =
                  reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + orow * p.ld_out + n0);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                o4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (lane == 0) bulk_wait_group_read<0>();
              __syncwarp();
              sdst[0] = make_uint4(pk[8 * h], pk[8 * h + 1], pk[8 * h + 2], pk[8 * h + 3]);
              sdst[1] = make_uint4(pk[8 * h + 4], pk[8 * h + 5], pk[8 * h + 6], pk[8 * h + 7]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                if (p.phases == 4)
                  tma_store_5d(&tmap_out, sb, n0 + 16 * h, ph & 1, up_j, ph >> 1, up_row);
                else
                  tma_store_2d(&tmap_out, sb, n0 + 16 * h, (int)(m - lane));
                bulk_commit_group();
              }
            }
            }
            if constexpr (CPG > 0) {
              // Statistics of the stored (rounded) values, per quadrant into
              // this accumulator's half of stat_smem.
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float2 f = Elem<D>::unpack(pk[j]);
                v[2 * j] = f.x;
                v[2 * j + 1] = f.y;
              }
              gn_chunk_stats<CPG>(v, lane, st + (quad * 64 + chunk * (32 / CPG)) * 2);
            }
          }
        }
        if constexpr (CPG > 0) {
          if (!p.out_f32) {
            // The slot's first warp merges the four quadrants of the slot's
            // groups and publishes one (mean, M2) per group of this tile. The
            // stat_smem halves alternate with the accumulators; a warp reaches
            // tile i + 2's writes only after the merging warp has passed tile
            // i + 1's barrier, i.e. finished reading tile i's half.
            slot_sync(sbar);
            constexpr int G = 32 / CPG;
            constexpr int kG = BLOCK_N / CPG;
            if (((warp - 2) & 3) == 0 && lane < CPW * G) {
              const int g = slot * CPW * G + lane;
              const float n = 32.0f * CPG;
              float ma = st[(0 * 64 + g) * 2], qa = st[(0 * 64 + g) * 2 + 1];
              float mb = st[(2 * 64 + g) * 2], qb = st[(2 * 64 + g) * 2 + 1];
              merge_equal_counts(ma, qa, st[(1 * 64 + g) * 2], st[(1 * 64 + g) * 2 + 1], n);
              merge_equal_counts(mb, qb, st[(3 * 64 + g) * 2], st[(3 * 64 + g) * 2 + 1], n);
              merge_equal_counts(ma, qa, mb, qb, 2.0f * n);
              float* dst = p.gn_part + ((long long)stat_slot * p.gn_groups + n_tile * kG + g) * 2;
              dst[0] = ma;
              dst[1] = qa;
            }
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (BLOCK_N != 16 && lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int sm_count(int device) {
  static std::atomic<int> counts[64];  // zero-initialized; atomic for concurrent callers
  if (device < 0 || device >= 64) return 148;
  if (counts[device] == 0) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, device);
    counts[device] = c > 0 ? c : 148;
  }
  return counts[device];
}

template <int BLOCK_N, int D, int CPG>
cudaError_t launch_typed(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                         const TcParams& p,
                         cudaStream_t stream) {
  using Cfg = TcConfig<BLOCK_N>;
  static std::atomic<bool> configured[64];  // zero-initialized; atomic for concurrent callers
  int device = 0;
  cudaGetDevice(&device);
  if (device >= 0 && device < 64 && !configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel<BLOCK_N, D, CPG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  const int tiles = p.num_m_tiles * p.phases * p.num_n_tiles;
  const int grid = tiles < sm_count(device) ? tiles : sm_count(device);
  conv_tc_kernel<BLOCK_N, D, CPG><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, to, p);
  return cudaGetLastError();
}

template <int BLOCK_N, int D>
cudaError_t launch_cpg(int cpg, const CUtensorMap& ta, const CUtensorMap& tb,
                       const CUtensorMap& to, const TcParams& p, cudaStream_t stream) {
  switch (cpg) {
    case 4: return launch_typed<BLOCK_N, D, 4>(ta, tb, to, p, stream);
    case 8: return launch_typed<BLOCK_N, D, 8>(ta, tb, to, p, stream);
    case 16: return launch_typed<BLOCK_N, D, 16>(ta, tb, to, p, stream);
    default: return launch_typed<BLOCK_N, D, 0>(ta, tb, to, p, stream);
  }
}

}  // namespace

namespace {
// OSOR_PIXEL_N_CONV=0 / OSOR_PAIR_CONV=0 in the environment keep layers off
// the pixel-N and CTA-pair kernels, for comparing against this one.
bool env_enabled(const char* name) {
  const char* v = getenv(name);
  return !(v && v[0] == '0');
}
bool tcn_enabled() {
  static const bool on = env_enabled("OSOR_PIXEL_N_CONV");
  return on;
}
bool pair_enabled() {
  static const bool on = env_enabled("OSOR_PAIR_CONV");
  return on;
}
}  // namespace

const char* conv_tc_check(const ConvTcArgs& a) {
  if (a.geglu) return pair_enabled() ? conv_tc2_check(a) : "GEGLU products run on CTA pairs";
  if (tcn_enabled() && conv_tcn_check(a) == nullptr) return nullptr;
  if (a.in_coef) {
    // The normalising transform lives in the row-shift kernels.
    if (pair_enabled() && conv_tc2_check(a) == nullptr) return nullptr;
    return "fused input GroupNorm needs a 3x3 stride-1 layer on the pixel-N or CTA-pair kernel";
  }
  if (a.upsample) {
    if (a.ksize != 2 || a.stride != 1 || a.out_nchw || a.out_f32)
      return "the fused upsample convolution takes 2x2 phase weights and a 16-bit output";
    if (a.out_h != a.in_h || a.out_w != a.in_w) return "upsample tile grid must be the input grid";
  } else if (a.ksize != 1 && a.ksize != 3) {
    return "tensor-core convolution supports 1x1 and 3x3 kernels";
  }
  if (a.stride != 1 && a.stride != 2) return "tensor-core convolution supports stride 1 and 2";
  if (a.cin <= 0 || a.cin % kBlockK != 0) return "input channels must be a multiple of 64";
  if (a.out_nchw) {
    if (a.cout <= 0 || a.cout > 16 || !a.out_f32 || a.residual || a.gn_part || a.row_scale)
      return "thin NCHW output needs 1..16 f32 channels without residual or statistics";
  } else if (a.cout <= 0 || a.cout % 128 != 0) {
    return "output channels must be a multiple of 128";
  }
  if (a.out_w <= 0 || a.out_h <= 0 || a.batch <= 0) return "empty convolution";
  const int tile_w = a.out_w >= kBlockM ? kBlockM : a.out_w;
  if (a.out_w % tile_w != 0 || kBlockM % tile_w != 0) return "output width must divide or be a multiple of 128";
  const int tile_h = kBlockM / tile_w;
  if (a.out_h % tile_h != 0) return "output rows do not fill whole 128-pixel tiles";
  if (a.pixel_stride % 8 != 0 || a.ldw % 8 != 0) return "row strides must be 16-byte multiples";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w)) & 15)
    return "operands must be 16-byte aligned";
  if (a.residual && (a.ld_res % 8 != 0 || (reinterpret_cast<uintptr_t>(a.residual) & 15)))
    return "residual must be 16-byte aligned";
  if (!a.out_nchw && !a.softmax_stats &&
      (a.ld_out % (a.out_f32 ? 4 : 8) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15)))
    return "output must be 16-byte aligned";
  if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15)) return "bias must be 16-byte aligned";
  if ((long long)a.batch * a.out_h * a.out_w > 0x7fffffffLL) return "problem too large";
  if (a.stride == 2 && 2 * tile_w > 256) return "stride-2 tile too wide";
  if (a.dtype != kBf16 && a.dtype != kF16) return "unknown 16-bit type";
  if (a.gn_part && (a.out_f32 || (a.gn_cpg != 4 && a.gn_cpg != 8 && a.gn_cpg != 16)))
    return "fused group-norm statistics need a 16-bit output and 4, 8 or 16 channels per group";
  if (a.softmax_stats || a.softmax_max) {
    if (a.softmax_stats && a.softmax_max) return "one softmax pass at a time";
    if (a.ksize != 1 || a.out_nchw || a.upsample || a.bias || a.residual || a.gn_part ||
        a.row_scale || a.out_f32)
      return "the softmax passes take a plain 1x1 product with a 16-bit output";
    if (a.softmax_stats &&
        (a.softmax_stats_ld < a.cout / conv_tc_softmax_block(a.cout) ||
         (reinterpret_cast<uintptr_t>(a.softmax_stats) & 7)))
      return "softmax statistics buffer is too small or misaligned";
  }
  return nullptr;
}

int conv_tc_softmax_block(int cout) {
  // Each epilogue warp covers BLOCK_N / 4 columns of a tile (two or one
  // 32-column chunks).
  return (cout % 256 == 0 ? 256 : 128) / 4;
}

cudaError_t conv_tc_launch(const ConvTcArgs& a, cudaStream_t stream) {
  // 3x3 layers with Cout <= 128 on rows of 256 pixels run with the pixels on
  // the MMA's N side (conv_tcn.cu); other layers with Cout 128 or a multiple
  // of 256 on CTA pairs (conv_tc2.cu); the rest (upsample phases, softmax
  // passes, odd tile counts) here.
  if (a.geglu) return conv_tc_check(a) == nullptr ? conv_tc2_launch(a, stream) : cudaErrorInvalidValue;
  if (tcn_enabled() && conv_tcn_check(a) == nullptr) return conv_tcn_launch(a, stream);
  if (pair_enabled() && conv_tc2_check(a) == nullptr) return conv_tc2_launch(a, stream);
  if (a.in_coef) return cudaErrorInvalidValue;
  EncodeTiledFn encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  const int tile_w = a.out_w >= kBlockM ? kBlockM : a.out_w;
  const int tile_h = kBlockM / tile_w;
  const int block_n = a.out_nchw ? 16 : ((a.cout % 256 == 0) ? 256 : 128);
  const CUtensorMapDataType tdt =
      a.dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;

  CUtensorMap ta, tb;
  {
    const cuuint64_t ps = (cuuint64_t)a.pixel_stride * 2;
    cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in_w, (cuuint64_t)a.in_h,
                          (cuuint64_t)a.batch};
    cuuint64_t strides[3] = {ps, ps * a.in_w, ps * a.in_w * a.in_h};
    cuuint32_t box[4] = {(cuuint32_t)kBlockK, (cuuint32_t)(tile_w * a.stride),
                         (cuuint32_t)(tile_h * a.stride), 1};
    cuuint32_t estr[4] = {1, (cuuint32_t)a.stride, (cuuint32_t)a.stride, 1};
    CUresult r = encode(&ta, tdt, 4, const_cast<void*>(static_cast<const void*>(a.x)), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  {
    const int k_total = a.ksize * a.ksize * a.cin;
    // Weight rows: for a thin output the 16 rows of its tile, zero-padded by
    // the caller when it allocated 16, else cout (the box reads the rows past
    // the tensor as zeros); four phase blocks of cout for the fused upsample;
    // else cout.
    const int rows = a.out_nchw ? (a.w_rows >= 16 ? 16 : a.cout)
                                : (a.upsample ? 4 * a.cout : a.cout);
    cuuint64_t dims[2] = {(cuuint64_t)k_total, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldw * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBlockK, (cuuint32_t)block_n};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tb, tdt, 2, const_cast<void*>(static_cast<const void*>(a.w)), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  TcParams p;
  p.tile_w = tile_w;
  p.tile_h = tile_h;
  p.tiles_x = a.out_w / tile_w;
  p.tiles_y = a.out_h / tile_h;
  p.num_m_tiles = a.batch * p.tiles_x * p.tiles_y;
  p.num_n_tiles = a.out_nchw ? 1 : a.cout / block_n;
  p.c_blocks = a.cin / kBlockK;
  p.k_blocks = a.ksize * a.ksize * p.c_blocks;
  p.ksize = a.ksize;
  p.stride = a.stride;
  p.pad = a.pad;
  p.n_out = a.cout;
  p.bias = a.bias;
  p.residual = a.residual;
  p.ld_res = a.ld_res;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.row_scale = a.row_scale;
  p.out_f32 = a.out_f32;
  const int cpg = a.gn_part ? a.gn_cpg : 0;
  p.gn_part = a.gn_part;
  p.gn_groups = cpg ? a.cout / cpg : 0;
  p.n_valid = a.cout;
  p.out_hw = (long long)a.out_h * a.out_w;
  p.phases = a.upsample ? 4 : 1;
  p.low_h = a.in_h;
  p.low_w = a.in_w;
  p.cout_total = a.upsample ? a.cout : 0;
  p.direct_store = a.upsample && a.in_w % 32 != 0;
  p.softmax_stats = a.softmax_stats;
  p.softmax_stats_ld = a.softmax_stats_ld;
  p.softmax_max = a.softmax_max;
  // Output tensor map for the epilogue's TMA stores (unused by the thin
  // NCHW output, which stores directly).
  CUtensorMap to = tb;
  if (!a.out_nchw && !a.softmax_stats) {
    CUresult r;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    if (a.upsample) {
      // Output pixel (img, 2i + a, 2j + b) of phase (a, b) and low-res pixel
      // (img, i, j) as dims (channel, b, j, a, img * low_h + i).
      const cuuint64_t row = (cuuint64_t)a.ld_out * 2;
      cuuint64_t dims[5] = {(cuuint64_t)a.cout, 2, (cuuint64_t)a.in_w, 2,
                            (cuuint64_t)a.batch * a.in_h};
      cuuint64_t strides[4] = {row, 2 * row, 2 * (cuuint64_t)a.in_w * row,
                               4 * (cuuint64_t)a.in_w * row};
      cuuint32_t box[5] = {16, 1, 32, 1, 1};
      r = encode(&to, tdt, 5, a.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const int esize = a.out_f32 ? 4 : 2;
      cuuint64_t dims[2] = {(cuuint64_t)a.cout, (cuuint64_t)p.num_m_tiles * kBlockM};
      cuuint64_t strides[1] = {(cuuint64_t)a.ld_out * esize};
      cuuint32_t box[2] = {(cuuint32_t)(32 / esize), 32};
      r = encode(&to, a.out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : tdt, 2, a.out, dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  if (a.out_nchw)
    return a.dtype == kF16 ? launch_typed<16, kF16, 0>(ta, tb, to, p, stream)
                           : launch_typed<16, kBf16, 0>(ta, tb, to, p, stream);
  if (a.dtype == kF16)
    return block_n == 256 ? launch_cpg<256, kF16>(cpg, ta, tb, to, p, stream)
                          : launch_cpg<128, kF16>(cpg, ta, tb, to, p, stream);
  return block_n == 256 ? launch_cpg<256, kBf16>(cpg, ta, tb, to, p, stream)
                        : launch_cpg<128, kBf16>(cpg, ta, tb, to, p, stream);
}

}  // namespace osor
