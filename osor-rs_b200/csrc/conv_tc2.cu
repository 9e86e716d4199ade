// Implicit-GEMM convolution on CTA pairs (2-SM tcgen05 MMA), N = BN output
// channels per pair tile: BN = 128 for Cout = 128, BN = 256 for Cout a
// multiple of 256 (Cout / 256 channel tiles).
//
// The one-CTA kernel (conv_tc.cu) re-fetches the whole weight matrix for
// every 128-pixel tile and reads both MMA operands from one SM's shared
// memory: per 128 x 256 x 16 instruction that is 12 KB of operand reads plus
// the stage's TMA writes, more than shared memory delivers at the tensor
// core's rate. Here two CTAs of a cluster cooperate on 256 pixels:
// `tcgen05.mma.cta_group::2` with M = 256, N = BN takes A rows 0..127 from
// the even CTA and 128..255 from the odd one, and B rows (output channels)
// 0..BN/2-1 / BN/2..BN-1 likewise, so each SM reads and stores only half of
// the weights. When that half fits (K <= 1152) it is loaded once per CTA and
// stays resident in shared memory for every tile the pair computes, and the
// pipeline stages carry only the A (input) tiles; otherwise each stage also
// carries the weight slices it needs.
//
// Row-shift mode (3x3, or the 2x2 upsample phases, stride 1, tiles of one
// 128-pixel output row): a stage holds 130 consecutive input pixels of one
// input row and channel block, and the ksize horizontal taps read it as views
// starting one pixel (one 128-byte swizzle row) apart, so a tile loads
// ksize * Cin / 64 stages instead of ksize^2 * Cin / 64.
//
// Fused nearest-2x upsample + 3x3 conv: as in conv_tc.cu, four 2x2 phase
// convolutions of the low-res input (4/9 of the FLOPs); each pair tile is one
// (m pair, phase, channel tile), and the epilogue stores low-res pixel
// (i, j)'s result at high-res pixel (2i + a, 2j + b) of phase (a, b).
//
// Roles per CTA (576 threads): warp 0 TMA producer, warp 1 TMEM allocator
// (both CTAs) and MMA issuer (even CTA only), warps 2..17 epilogue (four per
// TMEM lane quadrant, BN / 4 columns each, in 32-column chunks). The even CTA's barriers gate the
// MMAs: both CTAs' TMA loads complete on them, the MMA commits arrive on both
// CTAs' barriers (multicast commit), and both CTAs' epilogues release the
// accumulators on the even CTA's barrier. No TMA load uses cluster multicast.
//
// Fused input GroupNorm (FUSE = 1, row-shift 3x3 only): the input is the raw
// activation and per-channel GroupNorm coefficients come with it. Each CTA's
// loads complete on its own barrier, four transform warps normalise (+SiLU)
// the CTA's stage in place (gn_stage.cuh) and arrive on the even CTA's
// `ready` barrier, which gates the MMAs instead. 448 threads: warps 2..9
// epilogue (two per TMEM lane quadrant), warps 10..13 transform.
//
// GEGLU epilogue (GG = 1, its own instantiation: BN 256, no statistics or
// FUSE): the 1x1 product of a GEGLU input projection whose weight rows come
// as 128 value rows then their 128 gate rows per 256-row channel tile. An
// epilogue warp's two chunks of a tile are then a value chunk and its gate
// chunk; it stores value * gelu_erf(gate) at channel tile * 128 + chunk * 32
// of a cout / 2 wide output (FeedForward::forward, src/native/transformer.rs:
// 18-24).
//
// Reference counterpart: the same convolution as conv_tc.cu
// (BandedConv2d::forward_checked, src/native/conv.rs:54-145).
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "conv_epilogue.cuh"
#include "conv_tc.h"
#include "gn_stage.cuh"

namespace osor {
namespace {

constexpr int kM = 128;           // pixels per CTA
constexpr int kBK = 64;           // K block (one 128-byte swizzle row)
constexpr int kAB = kM * kBK * 2;            // A tile bytes (16 KB)
constexpr int kShiftRows = kM + 2;           // row-shift stage: 130 pixels
constexpr int kShiftAB = 17 * 1024;          // row-shift A bytes in a stage (>= 130 x 128 B)
constexpr int kMaxStages = 12;
constexpr int kMaxResidentKBlocks = 18;      // resident weights: K <= 1152
constexpr int kStat2 = 2 * 4 * 64 * 2 * 4;  // per accumulator: [quad][group](mean, M2)
constexpr int kSmem2 = 225 * 1024;

// Warp roles and shared-memory tail per variant: FUSE = 1 trades half of the
// epilogue warps for the four transform warps (the epilogue of a tile takes
// a small part of its MMA time) and a weight producer warp, and adds the
// `ready` and weight-ring barriers.
template <int FUSE>
struct Tc2Shape {
  static constexpr int kEpi = FUSE ? 8 : 16;  // epilogue warps, kEpi / 4 per lane quadrant
  static constexpr int kFirstXf = 2 + kEpi;   // first transform warp
  static constexpr int kBWarp = kFirstXf + kXfThreads / 32;  // FUSE: weight producer
  static constexpr int kThreads = 64 + 32 * kEpi + (FUSE ? kXfThreads + 32 : 0);
  static constexpr int kTail = FUSE ? 1024 : 256;  // barriers, TMEM address, abort flag
  static constexpr int kBudget = kSmem2 - 1024 - kTail - kStat2;  // stages + resident weights
};

// OSOR_ROW_SHIFT=0 in the environment keeps 3x3 / phase layers on one
// stage per tap (for comparison).
bool row_shift_enabled() {
  static const bool on = [] {
    const char* v = getenv("OSOR_ROW_SHIFT");
    return !(v && v[0] == '0');
  }();
  return on;
}

// B bytes per K block per CTA: BN / 2 weight rows of 64 channels.
template <int BN>
__host__ __device__ constexpr int b_block_bytes() {
  return (BN / 2) * kBK * 2;
}

struct Tc2Params {
  int num_m_tiles;         // even
  int n_tiles;             // Cout / BN
  int k_blocks, c_blocks;
  int ksize, stride, pad;
  int tiles_x, tiles_y, tile_w, tile_h;
  int row_shift;           // 1: row-shift stages (see above)
  // Fused nearest-2x upsample (phases == 4, ksize 2): the tile grid runs over
  // the low_h x low_w input and every tile is computed for the four output
  // phases (a, b) with weight rows [phase * cout_total, ...): pair tiles are
  // (m pair, phase, channel tile), and each low-res pixel's result lands on
  // high-res pixel (2i + a, 2j + b). phases == 1: plain convolution.
  int phases;
  int low_h, low_w;
  int cout_total;
  int units;               // stages per tile: k_blocks, or 3 * c_blocks in row-shift mode
  int b_resident;          // 1: weight half loaded once; 0: streamed with each stage
  int stages;              // pipeline depth (<= kMaxStages)
  int w_stages;            // FUSE with streamed weights: depth of the separate weight ring
  int stage_bytes;         // A bytes + streamed B bytes, 1 KB multiple
  int a_bytes;             // A bytes reserved at the start of a stage
  uint32_t a_tx;           // A bytes one CTA's load writes
  uint32_t b_tx;           // streamed B bytes one CTA's loads write per stage
  const float* bias;
  const void* residual;
  long long ld_res;
  void* out;
  long long ld_out;
  const float* row_scale;
  float* gn_part;
  int gn_groups;
  // FUSE = 1: GroupNorm(+SiLU) of the input from coef[img][c][4]; input rows
  // outside [in_y0, in_y1) are zero padding; in_w = input width.
  const float* in_coef;
  int in_c, in_silu, in_y0, in_y1, in_w;
  int geglu;               // GEGLU epilogue (ConvTcArgs::geglu); BN 256 without FUSE
};

// The four epilogue warps of one 32-column chunk (one per TMEM lane quadrant)
// synchronise on named barrier 2 + chunk, 128 threads; warps of different
// chunks never wait for each other.
__device__ __forceinline__ void chunk_sync(int bar) {
  asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool chunk_all(int bar, bool ok) {
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

template <int BN, int D, int CPG, int FUSE, int GG = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Tc2Shape<FUSE>::kThreads, 1)
    conv_tc2_kernel(const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_b, const Tc2Params p) {
  using Sh = Tc2Shape<FUSE>;
  constexpr int kEpiWarps = Sh::kEpi;
  constexpr int kBB = b_block_bytes<BN>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  // Resident weight half, or (FUSE, streamed) the weight ring of one tap per stage.
  uint8_t* smem_b = smem + p.stages * p.stage_bytes;
  uint8_t* tail = smem_b + (p.b_resident ? p.k_blocks * kBB : (FUSE ? p.w_stages * kBB : 0));
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* bfull = tempty + 2;
  uint64_t* drain = bfull + 1;
  uint64_t* ready = drain + 1;  // FUSE: stage normalised in both CTAs (even CTA's count)
  uint64_t* wfull = ready + kMaxStages;  // FUSE: weight ring (both CTAs' bytes, even CTA's)
  uint64_t* wempty = wfull + kMaxStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ready + (FUSE ? 3 * kMaxStages : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* stat_smem = reinterpret_cast<float*>(tail + Sh::kTail);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if (FUSE) mbar_init(&ready[s], 2 * kXfThreads / 32);  // transform warps of both CTAs
    }
    if (FUSE)
      for (int s = 0; s < p.w_stages; ++s) {
        mbar_init(&wfull[s], 1);
        mbar_init(&wempty[s], 1);
      }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    mbar_init(bfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // Pair tiles: (256-pixel pair of m tiles, channel tile), channel tile inner
  // so that clusters running together share input rows in L2.
  const int pairs = p.num_m_tiles / 2 * p.phases * p.n_tiles;
  const int cluster_id = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;
  const int tiles_per_image = p.tiles_x * p.tiles_y;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      if (p.b_resident) {
        // Weight half: rows [rank * 64, rank * 64 + 64), all K blocks.
        if (leader) mbar_arrive_expect_tx(bfull, 2u * p.k_blocks * kBB);
        for (int kb = 0; kb < p.k_blocks; ++kb)
          tma_load_2d_pair(smem_b + kb * kBB, &tmap_b, map_to_rank(smem_u32(bfull), 0), kb * kBK,
                           (int)rank * (BN / 2));
      }
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int pt = cluster_id; pt < pairs && ok; pt += clusters) {
        const int n_tile = pt % p.n_tiles;
        const int rest = pt / p.n_tiles;
        const int ph = rest % p.phases;
        const int m_tile = 2 * (rest / p.phases) + (int)rank;
        const int b_row = ph * p.cout_total + n_tile * BN + (int)rank * (BN / 2);
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
        for (int u = 0; u < p.units; ++u) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          int ky, kx, cb;
          if (p.row_shift) {
            ky = u / p.c_blocks;
            cb = u - ky * p.c_blocks;
            kx = 0;
          } else {
            const int tap = u / p.c_blocks;
            cb = u - tap * p.c_blocks;
            ky = tap / p.ksize;
            kx = tap - ky * p.ksize;
          }
          uint8_t* st = stages + stage * p.stage_bytes;
          if (FUSE) {
            // This CTA's transform warps wait for its own stage; the weights
            // come through their own ring (warp kBWarp).
            mbar_arrive_expect_tx(&full[stage], p.a_tx);
            tma_load_4d(st, &tmap_a, &full[stage], cb * kBK, ox + kx, oy + ky, img);
            if (++stage == p.stages) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          const uint32_t bar = map_to_rank(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2u * (p.a_tx + p.b_tx));
          tma_load_4d_pair(st, &tmap_a, bar, cb * kBK, ox + kx, oy + ky, img);
          if (!p.b_resident) {
            // The weight slices of this stage's taps: one, or the ksize kx
            // taps of row ky in row-shift mode.
            const int taps = p.row_shift ? p.ksize : 1;
            for (int t = 0; t < taps; ++t) {
              const int kb = p.row_shift ? (ky * p.ksize + t) * p.c_blocks + cb : u;
              tma_load_2d_pair(st + p.a_bytes + t * kBB, &tmap_b, bar, kb * kBK, b_row);
            }
          }
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = umma_idesc_f32acc(2 * kM, BN, Elem<D>::kUmmaFormat);
      bool ok = !p.b_resident || mbar_wait(bfull, 0, abort_flag);
      bool issued = false;
      int stage = 0;
      uint32_t phase = 0;
      int ws = 0;  // FUSE: weight ring
      uint32_t wph = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int pt = cluster_id; pt < pairs && ok; pt += clusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int u = 0; u < p.units; ++u) {
          if (!(FUSE ? mbar_wait_cluster(&ready[stage], phase, abort_flag)
                     : mbar_wait(&full[stage], phase, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stages + stage * p.stage_bytes);
          if (p.row_shift) {
            // Unit (ky, cb); tap kx reads the stage from pixel row kx on (the
            // 128-byte swizzle follows the address bits, so a view may start
            // on any row of a swizzle atom).
            const int ky = u / p.c_blocks;
            const int cb = u - ky * p.c_blocks;
#pragma unroll 1
            for (int kx = 0; kx < p.ksize; ++kx) {
              uint32_t b_addr;
              if (p.b_resident) {
                b_addr = smem_u32(smem_b + ((ky * p.ksize + kx) * p.c_blocks + cb) * kBB);
              } else if (FUSE) {
                if (!mbar_wait(&wfull[ws], wph, abort_flag)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                b_addr = smem_u32(smem_b + ws * kBB);
              } else {
                b_addr = a_addr + p.a_bytes + kx * kBB;
              }
#pragma unroll
              for (int k = 0; k < kBK / 16; ++k)
                umma_bf16_pair(d_tmem, sw128_kmajor_desc(a_addr + kx * 128 + k * 32),
                               sw128_kmajor_desc(b_addr + k * 32), idesc, (u | kx | k) != 0);
              issued = true;
              if (FUSE && !p.b_resident) {
                umma_commit_pair(&wempty[ws], 0x3);
                if (++ws == p.w_stages) {
                  ws = 0;
                  wph ^= 1;
                }
              }
            }
            if (!ok) break;
          } else {
            const uint32_t b_addr =
                p.b_resident ? smem_u32(smem_b + u * kBB) : a_addr + p.a_bytes;
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              umma_bf16_pair(d_tmem, sw128_kmajor_desc(a_addr + k * 32),
                             sw128_kmajor_desc(b_addr + k * 32), idesc, (u | k) != 0);
          }
          issued = true;
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok && issued) {
        umma_commit_pair(drain, 0x1);
        const uint32_t addr = smem_u32(drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(addr, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp < Sh::kFirstXf) {
    // ------------------------------------------------------------ epilogue
    // Warp (quad, slot) owns 32-column chunks slot, slot + kSlots, ... of the
    // BN accumulator columns.
    constexpr int kSlots = kEpiWarps / 4;
    constexpr int kChunks = BN / 32 / kSlots;
    const int quad = warp & 3;           // TMEM lanes quad*32 .. quad*32+31
    const int slot = (warp - 2) >> 2;    // 0 .. kSlots - 1
    const int cbar = 2 + slot;
    const int row = quad * 32 + lane;
    const uint32_t tempty_leader[2] = {map_to_rank(smem_u32(&tempty[0]), 0),
                                       map_to_rank(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int pt = cluster_id; pt < pairs; pt += clusters) {
      const int n_tile = pt % p.n_tiles;
      const int rest = pt / p.n_tiles;
      const int ph = rest % p.phases;
      const int m_tile = 2 * (rest / p.phases) + (int)rank;
      const long long m = (long long)m_tile * kM + row;
      // Output row of pixel m: itself, or for an upsample phase (a, b) the
      // high-res pixel (img, 2i + a, 2j + b) of low-res pixel (img, i, j);
      // GroupNorm tile slot: the image's tiles stay contiguous, phase-major.
      long long orow = m;
      int stat_tile = m_tile;
      if (p.phases == 4) {
        const long long low_hw = (long long)p.low_h * p.low_w;
        const long long im = m / low_hw;
        const long long rem = m - im * low_hw;
        const long long i = rem / p.low_w, j = rem - (rem / p.low_w) * p.low_w;
        orow = (im * 2 * p.low_h + 2 * i + (ph >> 1)) * (2LL * p.low_w) + 2 * j + (ph & 1);
        const int mt_img = m_tile / tiles_per_image;
        stat_tile = (mt_img * 4 + ph) * tiles_per_image + (m_tile - mt_img * tiles_per_image);
      }
      // The residual does not depend on the accumulator: start the first
      // chunk's loads before waiting for the MMAs.
      uint4 res[4];
      if (p.residual) {
        const uint4* r4 = reinterpret_cast<const uint4*>(
            static_cast<const uint16_t*>(p.residual) + m * p.ld_res + n_tile * BN + slot * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) res[j] = __ldg(r4 + j);
      }
      if (!chunk_all(cbar, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const float scale = p.row_scale ? __ldg(p.row_scale + m) : 1.0f;
      // GEGLU (GG): with BN 256 and four slots this warp's chunks are `slot`
      // (values) and `slot + 4` (their gates); the values wait here, rounded
      // to the 16-bit type as a stored projection would be.
      static_assert(!GG || (BN == 256 && kChunks == 2 && CPG == 0 && FUSE == 0),
                    "GEGLU epilogue: BN 256, four slots, no statistics");
      uint32_t gv[GG ? 16 : 1];
#pragma unroll 1
      for (int ci = 0; ci < kChunks; ++ci) {
        const int chunk = slot + kSlots * ci;
        uint32_t r[32];
        tmem_load_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + chunk * 32,
                             r);
        tmem_wait_ld();
        if (ci == kChunks - 1) {
          // This warp's part of the accumulator is in registers: release it
          // on the even CTA so the next tile's MMAs can start.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
        }
        const int n0 = n_tile * BN + chunk * 32;
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
            unpack8<D>(res[j], f);
#pragma unroll
            for (int t = 0; t < 8; ++t) v[8 * j + t] += f[t];
          }
          if (ci + 1 < kChunks) {
            const uint4* r4 = reinterpret_cast<const uint4*>(
                static_cast<const uint16_t*>(p.residual) + m * p.ld_res + n0 + kSlots * 32);
#pragma unroll
            for (int j = 0; j < 4; ++j) res[j] = __ldg(r4 + j);
          }
        }
        long long oc = n0;
        if constexpr (GG != 0) {
          if (ci == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) gv[j] = Elem<D>::pack(v[2 * j], v[2 * j + 1]);
            continue;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 a = Elem<D>::unpack(gv[j]);
            const float g0 = v[2 * j], g1 = v[2 * j + 1];
            v[2 * j] = a.x * (0.5f * g0 * (1.0f + erff(g0 * 0.70710678118654752f)));
            v[2 * j + 1] = a.y * (0.5f * g1 * (1.0f + erff(g1 * 0.70710678118654752f)));
          }
          oc = (long long)n_tile * (BN / 2) + slot * 32;
        }
        uint4* o4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + orow * p.ld_out + oc);
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = Elem<D>::pack(v[2 * j], v[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        if constexpr (CPG > 0) {
          // Statistics of the stored (rounded) values.
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float2 f = Elem<D>::unpack(pk[j]);
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
          }
          // Per-quadrant statistics into this accumulator's half of
          // stat_smem; the slot's first warp merges the four quadrants. The
          // halves alternate with the accumulators, and a warp reaches tile
          // i + 2's writes only after the merging warp has passed tile i + 1's
          // barriers, i.e. finished reading tile i's half. Within a tile the
          // chunks of one slot use disjoint groups.
          constexpr int G = 32 / CPG;
          float* st = stat_smem + acc * (4 * 64 * 2);
          gn_chunk_stats<CPG>(v, lane, st + (quad * 64 + chunk * G) * 2);
          chunk_sync(cbar);
          if (quad == 0 && lane < G) {
            const int g = chunk * G + lane;
            const float n = 32.0f * CPG;
            float ma = st[(0 * 64 + g) * 2], qa = st[(0 * 64 + g) * 2 + 1];
            float mb = st[(2 * 64 + g) * 2], qb = st[(2 * 64 + g) * 2 + 1];
            merge_equal_counts(ma, qa, st[(1 * 64 + g) * 2], st[(1 * 64 + g) * 2 + 1], n);
            merge_equal_counts(mb, qb, st[(3 * 64 + g) * 2], st[(3 * 64 + g) * 2 + 1], n);
            merge_equal_counts(ma, qa, mb, qb, 2.0f * n);
            float* dst =
                p.gn_part + ((long long)stat_tile * p.gn_groups + n_tile * (BN / CPG) + g) * 2;
            dst[0] = ma;
            dst[1] = qa;
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  } else if (FUSE && warp < Sh::kBWarp) {
    // ------------------------------------------------------------ transform
    // Same tile / unit order as the producer (plain 3x3, stride 1, one
    // 128-pixel row per tile): wait for this CTA's stage, normalise it,
    // publish it to the even CTA's MMA issuer.
    const int tid = threadIdx.x - 32 * Sh::kFirstXf;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    // Image of pair tile pt in this CTA; coefficients fetched one unit ahead.
    auto tile_img = [&](int pt) { return (2 * (pt / p.n_tiles) + (int)rank) / tiles_per_image; };
    float4 raw[8];
    if (cluster_id < pairs) gn_stage_coef_fetch(p.in_coef, tile_img(cluster_id), p.in_c, 0, tid, raw);
    for (int pt = cluster_id; pt < pairs && ok; pt += clusters) {
      const int m_tile = 2 * (pt / p.n_tiles) + (int)rank;
      const int img = m_tile / tiles_per_image;
      const int rem = m_tile - img * tiles_per_image;
      const int ty = rem / p.tiles_x;
      const int tx = rem - ty * p.tiles_x;
      const int ox = tx * p.tile_w - p.pad;
      const int oy = ty - p.pad;
      for (int u = 0; u < p.units; ++u) {
        const int ky = u / p.c_blocks;
        const int cb = u - ky * p.c_blocks;
        const int y = oy + ky;
        StageCoef<D> k;
        gn_stage_coef_prepare<D>(raw, p.in_silu != 0, k);
        {
          const int npt = u + 1 < p.units ? pt : pt + clusters;
          gn_stage_coef_fetch(p.in_coef, npt < pairs ? tile_img(npt) : img, p.in_c,
                              u + 1 < p.units ? (cb + 1) % p.c_blocks : 0, tid, raw);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag))) {
          ok = false;
          break;
        }
        gn_stage_apply<D>(stages + stage * p.stage_bytes, kShiftRows, ox, p.in_w,
                          y >= p.in_y0 && y < p.in_y1, k, p.in_silu != 0, tid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_release(map_to_rank(smem_u32(&ready[stage]), 0));
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (FUSE && lane == 0 && !p.b_resident) {
    // ------------------------------------------------------------ weight producer
    // FUSE: one 64-channel slice of this CTA's weight half per tap, in the
    // MMA's (tile, unit, kx) order; both CTAs' loads complete on the even
    // CTA's barrier.
    int ws = 0;
    uint32_t wph = 0;
    bool ok = true;
    for (int pt = cluster_id; pt < pairs && ok; pt += clusters) {
      const int b_row = (pt % p.n_tiles) * BN + (int)rank * (BN / 2);
      for (int u = 0; u < p.units && ok; ++u) {
        const int ky = u / p.c_blocks;
        const int cb = u - ky * p.c_blocks;
        for (int kx = 0; kx < p.ksize; ++kx) {
          if (!mbar_wait(&wempty[ws], wph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&wfull[ws], 2u * kBB);
          tma_load_2d_pair(smem_b + ws * kBB, &tmap_b, map_to_rank(smem_u32(&wfull[ws]), 0),
                           ((ky * p.ksize + kx) * p.c_blocks + cb) * kBK, b_row);
          if (++ws == p.w_stages) {
            ws = 0;
            wph ^= 1;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or arrivals are pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn2 encode_fn2() {
  static EncodeTiledFn2 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn2>(ptr);
    return static_cast<EncodeTiledFn2>(nullptr);
  }();
  return fn;
}

template <int BN, int D, int CPG, int FUSE, int GG = 0>
cudaError_t launch2(const CUtensorMap& ta, const CUtensorMap& tb, const Tc2Params& p,
                    cudaStream_t stream) {
  constexpr int kThreads2 = Tc2Shape<FUSE>::kThreads;
  // Per device: the shared-memory opt-in and how many pairs fit on the GPU at
  // once (not every SM need have a partner in its cluster-capable group, so
  // this can be below SMs / 2). The persistent grid never exceeds it: a pair
  // that had to wait for another to finish would double the kernel's time.
  static std::atomic<int> resident_pairs[64];  // zero-initialized; atomic for concurrent callers
  int device = 0;
  cudaGetDevice(&device);
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (resident_pairs[device] == 0) {
    cudaError_t e = cudaFuncSetAttribute(conv_tc2_kernel<BN, D, CPG, FUSE, GG>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2);
    if (e != cudaSuccess) return e;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(kThreads2, 1, 1);
    cfg.dynamicSmemBytes = kSmem2;
    cfg.stream = stream;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, conv_tc2_kernel<BN, D, CPG, FUSE, GG>, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorNotSupported;
    resident_pairs[device] = n < sms / 2 ? n : sms / 2;
  }
  const int pairs = p.num_m_tiles / 2 * p.phases * p.n_tiles;
  int clusters = resident_pairs[device];
  if (clusters > pairs) clusters = pairs;
  conv_tc2_kernel<BN, D, CPG, FUSE, GG><<<2 * clusters, kThreads2, kSmem2, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

}  // namespace

const char* conv_tc2_check(const ConvTcArgs& a) {
  if (a.out_nchw || a.out_f32 || a.softmax_stats || a.softmax_max)
    return "pair kernel: plain 16-bit output only";
  if (a.upsample && (a.ksize != 2 || a.stride != 1 || a.pad != 0 || a.residual ||
                     a.out_h != a.in_h || a.out_w != a.in_w))
    return "pair kernel: upsample takes 2x2 phase weights on the low-res grid";
  if (!a.upsample && a.ksize == 2) return "pair kernel: 2x2 kernels only as upsample phases";
  if (a.cout != 128 && (a.cout <= 0 || a.cout % 256 != 0))
    return "pair kernel: Cout 128 or a multiple of 256";
  if (a.ksize != 1 && a.ksize != 2 && a.ksize != 3) return "pair kernel: 1x1, 2x2 or 3x3";
  if (a.stride != 1 && a.stride != 2) return "pair kernel: stride 1 or 2";
  if (a.cin <= 0 || a.cin % kBK != 0) return "pair kernel: Cin % 64";
  if (a.out_w <= 0 || a.out_h <= 0 || a.batch <= 0) return "empty convolution";
  const int tile_w = a.out_w >= kM ? kM : a.out_w;
  if (a.out_w % tile_w != 0 || kM % tile_w != 0) return "pair kernel: tile width";
  const int tile_h = kM / tile_w;
  if (a.out_h % tile_h != 0) return "pair kernel: tile rows";
  const long long m_tiles = (long long)a.batch * (a.out_w / tile_w) * (a.out_h / tile_h);
  if (m_tiles % 2 != 0) return "pair kernel: odd tile count";
  if (a.stride == 2 && 2 * tile_w > 256) return "pair kernel: stride-2 tile too wide";
  if (a.pixel_stride % 8 != 0 || a.ldw % 8 != 0 || a.ld_out % 8 != 0) return "strides";
  if ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.w) |
       reinterpret_cast<uintptr_t>(a.out)) & 15)
    return "alignment";
  if (a.residual && (a.ld_res % 8 != 0 || (reinterpret_cast<uintptr_t>(a.residual) & 15)))
    return "residual alignment";
  if (a.bias && (reinterpret_cast<uintptr_t>(a.bias) & 15)) return "bias alignment";
  if (a.gn_part && a.gn_cpg != 4 && a.gn_cpg != 8 && a.gn_cpg != 16) return "statistics";
  if (a.dtype != kBf16 && a.dtype != kF16) return "dtype";
  if (m_tiles * kM > 0x7fffffffLL) return "problem too large";
  if (a.geglu && (a.ksize != 1 || a.upsample || a.in_coef || a.residual || a.gn_part ||
                  a.row_scale || a.cout % 256 != 0))
    return "pair kernel: GEGLU products are plain 1x1 with Cout a multiple of 256";
  if (a.in_coef) {
    if (a.upsample || a.ksize != 3 || a.stride != 1 || a.pad != 1 || tile_h != 1 ||
        !row_shift_enabled())
      return "pair kernel: fused input GroupNorm on row-shift 3x3 stride-1 tiles only";
    if (reinterpret_cast<uintptr_t>(a.in_coef) & 15) return "pair kernel: coefficient alignment";
    if (a.in_y0 < 0 || (a.in_y1 >= 0 && (a.in_y1 < a.in_y0 || a.in_y1 > a.in_h)))
      return "pair kernel: input row range";
  }
  return nullptr;
}

namespace {

template <int BN, int FUSE>
cudaError_t launch_cpg(int dtype, int cpg, const CUtensorMap& ta, const CUtensorMap& tb,
                       const Tc2Params& p, cudaStream_t stream) {
  if (p.geglu) {
    // Its own instantiation, so the other epilogues keep their registers.
    if constexpr (BN == 256 && FUSE == 0) {
      if (cpg != 0) return cudaErrorInvalidValue;
      return dtype == kF16 ? launch2<BN, kF16, 0, 0, 1>(ta, tb, p, stream)
                           : launch2<BN, kBf16, 0, 0, 1>(ta, tb, p, stream);
    } else {
      return cudaErrorInvalidValue;
    }
  }
  if (dtype == kF16) {
    switch (cpg) {
      case 4: return launch2<BN, kF16, 4, FUSE>(ta, tb, p, stream);
      case 8: return launch2<BN, kF16, 8, FUSE>(ta, tb, p, stream);
      case 16: return launch2<BN, kF16, 16, FUSE>(ta, tb, p, stream);
      default: return launch2<BN, kF16, 0, FUSE>(ta, tb, p, stream);
    }
  }
  switch (cpg) {
    case 4: return launch2<BN, kBf16, 4, FUSE>(ta, tb, p, stream);
    case 8: return launch2<BN, kBf16, 8, FUSE>(ta, tb, p, stream);
    case 16: return launch2<BN, kBf16, 16, FUSE>(ta, tb, p, stream);
    default: return launch2<BN, kBf16, 0, FUSE>(ta, tb, p, stream);
  }
}

template <int BN>
cudaError_t conv_tc2_launch_bn(const ConvTcArgs& a, cudaStream_t stream) {
  constexpr int kBB = b_block_bytes<BN>();
  EncodeTiledFn2 encode = encode_fn2();
  if (!encode) return cudaErrorNotSupported;
  const int tile_w = a.out_w >= kM ? kM : a.out_w;
  const int tile_h = kM / tile_w;
  const bool row_shift =
      row_shift_enabled() && (a.ksize == 3 || a.ksize == 2) && a.stride == 1 && tile_h == 1;
  const CUtensorMapDataType tdt =
      a.dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta, tb;
  {
    const cuuint64_t ps = (cuuint64_t)a.pixel_stride * 2;
    cuuint64_t dims[4] = {(cuuint64_t)a.cin, (cuuint64_t)a.in_w, (cuuint64_t)a.in_h,
                          (cuuint64_t)a.batch};
    cuuint64_t strides[3] = {ps, ps * a.in_w, ps * a.in_w * a.in_h};
    cuuint32_t box[4] = {(cuuint32_t)kBK, (cuuint32_t)(tile_w * a.stride),
                         (cuuint32_t)(tile_h * a.stride), 1};
    if (row_shift) box[1] = kShiftRows;
    cuuint32_t estr[4] = {1, (cuuint32_t)a.stride, (cuuint32_t)a.stride, 1};
    if (encode(&ta, tdt, 4, const_cast<void*>(a.x), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const int k_total = a.ksize * a.ksize * a.cin;
    cuuint64_t dims[2] = {(cuuint64_t)k_total, (cuuint64_t)(a.upsample ? 4 * a.cout : a.cout)};
    cuuint64_t strides[1] = {(cuuint64_t)a.ldw * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)(BN / 2)};
    cuuint32_t estr[2] = {1, 1};
    if (encode(&tb, tdt, 2, const_cast<void*>(a.w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  Tc2Params p;
  p.tile_w = tile_w;
  p.tile_h = tile_h;
  p.tiles_x = a.out_w / tile_w;
  p.tiles_y = a.out_h / tile_h;
  p.num_m_tiles = a.batch * p.tiles_x * p.tiles_y;
  p.n_tiles = a.cout / BN;
  p.phases = a.upsample ? 4 : 1;
  p.low_h = a.in_h;
  p.low_w = a.in_w;
  p.cout_total = a.upsample ? a.cout : 0;
  p.c_blocks = a.cin / kBK;
  p.k_blocks = a.ksize * a.ksize * p.c_blocks;
  p.ksize = a.ksize;
  p.stride = a.stride;
  p.pad = a.pad;
  p.row_shift = row_shift ? 1 : 0;
  p.units = row_shift ? a.ksize * p.c_blocks : p.k_blocks;
  // The weight half stays resident when one channel tile's K blocks fit
  // (Cout 128, K <= 1152); otherwise each stage carries its weight slices.
  p.b_resident =
      (p.n_tiles == 1 && p.phases == 1 && p.k_blocks * kBB <= kMaxResidentKBlocks * 8 * 1024) ? 1 : 0;
  p.a_bytes = row_shift ? kShiftAB : kAB;
  p.a_tx = row_shift ? kShiftRows * kBK * 2 : kAB;
  p.b_tx = p.b_resident ? 0 : (row_shift ? a.ksize : 1) * kBB;
  p.stage_bytes = p.a_bytes + (int)p.b_tx;
  const int fuse = a.in_coef ? 1 : 0;
  const int resident = p.b_resident ? p.k_blocks * kBB : 0;
  p.w_stages = 0;
  if (fuse) {
    // Pixel stages alone (the transform adds latency between a stage's load
    // and its MMAs, which a deeper pixel ring hides), streamed weights in a
    // ring of their own, one tap per stage.
    p.b_tx = 0;
    p.stage_bytes = p.a_bytes;
    const int budget = Tc2Shape<1>::kBudget - resident;
    if (p.b_resident) {
      p.stages = budget / p.stage_bytes;
    } else {
      p.stages = 6;
      p.w_stages = (budget - p.stages * p.stage_bytes) / kBB;
      if (p.w_stages > kMaxStages) p.w_stages = kMaxStages;
      if (p.w_stages < 2) return cudaErrorInvalidValue;
    }
  } else {
    p.stages = (Tc2Shape<0>::kBudget - resident) / p.stage_bytes;
  }
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  if (p.stages < 2) return cudaErrorInvalidValue;
  p.bias = a.bias;
  p.residual = a.residual;
  p.ld_res = a.ld_res;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.row_scale = a.row_scale;
  const int cpg = a.gn_part ? a.gn_cpg : 0;
  p.gn_part = a.gn_part;
  p.gn_groups = cpg ? a.cout / cpg : 0;
  p.in_coef = a.in_coef;
  p.in_c = a.cin;
  p.in_silu = a.in_silu;
  p.in_y0 = a.in_y0;
  p.in_y1 = a.in_y1 < 0 ? a.in_h : a.in_y1;
  p.in_w = a.in_w;
  p.geglu = a.geglu;
  if (fuse) return launch_cpg<BN, 1>(a.dtype, cpg, ta, tb, p, stream);
  return launch_cpg<BN, 0>(a.dtype, cpg, ta, tb, p, stream);
}

}  // namespace

cudaError_t conv_tc2_launch(const ConvTcArgs& a, cudaStream_t stream) {
  if (a.cout == 128) return conv_tc2_launch_bn<128>(a, stream);
  return conv_tc2_launch_bn<256>(a, stream);
}

}  // namespace osor
