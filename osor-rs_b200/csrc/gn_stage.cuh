// GroupNorm(+SiLU) of a convolution's input, applied in shared memory between
// the TMA load of a row-shift stage and the MMAs that read it.
//
// A GroupNorm whose statistics the producing convolution wrote (per-tile
// partials merged into per-channel coefficients by gn_tiles_coef_launch)
// then needs no pass of its own: the consuming 3x3 convolution loads the raw
// activation and four transform warps normalise each stage in place, so the
// normalised tensor never reaches HBM. f16 works on packed pairs with no
// conversion (h = x * a + b and y = h + h * tanh(h) as f16x2 FMAs and one
// tanh.approx.f16x2 per two elements, coefficients rounded to f16); bf16
// keeps the separate apply pass's f32 arithmetic and rounding (the unpack is
// a shift), so its results are that pass's bits.
//
// The decoder uses it only on request (OSOR_FUSED_INPUT_NORM=1): on B200 the
// fused convolutions measured 1.7-2x slower than the plain ones plus the
// separate pass. Each input row is normalised once per kernel row (three
// times, six with two channel tiles), and the transform's arithmetic did not
// overlap the MMAs whatever the ring depths, the batching of its shared-memory
// accesses, the waits' back-off or the placement of its warps.
//
// Reference counterpart: the resnet's norm -> SiLU -> conv sequence
// (Resnet::forward_checked, src/native/vae_encoder.rs:134-150, with
// StableGroupNorm::forward_silu at :83-85).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace osor {

constexpr int kXfThreads = 128;  // four transform warps, one per SM sub-partition

// One thread's coefficients for its eight channels of a stage: prepared as
// in gn_coef_prepare (y = x * a + b, pre-halved when SiLU follows).
template <int D>
struct StageCoef;

template <>
struct StageCoef<kF16> {
  uint32_t a[4], b[4];  // f16x2: channels (2j, 2j + 1) of the chunk
};
template <>
struct StageCoef<kBf16> {
  float a[8], b[8];
};

// Thread tid (0..127) of the transform always handles the logical 16-byte
// chunk (tid & 7) ^ ((tid >> 3) & 7), i.e. the same eight channels, of rows
// tid / 8 + 16 k. gn_stage_coef_fetch loads those channels' entries of
// coef[img][c][4] = (mean, rstd * gamma, beta, 0) for channel block cb (the
// transform issues it one unit ahead, so the loads' latency overlaps a
// stage's work); gn_stage_coef_prepare turns them into StageCoef.
__device__ __forceinline__ void gn_stage_coef_fetch(const float* __restrict__ coef, int img,
                                                    int channels, int cb, int tid,
                                                    float4 (&raw)[8]) {
  const int lc = (tid & 7) ^ ((tid >> 3) & 7);
  const float4* cf =
      reinterpret_cast<const float4*>(coef + ((long long)img * channels + cb * 64 + lc * 8) * 4);
#pragma unroll
  for (int j = 0; j < 8; ++j) raw[j] = __ldg(cf + j);
}

template <int D>
__device__ __forceinline__ void gn_stage_coef_prepare(const float4 (&raw)[8], bool silu,
                                                      StageCoef<D>& k) {
  float a[8], b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) gn_coef_prepare(raw[j].x, raw[j].y, raw[j].z, silu, a[j], b[j]);
  if constexpr (D == kF16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 ha = __floats2half2_rn(a[2 * j], a[2 * j + 1]);
      const __half2 hb = __floats2half2_rn(b[2 * j], b[2 * j + 1]);
      k.a[j] = *reinterpret_cast<const uint32_t*>(&ha);
      k.b[j] = *reinterpret_cast<const uint32_t*>(&hb);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      k.a[j] = a[j];
      k.b[j] = b[j];
    }
  }
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t x, uint32_t a, uint32_t b) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t htanh2_u32(uint32_t x) {
  uint32_t r;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

template <int D>
__device__ __forceinline__ uint4 gn_stage_vec(uint4 v, const StageCoef<D>& k, bool silu) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (D == kF16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t h = hfma2_u32(w[j], k.a[j], k.b[j]);
      w[j] = silu ? hfma2_u32(h, htanh2_u32(h), h) : h;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = gn_apply_prepared(__uint_as_float(w[j] << 16), k.a[2 * j], k.b[2 * j], silu);
      const float hi = gn_apply_prepared(__uint_as_float(w[j] & 0xffff0000u), k.a[2 * j + 1],
                                         k.b[2 * j + 1], silu);
      w[j] = Elem<kBf16>::pack(lo, hi);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Normalise rows [0, rows) of a row-shift stage in place. Row r holds the 64
// channels of one channel block of input pixel x0 + r of one input row as
// 128 bytes whose 16-byte chunks are XOR-swizzled by r & 7 (TMA's 128-byte
// swizzle on a 1024-byte aligned stage). Pixels outside [0, width) are the
// TMA zero fill and stay zero; when the input row itself is padding (row_ok
// false: outside the tensor, or an image-edge halo row of a band) the whole
// stage is written with zeros. A thread's chunks go in batches of kXfBatch:
// all loads, then the arithmetic, then all stores (chunk by chunk, a store
// that may alias the next load would serialise every chunk's latency).
constexpr int kXfBatch = 8;

template <int D>
__device__ __forceinline__ void gn_stage_apply(uint8_t* stage, int rows, int x0, int width,
                                               bool row_ok, const StageCoef<D>& k, bool silu,
                                               int tid) {
  const int q = tid & 7;
  const int r0 = tid >> 3;
  if (!row_ok) {
#pragma unroll 4
    for (int r = r0; r < rows; r += 16)
      *reinterpret_cast<uint4*>(stage + r * 128 + q * 16) = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
#pragma unroll 1
  for (int rb = r0; rb < rows; rb += 16 * kXfBatch) {
    uint4 v[kXfBatch];
    bool in[kXfBatch];
#pragma unroll
    for (int i = 0; i < kXfBatch; ++i) {
      const int r = rb + 16 * i;
      in[i] = r < rows && (unsigned)(x0 + r) < (unsigned)width;
      if (in[i]) v[i] = *reinterpret_cast<const uint4*>(stage + r * 128 + q * 16);
    }
#pragma unroll
    for (int i = 0; i < kXfBatch; ++i)
      if (in[i]) v[i] = gn_stage_vec<D>(v[i], k, silu);
#pragma unroll
    for (int i = 0; i < kXfBatch; ++i)
      if (in[i]) *reinterpret_cast<uint4*>(stage + (rb + 16 * i) * 128 + q * 16) = v[i];
  }
}

}  // namespace osor
