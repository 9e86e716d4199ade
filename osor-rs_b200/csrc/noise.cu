// Seeded standard-normal noise on the GPU (the reference's stored-seed
// contract, version 1: src/noise.rs:1-146).
//
// Each stream (0: posterior, 1: diffusion) is one xoshiro256** sequence seeded
// from SplitMix64; values are Box-Muller pairs computed in f64, rounded to
// f32, in row-major NCHW order. The sequence is inherently serial, so every
// thread takes a slice of kNoisePairs pairs and first jumps its own copy of
// the generator to the slice's start. The xoshiro256 state update is linear
// over GF(2) on the 256-bit state, so advancing by 2^k outputs is a fixed
// 256 x 256 bit matrix; the host builds the matrices for the powers of two a
// slice offset can contain once per process (by repeated squaring of the
// one-step matrix) and copies them to the device once per device. A thread's
// offset t * 2 * kNoisePairs is a sum of such powers.
#include <cstdint>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "noise.h"

namespace osor {
namespace {

constexpr int kNoisePairs = 64;        // pairs (128 values) per thread
constexpr int kNoiseSliceLog2 = 7;     // log2(2 * kNoisePairs) outputs per slice
constexpr int kNoiseJumps = 11;        // slice offsets below 2^(7 + 11) = 2^18 outputs
constexpr uint64_t kStride = 0x9E3779B97F4A7C15ull;

// Column c of jump matrix j: the state reached from basis state e_c after
// 2^(kNoiseSliceLog2 + j) steps. [j][c][word]
__device__ uint64_t g_noise_jumps[kNoiseJumps * 256 * 4];

__host__ __device__ inline uint64_t rotl64(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }

__host__ __device__ inline void xoshiro_step(uint64_t (&s)[4]) {
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
}

__host__ __device__ inline uint64_t xoshiro_next(uint64_t (&s)[4]) {
  const uint64_t result = rotl64(s[1] * 5, 7) * 9;
  xoshiro_step(s);
  return result;
}

__host__ __device__ inline void seed_stream(uint64_t seed, uint64_t stream, uint64_t (&s)[4]) {
  uint64_t mixer = seed + stream * kStride;
  for (int i = 0; i < 4; ++i) {
    mixer += kStride;
    uint64_t z = mixer;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    s[i] = z ^ (z >> 31);
  }
}

__host__ __device__ inline int ctz64(uint64_t v) {
#ifdef __CUDA_ARCH__
  return __ffsll((long long)v) - 1;
#else
  return __builtin_ctzll(v);
#endif
}

// state <- matrix (columns [256][4]) applied to state.
__host__ __device__ inline void apply_jump(const uint64_t* cols, uint64_t (&s)[4]) {
  uint64_t r0 = 0, r1 = 0, r2 = 0, r3 = 0;
  for (int w = 0; w < 4; ++w) {
    uint64_t bits = s[w];
    const uint64_t* c = cols + (size_t)w * 64 * 4;
    while (bits) {
      const int b = ctz64(bits);
      bits &= bits - 1;
      r0 ^= c[b * 4 + 0];
      r1 ^= c[b * 4 + 1];
      r2 ^= c[b * 4 + 2];
      r3 ^= c[b * 4 + 3];
    }
  }
  s[0] = r0;
  s[1] = r1;
  s[2] = r2;
  s[3] = r3;
}

template <typename O>
__device__ inline void put(void* out, int i, float v);
template <>
__device__ inline void put<float>(void* out, int i, float v) {
  static_cast<float*>(out)[i] = v;
}
template <>
__device__ inline void put<__half>(void* out, int i, float v) {
  static_cast<__half*>(out)[i] = __float2half_rn(v);
}
template <>
__device__ inline void put<__nv_bfloat16>(void* out, int i, float v) {
  static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
}

// grid (slices, 2 streams); one thread per slice of 2 * kNoisePairs values.
template <typename O>
__global__ void seeded_noise_kernel(uint64_t seed, int count, void* posterior, void* diffusion) {
  const int slice = blockIdx.x * blockDim.x + threadIdx.x;
  const int first = slice * 2 * kNoisePairs;
  if (first >= count) return;
  const uint64_t stream = blockIdx.y;
  void* out = stream == 0 ? posterior : diffusion;
  uint64_t s[4];
  seed_stream(seed, stream, s);
  for (int j = 0; j < kNoiseJumps; ++j)
    if ((slice >> j) & 1) apply_jump(g_noise_jumps + (size_t)j * 256 * 4, s);
  const double kTwoPi = 2.0 * 3.14159265358979323846;
  for (int k = 0; k < kNoisePairs; ++k) {
    const int i = first + 2 * k;
    if (i >= count) break;
    const double u1 = 1.0 - (double)(xoshiro_next(s) >> 11) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(xoshiro_next(s) >> 11) * (1.0 / 9007199254740992.0);
    const double radius = sqrt(-2.0 * log(u1));
    double sn, cs;
    sincos(kTwoPi * u2, &sn, &cs);
    put<O>(out, i, (float)(radius * cs));
    if (i + 1 < count) put<O>(out, i + 1, (float)(radius * sn));
  }
}

// Host: the jump matrices, built once per process.
const uint64_t* host_jumps() {
  static uint64_t table[kNoiseJumps * 256 * 4];
  static std::once_flag once;
  std::call_once(once, [] {
    // One-step matrix: column c = step(e_c).
    static uint64_t m[256 * 4];
    for (int c = 0; c < 256; ++c) {
      uint64_t s[4] = {0, 0, 0, 0};
      s[c / 64] = 1ull << (c % 64);
      xoshiro_step(s);
      memcpy(m + c * 4, s, sizeof(s));
    }
    // Square up to 2^kNoiseSliceLog2 steps, then keep the next kNoiseJumps powers.
    static uint64_t next[256 * 4];
    for (int k = 0; k < kNoiseSliceLog2 + kNoiseJumps; ++k) {
      if (k >= kNoiseSliceLog2) memcpy(table + (size_t)(k - kNoiseSliceLog2) * 256 * 4, m, sizeof(m));
      for (int c = 0; c < 256; ++c) {
        uint64_t s[4];
        memcpy(s, m + c * 4, sizeof(s));
        apply_jump(m, s);
        memcpy(next + c * 4, s, sizeof(s));
      }
      memcpy(m, next, sizeof(m));
    }
  });
  return table;
}

}  // namespace

cudaError_t seeded_noise_launch(uint64_t seed, int count, int dtype, void* posterior,
                                void* diffusion, cudaStream_t stream) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  static bool uploaded[64] = {false};
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    if (!uploaded[device]) {
      e = cudaMemcpyToSymbol(g_noise_jumps, host_jumps(), sizeof(g_noise_jumps));
      if (e != cudaSuccess) return e;
      uploaded[device] = true;
    }
  }
  if (count <= 0) return cudaSuccess;
  if (count > (1 << (kNoiseSliceLog2 + kNoiseJumps))) return cudaErrorInvalidValue;
  const int slices = (count + 2 * kNoisePairs - 1) / (2 * kNoisePairs);
  const dim3 grid((slices + 63) / 64, 2);
  if (dtype == kNoiseF32)
    seeded_noise_kernel<float><<<grid, 64, 0, stream>>>(seed, count, posterior, diffusion);
  else if (dtype == kNoiseF16)
    seeded_noise_kernel<__half><<<grid, 64, 0, stream>>>(seed, count, posterior, diffusion);
  else
    seeded_noise_kernel<__nv_bfloat16><<<grid, 64, 0, stream>>>(seed, count, posterior, diffusion);
  return cudaGetLastError();
}

}  // namespace osor
