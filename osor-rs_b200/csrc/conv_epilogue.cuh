// GroupNorm statistics of one 32-column chunk of a convolution epilogue.
#pragma once
#include "common.cuh"

namespace osor {

// (mean, M2) of two equal-count sets of n values each, merged in place into
// (mean, m2) (Chan et al.); symmetric in its operands, so both lanes of a
// shuffle pair compute identical results.
__device__ __forceinline__ void merge_equal_counts(float& mean, float& m2, float mo, float qo,
                                                   float n) {
  const float d = mo - mean;
  m2 = m2 + qo + d * d * (0.5f * n);
  mean = 0.5f * (mean + mo);
}

// v[32]: one pixel's values of 32 consecutive channels, held by each of the
// warp's 32 lanes (32 pixels). Computes, per group of CPG channels, the
// exact two-pass (mean, M2) of every lane's CPG values and merges them over
// the 32 lanes, writing (mean, M2) of group g to out[2 g], out[2 g + 1].
//
// The merge is a transpose-reduce: at each xor step a lane hands half of the
// groups it still carries to its partner and merges the other half, so the
// groups spread over the lanes (32 / CPG groups, 32 * CPG values each) with
// five merge steps of one or a few groups instead of one butterfly per group.
// The merge itself: afterwards lane l holds (mean, m2) of group l / CPG of
// the chunk (32 * CPG values).
template <int CPG>
__device__ __forceinline__ void gn_chunk_merge(const float (&v)[32], int lane, float& mean_out,
                                               float& m2_out) {
  constexpr int G = 32 / CPG;
  float mean[G], m2[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < CPG; ++c) s += v[g * CPG + c];
    const float mu = s * (1.0f / CPG);
    float q = 0.0f;
#pragma unroll
    for (int c = 0; c < CPG; ++c) {
      const float d = v[g * CPG + c] - mu;
      q += d * d;
    }
    mean[g] = mu;
    m2[g] = q;
  }
  float n = (float)CPG;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const int s = 16 >> k;
    const int carried = G >> k;
    const bool upper = (lane & s) != 0;
    if (carried >= 2) {
      const int half = carried / 2;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send_m = upper ? mean[i] : mean[i + half];
        const float send_q = upper ? m2[i] : m2[i + half];
        float keep_m = upper ? mean[i + half] : mean[i];
        float keep_q = upper ? m2[i + half] : m2[i];
        const float mo = __shfl_xor_sync(0xffffffffu, send_m, s);
        const float qo = __shfl_xor_sync(0xffffffffu, send_q, s);
        merge_equal_counts(keep_m, keep_q, mo, qo, n);
        mean[i] = keep_m;
        m2[i] = keep_q;
      }
    } else {
      const float mo = __shfl_xor_sync(0xffffffffu, mean[0], s);
      const float qo = __shfl_xor_sync(0xffffffffu, m2[0], s);
      merge_equal_counts(mean[0], m2[0], mo, qo, n);
    }
    n *= 2.0f;
  }
  mean_out = mean[0];
  m2_out = m2[0];
}

template <int CPG>
__device__ __forceinline__ void gn_chunk_stats(const float (&v)[32], int lane, float* out) {
  float mean, m2;
  gn_chunk_merge<CPG>(v, lane, mean, m2);
  // Lane l holds group l / CPG; the first lane of each run writes it.
  if ((lane & (CPG - 1)) == 0) {
    const int g = lane / CPG;
    out[2 * g] = mean;
    out[2 * g + 1] = m2;
  }
}

}  // namespace osor
