// Host interface of the GroupNorm(+SiLU) kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace osor {

// Shared-memory chunk capacity of the fused NCHW kernel and CTAs per SM.
constexpr int kGnFusedSmemBytes = 96 * 1024;
constexpr int kGnFusedCtasPerSm = 2;

// Standalone NCHW GroupNorm(+SiLU) with one HBM read and write per element
// (chunks re-read from L2): gn_nchw_l2_launch. Workspace: group counters (zeroed by the launch) and
// chunk partials.
struct GnL2Plan {
  int groups_total;
  long long count;
  long long chunk;
  int P;
  int grid;
  bool feasible;  // H * W a multiple of the 16-byte vector width, groups fit one wave
  size_t workspace_bytes;
};
GnL2Plan gn_nchw_l2_plan(int batch, int channels, long long spatial, int groups, int elem_bytes);
template <typename T>
cudaError_t gn_nchw_l2_launch(const T* x, T* y, const float* gamma, const float* beta, int batch,
                              int channels, long long spatial, int groups, float eps, int silu,
                              void* workspace, float* stats_out, cudaStream_t stream);

struct GnFusedPlan {
  int groups_total;
  long long count;
  long long chunk;
  int chunks_per_group;
  int grid;
  bool feasible;  // every chunk of a group fits in one wave of resident CTAs
  size_t workspace_bytes;
};
GnFusedPlan gn_fused_plan(int batch, int channels, long long spatial, int groups, int elem_bytes);

// Standalone NCHW GroupNorm(+SiLU), T = float, __nv_bfloat16 or __half. stats_out
// (nullable) receives [batch*groups][2] = (mean, biased variance).
// extra_arrivals / wait_ns exist for the wait-expiry test only: a group then
// waits for chunks_per_group + extra_arrivals arrivals (which never come) for
// at most wait_ns (0: the library's limit) before the kernel records
// kDevWaitTimeout and returns.
template <typename T>
cudaError_t gn_fused_launch(const T* x, T* y, const float* gamma, const float* beta, int batch,
                            int channels, long long spatial, int groups, float eps, int silu,
                            void* workspace, float* stats_out, cudaStream_t stream,
                            int extra_arrivals = 0, unsigned long long wait_ns = 0);

struct GnNhwcPlan {
  int threads;
  int chunks;
  long long pix_per_chunk;
  size_t partial_bytes, coef_bytes, workspace_bytes;
  int groups;
};
GnNhwcPlan gn_nhwc_plan(int batch, int channels, long long pixels, int groups);


// NHWC 16-bit (dtype kBf16 / kF16) GroupNorm(+SiLU): stats, finalize and
// apply kernels.
cudaError_t gn_nhwc_launch(int dtype, const void* x, void* y, const float* gamma, const float* beta,
                           int batch, int channels, long long pixels, int groups, float eps,
                           int silu, void* workspace, float* stats_out, cudaStream_t stream);

// NHWC GroupNorm(+SiLU) whose statistics were produced by the preceding
// tensor-core convolution (ConvTcArgs::gn_part): finalize from the per-tile
// (mean, M2) partials, then the streaming apply. pixels % 128 == 0. `coef` is
// batch * channels * 4 floats of scratch.
// Statistics only: mean_var[b][g] = (mean, var) of 16-bit NHWC x (workspace
// as gn_nhwc_plan's partials).
cudaError_t gn_nhwc_stats_launch(int dtype, const void* x, int batch, int channels,
                                 long long pixels, int groups, void* workspace, float* mean_var,
                                 cudaStream_t stream);
// Apply only, from `parts` sets of per-(image, group) (mean, var) over equal
// element counts, part_stats[p][b][g][2], merged in the kernel; coef is
// scratch of batch * channels * 4 floats.
cudaError_t gn_nhwc_apply_stats_launch(int dtype, const void* x, void* y, const float* gamma,
                                       const float* beta, const float* part_stats, int parts,
                                       int batch, int channels, long long pixels, int groups,
                                       float eps, int silu, float* coef, cudaStream_t stream);
// Finalize only: per-channel apply coefficients coef[b][c][4] = (mean,
// rstd * gamma, beta, 0) from the per-tile partials a convolution's epilogue
// wrote (pixels % 128 == 0), for a consumer that applies them itself.
cudaError_t gn_tiles_coef_launch(const float* tile_part, int batch, int channels,
                                 long long pixels, int groups, const float* gamma,
                                 const float* beta, float eps, float* coef, float* stats_out,
                                 cudaStream_t stream);
// Coefficients only: coef[b][c] = (mean, rstd * gamma, beta, 0) from `parts`
// equal-count (mean, var) sets part_stats[p][b][g][2] (as the apply above).
cudaError_t gn_coef_from_stats_launch(const float* part_stats, int parts, int batch, int channels,
                                      int groups, const float* gamma, const float* beta,
                                      float eps, float* coef, cudaStream_t stream);
cudaError_t gn_nhwc_apply_tiles_launch(int dtype, const void* x, void* y, const float* gamma,
                                       const float* beta, int batch, int channels,
                                       long long pixels, int groups, float eps, int silu,
                                       const float* tile_part, float* coef, float* stats_out,
                                       cudaStream_t stream);

}  // namespace osor
