// Host interface of the CUDA-core support kernels. `dtype` is the Dtype
// (kBf16 / kF16) of every 16-bit tensor of the call.
#pragma once
#include <cuda_runtime.h>

namespace osor {

enum : int { kLayoutNhwc16 = 0, kLayoutNchwF32 = 1 };

struct DirectConvArgs {
  int batch = 0, in_h = 0, in_w = 0, cin = 0;
  long long in_pixel_stride = 0;  // NHWC input only
  int ksize = 3, stride = 1, pad = 1;
  int out_h = 0, out_w = 0, cout = 0;
  long long out_pixel_stride = 0;  // NHWC output only
  long long ld_res = 0;            // NHWC residual row stride
};

// Direct convolution on CUDA cores for thin layers; weights 16-bit
// [cout][ksize*ksize*cin] in (ky, kx, ci) order, bias f32 (nullable),
// residual (NHWC output only, nullable).
cudaError_t direct_conv_launch(int dtype, const void* x, int in_mode, const void* w,
                               const float* bias, const void* residual, void* out, int out_mode,
                               const DirectConvArgs& a, cudaStream_t s);

cudaError_t upsample2x_nhwc_launch(const void* x, void* y, int batch, int h, int w, int c,
                                   cudaStream_t s);

// stats [rows][ld][2] = (max, sum of exp(v - max)) for `blocks` column blocks
// of each score row -> row_max[r] and inv_sum[r] = 1 / sum of exp(v - row_max).
cudaError_t softmax_merge_launch(const float* stats, int blocks, long long ld, int rows,
                                 float* row_max, float* inv_sum, cudaStream_t s);

cudaError_t transpose16_launch(const void* in, long long ld_in, void* out, long long ld_out,
                               int rows, int cols, cudaStream_t s);

// softmax(q k^T) v on CUDA cores, one warp per query (dim <= 512): n_q query
// rows of stride ld_q against n_kv key / value rows of stride ld_kv.
cudaError_t attention_rows_launch(int dtype, const void* q, long long ld_q, const void* k,
                                  const void* v, long long ld_kv, void* out, long long ld_out,
                                  int n_q, int n_kv, int dim, cudaStream_t s);

cudaError_t nchw_f32_to_nhwc16_launch(int dtype, const float* x, void* y, int batch, int c,
                                      long long hw, cudaStream_t s);
cudaError_t nhwc16_to_nchw_f32_launch(int dtype, const void* x, float* y, int batch, int c,
                                      long long hw, cudaStream_t s);
// Column matrix [B*h*w][ncols] (16-bit, ncols 64 or 128) of a thin-input
// k x k convolution over NCHW f32 x (k*k*cin <= ncols), with an optional
// per-pixel 1x1 pre-convolution pre_w [cin][cin] + pre_b applied to x first
// (nullable).
cudaError_t thin_columns_launch(int dtype, const float* x, void* cols, int batch, int cin, int h,
                                int w, int k, int pad, const float* pre_w, const float* pre_b,
                                cudaStream_t s, int ncols = 64);

}  // namespace osor
