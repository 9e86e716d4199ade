// Host interface of the kernels the SDXL UNet adds to the VAE set. Activations
// are NHWC 16-bit (`dtype` kBf16 / kF16) rows of `channels`; small embedding
// vectors are f32.
#pragma once
#include <cuda_runtime.h>

namespace osor {

// features[b] = (projection of the timestep [base], pooled [pooled_width],
// projections of the six time ids [6 * tp]); projections are sinusoidal,
// cosines first.
cudaError_t unet_time_features_launch(const float* time_ids, const float* pooled, int batch,
                                      float timestep, int base, int tp, int pooled_width,
                                      float* features, cudaStream_t s);

// y[r][o] = sum_k act(x[r][k]) * w[o][k] + bias[o] + bias2[o] for rows <= 8
// (act: identity or SiLU); w 16-bit [out_f][in_f]; bias / bias2 nullable.
cudaError_t rows_linear_launch(int dtype, const float* x, int rows, int in_f, const void* w,
                               const float* bias, const float* bias2, int out_f, int pre_silu,
                               float* y, cudaStream_t s);

// Per-row LayerNorm over `channels` (multiple of 8, at most 2048), f32
// statistics, affine f32 gamma / beta.
cudaError_t layer_norm_launch(int dtype, const void* x, void* y, const float* gamma,
                              const float* beta, long long rows, int channels, float eps,
                              cudaStream_t s);

// y[r][f] = x[r][f] * gelu_erf(x[r][features + f]); features multiple of 8.
// interleaved = 1: x rows are 256-column tiles of 128 values then their 128
// gates (the GEGLU product's order; features multiple of 128).
cudaError_t geglu_launch(int dtype, const void* x, void* y, long long rows, int features,
                         cudaStream_t s, int interleaved = 0);

// y[p] = a[p] (ca channels) followed by b[p] (cb channels); ca, cb multiples of 8.
cudaError_t concat_channels_launch(const void* a, int ca, const void* b, int cb, void* y,
                                   long long pixels, cudaStream_t s);

// Nearest resize to (out_h, out_w), source index min(n - 1, floor(i * (n / out)))
// in f64; channels multiple of 8.
cudaError_t resize_nearest_launch(const void* x, void* y, int batch, int in_h, int in_w,
                                  int out_h, int out_w, int channels, cudaStream_t s);

// y[b][p][c] = x[b][p][c] + image_bias[b * bias_stride + c] + residual[b][p][c]
// for c < channels; x rows have stride ld_x (>= channels), y and residual rows
// `channels`. image_bias / residual nullable; x == y allowed when ld_x ==
// channels.
cudaError_t channel_update_launch(int dtype, const void* x, long long ld_x, void* y, int channels,
                                  long long pixels_per_image, int batch, const float* image_bias,
                                  long long bias_stride, const void* residual, cudaStream_t s);

// Multi-head softmax(q k^T) v with f32 scores: head h of row i reads
// q[b][i][h*hd .. +hd) (q already scaled), keys / values k[b][j][h*hd ..),
// v[b][j][h*hd ..) and writes out[b][i][h*hd ..). Batch strides in elements;
// kv_batch_stride 0 shares one key / value set. hd in {32, 64, 128}.
cudaError_t attention_heads_launch(int dtype, const void* q, long long ld_q, long long q_bs,
                                   const void* k, const void* v, long long ld_kv, long long kv_bs,
                                   void* out, long long ld_out, long long out_bs, int batch,
                                   int heads, int n_q, int n_kv, int head_dim, cudaStream_t s);

// The tcgen05 kernel for head width 64 (attn_heads.cu): true when it takes
// the shapes (n_q a multiple of 256, strides multiples of 8 elements, 16-byte
// aligned operands, batch strides that do not overlap).
bool attn_heads64_tc_ok(const void* q, long long ld_q, long long q_bs, const void* k,
                        const void* v, long long ld_kv, long long kv_bs, const void* out,
                        long long ld_out, long long out_bs, int n_q, int n_kv);
// Same contract as attention_heads_launch with head_dim 64.
cudaError_t attn_heads64_tc_launch(int dtype, const void* q, long long ld_q, long long q_bs,
                                   const void* k, const void* v, long long ld_kv, long long kv_bs,
                                   void* out, long long ld_out, long long out_bs, int batch,
                                   int heads, int n_q, int n_kv, cudaStream_t s);

}  // namespace osor
