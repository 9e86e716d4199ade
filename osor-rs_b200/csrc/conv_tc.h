// Host interface of the tensor-core implicit-GEMM convolution kernel.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace osor {

// NHWC bf16 convolution (or GEMM) on tcgen05 tensor cores.
//   input   x[batch][in_h][in_w][pixel_stride] (bf16 or f16), first cin channels used
//   weight  w[cout][ldw], K = ksize*ksize*cin ordered (ky, kx, cin)
//   output  out[pixel][ld_out] (pixel = (b*out_h + oy)*out_w + ox), bf16 or f32
//   out = row_scale[pixel] * acc + bias[n] + residual[pixel][n]
// Zero padding: output (oy, ox) tap (ky, kx) reads input (oy*stride + ky - pad,
// ox*stride + kx - pad); reads outside the image are zero. A stride-2 3x3 with
// pad 0 therefore equals the reference's right/bottom zero pad then conv.
struct ConvTcArgs {
  int dtype = 0;  // Dtype of x, w, residual and a 16-bit output (kBf16 / kF16)
  const void* x = nullptr;
  int batch = 0, in_h = 0, in_w = 0, cin = 0;
  long long pixel_stride = 0;
  int ksize = 3, stride = 1, pad = 1;
  int out_h = 0, out_w = 0, cout = 0;
  const void* w = nullptr;
  long long ldw = 0;
  int w_rows = 0;  // weight rows allocated (>= cout; a thin tile reads 16, zeros past cout)
  const float* bias = nullptr;
  const void* residual = nullptr;
  long long ld_res = 0;
  void* out = nullptr;
  long long ld_out = 0;
  int out_f32 = 0;
  const float* row_scale = nullptr;
  // Optional GroupNorm partial statistics of the 16-bit output:
  // gn_part[m_tile][cout / gn_cpg][2] = (mean, M2) over each 128-pixel tile
  // and group of gn_cpg channels (gn_cpg 4, 8 or 16).
  float* gn_part = nullptr;
  int gn_cpg = 0;
  // Thin output: Cout <= 16 channels written as NCHW f32 planes
  // out[b][c][oy][ox] (out_f32 must be set); the weight buffer holds 16 rows,
  // rows >= cout zero.
  int out_nchw = 0;
  // Fused nearest-2x upsample + 3x3 conv: x is the low-res input
  // [batch][in_h][in_w], out is [batch][2 in_h][2 in_w][cout] (ld_out), ksize
  // is 2 and w holds the four phase weights [4 * cout][2 * 2 * cin] (phase
  // (a, b) = rows [(2a + b) * cout, ...)); out_h / out_w equal in_h / in_w.
  // GroupNorm partials (gn_part) are written per phase tile, image-major.
  int upsample = 0;
  // GEGLU product (1x1, Cout a multiple of 256, on CTA pairs): the weight
  // rows of each 256-row channel tile t hold the value rows t * 128 .. t * 128
  // + 127 of the projection and then the matching gate rows (bias alike); the
  // epilogue writes y[pixel][t * 128 + j] = value * gelu_erf(gate), cout / 2
  // channels (ld_out). No residual, statistics or row scale.
  int geglu = 0;
  // Softmax over each output row in two passes of the same product (the
  // attention scores, 1x1, no bias / residual / statistics, Cout a multiple
  // of 128). softmax_stats: no output is stored; for every row and every
  // block of conv_tc_softmax_block(cout) columns, (max, sum of exp(v - max))
  // goes to softmax_stats[row][block][2] (softmax_stats_ld blocks per row).
  // softmax_max: the 16-bit output is exp(v - softmax_max[row]).
  float* softmax_stats = nullptr;
  int softmax_stats_ld = 0;
  const float* softmax_max = nullptr;
  // Fused input GroupNorm(+SiLU): x is the raw activation and the kernel
  // normalises every loaded input tile with in_coef[b][c][4] = (mean,
  // rstd * gamma, beta, 0) (c < cin; the GroupNorm finalize's layout) before
  // the MMAs read it. Input rows outside [in_y0, in_y1) (in_y1 < 0: in_h)
  // are zero padding, as rows outside the tensor are; an extended band
  // tensor marks its image-edge halo rows this way. 3x3, stride 1, pad 1 on
  // the row-shift kernels only (conv_tc_check says which shapes).
  const float* in_coef = nullptr;
  int in_silu = 1;
  int in_y0 = 0, in_y1 = -1;
};

// Columns per (max, sum) partial of the softmax statistics pass.
int conv_tc_softmax_block(int cout);

// nullptr when the tensor-core kernel supports the shape, else a reason.
const char* conv_tc_check(const ConvTcArgs& a);
cudaError_t conv_tc_launch(const ConvTcArgs& a, cudaStream_t stream);

// 3x3 (pad 1) or 1x1 stride-1 convolution with Cout 64 / 128 (16-bit NHWC)
// or <= 16 (thin NCHW f32) and width % 256 == 0, with the pixels on the
// MMA's N side (256 per tile). conv_tc_launch dispatches to it first.
const char* conv_tcn_check(const ConvTcArgs& a);
cudaError_t conv_tcn_launch(const ConvTcArgs& a, cudaStream_t stream);

// Cout = 128 variant on CTA pairs with the weights resident in shared memory
// (plain 16-bit output, K <= 1152, an even number of 128-pixel tiles).
// conv_tc_launch dispatches to it when conv_tc2_check passes.
const char* conv_tc2_check(const ConvTcArgs& a);
cudaError_t conv_tc2_launch(const ConvTcArgs& a, cudaStream_t stream);

}  // namespace osor
