// Host interface of the fused GroupNorm(+SiLU) + thin 3x3 convolution (the
// VAE decoder's conv_norm_out + conv_out).
#pragma once
#include <cuda_runtime.h>

namespace osor {

// y[b][co][oy][ox] = bias[co] + sum over (ky, kx, ci) of
//   wz[(ky * 3 + kx) * 3 + co][ci] * S[b][oy + ky - 1][ox + kx - 1][ci],
// S = silu?(x * a + b) per channel from coef (zero outside the image).
//   x     NHWC 16-bit [batch][height][width][128] (dtype kBf16 / kF16)
//   coef  [batch][128][4] f32 (mean, rstd * gamma, beta, -), as
//         gn_tiles_coef_launch writes it
//   wz    16-bit [32][128]: rows 27..31 zero
//   out   NCHW f32 [batch][3][height][width]
struct GnConvOutArgs {
  int dtype = 0;
  const void* x = nullptr;
  int batch = 0, height = 0, width = 0, cin = 0;
  const float* coef = nullptr;
  int silu = 1;
  const void* wz = nullptr;
  const float* bias = nullptr;
  int cout = 0;
  float* out = nullptr;
  // normalize = 0: S = x, a plain 3x3 convolution (coef unused, may be null).
  int normalize = 1;
  // w_conv = 1: wz holds the convolution's own weights [cout][3][3][128]
  // (16-bit, rows of 9 * 128) instead of the tap matrix.
  int w_conv = 0;
};

// nullptr when the fused kernel takes the shape (Cin 128, Cout 3, width <=
// 1024), else a reason.
const char* gn_conv_out_check(const GnConvOutArgs& a);
cudaError_t gn_conv_out_launch(const GnConvOutArgs& a, cudaStream_t stream);

}  // namespace osor
