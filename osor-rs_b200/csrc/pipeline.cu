// Latent-space stages of the reference's inference pipeline around the VAE
// (src/pipeline.rs:720-860) and its DDPM scheduler arithmetic
// (src/scheduler.rs:128-340), in f32.
//
// Every product and sum is rounded on its own (__fmul_rn / __fadd_rn): the
// reference evaluates these stages as separate tensor operations without
// fused multiply-adds, and the scheduler's pinned f32 results depend on it.
#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "pipeline.h"

namespace osor {
namespace {

int blocks(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 32;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

// The reference's sigmoid: 1 / (exp(-x) + 1).
__device__ inline float sigmoid_ref(float x) { return __frcp_rn(__fadd_rn(expf(-x), 1.0f)); }

__device__ inline float predicted_original(float noisy, float out, float os, float ns, int kind,
                                           int clip, float range) {
  float p;
  if (kind == kPredictEpsilon)
    p = __fdiv_rn(__fsub_rn(noisy, __fmul_rn(out, ns)), os);
  else if (kind == kPredictSample)
    p = out;
  else
    p = __fsub_rn(__fmul_rn(noisy, os), __fmul_rn(out, ns));
  if (clip) p = fminf(fmaxf(p, -range), range);
  return p;
}

// One latent pixel (b, y, x) per thread-iteration: posterior sample, original
// latent, pooled mask and noisy latent into unet_input [B][9][h][w] =
// (noisy, mask, original); `sample` [B][4][h][w] is optional.
__global__ void prepare_kernel(const float* __restrict__ moments, const float* __restrict__ pnoise,
                               const float* __restrict__ dnoise, const float* __restrict__ mask,
                               float* __restrict__ unet_input, float* __restrict__ sample, int batch,
                               int h, int w, float scaling, float os, float ns) {
  const long long hw = (long long)h * w, total = (long long)batch * hw;
  const int W = w * 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / hw, p = i - b * hw;
    const int y = (int)(p / w), x = (int)(p - (long long)y * w);
    float* u = unet_input + b * 9 * hw + p;
    for (int c = 0; c < 4; ++c) {
      const float mean = moments[(b * 8 + c) * hw + p];
      const float logvar = fminf(fmaxf(moments[(b * 8 + 4 + c) * hw + p], -30.0f), 20.0f);
      const float std = expf(__fmul_rn(logvar, 0.5f));
      const float s = __fadd_rn(mean, __fmul_rn(std, pnoise[(b * 4 + c) * hw + p]));
      const float original = __fmul_rn(s, scaling);
      const float noisy =
          __fadd_rn(__fmul_rn(original, os), __fmul_rn(dnoise[(b * 4 + c) * hw + p], ns));
      if (sample) sample[(b * 4 + c) * hw + p] = s;
      u[c * hw] = noisy;
      u[(5 + c) * hw] = original;
    }
    // max_pool2d(8) of the image-resolution mask.
    const float* m = mask + b * (long long)hw * 64 + (long long)(y * 8) * W + x * 8;
    float mx = m[0];
    for (int dy = 0; dy < 8; ++dy)
      for (int dx = 0; dx < 8; ++dx) mx = fmaxf(mx, m[(long long)dy * W + dx]);
    u[4 * hw] = mx;
  }
}

// unet_output [B][5][h][w] and unet_input -> latent_alpha [B][1][h][w],
// predicted original and blend [B][4][h][w] (optional), and the decoder's
// latents = blend / scaling.
__global__ void finish_kernel(const float* __restrict__ unet_output,
                              const float* __restrict__ unet_input, float* __restrict__ alpha_out,
                              float* __restrict__ predicted, float* __restrict__ blend,
                              float* __restrict__ latents, int batch, long long hw, float os,
                              float ns, int kind, int clip, float range, float inv_scaling) {
  const long long total = (long long)batch * hw;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / hw, p = i - b * hw;
    const float a = sigmoid_ref(unet_output[(b * 5 + 4) * hw + p]);
    alpha_out[i] = a;
    const float one_minus = __fadd_rn(__fmul_rn(a, -1.0f), 1.0f);
    for (int c = 0; c < 4; ++c) {
      const float noisy = unet_input[(b * 9 + c) * hw + p];
      const float original = unet_input[(b * 9 + 5 + c) * hw + p];
      const float pred = predicted_original(noisy, unet_output[(b * 5 + c) * hw + p], os, ns,
                                            kind, clip, range);
      const float bl = __fadd_rn(__fmul_rn(a, pred), __fmul_rn(one_minus, original));
      const long long o = (b * 4 + c) * hw + p;
      if (predicted) predicted[o] = pred;
      if (blend) blend[o] = bl;
      latents[o] = __fmul_rn(bl, inv_scaling);
    }
  }
}

// Bilinear source coordinate with align_corners = false (pipeline.rs:864-884):
// x = clamp((i + 0.5) * source / target - 0.5, 0, source - 1) in f64.
__device__ inline void bilinear_axis(int i, int source, int target, int& lo, int& hi, float& wt) {
  double x = ((double)i + 0.5) * (double)source / (double)target - 0.5;
  x = fmin(fmax(x, 0.0), (double)(source - 1));
  lo = (int)floor(x);
  hi = min(lo + 1, source - 1);
  wt = (float)(x - (double)lo);
}

// decoded [B][3][H][W] raw RGB -> image = clamp(0.5 x + 0.5, 0, 1); latent
// alpha [B][1][h][w] -> alpha [B][1][H][W], vertical then horizontal pass.
__global__ void map_kernel(const float* __restrict__ decoded, const float* __restrict__ latent_alpha,
                           float* __restrict__ image, float* __restrict__ alpha, int batch, int H,
                           int W) {
  const int h = H / 8, w = W / 8;
  const long long HW = (long long)H * W, total = (long long)batch * HW;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / HW, p = i - b * HW;
    const int y = (int)(p / W), x = (int)(p - (long long)y * W);
    for (int c = 0; c < 3; ++c) {
      const long long o = (b * 3 + c) * HW + p;
      image[o] = fminf(fmaxf(__fadd_rn(__fmul_rn(decoded[o], 0.5f), 0.5f), 0.0f), 1.0f);
    }
    int y0, y1, x0, x1;
    float wy, wx;
    bilinear_axis(y, h, H, y0, y1, wy);
    bilinear_axis(x, w, W, x0, x1, wx);
    const float* la = latent_alpha + b * (long long)h * w;
    const float oy = __fadd_rn(__fmul_rn(wy, -1.0f), 1.0f);
    const float ox = __fadd_rn(__fmul_rn(wx, -1.0f), 1.0f);
    const float v0 = __fadd_rn(__fmul_rn(la[y0 * w + x0], oy), __fmul_rn(la[y1 * w + x0], wy));
    const float v1 = __fadd_rn(__fmul_rn(la[y0 * w + x1], oy), __fmul_rn(la[y1 * w + x1], wy));
    alpha[i] = __fadd_rn(__fmul_rn(v0, ox), __fmul_rn(v1, wx));
  }
}

__global__ void normalize_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = __fadd_rn(__fmul_rn(x[i], 2.0f), -1.0f);
}

__global__ void add_noise_kernel(const float* __restrict__ original, const float* __restrict__ noise,
                                 float* __restrict__ out, long long n, float os, float ns) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(__fmul_rn(original[i], os), __fmul_rn(noise[i], ns));
}

__global__ void predicted_kernel(const float* __restrict__ noisy, const float* __restrict__ out_m,
                                 float* __restrict__ out, long long n, float os, float ns, int kind,
                                 int clip, float range) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = predicted_original(noisy[i], out_m[i], os, ns, kind, clip, range);
}

}  // namespace

int scheduler_alphas(int num_train_timesteps, double beta_start, double beta_end, int schedule,
                     const double* trained_betas, float* out) {
  if (num_train_timesteps <= 0 || num_train_timesteps > 100000) return 1;
  if (!std::isfinite(beta_start) || !std::isfinite(beta_end) || beta_start < 0.0 ||
      beta_start >= 1.0 || beta_end < 0.0 || beta_end >= 1.0)
    return 1;
  if (schedule != kScheduleLinear && schedule != kScheduleScaledLinear) return 1;
  const int n = num_train_timesteps;
  if (trained_betas)
    for (int i = 0; i < n; ++i)
      if (!std::isfinite(trained_betas[i]) || trained_betas[i] < 0.0 || trained_betas[i] >= 1.0)
        return 1;
  float start, end;
  if (schedule == kScheduleScaledLinear) {
    start = (float)std::sqrt(beta_start);
    end = (float)std::sqrt(beta_end);
  } else {
    start = (float)beta_start;
    end = (float)beta_end;
  }
  const float step = n == 1 ? 0.0f : (end - start) / (float)(n - 1);
  double alpha = 1.0;
  for (int i = 0; i < n; ++i) {
    float beta;
    if (trained_betas) {
      beta = (float)trained_betas[i];
    } else {
      const float point = (i < n / 2 || n == 1) ? std::fmaf(step, (float)i, start)
                                                 : std::fmaf(-step, (float)(n - i - 1), end);
      beta = schedule == kScheduleScaledLinear ? point * point : point;
    }
    alpha *= (double)(1.0f - beta);
    const float stored = (float)alpha;
    if (!std::isfinite(stored) || stored <= 0.0f) return 2;
    out[i] = stored;
  }
  return 0;
}

void scheduler_scales(float alpha_t, float* os, float* ns) {
  *os = std::sqrt(alpha_t);
  *ns = std::sqrt(1.0f - alpha_t);
}

cudaError_t pipeline_prepare_launch(const float* moments, const float* posterior_noise,
                                    const float* diffusion_noise, const float* mask,
                                    float* unet_input, float* sample, int batch, int h, int w,
                                    float scaling, float alpha_t, cudaStream_t s) {
  float os, ns;
  scheduler_scales(alpha_t, &os, &ns);
  const long long total = (long long)batch * h * w;
  prepare_kernel<<<blocks(total, 256), 256, 0, s>>>(moments, posterior_noise, diffusion_noise,
                                                     mask, unet_input, sample, batch, h, w,
                                                     scaling, os, ns);
  return cudaGetLastError();
}

cudaError_t pipeline_finish_launch(const float* unet_output, const float* unet_input,
                                   float* latent_alpha, float* predicted, float* blend,
                                   float* latents, int batch, int h, int w, float alpha_t,
                                   int kind, int clip, float clip_range, float inv_scaling,
                                   cudaStream_t s) {
  float os, ns;
  scheduler_scales(alpha_t, &os, &ns);
  const long long hw = (long long)h * w;
  finish_kernel<<<blocks((long long)batch * hw, 256), 256, 0, s>>>(
      unet_output, unet_input, latent_alpha, predicted, blend, latents, batch, hw, os, ns, kind,
      clip, clip_range, inv_scaling);
  return cudaGetLastError();
}

cudaError_t pipeline_map_launch(const float* decoded, const float* latent_alpha, float* image,
                                float* alpha, int batch, int height, int width, cudaStream_t s) {
  const long long total = (long long)batch * height * width;
  map_kernel<<<blocks(total, 256), 256, 0, s>>>(decoded, latent_alpha, image, alpha, batch, height,
                                                 width);
  return cudaGetLastError();
}

cudaError_t pipeline_normalize_launch(const float* image, float* out, long long n,
                                      cudaStream_t s) {
  normalize_kernel<<<blocks(n, 256), 256, 0, s>>>(image, out, n);
  return cudaGetLastError();
}

cudaError_t scheduler_add_noise_launch(const float* original, const float* noise, float* out,
                                       long long n, float alpha_t, cudaStream_t s) {
  float os, ns;
  scheduler_scales(alpha_t, &os, &ns);
  add_noise_kernel<<<blocks(n, 256), 256, 0, s>>>(original, noise, out, n, os, ns);
  return cudaGetLastError();
}

cudaError_t scheduler_predicted_launch(const float* noisy, const float* model_output, float* out,
                                       long long n, float alpha_t, int kind, int clip,
                                       float clip_range, cudaStream_t s) {
  float os, ns;
  scheduler_scales(alpha_t, &os, &ns);
  predicted_kernel<<<blocks(n, 256), 256, 0, s>>>(noisy, model_output, out, n, os, ns, kind, clip,
                                                   clip_range);
  return cudaGetLastError();
}

}  // namespace osor
