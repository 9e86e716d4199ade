// Latent-space pipeline stages and DDPM scheduler arithmetic (f32): host
// interface.
#pragma once
#include <cuda_runtime.h>

namespace osor {

enum : int { kScheduleLinear = 0, kScheduleScaledLinear = 1 };
enum : int { kPredictEpsilon = 0, kPredictSample = 1, kPredictV = 2 };

// Cumulative alphas of the reference's scheduler (host). 0 on success, 1 for
// an invalid configuration, 2 when a cumulative alpha underflows.
int scheduler_alphas(int num_train_timesteps, double beta_start, double beta_end, int schedule,
                     const double* trained_betas, float* out);

cudaError_t pipeline_prepare_launch(const float* moments, const float* posterior_noise,
                                    const float* diffusion_noise, const float* mask,
                                    float* unet_input, float* sample, int batch, int h, int w,
                                    float scaling, float alpha_t, cudaStream_t s);
cudaError_t pipeline_finish_launch(const float* unet_output, const float* unet_input,
                                   float* latent_alpha, float* predicted, float* blend,
                                   float* latents, int batch, int h, int w, float alpha_t,
                                   int kind, int clip, float clip_range, float inv_scaling,
                                   cudaStream_t s);
cudaError_t pipeline_map_launch(const float* decoded, const float* latent_alpha, float* image,
                                float* alpha, int batch, int height, int width, cudaStream_t s);
// image * 2 - 1 (the encoder's input normalisation, pipeline.rs:721).
cudaError_t pipeline_normalize_launch(const float* image, float* out, long long n,
                                      cudaStream_t s);
cudaError_t scheduler_add_noise_launch(const float* original, const float* noise, float* out,
                                       long long n, float alpha_t, cudaStream_t s);
cudaError_t scheduler_predicted_launch(const float* noisy, const float* model_output, float* out,
                                       long long n, float alpha_t, int kind, int clip,
                                       float clip_range, cudaStream_t s);

}  // namespace osor
