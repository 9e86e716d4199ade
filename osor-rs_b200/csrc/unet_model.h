// SDXL inpainting UNet runtime: weights packed once into the layouts of the
// tensor-core products (zero rows up to a multiple of 128 output channels
// where that puts a product on the tensor cores), the fixed prompt's
// cross-attention keys / values computed at load, and one denoising call
// executed as a sequence of kernel launches on one stream. Activations come
// from a stream-ordered memory pool owned by the model.
#pragma once
#include <cuda_runtime.h>

#include "vae.h"

namespace osor {

struct Unet;

Status unet_create(const osor_tensor* tensors, size_t count, const osor_unet_config* cfg,
                   const float* context, int tokens, const float* pooled, int device, Unet** out);
void unet_destroy(Unet* m);
// input [B][9][h][w] f32 (device), time_ids [B][6] f32 (device) ->
// output [B][5][h][w] f32 (device).
Status unet_denoise(const Unet& m, const float* input, int timestep, const float* time_ids,
                    float* output, int batch, int height, int width, cudaStream_t s,
                    const volatile int* cancel);

}  // namespace osor
