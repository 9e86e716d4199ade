// Seeded standard-normal noise (the reference's stored-seed contract,
// version 1): host interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace osor {

// Output element types, numbered as the C ABI's OSOR_DTYPE_* codes.
enum : int { kNoiseBf16 = 0, kNoiseF16 = 1, kNoiseF32 = 2 };

// posterior / diffusion: `count` values each (count <= 2^18), stream 0 and 1
// of `seed`. The first call on a device copies the jump matrices to it
// (synchronously), so make it before any stream capture.
cudaError_t seeded_noise_launch(uint64_t seed, int count, int dtype, void* posterior,
                                void* diffusion, cudaStream_t stream);

}  // namespace osor
