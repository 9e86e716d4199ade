// Fused single-head attention (attn_fa.cu).
#pragma once
#include <cuda_runtime.h>

namespace osor {

// True when attn_fused_launch supports the shapes: tokens % 256 == 0, dim 256
// or 512, 16-byte aligned operands and row strides.
bool attn_fused_ok(int tokens, int dim, long long ld, long long ld_out, const void* q,
                   const void* k, const void* vt, const void* out);

// out[b][i][:] = softmax_j(q[b][i] . k[b][j]) v[b][j] for `batch` images of
// `tokens` rows; q / k rows of stride ld (scale already folded in), vt the
// per-image transposed values [batch][dim][tokens], out rows of stride ld_out.
// dtype: kBf16 / kF16 (all operands one 16-bit type).
cudaError_t attn_fused_launch(int dtype, const void* q, const void* k, long long ld,
                              const void* vt, void* out, long long ld_out, int batch, int tokens,
                              int dim, cudaStream_t stream);

// The CTA-pair attention (attn_pair.cu) at width 512: true when
// attn_pair_launch takes the shapes (tokens % 512 == 0, dim 512, 16-byte
// aligned operands and row strides).
bool attn_pair_ok(int tokens, int dim, long long ld, long long ld_out, const void* q,
                  const void* k, const void* vt, const void* out);
// Same contract as attn_fused_launch with dim = 512.
cudaError_t attn_pair_launch(int dtype, const void* q, const void* k, long long ld, const void* vt,
                             void* out, long long ld_out, int batch, int tokens, cudaStream_t stream);

}  // namespace osor
