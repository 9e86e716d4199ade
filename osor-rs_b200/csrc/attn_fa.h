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
// attn_pair_launch takes the shapes (n_q % 128 == 0, n_kv % 512 == 0, dim 512,
// 16-byte aligned operands, row strides multiples of 8 elements).
bool attn_pair_ok(int n_q, int n_kv, int dim, long long ld_q, long long ld_kv, long long ld_out,
                  const void* q, const void* k, const void* vt, const void* out);
// out[b][i][:] = softmax_j(q[b][i] . k[b][j]) v[b][j] for n_q query rows
// (stride ld_q) against n_kv key rows (stride ld_kv) per image; vt the
// per-image transposed values [batch][512][n_kv]; out rows of stride ld_out.
cudaError_t attn_pair_launch(int dtype, const void* q, long long ld_q, const void* k,
                             long long ld_kv, const void* vt, void* out, long long ld_out,
                             int batch, int n_q, int n_kv, cudaStream_t stream);

}  // namespace osor
