// CUDA-core kernels around the tensor-core contractions: thin convolutions
// (Cin or Cout below the tensor-core tile), nearest 2x upsampling, the
// attention softmax and V transpose, a CUDA-core attention for shapes the
// tensor-core tiles do not cover, layout conversions and the posterior
// elementwise op. 16-bit tensors are bf16 or f16 (Dtype), chosen per call.
#include "common.cuh"
#include "ops.h"

namespace osor {
namespace {

// ------------------------------------------------------------ direct conv
// One thread per output pixel and block of COB output channels.
// Weights: 16-bit [cout][ksize*ksize*cin] ordered (ky, kx, ci).
template <int D, int IN_MODE, int OUT_MODE, int COB>
__global__ void __launch_bounds__(128)
    direct_conv_kernel(const void* __restrict__ xin, const uint16_t* __restrict__ wbits,
                       const float* __restrict__ bias, const uint16_t* __restrict__ residual,
                       void* __restrict__ out, DirectConvArgs a) {
  using E = Elem<D>;
  using T = typename E::T;
  const T* w = reinterpret_cast<const T*>(wbits);
  const long long pix = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)a.batch * a.out_h * a.out_w;
  if (pix >= total) return;
  const int co0 = blockIdx.y * COB;
  const int ox = (int)(pix % a.out_w);
  const long long t = pix / a.out_w;
  const int oy = (int)(t % a.out_h);
  const int b = (int)(t / a.out_h);
  const long long kdim = (long long)a.ksize * a.ksize * a.cin;
  float acc[COB];
#pragma unroll
  for (int j = 0; j < COB; ++j) acc[j] = 0.0f;
  for (int ky = 0; ky < a.ksize; ++ky) {
    const int iy = oy * a.stride + ky - a.pad;
    if (iy < 0 || iy >= a.in_h) continue;
    for (int kx = 0; kx < a.ksize; ++kx) {
      const int ix = ox * a.stride + kx - a.pad;
      if (ix < 0 || ix >= a.in_w) continue;
      const long long wtap = (long long)(ky * a.ksize + kx) * a.cin;
      if (IN_MODE == kLayoutNhwc16) {
        const T* xp = static_cast<const T*>(xin) +
                      (((long long)b * a.in_h + iy) * a.in_w + ix) * a.in_pixel_stride;
        if ((a.cin & 7) == 0 && (a.in_pixel_stride & 7) == 0) {
          for (int ci = 0; ci < a.cin; ci += 8) {
            float xv[8];
            unpack8<D>(__ldg(reinterpret_cast<const uint4*>(xp + ci)), xv);
#pragma unroll
            for (int j = 0; j < COB; ++j) {
              if (co0 + j < a.cout) {
                float wv[8];
                unpack8<D>(__ldg(reinterpret_cast<const uint4*>(w + (long long)(co0 + j) * kdim +
                                                                wtap + ci)),
                           wv);
#pragma unroll
                for (int u = 0; u < 8; ++u) acc[j] += xv[u] * wv[u];
              }
            }
          }
        } else {
          for (int ci = 0; ci < a.cin; ++ci) {
            const float xv = E::to_f(xp[ci]);
#pragma unroll
            for (int j = 0; j < COB; ++j)
              if (co0 + j < a.cout) acc[j] += xv * E::to_f(w[(long long)(co0 + j) * kdim + wtap + ci]);
          }
        }
      } else {  // NCHW f32
        const float* xp = static_cast<const float*>(xin);
        for (int ci = 0; ci < a.cin; ++ci) {
          const float xv = __ldg(xp + (((long long)b * a.cin + ci) * a.in_h + iy) * a.in_w + ix);
#pragma unroll
          for (int j = 0; j < COB; ++j)
            if (co0 + j < a.cout) acc[j] += xv * E::to_f(w[(long long)(co0 + j) * kdim + wtap + ci]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < COB; ++j) {
    const int co = co0 + j;
    if (co >= a.cout) continue;
    float v = acc[j] + (bias ? __ldg(bias + co) : 0.0f);
    if (OUT_MODE == kLayoutNhwc16) {
      if (residual) v += E::to_f(reinterpret_cast<const T*>(residual)[pix * a.ld_res + co]);
      static_cast<T*>(out)[pix * a.out_pixel_stride + co] = E::from_f(v);
    } else {
      const long long o = (((long long)b * a.cout + co) * a.out_h + oy) * a.out_w + ox;
      static_cast<float*>(out)[o] = v;
    }
  }
}

template <int D, int IN_MODE, int OUT_MODE>
cudaError_t direct_dispatch(const void* x, const void* w, const float* bias, const void* residual,
                            void* out, const DirectConvArgs& a, cudaStream_t s) {
  const long long total = (long long)a.batch * a.out_h * a.out_w;
  const int threads = 128;
  const unsigned gx = (unsigned)((total + threads - 1) / threads);
  const uint16_t* wb = static_cast<const uint16_t*>(w);
  const uint16_t* rb = static_cast<const uint16_t*>(residual);
  if (a.cout <= 4) {
    direct_conv_kernel<D, IN_MODE, OUT_MODE, 4>
        <<<dim3(gx, (a.cout + 3) / 4), threads, 0, s>>>(x, wb, bias, rb, out, a);
  } else {
    direct_conv_kernel<D, IN_MODE, OUT_MODE, 8>
        <<<dim3(gx, (a.cout + 7) / 8), threads, 0, s>>>(x, wb, bias, rb, out, a);
  }
  return cudaGetLastError();
}

template <int D>
cudaError_t direct_typed(const void* x, int in_mode, const void* w, const float* bias,
                         const void* residual, void* out, int out_mode, const DirectConvArgs& a,
                         cudaStream_t s) {
  if (in_mode == kLayoutNhwc16 && out_mode == kLayoutNhwc16)
    return direct_dispatch<D, kLayoutNhwc16, kLayoutNhwc16>(x, w, bias, residual, out, a, s);
  if (in_mode == kLayoutNhwc16 && out_mode == kLayoutNchwF32)
    return direct_dispatch<D, kLayoutNhwc16, kLayoutNchwF32>(x, w, bias, residual, out, a, s);
  if (in_mode == kLayoutNchwF32 && out_mode == kLayoutNhwc16)
    return direct_dispatch<D, kLayoutNchwF32, kLayoutNhwc16>(x, w, bias, residual, out, a, s);
  return direct_dispatch<D, kLayoutNchwF32, kLayoutNchwF32>(x, w, bias, residual, out, a, s);
}

// ------------------------------------------------------------ upsample
__global__ void upsample2x_nhwc_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                       int h, int w, int vc, long long total_out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total_out;
       i += (long long)gridDim.x * blockDim.x) {
    const int v = (int)(i % vc);
    long long t = i / vc;
    const int ox = (int)(t % (2 * w));
    t /= (2 * w);
    const int oy = (int)(t % (2 * h));
    const long long b = t / (2 * h);
    y[i] = __ldg(x + ((b * h + oy / 2) * w + ox / 2) * vc + v);
  }
}

// ------------------------------------------------------------ softmax
// stats[row][block] = (max, sum of exp(v - max)) over the blocks of one score
// row -> the row's max and 1 / (sum of exp(v - row max)). One warp per row.
__global__ void softmax_merge_kernel(const float2* __restrict__ stats, int blocks, long long ld,
                                     int rows, float* __restrict__ row_max,
                                     float* __restrict__ inv_sum) {
  constexpr float kLog2e = 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float2* st = stats + row * ld;
  float m = -INFINITY;
  for (int b = lane; b < blocks; b += 32) m = fmaxf(m, st[b].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.0f;
  for (int b = lane; b < blocks; b += 32) {
    const float2 v = st[b];
    l += v.y * ex2_approx((v.x - m) * kLog2e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  if (lane == 0) {
    row_max[row] = m;
    inv_sum[row] = 1.0f / l;
  }
}

// ------------------------------------------------------------ transpose
// out[c][n] = in[n][c] of 16-bit elements; 32x32 tiles through shared memory.
__global__ void transpose16_kernel(const uint16_t* __restrict__ in, long long ld_in,
                                   uint16_t* __restrict__ out, long long ld_out, int rows,
                                   int cols) {
  __shared__ uint16_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[k][threadIdx.x] = in[(long long)r * ld_in + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[(long long)c * ld_out + r] = tile[threadIdx.x][k];
  }
}

// ------------------------------------------------------------ CUDA-core attention
// One warp per query row, online softmax over keys, fp32. q already scaled.
// q rows have stride ld_q, k/v rows stride ld_kv, out rows stride ld_out
// (elements).
template <int D>
__global__ void attention_rows_kernel(const uint16_t* __restrict__ qb, long long ld_q,
                                      const uint16_t* __restrict__ kb,
                                      const uint16_t* __restrict__ vb, long long ld,
                                      uint16_t* __restrict__ ob, long long ld_out, int n_q,
                                      int tokens, int dim) {
  using E = Elem<D>;
  using T = typename E::T;
  const T* q = reinterpret_cast<const T*>(qb);
  const T* k = reinterpret_cast<const T*>(kb);
  const T* v = reinterpret_cast<const T*>(vb);
  T* out = reinterpret_cast<T*>(ob);
  extern __shared__ float qs[];  // [warps][dim]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= n_q) return;
  float* qrow = qs + warp * dim;
  for (int c = lane; c < dim; c += 32) qrow[c] = E::to_f(q[row * ld_q + c]);
  __syncwarp();
  constexpr int kMaxPer = 16;  // dim <= 512
  float acc[kMaxPer];
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) acc[j] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  for (int t = 0; t < tokens; ++t) {
    float s = 0.0f;
    for (int c = lane; c < dim; c += 32) s += qrow[c] * E::to_f(k[(long long)t * ld + c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, s);
    const float corr = __expf(m - mn);
    const float pexp = __expf(s - mn);
    l = l * corr + pexp;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int c = lane + 32 * j;
      if (c < dim) acc[j] = acc[j] * corr + pexp * E::to_f(v[(long long)t * ld + c]);
    }
    m = mn;
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int c = lane + 32 * j;
    if (c < dim) out[row * ld_out + c] = E::from_f(acc[j] * inv);
  }
}

// ------------------------------------------------------------ layouts
template <int D>
__global__ void nchw_f32_to_nhwc16_kernel(const float* __restrict__ x, uint16_t* __restrict__ yb,
                                          int c, long long hw, long long total) {
  using E = Elem<D>;
  typename E::T* y = reinterpret_cast<typename E::T*>(yb);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    const long long pix = i / c;
    const long long b = pix / hw, p = pix % hw;
    y[i] = E::from_f(__ldg(x + (b * c + ch) * hw + p));
  }
}

template <int D>
__global__ void nhwc16_to_nchw_f32_kernel(const uint16_t* __restrict__ xb, float* __restrict__ y,
                                          int c, long long hw, long long total) {
  using E = Elem<D>;
  const typename E::T* x = reinterpret_cast<const typename E::T*>(xb);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i % hw;
    const long long t = i / hw;
    const int ch = (int)(t % c);
    const long long b = t / c;
    y[i] = E::to_f(x[(b * hw + p) * c + ch]);
  }
}

// Column matrix of a thin-input convolution: for output pixel (b, oy, ox),
// column j < k*k*cin holds input channel j % cin at tap j / cin = (ky, kx)
// (zero outside the image), columns up to ncols (64 or 128) are zero. With pre_w, every input
// pixel first goes through a 1x1 convolution pre_w [cin][cin] + pre_b (the
// decoder's post_quant_conv), and padding stays zero as in the reference
// (the second convolution pads the first one's output). One thread per pixel.
template <int D>
__global__ void thin_columns_kernel(const float* __restrict__ x, uint4* __restrict__ cols,
                                    int batch, int cin, int h, int w, int k, int pad,
                                    const float* __restrict__ pre_w,
                                    const float* __restrict__ pre_b, int ncols) {
  const long long pix = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long total = (long long)batch * h * w;
  if (pix >= total) return;
  const int ox = (int)(pix % w);
  const int oy = (int)((pix / w) % h);
  const long long b = pix / ((long long)w * h);
  const long long plane = (long long)h * w;
  const float* xb = x + b * cin * plane;
  const int used = k * k * cin;
#pragma unroll 1
  for (int j0 = 0; j0 < ncols; j0 += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      float val = 0.0f;
      if (j < used) {
        const int tap = j / cin, ci = j - tap * cin;
        const int iy = oy + tap / k - pad, ix = ox + tap % k - pad;
        if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
          const long long off = (long long)iy * w + ix;
          if (pre_w) {
            val = pre_b[ci];
            for (int c = 0; c < cin; ++c) val += pre_w[ci * cin + c] * __ldg(xb + c * plane + off);
          } else {
            val = __ldg(xb + ci * plane + off);
          }
        }
      }
      v[u] = val;
    }
    cols[pix * (ncols / 8) + j0 / 8] = pack8<D>(v);
  }
}

int blocks_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 32;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

}  // namespace

cudaError_t direct_conv_launch(int dtype, const void* x, int in_mode, const void* w,
                               const float* bias, const void* residual, void* out, int out_mode,
                               const DirectConvArgs& a, cudaStream_t s) {
  if (dtype == kF16) return direct_typed<kF16>(x, in_mode, w, bias, residual, out, out_mode, a, s);
  return direct_typed<kBf16>(x, in_mode, w, bias, residual, out, out_mode, a, s);
}

cudaError_t upsample2x_nhwc_launch(const void* x, void* y, int batch, int h, int w, int c,
                                   cudaStream_t s) {
  if (c % 8 != 0) return cudaErrorInvalidValue;
  const long long total = (long long)batch * 4 * h * w * (c / 8);
  upsample2x_nhwc_kernel<<<blocks_for(total, 256), 256, 0, s>>>(
      static_cast<const uint4*>(x), static_cast<uint4*>(y), h, w, c / 8, total);
  return cudaGetLastError();
}

cudaError_t softmax_merge_launch(const float* stats, int blocks, long long ld, int rows,
                                 float* row_max, float* inv_sum, cudaStream_t s) {
  const int warps = 8;
  softmax_merge_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      reinterpret_cast<const float2*>(stats), blocks, ld, rows, row_max, inv_sum);
  return cudaGetLastError();
}

cudaError_t transpose16_launch(const void* in, long long ld_in, void* out, long long ld_out,
                               int rows, int cols, cudaStream_t s) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose16_kernel<<<grid, dim3(32, 8), 0, s>>>(static_cast<const uint16_t*>(in), ld_in,
                                                   static_cast<uint16_t*>(out), ld_out, rows, cols);
  return cudaGetLastError();
}

cudaError_t attention_rows_launch(int dtype, const void* q, long long ld_q, const void* k,
                                  const void* v, long long ld_kv, void* out, long long ld_out,
                                  int n_q, int n_kv, int dim, cudaStream_t s) {
  if (dim > 512) return cudaErrorInvalidValue;
  const int warps = 4;
  const dim3 grid((n_q + warps - 1) / warps);
  const size_t smem = (size_t)warps * dim * sizeof(float);
  const uint16_t* qb = static_cast<const uint16_t*>(q);
  const uint16_t* kb = static_cast<const uint16_t*>(k);
  const uint16_t* vb = static_cast<const uint16_t*>(v);
  uint16_t* ob = static_cast<uint16_t*>(out);
  if (dtype == kF16)
    attention_rows_kernel<kF16><<<grid, warps * 32, smem, s>>>(qb, ld_q, kb, vb, ld_kv, ob, ld_out,
                                                               n_q, n_kv, dim);
  else
    attention_rows_kernel<kBf16><<<grid, warps * 32, smem, s>>>(qb, ld_q, kb, vb, ld_kv, ob,
                                                                ld_out, n_q, n_kv, dim);
  return cudaGetLastError();
}

cudaError_t nchw_f32_to_nhwc16_launch(int dtype, const float* x, void* y, int batch, int c,
                                      long long hw, cudaStream_t s) {
  const long long total = (long long)batch * c * hw;
  uint16_t* yb = static_cast<uint16_t*>(y);
  if (dtype == kF16)
    nchw_f32_to_nhwc16_kernel<kF16><<<blocks_for(total, 256), 256, 0, s>>>(x, yb, c, hw, total);
  else
    nchw_f32_to_nhwc16_kernel<kBf16><<<blocks_for(total, 256), 256, 0, s>>>(x, yb, c, hw, total);
  return cudaGetLastError();
}

cudaError_t nhwc16_to_nchw_f32_launch(int dtype, const void* x, float* y, int batch, int c,
                                      long long hw, cudaStream_t s) {
  const long long total = (long long)batch * c * hw;
  const uint16_t* xb = static_cast<const uint16_t*>(x);
  if (dtype == kF16)
    nhwc16_to_nchw_f32_kernel<kF16><<<blocks_for(total, 256), 256, 0, s>>>(xb, y, c, hw, total);
  else
    nhwc16_to_nchw_f32_kernel<kBf16><<<blocks_for(total, 256), 256, 0, s>>>(xb, y, c, hw, total);
  return cudaGetLastError();
}

cudaError_t thin_columns_launch(int dtype, const float* x, void* cols, int batch, int cin, int h,
                                int w, int k, int pad, const float* pre_w, const float* pre_b,
                                cudaStream_t s, int ncols) {
  if ((ncols != 64 && ncols != 128) || k * k * cin > ncols) return cudaErrorInvalidValue;
  const long long total = (long long)batch * h * w;
  const unsigned grid = (unsigned)((total + 127) / 128);
  uint4* c = static_cast<uint4*>(cols);
  if (dtype == kF16)
    thin_columns_kernel<kF16><<<grid, 128, 0, s>>>(x, c, batch, cin, h, w, k, pad, pre_w, pre_b,
                                                   ncols);
  else
    thin_columns_kernel<kBf16><<<grid, 128, 0, s>>>(x, c, batch, cin, h, w, k, pad, pre_w, pre_b,
                                                    ncols);
  return cudaGetLastError();
}

}  // namespace osor
