// CUDA kernels of the SDXL UNet beyond the VAE set: the time / added
// embedding inputs, small-row linear layers (time embeddings and every
// resnet's time_emb_proj in one launch), the transformer blocks' LayerNorm,
// GEGLU and multi-head attention, and the NHWC skip concatenation, nearest
// resize and per-image channel bias / narrowing epilogue. The convolutions,
// GroupNorm and linear projections over pixels run on the tensor-core and
// GroupNorm kernels shared with the VAE.
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "unet.h"

namespace osor {
namespace {

int grid_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = 148LL * 32;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------ time features
// Frequency i of a projection with `half` frequencies, in the reference's f32
// operation order: (i * f32(-ln 1e4)) * f32(1 / half), then exp.
__device__ __forceinline__ float projection_frequency(int i, int half) {
  const float neg_ln = (float)(-9.210340371976184);
  const float inv = (float)(1.0 / (double)half);
  return expf(((float)i * neg_ln) * inv);
}

// cos for the first half of a projection, sin for the second, of the f32
// product t * freq (evaluated in f64 and rounded once).
__device__ __forceinline__ float projection_value(float t, int r, int width) {
  const int half = width / 2;
  const int i = r < half ? r : r - half;
  const float arg = t * projection_frequency(i, half);
  return (float)(r < half ? cos((double)arg) : sin((double)arg));
}

__global__ void unet_time_features_kernel(const float* __restrict__ time_ids,
                                          const float* __restrict__ pooled, int batch, float t,
                                          int base, int tp, int pooled_width,
                                          float* __restrict__ features) {
  const int row_w = base + pooled_width + 6 * tp;
  const long long total = (long long)batch * row_w;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / row_w);
    const int r = (int)(i % row_w);
    float v;
    if (r < base) {
      v = projection_value(t, r, base);
    } else if (r < base + pooled_width) {
      v = pooled[r - base];
    } else {
      const int c = r - base - pooled_width;
      v = projection_value(time_ids[b * 6 + c / tp], c % tp, tp);
    }
    features[i] = v;
  }
}

// ------------------------------------------------------------ small-row linear
// One warp per output feature; the (activated) rows sit in shared memory.
constexpr int kLinearMaxRows = 8;
constexpr int kLinearSmemFloats = 12 * 1024;  // 48 KB

template <int D>
__global__ void __launch_bounds__(256)
    rows_linear_kernel(const float* __restrict__ x, int rows, int in_f,
                       const uint16_t* __restrict__ wbits, const float* __restrict__ bias,
                       const float* __restrict__ bias2, int out_f, int pre_silu,
                       float* __restrict__ y) {
  using E = Elem<D>;
  using T = typename E::T;
  __shared__ __align__(16) float xs[kLinearSmemFloats];
  for (int i = threadIdx.x; i < rows * in_f; i += blockDim.x) {
    float v = x[i];
    if (pre_silu) v = v / (1.0f + expf(-v));
    xs[i] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * (blockDim.x >> 5) + warp;
  if (o >= out_f) return;
  const T* w = reinterpret_cast<const T*>(wbits) + (long long)o * in_f;
  float acc[kLinearMaxRows];
#pragma unroll
  for (int r = 0; r < kLinearMaxRows; ++r) acc[r] = 0.0f;
  if ((in_f & 7) == 0) {
    for (int k = lane * 8; k < in_f; k += 256) {
      float wv[8];
      unpack8<D>(__ldg(reinterpret_cast<const uint4*>(w + k)), wv);
#pragma unroll
      for (int r = 0; r < kLinearMaxRows; ++r) {
        if (r < rows) {
          const float4 a = *reinterpret_cast<const float4*>(xs + r * in_f + k);
          const float4 c = *reinterpret_cast<const float4*>(xs + r * in_f + k + 4);
          acc[r] += wv[0] * a.x + wv[1] * a.y + wv[2] * a.z + wv[3] * a.w + wv[4] * c.x +
                    wv[5] * c.y + wv[6] * c.z + wv[7] * c.w;
        }
      }
    }
  } else {
    for (int k = lane; k < in_f; k += 32) {
      const float wv = E::to_f(w[k]);
#pragma unroll
      for (int r = 0; r < kLinearMaxRows; ++r)
        if (r < rows) acc[r] += wv * xs[r * in_f + k];
    }
  }
  const float add = (bias ? bias[o] : 0.0f) + (bias2 ? bias2[o] : 0.0f);
#pragma unroll
  for (int r = 0; r < kLinearMaxRows; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0 && r < rows) y[(long long)r * out_f + o] = v + add;
  }
}

// ------------------------------------------------------------ LayerNorm
constexpr int kLnMaxVec = 8;  // 8-channel vectors per lane: channels <= 2048

// VPL: 8-channel vectors per lane held in registers (ceil(C / 256) or more).
template <int D, int VPL>
__global__ void __launch_bounds__(256)
    layer_norm_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                      const float* __restrict__ gamma, const float* __restrict__ beta,
                      long long rows, int channels, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  const int vc = channels / 8;
  const uint4* src = x + row * vc;
  float v[VPL][8];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c8 = lane + 32 * j;
    if (c8 < vc) {
      unpack8<D>(__ldg(src + c8), v[j]);
#pragma unroll
      for (int u = 0; u < 8; ++u) s += v[j][u];
    }
  }
  const float mean = warp_sum(s) / (float)channels;
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c8 = lane + 32 * j;
    if (c8 < vc) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float d = v[j][u] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)channels + eps);
  uint4* dst = y + row * vc;
  // gamma / beta as 16-byte vectors (eight channels in four loads).
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int c8 = lane + 32 * j;
    if (c8 < vc) {
      const float4 ga = __ldg(g4 + 2 * c8), gb = __ldg(g4 + 2 * c8 + 1);
      const float4 ba = __ldg(b4 + 2 * c8), bb = __ldg(b4 + 2 * c8 + 1);
      const float gm[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      const float bt[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = (v[j][u] - mean) * rstd * gm[u] + bt[u];
      dst[c8] = pack8<D>(o);
    }
  }
}

// ------------------------------------------------------------ GEGLU
// interleaved = 0: row r holds the values in columns [0, features) and the
// gates in [features, 2 features). interleaved = 1: 256-column tiles of 128
// values then their 128 gates (the GEGLU product's weight-row order).
template <int D>
__global__ void geglu_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, long long rows,
                             int features, int interleaved) {
  const int vf = features / 8;
  const long long total = rows * vf;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / vf;
    const int c = (int)(i % vf);
    // 16 vectors of 8 channels per 128-channel block.
    const int vc = interleaved ? (c >> 4) * 32 + (c & 15) : c;
    const int vg = interleaved ? vc + 16 : vf + c;
    float a[8], g[8], o[8];
    unpack8<D>(__ldg(x + r * 2 * vf + vc), a);
    unpack8<D>(__ldg(x + r * 2 * vf + vg), g);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      o[u] = a[u] * (0.5f * g[u] * (1.0f + erff(g[u] * 0.70710678118654752f)));
    y[i] = pack8<D>(o);
  }
}

// ------------------------------------------------------------ layout ops
__global__ void concat_channels_kernel(const uint4* __restrict__ a, int va,
                                       const uint4* __restrict__ b, int vb,
                                       uint4* __restrict__ y, long long pixels) {
  const int vy = va + vb;
  const long long total = pixels * vy;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / vy;
    const int c = (int)(i % vy);
    y[i] = c < va ? __ldg(a + p * va + c) : __ldg(b + p * vb + (c - va));
  }
}

__global__ void resize_nearest_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                                      int batch, int in_h, int in_w, int out_h, int out_w,
                                      int vc) {
  const long long total = (long long)batch * out_h * out_w * vc;
  const double sh = (double)in_h / (double)out_h, sw = (double)in_w / (double)out_w;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % vc);
    long long t = i / vc;
    const int ox = (int)(t % out_w);
    t /= out_w;
    const int oy = (int)(t % out_h);
    const long long b = t / out_h;
    const int sy = min(in_h - 1, (int)((double)oy * sh));
    const int sx = min(in_w - 1, (int)((double)ox * sw));
    y[i] = __ldg(x + ((b * in_h + sy) * in_w + sx) * vc + c);
  }
}

// x and y may alias (in place when ld_x == channels): no __restrict__.
template <int D>
__global__ void channel_update_kernel(const uint4* x, long long vx, uint4* y, int vc,
                                      long long pixels_per_image, long long pixels,
                                      const float* __restrict__ image_bias, long long bias_stride,
                                      const uint4* __restrict__ residual) {
  const long long total = pixels * vc;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / vc;
    const int c8 = (int)(i % vc);
    float v[8];
    unpack8<D>(x[p * vx + c8], v);
    if (image_bias) {
      const float* bb = image_bias + (p / pixels_per_image) * bias_stride + c8 * 8;
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(bb));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(bb) + 1);
      v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
      v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
    }
    if (residual) {
      float r[8];
      unpack8<D>(__ldg(residual + i), r);
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] += r[u];
    }
    y[i] = pack8<D>(v);
  }
}

// ------------------------------------------------------------ multi-head attention
// Block: 4 warps. A query row is served by G = HD / 8 lanes; lane t of the
// group owns dims [4t, 4t + 4) and [HD/2 + 4t, HD/2 + 4t + 4), so that the
// group's float4 reads of a key row are contiguous. Key / value tiles of 32
// rows are converted to f32 in shared memory once per block and shared by its
// 4 * 32 / G query rows. Scores, the running max / sum and the output
// accumulators are f32; the softmax is rescaled once per tile.
constexpr int kAttnWarps = 4;
constexpr int kAttnKeys = 32;

template <int D>
__device__ __forceinline__ float4 unpack4(uint2 w) {
  const float2 a = Elem<D>::unpack(w.x), b = Elem<D>::unpack(w.y);
  return make_float4(a.x, a.y, b.x, b.y);
}

template <int D, int HD>
__global__ void __launch_bounds__(kAttnWarps * 32)
    attention_heads_kernel(const uint16_t* __restrict__ qb, long long ld_q, long long q_bs,
                           const uint16_t* __restrict__ kb, const uint16_t* __restrict__ vb,
                           long long ld_kv, long long kv_bs, uint16_t* __restrict__ ob,
                           long long ld_out, long long out_bs, int n_q, int n_kv) {
  constexpr int G = HD / 8;
  constexpr int RPW = 32 / G;
  constexpr int kRows = RPW * kAttnWarps;
  constexpr int VPR = HD / 8;  // 16-byte vectors per key row
  __shared__ __align__(16) float ks[kAttnKeys * HD];
  __shared__ __align__(16) float vs[kAttnKeys * HD];
  using E = Elem<D>;
  const int h = blockIdx.y;
  const long long b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / G, t = lane % G;
  const long long row = (long long)blockIdx.x * kRows + warp * RPW + sub;
  const bool valid = row < n_q;
  const long long rr = valid ? row : (long long)n_q - 1;
  const int d0 = 4 * t, d1 = HD / 2 + 4 * t;
  const uint16_t* qrow = qb + b * q_bs + rr * ld_q + (long long)h * HD;
  const float4 q0 = unpack4<D>(__ldg(reinterpret_cast<const uint2*>(qrow + d0)));
  const float4 q1 = unpack4<D>(__ldg(reinterpret_cast<const uint2*>(qrow + d1)));
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
  float m = -INFINITY, l = 0.0f;
  const uint16_t* kbase = kb + b * kv_bs + (long long)h * HD;
  const uint16_t* vbase = vb + b * kv_bs + (long long)h * HD;
  for (int j0 = 0; j0 < n_kv; j0 += kAttnKeys) {
    __syncthreads();  // the previous tile is consumed
    for (int i = threadIdx.x; i < kAttnKeys * VPR; i += kAttnWarps * 32) {
      const int kk = i / VPR, c = i % VPR;
      const int j = j0 + kk;
      float kf[8], vf[8];
      if (j < n_kv) {
        unpack8<D>(__ldg(reinterpret_cast<const uint4*>(kbase + (long long)j * ld_kv) + c), kf);
        unpack8<D>(__ldg(reinterpret_cast<const uint4*>(vbase + (long long)j * ld_kv) + c), vf);
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) kf[u] = vf[u] = 0.0f;
      }
      float4* kd = reinterpret_cast<float4*>(ks + kk * HD + c * 8);
      float4* vd = reinterpret_cast<float4*>(vs + kk * HD + c * 8);
      kd[0] = make_float4(kf[0], kf[1], kf[2], kf[3]);
      kd[1] = make_float4(kf[4], kf[5], kf[6], kf[7]);
      vd[0] = make_float4(vf[0], vf[1], vf[2], vf[3]);
      vd[1] = make_float4(vf[4], vf[5], vf[6], vf[7]);
    }
    __syncthreads();
    const int nk = min(kAttnKeys, n_kv - j0);
    float s[kAttnKeys];
    float mt = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < kAttnKeys; ++kk) {
      const float4 k0 = *reinterpret_cast<const float4*>(ks + kk * HD + d0);
      const float4 k1 = *reinterpret_cast<const float4*>(ks + kk * HD + d1);
      float p = q0.x * k0.x;
      p = fmaf(q0.y, k0.y, p);
      p = fmaf(q0.z, k0.z, p);
      p = fmaf(q0.w, k0.w, p);
      p = fmaf(q1.x, k1.x, p);
      p = fmaf(q1.y, k1.y, p);
      p = fmaf(q1.z, k1.z, p);
      p = fmaf(q1.w, k1.w, p);
#pragma unroll
      for (int o = G / 2; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      s[kk] = kk < nk ? p : -INFINITY;
      mt = fmaxf(mt, s[kk]);
    }
    const float mn = fmaxf(m, mt);
    const float corr = __expf(m - mn);
    l *= corr;
    a0.x *= corr; a0.y *= corr; a0.z *= corr; a0.w *= corr;
    a1.x *= corr; a1.y *= corr; a1.z *= corr; a1.w *= corr;
#pragma unroll
    for (int kk = 0; kk < kAttnKeys; ++kk) {
      const float p = __expf(s[kk] - mn);
      l += p;
      const float4 v0 = *reinterpret_cast<const float4*>(vs + kk * HD + d0);
      const float4 v1 = *reinterpret_cast<const float4*>(vs + kk * HD + d1);
      a0.x = fmaf(p, v0.x, a0.x); a0.y = fmaf(p, v0.y, a0.y);
      a0.z = fmaf(p, v0.z, a0.z); a0.w = fmaf(p, v0.w, a0.w);
      a1.x = fmaf(p, v1.x, a1.x); a1.y = fmaf(p, v1.y, a1.y);
      a1.z = fmaf(p, v1.z, a1.z); a1.w = fmaf(p, v1.w, a1.w);
    }
    m = mn;
  }
  if (valid) {
    const float inv = 1.0f / l;
    uint16_t* orow = ob + b * out_bs + row * ld_out + (long long)h * HD;
    reinterpret_cast<uint2*>(orow + d0)[0] =
        make_uint2(E::pack(a0.x * inv, a0.y * inv), E::pack(a0.z * inv, a0.w * inv));
    reinterpret_cast<uint2*>(orow + d1)[0] =
        make_uint2(E::pack(a1.x * inv, a1.y * inv), E::pack(a1.z * inv, a1.w * inv));
  }
}

// Head width 64 on the tensor cores (mma.sync m16n8k16, f32 accumulate),
// flash-style: each warp owns 16 query rows with Q held as A fragments; per
// 64-key tile, S = Q K^T lands in f32 accumulators, the online softmax runs on
// those fragments (row max / sum across the 4 lanes of a quad), P is repacked
// in registers as the A operand of O += P V. K and V tiles are staged in
// shared memory as [key][dim] rows of 72 elements (144 bytes: the eight rows of
// an ldmatrix phase fall in distinct banks); B fragments come from ldmatrix,
// transposed for V. Fragment layouts are the PTX ISA's for
// m16n8k16: lane = 4 * group + t; A holds (row group / group + 8, cols 2t,
// 2t + 1, +8), B (k 2t, 2t + 1, +8; n group), C (row group / group + 8,
// cols 2t, 2t + 1).
constexpr int kMmaWarps = 4;
constexpr int kMmaRows = 16 * kMmaWarps;  // query rows per block
constexpr int kMmaKeys = 64;              // keys per tile
constexpr int kMmaLd = 72;                // shared row stride in elements

template <int D>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if (D == kF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Four 8 x 8 16-bit matrices from shared memory; lanes 8m .. 8m + 7 give the
// row addresses of matrix m, and r[m] receives the lane's element pair of it:
// (row lane / 4, cols 2 (lane % 4), +1), or with .trans (rows 2 (lane % 4), +1,
// col lane / 4), i.e. a B fragment of the transposed storage.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const uint16_t* row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(row)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const uint16_t* row) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(row)));
}

template <int D>
__global__ void __launch_bounds__(kMmaWarps * 32)
    attention_heads64_mma_kernel(const uint16_t* __restrict__ qb, long long ld_q, long long q_bs,
                                 const uint16_t* __restrict__ kb, const uint16_t* __restrict__ vb,
                                 long long ld_kv, long long kv_bs, uint16_t* __restrict__ ob,
                                 long long ld_out, long long out_bs, int n_q, int n_kv) {
  constexpr int HD = 64;
  __shared__ __align__(16) uint16_t ks[kMmaKeys * kMmaLd];
  __shared__ __align__(16) uint16_t vs[kMmaKeys * kMmaLd];
  using E = Elem<D>;
  const int h = blockIdx.y;
  const long long b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const long long ra = (long long)blockIdx.x * kMmaRows + warp * 16 + g;
  const long long rb = ra + 8;
  const bool va = ra < n_q, vb8 = rb < n_q;
  const uint16_t* qbase = qb + b * q_bs + (long long)h * HD;
  uint32_t qa[4][4];
#pragma unroll
  for (int kst = 0; kst < 4; ++kst) {
    const int c0 = kst * 16 + 2 * t;
    qa[kst][0] = va ? __ldg(reinterpret_cast<const uint32_t*>(qbase + ra * ld_q + c0)) : 0u;
    qa[kst][1] = vb8 ? __ldg(reinterpret_cast<const uint32_t*>(qbase + rb * ld_q + c0)) : 0u;
    qa[kst][2] = va ? __ldg(reinterpret_cast<const uint32_t*>(qbase + ra * ld_q + c0 + 8)) : 0u;
    qa[kst][3] = vb8 ? __ldg(reinterpret_cast<const uint32_t*>(qbase + rb * ld_q + c0 + 8)) : 0u;
  }
  float o[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const uint16_t* kbase = kb + b * kv_bs + (long long)h * HD;
  const uint16_t* vbase = vb + b * kv_bs + (long long)h * HD;
  for (int j0 = 0; j0 < n_kv; j0 += kMmaKeys) {
    __syncthreads();  // the previous tile is consumed
    for (int i = threadIdx.x; i < kMmaKeys * (HD / 8); i += kMmaWarps * 32) {
      const int key = i >> 3, c = i & 7;
      const int j = j0 + key;
      uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
      if (j < n_kv) {
        kv = __ldg(reinterpret_cast<const uint4*>(kbase + (long long)j * ld_kv) + c);
        vv = __ldg(reinterpret_cast<const uint4*>(vbase + (long long)j * ld_kv) + c);
      }
      *reinterpret_cast<uint4*>(ks + key * kMmaLd + c * 8) = kv;
      *reinterpret_cast<uint4*>(vs + key * kMmaLd + c * 8) = vv;
    }
    __syncthreads();
    // S = Q K^T for 8 tiles of 8 keys. One ldmatrix gives the B fragments of
    // two key steps: matrices (dims 32 kp + 0, 8, 16, 24) of the tile's 8 keys.
    const int lrow = lane & 7, lmat = lane >> 3;
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t bk[4];
        ldsm_x4(bk, ks + (nt * 8 + lrow) * kMmaLd + 32 * kp + 8 * lmat);
        mma16816<D>(sc[nt], qa[2 * kp], bk[0], bk[1]);
        mma16816<D>(sc[nt], qa[2 * kp + 1], bk[2], bk[3]);
      }
    }
    // Mask keys past the end, then the tile's row maxima over the quad.
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int key = j0 + nt * 8 + 2 * t;
      if (key >= n_kv) sc[nt][0] = sc[nt][2] = -INFINITY;
      if (key + 1 >= n_kv) sc[nt][1] = sc[nt][3] = -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = __expf(m0 - mx0), c1 = __expf(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= c0;
      o[nt][1] *= c0;
      o[nt][2] *= c1;
      o[nt][3] *= c1;
    }
    // P = exp(S - max) as the A fragments of the 4 key steps of P V.
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = __expf(sc[nt][0] - m0), p1 = __expf(sc[nt][1] - m0);
      const float p2 = __expf(sc[nt][2] - m1), p3 = __expf(sc[nt][3] - m1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[nt >> 1][(nt & 1) * 2] = E::pack(p0, p1);
      pa[nt >> 1][(nt & 1) * 2 + 1] = E::pack(p2, p3);
    }
    // O += P V: transposed ldmatrix of [key][dim] rows gives the B fragments
    // (keys 2t, 2t + 1 of dim column g) of two key steps per load.
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t bv[4];
        ldsm_x4_trans(bv, vs + (32 * kp + 8 * lmat + lrow) * kMmaLd + nt * 8);
        mma16816<D>(o[nt], pa[2 * kp], bv[0], bv[1]);
        mma16816<D>(o[nt], pa[2 * kp + 1], bv[2], bv[3]);
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
  uint16_t* obase = ob + b * out_bs + (long long)h * HD + 2 * t;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    if (va)
      *reinterpret_cast<uint32_t*>(obase + ra * ld_out + nt * 8) =
          E::pack(o[nt][0] * i0, o[nt][1] * i0);
    if (vb8)
      *reinterpret_cast<uint32_t*>(obase + rb * ld_out + nt * 8) =
          E::pack(o[nt][2] * i1, o[nt][3] * i1);
  }
}

// Head width 64 takes the tcgen05 kernel (attn_heads.cu) where its shapes
// allow; OSOR_HEADS_TC=0 in the environment (read once) keeps the mma.sync
// kernel for every shape, for comparing.
bool heads_tc_enabled() {
  static const bool on = [] {
    const char* v = getenv("OSOR_HEADS_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int D>
cudaError_t attention_heads_typed(const void* q, long long ld_q, long long q_bs, const void* k,
                                  const void* v, long long ld_kv, long long kv_bs, void* out,
                                  long long ld_out, long long out_bs, int batch, int heads,
                                  int n_q, int n_kv, int head_dim, cudaStream_t s) {
  const uint16_t* qb = static_cast<const uint16_t*>(q);
  const uint16_t* kb = static_cast<const uint16_t*>(k);
  const uint16_t* vb = static_cast<const uint16_t*>(v);
  uint16_t* ob = static_cast<uint16_t*>(out);
  const dim3 block(kAttnWarps * 32);
  auto grid = [&](int rows) { return dim3((unsigned)((n_q + rows - 1) / rows), heads, batch); };
  switch (head_dim) {
    case 32:
      attention_heads_kernel<D, 32><<<grid(8 * kAttnWarps), block, 0, s>>>(
          qb, ld_q, q_bs, kb, vb, ld_kv, kv_bs, ob, ld_out, out_bs, n_q, n_kv);
      break;
    case 64:
      if (heads_tc_enabled() &&
          attn_heads64_tc_ok(q, ld_q, q_bs, k, v, ld_kv, kv_bs, out, ld_out, out_bs, n_q, n_kv))
        return attn_heads64_tc_launch(D, q, ld_q, q_bs, k, v, ld_kv, kv_bs, out, ld_out, out_bs,
                                      batch, heads, n_q, n_kv, s);
      attention_heads64_mma_kernel<D><<<grid(kMmaRows), dim3(kMmaWarps * 32), 0, s>>>(
          qb, ld_q, q_bs, kb, vb, ld_kv, kv_bs, ob, ld_out, out_bs, n_q, n_kv);
      break;
    case 128:
      attention_heads_kernel<D, 128><<<grid(2 * kAttnWarps), block, 0, s>>>(
          qb, ld_q, q_bs, kb, vb, ld_kv, kv_bs, ob, ld_out, out_bs, n_q, n_kv);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t unet_time_features_launch(const float* time_ids, const float* pooled, int batch,
                                      float timestep, int base, int tp, int pooled_width,
                                      float* features, cudaStream_t s) {
  const long long total = (long long)batch * (base + pooled_width + 6 * tp);
  unet_time_features_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      time_ids, pooled, batch, timestep, base, tp, pooled_width, features);
  return cudaGetLastError();
}

cudaError_t rows_linear_launch(int dtype, const float* x, int rows, int in_f, const void* w,
                               const float* bias, const float* bias2, int out_f, int pre_silu,
                               float* y, cudaStream_t s) {
  if (rows < 1 || rows > kLinearMaxRows || (long long)rows * in_f > kLinearSmemFloats)
    return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((out_f + 7) / 8);
  const uint16_t* wb = static_cast<const uint16_t*>(w);
  if (dtype == kF16)
    rows_linear_kernel<kF16><<<grid, 256, 0, s>>>(x, rows, in_f, wb, bias, bias2, out_f, pre_silu, y);
  else
    rows_linear_kernel<kBf16><<<grid, 256, 0, s>>>(x, rows, in_f, wb, bias, bias2, out_f, pre_silu, y);
  return cudaGetLastError();
}

cudaError_t layer_norm_launch(int dtype, const void* x, void* y, const float* gamma,
                              const float* beta, long long rows, int channels, float eps,
                              cudaStream_t s) {
  if (channels % 8 != 0 || channels / 8 > 32 * kLnMaxVec) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15)
    return cudaErrorInvalidValue;  // read as 16-byte vectors
  const unsigned grid = (unsigned)((rows + 7) / 8);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* yv = static_cast<uint4*>(y);
  const int vpl = (channels / 8 + 31) / 32;
  auto launch = [&](auto kernel) {
    kernel<<<grid, 256, 0, s>>>(xv, yv, gamma, beta, rows, channels, eps);
  };
  if (dtype == kF16) {
    if (vpl <= 2) launch(layer_norm_kernel<kF16, 2>);
    else if (vpl <= 3) launch(layer_norm_kernel<kF16, 3>);
    else if (vpl <= 5) launch(layer_norm_kernel<kF16, 5>);
    else launch(layer_norm_kernel<kF16, kLnMaxVec>);
  } else {
    if (vpl <= 2) launch(layer_norm_kernel<kBf16, 2>);
    else if (vpl <= 3) launch(layer_norm_kernel<kBf16, 3>);
    else if (vpl <= 5) launch(layer_norm_kernel<kBf16, 5>);
    else launch(layer_norm_kernel<kBf16, kLnMaxVec>);
  }
  return cudaGetLastError();
}

cudaError_t geglu_launch(int dtype, const void* x, void* y, long long rows, int features,
                         cudaStream_t s, int interleaved) {
  if (features % 8 != 0 || (interleaved && features % 128 != 0)) return cudaErrorInvalidValue;
  const long long total = rows * (features / 8);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* yv = static_cast<uint4*>(y);
  if (dtype == kF16)
    geglu_kernel<kF16><<<grid_for(total, 256), 256, 0, s>>>(xv, yv, rows, features, interleaved);
  else
    geglu_kernel<kBf16><<<grid_for(total, 256), 256, 0, s>>>(xv, yv, rows, features, interleaved);
  return cudaGetLastError();
}

cudaError_t concat_channels_launch(const void* a, int ca, const void* b, int cb, void* y,
                                   long long pixels, cudaStream_t s) {
  if (ca % 8 != 0 || cb % 8 != 0) return cudaErrorInvalidValue;
  const long long total = pixels * ((ca + cb) / 8);
  concat_channels_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      static_cast<const uint4*>(a), ca / 8, static_cast<const uint4*>(b), cb / 8,
      static_cast<uint4*>(y), pixels);
  return cudaGetLastError();
}

cudaError_t resize_nearest_launch(const void* x, void* y, int batch, int in_h, int in_w,
                                  int out_h, int out_w, int channels, cudaStream_t s) {
  if (channels % 8 != 0) return cudaErrorInvalidValue;
  const long long total = (long long)batch * out_h * out_w * (channels / 8);
  resize_nearest_kernel<<<grid_for(total, 256), 256, 0, s>>>(
      static_cast<const uint4*>(x), static_cast<uint4*>(y), batch, in_h, in_w, out_h, out_w,
      channels / 8);
  return cudaGetLastError();
}

cudaError_t channel_update_launch(int dtype, const void* x, long long ld_x, void* y, int channels,
                                  long long pixels_per_image, int batch, const float* image_bias,
                                  long long bias_stride, const void* residual, cudaStream_t s) {
  if (channels % 8 != 0 || ld_x % 8 != 0 || ld_x < channels || pixels_per_image <= 0)
    return cudaErrorInvalidValue;
  const long long pixels = pixels_per_image * batch;
  const long long total = pixels * (channels / 8);
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* yv = static_cast<uint4*>(y);
  const uint4* rv = static_cast<const uint4*>(residual);
  if (dtype == kF16)
    channel_update_kernel<kF16><<<grid_for(total, 256), 256, 0, s>>>(
        xv, ld_x / 8, yv, channels / 8, pixels_per_image, pixels, image_bias, bias_stride, rv);
  else
    channel_update_kernel<kBf16><<<grid_for(total, 256), 256, 0, s>>>(
        xv, ld_x / 8, yv, channels / 8, pixels_per_image, pixels, image_bias, bias_stride, rv);
  return cudaGetLastError();
}

cudaError_t attention_heads_launch(int dtype, const void* q, long long ld_q, long long q_bs,
                                   const void* k, const void* v, long long ld_kv, long long kv_bs,
                                   void* out, long long ld_out, long long out_bs, int batch,
                                   int heads, int n_q, int n_kv, int head_dim, cudaStream_t s) {
  if (dtype == kF16)
    return attention_heads_typed<kF16>(q, ld_q, q_bs, k, v, ld_kv, kv_bs, out, ld_out, out_bs,
                                       batch, heads, n_q, n_kv, head_dim, s);
  return attention_heads_typed<kBf16>(q, ld_q, q_bs, k, v, ld_kv, kv_bs, out, ld_out, out_bs,
                                      batch, heads, n_q, n_kv, head_dim, s);
}

}  // namespace osor
