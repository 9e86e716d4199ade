// GroupNorm(32) (+ SiLU) kernels.
//
// Reference semantics (src/native/vae_encoder.rs:21-85, metal_ops.rs:23-116):
// per (batch, group): mean over C/32 channels x H x W, variance of the
// centered values (never E[x^2] - E[x]^2 of raw values), normalized
// (x - mean) / sqrt(var + eps), then the per-channel affine, then SiLU.
// Statistics are fp32 throughout.
//
// Two code paths:
//  * gn_nchw_fused_kernel: standalone NCHW op. A group is one contiguous run
//    of memory. Persistent co-resident CTAs each hold one chunk of a group in
//    shared memory, compute the chunk's exact two-pass (count, mean, M2),
//    publish it, wait (bounded) until every chunk of the group has published,
//    merge the partials with Chan's formula in a fixed order (so every CTA
//    derives bit-identical statistics), then normalize from shared memory and
//    store. HBM traffic is one read and one write per element.
//  * gn_nhwc_{stats,finalize,apply}: the layout used between convolutions.
//    Stats accumulate per-channel sums of (x - anchor) and (x - anchor)^2,
//    anchor = the group's first element (the reference Metal kernel's anchor),
//    so partials add across chunks; finalize turns them into per-(batch,
//    channel) (mean, rstd * gamma, beta); apply streams x once with 16-byte
//    vectors.
#include <atomic>
#include "common.cuh"
#include "groupnorm.h"

namespace osor {
namespace {

__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

template <typename T>
__device__ __forceinline__ float silu_t(float v) {
  if constexpr (sizeof(T) == 2) {
    return silu_16(v);
  } else {
    return silu_f(v);
  }
}

// Element access for the standalone kernel: float, bf16 or f16 storage.
template <typename T>
struct Scalar;
template <>
struct Scalar<float> {
  static constexpr int V = 4;  // elements per 16-byte vector
  __device__ static void unpack(const uint4& q, float (&f)[4]) {
    f[0] = __uint_as_float(q.x);
    f[1] = __uint_as_float(q.y);
    f[2] = __uint_as_float(q.z);
    f[3] = __uint_as_float(q.w);
  }
  __device__ static float to_f(float v) { return v; }
  __device__ static float from_f(float v) { return v; }
  __device__ static void load(const float* p, float (&f)[4]) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    f[0] = q.x;
    f[1] = q.y;
    f[2] = q.z;
    f[3] = q.w;
  }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};
template <int D>
struct Scalar16 {
  using T = typename Elem<D>::T;
  static constexpr int V = 8;
  __device__ static float to_f(T v) { return Elem<D>::to_f(v); }
  __device__ static T from_f(float v) { return Elem<D>::from_f(v); }
  __device__ static void load(const T* p, float (&f)[8]) {
    unpack8<D>(*reinterpret_cast<const uint4*>(p), f);
  }
  __device__ static void unpack(const uint4& q, float (&f)[8]) { unpack8<D>(q, f); }
  __device__ static void store(T* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = pack8<D>(f);
  }
};
template <>
struct Scalar<__nv_bfloat16> : Scalar16<kBf16> {};
template <>
struct Scalar<__half> : Scalar16<kF16> {};

// Block-wide sum over 256 threads; result broadcast to all threads.
__device__ __forceinline__ float block_sum_256(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < 8 ? scratch[lane] : 0.0f;
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return __shfl_sync(0xffffffffu, t, 0);
}

constexpr int kFusedThreads = 256;

struct FusedParams {
  long long count;        // elements per group
  long long chunk;        // elements per chunk (last chunk of a group may be shorter)
  int chunks_per_group;
  int groups_total;       // batch * groups
  int groups;             // groups per image
  int channels;
  long long spatial;      // H * W
  float eps;
  int silu;
  int use_bulk;           // chunks are 16-byte aligned and sized
  float* partials;        // [groups_total, chunks_per_group, 3]
  int* arrive;            // [groups_total]
  float* stats_out;       // optional [groups_total, 2] (mean, var)
  int arrive_target;      // arrivals a group waits for: chunks_per_group (more only in the
                          // wait-expiry test, so that the wait runs out)
  unsigned long long wait_ns;  // limit of the cross-CTA group wait
};

template <typename T>
__global__ void __launch_bounds__(kFusedThreads)
    gn_nchw_fused_kernel(const T* __restrict__ x, T* __restrict__ y,
                         const float* __restrict__ gamma, const float* __restrict__ beta,
                         const FusedParams p) {
  using S = Scalar<T>;
  constexpr int V = S::V;
  // Two chunk buffers: the bulk load of the next item runs while this item's
  // statistics, group wait and normalization proceed.
  extern __shared__ __align__(128) uint8_t smem_raw[];
  T* bufs[2] = {reinterpret_cast<T*>(smem_raw), reinterpret_cast<T*>(smem_raw) + p.chunk};
  __shared__ float red[8];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  uint32_t bar_phase[2] = {0, 0};
  const int cpg = p.channels / p.groups;
  const long long items = (long long)p.groups_total * p.chunks_per_group;
  // Issues the bulk load of `it` into buffer `b` (thread 0, aligned path).
  auto issue = [&](long long it, int b) {
    const int g = (int)(it / p.chunks_per_group);
    const long long beg = (it - (long long)g * p.chunks_per_group) * p.chunk;
    const uint32_t bytes = (uint32_t)min(p.chunk, p.count - beg) * (uint32_t)sizeof(T);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(x + (long long)g * p.count + beg);
    mbar_arrive_expect_tx(&bars[b], bytes);
    for (uint32_t off = 0; off < bytes; off += 65536u)
      bulk_load(reinterpret_cast<uint8_t*>(bufs[b]) + off, src + off, min(65536u, bytes - off),
                &bars[b]);
  };
  bool pending[2] = {false, false};  // thread 0: a bulk load into buffer b is in flight
  if (p.use_bulk && threadIdx.x == 0 && (long long)blockIdx.x < items) {
    issue(blockIdx.x, 0);
    pending[0] = true;
  }
  int cur = 0;
  for (long long item = blockIdx.x; item < items; item += gridDim.x, cur ^= 1) {
    T* buf = bufs[cur];
    const int group = (int)(item / p.chunks_per_group);
    const int ci = (int)(item - (long long)group * p.chunks_per_group);
    const long long begin = (long long)ci * p.chunk;
    const int n = (int)min(p.chunk, p.count - begin);
    const long long base = (long long)group * p.count + begin;
    // ---- the chunk in shared memory
    if (p.use_bulk) {
      // The other buffer was released by the previous item's final barrier.
      if (threadIdx.x == 0 && item + gridDim.x < items) {
        issue(item + gridDim.x, cur ^ 1);
        pending[cur ^ 1] = true;
      }
      if (mbar_wait(&bars[cur], bar_phase[cur], &abort_flag)) pending[cur] = false;
      bar_phase[cur] ^= 1;
      __syncthreads();
      if (abort_flag) break;
    } else {
      for (int i = threadIdx.x; i < n; i += kFusedThreads) buf[i] = x[base + i];
      __syncthreads();
    }
    const bool vec = p.use_bulk;  // 16-byte aligned chunk in shared memory
    // ---- exact two-pass statistics of the chunk
    float s = 0.0f;
    if (vec) {
      for (int i = threadIdx.x * V; i < n; i += kFusedThreads * V) {
        float f[V];
        S::load(buf + i, f);
#pragma unroll
        for (int j = 0; j < V; ++j) s += f[j];
      }
    } else {
      for (int i = threadIdx.x; i < n; i += kFusedThreads) s += S::to_f(buf[i]);
    }
    const float chunk_mean = block_sum_256(s, red) / (float)n;
    float m2 = 0.0f;
    if (vec) {
      for (int i = threadIdx.x * V; i < n; i += kFusedThreads * V) {
        float f[V];
        S::load(buf + i, f);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float d = f[j] - chunk_mean;
          m2 += d * d;
        }
      }
    } else {
      for (int i = threadIdx.x; i < n; i += kFusedThreads) {
        const float d = S::to_f(buf[i]) - chunk_mean;
        m2 += d * d;
      }
    }
    m2 = block_sum_256(m2, red);
    if (threadIdx.x == 0) {
      float* slot = p.partials + ((long long)group * p.chunks_per_group + ci) * 3;
      slot[0] = (float)n;
      slot[1] = chunk_mean;
      slot[2] = m2;
      __threadfence();
      atomicAdd(p.arrive + group, 1);
      // ---- wait (bounded) until every chunk of the group has published
      const volatile int* arrived = p.arrive + group;
      const uint64_t t0 = global_timer_ns();
      bool ok = true;
      while (*arrived < p.arrive_target) {
        if (global_timer_ns() - t0 > p.wait_ns) {
          record_device_error(kDevWaitTimeout);
          ok = false;
          break;
        }
      }
      __threadfence();
      if (!ok) abort_flag = 1;
    }
    __syncthreads();
    if (abort_flag) break;
    // ---- merge the group's chunk partials, all threads at once:
    //   mean = sum(n_c mean_c) / N,  M2 = sum(M2_c) + sum(n_c (mean_c - mean)^2).
    // Every CTA of the group reduces the same values in the same order, so all
    // derive identical statistics. Loads go to L2 (__ldcg): other CTAs wrote them.
    const float* part = p.partials + (long long)group * p.chunks_per_group * 3;
    float s1 = 0.0f;
    for (int c = threadIdx.x; c < p.chunks_per_group; c += kFusedThreads)
      s1 += __ldcg(part + 3 * c) * __ldcg(part + 3 * c + 1);
    const float mean = block_sum_256(s1, red) / (float)p.count;
    float s2 = 0.0f;
    for (int c = threadIdx.x; c < p.chunks_per_group; c += kFusedThreads) {
      const float d = __ldcg(part + 3 * c + 1) - mean;
      s2 += __ldcg(part + 3 * c + 2) + __ldcg(part + 3 * c) * d * d;
    }
    const float var = block_sum_256(s2, red) / (float)p.count;
    const float rstd = 1.0f / sqrtf(var + p.eps);
    if (threadIdx.x == 0 && ci == 0 && p.stats_out) {
      p.stats_out[2 * group] = mean;
      p.stats_out[2 * group + 1] = var;
    }
    // ---- normalize from shared memory, one channel run at a time
    const int g = group % p.groups;
    const long long first = (long long)g * cpg * p.spatial + begin;  // offset inside the image
    int c = (int)(first / p.spatial);
    long long seg_end = (long long)(c + 1) * p.spatial - first;  // chunk-relative
    int pos = 0;
    while (pos < n) {
      const int end = (int)min((long long)n, seg_end);
      const float a = __ldg(gamma + c) * rstd;
      const float bsh = __ldg(beta + c);
      if (vec && (pos % V) == 0 && (end % V) == 0) {
        for (int i = pos + threadIdx.x * V; i < end; i += kFusedThreads * V) {
          float f[V];
          S::load(buf + i, f);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            float v = (f[j] - mean) * a + bsh;
            if (p.silu) v = silu_t<T>(v);
            f[j] = v;
          }
          S::store(y + base + i, f);
        }
      } else {
        for (int i = pos + threadIdx.x; i < end; i += kFusedThreads) {
          float v = (S::to_f(buf[i]) - mean) * a + bsh;
          if (p.silu) v = silu_t<T>(v);
          y[base + i] = S::from_f(v);
        }
      }
      pos = end;
      ++c;
      seg_end += p.spatial;
    }
    __syncthreads();  // the buffer is reused by the next item
  }
  // After an abandoned wait, let loads still in flight land before exiting.
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      if (!pending[b]) continue;
      const uint32_t addr = smem_u32(&bars[b]);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(addr, bar_phase[b]) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
  }
}

// --------------------------------------------------------------- NHWC path
constexpr int kNhwcThreads = 256;

// grid (chunks, batch). Each thread owns one 8-channel vector column and
// strides over the chunk's pixels; per-channel anchored sums are reduced over
// the threads sharing the column and written as partials[b][chunk][c][2].
template <int D>
__global__ void __launch_bounds__(kNhwcThreads)
    gn_nhwc_stats_kernel(const uint16_t* __restrict__ x, float* __restrict__ partials,
                         int channels, long long pixels, long long pix_per_chunk, int groups) {
  using E = Elem<D>;
  extern __shared__ float sred[];  // [rows][vc][16]
  const int vc = channels / 8;
  const int rows = blockDim.x / vc;
  const int col = threadIdx.x % vc;
  const int r0 = threadIdx.x / vc;
  const int b = blockIdx.y;
  const int cpg = channels / groups;
  const long long p_begin = (long long)blockIdx.x * pix_per_chunk;
  const long long p_end = min(pixels, p_begin + pix_per_chunk);
  const typename E::T* img =
      reinterpret_cast<const typename E::T*>(x) + (long long)b * pixels * channels;
  float anchor[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = col * 8 + j;
    anchor[j] = E::to_f(img[(c / cpg) * cpg]);
  }
  float s1[8], s2[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s1[j] = s2[j] = 0.0f;
  if (r0 < rows) {
    const uint4* src = reinterpret_cast<const uint4*>(img) + col;
    long long pix = p_begin + r0;
    // Four independent 16-byte loads in flight per thread.
    for (; pix + 3 * rows < p_end; pix += 4 * rows) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldcs(src + (pix + u * rows) * vc);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float f[8];
        unpack8<D>(q[u], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = f[j] - anchor[j];
          s1[j] += d;
          s2[j] += d * d;
        }
      }
    }
    for (; pix < p_end; pix += rows) {
      float f[8];
      unpack8<D>(__ldcs(src + pix * vc), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[j] - anchor[j];
        s1[j] += d;
        s2[j] += d * d;
      }
    }
    float* mine = sred + ((long long)r0 * vc + col) * 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mine[j] = s1[j];
      mine[8 + j] = s2[j];
    }
  }
  __syncthreads();
  // Reduce over rows: one thread per (column, value).
  for (int idx = threadIdx.x; idx < vc * 16; idx += blockDim.x) {
    const int c = idx / 16, j = idx % 16;
    float acc = 0.0f;
    for (int r = 0; r < rows; ++r) acc += sred[((long long)r * vc + c) * 16 + j];
    const int ch = c * 8 + (j & 7);
    float* out = partials + (((long long)b * gridDim.x + blockIdx.x) * channels + ch) * 2;
    out[j >> 3] = acc;
  }
}

// grid (groups, batch), 256 threads: combine partials of one (b, group) and
// write per-channel (mean, rstd * gamma, beta) for the apply kernel.
template <int D>
__global__ void __launch_bounds__(256)
    gn_nhwc_finalize_kernel(const uint16_t* __restrict__ x, const float* __restrict__ partials,
                            int chunks, int channels, long long pixels, int groups,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            float eps, float* __restrict__ coef, float* __restrict__ stats_out) {
  using E = Elem<D>;
  __shared__ float red[8];
  const int g = blockIdx.x, b = blockIdx.y;
  const int cpg = channels / groups;
  float s1 = 0.0f, s2 = 0.0f;
  const int items = chunks * cpg;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int ch = i / cpg, c = g * cpg + (i % cpg);
    const float* pp = partials + (((long long)b * chunks + ch) * channels + c) * 2;
    s1 += pp[0];
    s2 += pp[1];
  }
  s1 = block_sum_256(s1, red);
  s2 = block_sum_256(s2, red);
  const double count = (double)cpg * (double)pixels;
  const typename E::T* img = reinterpret_cast<const typename E::T*>(x);
  const float anchor = E::to_f(img[(long long)b * pixels * channels + g * cpg]);
  const float dm = (float)(s1 / count);
  const float mean = anchor + dm;
  float var = (float)(s2 / count) - dm * dm;
  var = fmaxf(var, 0.0f);
  const float rstd = 1.0f / sqrtf(var + eps);
  if (gamma) {
    for (int i = threadIdx.x; i < cpg; i += blockDim.x) {
      const int c = g * cpg + i;
      float* o = coef + ((long long)b * channels + c) * 4;
      o[0] = mean;
      o[1] = rstd * gamma[c];
      o[2] = beta[c];
      o[3] = 0.0f;
    }
  }
  if (threadIdx.x == 0 && stats_out) {
    stats_out[((long long)b * groups + g) * 2] = mean;
    stats_out[((long long)b * groups + g) * 2 + 1] = var;
  }
}

// coef[b][c] = (mean, rstd * gamma[c], beta[c], 0) from `parts` given
// per-(image, group) (mean, var) sets, part_stats[p][b][g][2], each over the
// same number of elements (e.g. equal row bands of one image held by several
// GPUs). The merge of equal counts is the mean of the means and
// var = mean(var_p) + mean((mean_p - mean)^2).
__global__ void gn_coef_from_stats_kernel(const float* __restrict__ part_stats, int parts,
                                          int batch, int channels, int groups,
                                          const float* __restrict__ gamma,
                                          const float* __restrict__ beta, float eps,
                                          float* __restrict__ coef) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // b * channels + c
  if (i >= batch * channels) return;
  const int b = i / channels, c = i - b * channels;
  const int g = c / (channels / groups);
  const long long set = (long long)batch * groups * 2;
  const float* ps = part_stats + ((long long)b * groups + g) * 2;
  float mean = 0.0f;
  for (int p = 0; p < parts; ++p) mean += ps[p * set];
  mean /= (float)parts;
  float var = 0.0f;
  for (int p = 0; p < parts; ++p) {
    const float d = ps[p * set] - mean;
    var += fmaxf(ps[p * set + 1], 0.0f) + d * d;
  }
  var /= (float)parts;
  const float rstd = 1.0f / sqrtf(var + eps);
  float* o = coef + (long long)i * 4;
  o[0] = mean;
  o[1] = rstd * gamma[c];
  o[2] = beta[c];
  o[3] = 0.0f;
}

// grid (groups, batch): combine the per-tile (mean, M2) partials that the
// producing convolution's epilogue wrote (tile_part[b*tiles + t][group][2],
// every tile holding `tile_count` elements of the group) and write the
// per-channel apply coefficients. With equal counts the group mean is the mean
// of tile means and M2 = sum M2_t + tile_count * sum (mean_t - mean)^2.
__global__ void __launch_bounds__(256)
    gn_tiles_finalize_kernel(const float* __restrict__ tile_part, int tiles, float tile_count,
                             int channels, int groups, const float* __restrict__ gamma,
                             const float* __restrict__ beta, float eps, float* __restrict__ coef,
                             float* __restrict__ stats_out) {
  __shared__ float red[8];
  const int g = blockIdx.x, b = blockIdx.y;
  const int cpg = channels / groups;
  const float* part = tile_part + (long long)b * tiles * groups * 2;
  float s = 0.0f;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) s += part[((long long)t * groups + g) * 2];
  const float mean = block_sum_256(s, red) / (float)tiles;
  float q = 0.0f;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const float* pp = part + ((long long)t * groups + g) * 2;
    const float d = pp[0] - mean;
    q += pp[1] + tile_count * d * d;
  }
  q = block_sum_256(q, red);
  const float var = fmaxf(q / (tile_count * (float)tiles), 0.0f);
  const float rstd = 1.0f / sqrtf(var + eps);
  for (int i = threadIdx.x; i < cpg; i += blockDim.x) {
    const int c = g * cpg + i;
    float* o = coef + ((long long)b * channels + c) * 4;
    o[0] = mean;
    o[1] = rstd * gamma[c];
    o[2] = beta[c];
    o[3] = 0.0f;
  }
  if (threadIdx.x == 0 && stats_out) {
    stats_out[((long long)b * groups + g) * 2] = mean;
    stats_out[((long long)b * groups + g) * 2 + 1] = var;
  }
}

// Streams x once: y = silu?((x - mean) * (rstd * gamma) + beta). grid (n, batch);
// each thread owns one 8-channel column of one image (coefficients held in
// registers) and keeps four 16-byte loads in flight.
template <int D>
__global__ void __launch_bounds__(256)
    gn_nhwc_apply_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                         const float* __restrict__ coef, int channels, long long pixels,
                         int silu) {
  const int vc = channels / 8;
  const int rows = blockDim.x / vc;
  const int col = threadIdx.x % vc;
  const int r0 = threadIdx.x / vc;
  if (r0 >= rows) return;
  const int b = blockIdx.y;
  float ca[8], cb[8];
  const float4* cf = reinterpret_cast<const float4*>(coef + ((long long)b * channels + col * 8) * 4);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 c = __ldg(cf + j);
    gn_coef_prepare(c.x, c.y, c.z, silu != 0, ca[j], cb[j]);
  }
  const uint4* src = x + (long long)b * pixels * vc + col;
  uint4* dst = y + (long long)b * pixels * vc + col;
  const long long stride = (long long)gridDim.x * rows;
  long long pix = (long long)blockIdx.x * rows + r0;
  auto apply = [&](const uint4& q) {
    float f[8];
    unpack8<D>(q, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = gn_apply_prepared(f[j], ca[j], cb[j], silu != 0);
    return pack8<D>(f);
  };
  for (; pix + 3 * stride < pixels; pix += 4 * stride) {
    uint4 q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) q[u] = __ldcs(src + (pix + u * stride) * vc);
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[(pix + u * stride) * vc] = apply(q[u]);
  }
  for (; pix < pixels; pix += stride) dst[pix * vc] = apply(__ldcs(src + pix * vc));
}

// Wide rows (C / 8 > 256 vectors, e.g. the 2560-channel skip concatenations
// of the UNet): each of the 256 threads owns the columns threadIdx.x + 256 * i
// of every pixel of its chunk, so no cross-thread reduction is needed; the
// partials layout is the one gn_nhwc_finalize_kernel reads.
constexpr int kWideCols = 4;  // C <= 8192

template <int D>
__global__ void __launch_bounds__(256)
    gn_nhwc_stats_wide_kernel(const uint16_t* __restrict__ x, float* __restrict__ partials,
                              int channels, long long pixels, long long pix_per_chunk,
                              int groups) {
  using E = Elem<D>;
  const int vc = channels / 8;
  const int cpg = channels / groups;
  const int b = blockIdx.y;
  const long long p_begin = (long long)blockIdx.x * pix_per_chunk;
  const long long p_end = min(pixels, p_begin + pix_per_chunk);
  const typename E::T* img =
      reinterpret_cast<const typename E::T*>(x) + (long long)b * pixels * channels;
  for (int col = threadIdx.x; col < vc; col += blockDim.x) {
    float anchor[8], s1[8], s2[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = col * 8 + j;
      anchor[j] = E::to_f(img[(c / cpg) * cpg]);
      s1[j] = s2[j] = 0.0f;
    }
    const uint4* src = reinterpret_cast<const uint4*>(img) + col;
    for (long long pix = p_begin; pix < p_end; ++pix) {
      float f[8];
      unpack8<D>(__ldcs(src + pix * vc), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[j] - anchor[j];
        s1[j] += d;
        s2[j] += d * d;
      }
    }
    float* out = partials + (((long long)b * gridDim.x + blockIdx.x) * channels + col * 8) * 2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      out[2 * j] = s1[j];
      out[2 * j + 1] = s2[j];
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256)
    gn_nhwc_apply_wide_kernel(const uint4* __restrict__ x, uint4* __restrict__ y,
                              const float* __restrict__ coef, int channels, long long pixels,
                              int silu) {
  const int vc = channels / 8;
  const int b = blockIdx.y;
  float ca[kWideCols][8], cb[kWideCols][8];
#pragma unroll
  for (int i = 0; i < kWideCols; ++i) {
    const int col = threadIdx.x + 256 * i;
    if (col < vc) {
      const float4* cf =
          reinterpret_cast<const float4*>(coef + ((long long)b * channels + col * 8) * 4);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 c = __ldg(cf + j);
        gn_coef_prepare(c.x, c.y, c.z, silu != 0, ca[i][j], cb[i][j]);
      }
    }
  }
  const uint4* src = x + (long long)b * pixels * vc;
  uint4* dst = y + (long long)b * pixels * vc;
  for (long long pix = blockIdx.x; pix < pixels; pix += gridDim.x) {
#pragma unroll
    for (int i = 0; i < kWideCols; ++i) {
      const int col = threadIdx.x + 256 * i;
      if (col < vc) {
        float f[8];
        unpack8<D>(__ldcs(src + pix * vc + col), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = gn_apply_prepared(f[j], ca[i][j], cb[i][j], silu != 0);
        dst[pix * vc + col] = pack8<D>(f);
      }
    }
  }
}

int num_sms() {
  int dev = 0, c = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
  return c > 0 ? c : 148;
}

// Bulk-copy apply: each CTA streams chunks of one image (kApplyChunk bytes,
// 16-byte vectors) through a ring of kApplyStages shared-memory buffers: a bulk
// load lands the chunk, the 256 threads normalise it in place (each thread
// always the same 8 channels, since 256 is a multiple of C / 8), and a bulk
// store writes it back. kApplyStages - 1 loads stay in flight per CTA.

template <int D, int kApplyChunk, int kApplyStages>
__global__ void __launch_bounds__(256)
    gn_nhwc_apply_bulk_kernel(const uint8_t* __restrict__ x, uint8_t* __restrict__ y,
                              const float* __restrict__ coef, int channels,
                              int chunks_per_image, long long chunks_total, int silu) {
  extern __shared__ __align__(128) uint8_t abuf[];
  __shared__ __align__(8) uint64_t full[kApplyStages];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kApplyStages; ++s) mbar_init(&full[s], 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  const int vc = channels / 8;
  const int octet = threadIdx.x % vc;
  long long issued = 0, consumed = 0;  // thread 0: loads issued / iterations finished
  auto load = [&](long long it) {
    const long long chunk = blockIdx.x + it * gridDim.x;
    if (chunk >= chunks_total) return;
    issued = it + 1;
    const int b = (int)(it % kApplyStages);
    mbar_arrive_expect_tx(&full[b], kApplyChunk);
    bulk_load(abuf + b * kApplyChunk, x + chunk * kApplyChunk, kApplyChunk, &full[b]);
  };
  if (threadIdx.x == 0)
    for (int it = 0; it < kApplyStages - 1; ++it) load(it);
  int img = -1;
  float ca[8], cb[8];
  for (long long it = 0;; ++it) {
    const long long chunk = blockIdx.x + it * gridDim.x;
    if (chunk >= chunks_total) break;
    const int b = (int)(it % kApplyStages);
    const int ci = (int)(chunk / chunks_per_image);
    if (ci != img) {
      img = ci;
      const float4* cf =
          reinterpret_cast<const float4*>(coef + ((long long)img * channels + octet * 8) * 4);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 c = __ldg(cf + j);
        gn_coef_prepare(c.x, c.y, c.z, silu != 0, ca[j], cb[j]);
      }
    }
    const bool ok = mbar_wait(&full[b], (uint32_t)((it / kApplyStages) & 1), &abort_flag);
    __syncthreads();
    if (!ok || abort_flag) break;
    consumed = it + 1;
    uint4* v = reinterpret_cast<uint4*>(abuf + b * kApplyChunk);
#pragma unroll
    for (int k = 0; k < kApplyChunk / 16 / 256; ++k) {
      float f[8];
      unpack8<D>(v[threadIdx.x + k * 256], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = gn_apply_prepared(f[j], ca[j], cb[j], silu != 0);
      v[threadIdx.x + k * 256] = pack8<D>(f);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0) {
      bulk_store(y + chunk * kApplyChunk, abuf + b * kApplyChunk, kApplyChunk);
      bulk_commit_group();
      // The previous iteration's store has finished reading its buffer, which
      // now takes the load kApplyStages - 1 chunks ahead.
      bulk_wait_group_read<1>();
      load(it + kApplyStages - 1);
    }
  }
  if (threadIdx.x == 0) {
    bulk_wait_group<0>();
    // After an abort, let the loads still in flight (iterations consumed ..
    // issued - 1) land before the CTA leaves.
    for (long long it = consumed; it < issued; ++it) {
      const uint32_t addr = smem_u32(&full[it % kApplyStages]);
      const uint32_t parity = (uint32_t)((it / kApplyStages) & 1);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(addr, parity) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
  }
}

// Chunk bytes, ring stages and CTAs per SM of the bulk-copy apply (measured in
// the decode against 16 KB x 4 x 3, 16 KB x 6 x 2 and 8 KB x 8 x 3: the larger
// chunks with two CTAs per SM move 5.3 TB/s against 4.2 for the first).
constexpr int kApplyChunk = 32768;
constexpr int kApplyStages = 3;
constexpr int kApplyCtas = 2;

template <int D>
cudaError_t apply_launch(const void* x, void* y, const float* coef, int batch, int channels,
                         long long pixels, int silu, cudaStream_t stream) {
  const long long image_bytes = pixels * channels * 2;
  if (256 % (channels / 8) == 0 && image_bytes % kApplyChunk == 0 &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0) {
    const int smem = kApplyStages * kApplyChunk;
    static std::atomic<bool> configured[64];  // zero-initialized; atomic for concurrent callers
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(gn_nhwc_apply_bulk_kernel<D, kApplyChunk, kApplyStages>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
    const int per_image = (int)(image_bytes / kApplyChunk);
    const long long total = (long long)per_image * batch;
    long long grid = (long long)num_sms() * kApplyCtas;
    if (grid > total) grid = total;
    gn_nhwc_apply_bulk_kernel<D, kApplyChunk, kApplyStages><<<(unsigned)grid, 256, smem, stream>>>(
        static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), coef, channels, per_image, total,
        silu);
    return cudaGetLastError();
  }
  const int vc = channels / 8;
  if (vc > 256) {
    long long bx = ((long long)num_sms() * 8 + batch - 1) / batch;
    if (bx > pixels) bx = pixels;
    if (bx < 1) bx = 1;
    gn_nhwc_apply_wide_kernel<D><<<dim3((unsigned)bx, batch), 256, 0, stream>>>(
        static_cast<const uint4*>(x), static_cast<uint4*>(y), coef, channels, pixels, silu);
    return cudaGetLastError();
  }
  const int rows = 256 / vc;
  const int threads = rows * vc;
  long long bx = ((long long)num_sms() * 8 + batch - 1) / batch;
  const long long need = (pixels + rows - 1) / rows;
  if (bx > need) bx = need;
  if (bx < 1) bx = 1;
  gn_nhwc_apply_kernel<D><<<dim3((unsigned)bx, batch), threads, 0, stream>>>(
      static_cast<const uint4*>(x), static_cast<uint4*>(y), coef, channels, pixels, silu);
  return cudaGetLastError();
}

// Per-chunk partial sums of every channel: the row-sharing kernel for C / 8
// <= 256 vectors, the column-owning one above that.
template <int D>
void stats_launch(const uint16_t* xs, float* partials, const GnNhwcPlan& plan, int batch,
                  int channels, long long pixels, int groups, cudaStream_t stream) {
  const int vc = channels / 8;
  if (vc > 256) {
    gn_nhwc_stats_wide_kernel<D><<<dim3(plan.chunks, batch), 256, 0, stream>>>(
        xs, partials, channels, pixels, plan.pix_per_chunk, groups);
    return;
  }
  const int rows = plan.threads / vc;
  const size_t sred = (size_t)rows * vc * 16 * sizeof(float);
  gn_nhwc_stats_kernel<D><<<dim3(plan.chunks, batch), plan.threads, sred, stream>>>(
      xs, partials, channels, pixels, plan.pix_per_chunk, groups);
}

template <int D>
cudaError_t gn_nhwc_typed(const void* x, void* y, const float* gamma, const float* beta, int batch,
                          int channels, long long pixels, int groups, float eps, int silu,
                          void* workspace, float* stats_out, cudaStream_t stream) {
  const GnNhwcPlan plan = gn_nhwc_plan(batch, channels, pixels, groups);
  float* partials = static_cast<float*>(workspace);
  float* coef = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                         (plan.partial_bytes + 255) / 256 * 256);
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  stats_launch<D>(xs, partials, plan, batch, channels, pixels, groups, stream);
  gn_nhwc_finalize_kernel<D><<<dim3(groups, batch), 256, 0, stream>>>(
      xs, partials, plan.chunks, channels, pixels, groups, gamma, beta, eps, coef, stats_out);
  return apply_launch<D>(x, y, coef, batch, channels, pixels, silu, stream);
}

}  // namespace

// ---------------------------------------------------------------- NCHW, L2-resident
// Standalone NCHW GroupNorm(+SiLU) with one HBM read and one HBM write per
// element. A group (CPG channels x H x W, contiguous in NCHW) is split into P
// chunks of up to kL2Chunk bytes handled by co-resident CTAs. Per chunk, one
// read from HBM accumulates sums of (x - a) and (x - a)^2 with the anchor a =
// the chunk's first element (the reference Metal kernel's anchoring), turned
// into the chunk's (n, mean, M2) and published with a counter; once all P
// chunks of the group have published (Chan merge in chunk order), the chunk
// is read again, normalised and written. Each CTA normalises a chunk two
// iterations after publishing it, so the group wait overlaps later chunks'
// reads and a group may span consecutive waves of the persistent grid. The
// second read was meant to hit L2, but the three chunks per CTA that are in
// flight (about 110 MB over the grid) together with the output stream do not
// stay there: profiled, the L2 hit rate is 2% and DRAM reads are twice the
// tensor, so the kernel moves 1.5x the algorithmic bytes. Waits are bounded.
constexpr int kL2Lag = 2;  // iterations between a chunk's statistics and its store

// CTA shape: many small CTAs per SM keep loads in flight while others wait
// on their group counters (measured against 512 x 2, 256 x 4, 256 x 3,
// 128 x 6 and 128 x 8 threads with 16-64 KB chunks: 128 x 8 with 32 KB
// chunks is fastest).
constexpr int kL2Threads = 128;
constexpr int kL2CtasPerSm = 8;
constexpr int kL2Unroll = 4;  // 16-byte loads in flight per thread
constexpr long long kL2Chunk = 32 * 1024;  // bytes

struct L2Params {
  long long count;  // elements per group
  long long chunk;  // elements per chunk (16-byte multiple); the last is shorter
  int P;            // chunks per group
  int groups_total, groups, channels;
  long long spatial;
  float eps;
  int silu;
  float* partials;  // [groups_total * P][3] (n, mean, M2)
  int* arrive;      // [groups_total]
  float* stats_out;
};

template <int THREADS>
__device__ __forceinline__ float block_sum_t(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < THREADS / 32 ? scratch[lane] : 0.0f;
#pragma unroll
  for (int o = THREADS / 64; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return __shfl_sync(0xffffffffu, t, 0);
}

template <typename T>
__global__ void __launch_bounds__(kL2Threads, kL2CtasPerSm)
    gn_nchw_l2_kernel(const T* __restrict__ x, T* __restrict__ y, const float* __restrict__ gamma,
                      const float* __restrict__ beta, const L2Params p) {
  using S = Scalar<T>;
  constexpr int V = S::V;
  __shared__ float red[2][kL2Threads / 32];
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  const long long items = (long long)p.groups_total * p.P;
  const int cpg = p.channels / p.groups;
  constexpr long long kStep = (long long)kL2Threads * V;

  auto pass1 = [&](long long item) {
    const int g = (int)(item / p.P);
    const int c = (int)(item - (long long)g * p.P);
    const long long begin = (long long)c * p.chunk;
    const long long n = min(p.chunk, p.count - begin);
    const T* src = x + (long long)g * p.count + begin;
    const float a = S::to_f(src[0]);
    float s1 = 0.0f, s2 = 0.0f;
    for (long long i0 = (long long)threadIdx.x * V; i0 < n; i0 += kStep * kL2Unroll) {
      uint4 raw[kL2Unroll];
#pragma unroll
      for (int u = 0; u < kL2Unroll; ++u)
        if (i0 + u * kStep < n) raw[u] = __ldcg(reinterpret_cast<const uint4*>(src + i0 + u * kStep));
#pragma unroll
      for (int u = 0; u < kL2Unroll; ++u)
        if (i0 + u * kStep < n) {
          float f[V];
          S::unpack(raw[u], f);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            const float d = f[j] - a;
            s1 += d;
            s2 = fmaf(d, d, s2);
          }
        }
    }
    // Both sums in one block reduction.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) {
      red[0][warp] = s1;
      red[1][warp] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float t1 = 0.0f, t2 = 0.0f;
      for (int w = 0; w < kL2Threads / 32; ++w) {
        t1 += red[0][w];
        t2 += red[1][w];
      }
      const float nf = (float)n;
      const float d = t1 / nf;  // mean - a
      float* dst = p.partials + item * 3;
      dst[0] = nf;
      dst[1] = a + d;
      dst[2] = fmaxf(t2 - t1 * d, 0.0f);
      __threadfence();
      atomicAdd(&p.arrive[g], 1);
    }
  };

  auto pass2 = [&](long long item) {
    const int g = (int)(item / p.P);
    const int c = (int)(item - (long long)g * p.P);
    if (threadIdx.x == 0) {
      const volatile int* ar = p.arrive + g;
      const uint64_t t0 = global_timer_ns();
      while (*ar < p.P) {
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          record_device_error(kDevWaitTimeout);
          failed = 1;
          break;
        }
      }
      __threadfence();
    }
    __syncthreads();
    if (failed) return;
    const float* part = p.partials + (long long)g * p.P * 3;
    float sm = 0.0f;
    for (int k = threadIdx.x; k < p.P; k += kL2Threads)
      sm += __ldcg(part + k * 3) * __ldcg(part + k * 3 + 1);
    const float mean = block_sum_t<kL2Threads>(sm, red[0]) / (float)p.count;
    float sq = 0.0f;
    for (int k = threadIdx.x; k < p.P; k += kL2Threads) {
      const float nk = __ldcg(part + k * 3), mk = __ldcg(part + k * 3 + 1);
      const float d = mk - mean;
      sq += __ldcg(part + k * 3 + 2) + nk * d * d;
    }
    const float var = fmaxf(block_sum_t<kL2Threads>(sq, red[0]) / (float)p.count, 0.0f);
    const float rstd = rsqrtf(var + p.eps);
    if (threadIdx.x == 0 && c == 0 && p.stats_out) {
      p.stats_out[g * 2] = mean;
      p.stats_out[g * 2 + 1] = var;
    }
    const long long begin = (long long)c * p.chunk;
    const long long n = min(p.chunk, p.count - begin);
    const long long base = (long long)g * p.count + begin;
    const int gi = g % p.groups;
    for (long long i0 = (long long)threadIdx.x * V; i0 < n; i0 += kStep * kL2Unroll) {
      uint4 raw[kL2Unroll];
#pragma unroll
      for (int u = 0; u < kL2Unroll; ++u)
        if (i0 + u * kStep < n)
          raw[u] = __ldcg(reinterpret_cast<const uint4*>(x + base + i0 + u * kStep));
#pragma unroll
      for (int u = 0; u < kL2Unroll; ++u) {
        const long long i = i0 + u * kStep;
        if (i < n) {
          // V consecutive elements never straddle a channel (spatial % V == 0).
          const int ch = gi * cpg + (int)((unsigned)(begin + i) / (unsigned)p.spatial);
          const float sc = rstd * __ldg(gamma + ch);
          const float sh = __ldg(beta + ch);
          float f[V];
          S::unpack(raw[u], f);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            float v = (f[j] - mean) * sc + sh;
            if (p.silu) v = silu_t<T>(v);
            f[j] = v;
          }
          S::store(y + base + i, f);
        }
      }
    }
  };

  // Normalise the chunk published kL2Lag iterations earlier: by then its
  // group has normally completed, so the wait rarely spins.
  for (long long it = 0;; ++it) {
    const long long item = blockIdx.x + it * gridDim.x;
    const long long prev = item - (long long)kL2Lag * gridDim.x;
    if (item < items) pass1(item);
    if (prev >= 0 && prev < items) pass2(prev);
    if (prev >= items || failed) break;
  }
}

// ------------------------------------------------------------ host wrappers

GnL2Plan gn_nchw_l2_plan(int batch, int channels, long long spatial, int groups, int elem_bytes) {
  GnL2Plan plan{};
  const int vec = 16 / elem_bytes;
  plan.groups_total = batch * groups;
  // Offsets within a group use 32-bit arithmetic.
  plan.feasible = spatial % vec == 0 && channels % groups == 0 &&
                  (long long)(channels / groups) * spatial < (1LL << 31);
  plan.count = (long long)(channels / groups) * spatial;
  plan.grid = num_sms() * kL2CtasPerSm;
  long long chunk = kL2Chunk / elem_bytes;
  // Every group must fit in one wave of the grid (P <= grid); chunks hold
  // whole 16-byte vectors and at most kL2Chunk bytes.
  if ((plan.count + chunk - 1) / chunk > plan.grid) {
    chunk = (plan.count + plan.grid - 1) / plan.grid;
    chunk = (chunk + vec - 1) / vec * vec;
    if (chunk * elem_bytes > kL2Chunk) plan.feasible = false;
  }
  chunk = (chunk + vec - 1) / vec * vec;
  plan.chunk = chunk;
  plan.P = (int)((plan.count + chunk - 1) / chunk);
  plan.workspace_bytes = ((size_t)plan.groups_total * sizeof(int) + 255) / 256 * 256 +
                         (size_t)plan.groups_total * plan.P * 3 * sizeof(float);
  return plan;
}

template <typename T>
cudaError_t gn_nchw_l2_launch(const T* x, T* y, const float* gamma, const float* beta, int batch,
                              int channels, long long spatial, int groups, float eps, int silu,
                              void* workspace, float* stats_out, cudaStream_t stream) {
  const GnL2Plan plan = gn_nchw_l2_plan(batch, channels, spatial, groups, (int)sizeof(T));
  if (!plan.feasible) return cudaErrorInvalidValue;
  L2Params p;
  p.count = plan.count;
  p.chunk = plan.chunk;
  p.P = plan.P;
  p.groups_total = plan.groups_total;
  p.groups = groups;
  p.channels = channels;
  p.spatial = spatial;
  p.eps = eps;
  p.silu = silu;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.arrive = reinterpret_cast<int*>(ws);
  p.partials = reinterpret_cast<float*>(ws + ((size_t)plan.groups_total * sizeof(int) + 255) / 256 * 256);
  p.stats_out = stats_out;
  cudaError_t e = cudaMemsetAsync(p.arrive, 0, (size_t)plan.groups_total * sizeof(int), stream);
  if (e != cudaSuccess) return e;
  const long long items = (long long)plan.groups_total * plan.P;
  int grid = plan.grid;
  if (items < grid) grid = (int)items;
  void* args[] = {(void*)&x, (void*)&y, (void*)&gamma, (void*)&beta, (void*)&p};
  // A cooperative launch guarantees that all CTAs are resident, which the
  // cross-CTA group wait needs.
  return cudaLaunchCooperativeKernel(reinterpret_cast<void*>(gn_nchw_l2_kernel<T>), dim3(grid),
                                     dim3(kL2Threads), args, 0, stream);
}

template cudaError_t gn_nchw_l2_launch<float>(const float*, float*, const float*, const float*,
                                              int, int, long long, int, float, int, void*, float*,
                                              cudaStream_t);
template cudaError_t gn_nchw_l2_launch<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*,
                                                      const float*, const float*, int, int,
                                                      long long, int, float, int, void*, float*,
                                                      cudaStream_t);
template cudaError_t gn_nchw_l2_launch<__half>(const __half*, __half*, const float*, const float*,
                                               int, int, long long, int, float, int, void*, float*,
                                               cudaStream_t);

GnFusedPlan gn_fused_plan(int batch, int channels, long long spatial, int groups, int elem_bytes) {
  GnFusedPlan plan{};
  plan.groups_total = batch * groups;
  plan.count = (long long)(channels / groups) * spatial;
  plan.grid = num_sms() * kGnFusedCtasPerSm;
  // Chunk capacity: fits kGnFusedSmemBytes, multiple of 16 bytes.
  // Chunk capacity: half of the shared memory (two buffers).
  const long long cap = kGnFusedSmemBytes / 2 / elem_bytes;
  long long chunks = (plan.count + cap - 1) / cap;
  if (chunks < 1) chunks = 1;
  const long long align = 16 / elem_bytes;
  long long chunk = (plan.count + chunks - 1) / chunks;
  chunk = (chunk + align - 1) / align * align;
  chunks = (plan.count + chunk - 1) / chunk;
  plan.chunk = chunk;
  plan.chunks_per_group = (int)chunks;
  plan.feasible = plan.chunks_per_group <= plan.grid;
  plan.workspace_bytes = (size_t)plan.groups_total * plan.chunks_per_group * 3 * sizeof(float) +
                         ((size_t)plan.groups_total * sizeof(int) + 255) / 256 * 256;
  return plan;
}

template <typename T>
cudaError_t gn_fused_launch(const T* x, T* y, const float* gamma, const float* beta, int batch,
                            int channels, long long spatial, int groups, float eps, int silu,
                            void* workspace, float* stats_out, cudaStream_t stream,
                            int extra_arrivals, unsigned long long wait_ns) {
  const GnFusedPlan plan = gn_fused_plan(batch, channels, spatial, groups, (int)sizeof(T));
  if (!plan.feasible) return cudaErrorInvalidValue;
  if (extra_arrivals < 0) return cudaErrorInvalidValue;
  FusedParams p;
  p.arrive_target = plan.chunks_per_group + extra_arrivals;
  p.wait_ns = wait_ns ? wait_ns : kWaitLimitNs;
  p.count = plan.count;
  p.chunk = plan.chunk;
  p.chunks_per_group = plan.chunks_per_group;
  p.groups_total = plan.groups_total;
  p.groups = groups;
  p.channels = channels;
  p.spatial = spatial;
  p.eps = eps;
  p.silu = silu;
  p.use_bulk = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
               ((reinterpret_cast<uintptr_t>(y) & 15) == 0) &&
               ((plan.count * (long long)sizeof(T)) % 16 == 0) &&
               ((plan.chunk * (long long)sizeof(T)) % 16 == 0);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.arrive = reinterpret_cast<int*>(ws);
  const size_t arrive_bytes = ((size_t)plan.groups_total * sizeof(int) + 255) / 256 * 256;
  p.partials = reinterpret_cast<float*>(ws + arrive_bytes);
  p.stats_out = stats_out;
  cudaError_t e = cudaMemsetAsync(p.arrive, 0, (size_t)plan.groups_total * sizeof(int), stream);
  if (e != cudaSuccess) return e;
  static std::atomic<bool> configured[64];  // zero-initialized; atomic for concurrent callers
  int device = 0;
  cudaGetDevice(&device);
  if (device >= 0 && device < 64 && !configured[device]) {
    e = cudaFuncSetAttribute(gn_nchw_fused_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kGnFusedSmemBytes);
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  const int smem = (int)(2 * plan.chunk * sizeof(T));
  const long long items = (long long)plan.groups_total * plan.chunks_per_group;
  int grid = plan.grid;
  if (items < grid) grid = (int)items;
  void* args[] = {(void*)&x, (void*)&y, (void*)&gamma, (void*)&beta, (void*)&p};
  // A cooperative launch guarantees that all CTAs are resident, which the
  // cross-CTA group wait relies on.
  return cudaLaunchCooperativeKernel((const void*)gn_nchw_fused_kernel<T>, dim3(grid),
                                     dim3(kFusedThreads), args, (size_t)smem, stream);
}

template cudaError_t gn_fused_launch<float>(const float*, float*, const float*, const float*, int,
                                            int, long long, int, float, int, void*, float*,
                                            cudaStream_t, int, unsigned long long);
template cudaError_t gn_fused_launch<__nv_bfloat16>(const __nv_bfloat16*, __nv_bfloat16*,
                                                    const float*, const float*, int, int, long long,
                                                    int, float, int, void*, float*, cudaStream_t,
                                                    int, unsigned long long);
template cudaError_t gn_fused_launch<__half>(const __half*, __half*, const float*, const float*,
                                             int, int, long long, int, float, int, void*, float*,
                                             cudaStream_t, int, unsigned long long);

GnNhwcPlan gn_nhwc_plan(int batch, int channels, long long pixels, int groups) {
  GnNhwcPlan plan{};
  const int vc = channels / 8;
  plan.threads = (kNhwcThreads / vc) * vc;
  const int target_ctas = num_sms() * 4;
  long long chunks = (target_ctas + batch - 1) / batch;
  if (chunks > pixels) chunks = pixels;
  if (chunks < 1) chunks = 1;
  plan.pix_per_chunk = (pixels + chunks - 1) / chunks;
  plan.chunks = (int)((pixels + plan.pix_per_chunk - 1) / plan.pix_per_chunk);
  plan.partial_bytes = (size_t)batch * plan.chunks * channels * 2 * sizeof(float);
  plan.coef_bytes = (size_t)batch * channels * 4 * sizeof(float);
  plan.workspace_bytes = (plan.partial_bytes + 255) / 256 * 256 + plan.coef_bytes;
  plan.groups = groups;
  return plan;
}

cudaError_t gn_tiles_coef_launch(const float* tile_part, int batch, int channels,
                                 long long pixels, int groups, const float* gamma,
                                 const float* beta, float eps, float* coef, float* stats_out,
                                 cudaStream_t stream) {
  const int tiles = (int)(pixels / 128);
  const float tile_count = 128.0f * (float)(channels / groups);
  gn_tiles_finalize_kernel<<<dim3(groups, batch), 256, 0, stream>>>(
      tile_part, tiles, tile_count, channels, groups, gamma, beta, eps, coef, stats_out);
  return cudaGetLastError();
}

cudaError_t gn_nhwc_apply_tiles_launch(int dtype, const void* x, void* y, const float* gamma,
                                       const float* beta, int batch, int channels,
                                       long long pixels, int groups, float eps, int silu,
                                       const float* tile_part, float* coef, float* stats_out,
                                       cudaStream_t stream) {
  const int tiles = (int)(pixels / 128);
  const float tile_count = 128.0f * (float)(channels / groups);
  gn_tiles_finalize_kernel<<<dim3(groups, batch), 256, 0, stream>>>(
      tile_part, tiles, tile_count, channels, groups, gamma, beta, eps, coef, stats_out);
  if (dtype == kF16) return apply_launch<kF16>(x, y, coef, batch, channels, pixels, silu, stream);
  return apply_launch<kBf16>(x, y, coef, batch, channels, pixels, silu, stream);
}

cudaError_t gn_nhwc_stats_launch(int dtype, const void* x, int batch, int channels,
                                 long long pixels, int groups, void* workspace, float* mean_var,
                                 cudaStream_t stream) {
  const GnNhwcPlan plan = gn_nhwc_plan(batch, channels, pixels, groups);
  float* partials = static_cast<float*>(workspace);
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  if (dtype == kF16) {
    stats_launch<kF16>(xs, partials, plan, batch, channels, pixels, groups, stream);
    gn_nhwc_finalize_kernel<kF16><<<dim3(groups, batch), 256, 0, stream>>>(
        xs, partials, plan.chunks, channels, pixels, groups, nullptr, nullptr, 0.0f, nullptr,
        mean_var);
  } else {
    stats_launch<kBf16>(xs, partials, plan, batch, channels, pixels, groups, stream);
    gn_nhwc_finalize_kernel<kBf16><<<dim3(groups, batch), 256, 0, stream>>>(
        xs, partials, plan.chunks, channels, pixels, groups, nullptr, nullptr, 0.0f, nullptr,
        mean_var);
  }
  return cudaGetLastError();
}

cudaError_t gn_nhwc_apply_stats_launch(int dtype, const void* x, void* y, const float* gamma,
                                       const float* beta, const float* part_stats, int parts,
                                       int batch, int channels, long long pixels, int groups,
                                       float eps, int silu, float* coef, cudaStream_t stream) {
  const int total = batch * channels;
  gn_coef_from_stats_kernel<<<(total + 255) / 256, 256, 0, stream>>>(
      part_stats, parts, batch, channels, groups, gamma, beta, eps, coef);
  if (dtype == kF16) return apply_launch<kF16>(x, y, coef, batch, channels, pixels, silu, stream);
  return apply_launch<kBf16>(x, y, coef, batch, channels, pixels, silu, stream);
}

cudaError_t gn_coef_from_stats_launch(const float* part_stats, int parts, int batch, int channels,
                                      int groups, const float* gamma, const float* beta,
                                      float eps, float* coef, cudaStream_t stream) {
  const int total = batch * channels;
  gn_coef_from_stats_kernel<<<(total + 255) / 256, 256, 0, stream>>>(
      part_stats, parts, batch, channels, groups, gamma, beta, eps, coef);
  return cudaGetLastError();
}

cudaError_t gn_nhwc_launch(int dtype, const void* x, void* y, const float* gamma, const float* beta,
                           int batch, int channels, long long pixels, int groups, float eps,
                           int silu, void* workspace, float* stats_out, cudaStream_t stream) {
  if (dtype == kF16)
    return gn_nhwc_typed<kF16>(x, y, gamma, beta, batch, channels, pixels, groups, eps, silu,
                               workspace, stats_out, stream);
  return gn_nhwc_typed<kBf16>(x, y, gamma, beta, batch, channels, pixels, groups, eps, silu,
                              workspace, stats_out, stream);
}

}  // namespace osor
