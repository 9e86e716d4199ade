// CPU oracle for the SDXL VAE hot path (TEST INFRASTRUCTURE, never product code).
//
// A plain C++ restatement of the reference crate's CPU F32 arithmetic for the
// VAE convolutions, group normalization, nearest upsampling and mid-block
// attention. Only the tests, the smoke check and the CPU-baseline legs of the
// benchmark load this library; the CUDA library never links or calls it.
//
// Parity anchors (paths inside the reference project):
//   conv        src/native/columns.rs:42-75 (Im2Col::fill_row: channel-major
//               columns, zero padding from bounds checks), :297-368
//               (conv2d_checked: bands of output rows sized by the scratch
//               budget, one weight[Cout, Cin*k*k] x columns GEMM per image),
//               src/native/conv.rs:13 (32 Mi element budget), :116-145 (bias
//               added after the GEMM).
//   groupnorm   src/native/vae_encoder.rs:14-16 (32 groups, eps 1e-6, staged
//               sums of at most 256-element factors), :21-35 (group_sum),
//               :55-81 (mean, centered variance, divide by sqrt(var+eps),
//               then affine), :83-85 (SiLU after the norm).
//   upsample    src/native/vae_decoder.rs:18-35 (nearest 2x).
//   attention   src/native/attention.rs:8 (64 Mi score budget), :27-84 (query
//               rows sliced to the budget), src/native/vae_encoder.rs:320-327
//               (softmax over keys, F32).
// The reference's GEMM (the gemm 0.19 crate behind candle-core 0.11 on CPU) is
// not vendored; its exact F32 accumulation order cannot be reproduced, so
// parity against this oracle is tolerance based. The SGEMM below is a packed,
// register-blocked kernel of our own that accumulates each output in K order.
//
// Build: oracle/build.sh (g++ -O3 -fopenmp -shared; one AVX2 and one AVX-512 build,
// chosen at load time from the host CPU's flags).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <omp.h>

namespace {

#if defined(__AVX512F__)
constexpr int kVL = 16;   // floats per vector register
constexpr int kMR = 12;   // micro-tile rows
#else
constexpr int kVL = 8;
constexpr int kMR = 6;
#endif
constexpr int kNV = 2;            // vectors per micro-tile row
constexpr int kNR = kNV * kVL;    // micro-tile columns
constexpr int kKC = 256;          // K block
constexpr int kMC = 8 * kMR;      // M block (multiple of kMR)
constexpr int kNC = 24 * kNR;     // N block per task (multiple of kNR)

typedef float vecf __attribute__((vector_size(kVL * 4)));

static inline vecf loadv(const float* p) {
  vecf v;
  std::memcpy(&v, p, sizeof(v));
  return v;
}
static inline void storev(float* p, vecf v) { std::memcpy(p, &v, sizeof(v)); }

// ctile[MR x NR] = sum_k Ap[k][0..MR) * Bp[k][0..NR), accumulated in K order.
static inline void micro_kernel(int kc, const float* __restrict ap, const float* __restrict bp,
                                float* __restrict ctile) {
  vecf c[kMR][kNV];
  for (int i = 0; i < kMR; ++i)
    for (int j = 0; j < kNV; ++j) c[i][j] = vecf{};
  for (int k = 0; k < kc; ++k) {
    vecf b[kNV];
    for (int j = 0; j < kNV; ++j) b[j] = loadv(bp + k * kNR + j * kVL);
    const float* a = ap + k * kMR;
    for (int i = 0; i < kMR; ++i) {
      const vecf av = vecf{} + a[i];
      for (int j = 0; j < kNV; ++j) c[i][j] += av * b[j];
    }
  }
  for (int i = 0; i < kMR; ++i)
    for (int j = 0; j < kNV; ++j) storev(ctile + i * kNR + j * kVL, c[i][j]);
}

// Pack A[ic:ic+mc, pc:pc+kc] (row-major, leading dim lda) into MR-row panels.
static void pack_a(const float* a, long lda, int mc, int kc, float* ap) {
  for (int ir = 0; ir < mc; ir += kMR) {
    const int mr = std::min(kMR, mc - ir);
    for (int k = 0; k < kc; ++k) {
      for (int i = 0; i < kMR; ++i) {
        ap[k * kMR + i] = i < mr ? a[(long)(ir + i) * lda + k] : 0.0f;
      }
    }
    ap += (long)kc * kMR;
  }
}

// Pack B[pc:pc+kc, jc:jc+nc] (row-major, leading dim ldb) into NR-column panels.
static void pack_b(const float* b, long ldb, int kc, int nc, float* bp) {
  for (int jr = 0; jr < nc; jr += kNR) {
    const int nr = std::min(kNR, nc - jr);
    for (int k = 0; k < kc; ++k) {
      const float* src = b + (long)k * ldb + jr;
      float* dst = bp + (long)k * kNR;
      if (nr == kNR) {
        std::memcpy(dst, src, sizeof(float) * kNR);
      } else {
        for (int j = 0; j < kNR; ++j) dst[j] = j < nr ? src[j] : 0.0f;
      }
    }
    bp += (long)kc * kNR;
  }
}

// C[M,N] = A[M,K] * B[K,N] (+ C when accumulate), all row-major.
// Parallel over N blocks; A is packed once and shared read-only.
static void sgemm(int m, int n, int k, const float* a, long lda, const float* b, long ldb,
                  float* c, long ldc, bool accumulate, int threads) {
  if (m <= 0 || n <= 0) return;
  if (k <= 0) {
    if (!accumulate)
      for (int i = 0; i < m; ++i) std::fill(c + (long)i * ldc, c + (long)i * ldc + n, 0.0f);
    return;
  }
  const int m_pad = (m + kMR - 1) / kMR * kMR;
  const int k_blocks = (k + kKC - 1) / kKC;
  std::vector<float> a_packed((size_t)m_pad * k);
  // Packed layout: for each K block pc, for each M block ic: panels.
  std::vector<size_t> a_offset((size_t)k_blocks * ((m + kMC - 1) / kMC));
  {
    size_t off = 0, idx = 0;
    for (int pc = 0; pc < k; pc += kKC) {
      const int kc = std::min(kKC, k - pc);
      for (int ic = 0; ic < m; ic += kMC) {
        const int mc = std::min(kMC, m - ic);
        a_offset[idx++] = off;
        off += (size_t)((mc + kMR - 1) / kMR * kMR) * kc;
      }
    }
  }
  const int m_blocks = (m + kMC - 1) / kMC;
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int t = 0; t < k_blocks * m_blocks; ++t) {
    const int pb = t / m_blocks, ib = t % m_blocks;
    const int pc = pb * kKC, ic = ib * kMC;
    pack_a(a + (long)ic * lda + pc, lda, std::min(kMC, m - ic), std::min(kKC, k - pc),
           a_packed.data() + a_offset[t]);
  }
  const int n_blocks = (n + kNC - 1) / kNC;
#pragma omp parallel num_threads(threads)
  {
    std::vector<float> b_packed((size_t)kKC * kNC);
    alignas(64) float ctile[kMR * kNR];
#pragma omp for schedule(dynamic, 1)
    for (int jb = 0; jb < n_blocks; ++jb) {
      const int jc = jb * kNC;
      const int nc = std::min(kNC, n - jc);
      for (int pb = 0; pb < k_blocks; ++pb) {
        const int pc = pb * kKC;
        const int kc = std::min(kKC, k - pc);
        pack_b(b + (long)pc * ldb + jc, ldb, kc, nc, b_packed.data());
        const bool add = accumulate || pb > 0;
        for (int ib = 0; ib < m_blocks; ++ib) {
          const int ic = ib * kMC;
          const int mc = std::min(kMC, m - ic);
          const float* ap_block = a_packed.data() + a_offset[(size_t)pb * m_blocks + ib];
          for (int jr = 0; jr < nc; jr += kNR) {
            const int nr = std::min(kNR, nc - jr);
            const float* bp = b_packed.data() + (long)(jr / kNR) * kc * kNR;
            for (int ir = 0; ir < mc; ir += kMR) {
              const int mr = std::min(kMR, mc - ir);
              micro_kernel(kc, ap_block + (long)(ir / kMR) * kc * kMR, bp, ctile);
              for (int i = 0; i < mr; ++i) {
                float* crow = c + (long)(ic + ir + i) * ldc + jc + jr;
                const float* trow = ctile + i * kNR;
                if (add) {
                  for (int j = 0; j < nr; ++j) crow[j] += trow[j];
                } else {
                  for (int j = 0; j < nr; ++j) crow[j] = trow[j];
                }
              }
            }
          }
        }
      }
    }
  }
}

int g_threads = 0;
int threads_or_default() { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

// Sum [rows, remaining] in the reference's staged order: repeatedly split the
// remaining extent by its largest factor <= 256 and sum contiguous runs of
// that factor; a prime remainder above 256 is summed directly.
void staged_group_sums(const float* xs, long rows, long count, float* out, int threads) {
  const long chunk = 256;
#pragma omp parallel num_threads(threads)
  {
    std::vector<float> work;
#pragma omp for schedule(dynamic, 1)
    for (long r = 0; r < rows; ++r) {
      work.assign(xs + r * count, xs + (r + 1) * count);
      long remaining = count;
      bool direct = false;
      while (remaining > chunk) {
        long factor = 0;
        for (long f = chunk; f >= 2; --f) {
          if (remaining % f == 0) { factor = f; break; }
        }
        if (factor == 0) { direct = true; break; }
        const long next = remaining / factor;
        for (long i = 0; i < next; ++i) {
          float s = 0.0f;
          for (long j = 0; j < factor; ++j) s += work[i * factor + j];
          work[i] = s;
        }
        remaining = next;
      }
      (void)direct;
      float s = 0.0f;
      for (long i = 0; i < remaining; ++i) s += work[i];
      out[r] = s;
    }
  }
}

}  // namespace

extern "C" {

void oracle_set_threads(int threads) { g_threads = threads; }
int oracle_threads(void) { return threads_or_default(); }

// C[M,N] = A[M,K] * B[K,N] (+C if accumulate); row-major, contiguous.
void oracle_sgemm(int m, int n, int k, const float* a, const float* b, float* c, int accumulate) {
  sgemm(m, n, k, a, k, b, n, c, n, accumulate != 0, threads_or_default());
}

// Convolution of NCHW F32 input with weight [Cout, Cin, k, k]; bias (nullable)
// is added after the GEMM. Output rows are produced in bands whose column
// scratch holds at most max_scratch_elements (min one row), mirroring
// columns.rs:326-360. Returns 0 on success, 1 on invalid shapes.
int oracle_conv2d(const float* x, const float* w, const float* bias, float* y, int batch,
                  int cin, int height, int width, int cout, int kernel, int stride, int padding,
                  long long max_scratch_elements) {
  if (kernel <= 0 || stride <= 0 || batch <= 0 || cin <= 0 || cout <= 0) return 1;
  const int ph = height + 2 * padding, pw = width + 2 * padding;
  if (ph < kernel || pw < kernel) return 1;
  const int oh = (ph - kernel) / stride + 1;
  const int ow = (pw - kernel) / stride + 1;
  const long rows_k = (long)cin * kernel * kernel;
  const long row_elements = (long)batch * rows_k * ow;
  long band = max_scratch_elements / row_elements;
  band = std::max(1L, std::min(band, (long)oh));
  const int threads = threads_or_default();
  // Column and band buffers persist across calls so that repeated calls do
  // not pay first-touch page faults (calls are serialised by the caller).
  static std::vector<float> columns;
  static std::vector<float> out_band;
  for (int row_start = 0; row_start < oh; row_start += (int)band) {
    const int rows = (int)std::min<long>(band, oh - row_start);
    const long pixels = (long)rows * ow;
    columns.resize((size_t)batch * rows_k * pixels);
    // Fill column row index = b*rows_k + c*k*k + ky*k + kx over the band.
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long index = 0; index < (long)batch * rows_k; ++index) {
      const long b = index / rows_k, tap = index % rows_k;
      const int c = (int)(tap / (kernel * kernel));
      const int ky = (int)((tap / kernel) % kernel), kx = (int)(tap % kernel);
      const float* plane = x + ((long)b * cin + c) * height * width;
      float* row = columns.data() + index * pixels;
      std::fill(row, row + pixels, 0.0f);
      for (int oy = 0; oy < rows; ++oy) {
        const long iy = (long)(row_start + oy) * stride + ky - padding;
        if (iy < 0 || iy >= height) continue;
        const float* in_row = plane + iy * width;
        float* out_row = row + (long)oy * ow;
        for (int ox = 0; ox < ow; ++ox) {
          const long ix = (long)ox * stride + kx - padding;
          if (ix >= 0 && ix < width) out_row[ox] = in_row[ix];
        }
      }
    }
    out_band.resize((size_t)cout * pixels);
    for (int b = 0; b < batch; ++b) {
      sgemm(cout, (int)pixels, (int)rows_k, w, rows_k, columns.data() + (long)b * rows_k * pixels,
            pixels, out_band.data(), pixels, false, threads);
      // Scatter the band into NCHW output and add the bias after the GEMM.
#pragma omp parallel for num_threads(threads) schedule(static)
      for (int o = 0; o < cout; ++o) {
        const float bo = bias ? bias[o] : 0.0f;
        float* dst = y + (((long)b * cout + o) * oh + row_start) * ow;
        const float* src = out_band.data() + (long)o * pixels;
        for (long p = 0; p < pixels; ++p) dst[p] = src[p] + bo;
      }
    }
  }
  return 0;
}

// GroupNorm over NCHW F32 [B, C, HW] with 32 groups; optional SiLU. Stats are
// written to mean_out / var_out (each B*32, nullable) for parity checks.
int oracle_group_norm(const float* x, const float* gamma, const float* beta, float* y, int batch,
                      int channels, long long spatial, double eps, int groups, int silu,
                      float* mean_out, float* var_out) {
  if (groups <= 0 || channels % groups != 0 || batch <= 0 || spatial <= 0) return 1;
  const long count = (long)(channels / groups) * spatial;
  const long rows = (long)batch * groups;
  const int threads = threads_or_default();
  std::vector<float> sums(rows), mean(rows), var(rows);
  staged_group_sums(x, rows, count, sums.data(), threads);
  const float inv_count = (float)(1.0 / (double)count);
  for (long r = 0; r < rows; ++r) mean[r] = sums[r] * inv_count;
  // Centered variance with the same staged summation.
  {
    std::vector<float> buf;
    for (long r = 0; r < rows; ++r) {
      buf.resize(count);
      const float* xr = x + r * count;
      const float m = mean[r];
#pragma omp parallel for num_threads(threads) schedule(static)
      for (long i = 0; i < count; ++i) {
        const float d = xr[i] - m;
        buf[i] = d * d;
      }
      float s;
      staged_group_sums(buf.data(), 1, count, &s, 1);
      var[r] = s * inv_count;
    }
  }
  const long per_channel = spatial;
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long r = 0; r < rows; ++r) {
    const float m = mean[r];
    const float denom = std::sqrt((float)(var[r] + (float)eps));
    const long g = r % groups;
    const float* xr = x + r * count;
    float* yr = y + r * count;
    for (long i = 0; i < count; ++i) {
      const long c = g * (channels / groups) + i / per_channel;
      float v = ((xr[i] - m) / denom) * gamma[c] + beta[c];
      if (silu) v = v / (1.0f + std::exp(-v));
      yr[i] = v;
    }
  }
  if (mean_out) std::copy(mean.begin(), mean.end(), mean_out);
  if (var_out) std::copy(var.begin(), var.end(), var_out);
  return 0;
}

// Nearest 2x upsample of NCHW F32.
void oracle_upsample_2x(const float* x, float* y, int batch, int channels, int height, int width) {
  const long planes = (long)batch * channels;
#pragma omp parallel for num_threads(threads_or_default()) schedule(static)
  for (long p = 0; p < planes; ++p) {
    const float* src = x + p * height * width;
    float* dst = y + p * 4L * height * width;
    for (int yy = 0; yy < 2 * height; ++yy) {
      const float* srow = src + (long)(yy / 2) * width;
      float* drow = dst + (long)yy * 2 * width;
      for (int xx = 0; xx < 2 * width; ++xx) drow[xx] = srow[xx / 2];
    }
  }
}

// softmax(q @ kt) @ v per batch entry, with query rows sliced so that one
// score slice holds at most max_score_elements (attention.rs:55-83).
// q [B, N, D], kt [B, D, M], v [B, M, D] -> out [B, N, D]. Returns 1 when the
// budget cannot hold a single score row.
int oracle_attention(const float* q, const float* kt, const float* v, float* out, int batch,
                     int queries, int tokens, int dim, long long max_score_elements) {
  const long row_elements = (long)batch * tokens;
  if (row_elements <= 0 || row_elements > max_score_elements) return 1;
  const long rows = std::min<long>(max_score_elements / row_elements, queries);
  const int threads = threads_or_default();
  std::vector<float> scores;
  for (long start = 0; start < queries; start += rows) {
    const long n = std::min<long>(rows, queries - start);
    scores.resize((size_t)n * tokens);
    for (int b = 0; b < batch; ++b) {
      const float* qb = q + ((long)b * queries + start) * dim;
      sgemm((int)n, tokens, dim, qb, dim, kt + (long)b * dim * tokens, tokens, scores.data(),
            tokens, false, threads);
#pragma omp parallel for num_threads(threads) schedule(static)
      for (long i = 0; i < n; ++i) {
        float* row = scores.data() + i * tokens;
        float mx = row[0];
        for (int j = 1; j < tokens; ++j) mx = std::max(mx, row[j]);
        float s = 0.0f;
        for (int j = 0; j < tokens; ++j) {
          row[j] = std::exp(row[j] - mx);
          s += row[j];
        }
        for (int j = 0; j < tokens; ++j) row[j] = row[j] / s;
      }
      sgemm((int)n, dim, tokens, scores.data(), tokens, v + (long)b * tokens * dim, dim,
            out + ((long)b * queries + start) * dim, dim, false, threads);
    }
  }
  return 0;
}

// Seeded standard-normal noise, version 1 of the reference's stored-seed
// contract (src/noise.rs:1-99): stream `stream` is a xoshiro256** generator
// whose four state words are the first four SplitMix64 outputs from
// seed + stream * 0x9E3779B97F4A7C15 (noise.rs:42-66); values are Box-Muller
// pairs in f64 - u1 = 1 - (top 53 bits of one output) * 2^-53, u2 from the
// next output, r = sqrt(-2 ln u1), angle = 2 pi u2, (r cos, r sin) - rounded to
// f32 (noise.rs:80-99). The published generators (SplitMix64, xoshiro256**)
// are restated here from their definitions.
void oracle_seeded_noise(uint64_t seed, uint64_t stream, long long count, float* out) {
  const uint64_t kStride = 0x9E3779B97F4A7C15ull;
  uint64_t mixer = seed + stream * kStride;
  uint64_t st[4];
  for (int i = 0; i < 4; ++i) {
    mixer += kStride;
    uint64_t z = mixer;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    st[i] = z ^ (z >> 31);
  }
  auto rotl = [](uint64_t v, int k) { return (v << k) | (v >> (64 - k)); };
  auto next = [&]() {
    const uint64_t result = rotl(st[1] * 5, 7) * 9;
    const uint64_t t = st[1] << 17;
    st[2] ^= st[0];
    st[3] ^= st[1];
    st[1] ^= st[2];
    st[0] ^= st[3];
    st[2] ^= t;
    st[3] = rotl(st[3], 45);
    return result;
  };
  auto unit = [&]() { return (double)(next() >> 11) * (1.0 / (double)(1ull << 53)); };
  const double kPi = 3.14159265358979323846;
  for (long long i = 0; i < count; i += 2) {
    const double u1 = 1.0 - unit();
    const double u2 = unit();
    const double radius = std::sqrt(-2.0 * std::log(u1));
    const double angle = 2.0 * kPi * u2;
    out[i] = (float)(radius * std::cos(angle));
    if (i + 1 < count) out[i + 1] = (float)(radius * std::sin(angle));
  }
}

}  // extern "C"
