// Row-band decode of one image over a group of GPUs (one rank per GPU), in
// C++ behind the C ABI: the whole-image decoder's kernels (tensor-core
// convolutions with GroupNorm statistics in their epilogues, the fused
// upsample phases, the CTA-pair attention, the fused conv_norm_out +
// conv_out) run on the rank's rows, with the exchanges of peer.cu between
// layers.
//
// Each activation is an *extended* band: rows 1..R are the rank's, rows 0
// and R + 1 halo rows. A 3x3 convolution runs over all R + 2 rows with zero
// padding, so its rows 1..R are exact once its input's halo rows hold the
// neighbours' rows (osor band halo exchange after each GroupNorm apply and
// before each upsample). GroupNorm statistics of rows 1..R come from the
// producing convolution's per-tile partials (tiles of 128 pixels lie within
// one row when the width is a multiple of 128) or a statistics pass, and the
// ranks' equal-count (mean, var) sets are all-gathered and merged before the
// apply. The mid-block attention gathers every rank's q|k|v rows (bulk
// gather) and attends the rank's queries to all keys. Nearest-2x upsampling
// of an extended band of R + 2 rows gives 2R + 4 rows whose rows 1..2R + 2
// are the upsampled band with exact halos, so no exchange follows it.
//
// Reference counterpart: VaeDecoder::forward (src/native/vae_decoder.rs
// :104-114) with the row-band geometry of the column convolution
// (src/native/conv.rs:96-108, src/native/columns.rs:335-362), which the
// reference runs one band after another on one device.
#include <algorithm>
#include <cstring>

#include "attn_fa.h"
#include "common.cuh"
#include "conv_out.h"
#include "conv_tc.h"
#include "groupnorm.h"
#include "ops.h"
#include "peer.h"
#include "profile.h"
#include "vae.h"

namespace osor {
namespace {

constexpr int kBandGroups = 32;
constexpr float kBandEps = 1e-6f;

size_t a256(size_t v) { return (v + 255) / 256 * 256; }

Status cuda_err(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::ok();
  return Status::err(OSOR_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Per-level shape of the band: R rows (without halos) of W pixels.
struct BandGeom {
  int ranks, rank, R, W;
};

// Workspace of one call.
struct BandBufs {
  size_t spare = 0;         // bytes before each extended tensor (one upsampled row)
  size_t act_bytes = 0;     // one activation buffer (spare included)
  size_t tstat_bytes = 0;
  uint8_t* act[4] = {};
  float* tstat[4] = {};
  float* coef = nullptr;    // [C][4]
  float* st_local = nullptr;  // [sets <= 4][32][2]
  float* st_all = nullptr;    // [ranks][sets][32][2]
  void* gn_ws = nullptr;
  size_t gn_bytes = 0;
  float* lat = nullptr;     // the band's latent rows, [4][rows][w] f32
  float* scores = nullptr;  // attention scratch when the pair kernel does not take the shape
  uint16_t* probs = nullptr;
  float* rowsum = nullptr;
  size_t total = 0;
};

bool pair_takes(int n_q, int n_kv, int c) {
  return c == 512 && n_q % 128 == 0 && n_kv % 512 == 0;
}

BandBufs band_layout(const Vae& m, int ranks, int h, int w) {
  BandBufs b;
  const int R = h / ranks;
  const int* ch = m.channels;
  const int rev[4] = {ch[3], ch[2], ch[1], ch[0]};
  size_t row_max = 0;   // widest row of any tensor (16-bit)
  size_t ext_max = 0;   // largest extended tensor, upsample outputs' extra rows included
  size_t px_max = 0;    // most pixels of any tensor a convolution produces
  for (int i = 0; i < 4; ++i) {
    const size_t wl = (size_t)w << i;
    const size_t rl = (size_t)R << i;
    const int cmax = std::max(rev[i], i ? rev[i - 1] : rev[0]);
    row_max = std::max(row_max, wl * cmax * 2);
    ext_max = std::max(ext_max, (rl + 4) * wl * cmax * 2);
    px_max = std::max(px_max, (rl + 4) * wl);
  }
  // q|k|v of the band's tokens and the keys' transposed values.
  const size_t tokens = (size_t)R * w;
  ext_max = std::max(ext_max, tokens * 3 * ch[3] * 2);
  ext_max = std::max(ext_max, tokens * ranks * ch[3] * 2);
  b.spare = a256(row_max);
  b.act_bytes = a256(b.spare + ext_max);
  b.tstat_bytes = a256((px_max / 128 + 1) * kBandGroups * 2 * sizeof(float));
  size_t g = 0;
  for (int i = 0; i < 4; ++i)
    for (int c : {ch[0], ch[1], ch[2], ch[3]})
      g = std::max(g, gn_nhwc_plan(1, c, (long long)((size_t)R << i) * ((size_t)w << i),
                                   kBandGroups)
                          .workspace_bytes);
  b.gn_bytes = a256(g);
  size_t off = 4 * b.act_bytes + 4 * b.tstat_bytes;
  const size_t coef_off = off;
  off += a256(512 * 4 * sizeof(float) * 2);
  const size_t st_off = off;
  off += a256(4 * kBandGroups * 2 * sizeof(float));
  const size_t sta_off = off;
  off += a256((size_t)ranks * 4 * kBandGroups * 2 * sizeof(float));
  const size_t gn_off = off;
  off += b.gn_bytes;
  const size_t lat_off = off;
  off += a256((size_t)4 * (R + 2) * w * sizeof(float));
  size_t scores_off = 0, probs_off = 0, rowsum_off = 0;
  const int n_q = R * w, n_kv = ranks * R * w;
  if (!pair_takes(n_q, n_kv, ch[3])) {
    scores_off = off;
    off += a256((size_t)n_q * (n_kv / 32 + 1) * 8 + (size_t)n_q * 4);
    probs_off = off;
    off += a256((size_t)n_q * n_kv * 2);
    rowsum_off = off;
    off += a256((size_t)n_q * 4);
  }
  b.total = off;
  // Offsets are stored as pointers relative to a null base; band_carve adds
  // the workspace address.
  b.coef = reinterpret_cast<float*>(coef_off);
  b.st_local = reinterpret_cast<float*>(st_off);
  b.st_all = reinterpret_cast<float*>(sta_off);
  b.gn_ws = reinterpret_cast<void*>(gn_off);
  b.lat = reinterpret_cast<float*>(lat_off);
  b.scores = reinterpret_cast<float*>(scores_off);
  b.probs = reinterpret_cast<uint16_t*>(probs_off);
  b.rowsum = reinterpret_cast<float*>(rowsum_off);
  return b;
}

BandBufs band_carve(BandBufs b, void* ws, bool attn_scratch) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  for (int i = 0; i < 4; ++i) {
    b.act[i] = base + i * b.act_bytes;
    b.tstat[i] = reinterpret_cast<float*>(base + 4 * b.act_bytes + i * b.tstat_bytes);
  }
  auto rel = [&](auto* p) { return reinterpret_cast<decltype(p)>(base + reinterpret_cast<uintptr_t>(p)); };
  b.coef = rel(b.coef);
  b.st_local = rel(b.st_local);
  b.st_all = rel(b.st_all);
  b.gn_ws = rel(static_cast<uint8_t*>(b.gn_ws));
  b.lat = rel(b.lat);
  if (attn_scratch) {
    b.scores = rel(b.scores);
    b.probs = rel(b.probs);
    b.rowsum = rel(b.rowsum);
  } else {
    b.scores = nullptr;
    b.probs = nullptr;
    b.rowsum = nullptr;
  }
  return b;
}

// One extended band tensor held in buffer `buf`: rows 0..R+1 at
// act[buf] + spare, `c` channels, and (when `stats`) the per-tile GroupNorm
// partials of its rows 1..R in tstat[buf] starting at tile `tile0`.
struct BT {
  int buf = 0;
  int c = 0;
  bool stats = false;
  long long tile0 = 0;
  // A fused upsample's partials are phase-major: four ranges of tiles, one
  // per output phase, `set_stride` tiles apart, each an equal share of the
  // band's pixels. Their statistics go out as four sets.
  int sets = 1;
  long long set_stride = 0;
};

struct Band {
  int dtype;
  const BandBufs& b;
  PeerGroup* g;
  cudaStream_t s;
  BandGeom geo;  // current level
  mutable int sets = 1;  // statistics sets per rank of the last band_stats
  uint8_t* ext(int buf) const { return b.act[buf] + b.spare; }
  long long row_bytes(int c) const { return (long long)geo.W * c * 2; }
  uint8_t* band_rows(const BT& t) const { return ext(t.buf) + row_bytes(t.c); }
  long long band_px() const { return (long long)geo.R * geo.W; }
};

// Band (mean, var) per group of t's rows 1..R into st_local (B.sets equal-
// count sets).
Status band_stats(const Band& B, const BT& t, const NormLayer& N) {
  const int low_w = t.sets == 4 ? B.geo.W / 2 : B.geo.W;
  if (t.stats && low_w % 128 == 0) {
    B.sets = t.sets;
    const long long px = B.band_px() / t.sets;
    OpScope scope("groupnorm", 0.0, 0.0, B.s, t.sets);
    for (int k = 0; k < t.sets; ++k) {
      const cudaError_t e = gn_tiles_coef_launch(
          B.b.tstat[t.buf] + (t.tile0 + k * t.set_stride) * kBandGroups * 2, 1, t.c, px,
          kBandGroups, N.gamma, N.beta, kBandEps, B.b.coef, B.b.st_local + k * kBandGroups * 2,
          B.s);
      if (e != cudaSuccess) return cuda_err(e, "band group-norm statistics");
    }
    return Status::ok();
  }
  B.sets = 1;
  const GnNhwcPlan plan = gn_nhwc_plan(1, t.c, B.band_px(), kBandGroups);
  if (plan.workspace_bytes > B.b.gn_bytes)
    return Status::err(OSOR_ERR_INVALID_INPUT, "band group-norm workspace too small");
  OpScope scope("groupnorm_stats", 0.0, 2.0 * B.band_px() * t.c, B.s, 2);
  return cuda_err(gn_nhwc_stats_launch(B.dtype, B.band_rows(t), 1, t.c, B.band_px(), kBandGroups,
                                       B.b.gn_ws, B.b.st_local, B.s),
                  "band group-norm statistics");
}

Status band_gather_stats(const Band& B) {
  const size_t bytes = (size_t)B.sets * kBandGroups * 2 * sizeof(float);
  OpScope scope("band_gather", 0.0, 2.0 * bytes * B.geo.ranks, B.s, 1);
  return cuda_err(band_gather_launch(B.g, B.b.st_local, bytes, B.b.st_all, B.s),
                  "band statistics gather");
}

Status band_halo(const Band& B, int buf, int c) {
  OpScope scope("band_halo", 0.0, 4.0 * B.row_bytes(c), B.s, 1);
  return cuda_err(band_halo_launch(B.g, B.ext(buf), B.row_bytes(c), B.geo.R, B.s), "band halo");
}

// The band's statistics (band_stats) to every rank and, with halo, t's raw
// edge rows to the neighbours (filling t's halo rows; zeros at the image's
// top and bottom) in one launch, so the ranks meet once per GroupNorm.
Status band_exchange(const Band& B, const BT& t, bool halo) {
  if (!halo) return band_gather_stats(B);
  const size_t bytes = (size_t)B.sets * kBandGroups * 2 * sizeof(float);
  OpScope scope("band_exchange", 0.0, 4.0 * B.row_bytes(t.c) + 2.0 * bytes * B.geo.ranks, B.s, 1);
  return cuda_err(band_halo_gather_launch(B.g, B.ext(t.buf), B.row_bytes(t.c), B.geo.R,
                                          B.b.st_local, bytes, B.b.st_all, B.s),
                  "band halo and statistics exchange");
}

// GroupNorm(+SiLU) of t into buffer yi (statistics merged over the ranks).
// With halo, t's raw halo rows come from the neighbours in the same exchange
// as the statistics and are normalised with the band (a row of the image is
// normalised alike on every rank), so y's halo rows are ready for the next
// convolution; the image's own top / bottom halo rows are zeroed in y (the
// convolution's zero padding). Without halo only rows 1..R are written.
Status band_gn(const Band& B, const BT& t, const NormLayer& N, bool silu, int yi, bool halo,
               BT* y) {
  Status st = band_stats(B, t, N);
  if (st.good()) st = band_exchange(B, t, halo);
  if (!st.good()) return st;
  const bool top = B.geo.rank == 0, bottom = B.geo.rank + 1 == B.geo.ranks;
  const int lo = halo && !top ? 0 : 1;
  const int hi = halo && !bottom ? B.geo.R + 2 : B.geo.R + 1;
  const long long rb = B.row_bytes(t.c);
  const long long px = (long long)(hi - lo) * B.geo.W;
  {
    OpScope scope("groupnorm", 0.0, 4.0 * px * t.c, B.s, 2);
    st = cuda_err(gn_nhwc_apply_stats_launch(B.dtype, B.ext(t.buf) + lo * rb, B.ext(yi) + lo * rb,
                                             N.gamma, N.beta, B.b.st_all, B.sets * B.geo.ranks,
                                             1, t.c, px, kBandGroups, kBandEps, silu ? 1 : 0,
                                             B.b.coef, B.s),
                  "band group-norm apply");
  }
  if (!st.good()) return st;
  if (halo && top)
    st = cuda_err(cudaMemsetAsync(B.ext(yi), 0, rb, B.s), "band top padding row");
  if (st.good() && halo && bottom)
    st = cuda_err(cudaMemsetAsync(B.ext(yi) + (long long)(B.geo.R + 1) * rb, 0, rb, B.s),
                  "band bottom padding row");
  y->buf = yi;
  y->c = t.c;
  y->stats = false;
  y->sets = 1;
  return st;
}

// Convolution of the extended tensor x (all R + 2 rows) into buffer oi's
// extended tensor, with the output's tile statistics.
Status band_conv(const Band& B, const ConvLayer& L, const BT& x, int oi, const uint8_t* residual,
                 BT* y) {
  bool produced = false;
  const int rows = B.geo.R + 2;
  Status st = run_conv(B.dtype, L, B.ext(x.buf), kLayoutNhwc16, 1, rows, B.geo.W, L.cin,
                       B.ext(oi), kLayoutNhwc16, L.cout, residual, L.cout, B.s, B.b.tstat[oi],
                       &produced);
  y->buf = oi;
  y->c = L.cout;
  y->stats = produced;
  y->tile0 = B.geo.W / 128;  // tiles of row 1 onwards (used when W % 128 == 0)
  return st;
}

// GroupNorm(+SiLU) of x followed by convolution L into buffer oi. When the
// convolution can normalise its own input, the ranks exchange the band
// statistics and x's raw halo rows (one rendezvous, as band_gn), the merged
// statistics become per-channel coefficients, and L reads x directly: rows
// of the extended tensor outside the image are its zero padding. Otherwise
// band_gn into buffer ti, then band_conv.
Status band_gn_conv(const Band& B, const BT& x, const NormLayer& N, bool silu, int ti,
                    const ConvLayer& L, int oi, const uint8_t* residual, BT* y) {
  const bool top = B.geo.rank == 0, bottom = B.geo.rank + 1 == B.geo.ranks;
  const int rows = B.geo.R + 2;
  InputNorm norm;
  norm.coef = B.b.coef;
  norm.silu = silu ? 1 : 0;
  norm.y0 = top ? 1 : 0;
  norm.y1 = bottom ? B.geo.R + 1 : rows;
  if (fused_input_norm_enabled() &&
      conv_takes_input_norm(B.dtype, L, B.ext(x.buf), 1, rows, B.geo.W, L.cin, B.ext(oi), L.cout,
                            residual, L.cout, norm)) {
    Status st = band_stats(B, x, N);
    if (st.good()) st = band_exchange(B, x, true);
    if (!st.good()) return st;
    {
      OpScope scope("groupnorm", 0.0, 0.0, B.s, 1);
      st = cuda_err(gn_coef_from_stats_launch(B.b.st_all, B.sets * B.geo.ranks, 1, x.c,
                                              kBandGroups, N.gamma, N.beta, kBandEps, B.b.coef,
                                              B.s),
                    "band group-norm coefficients");
    }
    if (!st.good()) return st;
    bool produced = false;
    st = run_conv(B.dtype, L, B.ext(x.buf), kLayoutNhwc16, 1, rows, B.geo.W, L.cin, B.ext(oi),
                  kLayoutNhwc16, L.cout, residual, L.cout, B.s, B.b.tstat[oi], &produced, &norm);
    y->buf = oi;
    y->c = L.cout;
    y->stats = produced;
    y->sets = 1;
    y->tile0 = B.geo.W / 128;
    return st;
  }
  BT t;
  Status st = band_gn(B, x, N, silu, ti, true, &t);
  if (st.good()) st = band_conv(B, L, t, oi, residual, y);
  return st;
}

Status band_resnet(const Band& B, const ResnetLayer& L, BT* x) {
  const int xi = x->buf;
  const int ti = (xi + 1) % 4, hi = (xi + 2) % 4, si = (xi + 3) % 4;
  const uint8_t* residual = B.ext(xi);
  Status st;
  BT sc, h, out;
  if (L.has_shortcut) {
    if (!(st = band_conv(B, L.shortcut, *x, si, nullptr, &sc)).good()) return st;
    residual = B.ext(si);
  }
  if (!(st = band_gn_conv(B, *x, L.n1, true, ti, L.c1, hi, nullptr, &h)).good()) return st;
  if (!(st = band_gn_conv(B, h, L.n2, true, ti, L.c2, xi, residual, &out)).good()) return st;
  *x = out;
  return Status::ok();
}

Status band_attention(const Band& B, const AttentionLayer& L, BT* x) {
  const int c = L.norm.c;
  const int xi = x->buf, ti = (xi + 1) % 4, qi = (xi + 2) % 4, oi = (xi + 3) % 4;
  const int n_q = (int)B.band_px();
  const int n_kv = n_q * B.geo.ranks;
  Status st;
  BT t;
  if (!(st = band_gn(B, *x, L.norm, false, ti, false, &t)).good()) return st;
  // q|k|v of the band's tokens: a 1x1 product over its R W pixels.
  uint8_t* qkv = B.b.act[qi];
  if (!(st = run_conv(B.dtype, L.qkv, B.band_rows(t), kLayoutNhwc16, 1, 1, n_q, c, qkv,
                      kLayoutNhwc16, 3 * c, nullptr, 0, B.s))
           .good())
    return st;
  const size_t part = (size_t)n_q * 3 * c * 2;
  if (const char* err = band_bulk_check(B.g, part)) return Status::err(OSOR_ERR_INVALID_INPUT, err);
  if (B.g->l.bulk_bytes != part)
    return Status::err(OSOR_ERR_INVALID_INPUT, "band bulk slots must equal the q|k|v part");
  {
    OpScope scope("band_bulk", 0.0, 2.0 * part * B.geo.ranks, B.s, 1);
    if (!(st = cuda_err(band_bulk_launch(B.g, qkv, part, B.s), "band q|k|v gather")).good())
      return st;
  }
  const uint16_t* all = reinterpret_cast<const uint16_t*>(bulk_slots(B.g));
  const uint16_t* q = all + (size_t)B.geo.rank * n_q * 3 * c;
  uint16_t* out = reinterpret_cast<uint16_t*>(B.b.act[oi]);
  st = attention_core(B.dtype, q, 3 * c, all + c, all + 2 * c, 3 * c, out, c, 1, n_q, n_kv, c,
                      B.b.scores, B.b.probs, B.b.rowsum, B.b.act[ti], B.s);
  if (!st.good()) return st;
  // Output projection + residual over the band rows, in place.
  bool produced = false;
  st = run_conv(B.dtype, L.out, out, kLayoutNhwc16, 1, 1, n_q, c, B.band_rows(*x), kLayoutNhwc16,
                c, B.band_rows(*x), c, B.s, B.b.tstat[xi], &produced);
  x->stats = produced;
  x->tile0 = 0;  // the product's tiles start at band row 1
  return st;
}

}  // namespace

Status vae_decode_band_sizes(const Vae& m, int ranks, int h, int w, BandSizes* out) {
  if (!m.has_decoder) return Status::err(OSOR_ERR_UNAVAILABLE, "model has no decoder");
  if (ranks < 1 || ranks > kMaxPeerRanks || h <= 0 || w <= 0 || h % ranks != 0)
    return Status::err(OSOR_ERR_INVALID_INPUT, "the latent height must divide into the ranks");
  if (h / ranks < 2) return Status::err(OSOR_ERR_INVALID_INPUT, "bands of at least two rows");
  const BandBufs b = band_layout(m, ranks, h, w);
  out->workspace = b.total;
  out->halo_row_bytes = b.spare;
  out->bulk_bytes = (size_t)(h / ranks) * w * 3 * m.channels[3] * 2;
  return Status::ok();
}

Status vae_decode_band(const Vae& m, PeerGroup* g, const float* latents, float* image_band, int h,
                       int w, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  BandSizes sizes;
  Status st = vae_decode_band_sizes(m, g->ranks, h, w, &sizes);
  if (!st.good()) return st;
  if (workspace_bytes < sizes.workspace)
    return Status::err(OSOR_ERR_INVALID_INPUT, "band decode workspace is too small");
  if (g->l.halo_bytes < sizes.halo_row_bytes)
    return Status::err(OSOR_ERR_INVALID_INPUT, "the peer group's halo slots are too small");
  if (g->l.gather_bytes < 4 * kBandGroups * 2 * sizeof(float))
    return Status::err(OSOR_ERR_INVALID_INPUT, "the peer group's gather slots are too small");
  for (int r = 0; r < g->ranks; ++r)
    if (!g->peers[r])
      return Status::err(OSOR_ERR_INVALID_INPUT, "a rank's arena is not mapped in the peer group");
  const int ranks = g->ranks, rank = g->rank;
  const int R = h / ranks, r0 = rank * R;
  const bool scratch = !pair_takes(R * w, ranks * R * w, m.channels[3]);
  const BandBufs b = band_carve(band_layout(m, ranks, h, w), workspace, scratch);
  Band B{m.dtype, b, g, s, BandGeom{ranks, rank, R, w}};
  const Decoder& d = m.dec;

  // post_quant_conv + conv_in (column GEMM) on latent rows [lo, hi): the
  // band with one row above and below where the image has them. The output
  // rows land at their extended positions; rows outside the image stay
  // unset (only the band rows and the exchanged halos are read later).
  const int lo = std::max(r0 - 1, 0), hi = std::min(r0 + R + 1, h);
  const int rows_in = hi - lo;
  if ((st = cuda_err(cudaMemcpy2DAsync(b.lat, (size_t)rows_in * w * sizeof(float),
                                       latents + (size_t)lo * w, (size_t)h * w * sizeof(float),
                                       (size_t)rows_in * w * sizeof(float), 4,
                                       cudaMemcpyDeviceToDevice, s),
                     "band latent rows"))
          .good() == false)
    return st;
  const ThinInputLayer& tin = d.conv_in_thin;
  const int c0 = tin.cols.cout;
  BT x;
  {
    const int ci = 1, xi = 0;
    {
      OpScope scope("thin_columns", 0.0, 4.0 * rows_in * w * tin.cin + 128.0 * rows_in * w, s, 1);
      st = cuda_err(thin_columns_launch(m.dtype, b.lat, b.act[ci], 1, tin.cin, rows_in, w, tin.k,
                                        tin.pad, tin.pre_w, tin.pre_b, s),
                    "band thin input columns");
    }
    if (!st.good()) return st;
    uint8_t* out = B.ext(xi) + (long long)(lo - (r0 - 1)) * w * c0 * 2;
    bool produced = false;
    st = run_conv(m.dtype, tin.cols, b.act[ci], kLayoutNhwc16, 1, rows_in, w, tin.cols.cin, out,
                  kLayoutNhwc16, c0, nullptr, 0, s, b.tstat[xi], &produced);
    if (!st.good()) return st;
    x.buf = xi;
    x.c = c0;
    x.stats = produced;
    x.tile0 = (long long)(r0 - lo) * (w / 128);  // band row 1 = latent row r0
  }
  // Mid block.
  if (!(st = band_resnet(B, d.mid.first, &x)).good()) return st;
  if (!(st = band_attention(B, d.mid.attn, &x)).good()) return st;
  if (!(st = band_resnet(B, d.mid.second, &x)).good()) return st;
  // Up blocks.
  for (const StageLayer& up : d.up) {
    for (const ResnetLayer& r : up.resnets)
      if (!(st = band_resnet(B, r, &x)).good()) return st;
    if (!up.resample) continue;
    // The upsampled band reads the neighbours' rows: exchange x's halos.
    if (!(st = band_halo(B, x.buf, x.c)).good()) return st;
    const ConvLayer& L = up.resample_conv;
    const int oi = (x.buf + 1) % 4;
    const long long hi_row = (long long)(2 * B.geo.W) * L.cout * 2;
    bool fused = false, phase_stats = false;
    if (L.w_up) {
      ConvTcArgs a;
      a.dtype = m.dtype;
      a.x = B.ext(x.buf);
      a.batch = 1;
      a.in_h = B.geo.R + 2;
      a.in_w = B.geo.W;
      a.cin = L.cin;
      a.pixel_stride = L.cin;
      a.ksize = 2;
      a.stride = 1;
      a.pad = 0;
      a.out_h = a.in_h;
      a.out_w = a.in_w;
      a.cout = L.cout;
      a.w = L.w_up;
      a.ldw = 4LL * L.cin;
      a.bias = L.bias;
      // 2R + 4 output rows starting one row before the new extended band.
      a.out = B.ext(oi) - hi_row;
      a.ld_out = L.cout;
      a.upsample = 1;
      const int cpg = L.cout % kBandGroups == 0 ? L.cout / kBandGroups : 0;
      if (B.geo.W % 128 == 0 && (cpg == 4 || cpg == 8 || cpg == 16)) {
        a.gn_part = b.tstat[oi];
        a.gn_cpg = cpg;
        phase_stats = true;
      }
      if (conv_tc_check(a) == nullptr) {
        const double px = 4.0 * a.in_h * a.in_w;
        OpScope scope("upconv_tc", 2.0 * px * L.cout * 4 * L.cin,
                      2.0 * a.in_h * a.in_w * L.cin + 2.0 * px * L.cout, s, 1);
        if (!(st = cuda_err(conv_tc_launch(a, s), "band upsample convolution")).good()) return st;
        fused = true;
      }
    }
    if (fused) {
      // Low-res rows 1..R of each phase's tiles are high-res band rows 1..2R.
      const long long low_tiles_per_row = B.geo.W / 128;
      x.stats = phase_stats;
      x.sets = 4;
      x.set_stride = (long long)(B.geo.R + 2) * low_tiles_per_row;
      x.tile0 = low_tiles_per_row;
      B.geo.R *= 2;
      B.geo.W *= 2;
      x.buf = oi;
      x.c = L.cout;
    } else {
      // Nearest 2x of all R + 2 rows, then the 3x3 convolution over the
      // upsampled extended band (rows 1 .. 2R + 2 of the upsampled rows).
      const int ui = oi;
      {
        OpScope scope("upsample", 0.0, 10.0 * (B.geo.R + 2) * B.geo.W * x.c, s, 1);
        st = cuda_err(upsample2x_nhwc_launch(B.ext(x.buf), B.ext(ui) - (long long)2 * B.geo.W * x.c * 2,
                                             1, B.geo.R + 2, B.geo.W, x.c, s),
                      "band upsample");
      }
      if (!st.good()) return st;
      B.geo.R *= 2;
      B.geo.W *= 2;
      BT u{ui, x.c, false, 0, 1, 0};
      BT y;
      if (!(st = band_conv(B, L, u, x.buf, nullptr, &y)).good()) return st;
      x = y;
    }
  }
  // conv_norm_out + SiLU + conv_out: coefficients from the merged band
  // statistics; the fused kernel reads the raw activation with the
  // neighbours' rows as its halo (exchanged first) and writes the image rows.
  const int Rf = B.geo.R, Wf = B.geo.W;
  if (!(st = band_stats(B, x, d.norm_out)).good()) return st;
  // Statistics and x's raw halo rows in one exchange (the fused kernel
  // normalises the halo rows itself).
  if (!(st = band_exchange(B, x, true)).good()) return st;
  const bool top = rank == 0, bottom = rank + 1 == ranks;
  const int first = top ? 1 : 0;
  const int height = Rf + 2 - (top ? 1 : 0) - (bottom ? 1 : 0);
  float* tmp = reinterpret_cast<float*>(b.act[(x.buf + 1) % 4]);
  GnConvOutArgs fa;
  fa.dtype = m.dtype;
  fa.x = B.ext(x.buf) + (long long)first * B.row_bytes(x.c);
  fa.batch = 1;
  fa.height = height;
  fa.width = Wf;
  fa.cin = d.norm_out.c;
  fa.coef = b.coef;
  fa.silu = 1;
  fa.wz = d.conv_out.w_z;
  fa.bias = d.conv_out.bias;
  fa.cout = d.conv_out.cout;
  fa.out = tmp;
  if (d.conv_out.w_z && gn_conv_out_check(fa) == nullptr) {
    const double px = (double)height * Wf;
    OpScope scope("gn_conv_out", 2.0 * px * fa.cout * 9 * fa.cin,
                  2.0 * px * fa.cin + 4.0 * px * fa.cout, s, 2);
    cudaError_t e = gn_coef_from_stats_launch(b.st_all, B.sets * ranks, 1, fa.cin, kBandGroups,
                                              d.norm_out.gamma, d.norm_out.beta, kBandEps, b.coef,
                                              s);
    if (e == cudaSuccess) e = gn_conv_out_launch(fa, s);
    if (!(st = cuda_err(e, "band group norm + conv_out")).good()) return st;
  } else {
    // GroupNorm apply over all rows with the merged coefficients' apply
    // (band rows, then the exchanged halos), then the thin convolution.
    const int ti = (x.buf + 2) % 4;
    {
      OpScope scope("groupnorm", 0.0, 4.0 * B.band_px() * x.c, s, 2);
      st = cuda_err(gn_nhwc_apply_stats_launch(m.dtype, B.band_rows(x),
                                               B.ext(ti) + B.row_bytes(x.c), d.norm_out.gamma,
                                               d.norm_out.beta, b.st_all, B.sets * ranks, 1, x.c,
                                               B.band_px(), kBandGroups, kBandEps, 1, b.coef, s),
                    "band group-norm apply");
    }
    if (!st.good()) return st;
    if (!(st = band_halo(B, ti, x.c)).good()) return st;
    // Convolve rows [first, first + height) of the normalized band, with the
    // image's own zero padding at its top and bottom.
    if (!(st = run_conv(m.dtype, d.conv_out, B.ext(ti) + (long long)first * B.row_bytes(x.c),
                        kLayoutNhwc16, 1, height, Wf, x.c, tmp, kLayoutNchwF32, 0, nullptr, 0,
                        s))
             .good())
      return st;
  }
  // Rows 1..Rf of the extended band are rows (1 - first) .. of tmp.
  const int skip = 1 - first;
  return cuda_err(cudaMemcpy2DAsync(image_band, (size_t)Rf * Wf * sizeof(float),
                                    tmp + (size_t)skip * Wf, (size_t)height * Wf * sizeof(float),
                                    (size_t)Rf * Wf * sizeof(float), (size_t)d.conv_out.cout,
                                    cudaMemcpyDeviceToDevice, s),
                  "band image rows");
}

}  // namespace osor
