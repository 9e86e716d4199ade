// SDXL inpainting UNet runtime behind osor_unet_create / osor_unet_denoise:
// Unet::new and Unet::forward (src/native.rs:127-379) with the resnet,
// transformer and block structure of src/native/{resnet,spatial,transformer,
// cross_blocks,unet_blocks}.rs. Activations are 16-bit NHWC; a transformer's
// tokens are the pixels of the NHWC image. The launch sequence and arguments
// are those of the Python host (osor_b200.unet.CudaUnetOps), so both give the
// same bits.
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "groupnorm.h"
#include "ops.h"
#include "profile.h"
#include "unet.h"
#include "unet_model.h"

namespace osor {

namespace {

constexpr int kGroups = 32;
constexpr float kResnetEps = 1e-5f;
constexpr float kTransformerGnEps = 1e-6f;
constexpr float kLayerNormEps = 1e-5f;
constexpr int kRowsLinearFloats = 12288;

Status cuda_err(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::ok();
  return Status::err(OSOR_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define OSOR_TRY(expr)                      \
  do {                                      \
    Status try_status_ = (expr);            \
    if (!try_status_.good()) return try_status_; \
  } while (0)

struct Product {
  int cin = 0, cout = 0, cpad = 0, k = 1;
  uint16_t* w = nullptr;  // [cpad][k*k*cin], rows >= cout zero
  float* bias = nullptr;  // [cpad] or null
  // GEGLU input projection with its rows in run_geglu_product's interleaved
  // order (value rows and their gate rows per 128 features).
  bool geglu = false;
};

struct Norm {
  int c = 0;
  float* gamma = nullptr;
  float* beta = nullptr;
};

struct ResnetL {
  Norm n1, n2;
  Product c1, c2, sc;
  bool has_sc = false;
  long long tb_off = 0;  // offset of this resnet's time bias in the stacked rows
};

struct TBlock {
  Norm ln1, ln2, ln3;
  Product qkv, out1, q2, out2, ff1, ff2;
  uint16_t* k2 = nullptr;  // prompt keys [tokens][C]
  uint16_t* v2 = nullptr;  // prompt values [tokens][C]
};

struct TransformerL {
  Norm norm;
  Product proj_in, proj_out;
  std::vector<TBlock> blocks;
  int heads = 1;
};

struct Level {
  std::vector<ResnetL> resnets;
  std::vector<TransformerL> attns;  // empty for a plain block
  bool resample = false;
  Product resample_conv;
};

int padded(int cout, int cin) {
  if (cin % 64 == 0 && cout % 128 != 0 && cout % 8 == 0) return (cout + 127) / 128 * 128;
  return cout;
}

}  // namespace

struct Unet {
  int device = 0;
  int dtype = kBf16;
  osor_unet_config cfg{};
  int tokens = 0;
  int base = 0, time_dim = 0, feat_w = 0;
  Product conv_in, conv_out;
  // conv_in as a 1x1 product over the 128-column matrix of its 81 taps x
  // channels (thin_columns_launch's order; 384 rows at SDXL width, rows past
  // 320 zero).
  Product conv_in_cols;
  Norm norm_out;
  uint16_t* emb_w1 = nullptr;
  float* emb_b1 = nullptr;
  uint16_t* emb_w2 = nullptr;
  float* emb_b2a = nullptr;
  float* emb_b2b = nullptr;
  uint16_t* temb_w = nullptr;
  float* temb_b = nullptr;
  int temb_rows = 0;
  float* pooled = nullptr;
  Level down[3], up[3];
  ResnetL mid0, mid1;
  TransformerL mid_attn;
  cudaMemPool_t pool = nullptr;
  std::vector<void*> allocations;
  ~Unet() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    for (void* p : allocations) cudaFree(p);
    if (pool) cudaMemPoolDestroy(pool);
    cudaSetDevice(prev);
  }
};

namespace {

// ------------------------------------------------------------------ loading
class Loader {
 public:
  Loader(const osor_tensor* t, size_t n, Unet* m) : m_(m) {
    for (size_t i = 0; i < n; ++i)
      if (t[i].name) by_name_[t[i].name] = &t[i];
  }

  // Host data of `name` checked against `shape` (trailing 1-dims not allowed).
  Status get(const std::string& name, std::initializer_list<int64_t> shape, const float** out) {
    auto it = by_name_.find(name);
    const osor_tensor* t = it == by_name_.end() ? nullptr : it->second;
    bool ok = t && t->data && t->ndim == (int)shape.size();
    int i = 0;
    for (int64_t d : shape) {
      if (!ok) break;
      ok = t->shape[i++] == d;
    }
    if (!ok)
      return Status::err(OSOR_ERR_INVALID_ARTIFACT,
                         "native model tensor missing or incompatible: " + name);
    *out = t->data;
    return Status::ok();
  }

  void own(void* p) { m_->allocations.push_back(p); }

  template <typename T>
  Status upload(const T* host, size_t n, T** dev) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, n * sizeof(T));
    if (e != cudaSuccess) return cuda_err(e, "weight allocation");
    m_->allocations.push_back(p);
    e = cudaMemcpy(p, host, n * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_err(e, "weight upload");
    *dev = static_cast<T*>(p);
    return Status::ok();
  }

  // 16-bit [rows][k*k*cin] (ky, kx, ci) of f32 [cout][cin][k][k]; rows >= cout zero.
  Status pack(const float* w, int cout, int cin, int k, int rows, uint16_t** dev) {
    std::vector<uint16_t> bits((size_t)rows * k * k * cin, 0);
    const int rc = osor_pack_conv_weight(w, bits.data(), cout, cin, k,
                                         m_->dtype == kF16 ? OSOR_DTYPE_F16 : OSOR_DTYPE_BF16);
    if (rc != OSOR_OK) return Status::err(rc, "weight packing");
    return upload(bits.data(), bits.size(), dev);
  }

  Status product_from(const float* w, const float* bias, int cout, int cin, int k, bool pad,
                      Product* p) {
    p->cin = cin;
    p->cout = cout;
    p->k = k;
    p->cpad = pad ? padded(cout, cin) : cout;
    OSOR_TRY(pack(w, cout, cin, k, p->cpad, &p->w));
    if (bias) {
      std::vector<float> b(p->cpad, 0.0f);
      std::memcpy(b.data(), bias, sizeof(float) * cout);
      OSOR_TRY(upload(b.data(), b.size(), &p->bias));
    }
    return Status::ok();
  }

  Status conv(const std::string& name, int cin, int cout, int k, Product* p, bool pad = true) {
    const float *w, *b;
    OSOR_TRY(get(name + ".weight", {cout, cin, k, k}, &w));
    OSOR_TRY(get(name + ".bias", {cout}, &b));
    return product_from(w, b, cout, cin, k, pad, p);
  }

  Status linear(const std::string& name, int cin, int cout, bool bias, Product* p) {
    const float *w, *b = nullptr;
    OSOR_TRY(get(name + ".weight", {cout, cin}, &w));
    if (bias) OSOR_TRY(get(name + ".bias", {cout}, &b));
    return product_from(w, b, cout, cin, 1, true, p);
  }

  Status norm(const std::string& name, int c, Norm* n) {
    const float *g, *b;
    OSOR_TRY(get(name + ".weight", {c}, &g));
    OSOR_TRY(get(name + ".bias", {c}, &b));
    n->c = c;
    OSOR_TRY(upload(g, c, &n->gamma));
    return upload(b, c, &n->beta);
  }

 private:
  Unet* m_;
  std::unordered_map<std::string, const osor_tensor*> by_name_;
};

// ------------------------------------------------------------------ forward
class Buf {
 public:
  Buf() = default;
  Buf(const Buf&) = delete;
  Buf& operator=(const Buf&) = delete;
  Buf(Buf&& o) noexcept : p_(o.p_), s_(o.s_) { o.p_ = nullptr; }
  Buf& operator=(Buf&& o) noexcept {
    release();
    p_ = o.p_;
    s_ = o.s_;
    o.p_ = nullptr;
    return *this;
  }
  ~Buf() { release(); }
  void* get() const { return p_; }
  cudaError_t alloc(size_t bytes, cudaMemPool_t pool, cudaStream_t s) {
    release();
    s_ = s;
    return cudaMallocFromPoolAsync(&p_, bytes, pool, s);
  }

 private:
  void release() {
    if (p_) cudaFreeAsync(p_, s_);
    p_ = nullptr;
  }
  void* p_ = nullptr;
  cudaStream_t s_ = nullptr;
};

// NHWC 16-bit tensor [b][h][w][c] (or an f32 buffer when used for rows).
struct Act {
  Buf buf;
  int b = 0, h = 0, w = 0, c = 0;
  uint16_t* p() const { return static_cast<uint16_t*>(buf.get()); }
  long long pixels() const { return (long long)b * h * w; }
};

class Run {
 public:
  Run(const Unet& m, cudaStream_t s, const volatile int* cancel)
      : m_(m), s_(s), cancel_(cancel) {}

  Status act(int b, int h, int w, int c, Act* a) {
    a->b = b;
    a->h = h;
    a->w = w;
    a->c = c;
    return cuda_err(a->buf.alloc((size_t)b * h * w * c * 2, m_.pool, s_), "activation allocation");
  }
  Status raw(size_t bytes, Buf* buf) {
    return cuda_err(buf->alloc(bytes, m_.pool, s_), "scratch allocation");
  }
  Status checkpoint() const {
    if (cancel_ && *cancel_) return Status::err(OSOR_ERR_CANCELLED, "inference was cancelled");
    return Status::ok();
  }

  // Product over pixels: [B, Ho, Wo, Cpad] (bias, and the residual when it
  // fuses) in `y`.
  Status raw_product(const Act& x, const Product& p, int stride, const uint16_t* residual,
                     Act* y) {
    const int pad = p.k / 2;
    const int oh = (x.h + 2 * pad - p.k) / stride + 1;
    const int ow = (x.w + 2 * pad - p.k) / stride + 1;
    OSOR_TRY(act(x.b, oh, ow, p.cpad, y));
    ConvLayer L;
    L.cin = p.cin;
    L.cout = p.cpad;
    L.k = p.k;
    L.stride = stride;
    L.pad = pad;
    L.pad_end = pad;
    L.w = p.w;
    L.bias = p.bias;
    return run_conv(m_.dtype, L, x.p(), kLayoutNhwc16, x.b, x.h, x.w, x.c, y->p(),
                    kLayoutNhwc16, p.cpad, residual, p.cpad, s_);
  }

  // CudaUnetOps.conv: the product, then (when padded or with a per-image
  // bias) the channel update that narrows it and adds bias / residual.
  Status conv(const Act& x, const Product& p, int stride, const Act* residual,
              const float* image_bias, Act* out) {
    const bool fused = p.cpad == p.cout && !image_bias;
    Act y;
    OSOR_TRY(raw_product(x, p, stride, fused && residual ? residual->p() : nullptr, &y));
    if (p.cpad == p.cout && !image_bias) {
      *out = std::move(y);
      return Status::ok();
    }
    Act o;
    if (p.cpad != p.cout) OSOR_TRY(act(y.b, y.h, y.w, p.cout, &o));
    uint16_t* dst = p.cpad == p.cout ? y.p() : o.p();
    {
      OpScope scope("channel_update", 0.0,
                    2.0 * y.pixels() * p.cout * (residual && !fused ? 3.0 : 2.0), s_, 1);
      OSOR_TRY(cuda_err(channel_update_launch(m_.dtype, y.p(), p.cpad, dst, p.cout,
                                              (long long)y.h * y.w, y.b, image_bias,
                                              m_.temb_rows, fused || !residual ? nullptr
                                                                               : residual->p(),
                                              s_),
                        "channel update"));
    }
    *out = p.cpad == p.cout ? std::move(y) : std::move(o);
    return Status::ok();
  }

  Status group_norm(const Act& x, const Norm& n, float eps, bool silu, Act* y) {
    OSOR_TRY(act(x.b, x.h, x.w, x.c, y));
    const long long pixels = (long long)x.h * x.w;
    const GnNhwcPlan plan = gn_nhwc_plan(x.b, x.c, pixels, kGroups);
    Buf ws;
    OSOR_TRY(raw(plan.workspace_bytes, &ws));
    OpScope scope("groupnorm", 0.0, 4.0 * x.b * x.c * pixels, s_, 3);
    return cuda_err(gn_nhwc_launch(m_.dtype, x.p(), y->p(), n.gamma, n.beta, x.b, x.c, pixels,
                                   kGroups, eps, silu ? 1 : 0, ws.get(), nullptr, s_),
                    "group norm");
  }

  Status layer_norm(const Act& x, const Norm& n, Act* y) {
    OSOR_TRY(act(x.b, x.h, x.w, x.c, y));
    OpScope scope("layernorm", 0.0, 4.0 * x.pixels() * x.c, s_, 1);
    return cuda_err(layer_norm_launch(m_.dtype, x.p(), y->p(), n.gamma, n.beta, x.pixels(), x.c,
                                      kLayerNormEps, s_),
                    "layer norm");
  }

  Status attend(const uint16_t* q, long long ld_q, const uint16_t* k, const uint16_t* v,
                long long ld_kv, long long kv_bs, int heads, int n_kv, const Act& shape,
                Act* out) {
    const int c = shape.c;
    const long long n = (long long)shape.h * shape.w;
    OSOR_TRY(act(shape.b, shape.h, shape.w, c, out));
    OpScope scope("attn_heads", 4.0 * shape.b * n * (double)n_kv * c,
                  2.0 * shape.b * c * (2.0 * n + (kv_bs ? 2.0 * n_kv : 0.0)) +
                      (kv_bs ? 0.0 : 4.0 * n_kv * c),
                  s_, 1);
    return cuda_err(attention_heads_launch(m_.dtype, q, ld_q, n * ld_q, k, v, ld_kv, kv_bs,
                                           out->p(), c, n * c, shape.b, heads, (int)n, n_kv,
                                           c / heads, s_),
                    "multi-head attention");
  }

  Status rows_linear(const float* x, int rows, int in_f, const uint16_t* w, const float* bias,
                     const float* bias2, int out_f, int pre_silu, float* y) {
    int chunk = kRowsLinearFloats / in_f;
    chunk = chunk < 1 ? 1 : (chunk > 8 ? 8 : chunk);
    for (int r0 = 0; r0 < rows; r0 += chunk) {
      const int r = rows - r0 < chunk ? rows - r0 : chunk;
      OpScope scope("rows_linear", 2.0 * r * in_f * out_f, 2.0 * in_f * out_f, s_, 1);
      OSOR_TRY(cuda_err(rows_linear_launch(m_.dtype, x + (long long)r0 * in_f, r, in_f, w, bias,
                                           bias2, out_f, pre_silu, y + (long long)r0 * out_f,
                                           s_),
                        "row linear"));
    }
    return Status::ok();
  }

  // ---------------------------------------------------------------- blocks
  Status resnet(const ResnetL& r, const Act& x, const float* tb, Act* out) {
    Act sc_buf;
    const Act* shortcut = &x;
    if (r.has_sc) {
      OSOR_TRY(conv(x, r.sc, 1, nullptr, nullptr, &sc_buf));
      shortcut = &sc_buf;
    }
    Act g1, h1, g2;
    OSOR_TRY(group_norm(x, r.n1, kResnetEps, true, &g1));
    OSOR_TRY(conv(g1, r.c1, 1, nullptr, tb + r.tb_off, &h1));
    OSOR_TRY(group_norm(h1, r.n2, kResnetEps, true, &g2));
    return conv(g2, r.c2, 1, shortcut, nullptr, out);
  }

  Status transformer(const TransformerL& t, const Act& x, Act* out) {
    Act g, xs;
    OSOR_TRY(group_norm(x, t.norm, kTransformerGnEps, false, &g));
    OSOR_TRY(conv(g, t.proj_in, 1, nullptr, nullptr, &xs));
    const int c = x.c;
    const long long n = (long long)x.h * x.w;
    for (const TBlock& blk : t.blocks) {
      OSOR_TRY(checkpoint());
      {  // self attention on the fused q|k|v product
        Act ln, qkv, o, next;
        OSOR_TRY(layer_norm(xs, blk.ln1, &ln));
        OSOR_TRY(raw_product(ln, blk.qkv, 1, nullptr, &qkv));
        const long long ld = blk.qkv.cpad;
        OSOR_TRY(attend(qkv.p(), ld, qkv.p() + c, qkv.p() + 2 * c, ld, n * ld, t.heads, (int)n,
                        xs, &o));
        OSOR_TRY(conv(o, blk.out1, 1, &xs, nullptr, &next));
        xs = std::move(next);
      }
      {  // cross attention on the prompt's keys / values
        Act ln, q, o, next;
        OSOR_TRY(layer_norm(xs, blk.ln2, &ln));
        OSOR_TRY(raw_product(ln, blk.q2, 1, nullptr, &q));
        OSOR_TRY(attend(q.p(), blk.q2.cpad, blk.k2, blk.v2, c, 0, t.heads, m_.tokens, xs, &o));
        OSOR_TRY(conv(o, blk.out2, 1, &xs, nullptr, &next));
        xs = std::move(next);
      }
      {  // GEGLU feed-forward
        Act ln, hidden, gated, next;
        OSOR_TRY(layer_norm(xs, blk.ln3, &ln));
        if (blk.ff1.geglu) {
          const int f = blk.ff1.cout / 2;
          OSOR_TRY(act(ln.b, ln.h, ln.w, f, &gated));
          const size_t need = geglu_product_workspace(m_.dtype, ln.b, ln.h, ln.w, ln.c, f);
          Buf ws;
          if (need) OSOR_TRY(raw(need, &ws));
          OSOR_TRY(run_geglu_product(m_.dtype, blk.ff1.w, blk.ff1.bias, ln.p(), ln.b, ln.h, ln.w,
                                     ln.c, f, gated.p(), ws.get(), need, s_));
          OSOR_TRY(conv(gated, blk.ff2, 1, &xs, nullptr, &next));
          xs = std::move(next);
          continue;
        }
        if (blk.ff1.cpad == blk.ff1.cout)
          OSOR_TRY(raw_product(ln, blk.ff1, 1, nullptr, &hidden));
        else
          OSOR_TRY(conv(ln, blk.ff1, 1, nullptr, nullptr, &hidden));
        const int f = blk.ff1.cout / 2;
        OSOR_TRY(act(hidden.b, hidden.h, hidden.w, f, &gated));
        {
          OpScope scope("geglu", 0.0, 6.0 * hidden.pixels() * f, s_, 1);
          OSOR_TRY(cuda_err(geglu_launch(m_.dtype, hidden.p(), gated.p(), hidden.pixels(), f, s_),
                            "GEGLU"));
        }
        OSOR_TRY(conv(gated, blk.ff2, 1, &xs, nullptr, &next));
        xs = std::move(next);
      }
    }
    OSOR_TRY(checkpoint());
    return conv(xs, t.proj_out, 1, &x, nullptr, out);
  }

  Status concat(const Act& a, const Act& b, Act* y) {
    OSOR_TRY(act(a.b, a.h, a.w, a.c + b.c, y));
    OpScope scope("concat", 0.0, 4.0 * a.pixels() * (a.c + b.c), s_, 1);
    return cuda_err(concat_channels_launch(a.p(), a.c, b.p(), b.c, y->p(), a.pixels(), s_),
                    "channel concatenation");
  }

  Status resize(const Act& x, int h, int w, Act* y) {
    OSOR_TRY(act(x.b, h, w, x.c, y));
    OpScope scope("resize", 0.0, 2.0 * x.b * x.c * ((double)x.h * x.w + (double)h * w), s_, 1);
    return cuda_err(resize_nearest_launch(x.p(), y->p(), x.b, x.h, x.w, h, w, x.c, s_),
                    "nearest resize");
  }

  Status forward(const float* input, int timestep, const float* time_ids, float* output, int b,
                 int h, int w) {
    const Unet& m = m_;
    const osor_unet_config& cfg = m.cfg;
    // Time and added embeddings, then every resnet's time bias.
    Buf feats, hidden, temb, tb;
    OSOR_TRY(raw((size_t)b * m.feat_w * 4, &feats));
    OSOR_TRY(raw((size_t)b * 2 * m.time_dim * 4, &hidden));
    OSOR_TRY(raw((size_t)b * m.time_dim * 4, &temb));
    OSOR_TRY(raw((size_t)b * m.temb_rows * 4, &tb));
    {
      OpScope scope("time_features", 0.0, 4.0 * b * m.feat_w, s_, 1);
      OSOR_TRY(cuda_err(unet_time_features_launch(time_ids, m.pooled, b, (float)timestep, m.base,
                                                  cfg.time_projection, cfg.pooled,
                                                  static_cast<float*>(feats.get()), s_),
                        "time features"));
    }
    OSOR_TRY(rows_linear(static_cast<float*>(feats.get()), b, m.feat_w, m.emb_w1, m.emb_b1,
                         nullptr, 2 * m.time_dim, 0, static_cast<float*>(hidden.get())));
    OSOR_TRY(rows_linear(static_cast<float*>(hidden.get()), b, 2 * m.time_dim, m.emb_w2,
                         m.emb_b2a, m.emb_b2b, m.time_dim, 1, static_cast<float*>(temb.get())));
    OSOR_TRY(rows_linear(static_cast<float*>(temb.get()), b, m.time_dim, m.temb_w, m.temb_b,
                         nullptr, m.temb_rows, 1, static_cast<float*>(tb.get())));
    const float* tbp = static_cast<const float*>(tb.get());

    // Activations are never modified after they are produced, so a skip and
    // the running activation share one buffer, as tensors do on the Python
    // host.
    using ActP = std::shared_ptr<Act>;
    ActP xs = std::make_shared<Act>();
    if (m.conv_in_cols.w) {
      // conv_in on tensor cores: the column matrix of the nine-channel input,
      // then a 1x1 product (narrowed from 384 to 320 channels).
      Act cols;
      OSOR_TRY(act(b, h, w, 128, &cols));
      {
        OpScope scope("thin_columns", 0.0, 4.0 * b * h * w * 9 + 256.0 * b * h * w, s_, 1);
        OSOR_TRY(cuda_err(thin_columns_launch(m.dtype, input, cols.p(), b, 9, h, w, 3, 1, nullptr,
                                              nullptr, s_, 128),
                          "thin input columns"));
      }
      OSOR_TRY(conv(cols, m.conv_in_cols, 1, nullptr, nullptr, xs.get()));
    } else {
      OSOR_TRY(act(b, h, w, m.conv_in.cout, xs.get()));
      ConvLayer L;
      L.cin = m.conv_in.cin;
      L.cout = m.conv_in.cout;
      L.k = 3;
      L.stride = 1;
      L.pad = 1;
      L.pad_end = 1;
      L.w = m.conv_in.w;
      L.bias = m.conv_in.bias;
      OSOR_TRY(run_conv(m.dtype, L, input, kLayoutNchwF32, b, h, w, m.conv_in.cin, xs->p(),
                        kLayoutNhwc16, m.conv_in.cout, nullptr, m.conv_in.cout, s_));
    }
    std::vector<ActP> residuals{xs};
    for (int i = 0; i < 3; ++i) {
      OSOR_TRY(checkpoint());
      const Level& lv = m.down[i];
      for (size_t j = 0; j < lv.resnets.size(); ++j) {
        ActP r = std::make_shared<Act>();
        OSOR_TRY(resnet(lv.resnets[j], *xs, tbp, r.get()));
        if (!lv.attns.empty()) {
          ActP t = std::make_shared<Act>();
          OSOR_TRY(transformer(lv.attns[j], *r, t.get()));
          r = t;
        }
        xs = r;
        residuals.push_back(xs);
      }
      if (lv.resample) {
        ActP d = std::make_shared<Act>();
        OSOR_TRY(conv(*xs, lv.resample_conv, 2, nullptr, nullptr, d.get()));
        xs = d;
        residuals.push_back(xs);
      }
    }
    OSOR_TRY(checkpoint());
    {
      ActP a = std::make_shared<Act>(), t = std::make_shared<Act>(), c = std::make_shared<Act>();
      OSOR_TRY(resnet(m.mid0, *xs, tbp, a.get()));
      OSOR_TRY(transformer(m.mid_attn, *a, t.get()));
      OSOR_TRY(resnet(m.mid1, *t, tbp, c.get()));
      xs = c;
    }
    for (int i = 0; i < 3; ++i) {
      OSOR_TRY(checkpoint());
      const Level& lv = m.up[i];
      const size_t count = lv.resnets.size();
      if (residuals.size() < count)
        return Status::err(OSOR_ERR_INVALID_ARTIFACT, "UNet residual topology is inconsistent");
      for (size_t j = 0; j < count; ++j) {
        ActP skip = residuals.back();
        residuals.pop_back();
        Act cat;
        OSOR_TRY(concat(*xs, *skip, &cat));
        ActP r = std::make_shared<Act>();
        OSOR_TRY(resnet(lv.resnets[j], cat, tbp, r.get()));
        if (!lv.attns.empty()) {
          ActP t = std::make_shared<Act>();
          OSOR_TRY(transformer(lv.attns[j], *r, t.get()));
          r = t;
        }
        xs = r;
      }
      if (lv.resample) {
        const Act& next = *residuals.back();
        Act up;
        ActP c = std::make_shared<Act>();
        OSOR_TRY(resize(*xs, next.h, next.w, &up));
        OSOR_TRY(conv(up, lv.resample_conv, 1, nullptr, nullptr, c.get()));
        xs = c;
      }
    }
    if (!residuals.empty())
      return Status::err(OSOR_ERR_INVALID_ARTIFACT, "UNet residual topology left unused tensors");
    OSOR_TRY(checkpoint());
    Act g;
    OSOR_TRY(group_norm(*xs, m.norm_out, kResnetEps, true, &g));
    ConvLayer L;
    L.cin = m.conv_out.cin;
    L.cout = m.conv_out.cout;
    L.k = 3;
    L.stride = 1;
    L.pad = 1;
    L.pad_end = 1;
    L.w = m.conv_out.w;
    L.bias = m.conv_out.bias;
    return run_conv(m.dtype, L, g.p(), kLayoutNhwc16, b, h, w, g.c, output, kLayoutNchwF32,
                    m.conv_out.cout, nullptr, m.conv_out.cout, s_);
  }

 private:
  const Unet& m_;
  cudaStream_t s_;
  const volatile int* cancel_;
};

}  // namespace

// ------------------------------------------------------------------ create
namespace {

Status load_resnet(Loader& ld, const std::string& p, int cin, int cout, int td, ResnetL* r,
                   std::vector<const float*>* temb_w, std::vector<const float*>* temb_b,
                   int* temb_rows) {
  OSOR_TRY(ld.norm(p + ".norm1", cin, &r->n1));
  OSOR_TRY(ld.conv(p + ".conv1", cin, cout, 3, &r->c1));
  OSOR_TRY(ld.norm(p + ".norm2", cout, &r->n2));
  OSOR_TRY(ld.conv(p + ".conv2", cout, cout, 3, &r->c2));
  r->has_sc = cin != cout;
  if (r->has_sc) OSOR_TRY(ld.conv(p + ".conv_shortcut", cin, cout, 1, &r->sc));
  const float *w, *b;
  OSOR_TRY(ld.get(p + ".time_emb_proj.weight", {cout, td}, &w));
  OSOR_TRY(ld.get(p + ".time_emb_proj.bias", {cout}, &b));
  temb_w->push_back(w);
  temb_b->push_back(b);
  r->tb_off = *temb_rows;
  *temb_rows += cout;
  return Status::ok();
}

Status load_transformer(Loader& ld, const std::string& p, int c, int depth, int heads,
                        int context, int tokens, const uint16_t* ctx16, int dtype,
                        TransformerL* t) {
  t->heads = heads;
  OSOR_TRY(ld.norm(p + ".norm", c, &t->norm));
  OSOR_TRY(ld.linear(p + ".proj_in", c, c, true, &t->proj_in));
  OSOR_TRY(ld.linear(p + ".proj_out", c, c, true, &t->proj_out));
  const float scale = (float)(1.0 / std::sqrt((double)(c / heads)));
  t->blocks.resize(depth);
  for (int d = 0; d < depth; ++d) {
    const std::string q = p + ".transformer_blocks." + std::to_string(d);
    TBlock& blk = t->blocks[d];
    OSOR_TRY(ld.norm(q + ".norm1", c, &blk.ln1));
    OSOR_TRY(ld.norm(q + ".norm2", c, &blk.ln2));
    OSOR_TRY(ld.norm(q + ".norm3", c, &blk.ln3));
    const float *wq, *wk, *wv, *cq, *ck, *cv;
    OSOR_TRY(ld.get(q + ".attn1.to_q.weight", {c, c}, &wq));
    OSOR_TRY(ld.get(q + ".attn1.to_k.weight", {c, c}, &wk));
    OSOR_TRY(ld.get(q + ".attn1.to_v.weight", {c, c}, &wv));
    std::vector<float> qkv((size_t)3 * c * c);
    for (size_t i = 0; i < (size_t)c * c; ++i) qkv[i] = wq[i] * scale;
    std::memcpy(qkv.data() + (size_t)c * c, wk, sizeof(float) * c * c);
    std::memcpy(qkv.data() + (size_t)2 * c * c, wv, sizeof(float) * c * c);
    OSOR_TRY(ld.product_from(qkv.data(), nullptr, 3 * c, c, 1, true, &blk.qkv));
    OSOR_TRY(ld.linear(q + ".attn1.to_out.0", c, c, true, &blk.out1));
    OSOR_TRY(ld.get(q + ".attn2.to_q.weight", {c, c}, &cq));
    std::vector<float> q2((size_t)c * c);
    for (size_t i = 0; i < q2.size(); ++i) q2[i] = cq[i] * scale;
    OSOR_TRY(ld.product_from(q2.data(), nullptr, c, c, 1, true, &blk.q2));
    OSOR_TRY(ld.linear(q + ".attn2.to_out.0", c, c, true, &blk.out2));
    {
      // GEGLU input projection: with 4c a multiple of 128 its rows are
      // interleaved (128 value rows, then their 128 gate rows) so that the
      // product's epilogue applies the gate.
      const float *fw, *fb;
      OSOR_TRY(ld.get(q + ".ff.net.0.proj.weight", {8 * c, c}, &fw));
      OSOR_TRY(ld.get(q + ".ff.net.0.proj.bias", {8 * c}, &fb));
      const int f = 4 * c;
      if (f % 128 == 0 && c % 8 == 0) {
        std::vector<float> iw((size_t)8 * c * c), ib((size_t)8 * c);
        for (int r = 0; r < 2 * f; ++r) {
          const int t = r / 256, j = r % 256;
          const int src = j < 128 ? t * 128 + j : f + t * 128 + (j - 128);
          std::memcpy(iw.data() + (size_t)r * c, fw + (size_t)src * c, sizeof(float) * c);
          ib[r] = fb[src];
        }
        OSOR_TRY(ld.product_from(iw.data(), ib.data(), 2 * f, c, 1, false, &blk.ff1));
        blk.ff1.geglu = true;
      } else {
        OSOR_TRY(ld.linear(q + ".ff.net.0.proj", c, 8 * c, true, &blk.ff1));
      }
    }
    OSOR_TRY(ld.linear(q + ".ff.net.2", 4 * c, c, true, &blk.ff2));
    // The prompt's keys / values: [tokens][context] x W^T on the device.
    OSOR_TRY(ld.get(q + ".attn2.to_k.weight", {c, context}, &ck));
    OSOR_TRY(ld.get(q + ".attn2.to_v.weight", {c, context}, &cv));
    for (int which = 0; which < 2; ++which) {
      Product kp;
      OSOR_TRY(ld.product_from(which == 0 ? ck : cv, nullptr, c, context, 1, false, &kp));
      uint16_t* out = nullptr;
      void* mem = nullptr;
      OSOR_TRY(cuda_err(cudaMalloc(&mem, (size_t)tokens * c * 2), "prompt key allocation"));
      ld.own(mem);
      out = static_cast<uint16_t*>(mem);
      ConvLayer L;
      L.cin = context;
      L.cout = c;
      L.k = 1;
      L.w = kp.w;
      OSOR_TRY(run_conv(dtype, L, ctx16, kLayoutNhwc16, 1, 1, tokens, context, out, kLayoutNhwc16,
                        c, nullptr, c, nullptr));
      (which == 0 ? blk.k2 : blk.v2) = out;
    }
  }
  return Status::ok();
}

}  // namespace

Status unet_create(const osor_tensor* tensors, size_t count, const osor_unet_config* cfg,
                   const float* context, int tokens, const float* pooled, int device, Unet** out) {
  if (!cfg || !context || !pooled || !out) return Status::err(OSOR_ERR_INVALID_INPUT, "null argument");
  if (cfg->dtype != OSOR_DTYPE_BF16 && cfg->dtype != OSOR_DTYPE_F16)
    return Status::err(OSOR_ERR_INVALID_INPUT, "dtype must be OSOR_DTYPE_BF16 or OSOR_DTYPE_F16");
  for (int i = 0; i < 3; ++i)
    if (cfg->channels[i] <= 0 || cfg->channels[i] % kGroups != 0 || cfg->channels[i] % 8 != 0 ||
        cfg->heads[i] <= 0 || cfg->channels[i] % cfg->heads[i] != 0 || cfg->depth[i] < 0)
      return Status::err(OSOR_ERR_INVALID_INPUT,
                         "UNet channels must be multiples of 32 divisible by the head count");
  if (cfg->depth[2] == 0)
    return Status::err(OSOR_ERR_INVALID_INPUT, "UNet middle block requires cross attention");
  if (cfg->layers < 1 || cfg->context <= 0 || cfg->pooled < 0 || cfg->time_projection < 2 ||
      cfg->time_projection % 2 != 0 || tokens < 1 || tokens > 1024)
    return Status::err(OSOR_ERR_INVALID_INPUT, "fixed conditioning must be [1, 1..=1024, context]");
  std::unique_ptr<Unet> m(new Unet());
  m->device = device;
  m->dtype = cfg->dtype == OSOR_DTYPE_F16 ? kF16 : kBf16;
  m->cfg = *cfg;
  m->tokens = tokens;
  m->base = cfg->channels[0];
  m->time_dim = 4 * m->base;
  m->feat_w = m->base + cfg->pooled + 6 * cfg->time_projection;
  int prev = 0;
  cudaGetDevice(&prev);
  OSOR_TRY(cuda_err(cudaSetDevice(device), "set device"));
  struct Restore {
    int d;
    ~Restore() { cudaSetDevice(d); }
  } restore{prev};
  {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    OSOR_TRY(cuda_err(cudaMemPoolCreate(&m->pool, &props), "memory pool"));
    uint64_t keep = ~0ull;
    OSOR_TRY(cuda_err(cudaMemPoolSetAttribute(m->pool, cudaMemPoolAttrReleaseThreshold, &keep),
                      "memory pool"));
  }
  Loader ld(tensors, count, m.get());
  const int td = m->time_dim, base = m->base;
  const int* ch = cfg->channels;
  // Prompt sequence in the model dtype, [tokens][context].
  uint16_t* ctx16 = nullptr;
  OSOR_TRY(ld.pack(context, tokens, cfg->context, 1, tokens, &ctx16));
  OSOR_TRY(ld.upload(pooled, (size_t)cfg->pooled > 0 ? cfg->pooled : 1, &m->pooled));
  OSOR_TRY(ld.conv("conv_in", 9, base, 3, &m->conv_in, false));
  {
    // conv_in's 3 x 3 x 9 taps as columns (tap-major, then channel) of a 1x1
    // product over 128 columns.
    const float *w, *b;
    OSOR_TRY(ld.get("conv_in.weight", {base, 9, 3, 3}, &w));
    OSOR_TRY(ld.get("conv_in.bias", {base}, &b));
    std::vector<float> cols((size_t)base * 128, 0.0f);
    for (int co = 0; co < base; ++co)
      for (int ci = 0; ci < 9; ++ci)
        for (int t = 0; t < 9; ++t)
          cols[(size_t)co * 128 + t * 9 + ci] = w[((size_t)co * 9 + ci) * 9 + t];
    OSOR_TRY(ld.product_from(cols.data(), b, base, 128, 1, true, &m->conv_in_cols));
  }
  {
    const float *w1t, *b1t, *w2t, *b2t, *w1a, *b1a, *w2a, *b2a;
    const int add_w = cfg->pooled + 6 * cfg->time_projection;
    OSOR_TRY(ld.get("time_embedding.linear_1.weight", {td, base}, &w1t));
    OSOR_TRY(ld.get("time_embedding.linear_1.bias", {td}, &b1t));
    OSOR_TRY(ld.get("time_embedding.linear_2.weight", {td, td}, &w2t));
    OSOR_TRY(ld.get("time_embedding.linear_2.bias", {td}, &b2t));
    OSOR_TRY(ld.get("add_embedding.linear_1.weight", {td, add_w}, &w1a));
    OSOR_TRY(ld.get("add_embedding.linear_1.bias", {td}, &b1a));
    OSOR_TRY(ld.get("add_embedding.linear_2.weight", {td, td}, &w2a));
    OSOR_TRY(ld.get("add_embedding.linear_2.bias", {td}, &b2a));
    // Block-diagonal first layers over (time projection | pooled, id projections).
    std::vector<float> w1((size_t)2 * td * m->feat_w, 0.0f);
    for (int o = 0; o < td; ++o) {
      std::memcpy(&w1[(size_t)o * m->feat_w], w1t + (size_t)o * base, sizeof(float) * base);
      std::memcpy(&w1[(size_t)(td + o) * m->feat_w + base], w1a + (size_t)o * add_w,
                  sizeof(float) * add_w);
    }
    OSOR_TRY(ld.pack(w1.data(), 2 * td, m->feat_w, 1, 2 * td, &m->emb_w1));
    std::vector<float> b1(2 * td);
    std::memcpy(b1.data(), b1t, sizeof(float) * td);
    std::memcpy(b1.data() + td, b1a, sizeof(float) * td);
    OSOR_TRY(ld.upload(b1.data(), b1.size(), &m->emb_b1));
    // Second layers side by side: their sum is emb + added.
    std::vector<float> w2((size_t)td * 2 * td);
    for (int o = 0; o < td; ++o) {
      std::memcpy(&w2[(size_t)o * 2 * td], w2t + (size_t)o * td, sizeof(float) * td);
      std::memcpy(&w2[(size_t)o * 2 * td + td], w2a + (size_t)o * td, sizeof(float) * td);
    }
    OSOR_TRY(ld.pack(w2.data(), td, 2 * td, 1, td, &m->emb_w2));
    OSOR_TRY(ld.upload(b2t, td, &m->emb_b2a));
    OSOR_TRY(ld.upload(b2a, td, &m->emb_b2b));
  }
  std::vector<const float*> temb_w, temb_b;
  std::vector<int> temb_c;
  int temb_rows = 0;
  auto resnet = [&](const std::string& p, int cin, int cout, ResnetL* r) {
    temb_c.push_back(cout);
    return load_resnet(ld, p, cin, cout, td, r, &temb_w, &temb_b, &temb_rows);
  };
  auto transformer = [&](const std::string& p, int c, int depth, int heads, TransformerL* t) {
    return load_transformer(ld, p, c, depth, heads, cfg->context, tokens, ctx16, m->dtype, t);
  };
  for (int i = 0; i < 3; ++i) {
    Level& lv = m->down[i];
    const int cin = i == 0 ? base : ch[i - 1];
    lv.resnets.resize(cfg->layers);
    if (cfg->depth[i] > 0) lv.attns.resize(cfg->layers);
    for (int j = 0; j < cfg->layers; ++j) {
      const std::string p = "down_blocks." + std::to_string(i);
      OSOR_TRY(resnet(p + ".resnets." + std::to_string(j), j == 0 ? cin : ch[i], ch[i],
                      &lv.resnets[j]));
      if (cfg->depth[i] > 0)
        OSOR_TRY(transformer(p + ".attentions." + std::to_string(j), ch[i], cfg->depth[i],
                             cfg->heads[i], &lv.attns[j]));
    }
    lv.resample = i + 1 < 3;
    if (lv.resample)
      OSOR_TRY(ld.conv("down_blocks." + std::to_string(i) + ".downsamplers.0.conv", ch[i], ch[i],
                       3, &lv.resample_conv));
  }
  OSOR_TRY(resnet("mid_block.resnets.0", ch[2], ch[2], &m->mid0));
  OSOR_TRY(transformer("mid_block.attentions.0", ch[2], cfg->depth[2], cfg->heads[2],
                       &m->mid_attn));
  OSOR_TRY(resnet("mid_block.resnets.1", ch[2], ch[2], &m->mid1));
  for (int i = 0; i < 3; ++i) {
    Level& lv = m->up[i];
    const int out_c = ch[2 - i];
    const int prev_c = i == 0 ? ch[2] : ch[3 - i];
    const int in_c = i + 1 == 3 ? base : ch[3 - i - 2];
    const int layers = cfg->layers + 1;
    lv.resnets.resize(layers);
    if (cfg->depth[2 - i] > 0) lv.attns.resize(layers);
    for (int j = 0; j < layers; ++j) {
      const int skip = j + 1 == layers ? in_c : out_c;
      const std::string p = "up_blocks." + std::to_string(i);
      OSOR_TRY(resnet(p + ".resnets." + std::to_string(j), (j == 0 ? prev_c : out_c) + skip,
                      out_c, &lv.resnets[j]));
      if (cfg->depth[2 - i] > 0)
        OSOR_TRY(transformer(p + ".attentions." + std::to_string(j), out_c, cfg->depth[2 - i],
                             cfg->heads[2 - i], &lv.attns[j]));
    }
    lv.resample = i + 1 < 3;
    if (lv.resample)
      OSOR_TRY(ld.conv("up_blocks." + std::to_string(i) + ".upsamplers.0.conv", out_c, out_c, 3,
                       &lv.resample_conv));
  }
  OSOR_TRY(ld.norm("conv_norm_out", base, &m->norm_out));
  OSOR_TRY(ld.conv("conv_out", base, 5, 3, &m->conv_out));
  // Every resnet's time_emb_proj stacked in execution order.
  {
    std::vector<float> w((size_t)temb_rows * td), b(temb_rows);
    size_t row = 0;
    for (size_t r = 0; r < temb_w.size(); ++r) {
      std::memcpy(&w[row * td], temb_w[r], sizeof(float) * temb_c[r] * td);
      std::memcpy(&b[row], temb_b[r], sizeof(float) * temb_c[r]);
      row += temb_c[r];
    }
    OSOR_TRY(ld.pack(w.data(), temb_rows, td, 1, temb_rows, &m->temb_w));
    OSOR_TRY(ld.upload(b.data(), b.size(), &m->temb_b));
    m->temb_rows = temb_rows;
  }
  OSOR_TRY(cuda_err(cudaDeviceSynchronize(), "UNet load"));
  *out = m.release();
  return Status::ok();
}

void unet_destroy(Unet* m) { delete m; }

Status unet_denoise(const Unet& m, const float* input, int timestep, const float* time_ids,
                    float* output, int batch, int height, int width, cudaStream_t s,
                    const volatile int* cancel) {
  if (!input || !time_ids || !output) return Status::err(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch < 1 || batch > 4 || height < 4 || height > 128 || width < 4 || width > 128)
    return Status::err(OSOR_ERR_INVALID_INPUT,
                       "UNet expects batch 1..=4, 9 channels and spatial dimensions 4..=128");
  if (timestep < 0) return Status::err(OSOR_ERR_INVALID_INPUT, "timestep must be non-negative");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(m.device);
  Status st;
  {
    Run run(m, s, cancel);
    st = run.checkpoint();
    if (st.good()) st = run.forward(input, timestep, time_ids, output, batch, height, width);
  }
  cudaSetDevice(prev);
  return st;
}

}  // namespace osor
