// VAE model runtime: weights repacked once to 16-bit tensor-core layouts, and
// the encoder / decoder graph executed as a sequence of kernel launches on one
// stream over a caller-provided workspace.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/osor_b200.h"

namespace osor {

struct Status {
  int code = OSOR_OK;
  std::string message;
  static Status ok() { return Status(); }
  static Status err(int c, std::string m) {
    Status s;
    s.code = c;
    s.message = std::move(m);
    return s;
  }
  bool good() const { return code == OSOR_OK; }
};

struct ConvLayer {
  int cin = 0, cout = 0, k = 1, stride = 1, pad = 0;
  int pad_end = 0;           // zero padding after the last row / column (encoder downsample: 1)
  const uint16_t* w = nullptr;  // 16-bit [w_rows][k*k*cin], (ky, kx, ci)
  const float* bias = nullptr;  // [cout]
  int w_rows = 0;               // allocated weight rows (>= cout; 16 for thin outputs)
  // For a 3x3 conv that follows a nearest 2x upsample: the four 2x2 phase
  // convolutions on the low-res input, [4 * cout][2][2][cin] (see
  // ConvTcArgs::upsample); nullptr otherwise.
  const uint16_t* w_up = nullptr;
  // For a thin 3x3 output (Cout <= 3): the per-pixel tap matrix of the fused
  // GroupNorm + conv kernel, 16-bit [32][cin], row (ky * 3 + kx) * cout + co
  // = w[co][ky][kx][:], rows past 9 * cout zero; nullptr otherwise.
  const uint16_t* w_z = nullptr;
};

// A convolution whose input has few channels (the image or the latent): run
// as a column matrix of 64 K-columns (thin_columns_launch) times `cols`, a
// 1x1 layer with Cin = 64. `pre_w`/`pre_b` (nullable) is a 1x1 convolution
// applied to every input pixel first (the decoder's post_quant_conv).
struct ThinInputLayer {
  int cin = 0, k = 3, pad = 1;
  ConvLayer cols;
  const float* pre_w = nullptr;
  const float* pre_b = nullptr;
};

struct NormLayer {
  int c = 0;
  float* gamma = nullptr;
  float* beta = nullptr;
};

struct ResnetLayer {
  NormLayer n1, n2;
  ConvLayer c1, c2;
  bool has_shortcut = false;
  ConvLayer shortcut;
};

struct AttentionLayer {
  NormLayer norm;
  ConvLayer qkv;  // 1x1, c -> 3c; q and k rows pre-scaled by c^-1/4
  ConvLayer out;  // 1x1, c -> c
};

struct MidLayer {
  ResnetLayer first, second;
  AttentionLayer attn;
};

struct StageLayer {
  std::vector<ResnetLayer> resnets;
  bool resample = false;  // upsample (decoder) / downsample (encoder)
  ConvLayer resample_conv;
};

struct Decoder {
  ThinInputLayer conv_in_thin;  // post_quant_conv + conv_in as one column GEMM
  MidLayer mid;
  std::vector<StageLayer> up;
  NormLayer norm_out;
  ConvLayer conv_out;
};

struct Encoder {
  ThinInputLayer conv_in_thin;
  std::vector<StageLayer> down;
  MidLayer mid;
  NormLayer norm_out;
  ConvLayer conv_out, quant;
};

// Per-call workspace layout (all parts 256-byte aligned).
struct WorkspacePlan {
  size_t act_bytes = 0;      // one activation buffer
  size_t tstat_bytes = 0;    // per-tile GroupNorm statistics of one activation buffer
  size_t f32_bytes = 0;      // thin f32 NCHW scratch
  size_t scores_bytes = 0;   // attention softmax partials for one image
  size_t probs_bytes = 0;    // attention probabilities (16-bit) for one image
  size_t rowsum_bytes = 0;
  size_t gn_bytes = 0;
  size_t total = 0;
};

struct Vae {
  int device = 0;
  int dtype = 0;  // Dtype of weights and activations
  int channels[4] = {128, 256, 512, 512};
  int layers = 2;
  bool has_decoder = false, has_encoder = false;
  Decoder dec;
  Encoder enc;
  std::vector<void*> allocations;
  ~Vae();
};

Status vae_create(const osor_tensor* tensors, size_t count, const osor_vae_config* cfg, int device,
                  Vae** out);
WorkspacePlan vae_workspace_plan(const Vae& m, int op, int batch, int height, int width);
Status vae_decode(const Vae& m, const float* latents, float* image, int batch, int h, int w,
                  void* workspace, size_t workspace_bytes, cudaStream_t stream,
                  const volatile int* cancel);
Status vae_encode(const Vae& m, const float* image, float* moments, int batch, int height,
                  int width, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                  const volatile int* cancel);

// Row-band decode of one image on one rank of a peer group (peer.h): the
// rank's rows [r R, (r + 1) R) of the latent (R = h / ranks) through the
// whole decoder, halo rows and GroupNorm statistics exchanged with the other
// ranks between layers and the mid-block attention's keys and values
// gathered from all of them. latents: the whole image [1, 4, h, w] f32 NCHW on
// every rank; image_band: this rank's rows of the f32 NCHW image,
// [1, 3, 8 R, 8 w].
struct PeerGroup;
struct BandSizes {
  size_t workspace = 0;       // bytes of device workspace per call
  size_t halo_row_bytes = 0;  // the peer group's halo slot size
  size_t bulk_bytes = 0;      // the peer group's bulk slot size (attention q|k|v part)
};
Status vae_decode_band_sizes(const Vae& m, int ranks, int h, int w, BandSizes* out);
Status vae_decode_band(const Vae& m, PeerGroup* g, const float* latents, float* image_band, int h,
                       int w, void* workspace, size_t workspace_bytes, cudaStream_t stream);

// Single-op entry points shared with the C ABI. in_mode / out_mode are
// kLayoutNhwc16 (16-bit of `dtype`) or kLayoutNchwF32.
// With gn_part set and a tensor-core shape whose Cout has 4, 8 or 16
// channels per group of 32, the epilogue also writes per-tile GroupNorm
// statistics of the output to gn_part and sets *gn_done.
//
// With norm set, x is the raw activation and the convolution applies
// GroupNorm(+SiLU) to its input itself (norm->coef[b][c][4] from the
// GroupNorm finalize; input rows outside [norm->y0, norm->y1), y1 < 0 for
// all rows, are zero padding): 16-bit NHWC in and out, and only the shapes
// conv_takes_input_norm accepts (others are refused with
// OSOR_ERR_INVALID_INPUT; the caller normalises separately instead).
struct InputNorm {
  const float* coef = nullptr;
  int silu = 1;
  int y0 = 0, y1 = -1;
};
Status run_conv(int dtype, const ConvLayer& L, const void* x, int in_mode, int batch, int in_h,
                int in_w, long long in_pixel_stride, void* out, int out_mode,
                long long out_pixel_stride, const void* residual, long long ld_res,
                cudaStream_t s, float* gn_part = nullptr, bool* gn_done = nullptr,
                const InputNorm* norm = nullptr);
// GEGLU feed-forward input: y[pixel][f] = value * gelu_erf(gate) of the 1x1
// product x W^T + bias with 2 * features weight rows in the interleaved order
// of ConvTcArgs::geglu (features a multiple of 128; x NHWC 16-bit [pixels][cin],
// y [pixels][features]). On CTA pairs the gate is applied in the product's
// epilogue and no workspace is used; other shapes store the product in
// `workspace` (geglu_product_workspace bytes) and gate it in a second pass.
size_t geglu_product_workspace(int dtype, int batch, int h, int w, int cin, int features);
Status run_geglu_product(int dtype, const uint16_t* weight, const float* bias, const void* x,
                         int batch, int h, int w, int cin, int features, void* y, void* workspace,
                         size_t workspace_bytes, cudaStream_t s);
bool conv_takes_input_norm(int dtype, const ConvLayer& L, const void* x, int batch, int in_h,
                           int in_w, long long in_pixel_stride, void* out,
                           long long out_pixel_stride, const void* residual, long long ld_res,
                           const InputNorm& norm);
// OSOR_FUSED_INPUT_NORM=1 in the environment (read once per process) lets
// the decoder's and band decoder's resnet convolutions apply their input
// GroupNorm themselves. Off by default: on B200 the fused 3x3 convolutions
// measured 1.7-2x slower than the separate apply pass plus the plain
// convolution (the transform warps' arithmetic does not overlap the MMAs).
bool fused_input_norm_enabled();

// softmax(q k^T) v for `batch` images: n_q query rows (stride ld_q) against
// n_kv key / value rows (stride ld_kv) per image. scores (softmax partials:
// n_q x n_kv / 32 x 2 + n_q floats), probs [n_q][n_kv] 16-bit, rowsum [n_q]
// and vt [dim][n_kv] are per-image scratch reused across images.
Status attention_core(int dtype, const void* q, long long ld_q, const void* k, const void* v,
                      long long ld_kv, void* out, long long ld_out, int batch, int n_q, int n_kv,
                      int dim, float* scores, void* probs, float* rowsum, void* vt,
                      cudaStream_t s);

}  // namespace osor
