/*
 * osor_b200 -- C ABI of the B200 (sm_100a) SDXL VAE hot path.
 *
 * This is the boundary a host binding calls: plain pointers, sizes and an
 * opaque model handle; no framework types. Every device pointer refers to
 * memory of the device the call runs on; `stream` is a cudaStream_t (NULL for
 * the legacy default stream). Calls enqueue work on `stream` and return once
 * it is enqueued; results are ready when the stream is synchronised.
 *
 * Each entry point names the reference (doublesharp/osor-rs) interface it
 * replaces, by path:line inside that project.
 */
#ifndef OSOR_B200_H
#define OSOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The first four errors mirror osor::Error (src/lib.rs:62-90):
 * InvalidInput, InvalidArtifact, Unavailable, Cancelled; the last two are
 * CUDA-level failures. A failed call leaves a message for
 * osor_last_error_message() on the calling thread. */
#define OSOR_OK 0
#define OSOR_ERR_INVALID_INPUT 1
#define OSOR_ERR_INVALID_ARTIFACT 2
#define OSOR_ERR_UNAVAILABLE 3
#define OSOR_ERR_CANCELLED 4
#define OSOR_ERR_CUDA 5
#define OSOR_ERR_TIMEOUT 6

/* Element types. Weights and activations of a model (and the 16-bit tensors
 * of an op call) are bf16 or f16; the reference's CUDA backend accepts both
 * model dtypes (src/runtime.rs:406-417). f32 is accepted by the standalone
 * group norm only. */
#define OSOR_DTYPE_BF16 0
#define OSOR_DTYPE_F16 1
#define OSOR_DTYPE_F32 2

/* Tensor layouts at the boundary. */
#define OSOR_LAYOUT_NHWC 0 /* [B][H][W][C], the internal layout (16-bit) */
#define OSOR_LAYOUT_NCHW 1 /* [B][C][H][W], the reference's layout */

/* Operations for osor_vae_workspace_size. */
#define OSOR_OP_DECODE 0
#define OSOR_OP_ENCODE 1

/* Model parts (bitmask) for osor_vae_config.parts. */
#define OSOR_PART_DECODER 1
#define OSOR_PART_ENCODER 2

typedef struct osor_vae osor_vae;

/* One named host float32 tensor of a diffusers-named VAE state dict, as the
 * reference's VarBuilder reads it (src/native/vae_encoder.rs:224-260,388-412;
 * src/native/vae_decoder.rs:62-101). */
typedef struct osor_tensor {
  const char* name;
  const float* data;
  int ndim;
  int64_t shape[4];
} osor_tensor;

/* Architecture::sdxl() VAE fields (src/native.rs:94-95) plus the model dtype
 * (LoadOptions::dtype, src/runtime.rs:137-160). */
typedef struct osor_vae_config {
  int channels[4]; /* block_out_channels, e.g. {128, 256, 512, 512} */
  int layers;      /* resnets per encoder down block (decoder: layers + 1) */
  int parts;       /* OSOR_PART_DECODER | OSOR_PART_ENCODER */
  int dtype;       /* OSOR_DTYPE_BF16 or OSOR_DTYPE_F16 */
} osor_vae_config;

/* Message of the last failed call on this thread ("" if none). */
const char* osor_last_error_message(void);

/* Library ABI version (major * 10000 + minor * 100 + patch). */
int osor_version(void);

/* OSOR_OK when `device` is an sm_100 GPU this library was built for, else
 * OSOR_ERR_UNAVAILABLE. Replaces Backend::Cuda{ordinal} device resolution
 * (src/runtime.rs:62-74). */
int osor_device_check(int device);

/* Synchronises `device`, returns its device-side status word (0 = no kernel
 * reported a problem; 1 = a bounded wait timed out) and clears it when
 * `reset` is non-zero. A negative value is -(status code) of a failed read. */
int osor_device_status(int device, int reset);

/* Builds a model from host float32 weights: repacks convolution weights to
 * 16-bit [Cout][ky][kx][Cin], folds the attention scale C^-1/4 into the q and
 * k projections and uploads everything to `device`. Missing or mis-shaped
 * tensors return OSOR_ERR_INVALID_ARTIFACT. Replaces NativeModel::new ->
 * VaeEncoder::new / VaeDecoder::new (src/native.rs:398-425,
 * src/native/vae_encoder.rs:388-412, src/native/vae_decoder.rs:62-101). */
int osor_vae_create(const osor_tensor* tensors, size_t count, const osor_vae_config* config,
                    int device, osor_vae** out);
void osor_vae_destroy(osor_vae* vae);

/* Bytes of device workspace osor_vae_decode / osor_vae_encode_moments need
 * for the given batch and spatial size (latent h, w for decode; image H, W
 * for encode). 0 when the shape is not admissible. */
size_t osor_vae_workspace_size(const osor_vae* vae, int op, int batch, int height, int width);

/* Decodes unscaled latents [B][4][h][w] f32 (device) into raw RGB
 * [B][3][8h][8w] f32 (device). `cancel` (nullable host flag) is polled
 * between blocks; when it reads non-zero the call stops enqueuing and returns
 * OSOR_ERR_CANCELLED. Replaces ModelBackend::decode / NativeModel::decode_checked
 * -> VaeDecoder::forward (src/pipeline.rs:66-67, src/native.rs:525-533,
 * src/native/vae_decoder.rs:104-114). */
int osor_vae_decode(const osor_vae* vae, const float* latents, float* image, int batch,
                    int latent_h, int latent_w, void* workspace, size_t workspace_bytes,
                    void* stream, const volatile int* cancel);

/* Encodes a normalized image [B][3][H][W] f32 in [-1, 1] (device) into raw
 * posterior moments [B][8][H/8][W/8] f32 (device). Replaces
 * ModelBackend::encode_moments / NativeModel::encode_moments_checked ->
 * VaeEncoder::forward (src/pipeline.rs:57, src/native.rs:487-501,
 * src/native/vae_encoder.rs:414-424). */
int osor_vae_encode_moments(const osor_vae* vae, const float* image, float* moments, int batch,
                            int height, int width, void* workspace, size_t workspace_bytes,
                            void* stream, const volatile int* cancel);

/* Host-side weight repack: w_oihw [Cout][Cin][k][k] f32 -> out (host,
 * Cout*k*k*Cin 16-bit patterns of `dtype`) in [Cout][ky][kx][Cin] order, the
 * layout osor_conv2d reads. Replaces the weight side of conv2d()
 * (src/native/conv.rs:149-182). */
int osor_pack_conv_weight(const float* w_oihw, uint16_t* out, int cout, int cin, int ksize,
                          int dtype);

/* 2-D convolution, square kernel, `pad` zero rows / columns before the first
 * and `pad_end` after the last (symmetric: pad_end = pad; the encoder's
 * downsampler, which pads one zero column / row on the right / bottom and then
 * convolves with stride 2 and no padding, is pad = 0, pad_end = 1). Output
 * size (H + pad + pad_end - k) / stride + 1. `dtype` (BF16 / F16) is the type
 * of the packed weight, the residual and any NHWC operand; in/out layout:
 * OSOR_LAYOUT_NHWC (16-bit) or OSOR_LAYOUT_NCHW (f32). bias f32 [Cout]
 * (nullable); residual NHWC [B][Ho][Wo][Cout] (nullable, NHWC output only) is
 * added after the bias. Tensor cores are used when the input is NHWC,
 * Cin % 64 == 0, the output tiles into 128-pixel blocks and either the output
 * is NHWC with Cout % 128 == 0 or NCHW f32 with Cout <= 16; other shapes run
 * a CUDA-core direct convolution. Replaces
 * BandedConv2d::forward_checked + add_bias (src/native/conv.rs:54-145) and the
 * residual add of Resnet::forward_checked (src/native/vae_encoder.rs:150). */
int osor_conv2d(const void* x, void* y, const void* weight_packed, const float* bias,
                const void* residual, int batch, int in_h, int in_w, int cin, int cout, int ksize,
                int stride, int pad, int pad_end, int in_layout, int out_layout, int dtype,
                void* stream);

/* Device workspace for osor_group_norm_silu (0: unsupported shape). */
size_t osor_group_norm_workspace_size(int batch, int channels, int height, int width, int layout,
                                      int dtype);

/* GroupNorm(32 groups) with optional SiLU, y = silu((x - mean) / sqrt(var +
 * eps) * gamma + beta) with fp32 statistics. OSOR_LAYOUT_NCHW (dtype F32,
 * BF16 or F16) runs one fused kernel that keeps each chunk of a group on chip
 * between the statistics and the normalization; OSOR_LAYOUT_NHWC (BF16 / F16)
 * runs the statistics / apply kernels used between convolutions. gamma/beta:
 * device f32 [C]. stats (nullable, device f32 [B*32][2]) receives (mean,
 * biased variance) per group. Replaces StableGroupNorm::forward /
 * forward_silu (src/native/vae_encoder.rs:55-105). */
int osor_group_norm_silu(const void* x, void* y, const float* gamma, const float* beta, int batch,
                         int channels, int height, int width, int layout, int dtype, float eps,
                         int silu, float* stats, void* workspace, size_t workspace_bytes,
                         void* stream);

/* GroupNorm(+SiLU) over NCHW tensors for callers that cannot allocate device
 * memory where they run the op, such as a host framework's enqueue callback
 * that owns all allocations or a serving loop that must not call the
 * allocator. It always runs the shared-memory-resident fused NCHW kernel
 * (osor_group_norm_silu may take the L2-resident one for the same shape), so
 * its results match osor_group_norm_silu's to rounding (statistics to 1e-4
 * relative, outputs to one unit in the last place of the 16-bit type). It
 * takes no workspace: the scratch lives in one fixed device array of 397312
 * bytes (32768 chunk partials plus 1024 group counters) that every GPU loading
 * the library keeps until exit. Shapes that need more scratch, and shapes whose
 * groups the fused kernel cannot hold in one wave of resident CTAs (which
 * osor_group_norm_silu still accepts), return OSOR_ERR_INVALID_INPUT before
 * any device work. The call runs on the device that owns x. The first call on
 * a device looks up the array's address with that device current, so make
 * that first call before any stream capture. All calls share the array (each
 * call clears its counters first); calls that overlap on the GPU race and must
 * not be issued. It calls no cudaMalloc / cudaFree. This entry point has no
 * counterpart in the reference. */
int osor_group_norm_silu_noalloc(const void* x, void* y, const float* gamma, const float* beta,
                                 int batch, int channels, int height, int width, int dtype,
                                 float eps, int silu, float* stats, void* stream);

/* Test hook for the device-side bounded waits (no counterpart in the
 * reference, whose own failure tests inject on the host, e.g. the
 * cancel-after-N-checkpoints test of src/native/conv.rs:190-216). Launches
 * the fused NCHW GroupNorm(+SiLU) kernel of osor_group_norm_silu with each
 * group's arrival target one above its chunk count, so every CTA's cross-CTA
 * group wait runs out after wait_ns (1 us .. 1 s) of %globaltimer. The kernel
 * then records code 1 (wait timeout) in the device status word, lets its
 * in-flight loads land and returns; y is left partly unwritten. Nothing
 * faults or traps, and the context stays usable: read the code with
 * osor_device_status(device, 1), then make normal calls. workspace: at least
 * osor_group_norm_workspace_size(..., OSOR_LAYOUT_NCHW, dtype) bytes. */
int osor_test_group_norm_wait_expiry(const void* x, void* y, const float* gamma,
                                     const float* beta, int batch, int channels, int height,
                                     int width, int dtype, unsigned long long wait_ns,
                                     void* workspace, size_t workspace_bytes, void* stream);

/* The statistics half of StableGroupNorm::forward_reference
 * (src/native/vae_encoder.rs:55-75) on 16-bit NHWC x: stats (device f32
 * [B][32][2]) receives each group's (mean, biased variance). With
 * osor_group_norm_apply it lets several GPUs that each hold a row band of one
 * image normalize it together: every band's statistics are gathered and merged
 * by the apply. workspace: osor_group_norm_workspace_size(..., NHWC, dtype). */
int osor_group_norm_stats(const void* x, int batch, int channels, int height, int width,
                          int dtype, float* stats, void* workspace, size_t workspace_bytes,
                          void* stream);

/* The normalization half (vae_encoder.rs:76-80, plus SiLU when `silu`, :103)
 * on 16-bit NHWC x -> y with statistics merged from `parts` sets part_stats
 * (device f32 [parts][B][32][2], each set over the same number of elements,
 * as osor_group_norm_stats writes them for equal bands): mean = mean of the
 * means, variance = mean of the variances + mean squared deviation of the
 * means. workspace: at least B * C * 16 bytes. */
int osor_group_norm_apply(const void* x, void* y, const float* gamma, const float* beta,
                          const float* part_stats, int parts, int batch, int channels, int height,
                          int width, int dtype, float eps, int silu, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Posterior and diffusion noise for a [batch, 3, height, width] job from a
 * seed: device tensors [batch, 4, height/8, width/8] of `dtype` (F32, F16 or
 * BF16), stream 0 into `posterior` and stream 1 into `diffusion`, bit-equal
 * in F32 to the reference's stored-seed contract version 1 (xoshiro256**
 * streams seeded by SplitMix64, Box-Muller pairs in f64 rounded to F32, NCHW
 * order). batch 1..4; height and width multiples of 8 in 32..1024. The first
 * call on a device copies an 88 KB jump table to it synchronously, so make it
 * before any stream capture. Replaces seeded_noise (src/noise.rs:107-146). */
int osor_seeded_noise(unsigned long long seed, int batch, int height, int width, int dtype,
                      void* posterior, void* diffusion, void* stream);

/* DDPM scheduler (src/scheduler.rs:128-340) and the latent-space stages of
 * the inference pipeline around the VAE (src/pipeline.rs:720-860), in F32.
 * Products and sums are rounded one by one, as the reference evaluates them.
 *
 * osor_scheduler_alphas: host function; alphas_cumprod receives
 * num_train_timesteps cumulative alphas (beta_schedule 0 = linear,
 * 1 = scaled_linear; trained_betas nullable) computed as Scheduler::new does
 * (scheduler.rs:128-221). */
int osor_scheduler_alphas(int num_train_timesteps, double beta_start, double beta_end,
                          int beta_schedule, const double* trained_betas, float* alphas_cumprod);

/* original * sqrt(a) + noise * sqrt(1 - a) over n device floats
 * (Scheduler::add_noise, scheduler.rs:278-297). */
int osor_scheduler_add_noise(const float* original, const float* noise, float* out, long long n,
                             float alpha_t, void* stream);

/* Predicted original sample (scheduler.rs:299-339); prediction_type 0 =
 * epsilon, 1 = sample, 2 = v_prediction; clamped to +-clip_range when
 * clip_sample. */
int osor_scheduler_predicted_original(const float* noisy, const float* model_output, float* out,
                                      long long n, float alpha_t, int prediction_type,
                                      int clip_sample, float clip_range, void* stream);

/* The encoder's input: normalized = image * 2 - 1 over [B][3][H][W]
 * (pipeline.rs:721). */
int osor_pipeline_normalize_image(const float* image, float* normalized, int batch, int height,
                                  int width, void* stream);

/* Stages before the denoiser (pipeline.rs:733-771): from the encoder's
 * moments [B][8][h][w], posterior / diffusion noise [B][4][h][w] and the mask
 * [B][1][H][W] (h = H/8, w = W/8), the UNet input [B][9][h][w] = (noisy
 * latent, max-pooled mask, original latent); sample [B][4][h][w] (nullable)
 * receives the posterior sample. alpha_t = alphas_cumprod[timestep]. */
int osor_pipeline_prepare(const float* moments, const float* posterior_noise,
                          const float* diffusion_noise, const float* mask, float* unet_input,
                          float* sample, int batch, int height, int width, float alpha_t,
                          double vae_scaling_factor, void* stream);

/* Stages after the denoiser (pipeline.rs:810-836): from its output
 * [B][5][h][w] and the UNet input, latent_alpha = sigmoid(channel 4)
 * [B][1][h][w], the predicted original and the alpha blend (both nullable,
 * [B][4][h][w]), and the decoder's input latents = blend / scaling. */
int osor_pipeline_finish(const float* unet_output, const float* unet_input, float* latent_alpha,
                         float* predicted, float* blend, float* latents, int batch, int height,
                         int width, float alpha_t, int prediction_type, int clip_sample,
                         float clip_range, double vae_scaling_factor, void* stream);

/* Display mapping (pipeline.rs:846-856, 862-896): image = clamp(0.5 decoded
 * + 0.5, 0, 1) [B][3][H][W]; alpha = bilinear 8x (align_corners = false) of
 * latent_alpha, [B][1][H][W]. */
int osor_pipeline_map(const float* decoded, const float* latent_alpha, float* image, float* alpha,
                      int batch, int height, int width, void* stream);

/* Nearest 2x upsample of 16-bit NHWC [B][H][W][C] -> [B][2H][2W][C], C % 8 == 0.
 * Replaces upsample_2x (src/native/vae_decoder.rs:18-35). */
int osor_upsample_2x(const void* x, void* y, int batch, int height, int width, int channels,
                     void* stream);

/* Device workspace for osor_attention. */
size_t osor_attention_workspace_size(int batch, int tokens, int dim);

/* out = softmax(q k^T) v per batch entry. q, k, v: device 16-bit (`dtype`)
 * [B][N][D] with row stride ld (elements, >= D), already scaled as the caller
 * wants (the VAE scales q and k by D^-1/4 each); out: [B][N][D]. Softmax
 * statistics are fp32. Replaces attend (src/native/attention.rs:10-25) for the
 * VAE mid-block attention (src/native/vae_encoder.rs:320-327). */
int osor_attention(const void* q, const void* k, const void* v, void* out, int batch, int tokens,
                   int dim, long long ld, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream);

/* Device workspace for osor_attention_kv. */
size_t osor_attention_kv_workspace_size(int batch, int n_q, int n_kv, int dim);

/* out = softmax(q k^T) v per batch entry with n_q query rows (row stride ld_q)
 * against n_kv key / value rows (row stride ld_kv); out: [B][n_q][D]
 * contiguous. The row band of one image on one GPU attends to the keys and
 * values gathered from every band. Replaces attend (src/native/attention.rs
 * :10-25), whose q and k already allow different row counts. */
int osor_attention_kv(const void* q, long long ld_q, const void* k, const void* v, long long ld_kv,
                      void* out, int batch, int n_q, int n_kv, int dim, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- UNet
 * Ops of the SDXL inpainting UNet (src/native.rs:112-379) beyond the VAE set.
 * Pixel tensors are 16-bit NHWC rows (`dtype` BF16 / F16, 16-byte aligned);
 * the convolutions, GroupNorm(+SiLU) (eps 1e-5 in resnets, 1e-6 before the
 * transformers) and the linear projections over pixels (1x1 osor_conv2d) are
 * the VAE entry points above. */

/* features (device f32 [B][base_channels + pooled_width + 6 * time_projection])
 * receives per batch entry the sinusoidal projection (cosines first) of
 * `timestep`, the pooled prompt embedding (device f32 [pooled_width], the same
 * for every entry) and the projections of the six time ids (device f32
 * [B][6]): the inputs of the time and added embeddings of Unet::forward
 * (src/native.rs:318-335). */
int osor_unet_time_features(const float* time_ids, const float* pooled, int batch, int timestep,
                            int base_channels, int time_projection, int pooled_width,
                            float* features, void* stream);

/* y[r][o] = sum_k act(x[r][k]) * w[o][k] + bias[o] + bias2[o] for 1..8 rows
 * (act = SiLU when pre_silu, else identity); x, y device f32, w 16-bit
 * [out][in] of `dtype`, bias / bias2 device f32 (nullable); rows * in <=
 * 12288. Replaces the TimestepEmbedding linears and the resnets'
 * time_emb_proj(silu(temb)) (src/native/resnet.rs:104-110): with every
 * resnet's projection stacked in one weight, one call gives all time biases. */
int osor_rows_linear(const float* x, int rows, int in_features, const void* weight,
                     const float* bias, const float* bias2, int out_features, int pre_silu,
                     int dtype, float* y, void* stream);

/* LayerNorm over the last axis of [rows][channels] (channels % 8 == 0, at most
 * 2048) with f32 statistics and f32 gamma / beta (all four pointers 16-byte
 * aligned). Replaces the transformer
 * blocks' nn::LayerNorm (src/native/spatial.rs:171-173). */
int osor_layer_norm(const void* x, void* y, const float* gamma, const float* beta, long long rows,
                    int channels, float eps, int dtype, void* stream);

/* y[r][f] = x[r][f] * gelu_erf(x[r][features + f]) for x [rows][2 * features]
 * (features % 8 == 0). Replaces FeedForward's exact-erf GEGLU gate
 * (src/native/transformer.rs:17-23). */
int osor_geglu(const void* x, void* y, long long rows, int features, int dtype, void* stream);

/* Column matrix of a thin-input k x k convolution (zero padding pad, stride
 * 1): x NCHW f32 [B][cin][H][W] -> cols 16-bit [B][H][W][ncols] (ncols 64 or
 * 128, k * k * cin <= ncols) with column (ky * k + kx) * cin + ci = x[b][ci]
 * [y + ky - pad][x + kx - pad] (zero outside the image) and the columns past
 * k * k * cin zero, so that the convolution is a 1x1 tensor-core product
 * over ncols input channels (the UNet's conv_in: 9 channels, 81 taps).
 * Replaces the column fill of conv2d_checked for thin inputs
 * (src/native/columns.rs:42-75, 297-368). */
int osor_thin_columns(const float* x, void* cols, int batch, int cin, int height, int width,
                      int ksize, int pad, int ncols, int dtype, void* stream);

/* FeedForward's input projection and GEGLU gate in one call: y[p][f] =
 * value * gelu_erf(gate) with (value, gate) = the 1x1 product x W^T + bias,
 * x NHWC [B][H][W][cin] 16-bit, y [B][H][W][features] 16-bit (features %
 * 128 == 0). weight_packed holds the projection's 2 * features rows
 * (osor_pack_conv_weight's layout) reordered per 128 features: rows t * 256 ..
 * t * 256 + 127 are value rows t * 128 .. t * 128 + 127 and the next 128 rows
 * the matching gate rows features + t * 128 ..; bias f32 [2 * features]
 * (nullable) in the same order. Shapes the CTA-pair kernel takes apply the
 * gate in the product's epilogue and need no workspace; others need
 * osor_linear_geglu_workspace_size bytes (the product is stored there and
 * gated in a second pass). Replaces FeedForward::forward's gate linear,
 * narrow and gelu_erf product (src/native/transformer.rs:18-24). */
size_t osor_linear_geglu_workspace_size(int batch, int height, int width, int cin, int features,
                                        int dtype);
int osor_linear_geglu(const void* x, void* y, const void* weight_packed, const float* bias,
                      int batch, int height, int width, int cin, int features, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream);

/* y[p] = (a[p], b[p]) for NHWC a [P][ca], b [P][cb] (ca, cb % 8 == 0).
 * Replaces Tensor::cat(&[xs, skip], 1) of the up blocks
 * (src/native/unet_blocks.rs:214-219, src/native/cross_blocks.rs:206). */
int osor_concat_channels(const void* a, int ca, const void* b, int cb, void* y, long long pixels,
                         int dtype, void* stream);

/* Nearest resize of NHWC [B][H][W][C] to [B][out_h][out_w][C] (C % 8 == 0),
 * source index min(n - 1, floor(i * (n / out))) in f64. Replaces
 * upsample_nearest2d to the next skip's size (src/native/unet_blocks.rs:222-235,
 * src/native.rs:356-367). */
int osor_resize_nearest(const void* x, void* y, int batch, int in_h, int in_w, int out_h,
                        int out_w, int channels, int dtype, void* stream);

/* y[b][p][c] = x[b][p][c] + image_bias[b * bias_stride + c] + residual[b][p][c]
 * for c < channels, with x rows of stride ld_x (>= channels, % 8 == 0) and y /
 * residual rows of `channels` (% 8 == 0); image_bias device f32 (16-byte
 * aligned, bias_stride % 4 == 0) and residual nullable. x == y (in place)
 * needs ld_x == channels. Adds a resnet's per-image time bias after conv1
 * (src/native/resnet.rs:104-110), and narrows a convolution computed with
 * zero-padded output channels. */
int osor_channel_update(const void* x, long long ld_x, void* y, int channels, int batch,
                        long long pixels_per_image, const float* image_bias,
                        long long bias_stride, const void* residual, int dtype, void* stream);

/* Multi-head out = softmax(q k^T) v per head with f32 scores and softmax:
 * head h of query row i of batch entry b reads q + b*q_batch_stride + i*ld_q +
 * h*head_dim (already scaled, e.g. by head_dim^-1/2), keys / values at
 * k / v + b*kv_batch_stride + j*ld_kv + h*head_dim, and writes out +
 * b*out_batch_stride + i*ld_out + h*head_dim. Strides in elements, multiples
 * of 8; kv_batch_stride 0 shares one key / value set (the fixed prompt) across
 * the batch. head_dim 32, 64 or 128. Replaces SelfAttention and
 * FixedCrossAttention's attend (src/native/spatial.rs:29-46, 83-158). */
int osor_attention_heads(const void* q, long long ld_q, long long q_batch_stride, const void* k,
                         const void* v, long long ld_kv, long long kv_batch_stride, void* out,
                         long long ld_out, long long out_batch_stride, int batch, int heads,
                         int n_q, int n_kv, int head_dim, int dtype, void* stream);

/* The UNet as one handle: weights packed and the prompt's cross-attention
 * keys / values computed at create, one call per denoising step. */
typedef struct osor_unet osor_unet;

/* Architecture fields of the UNet (src/native.rs:51-98; SDXL: channels {320,
 * 640, 1280}, depth {0, 2, 10} (0: a block without transformers), heads {5,
 * 10, 20}, context 2048, pooled 1280, time_projection 256, layers 2) and the
 * model dtype. */
typedef struct osor_unet_config {
  int channels[3];
  int depth[3];
  int heads[3];
  int context;
  int pooled;
  int time_projection;
  int layers;
  int dtype;
} osor_unet_config;

/* Builds the UNet from host float32 tensors with diffusers names and the fixed
 * prompt conditioning: `context` host f32 [tokens][config->context] (1..1024
 * tokens) and `pooled` host f32 [config->pooled]. A missing or misshaped
 * tensor returns OSOR_ERR_INVALID_ARTIFACT. Replaces Unet::new
 * (src/native.rs:127-258) inside NativeModel::new. */
int osor_unet_create(const osor_tensor* tensors, size_t count, const osor_unet_config* config,
                     const float* context, int tokens, const float* pooled, int device,
                     osor_unet** out);
void osor_unet_destroy(osor_unet* unet);

/* One denoising call: input [B][9][h][w] f32 (device), time_ids [B][6] f32
 * (device) -> output [B][5][h][w] f32 (device); B 1..4, h and w 4..128.
 * Activations come from a stream-ordered memory pool owned by the handle;
 * `cancel` (nullable host flag) is polled between blocks and transformer
 * layers. Replaces ModelBackend::denoise / NativeModel::denoise_checked
 * (src/pipeline.rs:54-68, src/native.rs:503-519). */
int osor_unet_denoise(const osor_unet* unet, const float* input, int timestep,
                      const float* time_ids, float* output, int batch, int height, int width,
                      void* stream, const volatile int* cancel);

/* ---- Row-band exchanges over peer memory (NVLink) ------------------------
 * A group of `ranks` processes, one GPU each, decoding one image in row bands
 * exchanges halo rows before each 3x3 convolution and GroupNorm statistics
 * before each normalisation. These entry points do it with peer stores into
 * the neighbours' device memory instead of NCCL calls: each rank creates an
 * arena, the ranks exchange the handles (OSOR_PEER_HANDLE_BYTES each, by any
 * host channel) and open every other rank's; the exchange kernels then take
 * the same arguments every call (their epochs live on the device), so a
 * decode that uses them can be captured in a CUDA graph. Every rank of the
 * group must issue the same exchanges in the same order. The exchange
 * itself has no counterpart in the reference, which runs its row bands one
 * after another on one device (band geometry: src/native/conv.rs:96-108). */
#define OSOR_PEER_HANDLE_BYTES 64
typedef struct osor_peer_group osor_peer_group;

/* Allocates this rank's arena on `device` (halo slots of halo_row_bytes,
 * all-gather slots of gather_bytes, one bulk slot of bulk_bytes per rank for
 * osor_vae_decode_band's attention keys and values, 0 for none) and writes
 * its IPC handle to handle_out. */
int osor_peer_group_create(int device, int ranks, int rank, size_t halo_row_bytes,
                           size_t gather_bytes, size_t bulk_bytes, osor_peer_group** out,
                           void* handle_out);
/* Maps rank `peer`'s arena (its handle from osor_peer_group_create). */
int osor_peer_group_open(osor_peer_group* group, int peer, const void* handle);
/* Waits for the device, unmaps the peers' arenas and frees this rank's (call
 * after every rank has finished its exchanges). */
void osor_peer_group_destroy(osor_peer_group* group);

/* Fills the halo rows of an extended band x [rows + 2][row_bytes] (rows
 * 1..rows are this rank's): row 0 from the rank above's last band row, row
 * rows + 1 from the rank below's first, zeros at the image's top and bottom;
 * this rank's rows 1 and `rows` go to its neighbours. */
int osor_band_halo(osor_peer_group* group, void* x, long long row_bytes, int rows, void* stream);

/* dst[r * bytes ..] = rank r's src for every rank of the group. */
int osor_band_gather(osor_peer_group* group, const void* src, size_t bytes, void* dst,
                     void* stream);

/* Row-band decode of one image on one rank of a peer group: sizes of the
 * per-call workspace, of the group's halo slots (halo_row_bytes) and of its
 * bulk slots (bulk_bytes) for `ranks` ranks and [1, 4, latent_h, latent_w]
 * latents (latent_h a multiple of ranks, bands of at least two rows). */
int osor_vae_decode_band_sizes(const osor_vae* vae, int ranks, int latent_h, int latent_w,
                               size_t* workspace_bytes, size_t* halo_row_bytes,
                               size_t* bulk_bytes);

/* The decoder over this rank's latent rows [r R, (r + 1) R), R = latent_h /
 * ranks, with halo rows, GroupNorm statistics and the mid-block attention's
 * keys and values exchanged with the group's other ranks over peer memory.
 * latents: the whole image's f32 NCHW [1, 4, latent_h, latent_w] on this
 * rank's device; image_band: this rank's rows of the raw decoded image, f32
 * NCHW [1, 3, 8 R, 8 latent_w]. Every rank of the group calls it together.
 * Replaces VaeDecoder::forward (src/native/vae_decoder.rs:104-114) for one
 * image spread over GPUs in the row-band geometry of src/native/conv.rs
 * :96-108. */
int osor_vae_decode_band(const osor_vae* vae, osor_peer_group* group, const float* latents,
                         float* image_band, int latent_h, int latent_w, void* workspace,
                         size_t workspace_bytes, void* stream);

/* One profiled op: kind ("conv_tc", "conv_direct", "groupnorm", ...),
 * algorithmic FLOPs and bytes, device time between the CUDA events recorded
 * on its stream, and the number of kernels it launched. */
typedef struct osor_profile_entry {
  char kind[32];
  double flops;
  double bytes;
  float ms;
  int launches;
} osor_profile_entry;

/* Starts recording CUDA events around every op this thread enqueues. Nothing
 * synchronises while recording. Replaces the per-stage timing of
 * Osor::infer_profiled (src/runtime.rs:514-540). */
void osor_profile_begin(void);

/* Stops recording, waits for the recorded events and writes up to
 * max_entries records (the total goes to *count). */
int osor_profile_end(osor_profile_entry* entries, int max_entries, int* count);

/* Number of kernels this library has launched in this process. */
long long osor_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* OSOR_B200_H */
