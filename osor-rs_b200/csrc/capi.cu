// extern "C" entry points declared in include/osor_b200.h.
#include <cmath>
#include <cstring>
#include <string>

#include "common.cuh"
#include "conv_tc.h"
#include "device_guard.h"
#include "groupnorm.h"
#include "noise.h"
#include "pipeline.h"
#include "ops.h"
#include "peer.h"
#include "profile.h"
#include "unet.h"
#include "unet_model.h"
#include "vae.h"

struct osor_vae {
  osor::Vae* impl;
};

struct osor_unet {
  osor::Unet* impl;
};

struct osor_peer_group {
  osor::PeerGroup* impl;
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
int report(const osor::Status& s) {
  if (s.good()) return OSOR_OK;
  return fail(s.code, s.message);
}
int cuda_fail(cudaError_t e, const char* what) {
  return fail(OSOR_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool is16(int dtype) { return dtype == OSOR_DTYPE_BF16 || dtype == OSOR_DTYPE_F16; }
int internal_dtype(int dtype) { return dtype == OSOR_DTYPE_F16 ? osor::kF16 : osor::kBf16; }

using osor::DeviceOf;

}  // namespace

namespace osor {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace osor

extern "C" {

const char* osor_last_error_message(void) { return g_last_error.c_str(); }

int osor_version(void) { return 100; }

int osor_device_check(int device) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(OSOR_ERR_UNAVAILABLE, "no CUDA device " + std::to_string(device));
  }
  cudaDeviceProp prop;
  if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
    return cuda_fail(e, "device properties");
  if (prop.major != 10 || prop.minor != 0)
    return fail(OSOR_ERR_UNAVAILABLE, std::string("device ") + prop.name +
                                          " is not sm_100; this library is built for sm_100a");
  return OSOR_OK;
}

int osor_device_status(int device, int reset) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int value = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&value, osor::g_device_status, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(osor::g_device_status, &zero, sizeof(int));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return -cuda_fail(e, "device status");
  return value;
}

int osor_vae_create(const osor_tensor* tensors, size_t count, const osor_vae_config* config,
                    int device, osor_vae** out) {
  if (!out || (!tensors && count)) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  *out = nullptr;
  int rc = osor_device_check(device);
  if (rc != OSOR_OK) return rc;
  osor::Vae* impl = nullptr;
  osor::Status s = osor::vae_create(tensors, count, config, device, &impl);
  if (!s.good()) return report(s);
  *out = new osor_vae{impl};
  return OSOR_OK;
}

void osor_vae_destroy(osor_vae* vae) {
  if (!vae) return;
  delete vae->impl;
  delete vae;
}

static bool decode_shape_ok(int batch, int h, int w) {
  // Admission rules of the reference pipeline (src/pipeline.rs:71-79): batch
  // 1..=4, image axes 32..=1024 in multiples of 8 -> latent axes 4..=128.
  return batch >= 1 && batch <= 4 && h >= 4 && w >= 4 && h <= 128 && w <= 128;
}
static bool encode_shape_ok(int batch, int h, int w) {
  return batch >= 1 && batch <= 4 && h >= 32 && w >= 32 && h <= 1024 && w <= 1024 && h % 8 == 0 &&
         w % 8 == 0;
}

size_t osor_vae_workspace_size(const osor_vae* vae, int op, int batch, int height, int width) {
  if (!vae) return 0;
  if (op == OSOR_OP_DECODE ? !decode_shape_ok(batch, height, width)
                           : !encode_shape_ok(batch, height, width))
    return 0;
  return osor::vae_workspace_plan(*vae->impl, op, batch, height, width).total;
}

int osor_vae_decode(const osor_vae* vae, const float* latents, float* image, int batch,
                    int latent_h, int latent_w, void* workspace, size_t workspace_bytes,
                    void* stream, const volatile int* cancel) {
  if (!vae || !latents || !image || !workspace)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!decode_shape_ok(batch, latent_h, latent_w))
    return fail(OSOR_ERR_INVALID_INPUT,
                "decode needs batch 1..=4 and latent axes 4..=128 (image axes 32..=1024)");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(vae->impl->device);
  osor::Status s = osor::vae_decode(*vae->impl, latents, image, batch, latent_h, latent_w,
                                    workspace, workspace_bytes,
                                    static_cast<cudaStream_t>(stream), cancel);
  cudaSetDevice(prev);
  return report(s);
}

int osor_vae_decode_band_sizes(const osor_vae* vae, int ranks, int latent_h, int latent_w,
                               size_t* workspace_bytes, size_t* halo_row_bytes,
                               size_t* bulk_bytes) {
  if (!vae || !workspace_bytes || !halo_row_bytes || !bulk_bytes)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!decode_shape_ok(1, latent_h, latent_w))
    return fail(OSOR_ERR_INVALID_INPUT, "band decode needs latent axes 4..=128");
  osor::BandSizes sz;
  osor::Status s = osor::vae_decode_band_sizes(*vae->impl, ranks, latent_h, latent_w, &sz);
  if (!s.good()) return report(s);
  *workspace_bytes = sz.workspace;
  *halo_row_bytes = sz.halo_row_bytes;
  *bulk_bytes = sz.bulk_bytes;
  return OSOR_OK;
}

int osor_vae_decode_band(const osor_vae* vae, osor_peer_group* group, const float* latents,
                         float* image_band, int latent_h, int latent_w, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!vae || !group || !group->impl || !latents || !image_band || !workspace)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!decode_shape_ok(1, latent_h, latent_w))
    return fail(OSOR_ERR_INVALID_INPUT, "band decode needs latent axes 4..=128");
  if (group->impl->device != vae->impl->device)
    return fail(OSOR_ERR_INVALID_INPUT, "the peer group and the model are on different devices");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(vae->impl->device);
  osor::Status s = osor::vae_decode_band(*vae->impl, group->impl, latents, image_band, latent_h,
                                         latent_w, workspace, workspace_bytes,
                                         static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  return report(s);
}

int osor_vae_encode_moments(const osor_vae* vae, const float* image, float* moments, int batch,
                            int height, int width, void* workspace, size_t workspace_bytes,
                            void* stream, const volatile int* cancel) {
  if (!vae || !image || !moments || !workspace)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!encode_shape_ok(batch, height, width))
    return fail(OSOR_ERR_INVALID_INPUT,
                "encode needs batch 1..=4 and image axes 32..=1024 in multiples of 8");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(vae->impl->device);
  osor::Status s = osor::vae_encode(*vae->impl, image, moments, batch, height, width, workspace,
                                    workspace_bytes, static_cast<cudaStream_t>(stream), cancel);
  cudaSetDevice(prev);
  return report(s);
}

int osor_pack_conv_weight(const float* w, uint16_t* out, int cout, int cin, int k, int dtype) {
  if (!w || !out || cout <= 0 || cin <= 0 || k <= 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid weight shape");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "weights must be BF16 or F16");
  for (int co = 0; co < cout; ++co)
    for (int ci = 0; ci < cin; ++ci)
      for (int ky = 0; ky < k; ++ky)
        for (int kx = 0; kx < k; ++kx) {
          const float v = w[(((size_t)co * cin + ci) * k + ky) * k + kx];
          uint16_t bits;
          if (dtype == OSOR_DTYPE_F16) {
            const __half h = __float2half_rn(v);
            std::memcpy(&bits, &h, 2);
          } else {
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            std::memcpy(&bits, &h, 2);
          }
          out[(((size_t)co * k + ky) * k + kx) * cin + ci] = bits;
        }
  return OSOR_OK;
}

int osor_conv2d(const void* x, void* y, const void* weight_packed, const float* bias,
                const void* residual, int batch, int in_h, int in_w, int cin, int cout, int ksize,
                int stride, int pad, int pad_end, int in_layout, int out_layout, int dtype,
                void* stream) {
  if (!x || !y || !weight_packed) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || in_h <= 0 || in_w <= 0 || cin <= 0 || cout <= 0 || ksize <= 0 || stride <= 0 ||
      pad < 0 || pad_end < 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid convolution shape");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "convolution dtype must be BF16 or F16");
  if ((in_layout != OSOR_LAYOUT_NHWC && in_layout != OSOR_LAYOUT_NCHW) ||
      (out_layout != OSOR_LAYOUT_NHWC && out_layout != OSOR_LAYOUT_NCHW))
    return fail(OSOR_ERR_INVALID_INPUT, "convolution layouts must be NHWC (16-bit) or NCHW (f32)");
  if (residual && out_layout != OSOR_LAYOUT_NHWC)
    return fail(OSOR_ERR_INVALID_INPUT, "a residual needs NHWC output");
  if (in_h + pad + pad_end < ksize || in_w + pad + pad_end < ksize)
    return fail(OSOR_ERR_INVALID_INPUT, "convolution input is smaller than its kernel");
  DeviceOf dev(x);
  osor::ConvLayer L;
  L.cin = cin;
  L.cout = cout;
  L.k = ksize;
  L.stride = stride;
  L.pad = pad;
  L.pad_end = pad_end;
  L.w = static_cast<const uint16_t*>(weight_packed);
  L.bias = bias;
  const int in_mode = in_layout == OSOR_LAYOUT_NHWC ? osor::kLayoutNhwc16 : osor::kLayoutNchwF32;
  const int out_mode = out_layout == OSOR_LAYOUT_NHWC ? osor::kLayoutNhwc16 : osor::kLayoutNchwF32;
  return report(osor::run_conv(internal_dtype(dtype), L, x, in_mode, batch, in_h, in_w, cin, y,
                               out_mode, cout, residual, cout, static_cast<cudaStream_t>(stream)));
}

namespace {
// The L2-resident NCHW GroupNorm takes 16-byte-aligned tensors whose H * W is
// a multiple of the vector width; OSOR_GN_NCHW_L2=0 in the environment keeps
// the shared-memory-resident kernel, for comparing.
bool nchw_l2_ok(const void* x, const void* y, int batch, int channels, long long spatial,
                int dtype) {
  static const bool on = [] {
    const char* v = getenv("OSOR_GN_NCHW_L2");
    return !(v && v[0] == '0');
  }();
  const int eb = dtype == OSOR_DTYPE_F32 ? 4 : 2;
  return on && aligned16(x) && aligned16(y) &&
         osor::gn_nchw_l2_plan(batch, channels, spatial, 32, eb).feasible;
}
}  // namespace

size_t osor_group_norm_workspace_size(int batch, int channels, int height, int width, int layout,
                                      int dtype) {
  if (batch <= 0 || channels <= 0 || channels % 32 != 0 || height <= 0 || width <= 0) return 0;
  const long long spatial = (long long)height * width;
  if (layout == OSOR_LAYOUT_NHWC) {
    // Up to 1024 16-byte vectors per pixel (C <= 8192): the wide kernels own
    // four 8-channel columns per thread.
    if (!is16(dtype) || channels / 8 > 1024) return 0;
    return osor::gn_nhwc_plan(batch, channels, spatial, 32).workspace_bytes;
  }
  if (layout != OSOR_LAYOUT_NCHW || (!is16(dtype) && dtype != OSOR_DTYPE_F32)) return 0;
  const int eb = dtype == OSOR_DTYPE_F32 ? 4 : 2;
  // Room for either NCHW kernel: the L2-resident two-pass one (16-byte
  // vectors along H * W) and the shared-memory-resident one.
  const osor::GnFusedPlan p = osor::gn_fused_plan(batch, channels, spatial, 32, eb);
  const osor::GnL2Plan q = osor::gn_nchw_l2_plan(batch, channels, spatial, 32, eb);
  size_t need = 0;
  if (p.feasible) need = p.workspace_bytes;
  if (q.feasible && q.workspace_bytes > need) need = q.workspace_bytes;
  return need;
}

int osor_group_norm_silu(const void* x, void* y, const float* gamma, const float* beta, int batch,
                         int channels, int height, int width, int layout, int dtype, float eps,
                         int silu, float* stats, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!x || !y || !gamma || !beta) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 32 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "VAE group normalization requires channels divisible by 32");
  const size_t need = osor_group_norm_workspace_size(batch, channels, height, width, layout, dtype);
  if (need == 0) return fail(OSOR_ERR_INVALID_INPUT, "unsupported group-norm shape, layout or dtype");
  if (!workspace || workspace_bytes < need)
    return fail(OSOR_ERR_INVALID_INPUT, "group-norm workspace is too small");
  DeviceOf dev(x);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long spatial = (long long)height * width;
  cudaError_t e;
  if (layout == OSOR_LAYOUT_NHWC) {
    if (!aligned16(x) || !aligned16(y))
      return fail(OSOR_ERR_INVALID_INPUT, "NHWC tensors must be 16-byte aligned");
    osor::OpScope scope("groupnorm", 0.0, 4.0 * batch * channels * spatial, s, 3);
    e = osor::gn_nhwc_launch(internal_dtype(dtype), x, y, gamma, beta, batch, channels, spatial, 32,
                             eps, silu, workspace, stats, s);
  } else if (nchw_l2_ok(x, y, batch, channels, spatial, dtype)) {
    osor::note_launches(1);
    // One HBM read and write per element; chunks re-read from L2.
    if (dtype == OSOR_DTYPE_F32)
      e = osor::gn_nchw_l2_launch<float>(static_cast<const float*>(x), static_cast<float*>(y),
                                         gamma, beta, batch, channels, spatial, 32, eps, silu,
                                         workspace, stats, s);
    else if (dtype == OSOR_DTYPE_BF16)
      e = osor::gn_nchw_l2_launch<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                                 static_cast<__nv_bfloat16*>(y), gamma, beta,
                                                 batch, channels, spatial, 32, eps, silu,
                                                 workspace, stats, s);
    else
      e = osor::gn_nchw_l2_launch<__half>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                          gamma, beta, batch, channels, spatial, 32, eps, silu,
                                          workspace, stats, s);
  } else if (dtype == OSOR_DTYPE_F32) {
    osor::note_launches(1);
    e = osor::gn_fused_launch<float>(static_cast<const float*>(x), static_cast<float*>(y), gamma,
                                     beta, batch, channels, spatial, 32, eps, silu, workspace, stats,
                                     s);
  } else if (dtype == OSOR_DTYPE_BF16) {
    osor::note_launches(1);
    e = osor::gn_fused_launch<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                             static_cast<__nv_bfloat16*>(y), gamma, beta, batch,
                                             channels, spatial, 32, eps, silu, workspace, stats, s);
  } else {
    osor::note_launches(1);
    e = osor::gn_fused_launch<__half>(static_cast<const __half*>(x), static_cast<__half*>(y), gamma,
                                      beta, batch, channels, spatial, 32, eps, silu, workspace,
                                      stats, s);
  }
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "group norm");
}

int osor_test_group_norm_wait_expiry(const void* x, void* y, const float* gamma,
                                     const float* beta, int batch, int channels, int height,
                                     int width, int dtype, unsigned long long wait_ns,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !y || !gamma || !beta) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 32 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "VAE group normalization requires channels divisible by 32");
  if (wait_ns < 1000ull || wait_ns > 1000000000ull)
    return fail(OSOR_ERR_INVALID_INPUT, "wait limit must lie in [1 us, 1 s]");
  if (dtype != OSOR_DTYPE_F32 && dtype != OSOR_DTYPE_BF16 && dtype != OSOR_DTYPE_F16)
    return fail(OSOR_ERR_INVALID_INPUT, "dtype must be F32, BF16 or F16");
  const long long spatial = (long long)height * width;
  const osor::GnFusedPlan plan =
      osor::gn_fused_plan(batch, channels, spatial, 32, dtype == OSOR_DTYPE_F32 ? 4 : 2);
  if (!plan.feasible)
    return fail(OSOR_ERR_INVALID_INPUT, "group is too large for the fused kernel's one wave");
  if (!workspace || workspace_bytes < plan.workspace_bytes)
    return fail(OSOR_ERR_INVALID_INPUT, "group-norm workspace is too small");
  DeviceOf dev(x);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  osor::note_launches(1);
  cudaError_t e;
  // One arrival more than the group's chunks: nothing ever provides it.
  if (dtype == OSOR_DTYPE_F32)
    e = osor::gn_fused_launch<float>(static_cast<const float*>(x), static_cast<float*>(y), gamma,
                                     beta, batch, channels, spatial, 32, 1e-6f, 1, workspace,
                                     nullptr, s, 1, wait_ns);
  else if (dtype == OSOR_DTYPE_BF16)
    e = osor::gn_fused_launch<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                             static_cast<__nv_bfloat16*>(y), gamma, beta, batch,
                                             channels, spatial, 32, 1e-6f, 1, workspace, nullptr, s,
                                             1, wait_ns);
  else
    e = osor::gn_fused_launch<__half>(static_cast<const __half*>(x), static_cast<__half*>(y), gamma,
                                      beta, batch, channels, spatial, 32, 1e-6f, 1, workspace,
                                      nullptr, s, 1, wait_ns);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "group norm wait-expiry test");
}

int osor_group_norm_stats(const void* x, int batch, int channels, int height, int width,
                          int dtype, float* stats, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (!x || !stats) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 32 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "VAE group normalization requires channels divisible by 32");
  const size_t need =
      osor_group_norm_workspace_size(batch, channels, height, width, OSOR_LAYOUT_NHWC, dtype);
  if (need == 0) return fail(OSOR_ERR_INVALID_INPUT, "unsupported group-norm shape or dtype");
  if (!workspace || workspace_bytes < need)
    return fail(OSOR_ERR_INVALID_INPUT, "group-norm workspace is too small");
  if (!aligned16(x)) return fail(OSOR_ERR_INVALID_INPUT, "NHWC tensors must be 16-byte aligned");
  DeviceOf dev(x);
  cudaError_t e = osor::gn_nhwc_stats_launch(internal_dtype(dtype), x, batch, channels,
                                             (long long)height * width, 32, workspace, stats,
                                             static_cast<cudaStream_t>(stream));
  osor::note_launches(2);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "group-norm statistics");
}

int osor_group_norm_apply(const void* x, void* y, const float* gamma, const float* beta,
                          const float* part_stats, int parts, int batch, int channels, int height,
                          int width, int dtype, float eps, int silu, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!x || !y || !gamma || !beta || !part_stats)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (parts <= 0) return fail(OSOR_ERR_INVALID_INPUT, "at least one statistics set is needed");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 32 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "VAE group normalization requires channels divisible by 32");
  const size_t need =
      osor_group_norm_workspace_size(batch, channels, height, width, OSOR_LAYOUT_NHWC, dtype);
  if (need == 0) return fail(OSOR_ERR_INVALID_INPUT, "unsupported group-norm shape or dtype");
  if (!workspace || workspace_bytes < (size_t)batch * channels * 4 * sizeof(float))
    return fail(OSOR_ERR_INVALID_INPUT, "group-norm workspace is too small");
  if (!aligned16(x) || !aligned16(y))
    return fail(OSOR_ERR_INVALID_INPUT, "NHWC tensors must be 16-byte aligned");
  DeviceOf dev(x);
  cudaError_t e = osor::gn_nhwc_apply_stats_launch(
      internal_dtype(dtype), x, y, gamma, beta, part_stats, parts, batch, channels,
      (long long)height * width, 32, eps, silu, static_cast<float*>(workspace),
      static_cast<cudaStream_t>(stream));
  osor::note_launches(2);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "group-norm apply");
}

int osor_seeded_noise(unsigned long long seed, int batch, int height, int width, int dtype,
                      void* posterior, void* diffusion, void* stream) {
  if (!posterior || !diffusion) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  auto valid_axis = [](int a) { return a >= 32 && a <= 1024 && a % 8 == 0; };
  if (batch < 1 || batch > 4 || !valid_axis(height) || !valid_axis(width))
    return fail(OSOR_ERR_INVALID_INPUT,
                "seeded noise needs batch 1..=4 and image axes that the model admits");
  if (dtype != OSOR_DTYPE_F32 && dtype != OSOR_DTYPE_F16 && dtype != OSOR_DTYPE_BF16)
    return fail(OSOR_ERR_INVALID_INPUT, "seeded noise dtype must be F32, F16, or BF16");
  DeviceOf dev(posterior);
  const int count = batch * 4 * (height / 8) * (width / 8);
  cudaError_t e = osor::seeded_noise_launch(seed, count, dtype, posterior, diffusion,
                                            static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "seeded noise");
}

int osor_scheduler_alphas(int num_train_timesteps, double beta_start, double beta_end,
                          int beta_schedule, const double* trained_betas, float* alphas_cumprod) {
  if (!alphas_cumprod) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  const int rc = osor::scheduler_alphas(num_train_timesteps, beta_start, beta_end, beta_schedule,
                                        trained_betas, alphas_cumprod);
  if (rc == 1) return fail(OSOR_ERR_INVALID_INPUT, "scheduler: invalid configuration");
  if (rc == 2) return fail(OSOR_ERR_INVALID_INPUT, "scheduler: cumulative alpha underflowed");
  return OSOR_OK;
}

namespace {
bool latent_job_ok(int batch, int height, int width) {
  auto valid_axis = [](int a) { return a >= 32 && a <= 1024 && a % 8 == 0; };
  return batch >= 1 && batch <= 4 && valid_axis(height) && valid_axis(width);
}
bool alpha_ok(float a) { return std::isfinite(a) && a > 0.0f && a <= 1.0f; }
}  // namespace

int osor_pipeline_prepare(const float* moments, const float* posterior_noise,
                          const float* diffusion_noise, const float* mask, float* unet_input,
                          float* sample, int batch, int height, int width, float alpha_t,
                          double vae_scaling_factor, void* stream) {
  if (!moments || !posterior_noise || !diffusion_noise || !mask || !unet_input)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!latent_job_ok(batch, height, width))
    return fail(OSOR_ERR_INVALID_INPUT, "image dimensions or batch exceed limits");
  if (!alpha_ok(alpha_t) || !(vae_scaling_factor > 0.0) || !std::isfinite(vae_scaling_factor))
    return fail(OSOR_ERR_INVALID_INPUT, "invalid cumulative alpha or VAE scaling factor");
  DeviceOf dev(moments);
  cudaError_t e = osor::pipeline_prepare_launch(
      moments, posterior_noise, diffusion_noise, mask, unet_input, sample, batch, height / 8,
      width / 8, (float)vae_scaling_factor, alpha_t, static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "pipeline prepare");
}

int osor_pipeline_finish(const float* unet_output, const float* unet_input, float* latent_alpha,
                         float* predicted, float* blend, float* latents, int batch, int height,
                         int width, float alpha_t, int prediction_type, int clip_sample,
                         float clip_range, double vae_scaling_factor, void* stream) {
  if (!unet_output || !unet_input || !latent_alpha || !latents)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!latent_job_ok(batch, height, width))
    return fail(OSOR_ERR_INVALID_INPUT, "image dimensions or batch exceed limits");
  if (!alpha_ok(alpha_t) || !(vae_scaling_factor > 0.0) || !std::isfinite(vae_scaling_factor))
    return fail(OSOR_ERR_INVALID_INPUT, "invalid cumulative alpha or VAE scaling factor");
  if (prediction_type < 0 || prediction_type > 2)
    return fail(OSOR_ERR_INVALID_INPUT, "unsupported prediction_type");
  if (clip_sample && !(clip_range > 0.0f && std::isfinite(clip_range)))
    return fail(OSOR_ERR_INVALID_INPUT, "invalid clip range");
  DeviceOf dev(unet_output);
  cudaError_t e = osor::pipeline_finish_launch(
      unet_output, unet_input, latent_alpha, predicted, blend, latents, batch, height / 8,
      width / 8, alpha_t, prediction_type, clip_sample, clip_range,
      (float)(1.0 / vae_scaling_factor), static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "pipeline finish");
}

int osor_pipeline_normalize_image(const float* image, float* normalized, int batch, int height,
                                  int width, void* stream) {
  if (!image || !normalized) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!latent_job_ok(batch, height, width))
    return fail(OSOR_ERR_INVALID_INPUT, "image dimensions or batch exceed limits");
  DeviceOf dev(image);
  cudaError_t e = osor::pipeline_normalize_launch(image, normalized, (long long)batch * 3 * height * width,
                                                  static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "pipeline normalize");
}

int osor_pipeline_map(const float* decoded, const float* latent_alpha, float* image, float* alpha,
                      int batch, int height, int width, void* stream) {
  if (!decoded || !latent_alpha || !image || !alpha)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!latent_job_ok(batch, height, width))
    return fail(OSOR_ERR_INVALID_INPUT, "image dimensions or batch exceed limits");
  DeviceOf dev(decoded);
  cudaError_t e = osor::pipeline_map_launch(decoded, latent_alpha, image, alpha, batch, height,
                                            width, static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "pipeline map");
}

int osor_scheduler_add_noise(const float* original, const float* noise, float* out, long long n,
                             float alpha_t, void* stream) {
  if (!original || !noise || !out) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (n <= 0 || n > 16LL * 1024 * 1024)
    return fail(OSOR_ERR_INVALID_INPUT, "scheduler tensor exceeds safety limit");
  if (!alpha_ok(alpha_t)) return fail(OSOR_ERR_INVALID_INPUT, "invalid cumulative alpha");
  DeviceOf dev(original);
  cudaError_t e = osor::scheduler_add_noise_launch(original, noise, out, n, alpha_t,
                                                   static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "scheduler add_noise");
}

int osor_scheduler_predicted_original(const float* noisy, const float* model_output, float* out,
                                      long long n, float alpha_t, int prediction_type,
                                      int clip_sample, float clip_range, void* stream) {
  if (!noisy || !model_output || !out) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (n <= 0 || n > 16LL * 1024 * 1024)
    return fail(OSOR_ERR_INVALID_INPUT, "scheduler tensor exceeds safety limit");
  if (!alpha_ok(alpha_t)) return fail(OSOR_ERR_INVALID_INPUT, "invalid cumulative alpha");
  if (prediction_type < 0 || prediction_type > 2)
    return fail(OSOR_ERR_INVALID_INPUT, "unsupported prediction_type");
  DeviceOf dev(noisy);
  cudaError_t e =
      osor::scheduler_predicted_launch(noisy, model_output, out, n, alpha_t, prediction_type,
                                       clip_sample, clip_range, static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "scheduler predicted_original");
}

int osor_upsample_2x(const void* x, void* y, int batch, int height, int width, int channels,
                     void* stream) {
  if (!x || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "upsample needs positive sizes and channels % 8 == 0");
  if (!aligned16(x) || !aligned16(y))
    return fail(OSOR_ERR_INVALID_INPUT, "tensors must be 16-byte aligned");
  DeviceOf dev(x);
  cudaError_t e = osor::upsample2x_nhwc_launch(x, y, batch, height, width, channels,
                                               static_cast<cudaStream_t>(stream));
  osor::note_launches(1);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "upsample");
}

namespace {
// Softmax scratch of the tensor-core attention: per-row (max, sum) partials
// over column blocks of at least 32 and the row maxima.
size_t attention_stats_bytes(int n_q, int n_kv) {
  return ((size_t)n_q * ((n_kv + 31) / 32) * 8 + (size_t)n_q * 4 + 255) / 256 * 256;
}
}  // namespace

size_t osor_attention_kv_workspace_size(int batch, int n_q, int n_kv, int dim) {
  (void)batch;
  if (n_q <= 0 || n_kv <= 0 || dim <= 0) return 0;
  const size_t a = attention_stats_bytes(n_q, n_kv);
  const size_t b = ((size_t)n_q * n_kv * 2 + 255) / 256 * 256;
  const size_t c = ((size_t)n_q * 4 + 255) / 256 * 256;
  const size_t d = ((size_t)n_kv * dim * 2 + 255) / 256 * 256;
  return a + b + c + d;
}

size_t osor_attention_workspace_size(int batch, int tokens, int dim) {
  return osor_attention_kv_workspace_size(batch, tokens, tokens, dim);
}

int osor_attention_kv(const void* q, long long ld_q, const void* k, const void* v, long long ld_kv,
                      void* out, int batch, int n_q, int n_kv, int dim, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || n_q <= 0 || n_kv <= 0 || dim <= 0 || dim > 512 || ld_q < dim || ld_kv < dim)
    return fail(OSOR_ERR_INVALID_INPUT, "attention tensor shapes are incompatible");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "attention dtype must be BF16 or F16");
  const size_t need = osor_attention_kv_workspace_size(batch, n_q, n_kv, dim);
  if (!workspace || workspace_bytes < need)
    return fail(OSOR_ERR_INVALID_INPUT, "attention workspace is too small");
  DeviceOf dev(q);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  float* scores = reinterpret_cast<float*>(w);
  w += attention_stats_bytes(n_q, n_kv);
  void* probs = w;
  w += ((size_t)n_q * n_kv * 2 + 255) / 256 * 256;
  float* rowsum = reinterpret_cast<float*>(w);
  w += ((size_t)n_q * 4 + 255) / 256 * 256;
  void* vt = w;
  // Batch entries are [n][D] blocks of stride n*ld inside q/k/v.
  osor::Status s;
  const uint16_t* qb = static_cast<const uint16_t*>(q);
  const uint16_t* kb = static_cast<const uint16_t*>(k);
  const uint16_t* vb = static_cast<const uint16_t*>(v);
  uint16_t* ob = static_cast<uint16_t*>(out);
  for (int b = 0; b < batch && s.good(); ++b) {
    const long long oq = (long long)b * n_q * ld_q, okv = (long long)b * n_kv * ld_kv;
    s = osor::attention_core(internal_dtype(dtype), qb + oq, ld_q, kb + okv, vb + okv, ld_kv,
                             ob + (long long)b * n_q * dim, dim, 1, n_q, n_kv, dim, scores, probs,
                             rowsum, vt, static_cast<cudaStream_t>(stream));
  }
  return report(s);
}

int osor_attention(const void* q, const void* k, const void* v, void* out, int batch, int tokens,
                   int dim, long long ld, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return osor_attention_kv(q, ld, k, v, ld, out, batch, tokens, tokens, dim, dtype, workspace,
                           workspace_bytes, stream);
}

// ---------------------------------------------------------------- UNet
int osor_unet_time_features(const float* time_ids, const float* pooled, int batch, int timestep,
                            int base_channels, int time_projection, int pooled_width,
                            float* features, void* stream) {
  if (!time_ids || !features || (pooled_width > 0 && !pooled))
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch < 1 || batch > 8 || timestep < 0 || base_channels < 2 || base_channels % 2 != 0 ||
      time_projection < 2 || time_projection % 2 != 0 || pooled_width < 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid time embedding shape");
  DeviceOf dev(features);
  osor::OpScope scope("time_features", 0.0,
                      4.0 * batch * (base_channels + pooled_width + 6 * time_projection),
                      static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::unet_time_features_launch(
      time_ids, pooled, batch, (float)timestep, base_channels, time_projection, pooled_width,
      features, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "time features");
}

int osor_rows_linear(const float* x, int rows, int in_features, const void* weight,
                     const float* bias, const float* bias2, int out_features, int pre_silu,
                     int dtype, float* y, void* stream) {
  if (!x || !weight || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (rows < 1 || rows > 8 || in_features < 1 || out_features < 1 ||
      (long long)rows * in_features > 12288)
    return fail(OSOR_ERR_INVALID_INPUT, "row linear takes 1..8 rows of at most 12288 values");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "linear weight dtype must be BF16 or F16");
  if (!aligned16(weight)) return fail(OSOR_ERR_INVALID_INPUT, "linear weight must be 16-byte aligned");
  DeviceOf dev(y);
  osor::OpScope scope("rows_linear", 2.0 * rows * in_features * out_features,
                      2.0 * in_features * out_features, static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::rows_linear_launch(internal_dtype(dtype), x, rows, in_features,
                                                 weight, bias, bias2, out_features, pre_silu,
                                                 y, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "row linear");
}

int osor_layer_norm(const void* x, void* y, const float* gamma, const float* beta, long long rows,
                    int channels, float eps, int dtype, void* stream) {
  if (!x || !y || !gamma || !beta) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (rows < 1 || channels < 8 || channels % 8 != 0 || channels > 2048 || !(eps >= 0.0f))
    return fail(OSOR_ERR_INVALID_INPUT, "layer norm needs rows of 8..2048 channels (multiple of 8)");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "layer norm dtype must be BF16 or F16");
  if (!aligned16(x) || !aligned16(y) || !aligned16(gamma) || !aligned16(beta))
    return fail(OSOR_ERR_INVALID_INPUT, "layer norm tensors must be 16-byte aligned");
  DeviceOf dev(x);
  osor::OpScope scope("layernorm", 0.0, 4.0 * rows * channels, static_cast<cudaStream_t>(stream),
                      1);
  const cudaError_t e = osor::layer_norm_launch(internal_dtype(dtype), x, y, gamma, beta, rows,
                                                channels, eps, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "layer norm");
}

int osor_geglu(const void* x, void* y, long long rows, int features, int dtype, void* stream) {
  if (!x || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (rows < 1 || features < 8 || features % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "GEGLU needs a positive multiple of 8 features");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "GEGLU dtype must be BF16 or F16");
  if (!aligned16(x) || !aligned16(y))
    return fail(OSOR_ERR_INVALID_INPUT, "GEGLU tensors must be 16-byte aligned");
  DeviceOf dev(x);
  osor::OpScope scope("geglu", 0.0, 6.0 * rows * features, static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::geglu_launch(internal_dtype(dtype), x, y, rows, features,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "GEGLU");
}

int osor_thin_columns(const float* x, void* cols, int batch, int cin, int height, int width,
                      int ksize, int pad, int ncols, int dtype, void* stream) {
  if (!x || !cols) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || cin <= 0 || height <= 0 || width <= 0 || ksize <= 0 || pad < 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid column-matrix shape");
  if ((ncols != 64 && ncols != 128) || ksize * ksize * cin > ncols)
    return fail(OSOR_ERR_INVALID_INPUT, "the taps x channels must fit 64 or 128 columns");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "column dtype must be BF16 or F16");
  if (!aligned16(cols)) return fail(OSOR_ERR_INVALID_INPUT, "columns must be 16-byte aligned");
  DeviceOf dev(x);
  osor::OpScope scope("thin_columns", 0.0, 4.0 * batch * height * width * cin +
                                               2.0 * ncols * batch * height * width,
                      static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e =
      osor::thin_columns_launch(internal_dtype(dtype), x, cols, batch, cin, height, width, ksize,
                                pad, nullptr, nullptr, static_cast<cudaStream_t>(stream), ncols);
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "column matrix");
}

size_t osor_linear_geglu_workspace_size(int batch, int height, int width, int cin, int features,
                                        int dtype) {
  if (batch <= 0 || height <= 0 || width <= 0 || cin <= 0 || cin % 8 != 0 || features <= 0 ||
      features % 128 != 0 || !is16(dtype))
    return 0;
  return osor::geglu_product_workspace(internal_dtype(dtype), batch, height, width, cin, features);
}

int osor_linear_geglu(const void* x, void* y, const void* weight_packed, const float* bias,
                      int batch, int height, int width, int cin, int features, int dtype,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !y || !weight_packed) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || cin <= 0 || cin % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid GEGLU product shape");
  if (features <= 0 || features % 128 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "GEGLU product needs a positive multiple of 128 features");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "GEGLU product dtype must be BF16 or F16");
  if (!aligned16(x) || !aligned16(y) || !aligned16(weight_packed) || (bias && !aligned16(bias)))
    return fail(OSOR_ERR_INVALID_INPUT, "GEGLU product operands must be 16-byte aligned");
  DeviceOf dev(x);
  return report(osor::run_geglu_product(internal_dtype(dtype),
                                        static_cast<const uint16_t*>(weight_packed), bias, x,
                                        batch, height, width, cin, features, y, workspace,
                                        workspace_bytes, static_cast<cudaStream_t>(stream)));
}

int osor_concat_channels(const void* a, int ca, const void* b, int cb, void* y, long long pixels,
                         int dtype, void* stream) {
  if (!a || !b || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (pixels < 1 || ca < 8 || cb < 8 || ca % 8 != 0 || cb % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "concatenated channel counts must be multiples of 8");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "concatenation dtype must be BF16 or F16");
  if (!aligned16(a) || !aligned16(b) || !aligned16(y))
    return fail(OSOR_ERR_INVALID_INPUT, "concatenated tensors must be 16-byte aligned");
  DeviceOf dev(y);
  osor::OpScope scope("concat", 0.0, 4.0 * pixels * (ca + cb), static_cast<cudaStream_t>(stream),
                      1);
  const cudaError_t e =
      osor::concat_channels_launch(a, ca, b, cb, y, pixels, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "channel concatenation");
}

int osor_resize_nearest(const void* x, void* y, int batch, int in_h, int in_w, int out_h,
                        int out_w, int channels, int dtype, void* stream) {
  if (!x || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch < 1 || in_h < 1 || in_w < 1 || out_h < 1 || out_w < 1 || channels < 8 ||
      channels % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid nearest resize shape");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "resize dtype must be BF16 or F16");
  if (!aligned16(x) || !aligned16(y))
    return fail(OSOR_ERR_INVALID_INPUT, "resized tensors must be 16-byte aligned");
  DeviceOf dev(x);
  osor::OpScope scope("resize", 0.0, 2.0 * batch * channels * ((double)in_h * in_w + (double)out_h * out_w),
                      static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::resize_nearest_launch(x, y, batch, in_h, in_w, out_h, out_w,
                                                    channels, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "nearest resize");
}

int osor_channel_update(const void* x, long long ld_x, void* y, int channels, int batch,
                        long long pixels_per_image, const float* image_bias,
                        long long bias_stride, const void* residual, int dtype, void* stream) {
  if (!x || !y) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch < 1 || pixels_per_image < 1 || channels < 8 || channels % 8 != 0 || ld_x < channels ||
      ld_x % 8 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "invalid channel update shape");
  if (x == y && ld_x != channels)
    return fail(OSOR_ERR_INVALID_INPUT, "an in-place channel update needs ld_x == channels");
  if (image_bias && (bias_stride < channels || bias_stride % 4 != 0))
    return fail(OSOR_ERR_INVALID_INPUT, "image bias rows must hold the channels, stride % 4 == 0");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "channel update dtype must be BF16 or F16");
  if (!aligned16(x) || !aligned16(y) || !aligned16(image_bias) || !aligned16(residual))
    return fail(OSOR_ERR_INVALID_INPUT, "channel update tensors must be 16-byte aligned");
  DeviceOf dev(x);
  osor::OpScope scope("channel_update", 0.0,
                      2.0 * batch * pixels_per_image * channels * (residual ? 3.0 : 2.0),
                      static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::channel_update_launch(internal_dtype(dtype), x, ld_x, y, channels,
                                                    pixels_per_image, batch, image_bias,
                                                    bias_stride, residual,
                                                    static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "channel update");
}

int osor_attention_heads(const void* q, long long ld_q, long long q_batch_stride, const void* k,
                         const void* v, long long ld_kv, long long kv_batch_stride, void* out,
                         long long ld_out, long long out_batch_stride, int batch, int heads,
                         int n_q, int n_kv, int head_dim, int dtype, void* stream) {
  if (!q || !k || !v || !out) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(OSOR_ERR_INVALID_INPUT, "attention head width must be 32, 64 or 128");
  const long long width = (long long)heads * head_dim;
  if (batch < 1 || batch > 65535 || heads < 1 || heads > 65535 || n_q < 1 || n_kv < 1 ||
      ld_q < width || ld_kv < width || ld_out < width)
    return fail(OSOR_ERR_INVALID_INPUT, "attention tensor shapes are incompatible");
  if (batch > 1 && (q_batch_stride < (long long)n_q * ld_q ||
                    out_batch_stride < (long long)n_q * ld_out ||
                    (kv_batch_stride != 0 && kv_batch_stride < (long long)n_kv * ld_kv)))
    return fail(OSOR_ERR_INVALID_INPUT, "attention batch strides overlap");
  if (q_batch_stride < 0 || kv_batch_stride < 0 || out_batch_stride < 0 ||
      ((ld_q | ld_kv | ld_out | q_batch_stride | kv_batch_stride | out_batch_stride) & 7) != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "attention strides must be non-negative multiples of 8");
  if (!is16(dtype)) return fail(OSOR_ERR_INVALID_INPUT, "attention dtype must be BF16 or F16");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(OSOR_ERR_INVALID_INPUT, "attention tensors must be 16-byte aligned");
  DeviceOf dev(q);
  osor::OpScope scope("attn_heads", 4.0 * batch * n_q * (double)n_kv * width,
                      2.0 * batch * width * (2.0 * n_q + (kv_batch_stride ? 2.0 * n_kv : 0.0)) +
                          (kv_batch_stride ? 0.0 : 4.0 * n_kv * width),
                      static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e = osor::attention_heads_launch(
      internal_dtype(dtype), q, ld_q, q_batch_stride, k, v, ld_kv, kv_batch_stride, out, ld_out,
      out_batch_stride, batch, heads, n_q, n_kv, head_dim, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "multi-head attention");
}

int osor_unet_create(const osor_tensor* tensors, size_t count, const osor_unet_config* config,
                     const float* context, int tokens, const float* pooled, int device,
                     osor_unet** out) {
  if (!tensors || !config || !context || !pooled || !out)
    return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  *out = nullptr;
  if (osor_device_check(device) != OSOR_OK) return OSOR_ERR_UNAVAILABLE;
  osor::Unet* impl = nullptr;
  osor::Status s = osor::unet_create(tensors, count, config, context, tokens, pooled, device, &impl);
  if (!s.good()) return report(s);
  *out = new osor_unet{impl};
  return OSOR_OK;
}

void osor_unet_destroy(osor_unet* unet) {
  if (!unet) return;
  osor::unet_destroy(unet->impl);
  delete unet;
}

int osor_unet_denoise(const osor_unet* unet, const float* input, int timestep,
                      const float* time_ids, float* output, int batch, int height, int width,
                      void* stream, const volatile int* cancel) {
  if (!unet || !unet->impl) return fail(OSOR_ERR_INVALID_INPUT, "null UNet handle");
  return report(osor::unet_denoise(*unet->impl, input, timestep, time_ids, output, batch, height,
                                   width, static_cast<cudaStream_t>(stream), cancel));
}

int osor_peer_group_create(int device, int ranks, int rank, size_t halo_row_bytes,
                           size_t gather_bytes, size_t bulk_bytes, osor_peer_group** out,
                           void* handle_out) {
  if (!out || !handle_out) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  *out = nullptr;
  if (osor_device_check(device) != OSOR_OK) return OSOR_ERR_UNAVAILABLE;
  static_assert(OSOR_PEER_HANDLE_BYTES == osor::kPeerHandleBytes, "handle size");
  osor::PeerGroup* g = nullptr;
  if (const char* err = osor::peer_group_create(device, ranks, rank, halo_row_bytes, gather_bytes,
                                                bulk_bytes, &g, handle_out))
    return fail(OSOR_ERR_INVALID_INPUT, err);
  *out = new osor_peer_group{g};
  return OSOR_OK;
}

int osor_peer_group_open(osor_peer_group* group, int peer, const void* handle) {
  if (!group || !group->impl || !handle) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (const char* err = osor::peer_group_open(group->impl, peer, handle))
    return fail(OSOR_ERR_CUDA, err);
  return OSOR_OK;
}

void osor_peer_group_destroy(osor_peer_group* group) {
  if (!group) return;
  osor::peer_group_destroy(group->impl);
  delete group;
}

int osor_band_halo(osor_peer_group* group, void* x, long long row_bytes, int rows, void* stream) {
  if (!group || !group->impl || !x) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!aligned16(x)) return fail(OSOR_ERR_INVALID_INPUT, "band halo: x must be 16-byte aligned");
  if (const char* err = osor::band_halo_check(group->impl, row_bytes, rows))
    return fail(OSOR_ERR_INVALID_INPUT, err);
  DeviceOf dev(x);
  osor::OpScope scope("band_halo", 0.0, 4.0 * row_bytes, static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e =
      osor::band_halo_launch(group->impl, x, row_bytes, rows, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "band halo");
}

int osor_band_gather(osor_peer_group* group, const void* src, size_t bytes, void* dst,
                     void* stream) {
  if (!group || !group->impl || !src || !dst) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (!aligned16(src) || !aligned16(dst))
    return fail(OSOR_ERR_INVALID_INPUT, "band gather: 16-byte aligned buffers");
  if (const char* err = osor::band_gather_check(group->impl, bytes))
    return fail(OSOR_ERR_INVALID_INPUT, err);
  DeviceOf dev(src);
  osor::OpScope scope("band_gather", 0.0, 2.0 * bytes, static_cast<cudaStream_t>(stream), 1);
  const cudaError_t e =
      osor::band_gather_launch(group->impl, src, bytes, dst, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? OSOR_OK : cuda_fail(e, "band gather");
}

}  // extern "C"
