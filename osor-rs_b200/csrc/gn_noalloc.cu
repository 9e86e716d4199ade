// GroupNorm(+SiLU) over NCHW tensors without any device allocation.
//
// Some callers cannot allocate device memory at the point where they run the
// op: a host framework's enqueue callback that owns every allocation and
// forbids new ones, or a serving loop that plans all memory up front and must
// not touch the allocator while it runs. For them this entry point keeps the
// fused kernel's scratch (one arrival counter per group and three floats per
// chunk of a group) in a fixed array in device memory that the library
// declares once. Every GPU that loads the library holds the array until the
// process exits.
//
// The call runs on the device that owns x (made current for the call, then
// restored), like osor_group_norm_silu, so the scratch it uses is that
// device's copy of the array.
//
// The array has a fixed size (kNoAllocScratchBytes); shapes whose scratch
// does not fit are rejected before any device work. The first call on a
// device looks up the array's device address (cudaGetSymbolAddress) with that
// device current; that first call should therefore come before any stream
// capture. All calls share the one array and it keeps the last call's
// contents: the arrival counters are cleared at the start of every call and
// the per-chunk partials are rewritten before they are read, so a call does
// not depend on what an earlier call left behind. Two calls whose kernels
// overlap on the GPU (different streams without ordering) race on the array
// and must not be issued.
#include <mutex>
#include <string>

#include "../../include/osor_b200.h"
#include "common.cuh"
#include "device_guard.h"
#include "groupnorm.h"

namespace osor {
// Sets the message osor_last_error_message() returns on this thread.
void set_last_error(const std::string& msg);
}  // namespace osor

namespace osor {
namespace {

// 32768 chunk partials (3 floats each) plus 1024 group counters: enough for
// batch 4 of the largest standalone shape, [*, 128, 1024, 1024] in 16-bit
// (4 * 32 groups * 171 chunks of 48 KiB = 21888 partials).
constexpr size_t kNoAllocScratchBytes = 32768 * 3 * sizeof(float) + 1024 * sizeof(int);

static __device__ __align__(256) unsigned char g_gn_noalloc_scratch[kNoAllocScratchBytes];

void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device (looked up once
// per device). Returns the CUDA error of the lookup.
cudaError_t scratch_address(void** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[device]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_gn_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return cudaSuccess;
}

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

}  // namespace
}  // namespace osor

extern "C" {

int osor_group_norm_silu_noalloc(const void* x, void* y, const float* gamma, const float* beta,
                                 int batch, int channels, int height, int width, int dtype,
                                 float eps, int silu, float* stats, void* stream) {
  using namespace osor;
  if (!x || !y || !gamma || !beta) return fail(OSOR_ERR_INVALID_INPUT, "null argument");
  if (batch <= 0 || height <= 0 || width <= 0 || channels <= 0 || channels % 32 != 0)
    return fail(OSOR_ERR_INVALID_INPUT, "VAE group normalization requires channels divisible by 32");
  if (dtype != OSOR_DTYPE_F32 && dtype != OSOR_DTYPE_BF16 && dtype != OSOR_DTYPE_F16)
    return fail(OSOR_ERR_INVALID_INPUT, "dtype must be F32, BF16 or F16");
  const long long spatial = (long long)height * width;
  const int eb = dtype == OSOR_DTYPE_F32 ? 4 : 2;
  const GnFusedPlan plan = gn_fused_plan(batch, channels, spatial, 32, eb);
  if (!plan.feasible)
    return fail(OSOR_ERR_INVALID_INPUT,
                "osor_group_norm_silu_noalloc runs only the shared-memory-resident kernel, and "
                "a group of this shape needs more chunks than one wave of its resident CTAs; "
                "osor_group_norm_silu (with a workspace) takes such shapes");
  if (plan.workspace_bytes > kNoAllocScratchBytes)
    return fail(OSOR_ERR_INVALID_INPUT,
                "shape needs " + std::to_string(plan.workspace_bytes) +
                    " bytes of scratch; the fixed no-allocation scratch holds " +
                    std::to_string(kNoAllocScratchBytes));
  // The scratch lookup and the launch both run on the device that owns x, as
  // the workspace entry point does: a stream of x's device and x's own copy of
  // the array, whichever device the calling thread had current.
  DeviceOf dev(x);
  void* scratch = nullptr;
  cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess) return fail(OSOR_ERR_CUDA, std::string("scratch lookup: ") + cudaGetErrorString(e));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == OSOR_DTYPE_F32)
    e = gn_fused_launch<float>(static_cast<const float*>(x), static_cast<float*>(y), gamma, beta,
                               batch, channels, spatial, 32, eps, silu, scratch, stats, s);
  else if (dtype == OSOR_DTYPE_BF16)
    e = gn_fused_launch<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                       static_cast<__nv_bfloat16*>(y), gamma, beta, batch, channels,
                                       spatial, 32, eps, silu, scratch, stats, s);
  else
    e = gn_fused_launch<__half>(static_cast<const __half*>(x), static_cast<__half*>(y), gamma, beta,
                                batch, channels, spatial, 32, eps, silu, scratch, stats, s);
  if (e != cudaSuccess) return fail(OSOR_ERR_CUDA, std::string("group norm: ") + cudaGetErrorString(e));
  return OSOR_OK;
}

}  // extern "C"
