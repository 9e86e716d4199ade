// Per-op CUDA-event profiling and a kernel launch counter.
//
// The reference times its pipeline per stage (Osor::infer_profiled,
// src/runtime.rs:514-540) by synchronising at each stage. Here every op of the
// VAE graph can be bracketed by CUDA events on its stream instead, so nothing
// synchronises inside the timed region; osor_profile_end reads the events.
#pragma once
#include <cuda_runtime.h>

namespace osor {

// Adds n to the process-wide count of kernels launched by this library.
void note_launches(int n);
long long launch_count();

// Records start / end events around one op on `stream` while profiling is
// enabled on the calling thread; no-op otherwise.
class OpScope {
 public:
  OpScope(const char* kind, double flops, double bytes, cudaStream_t stream, int launches);
  ~OpScope();
  OpScope(const OpScope&) = delete;
  OpScope& operator=(const OpScope&) = delete;

 private:
  int index_ = -1;
  cudaStream_t stream_ = nullptr;
};

}  // namespace osor
