// Per-op CUDA-event profiling (see profile.h) and the C ABI that reads it.
#include <atomic>
#include <cstring>
#include <vector>

#include "../../include/osor_b200.h"
#include "profile.h"

namespace osor {
namespace {

std::atomic<long long> g_launches{0};

struct Record {
  const char* kind;
  double flops, bytes;
  int launches;
  cudaEvent_t start, end;
};

struct ThreadProfile {
  bool enabled = false;
  std::vector<Record> records;
  std::vector<cudaEvent_t> pool;  // events reused across sessions
  size_t pool_used = 0;
  cudaEvent_t take() {
    if (pool_used == pool.size()) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
      pool.push_back(e);
    }
    return pool[pool_used++];
  }
};

thread_local ThreadProfile g_profile;

}  // namespace

void note_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

OpScope::OpScope(const char* kind, double flops, double bytes, cudaStream_t stream, int launches)
    : stream_(stream) {
  note_launches(launches);
  ThreadProfile& p = g_profile;
  if (!p.enabled) return;
  Record r{kind, flops, bytes, launches, p.take(), p.take()};
  if (!r.start || !r.end) return;
  cudaEventRecord(r.start, stream);
  index_ = (int)p.records.size();
  p.records.push_back(r);
}

OpScope::~OpScope() {
  if (index_ < 0) return;
  cudaEventRecord(g_profile.records[index_].end, stream_);
}

}  // namespace osor

extern "C" {

void osor_profile_begin(void) {
  osor::ThreadProfile& p = osor::g_profile;
  p.records.clear();
  p.pool_used = 0;
  p.enabled = true;
}

int osor_profile_end(osor_profile_entry* entries, int max_entries, int* count) {
  osor::ThreadProfile& p = osor::g_profile;
  p.enabled = false;
  int n = 0;
  int rc = OSOR_OK;
  for (const osor::Record& r : p.records) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.end) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.end) != cudaSuccess) {
      rc = OSOR_ERR_CUDA;
      ms = -1.0f;
    }
    if (entries && n < max_entries) {
      osor_profile_entry& e = entries[n];
      std::memset(e.kind, 0, sizeof(e.kind));
      std::strncpy(e.kind, r.kind, sizeof(e.kind) - 1);
      e.flops = r.flops;
      e.bytes = r.bytes;
      e.ms = ms;
      e.launches = r.launches;
    }
    ++n;
  }
  if (count) *count = n;
  p.records.clear();
  p.pool_used = 0;
  return rc;
}

long long osor_launch_count(void) { return osor::launch_count(); }

}  // extern "C"
