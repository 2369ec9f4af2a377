// Status reporting shared by every C-ABI entry point.
#include <atomic>
#include "common.cuh"

namespace cvhrf {
static thread_local int g_last_cuda_error = 0;
void set_last_cuda_error(int err) { g_last_cuda_error = err; }
static std::atomic<unsigned long long> g_launches{0};
void count_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
}  // namespace cvhrf

extern "C" const char* cvhrf_status_string(int status) {
  switch (status) {
    case CVHRF_OK: return "ok";
    case CVHRF_EINVAL: return "invalid argument";
    case CVHRF_EWORKSPACE: return "workspace too small";
    case CVHRF_ECUDA: return "CUDA runtime error";
    case CVHRF_EUNSUPPORTED: return "unsupported size";
    default: return "unknown status";
  }
}

extern "C" int cvhrf_last_cuda_error(void) { return cvhrf::g_last_cuda_error; }

extern "C" int cvhrf_version(void) { return 100; }

extern "C" unsigned long long cvhrf_kernel_launch_count(void) { return cvhrf::g_launches.load(); }
