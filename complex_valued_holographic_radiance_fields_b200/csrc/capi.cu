// Status reporting shared by every C-ABI entry point.
#include "common.cuh"

namespace cvhrf {
static thread_local int g_last_cuda_error = 0;
void set_last_cuda_error(int err) { g_last_cuda_error = err; }
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
