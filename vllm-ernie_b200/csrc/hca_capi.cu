// Status strings and version of the libhca_b200 C ABI.
#include "hca_common.cuh"

extern "C" const char* hca_status_string(int status) {
  switch (status) {
    case HCA_OK: return "ok";
    case HCA_E_INVALID: return "invalid argument (pointer, size, stride or alignment)";
    case HCA_E_UNSUPPORTED: return "shape not instantiated in this build";
    case HCA_E_CUDA: return "CUDA launch error";
    case HCA_E_WORKSPACE: return "workspace too small";
    case HCA_E_TOO_LARGE: return "needs more split-K scratch than HCA_NOALLOC_WORKSPACE_BYTES";
    default: return "unknown status";
  }
}

namespace hca {
const char*& last_cuda_error() {
  thread_local const char* msg = "no CUDA error recorded";
  return msg;
}
}  // namespace hca

extern "C" const char* hca_last_cuda_error(void) { return hca::last_cuda_error(); }

extern "C" int hca_version(void) { return 100; }
