// Chunked (WY/UT, chunk 64) prefill on the tensor cores.
#include "gdn_common.cuh"

namespace gdn {

// Error word written by bounded device-side waits (0 = no error).
__device__ unsigned g_device_error = 0;

bool chunked_supported(const ScanParams&) { return false; }
size_t chunked_workspace_bytes(const ScanParams&) { return 0; }
cudaError_t launch_chunked_scan(const ScanParams&, cudaStream_t) { return cudaErrorNotSupported; }

cudaError_t read_and_clear_device_error(unsigned* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (*code) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned));
  }
  return e;
}

}  // namespace gdn
