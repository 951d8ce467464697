// gdn_fused_block_noalloc: the fused block with its scratch in a static
// device array, for callers that cannot allocate device memory (see the
// declaration in gdn_api.h for who they are and the limits).
#include <mutex>

#include "gdn_common.cuh"

namespace {

// The scratch.  Host code must not pass `g_noalloc_scratch` itself to a
// kernel: in host code that name is a host-side stand-in, not a device
// address.  Its device address is looked up per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GDN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once
// per device with that device current.
gdn_status scratch_on_current_device(void** addr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return gdn::set_error(GDN_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return gdn::set_error(GDN_EUNSUPPORTED, "device ordinal %d is beyond the %d supported", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return gdn::set_error(GDN_ECUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", dev,
                            cudaGetErrorString(e));
    g_scratch_addr[dev] = ptr;
  }
  *addr = g_scratch_addr[dev];
  return GDN_OK;
}

}  // namespace

extern "C" gdn_status gdn_fused_block_noalloc(const gdn_block_args* args, gdn_stream_t stream) {
  if (!args) return gdn::set_error(GDN_EINVAL, "args is NULL");
  gdn_block_args a = *args;
  a.workspace = nullptr;
  a.workspace_bytes = 0;
  size_t need = 0;
  gdn_status st = gdn_block_workspace_size(&a, &need);
  if (st != GDN_OK) return st;
  if (need > (size_t)GDN_NOALLOC_SCRATCH_BYTES)
    return gdn::set_error(GDN_EUNSUPPORTED,
                          "gdn_fused_block_noalloc: this call needs %zu bytes of scratch but the static scratch "
                          "holds %zu (GDN_NOALLOC_SCRATCH_BYTES); split it into calls over fewer tokens",
                          need, (size_t)GDN_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  st = scratch_on_current_device(&scratch);
  if (st != GDN_OK) return st;
  a.workspace = scratch;
  a.workspace_bytes = GDN_NOALLOC_SCRATCH_BYTES;
  return gdn_fused_block(&a, stream);
}
