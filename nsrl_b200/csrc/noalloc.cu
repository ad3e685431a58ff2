// nsrl_linear_i16_i8_i16_noalloc: the linear for callers that cannot allocate
// device memory.
//
// The regular nsrl_linear_i16_i8_i16 asks its caller for a workspace of
// nsrl_linear_workspace_size() bytes (the byte planes of x and their row L1
// norms).  Some callers cannot provide one:
// - a shim that keeps nsrl-core's slice-in / slice-out signature with no
//   workspace argument (the reference's kernels are allocation-free, no_std);
// - a host path that must not call cudaMalloc / cudaFree, because those can
//   synchronise the device or fail under a memory budget that another
//   allocator owns.
// This entry point instead uses g_noalloc_scratch, a file-scope device array
// of NSRL_NOALLOC_SCRATCH_BYTES.  Every GPU that loads the library holds the
// array until the process exits.  Host code cannot use the array's name as a
// device address (it is a host-side stand-in), so the first call on each
// device looks the address up once with cudaGetSymbolAddress, with that
// device current, and caches it per device index; make that first call before
// any stream capture.  The cached address belongs to the device's primary
// context: a cudaDeviceReset after the first call (which unloads the module
// and its array) or a caller-made driver-API context is not supported.  All calls share the array and it keeps the last call's contents:
// the kernels that read it (the linear and the i32 prefix check) only read
// what the split kernel of the same call wrote, so nothing needs clearing.
// Calls that overlap on the GPU (two streams, or two host threads) race on the
// array and must be serialised by the caller.
#include <mutex>

#include "common.cuh"
#include "internal.h"

#define NSRL_NOALLOC_SCRATCH_BYTES (16u << 20)

static __device__ __align__(256) uint8_t g_noalloc_scratch[NSRL_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

}  // namespace

extern "C" {

size_t nsrl_linear_noalloc_scratch_bytes(void) { return NSRL_NOALLOC_SCRATCH_BYTES; }

nsrl_status nsrl_linear_i16_i8_i16_noalloc(const int16_t* x, size_t rows, const nsrl_linear_params* params,
                                           int16_t* y, nsrl_device_status* status, void* stream) {
  if (!params || params->input_dim == 0 || params->output_dim == 0) {
    nsrl::set_error("invalid shape: linear params");
    return NSRL_INVALID_SHAPE;
  }
  const size_t need = nsrl_linear_workspace_size(rows, params->input_dim, params->output_dim);
  if (need > NSRL_NOALLOC_SCRATCH_BYTES) {
    nsrl::set_error(
        "invalid shape: %zu rows x %zu inputs need %zu bytes of scratch, above the %u-byte static scratch of "
        "nsrl_linear_i16_i8_i16_noalloc (use nsrl_linear_i16_i8_i16 with a workspace)",
        rows, params->input_dim, need, (unsigned)NSRL_NOALLOC_SCRATCH_BYTES);
    return NSRL_INVALID_SHAPE;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    nsrl::set_error("cudaGetDevice: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    nsrl::set_error("device %d beyond the %d supported by the static scratch", dev, kMaxDevices);
    return NSRL_CUDA_ERROR;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        nsrl::set_error("cudaGetSymbolAddress(g_noalloc_scratch): %s", cudaGetErrorString(e));
        return NSRL_CUDA_ERROR;
      }
      g_noalloc_ptr[dev] = ptr;
    }
    scratch = g_noalloc_ptr[dev];
  }
  return nsrl_linear_i16_i8_i16(x, rows, params, y, scratch, NSRL_NOALLOC_SCRATCH_BYTES, status, stream);
}

}  // extern "C"
