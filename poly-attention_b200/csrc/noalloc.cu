// poly_pass_bwd_noalloc: the backward pass for callers that cannot allocate
// device memory.
//
// poly_pass_bwd needs a caller-provided workspace (the fp32 dQ accumulator
// and per-row statistics). Some callers have no way to provide one: hosts
// reaching this library through a thin FFI that only hands over existing
// tensors, processes whose device memory is fully pre-planned by another
// allocator, or code running where cudaMalloc is forbidden. For them this
// entry point takes its scratch from a fixed array compiled into the library
// and allocates nothing.
//
// Limits and sharing:
//   * the array is kNoAllocScratchBytes (8 MiB) per GPU, held by every GPU
//     that loads the library until the process exits; requests needing more
//     (poly_pass_bwd_workspace_size() > 8 MiB) are rejected with POLY_EINVAL;
//   * all calls on a device share the one array, so calls whose kernels
//     overlap on the GPU (different streams, or other threads) race and give
//     wrong results: serialise them;
//   * the array keeps whatever the previous call left in it; the kernels
//     clear or fully overwrite every part they read (the dQ accumulator is
//     zeroed on the stream first), so no stale state leaks into results;
//   * every call made outside stream capture resolves the array's device
//     address again (cudaGetSymbolAddress, with the call's device current),
//     so a device reset or a re-created primary context never leaves a stale
//     address behind; a call made during stream capture reuses the address
//     the device's last uncaptured call resolved, so the first call on each
//     device must come before any stream capture begins.
#include <mutex>
#include <string>

#include "common.cuh"

namespace poly {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

// Host code must never pass the name of this array to a kernel: on the host it
// is only a stand-in symbol. Its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

int scratch_for_current_device(cudaStream_t stream, void** out) {
  int dev = -1;
  int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device index out of range for the no-allocation scratch table");
    return POLY_EUNSUPPORTED;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  rc = cuda_status(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
  if (rc) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  } else if (!g_noalloc_ptr[dev]) {
    set_error("poly_pass_bwd_noalloc: the first call on a device must come before stream capture");
    return POLY_EINVAL;
  }
  *out = g_noalloc_ptr[dev];
  return POLY_OK;
}

}  // namespace
}  // namespace poly

extern "C" POLY_API size_t poly_noalloc_scratch_bytes(void) { return poly::kNoAllocScratchBytes; }

extern "C" POLY_API int poly_pass_bwd_noalloc(const PolyPassBwdArgs* args, void* stream) {
  if (!args) {
    poly::set_error("null args");
    return POLY_EINVAL;
  }
  const size_t need = poly_pass_bwd_workspace_size(args);
  if (need > poly::kNoAllocScratchBytes) {
    poly::set_error("poly_pass_bwd_noalloc: this problem needs " + std::to_string(need) +
                    " bytes of scratch, more than the built-in " + std::to_string(poly::kNoAllocScratchBytes) +
                    " bytes; use poly_pass_bwd with a caller-provided workspace");
    return POLY_EINVAL;
  }
  void* scratch = nullptr;
  const int rc = poly::scratch_for_current_device((cudaStream_t)stream, &scratch);
  if (rc) return rc;
  PolyPassBwdArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = poly::kNoAllocScratchBytes;
  return poly_pass_bwd(&a, stream);
}
