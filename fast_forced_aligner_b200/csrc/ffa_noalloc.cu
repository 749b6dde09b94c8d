// ffa_noalloc.cu -- an align entry point that allocates no memory.
//
// Some callers cannot allocate device memory at the time they align: code
// that runs inside a framework which owns every device allocation (and
// forbids cudaMalloc behind its back), real-time or embedded pipelines whose
// memory is fixed at start-up, or hosts that must not touch the driver's
// allocator while other work is in flight.  For them ffa_align_noalloc runs
// the ordinary ffa_align path with its scratch taken from fixed buffers that
// live in this library:
//   - device scratch: a file-scope __device__ array of kNoAllocScratchBytes
//     (64 MiB), held on each GPU that loads this code until the process exits;
//   - host staging: a static array of kNoAllocStagingBytes (2 MiB) from which
//     the per-call descriptor table is uploaded (pageable memory: the upload
//     is staged by the driver).
// Because every call shares these buffers -- and the host staging array
// serves every GPU of the process -- calls must be serialised across the
// whole process: one call in flight at a time, on any device, from any host
// thread (concurrent streams or threads race, on different GPUs too).  The
// scratch needs no clearing between calls: every byte a kernel reads is
// written earlier in the same call.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "ffa_b200.h"
#include "ffa_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t{64} << 20;
constexpr size_t kNoAllocStagingBytes = size_t{2} << 20;

// The device scratch.  Host code must not use its name as an address: it is
// a host-side stand-in, and the device address comes from
// cudaGetSymbolAddress (per device, below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
alignas(256) unsigned char g_noalloc_staging[kNoAllocStagingBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mutex;

int noalloc_fail(int code, const char* message) {
  ffa::set_last_error(message);  // readable through ffa_last_error()
  return code;
}

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device does it; make that call before any
// stream capture).
int scratch_on_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(FFA_ERR_CUDA, "ffa_align_noalloc: no usable current CUDA device");
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (err != cudaSuccess || p == nullptr)
        return noalloc_fail(FFA_ERR_CUDA, "ffa_align_noalloc: cudaGetSymbolAddress of the scratch failed");
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return FFA_OK;
}

}  // namespace

extern "C" {

int ffa_align_noalloc(const ffa_record* records, int64_t count, int mode, int flags,
                      const uint8_t* emission_validity, const ffa_outputs* outputs,
                      ffa_stream_t stream) {
  ffa_sizes sizes{};
  int rc = ffa_align_query(records, count, mode, flags, &sizes);
  if (rc != FFA_OK) return rc;  // message already in ffa_last_error()
  if (sizes.workspace_bytes > kNoAllocScratchBytes || sizes.staging_bytes > kNoAllocStagingBytes) {
    char msg[256];
    std::snprintf(msg, sizeof(msg),
                  "ffa_align_noalloc: batch needs %zu bytes of device scratch and %zu of staging; "
                  "this entry point holds %zu and %zu -- split the batch or use ffa_align",
                  sizes.workspace_bytes, sizes.staging_bytes, kNoAllocScratchBytes,
                  kNoAllocStagingBytes);
    return noalloc_fail(FFA_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  rc = scratch_on_current_device(&scratch);
  if (rc != FFA_OK) return rc;
  return ffa_align(records, count, mode, flags, emission_validity, outputs, g_noalloc_staging,
                   kNoAllocStagingBytes, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
