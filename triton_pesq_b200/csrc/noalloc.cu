// pesq_forward_noalloc: the PESQ forward pass with no caller workspace.
//
// Some callers of this library cannot hand us device scratch memory: a
// real-time audio callback or a plugin inside a host application must not call
// cudaMalloc (it may block, synchronise the device or be forbidden by the
// host's memory policy), and neither can code running while a stream is being
// captured into a CUDA graph in global capture mode.  This entry point gives
// them the MOS / loss / distances of a batch without any allocation: its
// scratch is one statically sized array in device memory that belongs to this
// file.
//
// Costs and rules of that choice:
//   * every GPU on which this file's module is loaded holds kNoAllocScratchBytes
//     (16 MiB) until the process exits -- with CUDA's default lazy module
//     loading that happens on the first call of this entry point on the device;
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress; make that first call before any stream capture;
//   * that address is cached per device ordinal for the primary context, the
//     one the CUDA runtime uses: after cudaDeviceReset (which tears down that
//     context, this module and its array with it) the cached address is
//     stale, and a context created through the driver API has an array of its
//     own at another address -- do not call this entry point after a device
//     reset in the same process, nor with a non-primary context current;
//   * all calls on a device share the one array, which keeps the contents of
//     the last call: calls whose GPU work overlaps (different streams, or
//     concurrent host threads without ordering) race on it and must be
//     serialised by the caller.  Nothing in the array has to start at zero:
//     every byte the forward pass reads is written earlier in the same call;
//   * a call whose workspace would exceed the array is rejected with
//     PESQ_ERR_WORKSPACE (the caller should then use pesq_forward with its own
//     workspace).  At 16 kHz that allows e.g. 64 utterances of 8 s; with
//     resampling the 16 kHz copy of the signals counts too (e.g. 4 x 10 s at
//     48 kHz).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/pesq_cuda.h"

namespace pesq {
int set_error(int code, const char* msg);
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return pesq::set_error(PESQ_ERR_CUDA, "pesq_forward_noalloc: no usable current CUDA device");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* addr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
    if (e != cudaSuccess || !addr)
      return pesq::set_error(PESQ_ERR_CUDA, "pesq_forward_noalloc: cudaGetSymbolAddress of the static scratch failed");
    g_scratch_addr[dev] = addr;
  }
  *out = g_scratch_addr[dev];
  return PESQ_OK;
}

}  // namespace

extern "C" int pesq_forward_noalloc(const pesq_plan* plan, void* stream, const float* ref, int64_t ld_ref,
                                    const float* deg, int64_t ld_deg, int64_t batch, int64_t n_src, float* d_symm,
                                    float* d_asymm, float* mos, float* loss) {
  if (!plan) return pesq::set_error(PESQ_ERR_INVALID_ARGUMENT, "pesq_forward_noalloc: NULL plan");
  // the plan's device must be current (as pesq_forward requires) before the
  // scratch lookup, which would otherwise load this module on another device
  int plan_dev = -1, cur_dev = -1;
  int rc = pesq_plan_device(plan, &plan_dev);
  if (rc) return rc;
  if (cudaGetDevice(&cur_dev) != cudaSuccess || cur_dev != plan_dev)
    return pesq::set_error(PESQ_ERR_INVALID_ARGUMENT,
                           "pesq_forward_noalloc: the plan was created on another device than the current one");
  size_t need = 0;
  rc = pesq_workspace_size(plan, batch, n_src, 0u, &need);
  if (rc) return rc;
  if (need > kNoAllocScratchBytes)
    return pesq::set_error(PESQ_ERR_WORKSPACE,
                           "pesq_forward_noalloc: this batch needs more scratch than the 16 MiB static array; "
                           "call pesq_forward with a workspace of pesq_workspace_size bytes instead");
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc) return rc;
  return pesq_forward(plan, stream, ref, ld_ref, deg, ld_deg, batch, n_src, 0u, scratch, kNoAllocScratchBytes,
                      d_symm, d_asymm, mos, loss);
}
