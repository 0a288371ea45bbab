// In-place multi-pass transform for callers that cannot allocate device
// memory.
//
// An in-place power-of-two transform longer than 4096 points needs a work
// area holding a copy of its input, because its first pass scatters rows
// across the whole transform (trnfft_exec_c2c takes that area from the
// caller).  Some callers cannot provide it: code running where cudaMalloc is
// off limits (inside another library's allocator or memory pool, in
// real-time audio callbacks that must not block or fail on allocation, or in
// embedding runtimes that hand out only fixed buffers).  This file gives them
// trnfft_exec_c2c_inplace_noalloc, which uses a fixed scratch array that the
// library reserves on every GPU that loads it and keeps until the process
// exits.  It allocates nothing.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/trnfft_b200.h"
#include "kernels.h"
#include "plan_internal.h"

namespace tfb {

// Largest batch * n the scratch holds: 2^21 complex values (16 MiB of
// device memory, real and imaginary planes of 2^21 floats each).
constexpr long long kNoAllocMaxElems = 1LL << 21;

static __device__ __align__(256) float g_noalloc_scratch[2 * kNoAllocMaxElems];

namespace {
constexpr int kMaxDev = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDev];  // device address of g_noalloc_scratch, per device
}  // namespace

// Device address of the scratch array on `device`, looked up once per device
// with that device current.  The name g_noalloc_scratch is only a host-side
// stand-in in host code, never a device address.
static int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= kMaxDev) return record_failure(TRNFFT_INVALID_VALUE, "exec_c2c_inplace_noalloc: device out of range");
  if (!g_scratch_addr[device]) {
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(device);
    void* p = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
      char msg[256];
      snprintf(msg, sizeof msg, "exec_c2c_inplace_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return record_failure(TRNFFT_CUDA_ERROR, msg);
    }
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return TRNFFT_SUCCESS;
}

}  // namespace tfb

extern "C" int trnfft_exec_c2c_inplace_noalloc(trnfft_plan_t plan, float* re, float* im, int64_t batch,
                                               int inverse, void* stream) {
  using namespace tfb;
  if (!plan) return record_failure(TRNFFT_INVALID_VALUE, "exec_c2c_inplace_noalloc: null plan");
  if (plan->algorithm != TRNFFT_ALG_MULTIPASS)
    return record_failure(TRNFFT_INVALID_VALUE,
                          "exec_c2c_inplace_noalloc: only power-of-two n > 4096 use scratch; call "
                          "trnfft_exec_c2c (which needs no work area for other sizes)");
  if (batch < 0) return record_failure(TRNFFT_INVALID_VALUE, "exec_c2c_inplace_noalloc: negative batch");
  if (batch == 0) return TRNFFT_SUCCESS;
  if (plan->n > kNoAllocMaxElems / batch) {
    char msg[256];
    snprintf(msg, sizeof msg,
             "exec_c2c_inplace_noalloc: batch*n = %lld*%lld exceeds the fixed scratch of %lld complex values",
             (long long)batch, (long long)plan->n, kNoAllocMaxElems);
    return record_failure(TRNFFT_INVALID_VALUE, msg);
  }
  void* scratch = nullptr;
  int rc = scratch_address(plan->device, &scratch);
  if (rc) return rc;
  // The scratch only receives a copy of the input, fully overwritten by every
  // call, so nothing in it has to start at zero.
  return trnfft_exec_c2c(plan, re, im, re, im, batch, inverse, scratch, stream);
}
