// C-ABI layer of trnfft_b200: plans, per-device tables, argument checking
// and dispatch to the kernel launchers.  See include/trnfft_b200.h.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/trnfft_b200.h"
#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

__device__ float2 g_tw[kTwN];

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TRNFFT_CUDA_ERROR, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
std::mutex g_init_mu;
bool g_dev_ready[kMaxDevices];

// Upload the W_8192 table to `device` (once per device, that device current).
int ensure_device_tables(int device) {
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (device < 0 || device >= kMaxDevices) return fail(TRNFFT_INVALID_VALUE, "device %d out of range", device);
  if (g_dev_ready[device]) return TRNFFT_SUCCESS;
  std::vector<float2> h(kTwN);
  for (int i = 0; i < kTwN; ++i) {
    const double a = -2.0 * M_PI * (double)i / (double)kTwN;
    h[i] = make_float2((float)std::cos(a), (float)std::sin(a));
  }
  cudaError_t e = cudaMemcpyToSymbol(g_tw, h.data(), sizeof(float2) * kTwN);
  if (e != cudaSuccess) return cuda_fail(e, "uploading twiddle table");
  g_dev_ready[device] = true;
  return TRNFFT_SUCCESS;
}

struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

int ilog2_exact(int64_t n) {
  if (n <= 0 || (n & (n - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace
}  // namespace tfb

using namespace tfb;

struct trnfft_plan_s {
  int64_t n = 0;
  int device = 0;
  int algorithm = TRNFFT_ALG_COPY;
  int logn = -1;
  int64_t m = 0;  // Bluestein padded length
  int logm = -1;
};

extern "C" {

int trnfft_abi_version(void) { return TRNFFT_B200_ABI_VERSION; }

const char* trnfft_last_error(void) { return g_err.c_str(); }

int trnfft_plan_create(trnfft_plan_t* plan, int64_t n, int device) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "plan_create: null plan pointer");
  *plan = nullptr;
  if (n < 1) return fail(TRNFFT_INVALID_VALUE, "plan_create: n must be >= 1 (got %lld)", (long long)n);
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(TRNFFT_INVALID_VALUE, "plan_create: no CUDA device %d", device);
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "plan_create: cannot select device %d", device);
  int rc = ensure_device_tables(device);
  if (rc) return rc;
  trnfft_plan_s* p = new (std::nothrow) trnfft_plan_s;
  if (!p) return fail(TRNFFT_ALLOC_FAILED, "plan_create: out of host memory");
  p->n = n;
  p->device = device;
  p->logn = ilog2_exact(n);
  if (n == 1) {
    p->algorithm = TRNFFT_ALG_COPY;
  } else if (p->logn >= 1 && p->logn <= 12) {
    p->algorithm = TRNFFT_ALG_STOCKHAM;
  } else if (p->logn > 12) {
    p->algorithm = TRNFFT_ALG_MULTIPASS;
  } else {
    p->algorithm = TRNFFT_ALG_BLUESTEIN;
    int64_t v = 2 * n - 2;
    int bl = 0;
    while (v >> bl) ++bl;
    p->m = int64_t(1) << bl;
    p->logm = bl;
  }
  *plan = p;
  return TRNFFT_SUCCESS;
}

int trnfft_plan_destroy(trnfft_plan_t plan) {
  if (!plan) return TRNFFT_SUCCESS;
  delete plan;
  return TRNFFT_SUCCESS;
}

int trnfft_plan_query(trnfft_plan_t plan, int* algorithm, int64_t* padded_n, int64_t batch,
                      int64_t* work_bytes) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "plan_query: null plan");
  if (algorithm) *algorithm = plan->algorithm;
  if (padded_n) *padded_n = plan->algorithm == TRNFFT_ALG_BLUESTEIN ? plan->m : plan->n;
  if (work_bytes) *work_bytes = 0;
  (void)batch;
  return TRNFFT_SUCCESS;
}

static int check_ptrs(const char* fn, std::initializer_list<const void*> ps, size_t align) {
  for (const void* p : ps) {
    if (!p) return fail(TRNFFT_INVALID_VALUE, "%s: null data pointer", fn);
    if (!aligned(p, align)) return fail(TRNFFT_INVALID_VALUE, "%s: pointer %p not %zu-byte aligned", fn, p, align);
  }
  return TRNFFT_SUCCESS;
}

int trnfft_exec_c2c(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out_re,
                    float* out_im, int64_t batch, int inverse, void* work, void* stream) {
  (void)work;
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2c: null plan");
  if (batch < 0) return fail(TRNFFT_INVALID_VALUE, "exec_c2c: negative batch");
  if (batch == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("exec_c2c", {in_re, in_im, out_re, out_im}, 4);
  if (rc) return rc;
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2c: cannot select device %d", plan->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n = plan->n;
  cudaError_t e = cudaSuccess;
  switch (plan->algorithm) {
    case TRNFFT_ALG_COPY: {
      const size_t bytes = sizeof(float) * (size_t)batch;
      if (out_re != in_re) e = cudaMemcpyAsync(out_re, in_re, bytes, cudaMemcpyDeviceToDevice, st);
      if (e == cudaSuccess && out_im != in_im)
        e = cudaMemcpyAsync(out_im, in_im, bytes, cudaMemcpyDeviceToDevice, st);
      break;
    }
    case TRNFFT_ALG_STOCKHAM: {
      RowArgs a{in_re, in_im, out_re, out_im, batch, n, n, inverse ? (float)(1.0 / (double)n) : 1.0f};
      e = launch_rows_c2c(plan->logn, inverse != 0, a, st);
      break;
    }
    default:
      return fail(TRNFFT_UNSUPPORTED, "exec_c2c: n=%lld not supported yet", (long long)n);
  }
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_r2c(trnfft_plan_t plan, const float* in, float* out_re, float* out_im,
                    int64_t batch, void* work, void* stream) {
  (void)work;
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_r2c: null plan");
  if (batch < 0) return fail(TRNFFT_INVALID_VALUE, "exec_r2c: negative batch");
  if (batch == 0) return TRNFFT_SUCCESS;
  const int64_t n = plan->n;
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_r2c: cannot select device %d", plan->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (plan->logn >= 2 && plan->logn <= 13) {
    int rc = check_ptrs("exec_r2c", {in}, 8);
    if (!rc) rc = check_ptrs("exec_r2c", {out_re, out_im}, 4);
    if (rc) return rc;
    RowArgs a{in, nullptr, out_re, out_im, batch, n, n / 2 + 1, 1.0f};
    e = launch_rows_r2c(plan->logn - 1, a, st);
  } else {
    return fail(TRNFFT_UNSUPPORTED, "exec_r2c: n=%lld not supported yet", (long long)n);
  }
  if (e != cudaSuccess) return cuda_fail(e, "exec_r2c");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_c2r(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out,
                    int64_t batch, void* work, void* stream) {
  (void)work;
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2r: null plan");
  if (batch < 0) return fail(TRNFFT_INVALID_VALUE, "exec_c2r: negative batch");
  if (batch == 0) return TRNFFT_SUCCESS;
  const int64_t n = plan->n;
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2r: cannot select device %d", plan->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (plan->logn >= 2 && plan->logn <= 13) {
    int rc = check_ptrs("exec_c2r", {out}, 8);
    if (!rc) rc = check_ptrs("exec_c2r", {in_re, in_im}, 4);
    if (rc) return rc;
    RowArgs a{in_re, in_im, out, nullptr, batch, n / 2 + 1, n, (float)(1.0 / (double)n)};
    e = launch_rows_c2r(plan->logn - 1, a, st);
  } else {
    return fail(TRNFFT_UNSUPPORTED, "exec_c2r: n=%lld not supported yet", (long long)n);
  }
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2r");
  return TRNFFT_SUCCESS;
}

}  // extern "C"
