// C-ABI layer of trnfft_b200: plans, per-device tables, argument checking
// and dispatch to the kernel launchers.  See include/trnfft_b200.h.
#include <cuda_runtime.h>

#include <cmath>
#include <complex>
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
#include "tma.cuh"

#include <cstdlib>

namespace tfb {

__device__ float2 g_tw[kTwN];
__device__ float2 g_twd[kTwN];

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

// Upload the W_16384 table and the level tables to `device` (once per device, that device current).
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
  // level tables D_L[k] = W_{2^L}^k, k < 2^(L-1), level L from offset 2^(L-1) - 1
  std::vector<float2> hd(kTwN, make_float2(1.f, 0.f));
  for (int L = 1; L <= kTwLog; ++L) {
    const int off = (1 << (L - 1)) - 1;
    for (int k = 0; k < (1 << (L - 1)); ++k) {
      const double a = -2.0 * M_PI * (double)k / (double)(1 << L);
      hd[off + k] = make_float2((float)std::cos(a), (float)std::sin(a));
    }
  }
  e = cudaMemcpyToSymbol(g_twd, hd.data(), sizeof(float2) * kTwN);
  if (e != cudaSuccess) return cuda_fail(e, "uploading the level twiddle tables");
  std::vector<double2> h64(4096);
  for (int i = 0; i < 4096; ++i) {
    const double a = -2.0 * M_PI * (double)i / 4096.0;
    h64[i] = make_double2(std::cos(a), std::sin(a));
  }
  e = upload_tw64(h64.data());
  if (e != cudaSuccess) return cuda_fail(e, "uploading the double-precision twiddle table");
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

// In-place iterative radix-2 FFT in double precision (forward sign), used
// only at plan creation to tabulate the Bluestein filter spectrum.
void host_fft_double(std::vector<std::complex<double>>& a) {
  const size_t n = a.size();
  for (size_t i = 1, j = 0; i < n; ++i) {
    size_t bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) std::swap(a[i], a[j]);
  }
  for (size_t len = 2; len <= n; len <<= 1) {
    const size_t h = len / 2;
    std::vector<std::complex<double>> w(h);
    for (size_t k = 0; k < h; ++k) w[k] = std::polar(1.0, -2.0 * M_PI * (double)k / (double)len);
    for (size_t i = 0; i < n; i += len)
      for (size_t k = 0; k < h; ++k) {
        const std::complex<double> u = a[i + k], v = a[i + k + h] * w[k];
        a[i + k] = u + v;
        a[i + k + h] = u - v;
      }
  }
}

}  // namespace

// Record a failure message for trnfft_last_error() from another translation unit.
int record_failure(int code, const char* msg) { return fail(code, "%s", msg); }

}  // namespace tfb

using namespace tfb;

#include "plan_internal.h"

// Two-level twiddle tables for W_n, n = 2^logn: W_n^e = hi[e >> s] * lo[e & (2^s - 1)].
static int make_twiddle_tables(trnfft_plan_s* p) {
  const int L = p->logn;
  const int sp = (L + 1) / 2;
  const int64_t nlo = int64_t(1) << sp, nhi = int64_t(1) << (L - sp);
  std::vector<float2> lo(nlo), hi(nhi);
  const double n = std::ldexp(1.0, L);
  for (int64_t i = 0; i < nlo; ++i) {
    const double a = -2.0 * M_PI * (double)i / n;
    lo[i] = make_float2((float)std::cos(a), (float)std::sin(a));
  }
  for (int64_t i = 0; i < nhi; ++i) {
    const double a = -2.0 * M_PI * (double)(i << sp) / n;
    hi[i] = make_float2((float)std::cos(a), (float)std::sin(a));
  }
  cudaError_t e = cudaMalloc(&p->tw_lo, sizeof(float2) * nlo);
  if (e == cudaSuccess) e = cudaMalloc(&p->tw_hi, sizeof(float2) * nhi);
  if (e != cudaSuccess) return fail(TRNFFT_ALLOC_FAILED, "plan_create: %s", cudaGetErrorString(e));
  e = cudaMemcpy(p->tw_lo, lo.data(), sizeof(float2) * nlo, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(p->tw_hi, hi.data(), sizeof(float2) * nhi, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "plan_create: uploading twiddle tables");
  p->tw_split = sp;
  return TRNFFT_SUCCESS;
}

static ColArgs col_base(const trnfft_plan_s* p) {
  ColArgs c;
  std::memset(&c, 0, sizeof c);
  c.O1 = 1;
  c.O2 = 1;
  c.O3 = 1;
  c.tw_modo = int64_t(1) << 62;
  c.scale = 1.f;
  c.nmask = p->n - 1;
  c.tw_split = p->tw_split;
  c.tw_hi = p->tw_hi;
  c.tw_lo = p->tw_lo;
  c.tw_mul = 1;
  return c;
}

static constexpr int kMaxColLog = 10;  // column passes transform up to 1024 points on chip
static constexpr int kMaxRowBlockLog = 14;  // contiguous rows up to 16384 points in one block
static constexpr int kMaxMultipassLog = 30;

// multi-pass digits of at most 2^max_digit_log() points (default 256; the
// environment variable TRNFFT_B200_MAX_DIGIT_LOG selects 6..10 for tuning)
static int max_digit_log() {
  static int v = [] {
    const char* e = getenv("TRNFFT_B200_MAX_DIGIT_LOG");
    int d = e ? atoi(e) : 8;
    return d < 6 ? 6 : (d > kMaxColLog ? kMaxColLog : d);
  }();
  return v;
}

// Contiguous rows of n = 2^p > 4096 points, out of place (in != out).
// n is split into m digits N_1..N_m (each <= 256 points; n = n_1 + N_1 n_2 +
// ... with n_1 fastest) and the output index is k = k_m + N_m (k_{m-1} + ...).
// Pass 1 transforms the slowest digit n_m and stores rows [n_1]...[n_{m-1}][k_m]
// (the transposing pass); passes 2..m transform n_{m-1}, ..., n_1 in place.
// After transforming digit j >= 2 the values are multiplied by
// W_N^{n_{j-1} * K_j * P_{j-1}}, K_j = sum_{i >= j} k_i Q_i, P_i = N_1..N_{i-1},
// Q_i = N_{i+1}..N_m: the twiddles of the Cooley-Tukey recursion on the
// leading digit, applied inside the pass that produces their operand.
static cudaError_t run_rows_multipass(const trnfft_plan_s* p, const float* xr, const float* xi, float* yr,
                                      float* yi, int64_t batch, bool inv, cudaStream_t st) {
  const int L = p->logn;
  if (L <= kMaxRowBlockLog) {
    // 8192 / 16384 points: one block per transform, one HBM round trip
    RowArgs a{xr, xi, yr, yi, batch, p->n, p->n, inv ? (float)(1.0 / (double)p->n) : 1.0f};
    return launch_rows_c2c(L, inv, a, st);
  }
  const long long N = p->n;
  const int md = max_digit_log();
  const int m0 = (L + md - 1) / md;
  const int m = m0 > 4 ? 4 : m0;
  if (m < 2 || m > 4) return cudaErrorInvalidValue;
  int lg[5] = {0, 0, 0, 0, 0};  // lg[1..m]
  for (int i = 1; i <= m; ++i) lg[i] = L / m + (i <= L % m ? 1 : 0);
  long long Nd[5], P[6];
  P[1] = 1;
  for (int i = 1; i <= m; ++i) {
    Nd[i] = 1LL << lg[i];
    P[i + 1] = P[i] * Nd[i];
  }
  auto Q = [&](int i) {  // N_{i+1} ... N_m
    long long q = 1;
    for (int t = i + 1; t <= m; ++t) q *= Nd[t];
    return q;
  };
  const float sc = inv ? (float)(1.0 / (double)N) : 1.f;
  cudaError_t e;
  {
    // pass 1: FFT over n_m (stride P_m).  Columns n_1; outer digits:
    // o1 = n_{m-1} (the twiddle digit), o2 = the digits n_2..n_{m-2} (m = 4: n_2), o3 = batch.
    ColArgs a = col_base(p);
    a.xr = xr; a.xi = xi; a.yr = yr; a.yi = yi;
    a.ncols = Nd[1];
    a.is_j = P[m];
    // output position of (n_1, ..., n_{m-1}, k_m) is sum_{i<m} n_i * (N_{i+1}..N_m) + k_m = n_i * Q(i)
    a.os_c = Q(1);
    if (m == 2) {
      a.O1 = 1;
      a.O2 = 1;
      a.has_tw = 1; a.tw_c = 1;  // W_N^{n_1 k_2}
    } else {
      a.O1 = Nd[m - 1]; a.is_o1 = P[m - 1]; a.os_o1 = Q(m - 1);
      a.has_tw = 1; a.tw_mul = P[m - 1]; a.tw_b = 1;  // W_N^{n_{m-1} k_m P_{m-1}}
      if (m == 4) {
        a.O2 = Nd[2]; a.is_o2 = P[2]; a.os_o2 = Q(2);
      }
    }
    a.O3 = batch; a.is_o3 = N; a.os_o3 = N;
    e = launch_colpass(lg[m], inv, 1, a, st);
    if (e != cudaSuccess) return e;
  }
  for (int j = m - 1; j >= 1; --j) {
    // in place, layout [n_1..n_{j-1}][n_j][k_{j+1}..k_m]: FFT over n_j (stride Q(j)),
    // columns = the already transformed fast digits (Q(j) of them), outer = slow digits.
    ColArgs b = col_base(p);
    b.xr = yr; b.xi = yi; b.yr = yr; b.yi = yi;
    b.ncols = Q(j);
    b.is_j = Q(j);
    b.os_k = Q(j);
    b.O1 = P[j]; b.is_o1 = Nd[j] * Q(j); b.os_o1 = Nd[j] * Q(j);
    b.O3 = batch; b.is_o3 = N; b.os_o3 = N;
    if (j >= 2) {
      // W_N^{n_{j-1} (k_j Q(j) + c) P_{j-1}}; n_{j-1} is the fastest digit of o1
      b.has_tw = 1; b.tw_modo = Nd[j - 1]; b.tw_mul = P[j - 1]; b.tw_a = 1; b.tw_b = Q(j);
    } else {
      b.scale = sc;
    }
    e = launch_colpass(lg[j], inv, 0, b, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

static int run_rows_multipass_plan(const trnfft_plan_s* p, const float* xr, const float* xi, float* yr, float* yi,
                                   int64_t batch, bool inv, cudaStream_t st) {
  cudaError_t e = run_rows_multipass(p, xr, xi, yr, yi, batch, inv, st);
  if (e != cudaSuccess) return cuda_fail(e, "multi-pass transform");
  return TRNFFT_SUCCESS;
}

// Transforms along the middle axis of an [outer][n][inner] array, inner > 1.
// tw (optional): after the transform, output (o, K, s) is multiplied by
// W_{tw->n}^{(coff + s) * K} using tw's tables (the four-step inter-pass twiddle).
// Peer scatter of the last pass (four-step exchange over NVLink), see ColArgs kind 2.
struct ScatterSpec {
  int npeers;
  float* re[8];
  float* im[8];
  int rows_log;
  long long ld, col0;
  long long max_blocks;  // grid cap of the scatter pass (0: none)
};

// ld_in / ld_out: floats between consecutive points of one column (default inner).
// With sc, the last pass stores into the peers' row buffers instead of yr/yi
// (yr/yi then only hold the first pass's output when there are two passes).
static cudaError_t run_axis(const trnfft_plan_s* p, const float* xr, const float* xi, float* yr, float* yi,
                            int64_t outer, int64_t inner, bool inv, cudaStream_t st,
                            const trnfft_plan_s* tw = nullptr, int64_t coff = 0, int64_t ld_in = 0,
                            int64_t ld_out = 0, const ScatterSpec* scs = nullptr) {
  auto scatter = [&](ColArgs& c, long long ka, long long kb) {
    c.sc_npeers = scs->npeers;
    for (int q = 0; q < scs->npeers; ++q) {
      c.sc_re[q] = scs->re[q];
      c.sc_im[q] = scs->im[q];
    }
    c.sc_ka = ka;
    c.sc_kb = kb;
    c.sc_rows_log = scs->rows_log;
    c.sc_ld = scs->ld;
    c.sc_col0 = scs->col0;
    c.max_blocks = scs->max_blocks;
  };
  if (ld_in <= 0) ld_in = inner;
  if (ld_out <= 0) ld_out = inner;
  auto extra_tw = [&](ColArgs& c, long long tw_c, long long tw_a) {
    c.has_tw = 1;
    c.nmask = tw->n - 1;
    c.tw_split = tw->tw_split;
    c.tw_hi = tw->tw_hi;
    c.tw_lo = tw->tw_lo;
    c.tw_mul = 1;
    c.tw_modo = int64_t(1) << 62;
    c.tw_a = tw_a;
    c.tw_b = 0;
    c.tw_c = tw_c;
    c.tw_coff = coff;
  };
  const int L = p->logn;
  const long long n = p->n;
  const float sc = inv ? (float)(1.0 / (double)n) : 1.f;
  if (L <= kMaxColLog) {
    ColArgs a = col_base(p);
    a.xr = xr; a.xi = xi; a.yr = yr; a.yi = yi;
    a.ncols = inner; a.O3 = outer; a.is_o3 = n * ld_in; a.is_j = ld_in;
    a.os_o3 = n * ld_out; a.os_k = ld_out; a.scale = sc;
    if (tw) extra_tw(a, 1, 0);  // e = (coff + s) * k
    if (scs) {
      scatter(a, 0, 1);  // K = k
      return launch_colpass(L, inv, 2, a, st);
    }
    return launch_colpass(L, inv, 0, a, st);
  }
  // n = L1*L2, point n1 + L1*n2, output k2 + L2*k1 (out of place first pass)
  const int l1 = L / 2, l2 = L - l1;
  const long long L1 = 1LL << l1, L2 = 1LL << l2;
  ColArgs a = col_base(p);  // FFT over n2; outer n1; output (n1*L2 + k2)*S + s; twiddle W_n^{n1 k2}
  a.xr = xr; a.xi = xi; a.yr = yr; a.yi = yi;
  a.ncols = inner; a.O1 = L1; a.O3 = outer; a.is_o1 = ld_in; a.is_o3 = n * ld_in; a.is_j = L1 * ld_in;
  a.os_o1 = L2 * ld_out; a.os_o3 = n * ld_out; a.os_k = ld_out;
  a.has_tw = 1; a.tw_b = 1;
  cudaError_t e = launch_colpass(l2, inv, 0, a, st);
  if (e != cudaSuccess) return e;
  ColArgs b = col_base(p);  // FFT over n1 in place; outer k2
  b.xr = yr; b.xi = yi; b.yr = yr; b.yi = yi;
  b.ncols = inner; b.O1 = L2; b.O3 = outer; b.is_o1 = ld_out; b.is_o3 = n * ld_out; b.is_j = L2 * ld_out;
  b.os_o1 = ld_out; b.os_o3 = n * ld_out; b.os_k = L2 * ld_out; b.scale = sc;
  // K = k2 + L2*k1 with k2 = o1 of this pass and k1 = its FFT index: e = (coff + s)*(o1 + L2*k)
  if (tw) {
    extra_tw(b, L2, 1);
    b.tw_modo = L2;  // o1 ranges over k2 < L2
  }
  if (scs) {
    scatter(b, 1, L2);  // K = k2 + L2*k1 with k2 = o1
    return launch_colpass(l1, inv, 2, b, st);
  }
  return launch_colpass(l1, inv, 0, b, st);
}

// Bluestein tables: chirp_k = exp(-i*pi*(k^2 mod 2n)/n) (exact integer
// reduction of the angle, then double trig) and H = FFT_m(h)/m with
// h_j = conj(chirp_j) for j < n, h_{m-j} = conj(chirp_j) for 0 < j < n.
static int make_bluestein_tables(trnfft_plan_s* p) {
  const int64_t n = p->n, m = p->m;
  std::vector<float2> c(n);
  std::vector<std::complex<double>> cd(n), h(m, 0.0);
  for (int64_t k = 0; k < n; ++k) {
    const int64_t e = (k * k) % (2 * n);
    const double ang = -M_PI * (double)e / (double)n;
    cd[k] = std::polar(1.0, ang);
    c[k] = make_float2((float)cd[k].real(), (float)cd[k].imag());
  }
  for (int64_t j = 0; j < n; ++j) h[j] = std::conj(cd[j]);
  for (int64_t j = 1; j < n; ++j) h[m - j] = std::conj(cd[j]);
  host_fft_double(h);
  std::vector<float2> hf(m);
  for (int64_t k = 0; k < m; ++k)
    hf[k] = make_float2((float)(h[k].real() / (double)m), (float)(h[k].imag() / (double)m));
  cudaError_t e = cudaMalloc(&p->chirp, sizeof(float2) * n);
  if (e == cudaSuccess) e = cudaMalloc(&p->H, sizeof(float2) * m);
  if (e != cudaSuccess) return fail(TRNFFT_ALLOC_FAILED, "plan_create: %s", cudaGetErrorString(e));
  e = cudaMemcpy(p->chirp, c.data(), sizeof(float2) * n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(p->H, hf.data(), sizeof(float2) * m, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "plan_create: uploading Bluestein tables");
  return TRNFFT_SUCCESS;
}

static constexpr int kMaxBluesteinLogM = 14;

static int run_rows_multipass_plan(const trnfft_plan_s* p, const float* xr, const float* xi, float* yr, float* yi,
                                   int64_t batch, bool inv, cudaStream_t st);

// Bluestein with m > 16384: chirp (n, float2), an m-point sub-plan, and
// H = FFT_m(h) computed on the device by the multi-pass kernels (planar).
static int make_large_bluestein(trnfft_plan_s* p) {
  const int64_t n = p->n, m = p->m;
  std::vector<float2> c(n);
  std::vector<float> hr(m, 0.f), hi(m, 0.f);
  for (int64_t k = 0; k < n; ++k) {
    const int64_t e = (k * k) % (2 * n);
    const double ang = -M_PI * (double)e / (double)n;
    c[k] = make_float2((float)std::cos(ang), (float)std::sin(ang));
  }
  for (int64_t j = 0; j < n; ++j) {
    hr[j] = c[j].x;
    hi[j] = -c[j].y;
  }
  for (int64_t j = 1; j < n; ++j) {
    hr[m - j] = c[j].x;
    hi[m - j] = -c[j].y;
  }
  trnfft_plan_t sub = nullptr;
  int rc = trnfft_plan_create(&sub, m, p->device);
  if (rc) return rc;
  p->sub = sub;
  float *dh = nullptr;
  cudaError_t e = cudaMalloc(&p->chirp, sizeof(float2) * n);
  if (e == cudaSuccess) e = cudaMalloc(&p->Hr, sizeof(float) * m);
  if (e == cudaSuccess) e = cudaMalloc(&p->Hi, sizeof(float) * m);
  if (e == cudaSuccess) e = cudaMalloc(&dh, sizeof(float) * 2 * m);
  if (e != cudaSuccess) {
    if (dh) cudaFree(dh);
    return fail(TRNFFT_ALLOC_FAILED, "plan_create: %s", cudaGetErrorString(e));
  }
  e = cudaMemcpy(p->chirp, c.data(), sizeof(float2) * n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dh, hr.data(), sizeof(float) * m, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(dh + m, hi.data(), sizeof(float) * m, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) rc = run_rows_multipass_plan(sub, dh, dh + m, p->Hr, p->Hi, 1, false, 0);
  if (e == cudaSuccess && rc == TRNFFT_SUCCESS) e = cudaDeviceSynchronize();
  cudaFree(dh);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "plan_create: Bluestein filter spectrum");
  return TRNFFT_SUCCESS;
}


// ---- double precision ------------------------------------------------------

static constexpr int kMaxF64Log = 24;        // power-of-two fp64 transforms up to 2^24 (two passes)
static constexpr int kMaxF64BlockLog = 12;   // one pass up to 4096 points

static std::mutex g_f64_mu;

template <class T>
static cudaError_t upload_new(T** dst, const std::vector<T>& h) {
  cudaError_t e = cudaMalloc(dst, sizeof(T) * h.size());
  if (e == cudaSuccess) e = cudaMemcpy(*dst, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice);
  return e;
}

// Tables of plan p for fp64 execution (its device current, g_f64_mu held).
static int enable_f64_locked(trnfft_plan_s* p) {
  if (p->f64) return TRNFFT_SUCCESS;
  cudaError_t e = cudaSuccess;
  if (p->algorithm == TRNFFT_ALG_STOCKHAM || p->algorithm == TRNFFT_ALG_MULTIPASS) {
    if (p->logn > kMaxF64Log)
      return fail(TRNFFT_UNSUPPORTED, "double precision: n=2^%d above the supported 2^%d", p->logn, kMaxF64Log);
    if (p->logn > kMaxF64BlockLog) {
      const int L = p->logn, sp = (L + 1) / 2;
      std::vector<double2> lo(size_t(1) << sp), hi(size_t(1) << (L - sp));
      const double n = std::ldexp(1.0, L);
      for (size_t i = 0; i < lo.size(); ++i) {
        const double a = -2.0 * M_PI * (double)i / n;
        lo[i] = make_double2(std::cos(a), std::sin(a));
      }
      for (size_t i = 0; i < hi.size(); ++i) {
        const double a = -2.0 * M_PI * (double)(i << sp) / n;
        hi[i] = make_double2(std::cos(a), std::sin(a));
      }
      e = upload_new(&p->tw64_lo, lo);
      if (e == cudaSuccess) e = upload_new(&p->tw64_hi, hi);
      p->tw64_split = sp;
    }
  } else if (p->algorithm == TRNFFT_ALG_BLUESTEIN || p->algorithm == TRNFFT_ALG_MIXED) {
    const int64_t n = p->n, m = p->m;
    if (p->logm > kMaxF64Log)
      return fail(TRNFFT_UNSUPPORTED, "double precision: Bluestein n=%lld (padded 2^%d) above 2^%d", (long long)n,
                  p->logm, kMaxF64Log);
    std::vector<double2> c(n), hf(m);
    std::vector<std::complex<double>> h(m, 0.0);
    for (int64_t k = 0; k < n; ++k) {
      const int64_t ex = (k * k) % (2 * n);
      const double ang = -M_PI * (double)ex / (double)n;
      c[k] = make_double2(std::cos(ang), std::sin(ang));
    }
    for (int64_t j = 0; j < n; ++j) h[j] = std::complex<double>(c[j].x, -c[j].y);
    for (int64_t j = 1; j < n; ++j) h[m - j] = std::complex<double>(c[j].x, -c[j].y);
    host_fft_double(h);
    for (int64_t k = 0; k < m; ++k) hf[k] = make_double2(h[k].real() / (double)m, h[k].imag() / (double)m);
    e = upload_new(&p->chirp64, c);
    if (e == cudaSuccess) e = upload_new(&p->H64, hf);
    if (e == cudaSuccess) {
      trnfft_plan_t sub = nullptr;
      int rc = trnfft_plan_create(&sub, m, p->device);
      if (rc) return rc;
      p->sub64 = sub;
      rc = enable_f64_locked(sub);
      if (rc) return rc;
    }
  }
  if (e != cudaSuccess) return fail(TRNFFT_ALLOC_FAILED, "double precision tables: %s", cudaGetErrorString(e));
  p->f64 = true;
  return TRNFFT_SUCCESS;
}

static int64_t f64_work_bytes(const trnfft_plan_s* p, int64_t batch) {
  if (p->algorithm == TRNFFT_ALG_BLUESTEIN || p->algorithm == TRNFFT_ALG_MIXED) {
    int64_t w = (int64_t)(2 * sizeof(double)) * p->m * batch;
    if (p->logm > kMaxF64BlockLog) w *= 2;
    return w;
  }
  if (p->algorithm != TRNFFT_ALG_COPY && p->logn > kMaxF64BlockLog) return (int64_t)(2 * sizeof(double)) * p->n * batch;
  return 0;
}

// float32 input / output planes of an fp64 transform (converted in the first kernel's loads and
// the last kernel's stores); null: the double planes are used
struct F32IO {
  const float* xr;
  const float* xi;
  float* yr;
  float* yi;
};

// Power-of-two fp64 transform of `batch` contiguous rows; `scale` multiplies the result.
static cudaError_t run_f64_pow2(const trnfft_plan_s* p, const double* xr, const double* xi, double* yr, double* yi,
                                int64_t batch, bool inv, double scale, double* work, cudaStream_t st,
                                const F32IO* io = nullptr) {
  const int L = p->logn;
  const long long N = p->n;
  F64SeqArgs a;
  std::memset(&a, 0, sizeof a);
  if (L <= kMaxF64BlockLog) {
    a.xr = xr; a.xi = xi; a.yr = yr; a.yi = yi;
    a.nseq = batch; a.inner = 1;
    a.in_outer = N; a.in_js = 1;
    a.out_outer = N; a.out_ks = 1;
    a.scale = scale;
    if (io) { a.xr32 = io->xr; a.xi32 = io->xi; a.yr32 = io->yr; a.yi32 = io->yi; }
    return launch_f64_seq(L, inv, a, st);
  }
  // N = N1 * N2, n = n1 N2 + n2, k = k1 + N1 k2:
  // A: columns n2, FFT over n1 (stride N2), times W_N^{n2 k1} -> work[k1][n2]
  // B: rows k1 of work, FFT over n2, stored at k1 + N1 k2 (natural order)
  const int l1 = L / 2, l2 = L - l1;
  const long long N1 = 1LL << l1, N2 = 1LL << l2;
  double* wr = work;
  double* wi = work + (size_t)N * batch;
  a.xr = xr; a.xi = xi; a.yr = wr; a.yi = wi;
  a.nseq = batch * N2; a.inner = N2;
  a.in_outer = N; a.in_cs = 1; a.in_js = N2;
  a.out_outer = N; a.out_cs = 1; a.out_ks = N2;
  a.tw_hi = p->tw64_hi; a.tw_lo = p->tw64_lo; a.tw_split = p->tw64_split;
  a.tw_mask = (unsigned long long)(N - 1); a.tw_off = 0;
  a.scale = 1.0;
  if (io) { a.xr32 = io->xr; a.xi32 = io->xi; }
  cudaError_t e = launch_f64_seq(l1, inv, a, st);
  if (e != cudaSuccess) return e;
  F64SeqArgs b;
  std::memset(&b, 0, sizeof b);
  b.xr = wr; b.xi = wi; b.yr = yr; b.yi = yi;
  b.nseq = batch * N1; b.inner = N1;
  b.in_outer = N; b.in_cs = N2; b.in_js = 1;
  b.out_outer = N; b.out_cs = 1; b.out_ks = N1;
  b.scale = scale;
  if (io) { b.yr32 = io->yr; b.yi32 = io->yi; }
  return launch_f64_seq(l2, inv, b, st);
}

static cudaError_t run_f64(const trnfft_plan_s* p, const double* xr, const double* xi, double* yr, double* yi,
                           int64_t batch, bool inv, double* work, cudaStream_t st, const F32IO* io = nullptr) {
  const double sc = inv ? 1.0 / (double)p->n : 1.0;
  if (p->algorithm == TRNFFT_ALG_COPY) {
    const void* sr = io ? (const void*)io->xr : (const void*)xr;
    const void* si = io ? (const void*)io->xi : (const void*)xi;
    void* dr = io ? (void*)io->yr : (void*)yr;
    void* di = io ? (void*)io->yi : (void*)yi;
    const size_t bytes = (io ? sizeof(float) : sizeof(double)) * (size_t)batch;
    cudaError_t e = cudaSuccess;
    if (dr != sr) e = cudaMemcpyAsync(dr, sr, bytes, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess && di != si) e = cudaMemcpyAsync(di, si, bytes, cudaMemcpyDeviceToDevice, st);
    return e;
  }
  if (p->algorithm != TRNFFT_ALG_BLUESTEIN && p->algorithm != TRNFFT_ALG_MIXED)
    return run_f64_pow2(p, xr, xi, yr, yi, batch, inv, sc, work, st, io);
  // Bluestein: chirp premultiply, m-point FFT, times H, unscaled inverse m-point FFT (1/m is in H), postmultiply
  const long long m = p->m;
  if (p->sub64 && p->sub64->logn <= kMaxF64BlueFusedLog) {
    // the whole chain in one kernel (the padded transforms stay in shared memory)
    F64BlueArgs fa;
    fa.xr = xr; fa.xi = xi; fa.yr = yr; fa.yi = yi;
    fa.chirp = p->chirp64; fa.H = p->H64;
    fa.batch = batch; fa.n = (int)p->n; fa.scale = sc;
    fa.xr32 = io ? io->xr : nullptr; fa.xi32 = io ? io->xi : nullptr;
    fa.yr32 = io ? io->yr : nullptr; fa.yi32 = io ? io->yi : nullptr;
    return launch_f64_blue_fused(p->sub64->logn, inv, fa, st);
  }
  double* ar = work;
  double* ai = work + (size_t)m * batch;
  double* sub_work = work + 2 * (size_t)m * batch;
  cudaError_t e = launch_f64_blue_pre(xr, xi, io ? io->xr : nullptr, io ? io->xi : nullptr, p->chirp64, ar, ai, batch,
                                      p->n, m, inv, st);
  if (e == cudaSuccess) e = run_f64_pow2(p->sub64, ar, ai, ar, ai, batch, false, 1.0, sub_work, st);
  if (e == cudaSuccess) e = launch_f64_blue_mul(ar, ai, p->H64, batch, m, inv, st);
  if (e == cudaSuccess) e = run_f64_pow2(p->sub64, ar, ai, ar, ai, batch, true, 1.0, sub_work, st);
  if (e == cudaSuccess)
    e = launch_f64_blue_post(ar, ai, p->chirp64, yr, yi, io ? io->yr : nullptr, io ? io->yi : nullptr, batch, p->n, m,
                             inv, sc, st);
  return e;
}

// Mixed-radix schedule of n (radices 16, 8, 4, 2, then 3, 5, 7), or 0 passes when
// n has another prime factor.  Larger power-of-two radices first: fewer passes.
static int mixed_schedule(int64_t n, int* radix) {
  int np = 0;
  int64_t v = n;
  while (v % 16 == 0 && np < 16) { radix[np++] = 16; v /= 16; }
  while (v % 8 == 0 && np < 16) { radix[np++] = 8; v /= 8; }
  while (v % 4 == 0 && np < 16) { radix[np++] = 4; v /= 4; }
  while (v % 2 == 0 && np < 16) { radix[np++] = 2; v /= 2; }
  for (int r : {5, 3, 7})
    while (v % r == 0 && np < 16) { radix[np++] = r; v /= r; }
  return v == 1 ? np : 0;
}

static constexpr int64_t kMaxMixedN = 8192;

// Mixed-radix plan tables: pass by pass, W_{ns R}^{k r} for k < ns, 1 <= r < R
// ([k][r-1]), computed in double and rounded once; and the packed radix codes.
static int mixed_code(int r) {
  switch (r) {
    case 2: return 0;
    case 3: return 1;
    case 4: return 2;
    case 5: return 3;
    case 7: return 4;
    case 8: return 5;
    default: return 6;  // 16
  }
}

static int make_mixed_tables(trnfft_plan_s* p) {
  std::vector<float2> t;
  long long ns = 1;
  p->codes = 0;
  for (int q = 0; q < p->npass; ++q) {
    const int R = p->radix[q];
    p->codes |= (unsigned long long)mixed_code(R) << (3 * q);
    // block of pass q: entry (r - 1) * ns + k = W_{ns R}^{k r} (r-major: the butterflies of a
    // warp, consecutive k, read consecutive entries for each r)
    for (int r = 1; r < R; ++r)
      for (long long k = 0; k < ns; ++k) {
        const long long e = (k * r) % (ns * R);
        const double a = -2.0 * M_PI * (double)e / (double)(ns * R);
        t.push_back(make_float2((float)std::cos(a), (float)std::sin(a)));
      }
    ns *= R;
  }
  if (t.empty()) t.push_back(make_float2(1.f, 0.f));
  cudaError_t e = cudaMalloc(&p->twn, sizeof(float2) * t.size());
  if (e == cudaSuccess) e = cudaMemcpy(p->twn, t.data(), sizeof(float2) * t.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(TRNFFT_ALLOC_FAILED, "plan_create: mixed-radix table: %s", cudaGetErrorString(e));
  return TRNFFT_SUCCESS;
}

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
  } else if (n <= kMaxMixedN && (p->npass = mixed_schedule(n, p->radix)) > 0 &&
             !getenv("TRNFFT_B200_NO_MIXED")) {
    // 7-smooth: direct mixed radix (the Bluestein length is kept for the fp64 path)
    p->algorithm = TRNFFT_ALG_MIXED;
    int64_t v = 2 * n - 2;
    int bl = 0;
    while (v >> bl) ++bl;
    p->m = int64_t(1) << bl;
    p->logm = bl;
    int rc2 = make_mixed_tables(p);
    if (rc2) {
      trnfft_plan_destroy(p);
      return rc2;
    }
  } else {
    p->algorithm = TRNFFT_ALG_BLUESTEIN;
    p->npass = 0;
    int64_t v = 2 * n - 2;
    int bl = 0;
    while (v >> bl) ++bl;
    p->m = int64_t(1) << bl;
    p->logm = bl;
    if (bl <= kMaxBluesteinLogM) {
      int rc2 = make_bluestein_tables(p);
      if (rc2) {
        trnfft_plan_destroy(p);
        return rc2;
      }
    } else if (bl <= kMaxMultipassLog) {
      int rc2 = make_large_bluestein(p);
      if (rc2) {
        trnfft_plan_destroy(p);
        return rc2;
      }
    }
  }
  if (p->logn > kMaxColLog && p->logn <= kMaxMultipassLog) {
    int rc3 = make_twiddle_tables(p);
    if (rc3) {
      trnfft_plan_destroy(p);
      return rc3;
    }
  }
  *plan = p;
  return TRNFFT_SUCCESS;
}

int trnfft_device_status(int device, int* status, int clear) {
  if (!status) return fail(TRNFFT_INVALID_VALUE, "device_status: null status pointer");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "device_status: cannot select device %d", device);
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(int));
  if (e == cudaSuccess && clear && v) {
    const int z = 0;
    e = cudaMemcpyToSymbol(g_dev_status, &z, sizeof(int));
  }
  if (e != cudaSuccess) return cuda_fail(e, "device_status");
  *status = v;
  return TRNFFT_SUCCESS;
}

int trnfft_plan_destroy(trnfft_plan_t plan) {
  if (!plan) return TRNFFT_SUCCESS;
  if (plan->chirp || plan->H) {
    DeviceGuard g(plan->device);
    if (plan->chirp) cudaFree(plan->chirp);
    if (plan->H) cudaFree(plan->H);
  }
  if (plan->tw_hi || plan->tw_lo || plan->Hr || plan->Hi) {
    DeviceGuard g(plan->device);
    if (plan->tw_hi) cudaFree(plan->tw_hi);
    if (plan->tw_lo) cudaFree(plan->tw_lo);
    if (plan->Hr) cudaFree(plan->Hr);
    if (plan->Hi) cudaFree(plan->Hi);
  }
  if (plan->twn) {
    DeviceGuard g(plan->device);
    cudaFree(plan->twn);
  }
  if (plan->tw64_hi || plan->tw64_lo || plan->chirp64 || plan->H64) {
    DeviceGuard g(plan->device);
    if (plan->tw64_hi) cudaFree(plan->tw64_hi);
    if (plan->tw64_lo) cudaFree(plan->tw64_lo);
    if (plan->chirp64) cudaFree(plan->chirp64);
    if (plan->H64) cudaFree(plan->H64);
  }
  if (plan->sub64) trnfft_plan_destroy(plan->sub64);
  if (plan->sub) trnfft_plan_destroy(plan->sub);
  delete plan;
  return TRNFFT_SUCCESS;
}

int trnfft_plan_query(trnfft_plan_t plan, int* algorithm, int64_t* padded_n, int64_t batch,
                      int64_t* work_bytes) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "plan_query: null plan");
  if (algorithm) *algorithm = plan->algorithm;
  if (padded_n) *padded_n = plan->algorithm == TRNFFT_ALG_BLUESTEIN ? plan->m : plan->n;
  // An in-place multi-pass transform needs a work area (a copy of the input);
  // a multi-pass Bluestein transform (m > 16384) always needs two m-point buffers.
  if (work_bytes) {
    if (plan->algorithm == TRNFFT_ALG_MULTIPASS)
      *work_bytes = (int64_t)(2 * sizeof(float)) * plan->n * batch;  // needed only above 16384 points
    else if (plan->algorithm == TRNFFT_ALG_BLUESTEIN && plan->sub)
      *work_bytes = (int64_t)(4 * sizeof(float)) * plan->m * batch;
    else
      *work_bytes = 0;
  }
  return TRNFFT_SUCCESS;
}

// [a, a + abytes) and [b, b + bbytes) share a byte
static bool ranges_overlap(const void* a, size_t abytes, const void* b, size_t bbytes) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + bbytes && y < x + abytes;
}

// How the output planes of a transform over `count` floats per plane relate
// to its input planes: 0 disjoint, 1 exactly in place (out_re == in_re and
// out_im == in_im), 2 any other overlap.
static int alias_kind(const float* in_re, const float* in_im, const float* out_re, const float* out_im,
                      size_t count) {
  const size_t b = count * sizeof(float);
  const bool any = ranges_overlap(in_re, b, out_re, b) || ranges_overlap(in_re, b, out_im, b) ||
                   ranges_overlap(in_im, b, out_re, b) || ranges_overlap(in_im, b, out_im, b);
  if (!any) return 0;
  return (in_re == out_re && in_im == out_im) ? 1 : 2;
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
  // One-pass kernels read each row whole before writing it: exactly in place
  // is fine, any other overlap of input and output planes is not.
  if (plan->algorithm != TRNFFT_ALG_MULTIPASS &&
      alias_kind(in_re, in_im, out_re, out_im, (size_t)n * (size_t)batch) == 2)
    return fail(TRNFFT_INVALID_VALUE, "exec_c2c: input and output planes overlap without being the same planes");
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
      // The bulk-copy (TMA) fed persistent kernel is opt-in
      // (TRNFFT_B200_ROW_KERNEL=tma): on B200 the plain kernel measured faster
      // because the row transform is bound by shared-memory instruction issue.
      static const bool use_tma = [] {
        const char* v = getenv("TRNFFT_B200_ROW_KERNEL");
        return v && strcmp(v, "tma") == 0;
      }();
      if (use_tma && rows_c2c_tma_ok(plan->logn, a))
        e = launch_rows_c2c_tma(plan->logn, inverse != 0, a, st);
      else
        e = launch_rows_c2c(plan->logn, inverse != 0, a, st);
      break;
    }
    case TRNFFT_ALG_MULTIPASS: {
      if (plan->logn > kMaxMultipassLog)
        return fail(TRNFFT_UNSUPPORTED, "exec_c2c: n=2^%d above the supported 2^%d", plan->logn, kMaxMultipassLog);
      const float* xr = in_re;
      const float* xi = in_im;
      // Rows of up to 16384 points are one pass in which every block reads a
      // whole row before writing it, so an exactly in-place call needs no copy.
      // More passes scatter rows across the whole transform: then any overlap
      // of input and output (in place, or planes that partly overlap) first
      // copies the input into the work area.
      const int ak = alias_kind(in_re, in_im, out_re, out_im, (size_t)n * (size_t)batch);
      if (ak == 2 || (ak == 1 && plan->logn > kMaxRowBlockLog)) {
        if (!work)
          return fail(TRNFFT_INVALID_VALUE, "exec_c2c: n=%lld with overlapping input and output needs the work area",
                      (long long)n);
        float* w = static_cast<float*>(work);
        const size_t cnt = (size_t)n * (size_t)batch;
        if (ranges_overlap(w, 2 * cnt * sizeof(float), in_re, cnt * sizeof(float)) ||
            ranges_overlap(w, 2 * cnt * sizeof(float), in_im, cnt * sizeof(float)) ||
            ranges_overlap(w, 2 * cnt * sizeof(float), out_re, cnt * sizeof(float)) ||
            ranges_overlap(w, 2 * cnt * sizeof(float), out_im, cnt * sizeof(float)))
          return fail(TRNFFT_INVALID_VALUE, "exec_c2c: the work area overlaps the data");
        e = cudaMemcpyAsync(w, in_re, cnt * sizeof(float), cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(w + cnt, in_im, cnt * sizeof(float), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) break;
        xr = w;
        xi = w + cnt;
      }
      e = run_rows_multipass(plan, xr, xi, out_re, out_im, batch, inverse != 0, st);
      break;
    }
    case TRNFFT_ALG_MIXED: {
      MixedArgs a;
      std::memset(&a, 0, sizeof a);
      a.xr = in_re; a.xi = in_im; a.yr = out_re; a.yi = out_im;
      a.batch = batch; a.n = (int)n; a.npass = plan->npass;
      a.codes = plan->codes;
      a.tw = plan->twn;
      a.scale = inverse ? (float)(1.0 / (double)n) : 1.f;
      e = launch_mixed(0, inverse != 0, a, st);
      break;
    }
    case TRNFFT_ALG_BLUESTEIN: {
      if (plan->sub) {
        if (!work) return fail(TRNFFT_INVALID_VALUE, "exec_c2c: Bluestein n=%lld needs the work area", (long long)n);
        const size_t mb = (size_t)plan->m * (size_t)batch;
        float* ar = static_cast<float*>(work);
        float *ai = ar + mb, *br = ai + mb, *bi = br + mb;
        const bool inv = inverse != 0;
        e = launch_blue_pre(in_re, in_im, plan->chirp, ar, ai, batch, n, plan->m, inv, st);
        if (e == cudaSuccess && run_rows_multipass_plan(plan->sub, ar, ai, br, bi, batch, false, st))
          return TRNFFT_CUDA_ERROR;
        if (e == cudaSuccess) e = launch_blue_mul(br, bi, plan->Hr, plan->Hi, batch, plan->m, inv, st);
        if (e == cudaSuccess && run_rows_multipass_plan(plan->sub, br, bi, ar, ai, batch, true, st))
          return TRNFFT_CUDA_ERROR;
        if (e == cudaSuccess)
          e = launch_blue_post(ar, ai, plan->chirp, out_re, out_im, batch, n, plan->m, inv,
                               inv ? (float)(1.0 / (double)n) : 1.f, st);
        break;
      }
      if (!plan->H)
        return fail(TRNFFT_UNSUPPORTED, "exec_c2c: Bluestein length n=%lld (padded %lld) above the supported "
                    "2^%d", (long long)n, (long long)plan->m, kMaxMultipassLog);
      BlueArgs a{in_re, in_im, out_re, out_im, batch, (int)n, plan->chirp, plan->H};
      e = launch_bluestein(plan->logm, 0, inverse != 0, a, st);
      break;
    }
    default:
      return fail(TRNFFT_UNSUPPORTED, "exec_c2c: n=%lld not supported yet", (long long)n);
  }
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_c2c_axis(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out_re,
                         float* out_im, int64_t outer, int64_t inner, int inverse, void* work, void* stream) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis: null plan");
  if (outer < 0 || inner < 1) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis: bad outer/inner");
  if (outer == 0) return TRNFFT_SUCCESS;
  if (inner == 1) return trnfft_exec_c2c(plan, in_re, in_im, out_re, out_im, outer, inverse, work, stream);
  int rc = check_ptrs("exec_c2c_axis", {in_re, in_im, out_re, out_im}, 4);
  if (rc) return rc;
  if (plan->algorithm == TRNFFT_ALG_COPY) {
    return trnfft_exec_c2c(plan, in_re, in_im, out_re, out_im, outer * inner, inverse, work, stream);
  }
  if (plan->logn < 1 || plan->logn > 2 * kMaxColLog)
    return fail(TRNFFT_UNSUPPORTED, "exec_c2c_axis: n=%lld (power of two up to 2^20 only)", (long long)plan->n);
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2c_axis: cannot select device %d", plan->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const float* xr = in_re;
  const float* xi = in_im;
  cudaError_t e = cudaSuccess;
  if (plan->logn > kMaxColLog && (in_re == out_re || in_im == out_im)) {
    if (!work) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis: in-place n=%lld needs the work area", (long long)plan->n);
    float* w = static_cast<float*>(work);
    const size_t cnt = (size_t)plan->n * outer * inner;
    e = cudaMemcpyAsync(w, in_re, cnt * sizeof(float), cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w + cnt, in_im, cnt * sizeof(float), cudaMemcpyDeviceToDevice, st);
    xr = w;
    xi = w + cnt;
  }
  if (e == cudaSuccess) e = run_axis(plan, xr, xi, out_re, out_im, outer, inner, inverse != 0, st);
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c_axis");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_stft(trnfft_plan_t plan, const float* signal, int64_t batch, int64_t length, int64_t hop,
                     const float* window, int center, int pad_mode, int normalized, int onesided,
                     int64_t frames, float* out_re, float* out_im, void* stream) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_stft: null plan");
  const int64_t n = plan->n;
  if (plan->logn < 2 || plan->logn > 13)
    return fail(TRNFFT_UNSUPPORTED, "exec_stft: n_fft=%lld (power of two 4..8192 only)", (long long)n);
  if (batch < 0 || length < 1 || hop < 1) return fail(TRNFFT_INVALID_VALUE, "exec_stft: bad batch/length/hop");
  if (pad_mode < 0 || pad_mode > 3) return fail(TRNFFT_INVALID_VALUE, "exec_stft: bad pad_mode %d", pad_mode);
  const int64_t pad = center ? n / 2 : 0;
  if (center && pad_mode == 0 && pad >= length)
    return fail(TRNFFT_INVALID_VALUE, "exec_stft: reflect padding %lld needs length > %lld", (long long)pad,
                (long long)pad);
  const int64_t lp = length + 2 * pad;
  if (lp < n) return fail(TRNFFT_INVALID_VALUE, "exec_stft: signal shorter than n_fft");
  const int64_t nf = 1 + (lp - n) / hop;
  if (frames != nf) return fail(TRNFFT_INVALID_VALUE, "exec_stft: frames=%lld, expected %lld", (long long)frames, (long long)nf);
  if (batch == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("exec_stft", {signal, window, out_re, out_im}, 4);
  if (rc) return rc;
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_stft: cannot select device %d", plan->device);
  StftArgs a{signal, window, out_re, out_im, batch, length, nf, hop, pad, pad_mode, onesided ? 1 : 0,
             normalized ? (float)(1.0 / std::sqrt((double)n)) : 1.f};
  cudaError_t e = launch_stft(plan->logn, a, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "exec_stft");
  return TRNFFT_SUCCESS;
}

int64_t trnfft_complex_linear_work_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return -1;
  return (int64_t)sizeof(float) * 6 * (M + N) * K;
}

// The complex linear map from split operands in the three-product form
//   P1 = Xr Wr^T,  P2 = Xi Wi^T,  P3 = (Xr + Xi)(Wr + Wi)^T,
//   Re = P1 - P2,  Im = P3 - P1 - P2,
// three tcgen05 GEMMs of three TF32 segments each (hi*hi + hi*lo + lo*hi), 9 tensor-core products
// instead of the 12 of the four-product form.  The first two GEMMs write P1 into yr and P2 into
// yi; the third combines them in its epilogue (and adds the biases).
// xs / ws: hi, lo of the real part, the imaginary part and their sum (six planes each).
// TRNFFT_B200_LINEAR_4M=1 selects the four-product form (two GEMMs of six segments: Re = Xr Wr^T -
// Xi Wi^T, Im = Xr Wi^T + Xi Wr^T), for measurement.
static bool linear_four_products() {
  static const bool v = [] {
    const char* e = getenv("TRNFFT_B200_LINEAR_4M");
    return e != nullptr && atoi(e) == 1;
  }();
  return v;
}

static int complex_linear_gemms4(float* const xs[6], const float* const ws[6], const float* br, const float* bi,
                                 float* yr, float* yi, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  GemmArgs ga;
  std::memset(&ga, 0, sizeof ga);
  for (int i = 0; i < 4; ++i) {
    ga.A[i] = xs[i];
    ga.B[i] = ws[i];
  }
  ga.na = 4;
  ga.nb = 4;
  ga.M = M; ga.N = N; ga.K = K; ga.lda = K; ga.ldb = K; ga.ldc = N;
  ga.nseg = 6;
  const int ra[6] = {0, 0, 1, 2, 2, 3}, rb[6] = {0, 1, 0, 2, 3, 2}, rn[6] = {0, 0, 0, 1, 1, 1};
  for (int i = 0; i < 6; ++i) { ga.seg_a[i] = ra[i]; ga.seg_b[i] = rb[i]; ga.seg_neg[i] = rn[i]; }
  ga.C = yr; ga.bias = br;
  cudaError_t e = launch_gemm_tf32(ga, st);
  if (e != cudaSuccess) return cuda_fail(e, "complex_linear: real part");
  const int ia[6] = {0, 0, 1, 2, 2, 3}, ib[6] = {2, 3, 2, 0, 1, 0};
  for (int i = 0; i < 6; ++i) { ga.seg_a[i] = ia[i]; ga.seg_b[i] = ib[i]; ga.seg_neg[i] = 0; }
  ga.C = yi; ga.bias = bi;
  e = launch_gemm_tf32(ga, st);
  if (e != cudaSuccess) return cuda_fail(e, "complex_linear: imaginary part");
  return TRNFFT_SUCCESS;
}

static int complex_linear_gemms(float* const xs[6], const float* const ws[6], const float* br, const float* bi,
                                float* yr, float* yi, int64_t M, int64_t N, int64_t K, cudaStream_t st) {
  if (linear_four_products()) return complex_linear_gemms4(xs, ws, br, bi, yr, yi, M, N, K, st);
  GemmArgs ga;
  std::memset(&ga, 0, sizeof ga);
  ga.na = 2;
  ga.nb = 2;
  ga.M = M; ga.N = N; ga.K = K; ga.lda = K; ga.ldb = K; ga.ldc = N;
  ga.nseg = 3;
  const int sa[3] = {0, 0, 1}, sb[3] = {0, 1, 0};
  for (int i = 0; i < 3; ++i) { ga.seg_a[i] = sa[i]; ga.seg_b[i] = sb[i]; ga.seg_neg[i] = 0; }
  static const char* what[3] = {"complex_linear: Xr Wr^T", "complex_linear: Xi Wi^T",
                                "complex_linear: (Xr+Xi)(Wr+Wi)^T"};
  for (int p = 0; p < 3; ++p) {
    ga.A[0] = xs[2 * p]; ga.A[1] = xs[2 * p + 1];
    ga.B[0] = ws[2 * p]; ga.B[1] = ws[2 * p + 1];
    ga.C = p == 1 ? yi : yr;
    ga.bias = p == 2 ? br : nullptr;
    ga.epi = p == 2 ? 1 : 0;
    ga.C2 = p == 2 ? yi : nullptr;
    ga.bias2 = p == 2 ? bi : nullptr;
    cudaError_t e = launch_gemm_tf32(ga, st);
    if (e != cudaSuccess) return cuda_fail(e, what[p]);
  }
  return TRNFFT_SUCCESS;
}

// hi / lo of x's real part, imaginary part and their sum into xs[0..5]
static cudaError_t split_complex(const float* xr, const float* xi, float* const xs[6], long long count,
                                 cudaStream_t st) {
  cudaError_t e = launch_split_tf32(xr, xs[0], xs[1], count, 1.f, st);
  if (e == cudaSuccess) e = launch_split_tf32(xi, xs[2], xs[3], count, 1.f, st);
  if (e == cudaSuccess) e = launch_split_tf32_sum(xr, xi, xs[4], xs[5], count, st);
  return e;
}

int trnfft_complex_linear(const float* xr, const float* xi, const float* wr, const float* wi, const float* br,
                          const float* bi, float* yr, float* yi, int64_t M, int64_t N, int64_t K, void* work,
                          int device, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(TRNFFT_INVALID_VALUE, "complex_linear: negative size");
  if (M == 0 || N == 0) return TRNFFT_SUCCESS;
  if (K % 4) return fail(TRNFFT_UNSUPPORTED, "complex_linear: K=%lld must be a multiple of 4", (long long)K);
  int rc = check_ptrs("complex_linear", {xr, xi, wr, wi, yr, yi, work}, 16);
  if (rc) return rc;
  if ((br == nullptr) != (bi == nullptr)) return fail(TRNFFT_INVALID_VALUE, "complex_linear: give both biases or none");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "complex_linear: cannot select device %d", device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* w = static_cast<float*>(work);
  const size_t mk = (size_t)M * K, nk = (size_t)N * K;
  float* xs[6];
  float* wsp[6];
  for (int i = 0; i < 6; ++i) {
    xs[i] = w + i * mk;
    wsp[i] = w + 6 * mk + i * nk;
  }
  cudaError_t e = split_complex(xr, xi, xs, (long long)mk, st);
  if (e == cudaSuccess) e = split_complex(wr, wi, wsp, (long long)nk, st);
  if (e != cudaSuccess) return cuda_fail(e, "complex_linear: split");
  const float* ws[6] = {wsp[0], wsp[1], wsp[2], wsp[3], wsp[4], wsp[5]};
  return complex_linear_gemms(xs, ws, br, bi, yr, yi, M, N, K, st);
}

int trnfft_split_tf32(const float* src, float* hi, float* lo, int64_t count, int device, void* stream) {
  if (count < 0) return fail(TRNFFT_INVALID_VALUE, "split_tf32: negative count");
  if (count == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("split_tf32", {src, hi, lo}, 16);
  if (rc) return rc;
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "split_tf32: cannot select device %d", device);
  cudaError_t e = launch_split_tf32(src, hi, lo, (long long)count, 1.f, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "split_tf32");
  return TRNFFT_SUCCESS;
}

int trnfft_split_tf32_sum(const float* a, const float* b, float* hi, float* lo, int64_t count, int device,
                          void* stream) {
  if (count < 0) return fail(TRNFFT_INVALID_VALUE, "split_tf32_sum: negative count");
  if (count == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("split_tf32_sum", {a, b, hi, lo}, 16);
  if (rc) return rc;
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "split_tf32_sum: cannot select device %d", device);
  cudaError_t e = launch_split_tf32_sum(a, b, hi, lo, (long long)count, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "split_tf32_sum");
  return TRNFFT_SUCCESS;
}

int trnfft_complex_linear_presplit(const float* xr, const float* xi, const float* w_split, const float* br,
                                   const float* bi, float* yr, float* yi, int64_t M, int64_t N, int64_t K, void* work,
                                   int device, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(TRNFFT_INVALID_VALUE, "complex_linear_presplit: negative size");
  if (M == 0 || N == 0) return TRNFFT_SUCCESS;
  if (K % 4) return fail(TRNFFT_UNSUPPORTED, "complex_linear_presplit: K=%lld must be a multiple of 4", (long long)K);
  int rc = check_ptrs("complex_linear_presplit", {xr, xi, w_split, yr, yi, work}, 16);
  if (rc) return rc;
  if ((br == nullptr) != (bi == nullptr))
    return fail(TRNFFT_INVALID_VALUE, "complex_linear_presplit: give both biases or none");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "complex_linear_presplit: cannot select device %d", device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float* w = static_cast<float*>(work);
  const size_t mk = (size_t)M * K, nk = (size_t)N * K;
  float* xs[6];
  const float* ws[6];
  for (int i = 0; i < 6; ++i) {
    xs[i] = w + i * mk;
    ws[i] = w_split + i * nk;
  }
  cudaError_t e = split_complex(xr, xi, xs, (long long)mk, st);
  if (e != cudaSuccess) return cuda_fail(e, "complex_linear_presplit: split");
  return complex_linear_gemms(xs, ws, br, bi, yr, yi, M, N, K, st);
}

int trnfft_exec_c2c_axis_tw(trnfft_plan_t plan, trnfft_plan_t tw_plan, const float* in_re, const float* in_im,
                            float* out_re, float* out_im, int64_t outer, int64_t inner, int64_t ld_in,
                            int64_t ld_out, int inverse, int64_t col_offset, void* stream) {
  if (!plan || !tw_plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: null plan");
  if (outer < 0 || inner < 1 || col_offset < 0) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: bad sizes");
  if (ld_in == 0) ld_in = inner;
  if (ld_out == 0) ld_out = inner;
  if (ld_in < inner || ld_out < inner) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: ld < inner");
  if (outer == 0) return TRNFFT_SUCCESS;
  if (plan->logn < 1 || plan->logn > 2 * kMaxColLog)
    return fail(TRNFFT_UNSUPPORTED, "exec_c2c_axis_tw: n=%lld (power of two up to 2^20 only)", (long long)plan->n);
  if (!tw_plan->tw_hi) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: twiddle plan must be a power of two > 1024");
  if (in_re == out_re || in_im == out_im)
    return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: out of place only");
  if (tw_plan->device != plan->device) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_axis_tw: plans on different devices");
  int rc = check_ptrs("exec_c2c_axis_tw", {in_re, in_im, out_re, out_im}, 4);
  if (rc) return rc;
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2c_axis_tw: cannot select device %d", plan->device);
  cudaError_t e = run_axis(plan, in_re, in_im, out_re, out_im, outer, inner, inverse != 0,
                           reinterpret_cast<cudaStream_t>(stream), tw_plan, col_offset, ld_in, ld_out);
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c_axis_tw");
  return TRNFFT_SUCCESS;
}

int trnfft_xbuf_alloc(int device, int64_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes <= 0) return fail(TRNFFT_INVALID_VALUE, "xbuf_alloc: bad arguments");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "xbuf_alloc: cannot select device %d", device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return fail(TRNFFT_ALLOC_FAILED, "xbuf_alloc: %s", cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "xbuf_alloc: cudaIpcGetMemHandle");
  }
  std::memcpy(ipc_handle, &h, sizeof h);
  *ptr = p;
  return TRNFFT_SUCCESS;
}

int trnfft_xbuf_free(int device, void* ptr) {
  DeviceGuard g(device);
  if (ptr) cudaFree(ptr);
  return TRNFFT_SUCCESS;
}

int trnfft_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int trnfft_ipc_open(int device, const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return fail(TRNFFT_INVALID_VALUE, "ipc_open: null argument");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "ipc_open: cannot select device %d", device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof h);
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_open: cudaIpcOpenMemHandle");
  return TRNFFT_SUCCESS;
}

int trnfft_ipc_close(int device, void* ptr) {
  DeviceGuard g(device);
  if (ptr) cudaIpcCloseMemHandle(ptr);
  return TRNFFT_SUCCESS;
}

int trnfft_exec_fourstep_scatter(trnfft_plan_t plan, trnfft_plan_t tw_plan, const float* in_re, const float* in_im,
                                 int64_t inner, int64_t ld_in, int inverse, int64_t col_offset, int npeers,
                                 float* const* peer_re, float* const* peer_im, int64_t rows_per_peer,
                                 int64_t peer_ld, int64_t peer_col0, void* work, void* stream) {
  if (!plan || !tw_plan || !peer_re || !peer_im) return fail(TRNFFT_INVALID_VALUE, "fourstep_scatter: null argument");
  if (npeers < 1 || npeers > 8) return fail(TRNFFT_INVALID_VALUE, "fourstep_scatter: 1..8 peers");
  if (plan->logn < 1 || plan->logn > 2 * kMaxColLog || !tw_plan->tw_hi)
    return fail(TRNFFT_UNSUPPORTED, "fourstep_scatter: column length must be a power of two <= 2^20");
  if (inner < 1 || ld_in < inner || rows_per_peer < 1 || rows_per_peer * npeers != plan->n ||
      peer_ld < peer_col0 + inner)
    return fail(TRNFFT_INVALID_VALUE, "fourstep_scatter: inconsistent sizes");
  int rc = check_ptrs("fourstep_scatter", {in_re, in_im}, 4);
  if (rc) return rc;
  ScatterSpec sc;
  sc.npeers = npeers;
  for (int q = 0; q < npeers; ++q) {
    if (!peer_re[q] || !peer_im[q]) return fail(TRNFFT_INVALID_VALUE, "fourstep_scatter: null peer buffer");
    sc.re[q] = peer_re[q];
    sc.im[q] = peer_im[q];
  }
  sc.rows_log = 0;
  while ((int64_t(1) << sc.rows_log) < rows_per_peer) ++sc.rows_log;
  // The scatter pass runs as a persistent grid of 4 blocks per SM looping over
  // its tiles: on B200 (2 GPUs, 2^30) this measured 7.6 ms per transform
  // against 9.9 ms with one block per tile, the peer stores then keep fewer
  // writes in flight.  TRNFFT_B200_SCATTER_BLOCKS overrides the cap (0: none).
  {
    const char* v = getenv("TRNFFT_B200_SCATTER_BLOCKS");
    if (v) {
      sc.max_blocks = atoll(v);
    } else {
      int sms = 0;
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, plan->device) != cudaSuccess) sms = 0;
      sc.max_blocks = 4LL * sms;
    }
  }
  sc.ld = peer_ld;
  sc.col0 = peer_col0;
  float* tr = nullptr;
  float* ti = nullptr;
  if (plan->logn > kMaxColLog) {
    if (!work) return fail(TRNFFT_INVALID_VALUE, "fourstep_scatter: n > 1024 needs the work area");
    tr = static_cast<float*>(work);
    ti = tr + (size_t)plan->n * inner;
  }
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "fourstep_scatter: cannot select device %d", plan->device);
  cudaError_t e = run_axis(plan, in_re, in_im, tr, ti, 1, inner, inverse != 0, reinterpret_cast<cudaStream_t>(stream),
                           tw_plan, col_offset, ld_in, inner, &sc);
  if (e != cudaSuccess) return cuda_fail(e, "fourstep_scatter");
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
  } else if (plan->algorithm == TRNFFT_ALG_MIXED) {
    int rc = check_ptrs("exec_r2c", {in, out_re, out_im}, 4);
    if (rc) return rc;
    MixedArgs a;
    std::memset(&a, 0, sizeof a);
    a.xr = in; a.yr = out_re; a.yi = out_im;
    a.batch = batch; a.n = (int)n; a.npass = plan->npass;
    a.codes = plan->codes;
    a.tw = plan->twn;
    a.scale = 1.f;
    e = launch_mixed(1, false, a, st);
  } else if (plan->algorithm == TRNFFT_ALG_BLUESTEIN && plan->H) {
    int rc = check_ptrs("exec_r2c", {in, out_re, out_im}, 4);
    if (rc) return rc;
    BlueArgs a{in, nullptr, out_re, out_im, batch, (int)n, plan->chirp, plan->H};
    e = launch_bluestein(plan->logm, 1, false, a, st);
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
  } else if (plan->algorithm == TRNFFT_ALG_MIXED) {
    int rc = check_ptrs("exec_c2r", {in_re, in_im, out}, 4);
    if (rc) return rc;
    MixedArgs a;
    std::memset(&a, 0, sizeof a);
    a.xr = in_re; a.xi = in_im; a.yr = out;
    a.batch = batch; a.n = (int)n; a.npass = plan->npass;
    a.codes = plan->codes;
    a.tw = plan->twn;
    a.scale = (float)(1.0 / (double)n);
    e = launch_mixed(2, true, a, st);
  } else if (plan->algorithm == TRNFFT_ALG_BLUESTEIN && plan->H) {
    int rc = check_ptrs("exec_c2r", {in_re, in_im, out}, 4);
    if (rc) return rc;
    BlueArgs a{in_re, in_im, out, nullptr, batch, (int)n, plan->chirp, plan->H};
    e = launch_bluestein(plan->logm, 2, true, a, st);
  } else {
    return fail(TRNFFT_UNSUPPORTED, "exec_c2r: n=%lld not supported yet", (long long)n);
  }
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2r");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_istft(trnfft_plan_t plan, const float* in_re, const float* in_im, int64_t batch, int64_t frames,
                      int64_t hop, const float* window, int center, int normalized, int onesided, int64_t out_len,
                      float* out, void* stream) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_istft: null plan");
  const int64_t n = plan->n;
  if (plan->logn < 2 || plan->logn > 13)
    return fail(TRNFFT_UNSUPPORTED, "exec_istft: n_fft=%lld (power of two 4..8192 only)", (long long)n);
  if (batch < 0 || frames < 1 || hop < 1 || out_len < 0)
    return fail(TRNFFT_INVALID_VALUE, "exec_istft: bad batch/frames/hop/out_len");
  if (batch == 0 || out_len == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("exec_istft", {in_re, in_im, window, out}, 4);
  if (rc) return rc;
  const int64_t nbins = onesided ? n / 2 + 1 : n;
  const size_t in_bytes = sizeof(float) * (size_t)batch * (size_t)nbins * (size_t)frames;
  const size_t out_bytes = sizeof(float) * (size_t)batch * (size_t)out_len;
  if (ranges_overlap(out, out_bytes, in_re, in_bytes) || ranges_overlap(out, out_bytes, in_im, in_bytes))
    return fail(TRNFFT_INVALID_VALUE, "exec_istft: the output overlaps the input spectrum");
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_istft: cannot select device %d", plan->device);
  IstftArgs a;
  std::memset(&a, 0, sizeof a);
  a.xr = in_re;
  a.xi = in_im;
  a.window = window;
  a.y = out;
  a.batch = batch;
  a.frames = frames;
  a.hop = hop;
  a.out_len = out_len;
  a.pad_front = center ? n / 2 : 0;
  a.exp_len = n + (frames - 1) * hop;
  a.total = a.exp_len > a.pad_front + out_len ? a.exp_len : a.pad_front + out_len;
  if (a.total >= (1LL << 31) - 16384)
    return fail(TRNFFT_UNSUPPORTED, "exec_istft: signals of 2^31 samples or more are not supported");
  if (hop > 8192) return fail(TRNFFT_UNSUPPORTED, "exec_istft: hop %lld above 8192 samples", (long long)hop);
  a.onesided = onesided ? 1 : 0;
  a.scale = (float)((normalized ? std::sqrt((double)n) : 1.0) / (double)n);
  cudaError_t e = launch_istft(plan->logn, a, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "exec_istft");
  return TRNFFT_SUCCESS;
}

int trnfft_complex_mask_apply(const float* mask_re, const float* mask_im, int64_t mask_count, const float* spec_re,
                              const float* spec_im, float* out_re, float* out_im, int64_t count, int device,
                              void* stream) {
  if (count < 0 || mask_count < 0) return fail(TRNFFT_INVALID_VALUE, "complex_mask_apply: negative size");
  if (count == 0) return TRNFFT_SUCCESS;
  if (mask_count == 0 || count % mask_count)
    return fail(TRNFFT_INVALID_VALUE, "complex_mask_apply: count %lld is not a multiple of mask_count %lld",
                (long long)count, (long long)mask_count);
  int rc = check_ptrs("complex_mask_apply", {mask_re, mask_im, spec_re, spec_im, out_re, out_im}, 4);
  if (rc) return rc;
  const size_t mb = sizeof(float) * (size_t)mask_count, cb = sizeof(float) * (size_t)count;
  for (const float* o : {out_re, out_im}) {
    const bool mask_ok = !(ranges_overlap(o, cb, mask_re, mb) || ranges_overlap(o, cb, mask_im, mb)) ||
                         (mask_count == count && (o == mask_re || o == mask_im));
    if (!mask_ok) return fail(TRNFFT_INVALID_VALUE, "complex_mask_apply: output overlaps a repeated mask");
  }
  if (ranges_overlap(out_re, cb, out_im, cb))
    return fail(TRNFFT_INVALID_VALUE, "complex_mask_apply: output planes overlap");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "complex_mask_apply: cannot select device %d", device);
  cudaError_t e = launch_cmul(mask_re, mask_im, mask_count, spec_re, spec_im, out_re, out_im, count,
                              reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "complex_mask_apply");
  return TRNFFT_SUCCESS;
}

int trnfft_plan_enable_f64(trnfft_plan_t plan) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "plan_enable_f64: null plan");
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "plan_enable_f64: cannot select device %d", plan->device);
  std::lock_guard<std::mutex> lk(g_f64_mu);
  return enable_f64_locked(plan);
}

int trnfft_plan_query_f64(trnfft_plan_t plan, int64_t batch, int64_t* work_bytes) {
  if (!plan || !work_bytes || batch < 0) return fail(TRNFFT_INVALID_VALUE, "plan_query_f64: bad arguments");
  *work_bytes = f64_work_bytes(plan, batch);
  return TRNFFT_SUCCESS;
}

int trnfft_exec_c2c_f64(trnfft_plan_t plan, const double* in_re, const double* in_im, double* out_re,
                        double* out_im, int64_t batch, int inverse, void* work, void* stream) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: null plan");
  if (batch < 0) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: negative batch");
  if (!plan->f64) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: call trnfft_plan_enable_f64 on the plan first");
  if (batch == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("exec_c2c_f64", {in_re, in_im, out_re, out_im}, 8);
  if (rc) return rc;
  const size_t cnt = (size_t)plan->n * (size_t)batch;
  const size_t b = cnt * sizeof(double);
  const bool partial = (ranges_overlap(in_re, b, out_re, b) || ranges_overlap(in_re, b, out_im, b) ||
                        ranges_overlap(in_im, b, out_re, b) || ranges_overlap(in_im, b, out_im, b)) &&
                       !(in_re == out_re && in_im == out_im);
  if (partial) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: input and output planes partly overlap");
  const int64_t wb = f64_work_bytes(plan, batch);
  if (wb > 0) {
    if (!work) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: n=%lld needs a work area of %lld bytes",
                           (long long)plan->n, (long long)wb);
    if (!aligned(work, 16)) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64: work area not 16-byte aligned");
  }
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2c_f64: cannot select device %d", plan->device);
  cudaError_t e = run_f64(plan, in_re, in_im, out_re, out_im, batch, inverse != 0, static_cast<double*>(work),
                          reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c_f64");
  return TRNFFT_SUCCESS;
}

int trnfft_exec_c2c_f64_f32io(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out_re,
                              float* out_im, int64_t batch, int inverse, void* work, void* stream) {
  if (!plan) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: null plan");
  if (batch < 0) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: negative batch");
  if (!plan->f64)
    return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: call trnfft_plan_enable_f64 on the plan first");
  if (batch == 0) return TRNFFT_SUCCESS;
  int rc = check_ptrs("exec_c2c_f64_f32io", {in_re, in_im, out_re, out_im}, 4);
  if (rc) return rc;
  const size_t b = (size_t)plan->n * (size_t)batch * sizeof(float);
  const bool partial = (ranges_overlap(in_re, b, out_re, b) || ranges_overlap(in_re, b, out_im, b) ||
                        ranges_overlap(in_im, b, out_re, b) || ranges_overlap(in_im, b, out_im, b)) &&
                       !(in_re == out_re && in_im == out_im);
  if (partial) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: input and output planes partly overlap");
  const int64_t wb = f64_work_bytes(plan, batch);
  if (wb > 0) {
    if (!work) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: n=%lld needs a work area of %lld bytes",
                           (long long)plan->n, (long long)wb);
    if (!aligned(work, 16)) return fail(TRNFFT_INVALID_VALUE, "exec_c2c_f64_f32io: work area not 16-byte aligned");
  }
  DeviceGuard g(plan->device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "exec_c2c_f64_f32io: cannot select device %d", plan->device);
  const F32IO io{in_re, in_im, out_re, out_im};
  cudaError_t e = run_f64(plan, nullptr, nullptr, nullptr, nullptr, batch, inverse != 0, static_cast<double*>(work),
                          reinterpret_cast<cudaStream_t>(stream), &io);
  if (e != cudaSuccess) return cuda_fail(e, "exec_c2c_f64_f32io");
  return TRNFFT_SUCCESS;
}

int trnfft_convert_f32_f64(const void* src, void* dst, int64_t count, int to_double, int device, void* stream) {
  if (count < 0 || (count && (!src || !dst))) return fail(TRNFFT_INVALID_VALUE, "convert_f32_f64: bad arguments");
  if (count == 0) return TRNFFT_SUCCESS;
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "convert_f32_f64: cannot select device %d", device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = to_double ? launch_f32_to_f64(static_cast<const float*>(src), static_cast<double*>(dst), count, st)
                            : launch_f64_to_f32(static_cast<const double*>(src), static_cast<float*>(dst), count, st);
  if (e != cudaSuccess) return cuda_fail(e, "convert_f32_f64");
  return TRNFFT_SUCCESS;
}

int trnfft_copy2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                  int device, void* stream) {
  if (dpitch < width || spitch < width || width < 0 || height < 0)
    return fail(TRNFFT_INVALID_VALUE, "copy2d: bad pitch/width/height");
  if (width == 0 || height == 0) return TRNFFT_SUCCESS;
  if (!dst || !src) return fail(TRNFFT_INVALID_VALUE, "copy2d: null pointer");
  DeviceGuard g(device);
  if (!g.ok) return fail(TRNFFT_CUDA_ERROR, "copy2d: cannot select device %d", device);
  cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dpitch, src, (size_t)spitch, (size_t)width, (size_t)height,
                                    cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "copy2d");
  return TRNFFT_SUCCESS;
}

}  // extern "C"
