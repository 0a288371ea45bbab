// Double-precision transforms: the accuracy mode precision="double".
//
// Reference: trnfft/fft_core.py:1306-1309 promotes the whole Bluestein
// pipeline to float64 in "double" mode (cast back at :1372-1374), and
// :1108-1110 runs power-of-two sizes up to 1024 as an fp64 DFT-GEMM on the
// host (_fft_via_gemm_double, :254-298); with float64 tensors its torch
// backend computes everything in float64.  Here every stage runs in fp64 on
// the GPU, on planar double arrays.
//
// One kernel, k_f64_seq, transforms C sequences of L = 2^LOGL <= 4096 points
// per block in shared memory (radix-4 Stockham passes, a final radix-2 when
// LOGL is odd).  Sequence s starts at (s / inner) * outer_stride +
// (s % inner) * cs and its element j sits j * js further on, for input and
// output separately, so the same kernel runs contiguous rows, strided columns
// and transposing stores.  An optional outer twiddle W_Ntw^{(s % inner) * k}
// (two-level fp64 table) multiplies output k: that is the inter-pass twiddle
// of the four-step split N = N1 * N2 used for N > 4096 (pass A over the
// strided columns with the twiddle, pass B over the rows with a transposing
// store, so the result is in natural order).  Bluestein sizes chain
// elementwise chirp kernels around two such transforms of the padded length.
// Twiddles inside a block come from a per-device table W_4096^i in double.
#include <cuda_runtime.h>

#include "kernels.h"

namespace tfb {

constexpr int kTw64Log = 12;
constexpr int kTw64N = 1 << kTw64Log;
__device__ double2 g_tw64[kTw64N];  // W_4096^i = exp(-2 pi i / 4096)^i, uploaded once per device

__device__ __forceinline__ double2 cmul64(double2 a, double2 b) {
  return make_double2(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}

template <bool INV>
__device__ __forceinline__ double2 tw64(int idx) {
  double2 w = g_tw64[idx];
  if (INV) w.y = -w.y;
  return w;
}

constexpr int kF64Threads = 256;

// sequences per block: about 4096 points (64 KB of shared memory), at most 16
template <int LOGL>
struct F64Geom {
  static constexpr int L = 1 << LOGL;
  static constexpr int C = (4096 / L) > 16 ? 16 : (4096 / L);
  static constexpr int NB4 = C * L / 4;  // radix-4 butterflies per pass
  static constexpr int NB2 = C * L / 2;
  static constexpr int BPT4 = (NB4 + kF64Threads - 1) / kF64Threads;
  static constexpr int BPT2 = (NB2 + kF64Threads - 1) / kF64Threads;
  static constexpr size_t smem = (size_t)C * L * sizeof(double2);
};

template <int LOGL, bool INV>
__device__ __forceinline__ void f64_block_fft(double2* sb) {
  using GM = F64Geom<LOGL>;
  constexpr int L = GM::L;
  // radix-4 passes, then radix-2 if LOGL is odd; ns = product of the earlier radices
#pragma unroll 1
  for (int lns = 0; lns + 2 <= LOGL; lns += 2) {
    const int ns = 1 << lns;
    double2 v[GM::BPT4 > 0 ? GM::BPT4 : 1][4];
#pragma unroll
    for (int q = 0; q < GM::BPT4; ++q) {
      const int t = threadIdx.x + q * kF64Threads;
      if (t < GM::NB4) {
        const int c = t / (L / 4), j = t % (L / 4);
#pragma unroll
        for (int r = 0; r < 4; ++r) v[q][r] = sb[c * L + j + r * (L / 4)];
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < GM::BPT4; ++q) {
      const int t = threadIdx.x + q * kF64Threads;
      if (t >= GM::NB4) continue;
      const int c = t / (L / 4), j = t % (L / 4);
      const int k = j & (ns - 1);
      double2 a0 = v[q][0], a1 = v[q][1], a2 = v[q][2], a3 = v[q][3];
      if (ns > 1) {
        // W_{4 ns}^{k r} = W_4096^{k r 4096 / (4 ns)}
        const int step = k << (kTw64Log - lns - 2);
        a1 = cmul64(a1, tw64<INV>(step));
        a2 = cmul64(a2, tw64<INV>(2 * step));
        a3 = cmul64(a3, tw64<INV>(3 * step));
      }
      const double2 s02 = make_double2(a0.x + a2.x, a0.y + a2.y), d02 = make_double2(a0.x - a2.x, a0.y - a2.y);
      const double2 s13 = make_double2(a1.x + a3.x, a1.y + a3.y), d13 = make_double2(a1.x - a3.x, a1.y - a3.y);
      // forward: X1 = d02 - i d13, X3 = d02 + i d13; the inverse swaps the signs
      const double2 md13 = INV ? make_double2(-d13.y, d13.x) : make_double2(d13.y, -d13.x);
      double2* y = sb + c * L;
      const int base = ((j >> lns) << (lns + 2)) + k;
      y[base] = make_double2(s02.x + s13.x, s02.y + s13.y);
      y[base + ns] = make_double2(d02.x + md13.x, d02.y + md13.y);
      y[base + 2 * ns] = make_double2(s02.x - s13.x, s02.y - s13.y);
      y[base + 3 * ns] = make_double2(d02.x - md13.x, d02.y - md13.y);
    }
    __syncthreads();
  }
  if constexpr (LOGL & 1) {
    constexpr int lns = LOGL - 1;
    constexpr int ns = 1 << lns;
    double2 v[GM::BPT2][2];
#pragma unroll
    for (int q = 0; q < GM::BPT2; ++q) {
      const int t = threadIdx.x + q * kF64Threads;
      if (t < GM::NB2) {
        const int c = t / (L / 2), j = t % (L / 2);
        v[q][0] = sb[c * L + j];
        v[q][1] = sb[c * L + j + L / 2];
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < GM::BPT2; ++q) {
      const int t = threadIdx.x + q * kF64Threads;
      if (t >= GM::NB2) continue;
      const int c = t / (L / 2), j = t % (L / 2);
      const int k = j & (ns - 1);
      double2 a0 = v[q][0], a1 = v[q][1];
      if (ns > 1) a1 = cmul64(a1, tw64<INV>(k << (kTw64Log - lns - 1)));
      const int base = ((j >> lns) << (lns + 1)) + k;
      sb[c * L + base] = make_double2(a0.x + a1.x, a0.y + a1.y);
      sb[c * L + base + ns] = make_double2(a0.x - a1.x, a0.y - a1.y);
    }
    __syncthreads();
  }
}

template <int LOGL, bool INV>
__global__ void __launch_bounds__(kF64Threads) k_f64_seq(F64SeqArgs a) {
  using GM = F64Geom<LOGL>;
  constexpr int L = GM::L;
  constexpr int C = GM::C;
  extern __shared__ double2 sb[];
  const long long s0 = (long long)blockIdx.x * C;
  int cn = C;
  if (s0 + cn > a.nseq) cn = (int)(a.nseq - s0);
  // load: walk the C x L tile along whichever axis is contiguous in memory
  const bool in_seq_fast = a.in_js != 1;  // neighbouring sequences adjacent: sequence index fastest
  for (int idx = threadIdx.x; idx < C * L; idx += kF64Threads) {
    int c, j;
    if (in_seq_fast) { c = idx % C; j = idx / C; } else { c = idx / L; j = idx % L; }
    double2 v = make_double2(0.0, 0.0);
    if (c < cn) {
      const long long s = s0 + c;
      const long long off = (s / a.inner) * a.in_outer + (s % a.inner) * a.in_cs + (long long)j * a.in_js;
      v = make_double2(a.xr[off], a.xi[off]);
    }
    sb[c * L + j] = v;
  }
  __syncthreads();
  f64_block_fft<LOGL, INV>(sb);
  const bool out_seq_fast = a.out_ks != 1;
  for (int idx = threadIdx.x; idx < C * L; idx += kF64Threads) {
    int c, k;
    if (out_seq_fast) { c = idx % C; k = idx / C; } else { c = idx / L; k = idx % L; }
    if (c >= cn) continue;
    const long long s = s0 + c;
    double2 v = sb[c * L + k];
    if (a.tw_hi) {
      const unsigned long long e =
          ((unsigned long long)((s % a.inner) + a.tw_off) * (unsigned long long)k) & a.tw_mask;
      double2 w = cmul64(a.tw_hi[e >> a.tw_split], a.tw_lo[e & ((1ULL << a.tw_split) - 1)]);
      if (INV) w.y = -w.y;
      v = cmul64(v, w);
    }
    const long long off = (s / a.inner) * a.out_outer + (s % a.inner) * a.out_cs + (long long)k * a.out_ks;
    a.yr[off] = v.x * a.scale;
    a.yi[off] = v.y * a.scale;
  }
}

template <int LOGL>
static cudaError_t launch_seq_l(const F64SeqArgs& a, bool inv, cudaStream_t st) {
  using GM = F64Geom<LOGL>;
  auto kern = inv ? k_f64_seq<LOGL, true> : k_f64_seq<LOGL, false>;
  if (GM::smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = (a.nseq + GM::C - 1) / GM::C;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, kF64Threads, GM::smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_f64_seq(int logl, bool inv, const F64SeqArgs& a, cudaStream_t st) {
  switch (logl) {
    case 1: return launch_seq_l<1>(a, inv, st);
    case 2: return launch_seq_l<2>(a, inv, st);
    case 3: return launch_seq_l<3>(a, inv, st);
    case 4: return launch_seq_l<4>(a, inv, st);
    case 5: return launch_seq_l<5>(a, inv, st);
    case 6: return launch_seq_l<6>(a, inv, st);
    case 7: return launch_seq_l<7>(a, inv, st);
    case 8: return launch_seq_l<8>(a, inv, st);
    case 9: return launch_seq_l<9>(a, inv, st);
    case 10: return launch_seq_l<10>(a, inv, st);
    case 11: return launch_seq_l<11>(a, inv, st);
    case 12: return launch_seq_l<12>(a, inv, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t upload_tw64(const double2* host_table) {
  return cudaMemcpyToSymbol(g_tw64, host_table, sizeof(double2) * kTw64N);
}

// ---- Bluestein chirp stages (fp64) ------------------------------------------
// a[b][j] = x[b][j] * chirp_j (conj for the inverse) for j < n, 0 for n <= j < m
__global__ void k_f64_blue_pre(const double* __restrict__ xr, const double* __restrict__ xi,
                               const double2* __restrict__ chirp, double* __restrict__ ar, double* __restrict__ ai,
                               long long batch, long long n, long long m, int inv) {
  const long long total = batch * m;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / m, j = i % m;
    double2 v = make_double2(0.0, 0.0);
    if (j < n) {
      double2 c = chirp[j];
      if (inv) c.y = -c.y;
      v = cmul64(make_double2(xr[b * n + j], xi[b * n + j]), c);
    }
    ar[i] = v.x;
    ai[i] = v.y;
  }
}

// a[b][k] *= H[k] (forward) or conj(H[(m - k) mod m]) (inverse: the spectrum of conj(h))
__global__ void k_f64_blue_mul(double* __restrict__ ar, double* __restrict__ ai, const double2* __restrict__ H,
                               long long batch, long long m, int inv) {
  const long long total = batch * m;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long k = i % m;
    double2 h = H[inv ? ((m - k) & (m - 1)) : k];
    if (inv) h.y = -h.y;
    const double2 v = cmul64(make_double2(ar[i], ai[i]), h);
    ar[i] = v.x;
    ai[i] = v.y;
  }
}

// y[b][j] = a[b][j] * chirp_j * scale for j < n
__global__ void k_f64_blue_post(const double* __restrict__ ar, const double* __restrict__ ai,
                                const double2* __restrict__ chirp, double* __restrict__ yr, double* __restrict__ yi,
                                long long batch, long long n, long long m, int inv, double scale) {
  const long long total = batch * n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / n, j = i % n;
    double2 c = chirp[j];
    if (inv) c.y = -c.y;
    const double2 v = cmul64(make_double2(ar[b * m + j], ai[b * m + j]), c);
    yr[i] = v.x * scale;
    yi[i] = v.y * scale;
  }
}

static unsigned ew_blocks(long long total) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long b = (total + 255) / 256;
  const long long cap = 8LL * sms;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

cudaError_t launch_f64_blue_pre(const double* xr, const double* xi, const double2* chirp, double* ar, double* ai,
                                long long batch, long long n, long long m, bool inv, cudaStream_t st) {
  k_f64_blue_pre<<<ew_blocks(batch * m), 256, 0, st>>>(xr, xi, chirp, ar, ai, batch, n, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_f64_blue_mul(double* ar, double* ai, const double2* H, long long batch, long long m, bool inv,
                                cudaStream_t st) {
  k_f64_blue_mul<<<ew_blocks(batch * m), 256, 0, st>>>(ar, ai, H, batch, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_f64_blue_post(const double* ar, const double* ai, const double2* chirp, double* yr, double* yi,
                                 long long batch, long long n, long long m, bool inv, double scale, cudaStream_t st) {
  k_f64_blue_post<<<ew_blocks(batch * n), 256, 0, st>>>(ar, ai, chirp, yr, yi, batch, n, m, inv ? 1 : 0, scale);
  return cudaGetLastError();
}

// float32 <-> float64 plane conversion (precision="double" on float32 tensors)
__global__ void k_f32_to_f64(const float* __restrict__ x, double* __restrict__ y, long long count) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = (double)x[i];
}
__global__ void k_f64_to_f32(const double* __restrict__ x, float* __restrict__ y, long long count) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = (float)x[i];
}

cudaError_t launch_f32_to_f64(const float* x, double* y, long long count, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  k_f32_to_f64<<<ew_blocks(count), 256, 0, st>>>(x, y, count);
  return cudaGetLastError();
}

cudaError_t launch_f64_to_f32(const double* x, float* y, long long count, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  k_f64_to_f32<<<ew_blocks(count), 256, 0, st>>>(x, y, count);
  return cudaGetLastError();
}

}  // namespace tfb
