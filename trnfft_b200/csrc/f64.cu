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
// store, so the result is in natural order).  Bluestein sizes whose padded
// length m is at most 8192 run as one fused kernel (k_f64_blue_small / _big:
// the padded transforms stay in shared memory); longer ones chain elementwise
// chirp kernels around two such transforms of the padded length.
// Twiddles inside a block come from a per-device table W_4096^i in double.
#include <cuda_runtime.h>

#include <cstdlib>

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
  static constexpr int LP = L;  // sequence pitch in shared memory
  static constexpr size_t smem = (size_t)C * LP * sizeof(double2);
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
        for (int r = 0; r < 4; ++r) v[q][r] = sb[c * GM::LP + j + r * (L / 4)];
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
        // W_{4 ns}^{k r} = W_4096^{k r 4096 / (4 ns)}: one table read, W^2k and W^3k by products
        const double2 w1 = tw64<INV>(k << (kTw64Log - lns - 2));
        const double2 w2 = cmul64(w1, w1);
        a1 = cmul64(a1, w1);
        a2 = cmul64(a2, w2);
        a3 = cmul64(a3, cmul64(w2, w1));
      }
      const double2 s02 = make_double2(a0.x + a2.x, a0.y + a2.y), d02 = make_double2(a0.x - a2.x, a0.y - a2.y);
      const double2 s13 = make_double2(a1.x + a3.x, a1.y + a3.y), d13 = make_double2(a1.x - a3.x, a1.y - a3.y);
      // forward: X1 = d02 - i d13, X3 = d02 + i d13; the inverse swaps the signs
      const double2 md13 = INV ? make_double2(-d13.y, d13.x) : make_double2(d13.y, -d13.x);
      double2* y = sb + c * GM::LP;
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
        v[q][0] = sb[c * GM::LP + j];
        v[q][1] = sb[c * GM::LP + j + L / 2];
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
      sb[c * GM::LP + base] = make_double2(a0.x + a1.x, a0.y + a1.y);
      sb[c * GM::LP + base + ns] = make_double2(a0.x - a1.x, a0.y - a1.y);
    }
    __syncthreads();
  }
}

template <int LOGL, bool INV>
__global__ void __launch_bounds__(kF64Threads, 3) k_f64_seq(F64SeqArgs a) {
  using GM = F64Geom<LOGL>;
  constexpr int L = GM::L;
  constexpr int C = GM::C;
  extern __shared__ double2 sb[];
  // per-sequence offsets, computed once per block (the 64-bit divisions stay out of the loops)
  __shared__ long long s_in[C], s_out[C];
  __shared__ unsigned long long s_tw[C];
  const long long s0 = (long long)blockIdx.x * C;
  int cn = C;
  if (s0 + cn > a.nseq) cn = (int)(a.nseq - s0);
  if (threadIdx.x < cn) {
    const long long s = s0 + threadIdx.x;
    const long long q = s / a.inner, r = s - q * a.inner;
    s_in[threadIdx.x] = q * a.in_outer + r * a.in_cs;
    s_out[threadIdx.x] = q * a.out_outer + r * a.out_cs;
    s_tw[threadIdx.x] = (unsigned long long)(r + a.tw_off);
  }
  __syncthreads();
  // load: walk the C x L tile along whichever axis is contiguous in memory
  const bool in_seq_fast = a.in_js != 1;  // neighbouring sequences adjacent: sequence index fastest
  for (int idx = threadIdx.x; idx < C * L; idx += kF64Threads) {
    int c, j;
    if (in_seq_fast) { c = idx % C; j = idx / C; } else { c = idx / L; j = idx % L; }
    double2 v = make_double2(0.0, 0.0);
    if (c < cn) {
      const long long off = s_in[c] + (long long)j * a.in_js;
      v = a.xr32 ? make_double2((double)a.xr32[off], (double)a.xi32[off]) : make_double2(a.xr[off], a.xi[off]);
    }
    sb[c * GM::LP + j] = v;
  }
  __syncthreads();
  f64_block_fft<LOGL, INV>(sb);
  const bool out_seq_fast = a.out_ks != 1;
  for (int idx = threadIdx.x; idx < C * L; idx += kF64Threads) {
    int c, k;
    if (out_seq_fast) { c = idx % C; k = idx / C; } else { c = idx / L; k = idx % L; }
    if (c >= cn) continue;
    double2 v = sb[c * GM::LP + k];
    if (a.tw_hi) {
      const unsigned long long e = (s_tw[c] * (unsigned long long)k) & a.tw_mask;
      double2 w = cmul64(a.tw_hi[e >> a.tw_split], a.tw_lo[e & ((1ULL << a.tw_split) - 1)]);
      if (INV) w.y = -w.y;
      v = cmul64(v, w);
    }
    const long long off = s_out[c] + (long long)k * a.out_ks;
    if (a.yr32) {
      a.yr32[off] = (float)(v.x * a.scale);
      a.yi32[off] = (float)(v.y * a.scale);
    } else {
      a.yr[off] = v.x * a.scale;
      a.yi[off] = v.y * a.scale;
    }
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
                               const float* __restrict__ xr32, const float* __restrict__ xi32,
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
      const long long o = b * n + j;
      v = cmul64(xr32 ? make_double2((double)xr32[o], (double)xi32[o]) : make_double2(xr[o], xi[o]), c);
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
                                float* __restrict__ yr32, float* __restrict__ yi32, long long batch, long long n,
                                long long m, int inv, double scale) {
  const long long total = batch * n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / n, j = i % n;
    double2 c = chirp[j];
    if (inv) c.y = -c.y;
    const double2 v = cmul64(make_double2(ar[b * m + j], ai[b * m + j]), c);
    if (yr32) {
      yr32[i] = (float)(v.x * scale);
      yi32[i] = (float)(v.y * scale);
    } else {
      yr[i] = v.x * scale;
      yi[i] = v.y * scale;
    }
  }
}

static unsigned ew_blocks(long long total) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long b = (total + 255) / 256;
  const long long cap = 8LL * sms;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

cudaError_t launch_f64_blue_pre(const double* xr, const double* xi, const float* xr32, const float* xi32,
                                const double2* chirp, double* ar, double* ai, long long batch, long long n, long long m,
                                bool inv, cudaStream_t st) {
  k_f64_blue_pre<<<ew_blocks(batch * m), 256, 0, st>>>(xr, xi, xr32, xi32, chirp, ar, ai, batch, n, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_f64_blue_mul(double* ar, double* ai, const double2* H, long long batch, long long m, bool inv,
                                cudaStream_t st) {
  k_f64_blue_mul<<<ew_blocks(batch * m), 256, 0, st>>>(ar, ai, H, batch, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_f64_blue_post(const double* ar, const double* ai, const double2* chirp, double* yr, double* yi,
                                 float* yr32, float* yi32, long long batch, long long n, long long m, bool inv,
                                 double scale, cudaStream_t st) {
  k_f64_blue_post<<<ew_blocks(batch * n), 256, 0, st>>>(ar, ai, chirp, yr, yi, yr32, yi32, batch, n, m, inv ? 1 : 0,
                                                        scale);
  return cudaGetLastError();
}

// ---- fused Bluestein (m <= 8192) -------------------------------------------
// The chain above makes five (m <= 4096) or seven (m = 8192) passes over the padded batch in
// HBM; here one block holds whole padded transforms in shared memory and does every stage:
// x read once, y written once.  m <= 4096: F64Geom's C transforms per 256-thread block and the
// radix-4 block FFT.  m = 8192 (128 KB of double2, one transform per block): radix-2 Stockham
// passes with 512 threads, each holding 8 butterflies (a radix-4 pass would hold 16 double2 per
// thread, more registers than a 512-thread block has); the last pass's twiddles W_8192^k are
// W_4096^(k/2), times W_8192 for odd k.

constexpr int kF64BigThreads = 512;

// Shared-memory slot of point i in the 8192-point kernels: one double2 of padding after every 8,
// so the strided radix-4 / radix-2 stores of the early passes (stride 4 ns double2) fall in
// distinct bank groups (33.6 M bank conflicts per launch without it, n = 4093 batch 4096);
// contiguous accesses stay contiguous within each group of 8 lanes.
__device__ __forceinline__ int f64p(int i) { return i + (i >> 3); }

// m = 8192 with 1024 threads: six radix-4 passes (2 butterflies of 4 values per thread) and a
// final radix-2 pass (4 butterflies per thread), half the shared-memory traffic of radix 2
constexpr int kF64Big4Threads = 1024;

template <int LOGL, bool INV>
__device__ __forceinline__ void f64_fft_r4_big(double2* sb, double2 w_half) {
  constexpr int NT = kF64Big4Threads;
  constexpr int L = 1 << LOGL;
  constexpr int BPT4 = L / 4 / NT;
  constexpr int BPT2 = L / 2 / NT;
  static_assert(BPT4 >= 1 && (LOGL & 1) && LOGL == kTw64Log + 1, "radix-4 block FFT geometry (m = 8192)");
#pragma unroll 1
  for (int lns = 0; lns + 2 <= LOGL; lns += 2) {
    const int ns = 1 << lns;
    double2 v[BPT4][4];
#pragma unroll
    for (int q = 0; q < BPT4; ++q) {
      const int j = threadIdx.x + q * NT;
#pragma unroll
      for (int r = 0; r < 4; ++r) v[q][r] = sb[f64p(j + r * (L / 4))];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < BPT4; ++q) {
      const int j = threadIdx.x + q * NT;
      const int k = j & (ns - 1);
      double2 a0 = v[q][0], a1 = v[q][1], a2 = v[q][2], a3 = v[q][3];
      if (ns > 1) {
        // W_{4 ns}^k = W_4096^(k 4096 / (4 ns)), lns <= 10: one table read, W^2k and W^3k by products
        const double2 w1 = tw64<INV>(k << (kTw64Log - lns - 2));
        const double2 w2 = cmul64(w1, w1);
        a1 = cmul64(a1, w1);
        a2 = cmul64(a2, w2);
        a3 = cmul64(a3, cmul64(w2, w1));
      }
      const double2 s02 = make_double2(a0.x + a2.x, a0.y + a2.y), d02 = make_double2(a0.x - a2.x, a0.y - a2.y);
      const double2 s13 = make_double2(a1.x + a3.x, a1.y + a3.y), d13 = make_double2(a1.x - a3.x, a1.y - a3.y);
      const double2 md13 = INV ? make_double2(-d13.y, d13.x) : make_double2(d13.y, -d13.x);
      const int base = ((j >> lns) << (lns + 2)) + k;
      sb[f64p(base)] = make_double2(s02.x + s13.x, s02.y + s13.y);
      sb[f64p(base + ns)] = make_double2(d02.x + md13.x, d02.y + md13.y);
      sb[f64p(base + 2 * ns)] = make_double2(s02.x - s13.x, s02.y - s13.y);
      sb[f64p(base + 3 * ns)] = make_double2(d02.x - md13.x, d02.y - md13.y);
    }
    __syncthreads();
  }
  {
    constexpr int lns = LOGL - 1;  // 12: W_8192^k = W_4096^(k/2) (x W_8192 for odd k)
    constexpr int ns = 1 << lns;
    double2 v[BPT2][2];
#pragma unroll
    for (int q = 0; q < BPT2; ++q) {
      const int j = threadIdx.x + q * NT;
      v[q][0] = sb[f64p(j)];
      v[q][1] = sb[f64p(j + L / 2)];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < BPT2; ++q) {
      const int j = threadIdx.x + q * NT;
      const int k = j & (ns - 1);
      double2 w = tw64<INV>(k >> 1);
      if (k & 1) w = cmul64(w, w_half);
      const double2 a0 = v[q][0], a1 = cmul64(v[q][1], w);
      const int base = ((j >> lns) << (lns + 1)) + k;
      sb[f64p(base)] = make_double2(a0.x + a1.x, a0.y + a1.y);
      sb[f64p(base + ns)] = make_double2(a0.x - a1.x, a0.y - a1.y);
    }
    __syncthreads();
  }
}

template <int LOGL, bool INV>
__device__ __forceinline__ void f64_fft_r2_big(double2* sb, double2 w_half) {
  constexpr int L = 1 << LOGL;
  constexpr int NB = L / 2;
  constexpr int BPT = NB / kF64BigThreads;
  static_assert(NB % kF64BigThreads == 0 && LOGL <= kTw64Log + 1, "radix-2 block FFT geometry");
#pragma unroll 1
  for (int lns = 0; lns < LOGL; ++lns) {
    const int ns = 1 << lns;
    double2 v[BPT][2];
#pragma unroll
    for (int q = 0; q < BPT; ++q) {
      const int j = threadIdx.x + q * kF64BigThreads;
      v[q][0] = sb[f64p(j)];
      v[q][1] = sb[f64p(j + NB)];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < BPT; ++q) {
      const int j = threadIdx.x + q * kF64BigThreads;
      const int k = j & (ns - 1);
      double2 a0 = v[q][0], a1 = v[q][1];
      if (lns > 0) {
        double2 w;
        if (lns + 1 <= kTw64Log) {
          w = tw64<INV>(k << (kTw64Log - lns - 1));  // W_{2 ns}^k
        } else {
          w = tw64<INV>(k >> 1);  // W_{2 ns}^k with 2 ns = 2 * 4096
          if (k & 1) w = cmul64(w, w_half);
        }
        a1 = cmul64(a1, w);
      }
      const int base = ((j >> lns) << (lns + 1)) + k;
      sb[f64p(base)] = make_double2(a0.x + a1.x, a0.y + a1.y);
      sb[f64p(base + ns)] = make_double2(a0.x - a1.x, a0.y - a1.y);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ double2 blue_chirp(const double2* chirp, int j, bool inv) {
  double2 c = chirp[j];
  if (inv) c.y = -c.y;
  return c;
}
__device__ __forceinline__ double2 blue_h(const double2* H, int k, int m, bool inv) {
  double2 h = H[inv ? ((m - k) & (m - 1)) : k];
  if (inv) h.y = -h.y;
  return h;
}

__device__ __forceinline__ double2 blue_load(const F64BlueArgs& a, long long o) {
  return a.xr32 ? make_double2((double)a.xr32[o], (double)a.xi32[o]) : make_double2(a.xr[o], a.xi[o]);
}
__device__ __forceinline__ void blue_store(const F64BlueArgs& a, long long o, double2 v) {
  if (a.yr32) {
    a.yr32[o] = (float)(v.x * a.scale);
    a.yi32[o] = (float)(v.y * a.scale);
  } else {
    a.yr[o] = v.x * a.scale;
    a.yi[o] = v.y * a.scale;
  }
}

// m <= 4096: C transforms per block (sequence c of the block is row blockIdx.x * C + c)
template <int LOGM, bool INV>
__global__ void __launch_bounds__(kF64Threads) k_f64_blue_small(F64BlueArgs a) {
  using GM = F64Geom<LOGM>;
  constexpr int M = GM::L;
  constexpr int C = GM::C;
  extern __shared__ double2 sb[];
  const long long r0 = (long long)blockIdx.x * C;
  const int n = a.n;
  for (int idx = threadIdx.x; idx < C * M; idx += kF64Threads) {
    const int c = idx / M, j = idx % M;
    const long long r = r0 + c;
    double2 v = make_double2(0.0, 0.0);
    if (j < n && r < a.batch) v = cmul64(blue_load(a, r * n + j), blue_chirp(a.chirp, j, INV));
    sb[c * GM::LP + j] = v;
  }
  __syncthreads();
  f64_block_fft<LOGM, false>(sb);
  for (int idx = threadIdx.x; idx < C * M; idx += kF64Threads) {
    const int s = (idx / M) * GM::LP + idx % M;
    sb[s] = cmul64(sb[s], blue_h(a.H, idx % M, M, INV));
  }
  __syncthreads();
  f64_block_fft<LOGM, true>(sb);  // unscaled: 1/m is folded into H
  for (int idx = threadIdx.x; idx < C * n; idx += kF64Threads) {
    const int c = idx / n, j = idx % n;
    const long long r = r0 + c;
    if (r >= a.batch) break;
    const double2 v = cmul64(sb[c * GM::LP + j], blue_chirp(a.chirp, j, INV));
    blue_store(a, r * n + j, v);
  }
}

// m = 8192: one transform per block; R4 selects the 1024-thread radix-4 block FFT
template <bool INV, bool R4>
__global__ void __launch_bounds__(R4 ? kF64Big4Threads : kF64BigThreads, 1) k_f64_blue_big(F64BlueArgs a) {
  constexpr int LOGM = 13;
  constexpr int M = 1 << LOGM;
  constexpr int NT = R4 ? kF64Big4Threads : kF64BigThreads;
  extern __shared__ double2 sb[];
  const long long r = blockIdx.x;
  const int n = a.n;
  double s, c;
  sincospi(2.0 / M, &s, &c);  // W_M = exp(-2 pi i / M)
  for (int j = threadIdx.x; j < M; j += NT) {
    double2 v = make_double2(0.0, 0.0);
    if (j < n) v = cmul64(blue_load(a, r * n + j), blue_chirp(a.chirp, j, INV));
    sb[f64p(j)] = v;
  }
  __syncthreads();
  if constexpr (R4) f64_fft_r4_big<LOGM, false>(sb, make_double2(c, -s));
  else f64_fft_r2_big<LOGM, false>(sb, make_double2(c, -s));
  for (int k = threadIdx.x; k < M; k += NT) sb[f64p(k)] = cmul64(sb[f64p(k)], blue_h(a.H, k, M, INV));
  __syncthreads();
  // unscaled inverse: 1/m is folded into H
  if constexpr (R4) f64_fft_r4_big<LOGM, true>(sb, make_double2(c, s));
  else f64_fft_r2_big<LOGM, true>(sb, make_double2(c, s));
  for (int j = threadIdx.x; j < n; j += NT) {
    const double2 v = cmul64(sb[f64p(j)], blue_chirp(a.chirp, j, INV));
    blue_store(a, r * n + j, v);
  }
}

// TRNFFT_B200_F64_BLUE_R2=1 selects the 512-thread radix-2 variant of the m = 8192 kernel.
static bool f64_blue_r2() {
  static const bool v = [] {
    const char* e = getenv("TRNFFT_B200_F64_BLUE_R2");
    return e != nullptr && atoi(e) == 1;
  }();
  return v;
}

template <int LOGM>
static cudaError_t launch_blue_small(bool inv, const F64BlueArgs& a, cudaStream_t st) {
  using GM = F64Geom<LOGM>;
  auto kern = inv ? k_f64_blue_small<LOGM, true> : k_f64_blue_small<LOGM, false>;
  if (GM::smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = (a.batch + GM::C - 1) / GM::C;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, kF64Threads, GM::smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_f64_blue_fused(int logm, bool inv, const F64BlueArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
  switch (logm) {
    case 1: return launch_blue_small<1>(inv, a, st);
    case 2: return launch_blue_small<2>(inv, a, st);
    case 3: return launch_blue_small<3>(inv, a, st);
    case 4: return launch_blue_small<4>(inv, a, st);
    case 5: return launch_blue_small<5>(inv, a, st);
    case 6: return launch_blue_small<6>(inv, a, st);
    case 7: return launch_blue_small<7>(inv, a, st);
    case 8: return launch_blue_small<8>(inv, a, st);
    case 9: return launch_blue_small<9>(inv, a, st);
    case 10: return launch_blue_small<10>(inv, a, st);
    case 11: return launch_blue_small<11>(inv, a, st);
    case 12: return launch_blue_small<12>(inv, a, st);
    case 13: {
      const bool r2 = f64_blue_r2();
      auto kern = r2 ? (inv ? k_f64_blue_big<true, false> : k_f64_blue_big<false, false>)
                     : (inv ? k_f64_blue_big<true, true> : k_f64_blue_big<false, true>);
      const size_t smem = sizeof(double2) * ((1 << 13) + (1 << 10));  // padded (f64p)
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      if (a.batch > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
      kern<<<(unsigned)a.batch, r2 ? kF64BigThreads : kF64Big4Threads, smem, st>>>(a);
      return cudaGetLastError();
    }
    default: return cudaErrorInvalidValue;
  }
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
