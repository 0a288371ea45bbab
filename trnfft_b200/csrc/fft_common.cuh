// Shared device-side building blocks of the trnfft_b200 FFT kernels.
//
// Data layout everywhere: planar float32 (separate re[] and im[] arrays),
// transforms batch-major, which is trnfft's ComplexTensor layout
// (trnfft/complex.py:16-33).
//
// The FFT engine is a register/shared-memory Stockham auto-sort FFT.  A
// length-N transform (N = 2^LOGN) is handled by T = N/E threads that each
// hold E complex values in registers.  Pass p applies radix R_p butterflies:
// butterfly b (0 <= b < N/R) reads x[b + r*N/R], multiplies by the twiddle
// W_{Ns*R}^{(b mod Ns)*r} (Ns = product of the earlier radices), runs an
// in-register R-point DFT and writes the result to
// ((b / Ns) * Ns * R + b mod Ns) + r*Ns.  The first pass reads natural order,
// the last pass writes natural order, so no bit reversal pass is needed and
// both the first load and the last store are unit-stride across threads.
// Between passes the values go through shared memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tfb {

// ---------------------------------------------------------------------------
// Compile-time trigonometry for the constant twiddles inside a radix-R
// butterfly (R <= 32).  Plain Taylor series evaluated in double precision by
// the C++ front end; |x| <= pi after reduction, 40 terms, error < 1e-15.
// ---------------------------------------------------------------------------
constexpr double kPi = 3.141592653589793238462643383279502884;

constexpr double ct_sin(double x) {
  double term = x, sum = x;
  for (int i = 1; i < 40; ++i) {
    term *= -x * x / ((2.0 * i) * (2.0 * i + 1.0));
    sum += term;
  }
  return sum;
}
constexpr double ct_cos(double x) {
  double term = 1.0, sum = 1.0;
  for (int i = 1; i < 40; ++i) {
    term *= -x * x / ((2.0 * i - 1.0) * (2.0 * i));
    sum += term;
  }
  return sum;
}
// angle 2*pi*k/n reduced to (-pi, pi]
constexpr double ct_angle(long k, long n) {
  long kk = ((k % n) + n) % n;
  if (2 * kk > n) kk -= n;
  return 2.0 * kPi * (double)kk / (double)n;
}

constexpr int ct_bitrev(int v, int bits) {
  int r = 0;
  for (int i = 0; i < bits; ++i) {
    r = (r << 1) | (v & 1);
    v >>= 1;
  }
  return r;
}
constexpr int ct_log2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

// (re, im) *= exp(sign * 2*pi*i * K / M), K and M compile-time.
template <int K, int M, bool INV>
__device__ __forceinline__ void cmul_const(float& re, float& im) {
  constexpr int k = ((K % M) + M) % M;
  if constexpr (k == 0) {
    return;
  } else if constexpr (2 * k == M) {
    re = -re;
    im = -im;
  } else if constexpr (4 * k == M) {
    // forward: multiply by -i ; inverse: by +i
    float t = re;
    if constexpr (INV) { re = -im; im = t; } else { re = im; im = -t; }
  } else if constexpr (4 * k == 3 * M) {
    float t = re;
    if constexpr (INV) { re = im; im = -t; } else { re = -im; im = t; }
  } else if constexpr (8 * k == M || 8 * k == 3 * M || 8 * k == 5 * M || 8 * k == 7 * M) {
    // odd multiples of 1/8 turn: c * (+-1 +- i) with c = sqrt(1/2)
    constexpr double ang = (INV ? 1.0 : -1.0) * ct_angle(k, M);
    constexpr float c = (float)ct_cos(ang);
    constexpr float s = (float)ct_sin(ang);
    // |c| == |s| here, so (re*c - im*s, re*s + im*c) = c*(re - im*(s/c)), ...
    constexpr float q = (s / c > 0.f) ? 1.f : -1.f;
    float nr = c * (re - q * im);
    float ni = c * (q * re + im);
    re = nr;
    im = ni;
  } else {
    constexpr double ang = (INV ? 1.0 : -1.0) * ct_angle(k, M);
    constexpr float c = (float)ct_cos(ang);
    constexpr float s = (float)ct_sin(ang);
    float nr = fmaf(re, c, -im * s);
    float ni = fmaf(re, s, im * c);
    re = nr;
    im = ni;
  }
}

// One radix-2 decimation-in-frequency butterfly stage of span S inside an
// R-point register DFT; J enumerates the R/2 butterflies of the stage.
template <int R, bool INV, int S, int J>
__device__ __forceinline__ void dif_bfly(float (&re)[R], float (&im)[R]) {
  if constexpr (J < R / 2) {
    constexpr int i = J % S;
    constexpr int lo = (J / S) * 2 * S + i;
    constexpr int hi = lo + S;
    float ar = re[lo], ai = im[lo], br = re[hi], bi = im[hi];
    re[lo] = ar + br;
    im[lo] = ai + bi;
    float dr = ar - br, di = ai - bi;
    cmul_const<i, 2 * S, INV>(dr, di);
    re[hi] = dr;
    im[hi] = di;
    dif_bfly<R, INV, S, J + 1>(re, im);
  }
}
template <int R, bool INV, int S>
__device__ __forceinline__ void dif_stages(float (&re)[R], float (&im)[R]) {
  dif_bfly<R, INV, S, 0>(re, im);
  if constexpr (S > 1) dif_stages<R, INV, S / 2>(re, im);
}

// In-register R-point DFT, R a power of two.  Output is left in bit-reversed
// order: X[k] is in slot ct_bitrev(k, log2 R).
template <int R, bool INV>
__device__ __forceinline__ void dft_reg(float (&re)[R], float (&im)[R]) {
  if constexpr (R > 1) dif_stages<R, INV, R / 2>(re, im);
}

// ---------------------------------------------------------------------------
// Twiddle table W_16384^i = exp(-2*pi*i*i/16384), i in [0, 16384), computed
// in double on the host and copied to every device once (a file-scope device
// array, so no allocation).  W_N^j for any N = 2^l <= 16384 is
// W_16384^(j << (14 - l)).
// ---------------------------------------------------------------------------
constexpr int kTwLog = 14;
constexpr int kTwN = 1 << kTwLog;
extern __device__ float2 g_tw[kTwN];

__device__ __forceinline__ float2 tw_lookup(int idx) { return __ldg(&g_tw[idx]); }

// Dense per-level tables D_L[k] = W_{2^L}^k for k < 2^(L-1), L = 1..14, level L stored from
// offset 2^(L-1) - 1 (16383 entries).  A Stockham pass needs W_{NS R}^{k 2^t} = D_{LNS+LR-t}[k]
// for consecutive k across a warp, so each of its table reads is contiguous.
extern __device__ float2 g_twd[kTwN];
__device__ __forceinline__ float2 tw_level(int L, int k) { return __ldg(&g_twd[(1 << (L - 1)) - 1 + k]); }

// Shared memory holds complex values interleaved (one float2 per element, so
// one 8-byte access moves a value) with one float2 of padding after every
// 2^SH elements.  With SH = log2 of the largest radix, the stride-R writes of
// the first Stockham pass land in distinct bank pairs within each half-warp.
template <int SH>
__device__ __forceinline__ int spad(int i) { return i + (i >> SH); }
template <int SH>
__host__ __device__ constexpr int spad_size(int n) { return n + (n >> SH); }

// ---------------------------------------------------------------------------
// Stockham pass schedule for N = 2^LOGN with E = 2^LOGE values per thread.
// The first pass takes the remainder radix when LOGE does not divide LOGN.
// ---------------------------------------------------------------------------
template <int LOGN, int LOGE>
struct Sched {
  static constexpr int LE = LOGE < LOGN ? LOGE : LOGN;
  static constexpr int N = 1 << LOGN;
  static constexpr int E = 1 << LE;
  static constexpr int T = N / E;  // threads per transform
  static constexpr int P = (LOGN + LE - 1) / LE;
  static constexpr int SH = LE;                    // shared-memory pad shift
  static constexpr int NP = N + (N >> LE);         // padded float2 slots per transform
  static constexpr int logr(int p) {
    return (LOGN % LE == 0) ? LE : (p == 0 ? LOGN % LE : LE);
  }
  static constexpr int logns(int p) {
    int s = 0;
    for (int q = 0; q < p; ++q) s += logr(q);
    return s;
  }
};

// Load the E values of pass p for thread j: v[q*R + r] = src(b + r*N/R),
// b = j + q*T.  `ld(index, re, im)` supplies the element.
template <int LOGN, int LOGE, int p, class Ld>
__device__ __forceinline__ void pass_load(int j, float (&vr)[Sched<LOGN, LOGE>::E],
                                          float (&vi)[Sched<LOGN, LOGE>::E], Ld ld) {
  using S = Sched<LOGN, LOGE>;
  constexpr int R = 1 << S::logr(p);
  constexpr int Q = S::E / R;
  constexpr int NR = S::N / R;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int b = j + q * S::T;
#pragma unroll
    for (int r = 0; r < R; ++r) ld(b + r * NR, vr[q * R + r], vi[q * R + r]);
  }
}

// Twiddle + in-register DFT + store of pass p.  `st(index, r, re, im)`
// receives every output element exactly once; output `index` = base + r*NS,
// and for each butterfly the calls come in increasing r (r is a compile-time
// constant after unrolling, so callers may branch on it for free).
template <int LOGN, int LOGE, int p, bool INV, class St>
__device__ __forceinline__ void pass_compute_store_qr(int j, float (&vr)[Sched<LOGN, LOGE>::E],
                                                      float (&vi)[Sched<LOGN, LOGE>::E], St st) {
  using S = Sched<LOGN, LOGE>;
  constexpr int LR = S::logr(p);
  constexpr int R = 1 << LR;
  constexpr int Q = S::E / R;
  constexpr int LNS = S::logns(p);
  constexpr int NS = 1 << LNS;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int b = j + q * S::T;
    const int k = b & (NS - 1);
    float ar[R], ai[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ar[r] = vr[q * R + r];
      ai[r] = vi[q * R + r];
    }
    if constexpr (NS > 1) {
      // W_{NS*R}^{k*r}.  The power-of-two exponents r = 2^t come from the level
      // tables (W_{NS*R}^{k 2^t} = D_{LNS+LR-t}[k]); every other r is the
      // product of the twiddle of its highest set bit and an already formed
      // twiddle (at most popcount(r)-1 roundings deep).
      float wr[R], wi[R];
      wr[0] = 1.f;
      wi[0] = 0.f;
#pragma unroll
      for (int r = 1; r < R; ++r) {
        const int hb = 1 << (31 - __clz(r));
        if (hb == r) {
          const float2 w = tw_level(LNS + LR - (31 - __clz(r)), k);
          wr[r] = w.x;
          wi[r] = INV ? -w.y : w.y;
        } else {
          const int lo = r - hb;
          wr[r] = fmaf(wr[hb], wr[lo], -wi[hb] * wi[lo]);
          wi[r] = fmaf(wr[hb], wi[lo], wi[hb] * wr[lo]);
        }
        const float xr = ar[r], xi = ai[r];
        ar[r] = fmaf(xr, wr[r], -xi * wi[r]);
        ai[r] = fmaf(xr, wi[r], xi * wr[r]);
      }
    }
    dft_reg<R, INV>(ar, ai);
    const int base = ((b >> LNS) << (LNS + LR)) + k;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int slot = ct_bitrev(r, LR);
      st(base + r * NS, q * R + r, r, ar[slot], ai[slot]);
    }
  }
}

// st(index, r, re, im); `pass_compute_store_qr` also passes the register
// slot q*R + r the value came from, so callers can keep outputs in (vr, vi).
template <int LOGN, int LOGE, int p, bool INV, class St>
__device__ __forceinline__ void pass_compute_store_r(int j, float (&vr)[Sched<LOGN, LOGE>::E],
                                                     float (&vi)[Sched<LOGN, LOGE>::E], St st) {
  pass_compute_store_qr<LOGN, LOGE, p, INV>(j, vr, vi,
                                            [&](int i, int, int r, float a, float b) { st(i, r, a, b); });
}

// Index of the output held in register slot q*R + r after pass p.
template <int LOGN, int LOGE, int p, class F>
__device__ __forceinline__ void pass_outputs(int j, F f) {
  using S = Sched<LOGN, LOGE>;
  constexpr int LR = S::logr(p);
  constexpr int R = 1 << LR;
  constexpr int Q = S::E / R;
  constexpr int LNS = S::logns(p);
  constexpr int NS = 1 << LNS;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int b = j + q * S::T;
    const int base = ((b >> LNS) << (LNS + LR)) + (b & (NS - 1));
#pragma unroll
    for (int r = 0; r < R; ++r) f(q * R + r, base + r * NS);
  }
}

// As pass_compute_store_r with `st(index, re, im)`.
template <int LOGN, int LOGE, int p, bool INV, class St>
__device__ __forceinline__ void pass_compute_store(int j, float (&vr)[Sched<LOGN, LOGE>::E],
                                                   float (&vi)[Sched<LOGN, LOGE>::E], St st) {
  pass_compute_store_r<LOGN, LOGE, p, INV>(j, vr, vi, [&](int i, int, float a, float b) { st(i, a, b); });
}

// Run passes [p, PEND) entirely through shared memory (`sb`: one transform,
// padded float2 layout).  The caller has already placed the pass-p input in
// shared memory and synchronised.  All threads of the block must call this.
template <int LOGN, int LOGE, bool INV, int p, int PEND>
__device__ __forceinline__ void smem_passes(int j, float2* sb) {
  if constexpr (p < PEND) {
    using S = Sched<LOGN, LOGE>;
    float vr[S::E], vi[S::E];
    pass_load<LOGN, LOGE, p>(j, vr, vi, [&](int i, float& a, float& b) {
      const float2 v = sb[spad<S::SH>(i)];
      a = v.x;
      b = v.y;
    });
    __syncthreads();
    pass_compute_store<LOGN, LOGE, p, INV>(j, vr, vi, [&](int i, float a, float b) {
      sb[spad<S::SH>(i)] = make_float2(a, b);
    });
    __syncthreads();
    smem_passes<LOGN, LOGE, INV, p + 1, PEND>(j, sb);
  }
}

}  // namespace tfb
