// Fused Bluestein (chirp-z) transform for any length n whose padded length
// m = 2^bitlen(2n-2) is at most 16384 (n <= 8192), one transform per group of
// threads, entirely on chip.
//
// Reference: trnfft/fft_core.py:1285-1376 computes
//   y = x * chirp, zero-pad to m, FFT(y) * FFT(h), IFFT, take n, * chirp
// with three radix-2 FFTs per call (FFT(h) is recomputed every call,
// fft_core.py:1349-1353) and six HBM round trips of host tensors.  Here:
//   * chirp_k = exp(-i*pi*(k^2 mod 2n)/n) is tabulated per plan in double and
//     rounded once (the reference's float32 angle pi*k*k/n loses ~1e-3 rad at
//     k ~ 4000, fft_core.py:1316-1320);
//   * H = FFT_m(h)/m, h = conj(chirp) with the circular wrap of
//     fft_core.py:1337-1345, is computed once per plan;
//   * one kernel does premultiply -> forward m-point Stockham FFT -> * H ->
//     inverse m-point FFT -> postmultiply, so x is read once and X written once;
//   * for m <= 8192 H and the chirp are copied into shared memory once per
//     block and the block loops over transforms (one resident grid), so the
//     per-point table reads of the two pointwise steps hit shared memory
//     instead of L2 (n = 4093, batch 4096 on B200: 0.28 ms per launch against
//     0.35 ms with the tables read through the read-only cache).
// The inverse transform uses conj(chirp) and H_inv[k] = conj(H[(m-k) mod m])
// (FFT of conj(h)), and scales by 1/n (fft_core.py:1369-1370).
#include <cstdlib>

#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGM>
struct BlueLogE {
  // 16 values per thread (radix-16 passes) up to m = 4096, where they beat the
  // radix-32 variant (~250 registers, one block per SM) measured on B200
  static constexpr int v = LOGM >= 13 ? 5 : 4;  // m >= 8192: radix-32 (measured faster there)
};

template <int LOGM, int LE_ = BlueLogE<LOGM>::v>
struct BlueGeom {
  static constexpr int LE = LE_;
  using S = Sched<LOGM, LE>;
  static constexpr int THREADS = S::T > 128 ? S::T : 128;
  // <= 128 registers per thread for the radix-16 kernels; the radix-32 ones keep all they need
  static constexpr int MINB = (LE == 5 || THREADS >= 512) ? 1 : 512 / THREADS;
  static constexpr int G = THREADS / S::T;
  static constexpr int MP = S::NP;
  static constexpr size_t work_smem = (size_t)G * MP * sizeof(float2);
  // H (m entries) and the chirp (n <= m/2 entries) stay in shared memory when they fit beside
  // the transforms (m <= 8192); the grid then loops over the transforms
  static constexpr size_t tab_smem = (size_t)(S::N + S::N / 2) * sizeof(float2);
  static constexpr bool TAB = work_smem + tab_smem <= 200 * 1024;
  static constexpr size_t smem = work_smem + (TAB ? tab_smem : 0);
};

// MODE 0: C2C, MODE 1: R2C (real rows -> n/2+1 bins), MODE 2: C2R (n/2+1 bins -> real rows).
// The real modes transform two rows at once: rows a = 2t and b = 2t+1 go in as
// a + i b (R2C; the two spectra are separated on chip from Z_k and Z_{n-k}),
// or their spectra as A + i B (C2R; the real and imaginary parts of the result
// are the two rows), half the work of a complex transform per row.
template <int LOGM, bool INV, int MODE, int LE_ = BlueLogE<LOGM>::v>
__global__ void __launch_bounds__(BlueGeom<LOGM, LE_>::THREADS, BlueGeom<LOGM, LE_>::MINB) k_bluestein(BlueArgs a) {
  using GM = BlueGeom<LOGM, LE_>;
  constexpr int LE = GM::LE;
  using S = Sched<LOGM, LE>;
  constexpr int M = S::N;
  extern __shared__ float sm[];
  const int g = threadIdx.x / S::T;
  const int j = threadIdx.x % S::T;
  const int n_all = a.n;
  float2* Hs = reinterpret_cast<float2*>(sm) + GM::G * GM::MP;
  float2* cs = Hs + M;
  if constexpr (GM::TAB) {
    for (int i = threadIdx.x; i < M; i += GM::THREADS) Hs[i] = __ldg(a.H + i);
    for (int i = threadIdx.x; i < n_all; i += GM::THREADS) cs[i] = __ldg(a.chirp + i);
    __syncthreads();
  }
  auto ldc = [&](int i) -> float2 {
    if constexpr (GM::TAB) return cs[i];
    else return __ldg(a.chirp + i);
  };
  auto ldh = [&](int i) -> float2 {
    if constexpr (GM::TAB) return Hs[i];
    else return __ldg(a.H + i);
  };
  const long long ntf_all = MODE == 0 ? a.batch : (a.batch + 1) / 2;
  for (long long tb = (long long)blockIdx.x * GM::G; tb < ntf_all; tb += (long long)gridDim.x * GM::G) {
    const long long t = tb + g;
    // the real modes pack rows 2t and 2t+1 into one complex transform
    const long long ntf = MODE == 0 ? a.batch : (a.batch + 1) / 2;
    const bool valid = t < ntf;
    const long long tt = valid ? t : 0;
    const long long row0 = MODE == 0 ? tt : 2 * tt;
    const bool has1 = MODE != 0 && row0 + 1 < a.batch;
    const int n = a.n;
    const int half = n / 2;
    float2* sb = reinterpret_cast<float2*>(sm) + g * GM::MP;
    const float csign = INV ? -1.f : 1.f;  // inverse uses conj(chirp)

    // ---- load + premultiply (pass 0 of the forward m-point FFT)
    float vr[S::E], vi[S::E];
    pass_load<LOGM, LE, 0>(j, vr, vi, [&](int i, float& r, float& m) {
      r = 0.f;
      m = 0.f;
      if (!valid || i >= n) return;
      float xr, xi;
      if constexpr (MODE == 0) {
        xr = __ldg(a.xr + tt * n + i);
        xi = __ldg(a.xi + tt * n + i);
      } else if constexpr (MODE == 1) {
        // z = a + i b for the real rows a = 2t, b = 2t+1
        xr = __ldg(a.xr + row0 * n + i);
        xi = has1 ? __ldg(a.xr + (row0 + 1) * n + i) : 0.f;
      } else {
        // Z = A + i B for the Hermitian extensions A, B of rows 2t, 2t+1 (trnfft/api.py:54-66);
        // the imaginary parts of bin 0 and (even n) bin n/2 do not contribute to a real result
        const long long h = half + 1;
        const int src = i <= half ? i : n - i;
        const float sg = i <= half ? 1.f : -1.f;
        const bool im_ok = !(src == 0 || 2 * src == n);
        const float ar = __ldg(a.xr + row0 * h + src);
        const float ai = im_ok ? sg * __ldg(a.xi + row0 * h + src) : 0.f;
        float br = 0.f, bi = 0.f;
        if (has1) {
          br = __ldg(a.xr + (row0 + 1) * h + src);
          bi = im_ok ? sg * __ldg(a.xi + (row0 + 1) * h + src) : 0.f;
        }
        xr = ar - bi;
        xi = ai + br;
      }
      const float2 c = ldc(i);
      const float ci = csign * c.y;
      r = fmaf(xr, c.x, -xi * ci);
      m = fmaf(xr, ci, xi * c.x);
    });
    auto sstore = [&](int i, float r, float m) {
      sb[spad<S::SH>(i)] = make_float2(r, m);
    };
    auto sload = [&](int i, float& r, float& m) {
      { const float2 v_ = sb[spad<S::SH>(i)]; r = v_.x; m = v_.y; }
    };
    if constexpr (S::P == 1) {
      // single-pass forward FFT: multiply by H in the store
      pass_compute_store<LOGM, LE, 0, false>(j, vr, vi, [&](int i, float r, float m) {
        float2 h = ldh(INV ? ((M - i) & (M - 1)) : i);
        if (INV) h.y = -h.y;
        sstore(i, fmaf(r, h.x, -m * h.y), fmaf(r, h.y, m * h.x));
      });
    } else {
      pass_compute_store<LOGM, LE, 0, false>(j, vr, vi, sstore);
      __syncthreads();
      smem_passes<LOGM, LE, false, 1, S::P - 1>(j, sb);
      pass_load<LOGM, LE, S::P - 1>(j, vr, vi, sload);
      __syncthreads();
      pass_compute_store<LOGM, LE, S::P - 1, false>(j, vr, vi, [&](int i, float r, float m) {
        float2 h = ldh(INV ? ((M - i) & (M - 1)) : i);
        if (INV) h.y = -h.y;
        sstore(i, fmaf(r, h.x, -m * h.y), fmaf(r, h.y, m * h.x));
      });
    }
    __syncthreads();

    // ---- inverse m-point FFT (unscaled; 1/m is folded into H) + postmultiply
    smem_passes<LOGM, LE, true, 0, S::P - 1>(j, sb);
    pass_load<LOGM, LE, S::P - 1>(j, vr, vi, sload);
    const float sc = INV ? 1.f / (float)n : 1.f;
    if constexpr (MODE == 1) __syncthreads();  // sb is rewritten below with the packed spectrum
    pass_compute_store<LOGM, LE, S::P - 1, true>(j, vr, vi, [&](int i, float r, float m) {
      if (!valid || i >= n) return;
      const float2 c = ldc(i);
      const float ci = csign * c.y;
      const float yr = fmaf(r, c.x, -m * ci) * sc;
      const float yi = fmaf(r, ci, m * c.x) * sc;
      if constexpr (MODE == 0) {
        a.yr[tt * n + i] = yr;
        a.yi[tt * n + i] = yi;
      } else if constexpr (MODE == 1) {
        sb[spad<S::SH>(i)] = make_float2(yr, yi);
      } else {
        a.yr[row0 * n + i] = yr;
        if (has1) a.yr[(row0 + 1) * n + i] = yi;
      }
    });
    if constexpr (MODE == 1) {
      // Z = FFT(a + i b): A_k = (Z_k + conj Z_{n-k}) / 2, B_k = (Z_k - conj Z_{n-k}) / (2i)
      __syncthreads();
      if (valid) {
        const long long h = half + 1;
        for (int k = j; k <= half; k += S::T) {
          const float2 z = sb[spad<S::SH>(k)];
          const float2 w = sb[spad<S::SH>(k == 0 ? 0 : n - k)];
          a.yr[row0 * h + k] = 0.5f * (z.x + w.x);
          a.yi[row0 * h + k] = 0.5f * (z.y - w.y);
          if (has1) {
            a.yr[(row0 + 1) * h + k] = 0.5f * (z.y + w.y);
            a.yi[(row0 + 1) * h + k] = 0.5f * (w.x - z.x);
          }
        }
      }
    }

    if constexpr (!GM::TAB) break;  // one block per transform group: no loop
    __syncthreads();  // this block's transform buffers are reused by its next transforms
  }
}

template <int LOGM, bool INV, int MODE, int LE_ = BlueLogE<LOGM>::v>
static cudaError_t launch_blue_t(const BlueArgs& a, cudaStream_t st) {
  using GM = BlueGeom<LOGM, LE_>;
  auto kern = k_bluestein<LOGM, INV, MODE, LE_>;
  if (GM::smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
    if (e != cudaSuccess) return e;
  }
  const long long ntf = MODE == 0 ? a.batch : (a.batch + 1) / 2;  // real modes: two rows per transform
  long long blocks = (ntf + GM::G - 1) / GM::G;
  if constexpr (GM::TAB) {
    // persistent: as many blocks as fit at once, each loading the tables once
    int dev = 0, sms = 0, per_sm = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GM::THREADS, GM::smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    if (blocks > (long long)sms * per_sm) blocks = (long long)sms * per_sm;
  }
  kern<<<(unsigned)blocks, GM::THREADS, GM::smem, st>>>(a);
  return cudaGetLastError();
}

// Values per thread for m >= 8192: C2C keeps 32 (radix-32 passes); the packed real modes at
// m = 8192 use 16 (twice the threads, half the registers each), measured on B200 with the tables
// in shared memory: rfft n = 4093 batch 4096 0.205 ms per launch against 0.252 ms with 32, while
// C2C measured the same either way (0.284 / 0.279 ms).  TRNFFT_B200_BLUE_LOGE=4 or 5 forces one
// choice for every mode, for measurement.
static int blue_loge_override() {
  static const int v = [] {
    const char* e = getenv("TRNFFT_B200_BLUE_LOGE");
    return e ? atoi(e) : 0;
  }();
  return v;
}

template <int LOGM>
static cudaError_t launch_blue_m(int mode, bool inv, const BlueArgs& a, cudaStream_t st) {
  if constexpr (LOGM >= 13) {
    const int ov = blue_loge_override();
    if (ov == 4 || (ov != 5 && LOGM == 13 && mode != 0)) {
      switch (mode) {
        case 0: return inv ? launch_blue_t<LOGM, true, 0, 4>(a, st) : launch_blue_t<LOGM, false, 0, 4>(a, st);
        case 1: return launch_blue_t<LOGM, false, 1, 4>(a, st);
        case 2: return launch_blue_t<LOGM, true, 2, 4>(a, st);
        default: return cudaErrorInvalidValue;
      }
    }
  }
  switch (mode) {
    case 0: return inv ? launch_blue_t<LOGM, true, 0>(a, st) : launch_blue_t<LOGM, false, 0>(a, st);
    case 1: return launch_blue_t<LOGM, false, 1>(a, st);
    case 2: return launch_blue_t<LOGM, true, 2>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bluestein(int logm, int mode, bool inv, const BlueArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
  switch (logm) {
    case 3: return launch_blue_m<3>(mode, inv, a, st);
    case 4: return launch_blue_m<4>(mode, inv, a, st);
    case 5: return launch_blue_m<5>(mode, inv, a, st);
    case 6: return launch_blue_m<6>(mode, inv, a, st);
    case 7: return launch_blue_m<7>(mode, inv, a, st);
    case 8: return launch_blue_m<8>(mode, inv, a, st);
    case 9: return launch_blue_m<9>(mode, inv, a, st);
    case 10: return launch_blue_m<10>(mode, inv, a, st);
    case 11: return launch_blue_m<11>(mode, inv, a, st);
    case 12: return launch_blue_m<12>(mode, inv, a, st);
    case 13: return launch_blue_m<13>(mode, inv, a, st);
    case 14: return launch_blue_m<14>(mode, inv, a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tfb
