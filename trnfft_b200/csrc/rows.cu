// Batched power-of-two transforms along contiguous rows, one whole transform
// per group of threads (single-CTA Stockham, N <= 16384 complex / 8192 real).
//
// Replaces the reference's per-stage radix-2 loop (trnfft/fft_core.py:53-117)
// and its NKI Stockham/butterfly kernels (trnfft/nki/stockham.py:55-235,
// trnfft/nki/butterfly.py:64-141): every stage of a transform stays on chip,
// so each element is read from HBM once and written once.
//
//   k_c2c  complex -> complex, forward or inverse (inverse scaled by 1/N)
//   k_r2c  real rows of length N = 2M -> N/2+1 bins, via one M-point complex
//          FFT of z[n] = x[2n] + i x[2n+1] and an on-chip split
//   k_c2r  N/2+1 bins -> real rows of length N = 2M (inverse of k_r2c; the
//          imaginary parts of bins 0 and N/2 do not contribute, as in
//          trnfft/api.py:49-68 where only the real part of the inverse
//          transform is returned)
#include "fft_common.cuh"
#include "kernels.h"
#include "tma.cuh"

#include <cstdlib>

namespace tfb {

constexpr int kRowThreads = 256;

template <int LOGN, int LOGE, int THR = kRowThreads>
struct RowGeom {
  using S = Sched<LOGN, LOGE>;
  static_assert(S::T <= THR && THR % S::T == 0, "one transform must fit in one block");
  static constexpr int THREADS = THR;
  static constexpr int G = THR / S::T;  // transforms per block
  static constexpr int NP = S::NP;
  static constexpr size_t smem = (size_t)G * NP * sizeof(float2);
};

// ----------------------------------------------------------------------------
template <int LOGN, int LOGE, bool INV, int MINB = 1, int THR = kRowThreads>
__global__ void __launch_bounds__(THR, MINB) k_c2c(RowArgs a) {
  using S = Sched<LOGN, LOGE>;
  using GM = RowGeom<LOGN, LOGE, THR>;
  extern __shared__ float sm[];
  const int g = threadIdx.x / S::T;
  const int j = threadIdx.x % S::T;
  const long long t = (long long)blockIdx.x * GM::G + g;
  const bool valid = t < a.batch;
  const long long tt = valid ? t : 0;
  const float* __restrict__ xr = a.xr + tt * a.in_stride;
  const float* __restrict__ xi = a.xi + tt * a.in_stride;
  float* __restrict__ yr = a.yr + tt * a.out_stride;
  float* __restrict__ yi = a.yi + tt * a.out_stride;
  const float sc = a.scale;

  float vr[S::E], vi[S::E];
  pass_load<LOGN, LOGE, 0>(j, vr, vi, [&](int i, float& r, float& m) {
    r = valid ? __ldg(xr + i) : 0.f;
    m = valid ? __ldg(xi + i) : 0.f;
  });
  auto gstore = [&](int i, float r, float m) {
    if (valid) {
      yr[i] = r * sc;
      yi[i] = m * sc;
    }
  };
  if constexpr (S::P == 1) {
    pass_compute_store<LOGN, LOGE, 0, INV>(j, vr, vi, gstore);
  } else {
    float2* sb = reinterpret_cast<float2*>(sm) + g * GM::NP;
    pass_compute_store<LOGN, LOGE, 0, INV>(j, vr, vi, [&](int i, float r, float m) {
      sb[spad<S::SH>(i)] = make_float2(r, m);
    });
    __syncthreads();
    smem_passes<LOGN, LOGE, INV, 1, S::P - 1>(j, sb);
    pass_load<LOGN, LOGE, S::P - 1>(j, vr, vi, [&](int i, float& r, float& m) {
      { const float2 v_ = sb[spad<S::SH>(i)]; r = v_.x; m = v_.y; }
    });
    pass_compute_store<LOGN, LOGE, S::P - 1, INV>(j, vr, vi, gstore);
  }
}

// Runs the M-point forward FFT of the packed row through all passes and
// leaves the result in shared memory.
template <int LOGM, int LOGE, bool INV, class Ld>
__device__ __forceinline__ void fft_to_smem(int j, float2* sb, Ld ld) {
  using S = Sched<LOGM, LOGE>;
  float vr[S::E], vi[S::E];
  pass_load<LOGM, LOGE, 0>(j, vr, vi, ld);
  pass_compute_store<LOGM, LOGE, 0, INV>(j, vr, vi, [&](int i, float r, float m) {
    sb[spad<S::SH>(i)] = make_float2(r, m);
  });
  __syncthreads();
  smem_passes<LOGM, LOGE, INV, 1, S::P>(j, sb);
}

// ----------------------------------------------------------------------------
// Real -> complex, N = 2M.  Row t of x (length N) -> row t of y (H = M+1 bins).
template <int LOGM, int LOGE, int MINB = 1, int THR = kRowThreads>
__global__ void __launch_bounds__(THR, MINB) k_r2c(RowArgs a) {
  using S = Sched<LOGM, LOGE>;
  using GM = RowGeom<LOGM, LOGE, THR>;
  constexpr int M = S::N;
  constexpr int LOGN = LOGM + 1;
  extern __shared__ float sm[];
  const int g = threadIdx.x / S::T;
  const int j = threadIdx.x % S::T;
  const long long t = (long long)blockIdx.x * GM::G + g;
  const bool valid = t < a.batch;
  const long long tt = valid ? t : 0;
  const float* __restrict__ x = a.xr + tt * a.in_stride;
  float* __restrict__ yr = a.yr + tt * a.out_stride;
  float* __restrict__ yi = a.yi + tt * a.out_stride;
  float2* sb = reinterpret_cast<float2*>(sm) + g * GM::NP;

  fft_to_smem<LOGM, LOGE, false>(j, sb, [&](int i, float& r, float& m) {
    if (valid) {
      const float2 v = __ldg(reinterpret_cast<const float2*>(x) + i);
      r = v.x;
      m = v.y;
    } else {
      r = 0.f;
      m = 0.f;
    }
  });
  // split: X_k = E_k + W_N^k O_k, E = (Z_k + conj Z_{M-k})/2, O = (Z_k - conj Z_{M-k})/(2i)
  for (int k = j; k <= M; k += S::T) {
    const int k0 = k & (M - 1);
    const int k1 = (M - k) & (M - 1);
    const float2 z = sb[spad<S::SH>(k0)], w2 = sb[spad<S::SH>(k1)];
    const float zr = z.x, zi = z.y, wr = w2.x, wi = w2.y;
    const float er = 0.5f * (zr + wr), ei = 0.5f * (zi - wi);
    const float orr = 0.5f * (zi + wi), oi = 0.5f * (wr - zr);
    const float2 w = tw_lookup(k << (kTwLog - LOGN));  // k <= M = N/2: index < table size
    if (valid) {
      yr[k] = er + (orr * w.x - oi * w.y);
      yi[k] = ei + (orr * w.y + oi * w.x);
    }
  }
}

// ----------------------------------------------------------------------------
// Complex -> real, N = 2M.  Row t of the spectrum (bins 0..M) -> real row t.
template <int LOGM, int LOGE, int MINB = 1, int THR = kRowThreads>
__global__ void __launch_bounds__(THR, MINB) k_c2r(RowArgs a) {
  using S = Sched<LOGM, LOGE>;
  using GM = RowGeom<LOGM, LOGE, THR>;
  constexpr int M = S::N;
  constexpr int LOGN = LOGM + 1;
  extern __shared__ float sm[];
  const int g = threadIdx.x / S::T;
  const int j = threadIdx.x % S::T;
  const long long t = (long long)blockIdx.x * GM::G + g;
  const bool valid = t < a.batch;
  const long long tt = valid ? t : 0;
  const float* __restrict__ xr = a.xr + tt * a.in_stride;
  const float* __restrict__ xi = a.xi + tt * a.in_stride;
  float* __restrict__ y = a.yr + tt * a.out_stride;
  float2* sb = reinterpret_cast<float2*>(sm) + g * GM::NP;
  const float sc = a.scale;  // 1/N

  // Z_k = E_k + i O_k with E_k = (X_k + conj X_{M-k})/2, O_k = (X_k - conj X_{M-k}) conj(W_N^k)/2
  fft_to_smem<LOGM, LOGE, true>(j, sb, [&](int k, float& r, float& m) {
    if (!valid) {
      r = 0.f;
      m = 0.f;
      return;
    }
    const int km = M - k;  // in [1, M]
    float ar = __ldg(xr + k), ai = (k == 0) ? 0.f : __ldg(xi + k);
    float br = __ldg(xr + km), bi = (km == M) ? 0.f : __ldg(xi + km);
    const float er = ar + br, ei = ai - bi;      // 2 E_k
    const float dr = ar - br, di = ai + bi;      // X_k - conj X_{M-k}
    const float2 w = tw_lookup(k << (kTwLog - LOGN));
    // 2 O_k = d * conj(w)
    const float orr = dr * w.x + di * w.y;
    const float oi = di * w.x - dr * w.y;
    // 2 Z_k = 2E + i 2O
    r = er - oi;
    m = ei + orr;
  });
  // The loads carry 2Z; the unscaled inverse M-point transform of 2Z is 2M z = N z,
  // so multiplying by sc = 1/N yields z = (x[2n], x[2n+1]).
  if (valid) {
    float2* yo = reinterpret_cast<float2*>(y);
    for (int n = j; n < M; n += S::T) {
      const float2 v = sb[spad<S::SH>(n)];
      yo[n] = make_float2(v.x * sc, v.y * sc);
    }
  }
}

// ----------------------------------------------------------------------------
// Row-kernel tuning variants (values per thread E = 2^LOGE, min resident
// blocks per SM).  Variant 0 is the default; the others are selectable with
// the environment variable TRNFFT_B200_ROW_VARIANT for measurement.
template <int LOGE_, int MINB_, int THR_ = kRowThreads>
struct RowVar {
  static constexpr int LOGE = LOGE_;
  static constexpr int MINB = MINB_;
  static constexpr int THR = THR_;
};

template <int LOGN, bool INV, class V>
static cudaError_t launch_c2c_v(const RowArgs& a, cudaStream_t st) {
  constexpr int LE = V::LOGE;
  using GM = RowGeom<LOGN, LE, V::THR>;
  auto kern = k_c2c<LOGN, LE, INV, V::MINB, V::THR>;
  const size_t smem = (Sched<LOGN, LE>::P == 1) ? 0 : GM::smem;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = (a.batch + GM::G - 1) / GM::G;
  kern<<<(unsigned)blocks, V::THR, smem, st>>>(a);
  return cudaGetLastError();
}

// Measured defaults (B200, batches of 8M complex values, L2 flushed before each
// launch): 128-thread blocks everywhere from N = 256; radix-32 passes with four
// resident blocks per SM for N = 512, 1024, 4096; radix-16 with six for 256, 2048.
template <int LOGN>
constexpr int default_row_variant() {
  return (LOGN == 8 || LOGN == 11) ? 10 : ((LOGN == 9 || LOGN == 10 || LOGN == 12) ? 8 : 0);
}

// N = 8192 and 16384: one transform per block, E = 32 with 256 / 512 threads
// (measured 4.0 / 3.2 TB/s on B200 against 3.5 / 2.7 for E = 16 with 512 /
// 1024 threads, which TRNFFT_B200_ROW_VARIANT=20 selects).
template <int LOGN, bool INV>
static cudaError_t launch_c2c_big_tma(const RowArgs& a, cudaStream_t st);

template <int LOGN, bool INV>
static cudaError_t launch_c2c_big(const RowArgs& a, cudaStream_t st, int variant) {
  static_assert(LOGN == 13 || LOGN == 14, "single-block rows up to 16384 points");
  if (variant == 20) return launch_c2c_v<LOGN, INV, RowVar<4, LOGN == 13 ? 2 : 1, (1 << LOGN) / 16>>(a, st);
  // contiguous rows with 16-byte aligned planes: the persistent bulk-copy kernel
  const bool bulk = ((reinterpret_cast<uintptr_t>(a.xr) | reinterpret_cast<uintptr_t>(a.xi)) & 15) == 0 &&
                    a.in_stride == (1LL << LOGN);
  if (variant != 21 && bulk) return launch_c2c_big_tma<LOGN, INV>(a, st);
  return launch_c2c_v<LOGN, INV, RowVar<5, LOGN == 13 ? 2 : 1, (1 << LOGN) / 32>>(a, st);
}

template <int LOGN, bool INV>
static cudaError_t launch_c2c_t(const RowArgs& a, cudaStream_t st, int variant) {
  if constexpr (LOGN >= 13) {
    return launch_c2c_big<LOGN, INV>(a, st, variant);
  } else {
  if (variant < 0) variant = default_row_variant<LOGN>();
  if constexpr (LOGN >= 8) {
    switch (variant) {
      case 1: return launch_c2c_v<LOGN, INV, RowVar<4, 3>>(a, st);
      case 2: return launch_c2c_v<LOGN, INV, RowVar<5, 1>>(a, st);
      case 3: return launch_c2c_v<LOGN, INV, RowVar<5, 2>>(a, st);
      case 5: return launch_c2c_v<LOGN, INV, RowVar<4, 2>>(a, st);
      case 6: return launch_c2c_v<LOGN, INV, RowVar<5, 3>>(a, st);
      case 7: return launch_c2c_v<LOGN, INV, RowVar<5, 4>>(a, st);
      case 8:
        if constexpr (LOGN <= 12 && (1 << LOGN) / 32 <= 128) return launch_c2c_v<LOGN, INV, RowVar<5, 4, 128>>(a, st);
        break;
      case 9:
        if constexpr ((1 << LOGN) / 32 <= 128) return launch_c2c_v<LOGN, INV, RowVar<5, 6, 128>>(a, st);
        break;
      case 10:
        if constexpr ((1 << LOGN) / 16 <= 128) return launch_c2c_v<LOGN, INV, RowVar<4, 6, 128>>(a, st);
        break;
      case 11:
        if constexpr ((1 << LOGN) / 32 <= 64) return launch_c2c_v<LOGN, INV, RowVar<5, 8, 64>>(a, st);
        break;
      case 12:
        if constexpr ((1 << LOGN) / 16 <= 128) return launch_c2c_v<LOGN, INV, RowVar<4, 8, 128>>(a, st);
        break;
      case 13:
        if constexpr ((1 << LOGN) / 32 <= 128) return launch_c2c_v<LOGN, INV, RowVar<5, 5, 128>>(a, st);
        break;
      case 14:
        if constexpr ((1 << LOGN) / 16 <= 64) return launch_c2c_v<LOGN, INV, RowVar<4, 10, 64>>(a, st);
        break;
      default: break;
    }
  }
  return launch_c2c_v<LOGN, INV, RowVar<4, 1>>(a, st);
  }
}

// Real transforms run an M = N/2 point complex FFT: same measured block shapes
// as the complex kernel of that length.
template <int LOGM, int MODE, class V>
static cudaError_t launch_real_v(const RowArgs& a, cudaStream_t st) {
  constexpr int LE = V::LOGE;
  using GM = RowGeom<LOGM, LE, V::THR>;
  auto kern = (MODE == 0) ? k_r2c<LOGM, LE, V::MINB, V::THR> : k_c2r<LOGM, LE, V::MINB, V::THR>;
  const size_t smem = GM::smem;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = (a.batch + GM::G - 1) / GM::G;
  kern<<<(unsigned)blocks, V::THR, smem, st>>>(a);
  return cudaGetLastError();
}

template <int LOGM, int MODE>
static cudaError_t launch_real_t(const RowArgs& a, cudaStream_t st) {
  constexpr int v = default_row_variant<LOGM>();
  if constexpr (v == 10) return launch_real_v<LOGM, MODE, RowVar<4, 6, 128>>(a, st);
  if constexpr (v == 8) return launch_real_v<LOGM, MODE, RowVar<5, 4, 128>>(a, st);
  return launch_real_v<LOGM, MODE, RowVar<4, 1>>(a, st);
}

cudaError_t launch_rows_c2c(int logn, bool inv, const RowArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
  static const int variant = [] {
    const char* v = getenv("TRNFFT_B200_ROW_VARIANT");
    return v ? atoi(v) : -1;
  }();
#define TFB_C2C_CASE(L) \
  case L: return inv ? launch_c2c_t<L, true>(a, st, variant) : launch_c2c_t<L, false>(a, st, variant);
  switch (logn) {
    TFB_C2C_CASE(1) TFB_C2C_CASE(2) TFB_C2C_CASE(3) TFB_C2C_CASE(4)
    TFB_C2C_CASE(5) TFB_C2C_CASE(6) TFB_C2C_CASE(7) TFB_C2C_CASE(8)
    TFB_C2C_CASE(9) TFB_C2C_CASE(10) TFB_C2C_CASE(11) TFB_C2C_CASE(12)
    TFB_C2C_CASE(13) TFB_C2C_CASE(14)
    default: return cudaErrorInvalidValue;
  }
#undef TFB_C2C_CASE
}

cudaError_t launch_rows_r2c(int logm, const RowArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
#define TFB_R_CASE(L) case L: return launch_real_t<L, 0>(a, st);
  switch (logm) {
    TFB_R_CASE(1) TFB_R_CASE(2) TFB_R_CASE(3) TFB_R_CASE(4) TFB_R_CASE(5) TFB_R_CASE(6)
    TFB_R_CASE(7) TFB_R_CASE(8) TFB_R_CASE(9) TFB_R_CASE(10) TFB_R_CASE(11) TFB_R_CASE(12)
    default: return cudaErrorInvalidValue;
  }
#undef TFB_R_CASE
}

cudaError_t launch_rows_c2r(int logm, const RowArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
#define TFB_R_CASE(L) case L: return launch_real_t<L, 1>(a, st);
  switch (logm) {
    TFB_R_CASE(1) TFB_R_CASE(2) TFB_R_CASE(3) TFB_R_CASE(4) TFB_R_CASE(5) TFB_R_CASE(6)
    TFB_R_CASE(7) TFB_R_CASE(8) TFB_R_CASE(9) TFB_R_CASE(10) TFB_R_CASE(11) TFB_R_CASE(12)
    default: return cudaErrorInvalidValue;
  }
#undef TFB_R_CASE
}

}  // namespace tfb

// ============================================================================
// Persistent, bulk-copy-fed variant of k_c2c.
//
// Each block loops over tiles of G consecutive transforms (G*N floats per
// plane, contiguous in HBM).  One thread keeps STAGES tiles in flight with
// 1-D bulk copies (cp.async.bulk, the TMA engine) into shared-memory stage
// buffers; the block runs the Stockham passes of the current tile while the
// next tiles stream in, so HBM reads never wait for the arithmetic.  The last
// pass stores straight from registers to HBM (unit stride across threads).
// ============================================================================
namespace tfb {
__device__ int g_dev_status;  // see tma.cuh
}

namespace tfb {

template <int LOGN, int LOGE, int STAGES>
struct TmaGeom {
  using S = Sched<LOGN, LOGE>;
  static constexpr int G = kRowThreads / S::T;
  static constexpr int TILE = G * S::N;  // floats per plane per tile
  static constexpr int NP = S::NP;
  static constexpr size_t stage_bytes = (size_t)2 * TILE * sizeof(float);
  static constexpr size_t xbytes = (size_t)G * NP * sizeof(float2);
  static constexpr size_t bar_off = STAGES * stage_bytes + xbytes;
  static constexpr size_t smem = bar_off + STAGES * sizeof(uint64_t);
};

template <int LOGN, int LOGE, bool INV, int STAGES>
__global__ void __launch_bounds__(kRowThreads) k_c2c_tma(RowArgs a, long long ntiles) {
  using S = Sched<LOGN, LOGE>;
  using GM = TmaGeom<LOGN, LOGE, STAGES>;
  static_assert(S::P >= 2, "bulk-copy variant needs at least two passes");
  extern __shared__ __align__(128) unsigned char smraw[];
  float* stages = reinterpret_cast<float*>(smraw);
  float* xbase = reinterpret_cast<float*>(smraw + STAGES * GM::stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smraw + GM::bar_off);
  const int tid = threadIdx.x;
  const int g = tid / S::T;
  const int j = tid % S::T;
  float2* sb = reinterpret_cast<float2*>(xbase) + g * GM::NP;
  const float sc = a.scale;

  auto issue = [&](long long tile, int s) {
    const long long row0 = tile * GM::G;
    const long long rows = (a.batch - row0) < GM::G ? (a.batch - row0) : GM::G;
    const uint32_t bytes = (uint32_t)(rows * S::N * sizeof(float));
    float* dst = stages + (size_t)s * 2 * GM::TILE;
    mbar_arrive_expect_tx(&bars[s], 2 * bytes);
    bulk_g2s(dst, a.xr + row0 * S::N, bytes, &bars[s]);
    bulk_g2s(dst + GM::TILE, a.xi + row0 * S::N, bytes, &bars[s]);
  };

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
    mbar_init_fence();
  }
  __syncthreads();
  long long issued = 0;  // meaningful in thread 0 only
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      const long long tile = blockIdx.x + (long long)s * gridDim.x;
      if (tile < ntiles) {
        issue(tile, s);
        ++issued;
      }
    }
  }

  long long it = 0;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int s = (int)(it % STAGES);
    const uint32_t parity = (uint32_t)((it / STAGES) & 1);
    const bool ok = __syncthreads_and(mbar_wait_bounded(&bars[s], parity));
    if (!ok) {
      if (tid == 0) atomicExch(&g_dev_status, kStatusWaitTimeout);
      break;
    }
    const long long t = tile * GM::G + g;
    const bool valid = t < a.batch;
    const float* str = stages + (size_t)s * 2 * GM::TILE + g * S::N;
    const float* sti = str + GM::TILE;
    float vr[S::E], vi[S::E];
    pass_load<LOGN, LOGE, 0>(j, vr, vi, [&](int i, float& r, float& m) {
      r = str[i];
      m = sti[i];
    });
    __syncthreads();  // stage s fully read by every thread
    if (tid == 0) {
      const long long next = tile + (long long)STAGES * gridDim.x;
      if (next < ntiles) {
        fence_proxy_async();
        issue(next, s);
        ++issued;
      }
    }
    pass_compute_store<LOGN, LOGE, 0, INV>(j, vr, vi, [&](int i, float r, float m) {
      sb[spad<S::SH>(i)] = make_float2(r, m);
    });
    __syncthreads();
    smem_passes<LOGN, LOGE, INV, 1, S::P - 1>(j, sb);
    pass_load<LOGN, LOGE, S::P - 1>(j, vr, vi, [&](int i, float& r, float& m) {
      { const float2 v_ = sb[spad<S::SH>(i)]; r = v_.x; m = v_.y; }
    });
    float* yr = a.yr + (valid ? t : 0) * a.out_stride;
    float* yi = a.yi + (valid ? t : 0) * a.out_stride;
    pass_compute_store<LOGN, LOGE, S::P - 1, INV>(j, vr, vi, [&](int i, float r, float m) {
      if (valid) {
        yr[i] = r * sc;
        yi[i] = m * sc;
      }
    });
  }
  // After a timeout, drain (bounded) every copy this block still has in flight
  // before its shared memory is released.
  if (tid == 0) {
    for (long long k = it; k < issued; ++k)
      (void)mbar_wait_bounded(&bars[k % STAGES], (uint32_t)((k / STAGES) & 1));
  }
}

template <int LOGN, bool INV, int LOGE, int STAGES>
static cudaError_t launch_c2c_tma_v(const RowArgs& a, cudaStream_t st) {
  using GM = TmaGeom<LOGN, LOGE, STAGES>;
  auto kern = k_c2c_tma<LOGN, LOGE, INV, STAGES>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0, per_sm = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRowThreads, GM::smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const long long ntiles = (a.batch + GM::G - 1) / GM::G;
  long long grid = (long long)sms * per_sm;
  if (grid > ntiles) grid = ntiles;
  kern<<<(unsigned)grid, kRowThreads, GM::smem, st>>>(a, ntiles);
  return cudaGetLastError();
}

// ============================================================================
// Persistent bulk-copy-fed kernel for rows of 8192 / 16384 points.
//
// A transform of this length fills half of an SM's registers (E = 32 values
// per thread), so only one block fits per SM and a plain kernel leaves HBM
// idle while it computes.  Here one block per SM loops over the rows: the
// next row streams into a planar stage buffer (one bulk copy per plane) as
// soon as the current row has been read into registers, and the Stockham
// exchanges between passes go through a single float plane (real parts,
// then imaginary parts), so stage + exchange fit in shared memory together.
// ============================================================================
template <int LOGN>
struct BigGeom {
  static constexpr int LE = 5;
  using S = Sched<LOGN, LE>;
  static constexpr int THREADS = S::T;
  static constexpr size_t stage_bytes = (size_t)2 * S::N * sizeof(float);
  static constexpr int XP = S::N + (S::N >> LE);  // padded floats of the exchange plane
  static constexpr size_t bar_off = (stage_bytes + (size_t)XP * sizeof(float) + 15) / 16 * 16;
  static constexpr size_t smem = bar_off + 16;
};

// pass p outputs (registers) -> pass p+1 inputs (registers), one plane at a time
template <int LOGN, int LE, int p>
__device__ __forceinline__ void exchange_planes(int j, float (&vr)[Sched<LOGN, LE>::E], float (&vi)[Sched<LOGN, LE>::E],
                                                float* xb) {
  using S = Sched<LOGN, LE>;
  __syncthreads();  // the previous readers of xb are done
  pass_outputs<LOGN, LE, p>(j, [&](int s, int i) { xb[spad<S::SH>(i)] = vr[s]; });
  __syncthreads();
  pass_load<LOGN, LE, p + 1>(j, vr, vi, [&](int i, float& r, float&) { r = xb[spad<S::SH>(i)]; });
  __syncthreads();
  pass_outputs<LOGN, LE, p>(j, [&](int s, int i) { xb[spad<S::SH>(i)] = vi[s]; });
  __syncthreads();
  pass_load<LOGN, LE, p + 1>(j, vr, vi, [&](int i, float&, float& m) { m = xb[spad<S::SH>(i)]; });
}

template <int LOGN, int LE, bool INV, int p, int PLAST>
__device__ __forceinline__ void big_mid_passes(int j, float (&vr)[Sched<LOGN, LE>::E], float (&vi)[Sched<LOGN, LE>::E],
                                               float* xb) {
  if constexpr (p < PLAST) {
    pass_compute_store_qr<LOGN, LE, p, INV>(j, vr, vi, [&](int, int s, int, float x, float y) {
      vr[s] = x;
      vi[s] = y;
    });
    exchange_planes<LOGN, LE, p>(j, vr, vi, xb);
    big_mid_passes<LOGN, LE, INV, p + 1, PLAST>(j, vr, vi, xb);
  }
}

template <int LOGN, bool INV>
__global__ void __launch_bounds__(BigGeom<LOGN>::THREADS, 1) k_c2c_big(RowArgs a) {
  using GM = BigGeom<LOGN>;
  using S = typename GM::S;
  constexpr int N = S::N;
  extern __shared__ __align__(128) unsigned char smraw[];
  float* stage = reinterpret_cast<float*>(smraw);
  float* xb = reinterpret_cast<float*>(smraw + GM::stage_bytes);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smraw + GM::bar_off);
  const int tid = threadIdx.x;
  const int j = tid;
  const float sc = a.scale;
  auto issue = [&](long long row) {
    mbar_arrive_expect_tx(bar, 2u * N * (uint32_t)sizeof(float));
    bulk_g2s(stage, a.xr + row * N, N * (uint32_t)sizeof(float), bar);
    bulk_g2s(stage + N, a.xi + row * N, N * (uint32_t)sizeof(float), bar);
  };
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_init_fence();
  }
  __syncthreads();
  long long issued = 0;  // meaningful in thread 0 only
  if (tid == 0 && (long long)blockIdx.x < a.batch) {
    issue(blockIdx.x);
    ++issued;
  }
  long long it = 0;
  for (long long row = blockIdx.x; row < a.batch; row += gridDim.x, ++it) {
    const bool ok = __syncthreads_and(mbar_wait_bounded(bar, (uint32_t)(it & 1)));
    if (!ok) {
      if (tid == 0) atomicExch(&g_dev_status, kStatusWaitTimeout);
      break;
    }
    float vr[S::E], vi[S::E];
    pass_load<LOGN, GM::LE, 0>(j, vr, vi, [&](int i, float& r, float& m) {
      r = stage[i];
      m = stage[N + i];
    });
    __syncthreads();  // the stage has been read by every thread
    if (tid == 0) {
      const long long next = row + gridDim.x;
      if (next < a.batch) {
        fence_proxy_async();
        issue(next);
        ++issued;
      }
    }
    big_mid_passes<LOGN, GM::LE, INV, 0, S::P - 1>(j, vr, vi, xb);
    float* yr = a.yr + row * a.out_stride;
    float* yi = a.yi + row * a.out_stride;
    pass_compute_store<LOGN, GM::LE, S::P - 1, INV>(j, vr, vi, [&](int i, float r, float m) {
      yr[i] = r * sc;
      yi[i] = m * sc;
    });
  }
  // after a timeout, drain (bounded) the copy still in flight before the
  // block's shared memory is released
  if (tid == 0) {
    for (long long k = it; k < issued; ++k) (void)mbar_wait_bounded(bar, (uint32_t)(k & 1));
  }
}

template <int LOGN, bool INV>
static cudaError_t launch_c2c_big_tma(const RowArgs& a, cudaStream_t st) {
  using GM = BigGeom<LOGN>;
  auto kern = k_c2c_big<LOGN, INV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  long long grid = sms;
  if (grid > a.batch) grid = a.batch;
  kern<<<(unsigned)grid, GM::THREADS, GM::smem, st>>>(a);
  return cudaGetLastError();
}

bool rows_c2c_tma_ok(int logn, const RowArgs& a) {
  // 16-byte aligned planes with contiguous rows, two or more passes
  const bool al = ((reinterpret_cast<uintptr_t>(a.xr) | reinterpret_cast<uintptr_t>(a.xi)) & 15) == 0;
  return al && logn >= 6 && logn <= 12 && a.in_stride == (1LL << logn);
}

cudaError_t launch_rows_c2c_tma(int logn, bool inv, const RowArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
  static const int stages = [] {
    const char* v = getenv("TRNFFT_B200_TMA_STAGES");
    return (v && atoi(v) == 3) ? 3 : 2;
  }();
#define TFB_TMA_CASE(L)                                                                      \
  case L:                                                                                    \
    if (stages == 3)                                                                         \
      return inv ? launch_c2c_tma_v<L, true, 4, 3>(a, st) : launch_c2c_tma_v<L, false, 4, 3>(a, st); \
    return inv ? launch_c2c_tma_v<L, true, 4, 2>(a, st) : launch_c2c_tma_v<L, false, 4, 2>(a, st);
  switch (logn) {
    TFB_TMA_CASE(6) TFB_TMA_CASE(7) TFB_TMA_CASE(8) TFB_TMA_CASE(9)
    TFB_TMA_CASE(10) TFB_TMA_CASE(11) TFB_TMA_CASE(12)
    default: return cudaErrorInvalidValue;
  }
#undef TFB_TMA_CASE
}

}  // namespace tfb
