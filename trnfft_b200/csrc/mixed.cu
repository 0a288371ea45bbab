// Direct mixed-radix transforms for 7-smooth lengths (n = 2^a 3^b 5^c 7^d,
// not a power of two, n <= 8192), one whole transform per group of threads.
//
// Reference: every n that is not a power of two goes through Bluestein in
// trnfft (fft_core.py:44-50 -> _bluestein, :1285-1376): three power-of-two
// FFTs of the padded length m = 2^bitlen(2n-2) (m = 2048 for n = 1000, 16384
// for n = 6000).  For lengths whose prime factors are all small, a
// Stockham transform with radix 2/3/4/5/7/8/16 passes does the same DFT with
// one n-point transform: several times fewer operations and still one HBM
// read and one HBM write per element.  Results agree with the reference's to
// float32 rounding (both are the DFT of the same input).
//
// Pass p has radix R and span ns = R_0 ... R_{p-1}: butterfly b < n/R reads
// x[b + r n/R], multiplies by W_{ns R}^{(b mod ns) r} (a per-plan table laid
// out pass by pass, [k][r], computed in double), runs an R-point DFT in
// registers and writes
// y[(b / ns) ns R + (b mod ns) + r ns].  The first pass reads HBM directly
// (unit stride across threads) and the last writes HBM directly; the passes
// in between alternate between two padded float2 rows in shared memory.  The radix of
// each pass is a run-time value: a switch picks the register-resident pass
// specialised for it.
#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGNMAX>
struct MixGeom {
  static constexpr int NMAX = 1 << LOGNMAX;
  static constexpr int T = NMAX / 16 < 4 ? 4 : NMAX / 16;  // threads per transform: ~16 values each
  static constexpr int G = T >= 256 ? 1 : 256 / T;         // transforms per block
  static constexpr int THREADS = G * T;
  static constexpr int MINB = 1024 / THREADS >= 4 ? 4 : 1024 / THREADS;  // <= 64 registers a thread
};

__host__ __device__ __forceinline__ int mpad(int i) { return i + (i >> 5); }

// In-register R-point DFT in natural output order (X_k in slot k).
template <int R, bool INV>
__device__ __forceinline__ void dft_any(float (&re)[R], float (&im)[R]) {
  if constexpr ((R & (R - 1)) == 0) {
    dft_reg<R, INV>(re, im);  // bit-reversed output order
    float tr[R], ti[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      tr[k] = re[ct_bitrev(k, ct_log2(R))];
      ti[k] = im[ct_bitrev(k, ct_log2(R))];
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      re[k] = tr[k];
      im[k] = ti[k];
    }
  } else {
    // odd R: X_k = x_0 + sum_{j=1}^{(R-1)/2} [(x_j + x_{R-j}) cos(2 pi j k / R)
    //                                          -+ i (x_j - x_{R-j}) sin(2 pi j k / R)]
    constexpr int H = (R - 1) / 2;
    float sr[H + 1], si[H + 1], dr[H + 1], di[H + 1];
#pragma unroll
    for (int j = 1; j <= H; ++j) {
      sr[j] = re[j] + re[R - j];
      si[j] = im[j] + im[R - j];
      dr[j] = re[j] - re[R - j];
      di[j] = im[j] - im[R - j];
    }
    float outr[R], outi[R];
    float s0r = re[0], s0i = im[0];
#pragma unroll
    for (int j = 1; j <= H; ++j) {
      s0r += sr[j];
      s0i += si[j];
    }
    outr[0] = s0r;
    outi[0] = s0i;
#pragma unroll
    for (int k = 1; k <= H; ++k) {
      float ar = re[0], ai = im[0], br = 0.f, bi = 0.f;
#pragma unroll
      for (int j = 1; j <= H; ++j) {
        const float c = (float)ct_cos(ct_angle((long)j * k, R));
        const float s = (float)ct_sin(ct_angle((long)j * k, R));
        ar = fmaf(sr[j], c, ar);
        ai = fmaf(si[j], c, ai);
        br = fmaf(dr[j], s, br);
        bi = fmaf(di[j], s, bi);
      }
      // forward: X_k = A - i B, X_{R-k} = A + i B with B = sum d_j sin; inverse swaps
      if (INV) {
        outr[k] = ar - bi;
        outi[k] = ai + br;
        outr[R - k] = ar + bi;
        outi[R - k] = ai - br;
      } else {
        outr[k] = ar + bi;
        outi[k] = ai - br;
        outr[R - k] = ar - bi;
        outi[R - k] = ai + br;
      }
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      re[k] = outr[k];
      im[k] = outi[k];
    }
  }
}

// One pass of radix R from `src` to `dst` (padded float2 rows in shared
// memory).  FIRST: inputs from HBM through `ld(i, re, im)` (all of a thread's
// loads are issued before any arithmetic, to keep HBM requests in flight);
// LAST: outputs to HBM through `st(i, re, im)`.  Middle passes load, transform
// and store one butterfly at a time (the two buffers alternate), so a thread
// holds only R values.  `twp` is this pass's twiddle block: entry
// (r-1)*ns + k = W_{ns R}^{k r}, so for each r the butterflies of a warp
// (consecutive k) read consecutive entries.
template <int R, bool INV, int LOGNMAX, bool FIRST, bool LAST, class Ld, class St>
__device__ __forceinline__ void mix_pass(const float2* src, float2* dst, int j0, int n, int ns,
                                         const float2* __restrict__ twp, Ld ld, St st) {
  using GM = MixGeom<LOGNMAX>;
  constexpr int Q = (16 + R - 1) / R;  // butterflies per thread (n <= NMAX = 16 T)
  const int nb = n / R;
  auto butterfly = [&](int b, float (&vr)[R], float (&vi)[R]) {
    const int hi = b / ns;
    const int k = b - hi * ns;
    if (ns > 1) {
#pragma unroll
      for (int r = 1; r < R; ++r) {
        float2 w = __ldg(twp + (r - 1) * ns + k);
        if (INV) w.y = -w.y;
        const float xr = vr[r], xi = vi[r];
        vr[r] = fmaf(xr, w.x, -xi * w.y);
        vi[r] = fmaf(xr, w.y, xi * w.x);
      }
    }
    dft_any<R, INV>(vr, vi);
    const int base = hi * ns * R + k;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = base + r * ns;
      if constexpr (LAST) {
        st(i, vr[r], vi[r]);
      } else {
        dst[mpad(i)] = make_float2(vr[r], vi[r]);
      }
    }
  };
  if constexpr (FIRST) {
    float vr[Q][R], vi[Q][R];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int b = j0 + q * GM::T;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (b < nb) {
          ld(b + r * nb, vr[q][r], vi[q][r]);
        } else {
          vr[q][r] = 0.f;
          vi[q][r] = 0.f;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int b = j0 + q * GM::T;
      if (b < nb) butterfly(b, vr[q], vi[q]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int b = j0 + q * GM::T;
      if (b >= nb) break;
      float vr[R], vi[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float2 v = src[mpad(b + r * nb)];
        vr[r] = v.x;
        vi[r] = v.y;
      }
      butterfly(b, vr, vi);
    }
  }
  if constexpr (!LAST) __syncthreads();
}

// Radix codes (3 bits per pass in MixedArgs::codes): 0..6 = 2, 3, 4, 5, 7, 8, 16.
__host__ __device__ constexpr int mix_radix_of(int code) {
  return code == 0 ? 2 : code == 1 ? 3 : code == 2 ? 4 : code == 3 ? 5 : code == 4 ? 7 : code == 5 ? 8 : 16;
}

template <bool INV, int LOGNMAX, bool FIRST, bool LAST, class Ld, class St>
__device__ __forceinline__ void mix_pass_r(int code, const float2* src, float2* dst, int j0, int n, int ns,
                                           const float2* twp, Ld ld, St st) {
  switch (code) {
    case 0: mix_pass<2, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    case 1: mix_pass<3, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    case 2: mix_pass<4, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    case 3: mix_pass<5, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    case 4: mix_pass<7, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    case 5: mix_pass<8, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
    default: mix_pass<16, INV, LOGNMAX, FIRST, LAST>(src, dst, j0, n, ns, twp, ld, st); break;
  }
}

// MODE 0: C2C; MODE 1: R2C (real rows -> n/2+1 bins); MODE 2: C2R (n/2+1 bins -> real rows).
// The real modes transform two rows at once (a + i b in, the two spectra separated on chip;
// or A + i B in, real and imaginary parts out as the two rows).
template <int LOGNMAX, bool INV, int MODE>
__global__ void __launch_bounds__(MixGeom<LOGNMAX>::THREADS, MixGeom<LOGNMAX>::MINB) k_mixed(MixedArgs a) {
  using GM = MixGeom<LOGNMAX>;
  extern __shared__ float2 sm2[];
  const int g = threadIdx.x / GM::T;
  const int j0 = threadIdx.x % GM::T;
  const int n = a.n;
  const long long t = (long long)blockIdx.x * GM::G + g;
  // the real modes pack rows 2t and 2t+1 into one complex transform
  const long long ntf = MODE == 0 ? a.batch : (a.batch + 1) / 2;
  const bool valid = t < ntf;
  const long long tt = valid ? t : 0;
  const long long row0 = MODE == 0 ? tt : 2 * tt;
  const bool has1 = MODE != 0 && row0 + 1 < a.batch;
  float2* buf0 = sm2 + g * 2 * a.pitch;
  float2* buf1 = buf0 + a.pitch;
  const int half = n / 2;
  const long long hbins = half + 1;
  auto ld = [&](int i, float& r, float& m) {
    r = 0.f;
    m = 0.f;
    if (!valid) return;
    if constexpr (MODE == 0) {
      r = __ldg(a.xr + tt * n + i);
      m = __ldg(a.xi + tt * n + i);
    } else if constexpr (MODE == 1) {
      // z = a + i b for the real rows a = 2t, b = 2t+1
      r = __ldg(a.xr + row0 * n + i);
      m = has1 ? __ldg(a.xr + (row0 + 1) * n + i) : 0.f;
    } else {
      // Z = A + i B for the Hermitian extensions A, B of rows 2t, 2t+1 (trnfft/api.py:54-66);
      // the imaginary parts of bin 0 and (even n) bin n/2 do not contribute to a real result
      const int src = i <= half ? i : n - i;
      const float sg = i <= half ? 1.f : -1.f;
      const bool im_ok = !(src == 0 || 2 * src == n);
      const float ar = __ldg(a.xr + row0 * hbins + src);
      const float ai = im_ok ? sg * __ldg(a.xi + row0 * hbins + src) : 0.f;
      float br = 0.f, bi = 0.f;
      if (has1) {
        br = __ldg(a.xr + (row0 + 1) * hbins + src);
        bi = im_ok ? sg * __ldg(a.xi + (row0 + 1) * hbins + src) : 0.f;
      }
      r = ar - bi;
      m = ai + br;
    }
  };
  float2* zb = buf1;  // MODE 1: the packed spectrum Z is gathered here before the split
  auto st = [&](int i, float r, float m) {
    if constexpr (MODE == 0) {
      if (!valid) return;
      a.yr[tt * n + i] = r * a.scale;
      a.yi[tt * n + i] = m * a.scale;
    } else if constexpr (MODE == 1) {
      zb[mpad(i)] = make_float2(r, m);
    } else {
      if (!valid) return;
      a.yr[row0 * n + i] = r * a.scale;
      if (has1) a.yr[(row0 + 1) * n + i] = m * a.scale;
    }
  };
  const int P = a.npass;
  const unsigned long long codes = a.codes;
  int code = (int)(codes & 7);
  if (P == 1) {
    mix_pass_r<INV, LOGNMAX, true, true>(code, buf0, buf1, j0, n, 1, a.tw, ld, st);
  } else {
    // per-pass twiddle blocks follow each other: pass p takes ns_p * (R_p - 1) entries
    int ns = 1;
    long long off = 0;
    mix_pass_r<INV, LOGNMAX, true, false>(code, buf1, buf0, j0, n, ns, a.tw + off, ld, st);
    off += (long long)ns * (mix_radix_of(code) - 1);
    ns *= mix_radix_of(code);
    float2* src = buf0;
    float2* dst = buf1;
    for (int p = 1; p < P - 1; ++p) {
      code = (int)((codes >> (3 * p)) & 7);
      mix_pass_r<INV, LOGNMAX, false, false>(code, src, dst, j0, n, ns, a.tw + off, ld, st);
      off += (long long)ns * (mix_radix_of(code) - 1);
      ns *= mix_radix_of(code);
      float2* tmp = src;
      src = dst;
      dst = tmp;
    }
    zb = dst;  // the last pass reads src; MODE 1 writes Z into the other row buffer
    code = (int)((codes >> (3 * (P - 1))) & 7);
    mix_pass_r<INV, LOGNMAX, false, true>(code, src, dst, j0, n, ns, a.tw + off, ld, st);
  }
  if constexpr (MODE == 1) {
    // Z = FFT(a + i b): A_k = (Z_k + conj Z_{n-k}) / 2, B_k = (Z_k - conj Z_{n-k}) / (2i)
    __syncthreads();
    if (valid) {
      for (int k = j0; k <= half; k += GM::T) {
        const float2 z = zb[mpad(k)];
        const float2 w = zb[mpad(k == 0 ? 0 : n - k)];
        a.yr[row0 * hbins + k] = 0.5f * (z.x + w.x);
        a.yi[row0 * hbins + k] = 0.5f * (z.y - w.y);
        if (has1) {
          a.yr[(row0 + 1) * hbins + k] = 0.5f * (z.y + w.y);
          a.yi[(row0 + 1) * hbins + k] = 0.5f * (w.x - z.x);
        }
      }
    }
  }
}

template <int LOGNMAX, bool INV, int MODE>
static cudaError_t launch_mixed_t(MixedArgs a, cudaStream_t st) {
  using GM = MixGeom<LOGNMAX>;
  a.pitch = mpad(a.n) + 1;
  const size_t smem = (size_t)GM::G * 2 * a.pitch * sizeof(float2);
  auto kern = k_mixed<LOGNMAX, INV, MODE>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long ntf = MODE == 0 ? a.batch : (a.batch + 1) / 2;  // real modes: two rows per transform
  const long long blocks = (ntf + GM::G - 1) / GM::G;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, GM::THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

template <int LOGNMAX>
static cudaError_t launch_mixed_c(int mode, bool inv, const MixedArgs& a, cudaStream_t st) {
  switch (mode) {
    case 0: return inv ? launch_mixed_t<LOGNMAX, true, 0>(a, st) : launch_mixed_t<LOGNMAX, false, 0>(a, st);
    case 1: return launch_mixed_t<LOGNMAX, false, 1>(a, st);
    case 2: return launch_mixed_t<LOGNMAX, true, 2>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_mixed(int mode, bool inv, const MixedArgs& a, cudaStream_t st) {
  if (a.batch <= 0) return cudaSuccess;
  if (a.n <= 64) return launch_mixed_c<6>(mode, inv, a, st);
  if (a.n <= 256) return launch_mixed_c<8>(mode, inv, a, st);
  if (a.n <= 1024) return launch_mixed_c<10>(mode, inv, a, st);
  if (a.n <= 4096) return launch_mixed_c<12>(mode, inv, a, st);
  if (a.n <= 8192) return launch_mixed_c<13>(mode, inv, a, st);
  return cudaErrorInvalidValue;
}

}  // namespace tfb
