// Column-tile FFT pass: the building block of the multi-pass large-N
// transforms and of transforms along a strided axis (fft2 / fftn).
//
// A tile is CT neighbouring "columns" (unit stride in HBM) of L-point
// transforms whose points are `is_j` floats apart.  The block loads the tile
// with coalesced reads (CT consecutive floats per point), keeps each column
// as one padded float2 transform in shared memory, runs every Stockham pass
// of the L-point FFT on chip, applies an optional twiddle W_N^e, and stores
// the tile either column-wise again (KIND 0, in place allowed) or row-wise
// (KIND 1: column c becomes a contiguous run of L outputs, which is the
// transposition step of the four-step / six-step algorithm).
//
// Four-step reference: trnfft/nki/multicore.py:151-219 (column DFTs, twiddle
// exp(sign*2*pi*i*l*k1/N), row DFTs, column-major flatten), which runs the
// twiddle on the host and materialises two transposes.  Here the twiddle is
// fused into the pass that produces its operand and the transposes are the
// store pattern of the first pass.
#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGL>
struct ColGeom {
  static constexpr int LE = 4;
  using S = Sched<LOGL, LE>;
  static constexpr int L = S::N;
  static constexpr int CT0 = 256 / S::T;
  static constexpr int CT = CT0 < 8 ? 8 : (CT0 > 64 ? 64 : CT0);
  static constexpr int THREADS = CT * S::T;
  static constexpr int MINB = THREADS >= 1024 ? 1 : 1024 / THREADS;  // >= 1024 resident threads per SM
  // column pitch in float2: CT columns of one half-warp land in distinct banks
  static constexpr int R16 = CT >= 16 ? 1 : 16 / CT;
  static constexpr int PITCH = S::NP + ((R16 - (S::NP % 16)) + 16) % 16;
  static constexpr size_t smem = (size_t)CT * PITCH * sizeof(float2);
};

// W_N^e for e already reduced mod N (N = 2^logN <= 2^30): two-level table.
__device__ __forceinline__ float2 twiddle2(const ColArgs& a, uint32_t e) {
  const float2 hi = __ldg(a.tw_hi + (e >> a.tw_split));
  const float2 lo = __ldg(a.tw_lo + (e & ((1u << a.tw_split) - 1u)));
  return make_float2(hi.x * lo.x - hi.y * lo.y, hi.x * lo.y + hi.y * lo.x);
}

template <int LOGL, bool INV, int KIND>
__global__ void __launch_bounds__(ColGeom<LOGL>::THREADS, ColGeom<LOGL>::MINB) k_col(ColArgs a) {
  using GM = ColGeom<LOGL>;
  using S = typename GM::S;
  constexpr int L = GM::L;
  constexpr int CT = GM::CT;
  constexpr int THREADS = GM::THREADS;
  constexpr int ITER = CT * L / THREADS;  // elements per thread in the tile load/store
  constexpr int RSTEP = THREADS / CT;     // rows advanced per iteration (column-wise mapping)
  static_assert(THREADS % CT == 0 && (CT * L) % THREADS == 0, "tile mapping");
  extern __shared__ float2 sm2[];
  const int tid = threadIdx.x;
  const long long tile = blockIdx.x;
  const long long ncb = (a.ncols + CT - 1) / CT;
  const long long cb = tile % ncb;
  long long rest = tile / ncb;
  const long long o1 = rest % a.O1;
  rest /= a.O1;
  const long long o2 = rest % a.O2;
  const long long o3 = rest / a.O2;
  const long long c0 = cb * CT;
  const long long ibase = o1 * a.is_o1 + o2 * a.is_o2 + o3 * a.is_o3;
  const long long obase = o1 * a.os_o1 + o2 * a.os_o2 + o3 * a.os_o3;

  // ---- tile load: thread owns column cl and rows r0 + i*RSTEP; every load is
  // issued before the first shared-memory store.
  const int cl = tid % CT;
  const int r0 = tid / CT;
  const bool colok = c0 + cl < a.ncols;
  {
    const long long base = ibase + c0 + cl + (long long)r0 * a.is_j;
    const float* __restrict__ pr = a.xr + base;
    const float* __restrict__ pi = a.xi + base;
    const long long step = (long long)RSTEP * a.is_j;
    float vr[ITER], vi[ITER];
#pragma unroll
    for (int i = 0; i < ITER; ++i) {
      vr[i] = colok ? __ldg(pr + i * step) : 0.f;
      vi[i] = colok ? __ldg(pi + i * step) : 0.f;
    }
    float2* dst = sm2 + cl * GM::PITCH;
#pragma unroll
    for (int i = 0; i < ITER; ++i) dst[spad<S::SH>(r0 + i * RSTEP)] = make_float2(vr[i], vi[i]);
  }
  __syncthreads();
  {
    const int col = tid / S::T;
    const int j = tid % S::T;
    smem_passes<LOGL, GM::LE, INV, 0, S::P>(j, sm2 + col * GM::PITCH);
  }

  // ---- twiddle + store.  The exponent for output k of column cg is
  // e = tw_mul*(o1*(tw_a*cg + tw_b*k) + tw_c*cg*k) = A1*cg + k*(B1 + C1*cg),
  // evaluated mod 2^32 and then reduced mod N (N divides 2^32).  Along each
  // thread's sequence of outputs the exponent grows by a fixed step, so the
  // twiddle is carried by complex multiplication and re-read from the table
  // every kAnchor outputs (bounded rounding growth, few scattered lookups).
  constexpr int kAnchor = 8;
  const uint32_t nmask = (uint32_t)a.nmask;
  const long long od = o1 % a.tw_modo;  // the input digit this twiddle multiplies
  const uint32_t A1 = (uint32_t)(a.tw_mul * od * a.tw_a);
  const uint32_t B1 = (uint32_t)(a.tw_mul * od * a.tw_b);
  const uint32_t C1 = (uint32_t)(a.tw_mul * a.tw_c);
  const bool tw = a.has_tw != 0;
  const float sc = a.scale;
  auto cmul = [](float2 x, float2 y) { return make_float2(x.x * y.x - x.y * y.y, x.x * y.y + x.y * y.x); };
  auto look = [&](uint32_t e) {
    float2 w = twiddle2(a, e & nmask);
    if (INV) w.y = -w.y;
    return w;
  };
  if constexpr (KIND == 2) {
    // column-wise like kind 0, each output stored into its owner rank's row
    // buffer (peer memory over NVLink for the other ranks)
    if (colok) {
      const long long cg = c0 + cl;
      const float2* src = sm2 + cl * GM::PITCH;
      const uint32_t cgt = (uint32_t)(cg + a.tw_coff);
      const uint32_t de = B1 + C1 * cgt;
      const uint32_t e0 = A1 * cgt + (uint32_t)r0 * de;
      float2 w = make_float2(1.f, 0.f), d = w;
      if (tw) d = look((uint32_t)RSTEP * de);
#pragma unroll
      for (int i = 0; i < ITER; ++i) {
        const int k = r0 + i * RSTEP;
        float2 v = src[spad<S::SH>(k)];
        if (tw) {
          w = (i % kAnchor == 0) ? look(e0 + (uint32_t)i * RSTEP * de) : cmul(w, d);
          v = cmul(v, w);
        }
        const long long K = o1 * a.sc_ka + (long long)k * a.sc_kb;
        const int q = (int)(K / a.sc_rows);
        const long long off = (K - (long long)q * a.sc_rows) * a.sc_ld + a.sc_col0 + cg;
        if (q < a.sc_npeers) {
          a.sc_re[q][off] = v.x * sc;
          a.sc_im[q][off] = v.y * sc;
        }
      }
    }
    __threadfence_system();
  } else if constexpr (KIND == 0) {
    // column-wise, same thread mapping as the load: k = r0 + i*RSTEP
    if (colok) {
      const long long cg = c0 + cl;
      const long long base = obase + cg + (long long)r0 * a.os_k;
      float* __restrict__ qr = a.yr + base;
      float* __restrict__ qi = a.yi + base;
      const long long step = (long long)RSTEP * a.os_k;
      const float2* src = sm2 + cl * GM::PITCH;
      const uint32_t cgt = (uint32_t)(cg + a.tw_coff);
      const uint32_t de = B1 + C1 * cgt;
      const uint32_t e0 = A1 * cgt + (uint32_t)r0 * de;
      float2 w = make_float2(1.f, 0.f), d = w;
      if (tw) d = look((uint32_t)RSTEP * de);
#pragma unroll
      for (int i = 0; i < ITER; ++i) {
        float2 v = src[spad<S::SH>(r0 + i * RSTEP)];
        if (tw) {
          w = (i % kAnchor == 0) ? look(e0 + (uint32_t)i * RSTEP * de) : cmul(w, d);
          v = cmul(v, w);
        }
        qr[i * step] = v.x * sc;
        qi[i * step] = v.y * sc;
      }
    }
  } else {
    // row-wise: consecutive threads take consecutive k of one column
    float* __restrict__ qr0 = a.yr + obase;
    float* __restrict__ qi0 = a.yi + obase;
    if constexpr (THREADS <= L) {
      constexpr int R = L / THREADS;  // k = q*THREADS + tid, columns c = 0..CT-1
#pragma unroll
      for (int q = 0; q < R; ++q) {
        const int k = q * THREADS + tid;
        const uint32_t mstep = A1 + C1 * (uint32_t)k;  // exponent step per column
        const uint32_t coff = (uint32_t)a.tw_coff;
        float2 w = make_float2(1.f, 0.f), m = w;
        if (tw) m = look(mstep);
#pragma unroll
        for (int c = 0; c < CT; ++c) {
          const long long cg = c0 + c;
          if (cg < a.ncols) {
            float2 v = sm2[c * GM::PITCH + spad<S::SH>(k)];
            if (tw) {
              w = (c % kAnchor == 0)
                      ? look(A1 * ((uint32_t)cg + coff) + (uint32_t)k * (B1 + C1 * ((uint32_t)cg + coff)))
                      : cmul(w, m);
              v = cmul(v, w);
            }
            const long long off = cg * a.os_c + k;
            qr0[off] = v.x * sc;
            qi0[off] = v.y * sc;
          }
        }
      }
    } else {
      constexpr int CPI = THREADS / L;  // columns per iteration; k fixed per thread
      const int k = tid % L;
      const int cst = tid / L;
      const uint32_t mstep = (uint32_t)CPI * (A1 + C1 * (uint32_t)k);
      float2 w = make_float2(1.f, 0.f), m = w;
      if (tw) m = look(mstep);
#pragma unroll
      for (int i = 0; i < ITER; ++i) {
        const int c = i * CPI + cst;
        const long long cg = c0 + c;
        float2 v = sm2[c * GM::PITCH + spad<S::SH>(k)];
        if (tw) {
          const uint32_t cgt = (uint32_t)cg + (uint32_t)a.tw_coff;
          w = (i % kAnchor == 0) ? look(A1 * cgt + (uint32_t)k * (B1 + C1 * cgt)) : cmul(w, m);
          v = cmul(v, w);
        }
        if (cg < a.ncols) {
          const long long off = cg * a.os_c + k;
          qr0[off] = v.x * sc;
          qi0[off] = v.y * sc;
        }
      }
    }
  }
}

template <int LOGL, bool INV, int KIND>
static cudaError_t launch_col_t(const ColArgs& a, cudaStream_t st) {
  using GM = ColGeom<LOGL>;
  auto kern = k_col<LOGL, INV, KIND>;
  if (GM::smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e0 = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e0 != cudaSuccess) return e0;
  const long long ncb = (a.ncols + GM::CT - 1) / GM::CT;
  const long long tiles = ncb * a.O1 * a.O2 * a.O3;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)tiles, GM::THREADS, GM::smem, st>>>(a);
  return cudaGetLastError();
}

template <int LOGL>
static cudaError_t launch_col_l(bool inv, int kind, const ColArgs& a, cudaStream_t st) {
  if (kind == 0) return inv ? launch_col_t<LOGL, true, 0>(a, st) : launch_col_t<LOGL, false, 0>(a, st);
  if (kind == 2) return inv ? launch_col_t<LOGL, true, 2>(a, st) : launch_col_t<LOGL, false, 2>(a, st);
  return inv ? launch_col_t<LOGL, true, 1>(a, st) : launch_col_t<LOGL, false, 1>(a, st);
}

cudaError_t launch_colpass(int logl, bool inv, int kind, const ColArgs& a, cudaStream_t st) {
  switch (logl) {
    case 1: return launch_col_l<1>(inv, kind, a, st);
    case 2: return launch_col_l<2>(inv, kind, a, st);
    case 3: return launch_col_l<3>(inv, kind, a, st);
    case 4: return launch_col_l<4>(inv, kind, a, st);
    case 5: return launch_col_l<5>(inv, kind, a, st);
    case 6: return launch_col_l<6>(inv, kind, a, st);
    case 7: return launch_col_l<7>(inv, kind, a, st);
    case 8: return launch_col_l<8>(inv, kind, a, st);
    case 9: return launch_col_l<9>(inv, kind, a, st);
    case 10: return launch_col_l<10>(inv, kind, a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tfb
