// Column-tile FFT pass: the building block of the multi-pass large-N
// transforms and of transforms along a strided axis (fft2 / fftn).
//
// A tile is CT neighbouring "columns" (unit stride in HBM) of L-point
// transforms whose points are `is_j` floats apart.  Thread (column, lane)
// loads its first-pass inputs straight from HBM (a warp reads one contiguous
// run of 32 columns per point), the middle Stockham passes exchange through
// a shared [L][CT+1] tile, and the last pass applies an optional twiddle
// W_N^e in registers and stores either column-wise (KIND 0, in place
// allowed), into the owning rank's row buffer (KIND 2, the four-step exchange
// over NVLink), or row-wise through shared memory (KIND 1: column c becomes a
// contiguous run of L outputs, the transposition step of the four-step /
// six-step algorithm).
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
  static constexpr int T = S::T;  // threads per column
  // columns per tile: a warp covers 32 (or 16 for L >= 512) neighbouring
  // columns at one butterfly index, so every global access of a warp is one
  // contiguous 128-byte run (64-byte runs lose up to half the HBM bandwidth
  // when the rows are a large power of two apart); small L take several such
  // groups to keep 128+ threads.  Only L = 1024 falls back to 16 columns (a
  // 32-column tile would not fit in shared memory).
  static constexpr int CW = 32 * T <= 1024 ? 32 : 16;
  static constexpr int G = CW * T >= 128 ? 1 : 128 / (CW * T);
  static constexpr int CT = CW * G;
  static constexpr int THREADS = CT * T;
  static constexpr int MINB = THREADS >= 1024 ? 1 : 1024 / THREADS;  // >= 1024 resident threads per SM
  // shared tile [L][CT] of float2 with an odd pitch: a warp's accesses at one
  // point index are contiguous, and the row-wise read-out (consecutive points
  // of one column) steps 2*SP banks, conflict-free per half-warp.
  static constexpr int SP = CT + 1;
  static constexpr size_t smem_bytes(int kind) {
    return (S::P > 1 || kind == 1) ? (size_t)L * SP * sizeof(float2) : 0;
  }
};

// W_N^e for e already reduced mod N (N = 2^logN <= 2^30): two-level table.
__device__ __forceinline__ float2 twiddle2(const ColArgs& a, uint32_t e) {
  const float2 hi = __ldg(a.tw_hi + (e >> a.tw_split));
  const float2 lo = __ldg(a.tw_lo + (e & ((1u << a.tw_split) - 1u)));
  return make_float2(hi.x * lo.x - hi.y * lo.y, hi.x * lo.y + hi.y * lo.x);
}

// Stockham passes p .. PLAST-1 of one column through shared memory: on entry
// (vr, vi) hold pass p's inputs, on return pass PLAST's inputs.  `col` points
// at the column's first element; point i lives at col[i * SP].
template <int LOGL, int LE, bool INV, int p, int PLAST, int SP>
__device__ __forceinline__ void col_mid_passes(int j, float (&vr)[Sched<LOGL, LE>::E],
                                               float (&vi)[Sched<LOGL, LE>::E], float2* col) {
  if constexpr (p < PLAST) {
    if constexpr (p > 0) __syncthreads();  // pass p's inputs have been read by every thread
    pass_compute_store<LOGL, LE, p, INV>(j, vr, vi, [&](int i, float x, float y) { col[i * SP] = make_float2(x, y); });
    __syncthreads();
    pass_load<LOGL, LE, p + 1>(j, vr, vi, [&](int i, float& x, float& y) {
      const float2 v = col[i * SP];
      x = v.x;
      y = v.y;
    });
    col_mid_passes<LOGL, LE, INV, p + 1, PLAST, SP>(j, vr, vi, col);
  }
}

// x / d and x mod d for the tile decode: shift and mask when d = 2^lg
__device__ __forceinline__ uint32_t qdiv(uint32_t x, uint32_t d, int lg) { return lg >= 0 ? x >> lg : x / d; }
__device__ __forceinline__ uint32_t qmod(uint32_t x, uint32_t d, int lg) {
  return lg >= 0 ? x & ((1u << lg) - 1u) : x % d;
}

// OFF: the integer type of element offsets inside one tile (int when they all
// fit in 31 bits, which saves the 64-bit multiplies of every access).
template <int LOGL, bool INV, int KIND, class OFF>
__device__ __forceinline__ void col_tile(const ColArgs& a, const uint32_t tile, float* const* s_re,
                                         float* const* s_im) {
  using GM = ColGeom<LOGL>;
  using S = typename GM::S;
  constexpr int L = GM::L;
  constexpr int CT = GM::CT;
  constexpr int SP = GM::SP;
  constexpr int THREADS = GM::THREADS;
  constexpr int PL = S::P - 1;                        // the last Stockham pass
  constexpr int NSL = 1 << S::logns(PL);              // its output stride
  extern __shared__ float2 sm2[];
  const int tid = threadIdx.x;
  const uint32_t cb = qmod(tile, a.d_ncb, a.lg_ncb);
  uint32_t rest = qdiv(tile, a.d_ncb, a.lg_ncb);
  const uint32_t o1 = qmod(rest, a.d_O1, a.lg_O1);
  rest = qdiv(rest, a.d_O1, a.lg_O1);
  const uint32_t o2 = qmod(rest, a.d_O2, a.lg_O2);
  const uint32_t o3 = qdiv(rest, a.d_O2, a.lg_O2);
  const long long c0 = (long long)cb * CT;
  const long long ibase = (long long)o1 * a.is_o1 + (long long)o2 * a.is_o2 + (long long)o3 * a.is_o3;
  const long long obase = (long long)o1 * a.os_o1 + (long long)o2 * a.os_o2 + (long long)o3 * a.os_o3;

  // thread = (column cl, butterfly lane j); pass 0 reads straight from HBM
  const int cl = tid % CT;
  const int j = tid / CT;
  const bool colok = c0 + cl < a.ncols;
  const long long cg = c0 + cl;
  float vr[S::E], vi[S::E];
  {
    const float* __restrict__ pr = a.xr + ibase + cg;
    const float* __restrict__ pi = a.xi + ibase + cg;
    const OFF is = (OFF)a.is_j;
    pass_load<LOGL, GM::LE, 0>(j, vr, vi, [&](int n, float& x, float& y) {
      x = colok ? __ldg(pr + (OFF)n * is) : 0.f;
      y = colok ? __ldg(pi + (OFF)n * is) : 0.f;
    });
  }
  float2* col = sm2 + cl;
  col_mid_passes<LOGL, GM::LE, INV, 0, PL, SP>(j, vr, vi, col);

  // ---- last pass + twiddle + store.  The exponent for output k of column cg
  // is e = tw_mul*(o1*(tw_a*cg + tw_b*k) + tw_c*cg*k) = A1*cg + k*(B1 + C1*cg),
  // evaluated mod 2^32 and then reduced mod N (N divides 2^32).  A thread's
  // outputs of one butterfly are k = b + r*NSL, so the twiddle is carried by
  // complex multiplication with W^(NSL*de) and re-read from the table every
  // kAnchor outputs (bounded rounding growth, few scattered lookups).
  constexpr int kAnchor = 8;
  const uint32_t nmask = (uint32_t)a.nmask;
  const uint32_t od = qmod(o1, a.d_modo, a.lg_modo);  // the input digit this twiddle multiplies
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
  if constexpr (KIND == 0 || KIND == 2) {
    const uint32_t cgt = (uint32_t)(cg + a.tw_coff);
    const uint32_t de = B1 + C1 * cgt;
    const uint32_t ea = A1 * cgt;
    float2 w = make_float2(1.f, 0.f), d = w;
    if (tw) d = look((uint32_t)NSL * de);
    const bool scaled = sc != 1.f;
    auto twid = [&](int k, int r, float x, float y) {
      float2 v = make_float2(x, y);
      if (tw) {  // the scale rides on the anchored twiddle
        if (r % kAnchor == 0) {
          w = look(ea + (uint32_t)k * de);
          w.x *= sc;
          w.y *= sc;
        } else {
          w = cmul(w, d);
        }
        v = cmul(v, w);
      } else if (scaled) {
        v.x *= sc;
        v.y *= sc;
      }
      return v;
    };
    if constexpr (KIND == 0) {
      float* __restrict__ qr = a.yr + obase + cg;
      float* __restrict__ qi = a.yi + obase + cg;
      const OFF os = (OFF)a.os_k;
      pass_compute_store_r<LOGL, GM::LE, PL, INV>(j, vr, vi, [&](int k, int r, float x, float y) {
        const float2 v = twid(k, r, x, y);
        if (colok) {
          qr[(OFF)k * os] = v.x;
          qi[(OFF)k * os] = v.y;
        }
      });
    } else {
      // each output goes to its owner rank's row buffer (peer memory over
      // NVLink for the other ranks): K = o1*ka + k*kb, rank K >> rows_log
      const OFF kbase = (OFF)o1 * (OFF)a.sc_ka;
      const OFF rmask = ((OFF)1 << a.sc_rows_log) - 1;
      const OFF ccol = (OFF)(a.sc_col0 + cg);
      const OFF kb = (OFF)a.sc_kb, ld = (OFF)a.sc_ld;
      pass_compute_store_r<LOGL, GM::LE, PL, INV>(j, vr, vi, [&](int k, int r, float x, float y) {
        const float2 v = twid(k, r, x, y);
        const OFF K = kbase + (OFF)k * kb;
        const int q = (int)(K >> a.sc_rows_log);
        const OFF off = (K & rmask) * ld + ccol;
        if (colok && q < a.sc_npeers) {
          s_re[q][off] = v.x;
          s_im[q][off] = v.y;
        }
      });
    }
  } else {
    // row-wise (transposing) store: the last pass goes to shared memory, then
    // consecutive threads take consecutive k of one column
    if constexpr (PL > 0) __syncthreads();
    pass_compute_store<LOGL, GM::LE, PL, INV>(j, vr, vi, [&](int i, float x, float y) { col[i * SP] = make_float2(x, y); });
    __syncthreads();
    float* __restrict__ qr0 = a.yr + obase + c0 * a.os_c;
    float* __restrict__ qi0 = a.yi + obase + c0 * a.os_c;
    static_assert(THREADS % L == 0, "row-wise store mapping");
    constexpr int CPI = THREADS / L;  // columns per iteration; k fixed per thread
    const int k = tid % L;
    const int cst = tid / L;
    const uint32_t mstep = (uint32_t)CPI * (A1 + C1 * (uint32_t)k);
    float2 w = make_float2(1.f, 0.f), m = w;
    if (tw) m = look(mstep);
#pragma unroll
    for (int i = 0; i < CT / CPI; ++i) {
      const int c = i * CPI + cst;
      const long long cgc = c0 + c;
      float2 v = sm2[k * SP + c];
      if (tw) {
        const uint32_t cgt = (uint32_t)cgc + (uint32_t)a.tw_coff;
        w = (i % kAnchor == 0) ? look(A1 * cgt + (uint32_t)k * (B1 + C1 * cgt)) : cmul(w, m);
        v = cmul(v, w);
      }
      if (cgc < a.ncols) {
        const OFF off = (OFF)c * (OFF)a.os_c + k;
        qr0[off] = v.x * sc;
        qi0[off] = v.y * sc;
      }
    }
  }
}

// One tile per iteration; the grid is the tile count unless ColArgs.max_blocks
// caps it (the scatter pass then leaves SMs to a concurrent kernel).
template <int LOGL, bool INV, int KIND, class OFF>
__global__ void __launch_bounds__(ColGeom<LOGL>::THREADS, ColGeom<LOGL>::MINB) k_col(ColArgs a) {
  __shared__ float* s_ptr[16];  // kind 2: the peers' row buffers, re then im
  if constexpr (KIND == 2) {
    if (threadIdx.x < (unsigned)a.sc_npeers) {
      s_ptr[threadIdx.x] = a.sc_re[threadIdx.x];
      s_ptr[8 + threadIdx.x] = a.sc_im[threadIdx.x];
    }
    __syncthreads();
  }
  for (uint32_t tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x) {
    col_tile<LOGL, INV, KIND, OFF>(a, tile, s_ptr, s_ptr + 8);
    if (tile + gridDim.x < a.ntiles) __syncthreads();  // the tile's shared memory is free again
  }
  if constexpr (KIND == 2) __threadfence_system();
}

static int ilog2_exact(long long v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int l = 0;
  while ((1LL << l) < v) ++l;
  return l;
}

// largest element offset a tile touches relative to its base pointers
template <int LOGL>
static bool offsets_fit_31(const ColArgs& a, int kind) {
  using GM = ColGeom<LOGL>;
  const long long lim = 1LL << 31;
  const long long L = GM::L, CT = GM::CT;
  if ((L - 1) * a.is_j + CT >= lim) return false;
  if (kind == 0 && (L - 1) * a.os_k + CT >= lim) return false;
  if (kind == 1 && (CT - 1) * a.os_c + L >= lim) return false;
  if (kind == 2) {
    const long long kmax = (a.O1 - 1) * a.sc_ka + (L - 1) * a.sc_kb;
    if (kmax >= lim || (1LL << a.sc_rows_log) * a.sc_ld >= lim || a.sc_col0 + a.ncols >= lim) return false;
  }
  return true;
}

template <int LOGL, bool INV, int KIND, class OFF>
static cudaError_t launch_col_o(const ColArgs& a, cudaStream_t st) {
  using GM = ColGeom<LOGL>;
  auto kern = k_col<LOGL, INV, KIND, OFF>;
  constexpr size_t smem = GM::smem_bytes(KIND);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e0 = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e0 != cudaSuccess) return e0;
  const long long ncb = (a.ncols + GM::CT - 1) / GM::CT;
  const long long tiles = ncb * a.O1 * a.O2 * a.O3;
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  ColArgs b = a;
  b.d_ncb = (uint32_t)ncb;
  b.lg_ncb = ilog2_exact(ncb);
  b.d_O1 = (uint32_t)a.O1;
  b.lg_O1 = ilog2_exact(a.O1);
  b.d_O2 = (uint32_t)a.O2;
  b.lg_O2 = ilog2_exact(a.O2);
  // o1 mod tw_modo: the identity when tw_modo >= O1
  if (a.tw_modo >= a.O1) {
    b.d_modo = 0;
    b.lg_modo = 31;
  } else {
    b.d_modo = (uint32_t)a.tw_modo;
    b.lg_modo = ilog2_exact(a.tw_modo);
  }
  b.ntiles = (uint32_t)tiles;
  long long grid = tiles;
  if (a.max_blocks > 0 && a.max_blocks < grid) grid = a.max_blocks;
  kern<<<(unsigned)grid, GM::THREADS, smem, st>>>(b);
  return cudaGetLastError();
}

template <int LOGL, bool INV, int KIND>
static cudaError_t launch_col_t(const ColArgs& a, cudaStream_t st) {
  if (offsets_fit_31<LOGL>(a, KIND)) return launch_col_o<LOGL, INV, KIND, int>(a, st);
  return launch_col_o<LOGL, INV, KIND, long long>(a, st);
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
