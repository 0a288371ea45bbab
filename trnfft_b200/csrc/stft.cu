// Fused short-time Fourier transform for power-of-two n_fft (4 .. 8192).
//
// Reference: trnfft/api.py:291-365 pads the signal (F.pad, reflect by
// default), gathers every frame into a (..., frames, n_fft) tensor, multiplies
// by the window, runs a full complex FFT of each real frame, slices the
// one-sided bins and transposes to (..., freq, time) -- five HBM round trips
// of a tensor twice the signal's size.  Here one kernel reads each frame's
// samples straight from the waveform (interior frames as aligned float2 pairs;
// frames that reach into the padding map their indices by pad_mode), applies
// the window, transforms the real frame as an n_fft/2-point complex FFT of
// z[n] = x[2n] + i x[2n+1] plus an on-chip split, and writes the bins in the
// (freq, time) layout: a block owns G consecutive frames of one waveform, so
// each frequency row receives G contiguous floats per store.
#include <cstdlib>

#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGM, int TB = 128>
struct StftGeom {
  static constexpr int LE = 4;
  using S = Sched<LOGM, LE>;
  static constexpr int G0 = TB / S::T;
  static constexpr int G = G0 < 1 ? 1 : G0;  // frames per block
  static constexpr int THREADS = G * S::T;
  static constexpr int MINB = THREADS >= 1024 ? 1 : 1024 / THREADS;
  // frame pitch = 2 (mod 16) float2: in the split read-out a half-warp covers 8 frames x 2
  // neighbouring bins, which then fall on 16 distinct bank pairs
  static constexpr int FP = S::NP + ((2 - S::NP % 16) + 16) % 16;
  static constexpr size_t smem = (size_t)G * FP * sizeof(float2);
};

__device__ __forceinline__ long long stft_src(long long i, long long L, int mode) {
  // map an index of the padded signal (already shifted by -pad) into [0, L); -1 = zero
  if (i >= 0 && i < L) return i;
  switch (mode) {
    case 0:  // reflect (edge sample not repeated)
      if (i < 0) i = -i;
      if (i >= L) i = 2 * (L - 1) - i;
      return i;
    case 1:  // constant (zeros)
      return -1;
    case 2:  // replicate
      return i < 0 ? 0 : L - 1;
    default: {  // circular
      long long r = i % L;
      return r < 0 ? r + L : r;
    }
  }
}

template <int LOGM, int TB>
__global__ void __launch_bounds__(StftGeom<LOGM, TB>::THREADS, StftGeom<LOGM, TB>::MINB) k_stft(StftArgs a) {
  using GM = StftGeom<LOGM, TB>;
  using S = typename GM::S;
  constexpr int M = S::N;
  constexpr int N = 2 * M;
  constexpr int LOGN = LOGM + 1;
  extern __shared__ float2 sm2[];
  const int g = threadIdx.x / S::T;
  const int j = threadIdx.x % S::T;
  // block -> (waveform, frame group) in 32-bit arithmetic (blocks < 2^31)
  const uint32_t nfb = (uint32_t)((a.frames + GM::G - 1) / GM::G);
  const long long b = blockIdx.x / nfb;
  const long long f0 = (long long)(blockIdx.x % nfb) * GM::G;
  const long long f = f0 + g;
  const bool valid = f < a.frames;
  const float* __restrict__ x = a.x + b * a.len;
  const float* __restrict__ w = a.window;
  float2* sb = sm2 + g * GM::FP;
  const long long base = f * a.hop - a.pad;

  float vr[S::E], vi[S::E];
  // interior frames (no padding involved) with an even start read sample pairs as float2
  const bool fast = valid && base >= 0 && base + N <= a.len && ((((uintptr_t)(x + base)) | (uintptr_t)w) & 7) == 0;
  if (__syncthreads_and(fast || !valid)) {
    const float2* x2 = reinterpret_cast<const float2*>(x + (valid ? base : 0));
    const float2* w2 = reinterpret_cast<const float2*>(w);
    pass_load<LOGM, GM::LE, 0>(j, vr, vi, [&](int n, float& r, float& m) {
      if (valid) {
        const float2 v = __ldg(x2 + n);
        const float2 ww = __ldg(w2 + n);
        r = v.x * ww.x;
        m = v.y * ww.y;
      } else {
        r = 0.f;
        m = 0.f;
      }
    });
  } else {
    pass_load<LOGM, GM::LE, 0>(j, vr, vi, [&](int n, float& r, float& m) {
      r = 0.f;
      m = 0.f;
      if (!valid) return;
      const long long s0 = stft_src(base + 2 * n, a.len, a.pad_mode);
      const long long s1 = stft_src(base + 2 * n + 1, a.len, a.pad_mode);
      if (s0 >= 0) r = __ldg(x + s0) * __ldg(w + 2 * n);
      if (s1 >= 0) m = __ldg(x + s1) * __ldg(w + 2 * n + 1);
    });
  }
  pass_compute_store<LOGM, GM::LE, 0, false>(j, vr, vi, [&](int i, float r, float m) {
    sb[spad<S::SH>(i)] = make_float2(r, m);
  });
  __syncthreads();
  smem_passes<LOGM, GM::LE, false, 1, S::P>(j, sb);

  // split + store: X_k = E_k + W_N^k O_k; lanes run over the block's frames
  const int nbins = a.onesided ? M + 1 : N;
  const long long F = a.frames;
  float* __restrict__ yr = a.yr + b * (long long)nbins * F;
  float* __restrict__ yi = a.yi + b * (long long)nbins * F;
  if (a.onesided) {
    // bins k and M-k from one pair of loads: with T = W_N^k O_k, X_k = E_k + T and
    // X_{M-k} = conj(E_k - T) (W_N^{M-k} = -conj(W_N^k), E_{M-k} = conj(E_k), O_{M-k} = conj(O_k))
    for (int idx = threadIdx.x; idx < (M / 2 + 1) * GM::G; idx += GM::THREADS) {
      const int gg = idx % GM::G;
      const int k = idx / GM::G;
      const long long ff = f0 + gg;
      if (ff >= F) continue;
      const float2* fb = sm2 + gg * GM::FP;
      const float2 z = fb[spad<S::SH>(k & (M - 1))];
      const float2 v = fb[spad<S::SH>((M - k) & (M - 1))];
      const float er = 0.5f * (z.x + v.x), ei = 0.5f * (z.y - v.y);
      const float orr = 0.5f * (z.y + v.y), oi = 0.5f * (v.x - z.x);
      const float2 tw = tw_lookup(k << (kTwLog - LOGN));
      const float tr = orr * tw.x - oi * tw.y;
      const float ti = orr * tw.y + oi * tw.x;
      yr[(long long)k * F + ff] = (er + tr) * a.scale;
      yi[(long long)k * F + ff] = (ei + ti) * a.scale;
      if (2 * k != M) {
        yr[(long long)(M - k) * F + ff] = (er - tr) * a.scale;
        yi[(long long)(M - k) * F + ff] = (ti - ei) * a.scale;
      }
    }
    return;
  }
  for (int idx = threadIdx.x; idx < nbins * GM::G; idx += GM::THREADS) {
    const int gg = idx % GM::G;
    const int k = idx / GM::G;
    const long long ff = f0 + gg;
    if (ff >= F) continue;
    const bool mirror = k > M;
    const int kk = mirror ? N - k : k;
    const float2* fb = sm2 + gg * GM::FP;
    const float2 z = fb[spad<S::SH>(kk & (M - 1))];
    const float2 v = fb[spad<S::SH>((M - kk) & (M - 1))];
    const float er = 0.5f * (z.x + v.x), ei = 0.5f * (z.y - v.y);
    const float orr = 0.5f * (z.y + v.y), oi = 0.5f * (v.x - z.x);
    const float2 tw = tw_lookup(kk << (kTwLog - LOGN));
    float xr = er + (orr * tw.x - oi * tw.y);
    float xi = ei + (orr * tw.y + oi * tw.x);
    if (mirror) xi = -xi;
    yr[(long long)k * F + ff] = xr * a.scale;
    yi[(long long)k * F + ff] = xi * a.scale;
  }
}

// TRNFFT_B200_STFT_THREADS (128, 256 or 512) sets the frames per block (threads / (n_fft/32)),
// for measurement; 128 by default.
static int stft_block_threads() {
  static const int v = [] {
    const char* e = getenv("TRNFFT_B200_STFT_THREADS");
    const int t = e ? atoi(e) : 128;
    return (t == 256 || t == 512) ? t : 128;
  }();
  return v;
}

template <int LOGM, int TB>
static cudaError_t launch_stft_tb(const StftArgs& a, cudaStream_t st) {
  using GM = StftGeom<LOGM, TB>;
  auto kern = k_stft<LOGM, TB>;
  if (GM::smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GM::smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = a.batch * ((a.frames + GM::G - 1) / GM::G);
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, GM::THREADS, GM::smem, st>>>(a);
  return cudaGetLastError();
}

template <int LOGM>
static cudaError_t launch_stft_t(const StftArgs& a, cudaStream_t st) {
  switch (stft_block_threads()) {
    case 256: return launch_stft_tb<LOGM, 256>(a, st);
    case 512: return launch_stft_tb<LOGM, 512>(a, st);
    default: return launch_stft_tb<LOGM, 128>(a, st);
  }
}

cudaError_t launch_stft(int logn, const StftArgs& a, cudaStream_t st) {
  switch (logn - 1) {
    case 1: return launch_stft_t<1>(a, st);
    case 2: return launch_stft_t<2>(a, st);
    case 3: return launch_stft_t<3>(a, st);
    case 4: return launch_stft_t<4>(a, st);
    case 5: return launch_stft_t<5>(a, st);
    case 6: return launch_stft_t<6>(a, st);
    case 7: return launch_stft_t<7>(a, st);
    case 8: return launch_stft_t<8>(a, st);
    case 9: return launch_stft_t<9>(a, st);
    case 10: return launch_stft_t<10>(a, st);
    case 11: return launch_stft_t<11>(a, st);
    case 12: return launch_stft_t<12>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tfb
