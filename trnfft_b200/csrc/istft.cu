// Fused inverse short-time Fourier transform (windowed overlap-add) for
// power-of-two n_fft (4 .. 8192).
//
// Reference: trnfft/api.py:368-470 rebuilds the full spectrum of every frame
// (Hermitian extension, api.py:396-409), runs a complex inverse FFT per frame,
// then loops over the frames in Python twice (api.py:438-448): once for the
// windowed sum and the squared-window envelope, once for the raw sum; samples
// whose envelope exceeds 1e-8 are divided by it, the others take the raw sum
// (api.py:450-452); finally the centre padding is cut and the result trimmed
// or zero-padded to `length` (api.py:454-468).
//
// Here one kernel does all of it.  A block owns one segment of SEG output
// samples of one signal.  It walks over the frames that touch the segment in
// chunks of G frames: it stages the chunk's spectrum columns ([bins][G], the
// G frames are contiguous in the (freq, time) layout, so every load is a run
// of G floats), runs G real inverse transforms on chip (an n_fft/2-point
// complex FFT of Z_k = E_k + i O_k, the same packing as the forward real
// kernels), and adds each frame's samples, windowed and raw, into two
// segment accumulators in shared memory.  The envelope sum_f w[t - f hop]^2 is
// evaluated per sample from the window, and every output sample is written
// exactly once.  Frames shared by two neighbouring segments are transformed by
// both blocks (a few percent extra arithmetic, no extra writes).
#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGM>
struct IstftGeom {
  static constexpr int LE = 4;
  using S = Sched<LOGM, LE>;
  static constexpr int G0 = 128 / S::T;
  static constexpr int G = G0 < 1 ? 1 : G0;  // frames per chunk
  static constexpr int THREADS = G * S::T;  // every thread owns a slice of one frame
  static constexpr int M = S::N;
  static constexpr int FP = S::NP + ((2 - S::NP % 16) + 16) % 16;  // frame pitch (float2)
  // frames (float2) + spectrum tile (2 planes of (M+1) x G floats); the segment
  // accumulators (2 x SEG floats) follow, sized at launch
  static constexpr size_t fixed_smem = (size_t)G * FP * sizeof(float2) + 2 * (size_t)(M + 1) * G * sizeof(float);
};

template <int LOGM>
__global__ void __launch_bounds__(IstftGeom<LOGM>::THREADS) k_istft(IstftArgs a) {
  using GM = IstftGeom<LOGM>;
  using S = typename GM::S;
  constexpr int M = S::N;
  constexpr int N = 2 * M;
  constexpr int LOGN = LOGM + 1;
  constexpr int G = GM::G;
  extern __shared__ float2 sm2[];
  float2* frames = sm2;
  float* tre = reinterpret_cast<float*>(sm2 + G * GM::FP);
  float* tim = tre + (M + 1) * G;
  float* acc_w = tim + (M + 1) * G;
  float* acc_r = acc_w + a.seg;

  const long long b = blockIdx.x / a.nseg;
  const long long t0 = (long long)(blockIdx.x % a.nseg) * a.seg;
  const long long t1 = min(t0 + a.seg, a.total);
  const int tid = threadIdx.x;
  const int g = tid / S::T;
  const int j = tid % S::T;
  const long long hop = a.hop;
  const long long F = a.frames;
  const int nbins = a.onesided ? M + 1 : N;
  const float* __restrict__ xr = a.xr + b * (long long)nbins * F;
  const float* __restrict__ xi = a.xi + b * (long long)nbins * F;
  const float* __restrict__ w = a.window;

  for (int i = tid; i < a.seg; i += GM::THREADS) {
    acc_w[i] = 0.f;
    acc_r[i] = 0.f;
  }
  // frames f with [f hop, f hop + N) meeting [t0, t1)
  long long flo = t0 - N + 1 <= 0 ? 0 : (t0 - N + 1 + hop - 1) / hop;
  long long fhi = (t1 - 1) / hop;
  if (fhi > F - 1) fhi = F - 1;

  for (long long fc = flo; fc <= fhi; fc += G) {
    // stage the chunk's spectrum: tile[k][gg], k in [0, M]
    for (int idx = tid; idx < (M + 1) * G; idx += GM::THREADS) {
      const int gg = idx % G;
      const int k = idx / G;
      const long long f = fc + gg;
      float r = 0.f, m = 0.f;
      if (f <= fhi) {
        r = __ldg(xr + (long long)k * F + f);
        m = __ldg(xi + (long long)k * F + f);
        if (!a.onesided) {
          // real part of the full inverse transform = C2R of (X_k + conj X_{N-k}) / 2
          const int km = (N - k) & (N - 1);
          r = 0.5f * (r + __ldg(xr + (long long)km * F + f));
          m = 0.5f * (m - __ldg(xi + (long long)km * F + f));
        }
      }
      tre[idx] = r;
      tim[idx] = m;
    }
    __syncthreads();
    {
      float2* sb = frames + g * GM::FP;
      float vr[S::E], vi[S::E];
      // 2 Z_k = (X_k + conj X_{M-k}) + i (X_k - conj X_{M-k}) conj(W_N^k)
      pass_load<LOGM, GM::LE, 0>(j, vr, vi, [&](int k, float& r, float& m) {
        const int km = M - k;
        const float ar = tre[k * G + g], ai = (k == 0) ? 0.f : tim[k * G + g];
        const float br = tre[km * G + g], bi = (km == M) ? 0.f : tim[km * G + g];
        const float er = ar + br, ei = ai - bi;
        const float dr = ar - br, di = ai + bi;
        const float2 tw = tw_lookup(k << (kTwLog - LOGN));
        const float orr = dr * tw.x + di * tw.y;
        const float oi = di * tw.x - dr * tw.y;
        r = er - oi;
        m = ei + orr;
      });
      pass_compute_store<LOGM, GM::LE, 0, true>(j, vr, vi, [&](int i, float r, float m) {
        sb[spad<S::SH>(i)] = make_float2(r, m);
      });
    }
    __syncthreads();
    smem_passes<LOGM, GM::LE, true, 1, S::P>(j, frames + g * GM::FP);
    // overlap-add of the chunk into the segment
    const long long fend = min(fc + G - 1, fhi);
    for (long long t = t0 + tid; t < t1; t += GM::THREADS) {
      float sw = 0.f, sr = 0.f;
      for (long long f = fc; f <= fend; ++f) {
        const long long off = t - f * hop;
        if (off < 0 || off >= N) continue;
        const float2 z = frames[(int)(f - fc) * GM::FP + spad<S::SH>((int)(off >> 1))];
        const float v = ((off & 1) ? z.y : z.x) * a.scale;
        sw = fmaf(v, __ldg(w + off), sw);
        sr += v;
      }
      acc_w[t - t0] += sw;
      acc_r[t - t0] += sr;
    }
    __syncthreads();
  }

  // envelope, normalisation, centre trim and length
  float* __restrict__ y = a.y + b * a.out_len;
  for (long long t = t0 + tid; t < t1; t += GM::THREADS) {
    const long long o = t - a.pad_front;
    if (o < 0 || o >= a.out_len) continue;
    float out = 0.f;
    if (t < a.exp_len) {
      long long f0 = t - N + 1 <= 0 ? 0 : (t - N + 1 + hop - 1) / hop;
      long long f1 = t / hop;
      if (f1 > F - 1) f1 = F - 1;
      float env = 0.f;
      for (long long f = f0; f <= f1; ++f) {
        const float ww = __ldg(w + (t - f * hop));
        env = fmaf(ww, ww, env);
      }
      out = env > 1e-8f ? acc_w[t - t0] / env : acc_r[t - t0];
    }
    y[o] = out;
  }
}

template <int LOGM>
static cudaError_t launch_istft_t(IstftArgs a, cudaStream_t st) {
  using GM = IstftGeom<LOGM>;
  // segment: up to 4 chunks of G frames' worth of hops, about 4096 samples
  long long seg = (long long)GM::G * a.hop;
  long long cps = seg > 0 ? 4096 / seg : 1;
  if (cps < 1) cps = 1;
  if (cps > 4) cps = 4;
  seg *= cps;
  if (seg > 16384) seg = 16384;
  if (seg < 1) seg = 1;
  a.seg = (int)seg;
  a.nseg = (a.total + seg - 1) / seg;
  const size_t smem = GM::fixed_smem + 2 * (size_t)seg * sizeof(float);
  auto kern = k_istft<LOGM>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long blocks = a.batch * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  kern<<<(unsigned)blocks, GM::THREADS, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_istft(int logn, const IstftArgs& a, cudaStream_t st) {
  switch (logn - 1) {
    case 1: return launch_istft_t<1>(a, st);
    case 2: return launch_istft_t<2>(a, st);
    case 3: return launch_istft_t<3>(a, st);
    case 4: return launch_istft_t<4>(a, st);
    case 5: return launch_istft_t<5>(a, st);
    case 6: return launch_istft_t<6>(a, st);
    case 7: return launch_istft_t<7>(a, st);
    case 8: return launch_istft_t<8>(a, st);
    case 9: return launch_istft_t<9>(a, st);
    case 10: return launch_istft_t<10>(a, st);
    case 11: return launch_istft_t<11>(a, st);
    case 12: return launch_istft_t<12>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tfb
