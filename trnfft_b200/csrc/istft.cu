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
// Here one kernel does all of it.  A block owns the samples of P consecutive
// frame starts of one signal (a segment of P * hop samples) and transforms
// the P + H frames that touch it (H = ceil(n_fft / hop) - 1 earlier frames
// reach into the segment), in chunks of G frames: it stages the chunk's
// spectrum columns ([bins][G]; the G frames are contiguous in the (freq, time)
// layout, so every load is a run of G floats), runs G real inverse transforms
// on chip (an n_fft/2-point complex FFT of Z_k = E_k + i O_k, the packing of
// the forward real kernels), and overlap-adds: each thread owns a fixed
// residue class of the segment's samples and sums, in registers and in frame
// order like the reference's loop, the windowed value, the raw value and the
// squared window of the frames that cover each of its samples.  When P + H
// frames fit in one chunk (n_fft = 2 hop: 8 frames for 7 frame starts) the
// block normalises and writes its samples at once; otherwise the sums go into
// three segment accumulators in shared memory once per chunk.  Every output
// sample is written exactly once, without atomics.
#include <cstdlib>

#include "fft_common.cuh"
#include "kernels.h"

namespace tfb {

template <int LOGM, int TB = 128>
struct IstftGeom {
  static constexpr int LE = 4;
  using S = Sched<LOGM, LE>;
  static constexpr int G0 = TB / S::T;
  static constexpr int G = G0 < 1 ? 1 : G0;  // frames per chunk
  static constexpr int THREADS = G * S::T;  // every thread owns a slice of one frame
  static constexpr int M = S::N;
  static constexpr int FP = S::NP + ((2 - S::NP % 16) + 16) % 16;  // frame pitch (float2)
  // the spectrum tile (2 planes of (M+1) x G floats) shares its space with the frames
  // (float2): it is read into registers before the first pass writes the frames
  // tile floats per bin.  In the C2R pre-processing a warp reads bins k = j + T r of its
  // FW = 32 / T frames (lanes: FW frames x T consecutive j): a pitch of FW x (odd) puts the
  // warp's 32 loads in 32 distinct banks
  static constexpr int FW = S::T < 32 ? 32 / S::T : 1;
  static constexpr int TPO = (G + FW - 1) / FW;
  static constexpr int TP = FW * (TPO % 2 ? TPO : TPO + 1);
  static constexpr size_t tile_bytes = 2 * (size_t)(M + 1) * TP * sizeof(float);
  static constexpr size_t frame_bytes = (size_t)G * FP * sizeof(float2);
  // ... followed by the segment accumulators (3 x SEG floats), sized at launch
  static constexpr size_t fixed_smem = ((tile_bytes > frame_bytes ? tile_bytes : frame_bytes) + 15) / 16 * 16;
  // resident blocks per SM: up to 8, and 1024 threads' worth in all (64 registers per thread)
  static constexpr int MINB = THREADS >= 1024 ? 1 : (1024 / THREADS < 8 ? 1024 / THREADS : 8);
};

// 4-byte asynchronous global -> shared copy; src_bytes = 0 fills zero
__device__ __forceinline__ void cp_async4(float* smem, const float* gmem, int src_bytes) {
  const unsigned sa = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

template <int LOGM, int TB>
__global__ void __launch_bounds__(IstftGeom<LOGM, TB>::THREADS, IstftGeom<LOGM, TB>::MINB) k_istft(IstftArgs a) {
  using GM = IstftGeom<LOGM, TB>;
  using S = typename GM::S;
  constexpr int M = S::N;
  constexpr int N = 2 * M;
  constexpr int LOGN = LOGM + 1;
  constexpr int G = GM::G;
  extern __shared__ float2 sm2[];
  float2* frames = sm2;
  float* tre = reinterpret_cast<float*>(sm2);  // aliases the frames (see IstftGeom)
  float* tim = tre + (M + 1) * GM::TP;
  float* acc_w = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(sm2) + GM::fixed_smem);
  float* acc_r = acc_w + a.seg;      // unwindowed overlap-add
  float* acc_e = acc_r + a.seg;      // envelope sum_f w[t - f hop]^2

  const long long b = blockIdx.x / a.nseg;
  // 32-bit sample indices within one signal (the host rejects signals of 2^31 samples)
  const int t0 = (int)((blockIdx.x % a.nseg) * (long long)a.seg);
  const int t1 = (int)min((long long)t0 + a.seg, a.total);
  const int tid = threadIdx.x;
  const int g = tid / S::T;
  const int j = tid % S::T;
  const int hop = (int)a.hop;
  const int F = (int)a.frames;
  const int nbins = a.onesided ? M + 1 : N;
  const float* __restrict__ xr = a.xr + b * (long long)nbins * F;
  const float* __restrict__ xi = a.xi + b * (long long)nbins * F;
  const float* __restrict__ w = a.window;

  // frames f with [f hop, f hop + N) meeting [t0, t1)
  const int flo = t0 - N + 1 <= 0 ? 0 : (t0 - N + hop) / hop;
  int fhi = (t1 - 1) / hop;
  if (fhi > F - 1) fhi = F - 1;
  if (flo > fhi) {
    // no frame reaches these samples (a requested length past the frames): zeros
    for (int t = t0 + tid; t < t1; t += GM::THREADS) {
      const long long o = (long long)t - a.pad_front;
      if (o >= 0 && o < a.out_len) a.y[b * a.out_len + o] = 0.f;
    }
    return;
  }
  // one chunk covers all the block's frames: no segment accumulators (see the overlap-add);
  // the launcher allocates them only when its geometry can give a block more than one chunk
  const bool single = fhi - flo < G;
  if (!single) {
    for (int i = tid; i < a.seg; i += GM::THREADS) {
      acc_w[i] = 0.f;
      acc_r[i] = 0.f;
      acc_e[i] = 0.f;
    }
  }

  for (int fc = flo; fc <= fhi; fc += G) {
    // stage the chunk's spectrum: tile[k][gg], k in [0, M]; the G frames of a bin are
    // contiguous in memory.  One-sided spectra go through asynchronous 4-byte copies, all in
    // flight at once (frames past the last one are zero-filled).
    if (a.onesided) {
      for (int idx = tid; idx < (M + 1) * G; idx += GM::THREADS) {
        const int gg = idx % G;
        const int k = idx / G;
        const int f = fc + gg;
        const bool in = f <= fhi;
        const long long off = in ? (long long)k * F + f : 0;
        cp_async4(tre + k * GM::TP + gg, xr + off, in ? 4 : 0);
        cp_async4(tim + k * GM::TP + gg, xi + off, in ? 4 : 0);
      }
      cp_async_wait_all();
    } else {
      for (int idx = tid; idx < (M + 1) * G; idx += GM::THREADS) {
        const int gg = idx % G;
        const int k = idx / G;
        const int f = fc + gg;
        float r = 0.f, m = 0.f;
        if (f <= fhi) {
          // real part of the full inverse transform = C2R of (X_k + conj X_{N-k}) / 2
          const int km = (N - k) & (N - 1);
          r = 0.5f * (__ldg(xr + (long long)k * F + f) + __ldg(xr + (long long)km * F + f));
          m = 0.5f * (__ldg(xi + (long long)k * F + f) - __ldg(xi + (long long)km * F + f));
        }
        tre[k * GM::TP + gg] = r;
        tim[k * GM::TP + gg] = m;
      }
    }
    __syncthreads();
    {
      float2* sb = frames + g * GM::FP;
      float vr[S::E], vi[S::E];
      // 2 Z_k = (X_k + conj X_{M-k}) + i (X_k - conj X_{M-k}) conj(W_N^k)
      pass_load<LOGM, GM::LE, 0>(j, vr, vi, [&](int k, float& r, float& m) {
        const int km = M - k;
        const float ar = tre[k * GM::TP + g], ai = (k == 0) ? 0.f : tim[k * GM::TP + g];
        const float br = tre[km * GM::TP + g], bi = (km == M) ? 0.f : tim[km * GM::TP + g];
        const float er = ar + br, ei = ai - bi;
        const float dr = ar - br, di = ai + bi;
        const float2 tw = tw_level(LOGN, k);  // W_N^k, k < M = 2^(LOGN-1)
        const float orr = dr * tw.x + di * tw.y;
        const float oi = di * tw.x - dr * tw.y;
        r = er - oi;
        m = ei + orr;
      });
      __syncthreads();  // the tile is read: the frames may overwrite it
      pass_compute_store<LOGM, GM::LE, 0, true>(j, vr, vi, [&](int i, float r, float m) {
        sb[spad<S::SH>(i)] = make_float2(r, m);
      });
    }
    __syncthreads();
    smem_passes<LOGM, GM::LE, true, 1, S::P>(j, frames + g * GM::FP);
    __syncthreads();
    // overlap-add.  Thread tid owns the samples t = t0 + tid (mod THREADS) and sums, in frame
    // order as the reference's loop does, the chunk's frames that cover t (at most
    // ceil(n_fft / hop) of them) in registers: windowed, raw and squared window.  A block whose
    // frames fit in one chunk normalises and writes its samples right away; otherwise the sums
    // go into the segment accumulators once per chunk.
    const int fe = fc + G - 1 < fhi ? fc + G - 1 : fhi;
    for (int t = t0 + tid; t < t1; t += GM::THREADS) {
      // frames f with f hop <= t < f hop + N, within [fc, fe]
      int fa = t < N ? 0 : (t - N) / hop + 1;
      int fb = t / hop;
      if (fa < fc) fa = fc;
      if (fb > fe) fb = fe;
      float sw = 0.f, sr = 0.f, se = 0.f;
      for (int f = fa; f <= fb; ++f) {
        const int off = t - f * hop;
        const float2 z = frames[(f - fc) * GM::FP + spad<S::SH>(off >> 1)];
        const float v = ((off & 1) ? z.y : z.x) * a.scale;
        const float ww = __ldg(w + off);
        sw = fmaf(v, ww, sw);
        sr += v;
        se = fmaf(ww, ww, se);
      }
      if (single) {
        const long long o = (long long)t - a.pad_front;
        if (o >= 0 && o < a.out_len) {
          float out = 0.f;
          if (t < a.exp_len) out = se > 1e-8f ? sw / se : sr;
          a.y[b * a.out_len + o] = out;
        }
      } else if (fa <= fb) {
        acc_w[t - t0] += sw;
        acc_r[t - t0] += sr;
        acc_e[t - t0] += se;
      }
    }
    __syncthreads();
  }
  if (single) return;  // written above

  // normalisation, centre trim and length
  float* __restrict__ y = a.y + b * a.out_len;
  for (int t = t0 + tid; t < t1; t += GM::THREADS) {
    const long long o = (long long)t - a.pad_front;
    if (o < 0 || o >= a.out_len) continue;
    float out = 0.f;
    if (t < a.exp_len) {
      const float env = acc_e[t - t0];
      out = env > 1e-8f ? acc_w[t - t0] / env : acc_r[t - t0];
    }
    y[o] = out;
  }
}

template <int LOGM, int TB>
static cudaError_t launch_istft_tb(IstftArgs a, cudaStream_t st) {
  using GM = IstftGeom<LOGM, TB>;
  constexpr int N = 2 * GM::M;
  // A block owns P consecutive frame starts (its segment is P * hop samples) and needs the
  // H = ceil(N / hop) - 1 frames before them: P + H = K * G frames, K whole chunks.
  const long long H = (N - 1) / a.hop;
  long long K = (H + GM::G) / GM::G;  // smallest K with K * G > H
  if (K < 1) K = 1;
  long long P = K * GM::G - H;
  long long seg = P * a.hop;
  // with one chunk (K = 1) every block's frames fit in it and the overlap-add needs no segment
  // accumulators; otherwise keep the three accumulators within 96 KB
  while (K > 1 && seg * 12 > 96 * 1024 && P > 1) {
    --P;
    seg = P * a.hop;
  }
  if (seg > (1 << 30) || (K > 1 && seg * 12 > 96 * 1024)) return cudaErrorInvalidValue;  // hop beyond 8192
  a.seg = (int)seg;
  a.nseg = (a.total + seg - 1) / seg;
  const size_t smem = GM::fixed_smem + (K > 1 ? 3 * (size_t)seg * sizeof(float) : 0);
  auto kern = k_istft<LOGM, TB>;
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

// TRNFFT_B200_ISTFT_THREADS (128, 256 or 512) sets the frames per chunk (threads / (n_fft/32)),
// for measurement; 128 by default.
static int istft_block_threads() {
  static const int v = [] {
    const char* e = getenv("TRNFFT_B200_ISTFT_THREADS");
    const int t = e ? atoi(e) : 128;
    return (t == 256 || t == 512) ? t : 128;
  }();
  return v;
}

template <int LOGM>
static cudaError_t launch_istft_t(const IstftArgs& a, cudaStream_t st) {
  switch (istft_block_threads()) {
    case 256: return launch_istft_tb<LOGM, 256>(a, st);
    case 512: return launch_istft_tb<LOGM, 512>(a, st);
    default: return launch_istft_tb<LOGM, 128>(a, st);
  }
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
