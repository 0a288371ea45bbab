// Bluestein (chirp-z) for lengths whose padded length m exceeds what one
// block holds on chip (m > 16384): the same algorithm as bluestein.cu
// (trnfft/fft_core.py:1285-1376) split into passes over a caller-provided
// work area, with the m-point transforms done by the multi-pass kernels.
//   pre : A[i] = x[i] * chirp_i (i < n), 0 (n <= i < m)
//   FFT : B = FFT_m(A)
//   mul : B *= H   (H = FFT_m(h), h = conj(chirp) with circular wrap; the
//                   inverse transform uses conj(H[(m-k) mod m]))
//   IFFT: A = IFFT_m(B)   (scaled by 1/m)
//   post: y[k] = A[k] * chirp_k (* 1/n for the inverse), k < n
// Every kernel is a grid-stride elementwise pass (HBM bound).
#include "kernels.h"

namespace tfb {

__global__ void k_blue_pre(const float* __restrict__ xr, const float* __restrict__ xi, const float2* __restrict__ chirp,
                           float* __restrict__ ar, float* __restrict__ ai, long long batch, long long n, long long m,
                           int inverse) {
  const long long total = batch * m;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long b = t / m, i = t - b * m;
    float r = 0.f, q = 0.f;
    if (i < n) {
      const float2 c = __ldg(chirp + i);
      const float ci = inverse ? -c.y : c.y;
      const float x0 = __ldg(xr + b * n + i), x1 = __ldg(xi + b * n + i);
      r = fmaf(x0, c.x, -x1 * ci);
      q = fmaf(x0, ci, x1 * c.x);
    }
    ar[t] = r;
    ai[t] = q;
  }
}

__global__ void k_blue_mul(float* __restrict__ br, float* __restrict__ bi, const float* __restrict__ hr,
                           const float* __restrict__ hi, long long batch, long long m, int inverse) {
  const long long total = batch * m;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long k = t % m;
    float h0, h1;
    if (inverse) {
      const long long km = (m - k) & (m - 1);
      h0 = __ldg(hr + km);
      h1 = -__ldg(hi + km);
    } else {
      h0 = __ldg(hr + k);
      h1 = __ldg(hi + k);
    }
    const float v0 = br[t], v1 = bi[t];
    br[t] = fmaf(v0, h0, -v1 * h1);
    bi[t] = fmaf(v0, h1, v1 * h0);
  }
}

__global__ void k_blue_post(const float* __restrict__ ar, const float* __restrict__ ai, const float2* __restrict__ chirp,
                            float* __restrict__ yr, float* __restrict__ yi, long long batch, long long n, long long m,
                            int inverse, float scale) {
  const long long total = batch * n;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    const long long b = t / n, k = t - b * n;
    const float2 c = __ldg(chirp + k);
    const float ci = inverse ? -c.y : c.y;
    const float v0 = __ldg(ar + b * m + k), v1 = __ldg(ai + b * m + k);
    yr[t] = fmaf(v0, c.x, -v1 * ci) * scale;
    yi[t] = fmaf(v0, ci, v1 * c.x) * scale;
  }
}

static unsigned grid_for(long long total) {
  long long g = (total + 255) / 256;
  if (g > 148LL * 32) g = 148LL * 32;
  return (unsigned)(g < 1 ? 1 : g);
}

cudaError_t launch_blue_pre(const float* xr, const float* xi, const float2* chirp, float* ar, float* ai,
                            long long batch, long long n, long long m, bool inv, cudaStream_t st) {
  k_blue_pre<<<grid_for(batch * m), 256, 0, st>>>(xr, xi, chirp, ar, ai, batch, n, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_blue_mul(float* br, float* bi, const float* hr, const float* hi, long long batch, long long m,
                            bool inv, cudaStream_t st) {
  k_blue_mul<<<grid_for(batch * m), 256, 0, st>>>(br, bi, hr, hi, batch, m, inv ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_blue_post(const float* ar, const float* ai, const float2* chirp, float* yr, float* yi,
                             long long batch, long long n, long long m, bool inv, float scale, cudaStream_t st) {
  k_blue_post<<<grid_for(batch * n), 256, 0, st>>>(ar, ai, chirp, yr, yi, batch, n, m, inv ? 1 : 0, scale);
  return cudaGetLastError();
}

}  // namespace tfb
