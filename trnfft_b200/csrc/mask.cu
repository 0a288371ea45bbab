// Fused complex mask application y = mask * spec on planar float32 operands.
//
// Reference: trnfft/nki/dispatch.py:105-113 (complex_mask_apply) and its NKI
// kernel dispatch.py:347-417 compute (a_re b_re - a_im b_im) + i (a_re b_im +
// a_im b_re) in one pass instead of six torch element-wise ops.  Here one
// grid-stride kernel reads the four planes once and writes the two output
// planes once (24 bytes per complex element, the HBM floor).  The mask may be
// shorter than the spectrogram and repeat along the leading axes (a mask of
// shape (freq, time) applied to every signal of a (batch, freq, time)
// spectrogram): element i uses mask element i mod mcount.  Planes whose
// pointers and lengths are multiples of 4 floats move as float4.
#include "kernels.h"

namespace tfb {

__device__ __forceinline__ void cmul4(const float4& ar, const float4& ai, const float4& br, const float4& bi,
                                      float4& yr, float4& yi) {
  yr.x = fmaf(ar.x, br.x, -ai.x * bi.x);
  yr.y = fmaf(ar.y, br.y, -ai.y * bi.y);
  yr.z = fmaf(ar.z, br.z, -ai.z * bi.z);
  yr.w = fmaf(ar.w, br.w, -ai.w * bi.w);
  yi.x = fmaf(ar.x, bi.x, ai.x * br.x);
  yi.y = fmaf(ar.y, bi.y, ai.y * br.y);
  yi.z = fmaf(ar.z, bi.z, ai.z * br.z);
  yi.w = fmaf(ar.w, bi.w, ai.w * br.w);
}

// count4 / mcount4 in float4 units; mask index advances with the grid stride
__global__ void __launch_bounds__(256) k_cmul_v4(const float4* __restrict__ mr, const float4* __restrict__ mi,
                                                 long long mcount4, const float4* __restrict__ sr,
                                                 const float4* __restrict__ si, float4* __restrict__ yr,
                                                 float4* __restrict__ yi, long long count4) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long m = i % mcount4;
  const long long step = stride % mcount4;
  for (; i < count4; i += stride) {
    float4 a, b;
    cmul4(__ldg(mr + m), __ldg(mi + m), __ldcs(sr + i), __ldcs(si + i), a, b);
    __stcs(yr + i, a);
    __stcs(yi + i, b);
    m += step;
    if (m >= mcount4) m -= mcount4;
  }
}

__global__ void __launch_bounds__(256) k_cmul_scalar(const float* __restrict__ mr, const float* __restrict__ mi,
                                                     long long mcount, const float* __restrict__ sr,
                                                     const float* __restrict__ si, float* __restrict__ yr,
                                                     float* __restrict__ yi, long long count) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long m = i % mcount;
  const long long step = stride % mcount;
  for (; i < count; i += stride) {
    const float ar = __ldg(mr + m), ai = __ldg(mi + m), br = __ldg(sr + i), bi = __ldg(si + i);
    yr[i] = fmaf(ar, br, -ai * bi);
    yi[i] = fmaf(ar, bi, ai * br);
    m += step;
    if (m >= mcount) m -= mcount;
  }
}

cudaError_t launch_cmul(const float* mr, const float* mi, long long mcount, const float* sr, const float* si,
                        float* yr, float* yi, long long count, cudaStream_t st) {
  if (count <= 0) return cudaSuccess;
  if (mcount <= 0) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uintptr_t al = reinterpret_cast<uintptr_t>(mr) | reinterpret_cast<uintptr_t>(mi) |
                       reinterpret_cast<uintptr_t>(sr) | reinterpret_cast<uintptr_t>(si) |
                       reinterpret_cast<uintptr_t>(yr) | reinterpret_cast<uintptr_t>(yi);
  const bool v4 = (al & 15) == 0 && (count & 3) == 0 && (mcount & 3) == 0;
  const long long units = v4 ? count / 4 : count;
  // persistent grid: 8 blocks of 256 threads per SM (enough loads in flight for HBM)
  long long blocks = (units + 255) / 256;
  const long long cap = 8LL * sms;
  if (blocks > cap) blocks = cap;
  if (v4) {
    k_cmul_v4<<<(unsigned)blocks, 256, 0, st>>>(
        reinterpret_cast<const float4*>(mr), reinterpret_cast<const float4*>(mi), mcount / 4,
        reinterpret_cast<const float4*>(sr), reinterpret_cast<const float4*>(si), reinterpret_cast<float4*>(yr),
        reinterpret_cast<float4*>(yi), units);
  } else {
    k_cmul_scalar<<<(unsigned)blocks, 256, 0, st>>>(mr, mi, mcount, sr, si, yr, yi, count);
  }
  return cudaGetLastError();
}

}  // namespace tfb
