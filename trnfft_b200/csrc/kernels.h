// Internal launcher interface between the C-ABI layer (capi.cu) and the
// kernel translation units.  Not part of the public boundary.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tfb {

// Rows of a batch, row r of the input at xr/xi + r*in_stride, of the output
// at yr/yi + r*out_stride (strides in floats).
struct RowArgs {
  const float* xr;
  const float* xi;
  float* yr;
  float* yi;
  long long batch;
  long long in_stride;
  long long out_stride;
  float scale;
};

// Fused Bluestein transforms (bluestein.cu).  mode 0: C2C rows of n,
// mode 1: R2C (rows of n reals -> n/2+1 bins), mode 2: C2R (n/2+1 bins -> n reals).
struct BlueArgs {
  const float* xr;
  const float* xi;
  float* yr;
  float* yi;
  long long batch;
  int n;
  const float2* chirp;  // n entries, exp(-i*pi*(k^2 mod 2n)/n)
  const float2* H;      // m entries, FFT_m(h) / m
};

cudaError_t launch_bluestein(int logm, int mode, bool inv, const BlueArgs& a, cudaStream_t st);

cudaError_t launch_rows_c2c(int logn, bool inv, const RowArgs& a, cudaStream_t st);
bool rows_c2c_tma_ok(int logn, const RowArgs& a);
cudaError_t launch_rows_c2c_tma(int logn, bool inv, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_r2c(int logm, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_c2r(int logm, const RowArgs& a, cudaStream_t st);

}  // namespace tfb
