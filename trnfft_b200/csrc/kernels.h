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

cudaError_t launch_rows_c2c(int logn, bool inv, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_r2c(int logm, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_c2r(int logm, const RowArgs& a, cudaStream_t st);

}  // namespace tfb
