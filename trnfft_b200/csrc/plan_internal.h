// Definition of the opaque plan object behind trnfft_plan_t (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/trnfft_b200.h"

struct trnfft_plan_s {
  int64_t n = 0;
  int device = 0;
  int algorithm = TRNFFT_ALG_COPY;
  int logn = -1;
  int64_t m = 0;  // Bluestein padded length
  int logm = -1;
  float2* chirp = nullptr;  // Bluestein: n entries
  float2* H = nullptr;      // Bluestein: m entries
  float2* tw_hi = nullptr;  // power of two n > 1024: W_n^(i << tw_split)
  float2* tw_lo = nullptr;  // power of two n > 1024: W_n^i, i < 2^tw_split
  int tw_split = 0;
  // Bluestein with m > 16384 (multi-pass): m-point sub-plan and H = FFT_m(h), planar
  struct trnfft_plan_s* sub = nullptr;
  float* Hr = nullptr;
  float* Hi = nullptr;
  // mixed radix (TRNFFT_ALG_MIXED): pass radices and W_n^i, i < n
  int npass = 0;
  int radix[16] = {0};
  unsigned long long codes = 0;  // 3 bits per pass, see MixedArgs
  float2* twn = nullptr;
  // double precision (trnfft_plan_enable_f64): power of two n > 4096: two-level
  // table of W_n; Bluestein: chirp and H = FFT_m(h)/m in double, and an m-point
  // sub-plan (also fp64-enabled) for the padded transforms
  bool f64 = false;
  double2* tw64_hi = nullptr;
  double2* tw64_lo = nullptr;
  int tw64_split = 0;
  double2* chirp64 = nullptr;
  double2* H64 = nullptr;
  struct trnfft_plan_s* sub64 = nullptr;
};
