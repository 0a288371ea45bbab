// Internal launcher interface between the C-ABI layer (capi.cu) and the
// kernel translation units.  Not part of the public boundary.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tfb {

int record_failure(int code, const char* msg);

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

// Direct mixed-radix transforms of 7-smooth n <= 8192 (mixed.cu); modes as
// BlueArgs.  Pass p's radix has code (codes >> 3p) & 7 (0..6 = 2, 3, 4, 5, 7,
// 8, 16); tw holds, pass after pass, W_{ns R}^{k r} at k*(R-1) + r-1 for
// k < ns (ns = product of the earlier radices), 1 <= r < R.
struct MixedArgs {
  const float* xr;
  const float* xi;
  float* yr;
  float* yi;
  long long batch;
  int n;
  int npass;
  unsigned long long codes;
  const float2* tw;
  float scale;
  int pitch;  // set by the launcher
};

cudaError_t launch_mixed(int mode, bool inv, const MixedArgs& a, cudaStream_t st);

// Column-tile FFT pass (colpass.cu).  Tile = CT neighbouring columns
// c in [c0, c0+CT) of L-point transforms, for outer block (o1, o2, o3).
// Point j of column c is read at
//   x + o1*is_o1 + o2*is_o2 + o3*is_o3 + c + j*is_j
// and output k goes to
//   kind 0: y + o1*os_o1 + o2*os_o2 + o3*os_o3 + c + k*os_k
//   kind 1: y + o1*os_o1 + o2*os_o2 + o3*os_o3 + c*os_c + k
// after multiplication by W_N^e,
//   e = tw_mul*((o1 mod tw_modo)*(tw_a*c' + tw_b*k) + tw_c*c'*k)  (mod N),
// c' = c + tw_coff,
// with W_N^e = tw_hi[e >> tw_split] * tw_lo[e & (2^tw_split - 1)].
struct ColArgs {
  const float* xr;
  const float* xi;
  float* yr;
  float* yi;
  long long ncols, O1, O2, O3;
  long long is_o1, is_o2, is_o3, is_j;
  long long os_o1, os_o2, os_o3, os_k, os_c;
  int has_tw;
  long long tw_mul, tw_a, tw_b, tw_c, tw_modo;
  long long tw_coff;  // added to the column index in the twiddle exponent
  long long nmask;
  int tw_split;
  const float2* tw_hi;
  const float2* tw_lo;
  float scale;
  // kind 2 (scatter to peers): output k of outer block o1 has global index
  // K = o1*sc_ka + k*sc_kb and goes to rank q = K >> sc_rows_log, row
  // K mod 2^sc_rows_log, column sc_col0 + c of that rank's row buffer (sc_ld
  // floats per row).
  int sc_npeers;
  int sc_rows_log;
  // filled by launch_colpass: 32-bit tile decode (log2 >= 0 selects shift and
  // mask for a power of two, else division) and whether every element offset
  // inside a tile fits in 31 bits
  uint32_t d_ncb, d_O1, d_O2, d_modo;
  int lg_ncb, lg_O1, lg_O2, lg_modo;
  uint32_t ntiles;   // filled by launch_colpass
  long long max_blocks;  // > 0: cap on the grid (tiles loop), 0: one block per tile
  float* sc_re[8];
  float* sc_im[8];
  long long sc_ka, sc_kb, sc_ld, sc_col0;
};

cudaError_t launch_colpass(int logl, bool inv, int kind, const ColArgs& a, cudaStream_t st);

// Fused STFT (stft.cu): frame f of waveform b covers padded samples
// [f*hop, f*hop + n) = original [f*hop - pad, ...) mapped by pad_mode
// (0 reflect, 1 constant, 2 replicate, 3 circular); output (batch, bins, frames).
struct StftArgs {
  const float* x;
  const float* window;  // n_fft entries
  float* yr;
  float* yi;
  long long batch, len, frames, hop, pad;
  int pad_mode;
  int onesided;
  float scale;
};

cudaError_t launch_stft(int logn, const StftArgs& a, cudaStream_t st);

// Fused inverse STFT (istft.cu): input planes (batch, bins, frames) with bins =
// n/2+1 (onesided) or n; output (batch, out_len): sample o is overlap-add
// position t = o + pad_front (zero where t >= exp_len = n + (frames-1)*hop).
// scale multiplies every inverse-transformed sample (1/n, times sqrt(n) when
// the forward transform was normalised).  seg / nseg are set by the launcher.
struct IstftArgs {
  const float* xr;
  const float* xi;
  const float* window;  // n entries
  float* y;
  long long batch, frames, hop, out_len, pad_front, exp_len, total;
  int onesided;
  float scale;
  int seg;
  long long nseg;
};

cudaError_t launch_istft(int logn, const IstftArgs& a, cudaStream_t st);

// Double-precision sequence transforms (f64.cu): nseq sequences of 2^logl
// points; sequence s starts at (s / inner) * outer + (s % inner) * cs and its
// points are js apart (in_* for the input, out_* / ks for the output).  With
// tw_hi set, output k of sequence s is multiplied by W^e, e = ((s % inner) +
// tw_off) * k & tw_mask, from the two-level table hi[e >> split] * lo[e & ...].
struct F64SeqArgs {
  const double* xr;
  const double* xi;
  double* yr;
  double* yi;
  long long nseq, inner;
  long long in_outer, in_cs, in_js;
  long long out_outer, out_cs, out_ks;
  const double2* tw_hi;
  const double2* tw_lo;
  int tw_split;
  unsigned long long tw_mask;
  long long tw_off;
  double scale;
  // float32 input / output planes: when set they replace xr/xi (yr/yi), converted on load (store)
  const float* xr32;
  const float* xi32;
  float* yr32;
  float* yi32;
};

cudaError_t launch_f64_seq(int logl, bool inv, const F64SeqArgs& a, cudaStream_t st);
cudaError_t launch_f64_blue_pre(const double* xr, const double* xi, const float* xr32, const float* xi32,
                                const double2* chirp, double* ar, double* ai, long long batch, long long n, long long m,
                                bool inv, cudaStream_t st);
cudaError_t launch_f64_blue_mul(double* ar, double* ai, const double2* H, long long batch, long long m, bool inv,
                                cudaStream_t st);
cudaError_t launch_f64_blue_post(const double* ar, const double* ai, const double2* chirp, double* yr, double* yi,
                                 float* yr32, float* yi32, long long batch, long long n, long long m, bool inv,
                                 double scale, cudaStream_t st);
cudaError_t launch_f32_to_f64(const float* x, double* y, long long count, cudaStream_t st);
cudaError_t launch_f64_to_f32(const double* x, float* y, long long count, cudaStream_t st);
// Upload W_4096^i in double to the current device (f64.cu), once per device.
cudaError_t upload_tw64(const double2* host_table);

// Fused fp64 Bluestein for padded lengths m = 2^logm <= 8192: chirp premultiply, m-point FFT,
// times H, unscaled inverse m-point FFT, chirp postmultiply and scale in one kernel (f64.cu).
struct F64BlueArgs {
  const double* xr;
  const double* xi;
  double* yr;
  double* yi;
  const double2* chirp;
  const double2* H;
  long long batch;
  int n;
  double scale;
  const float* xr32;  // float32 planes replacing xr/xi (yr/yi) when set
  const float* xi32;
  float* yr32;
  float* yi32;
};
constexpr int kMaxF64BlueFusedLog = 13;
cudaError_t launch_f64_blue_fused(int logm, bool inv, const F64BlueArgs& a, cudaStream_t st);

// Element-wise complex product y = m[i mod mcount] * s[i] (mask.cu), i < count.
cudaError_t launch_cmul(const float* mr, const float* mi, long long mcount, const float* sr, const float* si,
                        float* yr, float* yi, long long count, cudaStream_t st);

// TF32 tensor-core GEMM with signed K-segments (gemm_tf32.cu):
// C = sum_s (seg_neg[s] ? -1 : 1) * A[seg_a[s]] * B[seg_b[s]]^T (+ bias),
// A_i: M x K (lda), B_i: N x K (ldb), C: M x N (ldc), row-major float32.
#define GEMM_MAX_SEGS 6
struct GemmArgs {
  const float* A[4];
  int na;
  const float* B[4];
  int nb;
  int nseg;
  int seg_a[GEMM_MAX_SEGS];
  int seg_b[GEMM_MAX_SEGS];
  int seg_neg[GEMM_MAX_SEGS];
  float* C;
  const float* bias;
  long long M, N, K, lda, ldb, ldc;
  // epi = 0: C = acc (+ bias).  epi = 1 (three-product complex form): C holds P1 and C2 holds
  // P2 on entry; the epilogue writes C = P1 - P2 (+ bias) and C2 = acc - P1 - P2 (+ bias2).
  int epi;
  float* C2;
  const float* bias2;
};

cudaError_t launch_gemm_tf32(const GemmArgs& g, cudaStream_t st);
cudaError_t launch_split_tf32(const float* x, float* hi, float* lo, long long n, float scale, cudaStream_t st);
// hi / lo of x + y (the operands of the third product of the three-product complex form)
cudaError_t launch_split_tf32_sum(const float* x, const float* y, float* hi, float* lo, long long n, cudaStream_t st);

// Multi-pass Bluestein helpers (bluestein_large.cu).
cudaError_t launch_blue_pre(const float* xr, const float* xi, const float2* chirp, float* ar, float* ai,
                            long long batch, long long n, long long m, bool inv, cudaStream_t st);
cudaError_t launch_blue_mul(float* br, float* bi, const float* hr, const float* hi, long long batch, long long m,
                            bool inv, cudaStream_t st);
cudaError_t launch_blue_post(const float* ar, const float* ai, const float2* chirp, float* yr, float* yi,
                             long long batch, long long n, long long m, bool inv, float scale, cudaStream_t st);

cudaError_t launch_rows_c2c(int logn, bool inv, const RowArgs& a, cudaStream_t st);
bool rows_c2c_tma_ok(int logn, const RowArgs& a);
cudaError_t launch_rows_c2c_tma(int logn, bool inv, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_r2c(int logm, const RowArgs& a, cudaStream_t st);
cudaError_t launch_rows_c2r(int logm, const RowArgs& a, cudaStream_t st);

}  // namespace tfb
