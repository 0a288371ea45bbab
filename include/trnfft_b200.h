/*
 * trnfft_b200 -- C ABI of the B200 (sm_100a) FFT hot path.
 *
 * This is the drop-in boundary underneath the Python package trnfft_b200,
 * which mirrors the public API of trnsci/trnfft.  The reference reaches its
 * device kernels through the Python dispatch layer trnfft/nki/dispatch.py
 * (set_backend/_use_nki, dispatch.py:50-71) and the device ladder
 * trnfft/fft_core.py:1063-1150; every entry point below replaces one call
 * site of that ladder, cited beside it.
 *
 * Conventions
 *   - Data are float32, planar (separate real and imaginary arrays), the
 *     layout of trnfft.ComplexTensor (trnfft/complex.py:16-33).  Transforms
 *     are batch-major and contiguous: transform b occupies [b*n, (b+1)*n).
 *   - All pointers are device pointers on the plan's device.  Outputs are
 *     allocated by the caller; no entry point allocates device memory except
 *     trnfft_plan_create (plan tables).
 *   - `stream` is a cudaStream_t passed as void*.  Work is enqueued on it and
 *     the call returns without synchronising.
 *   - Every function returns a trnfft_status; on failure
 *     trnfft_last_error() (thread-local) describes the cause.  Nothing throws
 *     across the boundary.
 *   - Forward transforms use exp(-2*pi*i*j*k/n); inverse transforms use
 *     exp(+2*pi*i*j*k/n) and are scaled by 1/n, like fft_core
 *     (trnfft/fft_core.py:114-116, 1369-1370).
 */
#ifndef TRNFFT_B200_H
#define TRNFFT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRNFFT_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define TRNFFT_API __attribute__((visibility("default")))
#else
#define TRNFFT_API
#endif

typedef enum {
  TRNFFT_SUCCESS = 0,
  TRNFFT_INVALID_VALUE = 1, /* bad size, null pointer, misaligned pointer */
  TRNFFT_UNSUPPORTED = 2,   /* size or mode this build does not implement */
  TRNFFT_CUDA_ERROR = 3,    /* a CUDA runtime call or kernel launch failed */
  TRNFFT_ALLOC_FAILED = 4,  /* plan table allocation failed */
  TRNFFT_INTERNAL = 5
} trnfft_status;

/* Algorithm chosen by a plan (trnfft/plan.py:14-16 has COOLEY_TUKEY and
 * BLUESTEIN; the B200 build splits power-of-two sizes by whether one
 * transform fits on chip). */
typedef enum {
  TRNFFT_ALG_COPY = 0,      /* n == 1 */
  TRNFFT_ALG_STOCKHAM = 1,  /* power of two, n <= 4096: one pass over HBM */
  TRNFFT_ALG_MULTIPASS = 2, /* power of two, n > 4096: one pass up to 16384, else 2-4 passes */
  TRNFFT_ALG_BLUESTEIN = 3, /* any other n: fused chirp-z, one pass over HBM */
  TRNFFT_ALG_MIXED = 4      /* 7-smooth n <= 8192 (not a power of two): direct mixed-radix, one pass */
} trnfft_algorithm;

typedef struct trnfft_plan_s* trnfft_plan_t;

/* ABI version of the loaded library (TRNFFT_B200_ABI_VERSION). */
TRNFFT_API int trnfft_abi_version(void);

/* Thread-local description of the last failure on this thread. */
TRNFFT_API const char* trnfft_last_error(void);

/* Create a plan for length-n transforms on CUDA device `device`.
 * Replaces trnfft.plan.create_plan (trnfft/plan.py:34-46): the algorithm
 * choice (power of two or Bluestein with padded_n = 2^bitlen(2n-2)) is the
 * reference's, and unlike the reference the plan owns device tables
 * (Bluestein chirp and filter spectrum).  Synchronises the device. */
TRNFFT_API int trnfft_plan_create(trnfft_plan_t* plan, int64_t n, int device);

/* Device status word of the library's kernels on `device`: 0 when all is
 * well, 1 when a kernel gave up a bounded wait for its own bulk copies
 * (it then skips its remaining work instead of hanging).  With clear != 0
 * the word is reset.  Synchronous.  No counterpart in the reference (whose
 * kernels have no device-side waits). */
TRNFFT_API int trnfft_device_status(int device, int* status, int clear);

/* Release a plan and its device tables. */
TRNFFT_API int trnfft_plan_destroy(trnfft_plan_t plan);

/* Plan properties: algorithm (trnfft_algorithm), padded length (Bluestein m,
 * else n) and the work-area bytes that an IN-PLACE trnfft_exec_c2c needs for
 * `batch` transforms (0 when none; out-of-place calls never need one). Replaces FFTPlan's fields (trnfft/plan.py:19-28). */
TRNFFT_API int trnfft_plan_query(trnfft_plan_t plan, int* algorithm, int64_t* padded_n, int64_t batch,
                      int64_t* work_bytes);

/* Batched complex-to-complex transform along contiguous rows.
 * Replaces fft_core(x, inverse) (trnfft/fft_core.py:22-50) -> _cooley_tukey
 * (fft_core.py:53-117) / _bluestein (fft_core.py:1285-1376), reached from
 * trnfft.fft / trnfft.ifft (trnfft/api.py:22-35).
 * Power-of-two 4096 < n <= 16384 run as one row pass (one transform per
 * block); larger n (up to 2^30) as two to four column-tile passes
 * (four-step / six-step, trnfft/nki/multicore.py:151-219).  Exactly
 * in-place calls (out_re == in_re and out_im == in_im) are allowed and need
 * no work area up to n = 16384; above that an in-place call needs `work`, a
 * device buffer of trnfft_plan_query's work_bytes, disjoint from the data.
 * Output planes that overlap the input in any other way are rejected
 * (TRNFFT_INVALID_VALUE) up to n = 16384 and copied aside through `work`
 * above it.  Out-of-place calls need no work area (NULL). */
TRNFFT_API int trnfft_exec_c2c(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out_re,
                    float* out_im, int64_t batch, int inverse, void* work, void* stream);

/* Transforms along the middle axis of a contiguous [outer][n][inner] array
 * (element (o, j, s) at o*n*inner + j*inner + s), for power-of-two n up to
 * 2^20 (inner == 1 is exactly trnfft_exec_c2c).  Replaces the per-axis
 * transpose + contiguous copy + fft_core + transpose back of
 * _fft_along_dim (trnfft/api.py:496-516) used by fft2/fftn/ifftn
 * (trnfft/api.py:105-167): the column tiles are read in place.
 * An in-place call with n > 1024 needs `work` of plan_query's size for
 * batch = outer*inner. */
TRNFFT_API int trnfft_exec_c2c_axis(trnfft_plan_t plan, const float* in_re, const float* in_im,
                                    float* out_re, float* out_im, int64_t outer, int64_t inner,
                                    int inverse, void* work, void* stream);

/* In-place complex transform that allocates nothing, for callers that cannot
 * call cudaMalloc or hand over a work area (code running inside another
 * allocator or memory pool, real-time callbacks that must not allocate,
 * runtimes that only lend fixed buffers).  No counterpart in the reference.
 *
 * Only power-of-two n > 4096 (the multi-pass plans; 8192 and 16384 run in
 * place without touching the scratch, larger n copy their input into it) and
 * batch * n <= 2^21 complex values: the scratch is a fixed 16 MiB device
 * array that every GPU loading the library keeps until process exit.
 * Larger requests fail with TRNFFT_INVALID_VALUE.  The first call on a device
 * looks up the array's device address (make that first call before any
 * stream capture).  All calls on a device share the one array, so calls
 * whose work overlaps on the GPU (different streams, or different host
 * threads without ordering) race and corrupt each other's results;
 * serialise them.  The array keeps the last call's contents; nothing in it
 * needs clearing because every call overwrites what it reads. */
TRNFFT_API int trnfft_exec_c2c_inplace_noalloc(trnfft_plan_t plan, float* re, float* im, int64_t batch,
                                               int inverse, void* stream);

/* Double precision.  trnfft_plan_enable_f64 builds the plan's fp64 tables
 * (power of two n up to 2^24; any other n whose Bluestein length m is at most
 * 2^24); it allocates device memory and synchronises, so call it before any
 * stream capture.  trnfft_plan_query_f64 gives the work-area bytes
 * trnfft_exec_c2c_f64 needs for `batch` transforms (0 for powers of two up to
 * 4096).  trnfft_exec_c2c_f64 is trnfft_exec_c2c on planar float64 data with
 * every stage (twiddles, chirp, filter spectrum, butterflies) in fp64.
 * Replaces the reference's accuracy mode precision="double": the fp64
 * Bluestein pipeline (trnfft/fft_core.py:1306-1309, 1372-1374) and the fp64
 * DFT-GEMM for power-of-two n (_fft_via_gemm_double, fft_core.py:254-298,
 * selected at :1108-1110), and its torch backend on float64 tensors.
 * In-place calls are allowed; partly overlapping planes are rejected. */
TRNFFT_API int trnfft_plan_enable_f64(trnfft_plan_t plan);
TRNFFT_API int trnfft_plan_query_f64(trnfft_plan_t plan, int64_t batch, int64_t* work_bytes);
TRNFFT_API int trnfft_exec_c2c_f64(trnfft_plan_t plan, const double* in_re, const double* in_im, double* out_re,
                                   double* out_im, int64_t batch, int inverse, void* work, void* stream);

/* trnfft_exec_c2c_f64 on planar float32 input and output: every stage runs in
 * float64 (precision="double" on float32 tensors, trnfft/fft_core.py:1306-1309,
 * 1372-1374 cast to float64 and back); the widening happens in the first
 * kernel's loads and the narrowing in the last kernel's stores, so no float64
 * copy of the data is made.  Pointers 4-byte aligned; the same work area as
 * trnfft_exec_c2c_f64 (trnfft_plan_query_f64). */
TRNFFT_API int trnfft_exec_c2c_f64_f32io(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out_re,
                                         float* out_im, int64_t batch, int inverse, void* work, void* stream);

/* Convert `count` values between float32 and float64 on `device` (to_double
 * != 0: float -> double).  Used to run float32 data through the fp64
 * transforms of precision="double" (the reference casts with .double() and
 * back, fft_core.py:1308-1309, 1372-1374). */
TRNFFT_API int trnfft_convert_f32_f64(const void* src, void* dst, int64_t count, int to_double, int device,
                                      void* stream);

/* Short-time Fourier transform of `batch` real signals of `length` samples,
 * power-of-two n_fft = plan n (4..8192).  Replaces trnfft.stft
 * (trnfft/api.py:291-365): frames start every `hop` samples of the signal
 * padded by n_fft/2 on both sides when `center` (pad_mode 0 reflect,
 * 1 constant, 2 replicate, 3 circular, as torch.nn.functional.pad), are
 * multiplied by `window` (n_fft floats, already zero-padded to n_fft), and
 * transformed; `normalized` scales by 1/sqrt(n_fft).  Output planes are
 * (batch, bins, frames) with bins = n_fft/2+1 (onesided) or n_fft, and
 * frames = 1 + (length + 2*pad - n_fft) / hop, which the caller passes as a
 * check. */
TRNFFT_API int trnfft_exec_stft(trnfft_plan_t plan, const float* signal, int64_t batch, int64_t length,
                                int64_t hop, const float* window, int center, int pad_mode, int normalized,
                                int onesided, int64_t frames, float* out_re, float* out_im, void* stream);

/* Inverse short-time Fourier transform with windowed overlap-add, power-of-two
 * n_fft = plan n (4..8192).  Replaces trnfft.istft (trnfft/api.py:368-470):
 * each frame of the (batch, bins, frames) planes (bins = n_fft/2+1 when
 * `onesided`, else n_fft, of which the real part of the inverse transform is
 * used) is inverse-transformed, multiplied by `window` (n_fft floats, already
 * zero-padded) and overlap-added every `hop` samples; samples whose envelope
 * sum_f window[t - f*hop]^2 exceeds 1e-8 are divided by it, the others keep
 * the unwindowed sum (api.py:450-452).  `normalized` undoes the forward
 * 1/sqrt(n_fft).  `out` receives batch rows of out_len samples starting at
 * overlap-add position n_fft/2 when `center` (else 0), zero past
 * n_fft + (frames-1)*hop; the caller derives out_len from `length` as
 * api.py:454-468 does.  One kernel, one pass over the spectrum.  hop up to
 * 8192 samples and signals below 2^31 samples (else TRNFFT_UNSUPPORTED). */
TRNFFT_API int trnfft_exec_istft(trnfft_plan_t plan, const float* in_re, const float* in_im, int64_t batch,
                                 int64_t frames, int64_t hop, const float* window, int center, int normalized,
                                 int onesided, int64_t out_len, float* out, void* stream);

/* Element-wise complex product out = mask * spec over `count` elements of
 * planar float32 data, where element i uses mask element i % mask_count
 * (mask_count divides count: a mask repeated over the leading axes).
 * Replaces trnfft.nki.dispatch.complex_mask_apply (trnfft/nki/dispatch.py:
 * 105-113) and its fused NKI kernel (dispatch.py:347-417).  The output may be
 * the spectrogram's planes (in place); it may be the mask's planes only when
 * mask_count == count.  On CUDA device `device`, enqueued on `stream`. */
TRNFFT_API int trnfft_complex_mask_apply(const float* mask_re, const float* mask_im, int64_t mask_count,
                                         const float* spec_re, const float* spec_im, float* out_re, float* out_im,
                                         int64_t count, int device, void* stream);

/* Work-area bytes trnfft_complex_linear needs: the TF32 hi/lo splits of the
 * real part, the imaginary part and their sum, for x and for W:
 * 6*(M+N)*K floats.  -1 for negative sizes. */
TRNFFT_API int64_t trnfft_complex_linear_work_bytes(int64_t M, int64_t N, int64_t K);

/* Complex linear map y = x W^T (+ b) on planar complex operands:
 * x (M x K), W (N x K, the nn.Linear weight layout), y (M x N), row-major,
 * b (N) optional (both parts or neither).  Replaces ComplexLinear.forward
 * (trnfft/nn.py:33-49) and trnfft.nki.dispatch.complex_linear
 * (trnfft/nki/dispatch.py:91-102): three tcgen05 TF32 tensor-core GEMMs in
 * the three-product form P1 = Xr Wr^T, P2 = Xi Wi^T, P3 = (Xr+Xi)(Wr+Wi)^T,
 * Re = P1 - P2, Im = P3 - P1 - P2, each with the 3xTF32 split
 * (hi*hi + hi*lo + lo*hi), float32 accuracy.  K must be a
 * multiple of 4; all pointers 16-byte aligned; `work` holds
 * trnfft_complex_linear_work_bytes(M, N, K) bytes. */
TRNFFT_API int trnfft_complex_linear(const float* xr, const float* xi, const float* wr, const float* wi,
                                     const float* br, const float* bi, float* yr, float* yi, int64_t M,
                                     int64_t N, int64_t K, void* work, int device, void* stream);

/* TF32 hi/lo split of `count` floats (hi = x rounded to TF32, lo = the TF32
 * rounding of x - hi), the operands of the 3xTF32 products; 16-byte aligned
 * pointers.  With trnfft_complex_linear_presplit a caller splits a weight
 * once and reuses it across calls (ComplexLinear caches it per weight
 * version), instead of re-splitting W on every forward. */
TRNFFT_API int trnfft_split_tf32(const float* src, float* hi, float* lo, int64_t count, int device, void* stream);

/* trnfft_split_tf32 of a + b (the sum rounded once to float32): the split of
 * Wr + Wi that the third product of trnfft_complex_linear_presplit uses. */
TRNFFT_API int trnfft_split_tf32_sum(const float* a, const float* b, float* hi, float* lo, int64_t count, int device,
                                     void* stream);

/* trnfft_complex_linear with W already split: w_split holds six N x K planes
 * in the order Wr_hi, Wr_lo, Wi_hi, Wi_lo, Ws_hi, Ws_lo (trnfft_split_tf32 of
 * W_re and W_im, trnfft_split_tf32_sum of the two).  `work` holds the split
 * of x: 6*M*K floats.  Replaces
 * ComplexLinear.forward (trnfft/nn.py:33-49) for a weight that did not change
 * since it was split. */
TRNFFT_API int trnfft_complex_linear_presplit(const float* xr, const float* xi, const float* w_split,
                                              const float* br, const float* bi, float* yr, float* yi, int64_t M,
                                              int64_t N, int64_t K, void* work, int device, void* stream);

/* The column step of the four-step FFT across GPUs: transforms along the
 * middle axis of [outer][n][inner] (plan n, power of two <= 2^20, out of
 * place; ld_in / ld_out floats between the points of a column, 0 = inner,
 * so a column sub-block of a wider array can be read and written densely)
 * and multiplies output (o, K, s) by W_M^{(col_offset + s) * K},
 * M = tw_plan n (a power of two > 1024; its tables are used).  Replaces the
 * column DFTs + host twiddle of _stage_parallel_fft
 * (trnfft/nki/multicore.py:189-204) with one fused pass. */
TRNFFT_API int trnfft_exec_c2c_axis_tw(trnfft_plan_t plan, trnfft_plan_t tw_plan, const float* in_re,
                                       const float* in_im, float* out_re, float* out_im, int64_t outer,
                                       int64_t inner, int64_t ld_in, int64_t ld_out, int inverse,
                                       int64_t col_offset, void* stream);

/* Exchange buffers for the four-step FFT across GPUs, shared between
 * processes with CUDA IPC (no multicast objects).  trnfft_xbuf_alloc
 * allocates `bytes` on `device` and writes its IPC handle
 * (trnfft_ipc_handle_bytes() bytes) to ipc_handle; trnfft_ipc_open maps a
 * peer's buffer on `device`.  No counterpart in the reference (its
 * multi-core path has no collectives, trnfft/nki/multicore.py:39-55). */
TRNFFT_API int trnfft_ipc_handle_bytes(void);
TRNFFT_API int trnfft_xbuf_alloc(int device, int64_t bytes, void** ptr, void* ipc_handle);
TRNFFT_API int trnfft_xbuf_free(int device, void* ptr);
TRNFFT_API int trnfft_ipc_open(int device, const void* ipc_handle, void** ptr);
TRNFFT_API int trnfft_ipc_close(int device, void* ptr);

/* The column step of the four-step FFT across `npeers` GPUs with the
 * exchange fused in: like trnfft_exec_c2c_axis_tw on this rank's column
 * block [n][inner] (ld_in floats per point), but the output of global row
 * K (0 <= K < n) is stored by this kernel into rank K / rows_per_peer's row
 * buffer peer_re/peer_im[q] at row K % rows_per_peer, columns
 * peer_col0 .. peer_col0+inner (peer_ld floats per row): NVLink peer stores
 * replace the all-to-all of the reference's host-side transpose
 * (trnfft/nki/multicore.py:189-217).  The caller orders the ranks before
 * (peers done reading) and after (all stores landed) the call.  n > 1024
 * needs `work` of 2*n*inner floats.  Every peer_re[q] / peer_im[q] must map
 * at least rows_per_peer * peer_ld floats: the library cannot see the size of
 * another process's allocation, and a smaller buffer receives stores past its
 * end. */
TRNFFT_API int trnfft_exec_fourstep_scatter(trnfft_plan_t plan, trnfft_plan_t tw_plan, const float* in_re,
                                            const float* in_im, int64_t inner, int64_t ld_in, int inverse,
                                            int64_t col_offset, int npeers, float* const* peer_re,
                                            float* const* peer_im, int64_t rows_per_peer, int64_t peer_ld,
                                            int64_t peer_col0, void* work, void* stream);

/* Strided block copy on `stream` (device `device` current): `height` rows of
 * `width` bytes from src (rows spitch bytes apart) to dst (dpitch apart),
 * either side local or a peer's buffer mapped with trnfft_ipc_open; the copy
 * engines move it over NVLink.  The exchange step of fft2 across GPUs: each
 * rank writes its column blocks straight into the owners' buffers, replacing
 * the reference's transpose (trnfft/api.py:496-516) without a transposing
 * kernel or an all-to-all staging copy.  No counterpart in the reference (its
 * transforms run on one device). */
TRNFFT_API int trnfft_copy2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width,
                             int64_t height, int device, void* stream);

/* Batched real-to-complex transform: rows of n reals -> rows of n/2+1 bins.
 * Replaces trnfft.rfft (trnfft/api.py:38-46), which runs a full complex
 * transform of the real row and keeps the first n//2+1 bins. */
TRNFFT_API int trnfft_exec_r2c(trnfft_plan_t plan, const float* in, float* out_re, float* out_im,
                    int64_t batch, void* work, void* stream);

/* Batched complex-to-real transform: rows of n/2+1 bins -> rows of n reals,
 * scaled by 1/n.  Replaces trnfft.irfft (trnfft/api.py:49-68): the result is
 * the real part of the inverse transform of the Hermitian extension, so the
 * imaginary parts of bin 0 and (even n) bin n/2 do not contribute. */
TRNFFT_API int trnfft_exec_c2r(trnfft_plan_t plan, const float* in_re, const float* in_im, float* out,
                    int64_t batch, void* work, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRNFFT_B200_H */
