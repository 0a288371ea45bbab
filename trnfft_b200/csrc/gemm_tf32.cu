// Tensor-core (tcgen05 / TMEM) TF32 GEMM with signed K-segments:
//
//   C[M x N] = sum_s  sign_s * A_s[M x K] * B_s[N x K]^T     (+ bias[N])
//
// A_s and B_s are row-major float32 arrays whose low 13 mantissa bits are
// ignored by the TF32 tensor-core datapath.  With A = A_hi + A_lo (A_hi the
// TF32 part, A_lo the remainder, both produced by k_split_tf32) the three
// segments A_hi*B_hi + A_hi*B_lo + A_lo*B_hi form the 3xTF32 product, which
// keeps float32 accuracy.  The complex product of a planar complex
// X (M x K) with W^T (W: N x K), as in ComplexLinear (trnfft/nn.py:33-49,
// trnfft/nki/dispatch.py:267-345), runs in the three-product form
//   P1 = Xr Wr^T, P2 = Xi Wi^T, P3 = (Xr + Xi)(Wr + Wi)^T,
//   Re = P1 - P2, Im = P3 - P1 - P2:
// three GEMMs of three segments (9 TF32 products instead of the 12 of
// Re = Xr Wr^T - Xi Wi^T, Im = Xr Wi^T + Xi Wr^T); the third GEMM's epilogue
// (epi = 1) combines the three products and adds the biases.
//
// Accumulation: the tensor core's in-place float32 accumulation has a
// systematic rounding bias that grows linearly with K (measured: 9e-5
// relative at K = 4096 on positive data).  So partial sums over at most 6
// TF32 segments x 32 of K are accumulated in one of two TMEM buffers, and the
// epilogue warps add each into round-to-nearest float32 registers while the
// next accumulates into the other buffer.
//
// Kernel structure (one CTA per 128 x 256 output tile, 320 threads):
//   warp 0   : one thread issues 2-D TMA loads (SWIZZLE_128B, no multicast)
//              of a 128 x 32 A tile and a 256 x 32 B tile per stage;
//   warp 1   : allocates 512 TMEM columns, one thread issues tcgen05.mma
//              (M=128, N=256, K=8, kind::tf32) and commits each stage back to
//              the producer and each accumulation group to the epilogue;
//   warps 2-9: epilogue, tcgen05.ld of the partial sums (each warp 32 TMEM
//              lanes x 128 columns), float32 accumulation; at the end the
//              block goes through shared memory (the free stage buffers) so
//              that global memory sees 128-byte row runs.
// Every wait is bounded: on timeout the CTA records the device status word,
// drains what it issued (bounded), frees its TMEM and exits.
#include <atomic>
#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "tma.cuh"

namespace tfb {

namespace gemm {

constexpr int BM = 128, BN = 256, BK = 32;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;  // 16 KiB
constexpr int B_BYTES = BN * BK * 4;  // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;  // two warps per TMEM lane quarter, 128 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;  // two 256-column accumulators
constexpr size_t SMEM = 1024 /*align slack*/ + (size_t)STAGES * STAGE_BYTES + 256;
static_assert(SMEM <= 227 * 1024, "shared memory budget");
static_assert(EPI_WARPS * 32 * 129 * 4 <= STAGES * STAGE_BYTES, "epilogue staging fits in the stage buffers");

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;            // descriptor version
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D f32, A/B tf32, K-major, M=128, N=256, optional B negate.
__host__ __device__ constexpr uint32_t idesc_tf32(bool negate_b) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((negate_b ? 1u : 0u) << 14) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace gemm

// Epilogue of one warp's 32 x 128 accumulator block (rows row0.., columns col0..; lane l holds
// row row0 + l).  The block goes through this warp's region of shared memory (32 rows, pitch
// 129 floats: conflict-free both ways) so that global memory is read and written in 128-byte
// row runs instead of one row per lane.  Called after the tile's last drain, when the stage
// buffers that hold the region are no longer read by the tensor core or written by TMA.
__device__ __forceinline__ void gemm_store_block(const float (&acc)[128], float* stile, int lane,
                                                 float* __restrict__ C, float* __restrict__ C2,
                                                 const float* __restrict__ bias, const float* __restrict__ bias2,
                                                 int epi, int row0, int col0, int M, int N, long long ldc) {
  fence_proxy_async();
#pragma unroll
  for (int j = 0; j < 128; ++j) stile[lane * 129 + j] = acc[j];
  __syncwarp();
  float b1[4], b2[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int gc = col0 + c * 32 + lane;
    b1[c] = (bias && gc < N) ? __ldg(bias + gc) : 0.f;
    b2[c] = (bias2 && gc < N) ? __ldg(bias2 + gc) : 0.f;
  }
  for (int r = 0; r < 32; ++r) {
    const int row = row0 + r;
    if (row >= M) break;
    float* c1 = C + (long long)row * ldc + col0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = c * 32 + lane;
      if (col0 + col >= N) continue;
      const float v = stile[r * 129 + col];
      if (epi == 0) {
        c1[col] = v + b1[c];
      } else {
        float* c2 = C2 + (long long)row * ldc + col0;
        const float p1 = c1[col], p2 = c2[col];
        c1[col] = (p1 - p2) + b1[c];
        c2[col] = (v - p1 - p2) + b2[c];
      }
    }
  }
}

struct GemmSegs {
  int nseg;
  int kacc;  // K blocks accumulated in one TMEM buffer between drains
  int a_idx[GEMM_MAX_SEGS];
  int b_idx[GEMM_MAX_SEGS];
  int neg[GEMM_MAX_SEGS];
};

__global__ void __launch_bounds__(gemm::THREADS, 1)
    k_gemm_tf32(const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap ma1,
                const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap ma3,
                const __grid_constant__ CUtensorMap mb0, const __grid_constant__ CUtensorMap mb1,
                const __grid_constant__ CUtensorMap mb2, const __grid_constant__ CUtensorMap mb3, GemmSegs segs,
                float* __restrict__ C, const float* __restrict__ bias, int M, int N, int K, long long ldc,
                int epi, float* __restrict__ C2, const float* __restrict__ bias2) {
  using namespace gemm;
  extern __shared__ __align__(1024) unsigned char smraw[];
  // 1024-byte aligned stage buffers (the 128-byte swizzle pattern repeats every 1024 bytes)
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // 2: partial sum of a K block ready in TMEM buffer p
  uint64_t* acc_empty = acc_full + 2;    // 2: epilogue has drained TMEM buffer p
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * BM;
  const int kblocks = (K + BK - 1) / BK;
  const int iters = kblocks * segs.nseg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int p = 0; p < 2; ++p) {
      mbar_init(&acc_full[p], 1);
      mbar_init(&acc_empty[p], EPI_WARPS);
    }
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  volatile int* vabort = abort_flag;

  const CUtensorMap* amaps[4] = {&ma0, &ma1, &ma2, &ma3};
  const CUtensorMap* bmaps[4] = {&mb0, &mb1, &mb2, &mb3};

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer
      int issued = 0;
      for (int it = 0; it < iters; ++it) {
        const int s = it % STAGES;
        const int round = it / STAGES;
        if (round > 0 && !mbar_wait_bounded(&empty[s], (round - 1) & 1)) {
          atomicExch(abort_flag, 1);
          break;
        }
        if (*vabort) break;
        const int kb = it / segs.nseg;
        const int sg = it % segs.nseg;
        unsigned char* sa = base + s * STAGE_BYTES;
        unsigned char* sb = sa + A_BYTES;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        tma_load_2d(sa, amaps[segs.a_idx[sg]], kb * BK, m0, &full[s]);
        tma_load_2d(sb, bmaps[segs.b_idx[sg]], kb * BK, n0, &full[s]);
        ++issued;
      }
      if (*vabort) {
        // drain: issued stages must land before shared memory is released
        for (int it = (issued > STAGES ? issued - STAGES : 0); it < issued; ++it)
          (void)mbar_wait_bounded(&full[it % STAGES], (it / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t base_addr = smem_u32(base);
      for (int kb = 0; kb < kblocks && !*vabort; ++kb) {
        const int grp = kb / segs.kacc;  // accumulation group: one TMEM buffer, one drain
        const int p = grp & 1;
        const bool first = kb % segs.kacc == 0;
        if (first && grp >= 2 && !mbar_wait_bounded(&acc_empty[p], ((grp >> 1) - 1) & 1)) {
          atomicExch(abort_flag, 1);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dacc = tmem + (uint32_t)(p * BN);
        bool ok = true;
        for (int sg = 0; sg < segs.nseg; ++sg) {
          const int it = kb * segs.nseg + sg;
          const int s = it % STAGES;
          if (!mbar_wait_bounded(&full[s], (it / STAGES) & 1) || *vabort) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t idesc = idesc_tf32(segs.neg[sg] != 0);
          const uint32_t sa = base_addr + s * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // advance 8 tf32 = 32 bytes along K inside the swizzled 128-byte row
            mma_tf32(dacc, smem_desc_sw128(sa + k * 32), smem_desc_sw128(sb + k * 32), idesc,
                     (!first || sg > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) {
          atomicExch(abort_flag, 1);
          break;
        }
        if (kb % segs.kacc == segs.kacc - 1 || kb == kblocks - 1) mma_commit(&acc_full[p]);
      }
      if (*vabort) {
        // release epilogue warps that may be waiting
        mbar_arrive(&acc_full[0]);
        mbar_arrive(&acc_full[1]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9): TMEM lanes 32*(warp%4), columns 128*h .. +127
    const int q = warp % 4;
    const int h = (warp - 2) / 4;
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.f;
    bool good = true;
    const int ngroups = (kblocks + segs.kacc - 1) / segs.kacc;
    for (int grp = 0; grp < ngroups; ++grp) {
      const int p = grp & 1;
      if (!mbar_wait_bounded(&acc_full[p], (grp >> 1) & 1)) {
        atomicExch(abort_flag, 1);
        good = false;
        break;
      }
      if (*vabort) {
        good = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(p * BN + h * 128 + c * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] += __uint_as_float(v[j]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[p]);
    }
    if (good && !*vabort)
      gemm_store_block(acc, reinterpret_cast<float*>(base) + (warp - 2) * (32 * 129), lane, C, C2, bias, bias2, epi,
                       m0 + q * 32, n0 + h * 128, M, N, ldc);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
  if (threadIdx.x == 0 && *vabort) atomicExch(&g_dev_status, kStatusWaitTimeout);
}

// ---------------------------------------------------------------------------
// Two-SM variant (tcgen05 cta_group::2): a cluster of two CTAs (cluster dims
// (2, 1, 1), the pair along x) computes a 256 x 256 output tile.  CTA r of the pair stages rows r*128.. of the A tile
// and rows r*128.. of the B tile (128 x 32 each, 32 KiB per stage, 6 stages);
// the even CTA issues tcgen05.mma.cta_group::2 with M = 256, N = 256, which
// reads both CTAs' shared memory and accumulates rows r*128.. of the tile in
// CTA r's TMEM.  Per CTA that is the same 128 x 256 output as the one-CTA
// kernel with two thirds of its shared-memory operand traffic (32 KiB instead
// of 48 KiB written by TMA and read by the tensor core per 32-wide K step).
//   * both CTAs' TMA loads report their bytes to the even CTA's full barrier
//     (`.cta_group::2` form; no multicast), which expects 64 KiB per stage;
//   * the even CTA's commits arrive on the empty / accumulator-ready
//     barriers of both CTAs (tcgen05.commit multicast to the pair);
//   * the epilogue warps of both CTAs release a TMEM buffer by arriving on
//     the even CTA's accumulator-free barrier (16 arrivals).
// Every wait is bounded; a CTA that gives up records the status word, waits a
// bounded time for copies in flight, and meets its peer at the final cluster
// barrier before freeing TMEM.
namespace gemm2 {
constexpr int BM = 128, BN = 256, BK = 32;  // BM / BN: this CTA's rows / the pair's columns
constexpr int HALF_N = BN / 2;
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK * 4;      // 16 KiB
constexpr int B_BYTES = HALF_N * BK * 4;  // 16 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
static_assert(SMEM <= 227 * 1024, "shared memory budget");
static_assert(EPI_WARPS * 32 * 129 * 4 <= STAGES * STAGE_BYTES, "epilogue staging fits in the stage buffers");

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive (once) on `bar` at the same offset in both CTAs of the pair when the MMAs issued so far complete
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_cluster_bounded(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i)
    if (try_wait_cluster(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void settle_after_abort() {
  // bounded pause (~200 us) so that bulk copies already issued land before shared memory is released
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < 200000ull);
}
// M = 256 (the pair), N = 256, tf32 in, f32 accumulate, K-major, optional B negate
__host__ __device__ constexpr uint32_t idesc_pair(bool negate_b) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((negate_b ? 1u : 0u) << 14) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(256 >> 4) << 24);
}
}  // namespace gemm2

__global__ void __launch_bounds__(gemm2::THREADS, 1)
    k_gemm_tf32_pair(const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap ma1,
                     const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap ma3,
                     const __grid_constant__ CUtensorMap mb0, const __grid_constant__ CUtensorMap mb1,
                     const __grid_constant__ CUtensorMap mb2, const __grid_constant__ CUtensorMap mb3,
                     GemmSegs segs, float* __restrict__ C, const float* __restrict__ bias, int M, int N, int K,
                     long long ldc, int epi, float* __restrict__ C2, const float* __restrict__ bias2) {
  using namespace gemm2;
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * STAGE_BYTES);  // used in the even CTA
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // 2
  uint64_t* acc_empty = acc_full + 2;   // 2, used in the even CTA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // 1-D grid of clusters (2, 1, 1); cluster c covers column tile c % ntn of row-tile pair c / ntn
  // (column tiles vary fastest, so the CTAs resident at one time share their A rows in L2)
  const uint32_t rank = cta_rank();  // == blockIdx.x & 1
  const bool leader = rank == 0;
  const int ntn = (N + BN - 1) / BN;
  const int cid = blockIdx.x >> 1;
  const int n0 = (cid % ntn) * BN;
  const int m0 = ((cid / ntn) * 2 + (int)rank) * BM;
  const int kblocks = (K + BK - 1) / BK;
  const int iters = kblocks * segs.nseg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int p = 0; p < 2; ++p) {
      mbar_init(&acc_full[p], 1);
      mbar_init(&acc_empty[p], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();  // barrier init and TMEM allocation visible to both CTAs
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  volatile int* vabort = abort_flag;

  const CUtensorMap* amaps[4] = {&ma0, &ma1, &ma2, &ma3};
  const CUtensorMap* bmaps[4] = {&mb0, &mb1, &mb2, &mb3};

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs): own A rows and own half of the B rows
      const uint32_t full0 = map_rank(full, 0);
      for (int it = 0; it < iters; ++it) {
        const int s = it % STAGES;
        const int round = it / STAGES;
        if (round > 0 && !mbar_wait_bounded(&empty[s], (round - 1) & 1)) {
          atomicExch(abort_flag, 1);
          break;
        }
        if (*vabort) break;
        const int kb = it / segs.nseg;
        const int sg = it % segs.nseg;
        unsigned char* sa = base + s * STAGE_BYTES;
        unsigned char* sb = sa + A_BYTES;
        if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
        const uint32_t fb = full0 + (uint32_t)(s * sizeof(uint64_t));
        tma_load_2d_pair(sa, amaps[segs.a_idx[sg]], kb * BK, m0, fb);
        tma_load_2d_pair(sb, bmaps[segs.b_idx[sg]], kb * BK, n0 + (int)rank * HALF_N, fb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (even CTA)
      const uint32_t base_addr = smem_u32(base);
      for (int kb = 0; kb < kblocks && !*vabort; ++kb) {
        const int grp = kb / segs.kacc;  // accumulation group: one TMEM buffer, one drain
        const int p = grp & 1;
        const bool first = kb % segs.kacc == 0;
        if (first && grp >= 2 && !wait_cluster_bounded(&acc_empty[p], ((grp >> 1) - 1) & 1)) {
          atomicExch(abort_flag, 1);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dacc = tmem + (uint32_t)(p * BN);
        bool ok = true;
        for (int sg = 0; sg < segs.nseg; ++sg) {
          const int it = kb * segs.nseg + sg;
          const int s = it % STAGES;
          if (!mbar_wait_bounded(&full[s], (it / STAGES) & 1) || *vabort) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t idesc = idesc_pair(segs.neg[sg] != 0);
          const uint32_t sa = base_addr + s * STAGE_BYTES;
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k)
            mma_tf32_pair(dacc, gemm::smem_desc_sw128(sa + k * 32), gemm::smem_desc_sw128(sb + k * 32), idesc,
                          (!first || sg > 0 || k > 0) ? 1u : 0u);
          mma_commit_pair(&empty[s]);
        }
        if (!ok) {
          atomicExch(abort_flag, 1);
          break;
        }
        if (kb % segs.kacc == segs.kacc - 1 || kb == kblocks - 1) mma_commit_pair(&acc_full[p]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs): this CTA's 128 rows of the pair tile
    const int q = warp % 4;
    const int h = (warp - 2) / 4;
    const uint32_t acc_empty0 = map_rank(acc_empty, 0);
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.f;
    bool good = true;
    const int ngroups = (kblocks + segs.kacc - 1) / segs.kacc;
    for (int grp = 0; grp < ngroups; ++grp) {
      const int p = grp & 1;
      if (!mbar_wait_bounded(&acc_full[p], (grp >> 1) & 1)) {
        atomicExch(abort_flag, 1);
        good = false;
        break;
      }
      if (*vabort) {
        good = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(p * BN + h * 128 + c * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] += __uint_as_float(v[j]);
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) remote_arrive(acc_empty0 + (uint32_t)(p * sizeof(uint64_t)));
    }
    if (good && !*vabort)
      gemm_store_block(acc, reinterpret_cast<float*>(base) + (warp - 2) * (32 * 129), lane, C, C2, bias, bias2, epi,
                       m0 + q * 32, n0 + h * 128, M, N, ldc);
  }
  __syncthreads();
  if (*vabort) {
    if (threadIdx.x == 0) {
      atomicExch(&g_dev_status, kStatusWaitTimeout);
      settle_after_abort();
    }
    __syncthreads();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();  // the peer no longer reads this CTA's shared memory or arrives on its barriers
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// hi = x with the 13 low mantissa bits cleared (exactly representable in
// TF32), lo = x - hi (exact in float32; the tensor core keeps its top 10
// mantissa bits, so hi + lo carries ~21 bits of x).
__global__ void k_split_tf32(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo, long long n,
                             float scale) {
  long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4;
  const long long stride = (long long)gridDim.x * blockDim.x * 4;
  for (; i < n; i += stride) {
    if (i + 3 < n) {
      float4 v = *reinterpret_cast<const float4*>(x + i);
      float4 h, l;
      float* pv = &v.x;
      float* ph = &h.x;
      float* pl = &l.x;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float s = pv[t] * scale;
        ph[t] = __uint_as_float(__float_as_uint(s) & 0xFFFFE000u);
        pl[t] = s - ph[t];
      }
      *reinterpret_cast<float4*>(hi + i) = h;
      *reinterpret_cast<float4*>(lo + i) = l;
    } else {
      for (long long t = i; t < n; ++t) {
        const float s = x[t] * scale;
        hi[t] = __uint_as_float(__float_as_uint(s) & 0xFFFFE000u);
        lo[t] = s - hi[t];
      }
    }
  }
}

// hi / lo split of x + y (the sum rounded once to float32)
__global__ void k_split_tf32_sum(const float* __restrict__ x, const float* __restrict__ y, float* __restrict__ hi,
                                 float* __restrict__ lo, long long n) {
  long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4;
  const long long stride = (long long)gridDim.x * blockDim.x * 4;
  for (; i < n; i += stride) {
    if (i + 3 < n) {
      const float4 a = *reinterpret_cast<const float4*>(x + i);
      const float4 b = *reinterpret_cast<const float4*>(y + i);
      const float s[4] = {a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w};
      float h[4], l[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        h[t] = __uint_as_float(__float_as_uint(s[t]) & 0xFFFFE000u);
        l[t] = s[t] - h[t];
      }
      *reinterpret_cast<float4*>(hi + i) = make_float4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<float4*>(lo + i) = make_float4(l[0], l[1], l[2], l[3]);
    } else {
      for (long long t = i; t < n; ++t) {
        const float sv = x[t] + y[t];
        hi[t] = __uint_as_float(__float_as_uint(sv) & 0xFFFFE000u);
        lo[t] = sv - hi[t];
      }
    }
  }
}

cudaError_t launch_split_tf32_sum(const float* x, const float* y, float* hi, float* lo, long long n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const long long v4 = (n + 3) / 4;
  long long blocks = (v4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_split_tf32_sum<<<(unsigned)blocks, 256, 0, st>>>(x, y, hi, lo, n);
  return cudaGetLastError();
}

cudaError_t launch_split_tf32(const float* x, float* hi, float* lo, long long n, float scale, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const long long v4 = (n + 3) / 4;
  long long blocks = (v4 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_split_tf32<<<(unsigned)blocks, 256, 0, st>>>(x, hi, lo, n, scale);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// host side: tensor maps through the driver entry point (no libcuda link)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// rows x cols row-major float32 (cols contiguous, ld floats between rows), box BK x box_rows
static bool make_map(CUtensorMap* m, const float* ptr, long long rows, long long cols, long long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {(cuuint32_t)gemm::BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static constexpr int kGemmMaxDevices = 64;

// TRNFFT_B200_GEMM_PAIR=1 selects the two-SM kernel (k_gemm_tf32_pair), 0 the one-CTA kernel.
static bool gemm_pair_enabled() {
  static const bool v = [] {
    const char* e = getenv("TRNFFT_B200_GEMM_PAIR");
    return e != nullptr && atoi(e) == 1;
  }();
  return v;
}

cudaError_t launch_gemm_tf32(const GemmArgs& g, cudaStream_t st) {
  using namespace gemm;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return cudaSuccess;
  if (g.nseg < 1 || g.nseg > GEMM_MAX_SEGS || g.na < 1 || g.na > 4 || g.nb < 1 || g.nb > 4)
    return cudaErrorInvalidValue;
  if ((g.K % 4) != 0 || (g.lda % 4) != 0 || (g.ldb % 4) != 0) return cudaErrorInvalidValue;  // 16-byte rows
  if (g.epi != 0 && (g.epi != 1 || g.C2 == nullptr)) return cudaErrorInvalidValue;
  const bool pair = gemm_pair_enabled();
  CUtensorMap am[4], bm[4];
  for (int i = 0; i < 4; ++i) {
    const float* pa = g.A[i < g.na ? i : 0];
    const float* pb = g.B[i < g.nb ? i : 0];
    if (!make_map(&am[i], pa, g.M, g.K, g.lda, BM)) return cudaErrorInvalidValue;
    if (!make_map(&bm[i], pb, g.N, g.K, g.ldb, pair ? gemm2::HALF_N : BN)) return cudaErrorInvalidValue;
  }
  GemmSegs segs;
  segs.nseg = g.nseg;
  // The tensor core's in-place float32 accumulation is biased, so partial sums are drained into
  // round-to-nearest registers every 6 TF32 segments x 32 of K at most: a K block of up to three
  // segments accumulates two K blocks per TMEM buffer (half the drains), longer ones one.
  segs.kacc = g.nseg <= 3 ? 2 : 1;
  for (int s = 0; s < g.nseg; ++s) {
    segs.a_idx[s] = g.seg_a[s];
    segs.b_idx[s] = g.seg_b[s];
    segs.neg[s] = g.seg_neg[s];
  }
  // The dynamic shared-memory opt-in is a per-device function attribute: set
  // it once per device (the current one), under a flag per device that
  // concurrent first calls may both pass (setting it twice is harmless).
  static std::atomic<bool> attr_done[kGemmMaxDevices];
  int dev = 0;
  cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= kGemmMaxDevices || !attr_done[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tf32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k_gemm_tf32_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm2::SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kGemmMaxDevices) attr_done[dev].store(true, std::memory_order_release);
  }
  if (pair) {
    // clusters of two CTAs, one per pair of 128-row tiles (rows past M load zeros and store nothing)
    const long long pairs = (g.M + 2 * gemm2::BM - 1) / (2 * gemm2::BM);
    const long long ntn = (g.N + gemm2::BN - 1) / gemm2::BN;
    if (2 * pairs * ntn > 0x7fffffffLL) return cudaErrorInvalidValue;
    dim3 grid2((unsigned)(2 * pairs * ntn), 1, 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid2;
    cfg.blockDim = dim3(gemm2::THREADS, 1, 1);
    cfg.dynamicSmemBytes = gemm2::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = cudaLaunchKernelEx(&cfg, k_gemm_tf32_pair, am[0], am[1], am[2], am[3], bm[0], bm[1], bm[2],
                                        bm[3], segs, g.C, g.bias, (int)g.M, (int)g.N, (int)g.K, g.ldc, g.epi, g.C2,
                                        g.bias2);
    return le != cudaSuccess ? le : cudaGetLastError();
  }
  dim3 grid((unsigned)((g.N + BN - 1) / BN), (unsigned)((g.M + BM - 1) / BM));
  k_gemm_tf32<<<grid, THREADS, SMEM, st>>>(am[0], am[1], am[2], am[3], bm[0], bm[1], bm[2], bm[3], segs, g.C,
                                           g.bias, (int)g.M, (int)g.N, (int)g.K, g.ldc, g.epi, g.C2, g.bias2);
  return cudaGetLastError();
}

}  // namespace tfb
