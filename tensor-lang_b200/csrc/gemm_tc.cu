// Split-precision fp32 GEMM on the sm_100a tensor cores: tcgen05.mma with
// the accumulator in tensor memory, operands staged by TMA.
//
// Serves matmul (kernel_generator.py:501-525), linear (:1584-1661) and the
// matmul/linear VJPs (autograd.py:520-537, 619-646), in float32:
//   C[M,N] (+)= op(A)[M,K] @ op(B)[K,N] (+ bias[N]) (relu)
//
// fp32 accuracy from TF32 tensor cores: the tensor core reads an fp32
// operand as TF32 by dropping the low 13 mantissa bits, so the raw operand
// is the "hi" part; a pre-pass writes lo = x - trunc_tf32(x) (exact in fp32)
// to a workspace, and each 8-deep k-step issues three MMAs, hi*hi + hi*lo +
// lo*hi, accumulating in fp32 in TMEM (the dropped lo*lo term is ~2^-22
// relative).
//
// The TF32+bf16 scheme keeps hi*hi on the TF32 path and folds
// both correction terms into one bf16 MMA over a K-concatenated pair:
//   [bf16(A) | bf16(loA)] . [bf16(loB) | bf16(B)]  =  A*loB + loA*B  (+ ~2^-19)
// A pre-pass writes each operand's pair matrix in the operand's own major
// order: for a K-major operand 32 values then 32 lows per 32-deep k-block
// along each row (one 128-byte swizzled row holds a k-block's pair); for an
// MN-major operand 32 rows of values then 32 rows of lows per k-block, each
// row spanning M or N (64-wide MN-major boxes) -- no transpose.  Per 8-deep k-step this is one
// TF32 MMA plus half a bf16 MMA of the same shape: 2 TF32 MMA-times instead of
// 3.  Per product the error is below 9 * 2^-20 relative (lo*lo dropped,
// bf16 rounding of the correction operands).
//
// The BF16X3 scheme (the default) splits each operand into two bf16 terms,
// a = a0 + a1 with a0 = bf16(a) and a1 = bf16(a - a0) (16 significant bits),
// and keeps the three leading products a0*b0 + a0*b1 + a1*b0: a0*b0 reads
// the value halves of the pair tiles, and the pair MMA over [a0|a1].[b1|b0]
// adds both cross terms, so the fp32 operands are never loaded.  Per
// 32-deep k-block the tensor core does 3 bf16 MMA-times (TF32+bf16: 4) and a
// CTA loads 32 KB (TF32+bf16: 64 KB).  Per product the error is below
// ~3 * 2^-16 relative (a1*b1 dropped, bf16 rounding of a1 and b1); measured
// on N(0,1) data at K = 4096-65536: max 5e-6 relative to max|C|, against
// 1.6e-6 for TF32+bf16.
//
// One CTA computes a 128 x 256 tile with 10 warps:
//   warp 0 lane 0   TMA producer (2-stage ring of hi/lo tiles of A and B)
//   warp 1          TMEM allocation; lane 0 issues the MMAs
//   warps 2-9       epilogue: drain each finished TMEM chunk into fp32
//                   registers (round to nearest), then bias, relu,
//                   accumulate, store
// K-major operands (A as stored, B^T as stored) are one TMA box per tile in
// the 128-byte swizzle; MN-major operands (A^T, and B stored [K][N]) are
// 32-wide boxes, one per 32 rows of M or N, in the 128-byte swizzle with
// 32-byte atoms (the layout tcgen05 requires for MN-major tf32).  No TMA
// multicast is used.  Every mbarrier wait is bounded: on timeout the kernel
// records TL_ERR_TIMEOUT in a device flag (tl_device_error) and falls
// through to free its TMEM and exit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "tl_common.cuh"

namespace tl {

__device__ int g_device_error = 0;

namespace {

constexpr int BM = 128, BN = 256, BK = 32, STAGES = 2;
// k-blocks per TMEM accumulation chunk (256 deep): each drain reads the whole
// accumulator out of tensor memory and slows the MMAs while it runs, so
// chunks are as long as the accuracy allows.  Measured max rel err at
// K = 4096-65536 (BF16X3): 4.5e-6 with 8, 4.4e-6 with 4; one chunk for all
// of K reaches 2e-4.  8 is 2.6% faster than 4.
constexpr int KC = 8;
// CTA-pair epilogue drains TMEM 16 columns per load (true) or 32 (false)
constexpr bool kDrain16 = true;
constexpr int A_TILE = BM * BK * 4;            // 16 KB
constexpr int B_TILE = BN * BK * 4;            // 32 KB
constexpr int STAGE_BYTES = 2 * A_TILE + 2 * B_TILE;  // hi + lo of A and B: 96 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int TMEM_COLS = 512;                 // two BN-wide accumulators, used alternately
constexpr int EPI_WARPS = 8;                   // 2 per TMEM lane quarter, BN/2 columns each
constexpr int THREADS = 64 + 32 * EPI_WARPS;   // producer warp, MMA warp, epilogue warps
constexpr unsigned long long kWaitLimitNs = 2000000000ULL;  // 2 s: far above any normal wait

// ---------------------------------------------------------------- PTX -----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: gives up after kWaitLimitNs, flags TL_ERR_TIMEOUT in the
// device error word and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  atomicExch(&g_device_error, TL_ERR_TIMEOUT);
  return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate = 1u) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  // load and wait in one asm statement: the destination registers are only
  // valid after tcgen05.wait::ld, so nothing may read them in between
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 columns of this warp's 32 TMEM lanes (half the registers of tmem_ld32)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor with the tcgen05 version bits.
//   K-major operands:  128-byte swizzle (16-byte atoms, 8-row period), layout 2
//   MN-major operands: 128-byte swizzle with 32-byte atoms (4-row period), layout 1
//                      -- the only shared-memory layout tcgen05 accepts for
//                      MN-major 32-bit (tf32) operands
constexpr uint32_t kLayoutSW128 = 2, kLayoutSW128Atom32 = 1;
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)layout << 61;
  return d;
}
// K-major tile: rows of 128 B (32 tf32 along K), 8-row groups 1024 B apart;
// one 8-deep k-step is a 32-byte advance inside the swizzled row.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int k) {
  return smem_desc(tile + 32 * k, 16, 1024, kLayoutSW128);
}
// MN-major tile: 32-wide chunks of BK rows (128 B per K-row) 4 KB apart;
// 4-row swizzle groups 512 B apart; one 8-deep k-step is 8 rows = 1024 B.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int k) {
  return smem_desc(tile + 1024 * k, 4096, 512, kLayoutSW128Atom32);
}

// Instruction descriptor: kind::tf32, fp32 accumulate, M=128, N=BN.
template <int A_MN, int B_MN>
__host__ __device__ constexpr uint32_t idesc_tf32() {
  return (1u << 4)                 // D format: f32
         | (2u << 7)               // A format: tf32
         | (2u << 10)              // B format: tf32
         | ((uint32_t)A_MN << 15)  // A major (1 = MN)
         | ((uint32_t)B_MN << 16)  // B major (1 = MN)
         | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// Instruction descriptor: kind::f16 with bf16 A and B, fp32 accumulate,
// M=128, N=BN; A_MN / B_MN = 1 for an MN-major operand.
template <int A_MN, int B_MN>
__host__ __device__ constexpr uint32_t idesc_bf16() {
  return (1u << 4)     // D format: f32
         | (1u << 7)   // A format: bf16
         | (1u << 10)  // B format: bf16
         | ((uint32_t)A_MN << 15) | ((uint32_t)B_MN << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// MN-major bf16 pair tile: 64-wide chunks (128 B per pair row, 128-byte
// swizzle) of 64 pair rows, 8 KB apart; 8-row groups 1 KB apart; one 16-deep
// k-step is 16 rows = 2 KB.
constexpr int PAIR_MN_CHUNK = 64 * 64 * 2;
constexpr uint32_t kLayoutSW128Pair = 2;
__device__ __forceinline__ uint64_t mn16_desc(uint32_t tile, int k) {
  uint64_t d = 0;
  const uint32_t saddr = tile + 2048u * (uint32_t)k;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((PAIR_MN_CHUNK >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((1024 >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)kLayoutSW128Pair << 61;
  return d;
}

// Operand schemes
constexpr int kScheme3xTF32 = 0;    // lo tiles fp32: hi*hi + hi*lo + lo*hi, all TF32
constexpr int kSchemeTF32BF16 = 1;  // pair tiles bf16: hi*hi TF32 + one bf16 pair MMA
constexpr int kSchemeBF16X3 = 2;    // pair tiles only: v*v + one bf16 pair MMA, all bf16

struct Params {
  int M, N, K;
  float* C;
  int64_t ldc;
  const float* bias;
  int accumulate;
  int epilogue;
  const float* mask;  // relu-mask epilogue: C = v * (mask > 0), or null
  int64_t ldm;
  int splits;         // CTA-pair kernel: K split this many ways (1: no split)
  float* partial;     // [splits][M][N] raw sums when splits > 1
  int tpc = 1;        // CTA-pair kernel: tiles each cluster computes in turn
  int clc = 0;        // CTA-pair kernel: take pending clusters' tiles (cluster launch control)
  int tma_store = 0;  // CTA-pair kernel: results leave through shared memory and TMA stores
};

// Split-K partial of one thread's BN/2 columns of row `row` (no epilogue).
__device__ __forceinline__ void store_partial(const Params& p, int split, int row, int nb0,
                                              const float (&sum)[BN / 2]) {
  if (row >= p.M || nb0 >= p.N) return;
  float* prow = p.partial + ((int64_t)split * p.M + row) * p.N + nb0;
  if (nb0 + BN / 2 <= p.N && (p.N % 4 == 0)) {
    float4* p4 = reinterpret_cast<float4*>(prow);
#pragma unroll
    for (int j = 0; j < BN / 8; ++j)
      __stcg(p4 + j, make_float4(sum[4 * j], sum[4 * j + 1], sum[4 * j + 2], sum[4 * j + 3]));
  } else {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j)
      if (nb0 + j < p.N) prow[j] = sum[j];
  }
}

// Epilogue of one thread's BN/2 columns of row `row` (bias, relu, relu mask,
// accumulate, store); shared by the single-CTA and CTA-pair kernels.
__device__ __forceinline__ void store_row(const Params& p, int row, int nb0, float (&sum)[BN / 2]) {
  if (row >= p.M || nb0 >= p.N) return;
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j)
      if (nb0 + j < p.N) sum[j] += __ldg(&p.bias[nb0 + j]);
  }
  if (p.epilogue == TL_EPI_RELU) {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) sum[j] = fmaxf(0.f, sum[j]);
  }
  const bool full = nb0 + BN / 2 <= p.N;
  if (p.mask) {
    const float* mrow = p.mask + (int64_t)row * p.ldm + nb0;
    if (full && (p.ldm % 4 == 0) && (((uintptr_t)p.mask & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(mrow) + j);
        sum[4 * j] = __fmul_rn(sum[4 * j], q.x > 0.f ? 1.f : 0.f);
        sum[4 * j + 1] = __fmul_rn(sum[4 * j + 1], q.y > 0.f ? 1.f : 0.f);
        sum[4 * j + 2] = __fmul_rn(sum[4 * j + 2], q.z > 0.f ? 1.f : 0.f);
        sum[4 * j + 3] = __fmul_rn(sum[4 * j + 3], q.w > 0.f ? 1.f : 0.f);
      }
    } else {
#pragma unroll
      for (int j = 0; j < BN / 2; ++j)
        if (nb0 + j < p.N) sum[j] = __fmul_rn(sum[j], mrow[j] > 0.f ? 1.f : 0.f);
    }
  }
  float* crow = p.C + (int64_t)row * p.ldc + nb0;
  if (full && (p.ldc % 4 == 0) && (((uintptr_t)p.C & 15) == 0)) {
    float4* c4 = reinterpret_cast<float4*>(crow);
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
      float4 o = make_float4(sum[4 * j], sum[4 * j + 1], sum[4 * j + 2], sum[4 * j + 3]);
      if (p.accumulate) {
        float4 q = c4[j];
        o.x += q.x; o.y += q.y; o.z += q.z; o.w += q.w;
      }
      c4[j] = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j)
      if (nb0 + j < p.N) crow[j] = p.accumulate ? crow[j] + sum[j] : sum[j];
  }
}

// TA: 0 = A stored [M][K] (K-major), 1 = A stored [K][M] (MN-major)
// TB: 0 = B stored [K][N] (MN-major), 1 = B stored [N][K] (K-major)
//
// The tensor core's fp32 accumulator rounds its additions toward zero, so a
// long K run accumulated in one TMEM accumulator drifts (a relative bias of
// ~1e-5 at K=4096, growing with K).  The MMAs therefore accumulate chunks of
// KC k-blocks, alternately into two TMEM accumulators, and the epilogue warps
// add each finished chunk into fp32 registers with round-to-nearest while
// the tensor core fills the other accumulator.
//
// SCHEME kSchemeTF32BF16: tmAlo / tmBlo are the bf16 pair matrices, always
// K-major ([rows][2*Kp], one 64-wide box per k-block).
template <int TA, int TB, int SCHEME>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmAlo,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmBlo,
                   Params p) {
  constexpr bool PAIR = SCHEME != kScheme3xTF32;  // bf16 pair tiles
  constexpr bool X3 = SCHEME == kSchemeBF16X3;    // pair tiles only, no fp32 tiles
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                  // [STAGES] TMA -> MMA
  uint64_t* empty = bars + STAGES;        // [STAGES] MMA -> TMA
  uint64_t* acc_full = bars + 2 * STAGES; // [2] MMA -> epilogue (chunk finished)
  uint64_t* acc_free = acc_full + 2;      // [2] epilogue -> MMA (chunk drained)
  uint32_t* tmem_slot = (uint32_t*)(acc_free + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nk = (p.K + BK - 1) / BK;
  const int nchunks = (nk + KC - 1) / KC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_free[b]), EPI_WARPS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (kb >= STAGES && !mbar_wait(smem_u32(&empty[s]), ph ^ 1)) break;
        unsigned char* st = smem + s * STAGE_BYTES;
        const uint32_t sA = smem_u32(st), sAl = sA + A_TILE;
        const uint32_t sB = sAl + A_TILE, sBl = sB + B_TILE;
        const uint32_t fb = smem_u32(&full[s]);
        // the bf16 pair tiles are as large as the fp32 tiles (A_TILE, B_TILE)
        mbar_expect_tx(fb, X3 ? A_TILE + B_TILE : STAGE_BYTES);
        const int k0 = kb * BK;
        if (X3) {
          // no fp32 tiles
        } else if (TA == 0) {
          tma_load_2d(sA, &tmA, fb, k0, m0);
          if (!PAIR) tma_load_2d(sAl, &tmAlo, fb, k0, m0);
        } else {
#pragma unroll
          for (int c = 0; c < BM / 32; ++c) {
            tma_load_2d(sA + c * 4096, &tmA, fb, m0 + 32 * c, k0);
            if (!PAIR) tma_load_2d(sAl + c * 4096, &tmAlo, fb, m0 + 32 * c, k0);
          }
        }
        if (X3) {
          // no fp32 tiles
        } else if (TB == 1) {
          tma_load_2d(sB, &tmB, fb, k0, n0);
          if (!PAIR) tma_load_2d(sBl, &tmBlo, fb, k0, n0);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) {
            tma_load_2d(sB + c * 4096, &tmB, fb, n0 + 32 * c, k0);
            if (!PAIR) tma_load_2d(sBl + c * 4096, &tmBlo, fb, n0 + 32 * c, k0);
          }
        }
        if (PAIR) {  // k-block kb of the pair matrices starts at pair index 64*kb = 2*k0
          if (TA == 0) {
            tma_load_2d(sAl, &tmAlo, fb, 2 * k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d(sAl + c * PAIR_MN_CHUNK, &tmAlo, fb, m0 + 64 * c, 2 * k0);
          }
          if (TB == 1) {
            tma_load_2d(sBl, &tmBlo, fb, 2 * k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(sBl + c * PAIR_MN_CHUNK, &tmBlo, fb, n0 + 64 * c, 2 * k0);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32<TA, TB ? 0 : 1>();
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int b = c & 1;
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        if (c >= 2 && !mbar_wait(smem_u32(&acc_free[b]), ((c >> 1) - 1) & 1)) break;
        fence_after();
        const int kb_end = min(nk, (c + 1) * KC);
        for (int kb = c * KC; kb < kb_end; ++kb) {
          const int s = kb % STAGES;
          const uint32_t ph = (kb / STAGES) & 1;
          if (!mbar_wait(smem_u32(&full[s]), ph)) {
            ok = false;
            break;
          }
          fence_after();
          unsigned char* st = smem + s * STAGE_BYTES;
          const uint32_t sA = smem_u32(st), sAl = sA + A_TILE;
          const uint32_t sB = sAl + A_TILE, sBl = sB + B_TILE;
          if constexpr (X3) {
            // values x values: the A pair's first half (k-steps 0, 1) with
            // the B pair's second half (k-steps 2, 3; B pairs hold lows first)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
              mma_bf16(acc, TA ? mn16_desc(sAl, k) : kmajor_desc(sAl, k),
                       TB ? kmajor_desc(sBl, k + 2) : mn16_desc(sBl, k + 2),
                       idesc_bf16<TA, TB ? 0 : 1>(), first);
            }
          } else if constexpr (PAIR) {
#pragma unroll
            for (int k = 0; k < BK / 8; ++k) {
              const uint64_t a = TA ? mnmajor_desc(sA, k) : kmajor_desc(sA, k);
              const uint64_t bh = TB ? kmajor_desc(sB, k) : mnmajor_desc(sB, k);
              const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
              mma_tf32(acc, a, bh, idesc, first);
            }
          }
          if constexpr (PAIR) {
            // 64 bf16 per row (32 values, 32 lows): 4 k-steps of 16, each a 32-byte advance
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_bf16(acc, TA ? mn16_desc(sAl, k) : kmajor_desc(sAl, k),
                       TB ? kmajor_desc(sBl, k) : mn16_desc(sBl, k), idesc_bf16<TA, TB ? 0 : 1>());
          } else {
#pragma unroll
            for (int k = 0; k < BK / 8; ++k) {
              const uint64_t a = TA ? mnmajor_desc(sA, k) : kmajor_desc(sA, k);
              const uint64_t al = TA ? mnmajor_desc(sAl, k) : kmajor_desc(sAl, k);
              const uint64_t bh = TB ? kmajor_desc(sB, k) : mnmajor_desc(sB, k);
              const uint64_t bl = TB ? kmajor_desc(sBl, k) : mnmajor_desc(sBl, k);
              const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
              mma_tf32(acc, a, bh, idesc, first);
              mma_tf32(acc, a, bl, idesc, 1u);
              mma_tf32(acc, al, bh, idesc, 1u);
            }
          }
          mma_commit(smem_u32(&empty[s]));  // frees the stage when these MMAs finish
        }
        mma_commit(smem_u32(&acc_full[b]));  // chunk ready for the epilogue
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int e = warp - 2;                    // 0..EPI_WARPS-1
    const int quarter = warp & 3;              // TMEM lanes this warp may access
    const int half = e >= 4 ? 1 : 0;           // which BN/2 columns it owns
    const int row = m0 + quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float sum[BN / 2];
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) sum[j] = 0.f;
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int b = c & 1;
      if (!mbar_wait(smem_u32(&acc_full[b]), (c >> 1) & 1)) {
        ok = false;
        break;
      }
      fence_after();
      __syncwarp();
      const uint32_t base = tmem + lane_base + (uint32_t)(b * BN + half * (BN / 2));
#pragma unroll
      for (int q = 0; q < BN / 64; ++q) {
        float v[32];
        tmem_ld32(base + q * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[q * 32 + j] = __fadd_rn(sum[q * 32 + j], v[j]);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_free[b])) : "memory");
    }
    if (ok) store_row(p, row, n0 + half * (BN / 2), sum);
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------- CTA-pair kernel ---
// A cluster of two CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2
// on the two SMs of a pair.  CTA r (rank in the cluster) loads rows
// m0+128r..+127 of A and rows n0+128r..+127 of B (the N axis) for every
// k-block into its own shared memory; the leader (rank 0) issues the MMAs,
// which read both CTAs' tiles and accumulate 128 x 256 in each CTA's tensor
// memory.  Per CTA a k-block moves 64 KB under TF32+bf16 (three stages fit)
// instead of the single-CTA tile's 96 KB for the same MMA work, and 32 KB
// under BF16X3 (six stages).  On launches of many waves a cluster computes up
// to four tiles in turn (Params.tpc), its ring and accumulators running on
// across them, so one tile's store overlaps the next tile's MMAs.
//
// Barriers: every TMA load of both CTAs completes on the leader's full[s]
// (the .cta_group::2 form of the load may signal the peer CTA's barrier);
// the leader's MMA commits arrive on empty[s] and acc_full[b] of both CTAs
// (commit multicast); both CTAs' epilogue warps arrive on the leader's
// acc_free[b].  Cluster barriers after set-up and before TMEM release keep
// either CTA from touching a peer that is not ready or has left.
constexpr int STAGES2 = 3;
constexpr int HB = 128;                            // B rows (N) held per CTA
constexpr int B_HALF = HB * BK * 4;                // 16 KB
constexpr int STAGE2_BYTES = 2 * A_TILE + 2 * B_HALF;  // 64 KB per CTA
// Epilogue staging for TMA stores: one 32 x 32 fp32 tile (4 KB, 128-byte
// swizzle) per epilogue warp.
constexpr int STG_TILE = 32 * 32 * 4;
constexpr int STG_BYTES = EPI_WARPS * STG_TILE;
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + STG_BYTES + 1024 + 512;
static_assert(SMEM2_BYTES <= 227 * 1024, "CTA-pair kernel shared memory");
// The BF16X3 scheme stages only the two pair tiles (32 KB per CTA), so twice
// as many stages fit in the same shared memory.
template <int SCHEME>
struct Ring2 {
  static constexpr bool X3 = SCHEME == kSchemeBF16X3;
  static constexpr int kBytes = X3 ? 2 * A_TILE : STAGE2_BYTES;
  static constexpr int kStages = X3 ? 2 * STAGES2 : STAGES2;
  static_assert(kBytes * kStages == STAGE2_BYTES * STAGES2, "ring fits the allocation");
};

// Tile g of a CTA-pair launch, over (split, M tile, N tile) with the N tiles
// fastest -- consecutive tiles share their A rows in L2 -- and, with split K,
// all tiles of split 0 first, then split 1, ...; kb0 / nk: the split's k-blocks.
struct Tile2 {
  int split, m0, n0, kb0, nk;
};
__device__ __forceinline__ Tile2 tile2_of(const Params& p, int g, int m_tiles, int n_tiles,
                                          int nk_all) {
  Tile2 t;
  const int per = m_tiles * n_tiles;
  t.split = g / per;
  const int r = g - t.split * per;
  t.m0 = (r / n_tiles) * 256;
  t.n0 = (r % n_tiles) * 256;
  t.kb0 = (int)((int64_t)t.split * nk_all / p.splits);
  t.nk = (int)((int64_t)(t.split + 1) * nk_all / p.splits) - t.kb0;
  return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
// TMA stores of a staged 32 x 32 fp32 tile (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"((uint64_t)map), "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"((uint64_t)map), "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// the staging tile may be written again once earlier stores have read it
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t a, float x, float y, float z, float w) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w)
               : "memory");
}

// store_row's bias, relu and relu-VJP mask, in place and in the same order
// (so the stored values are the same bits), for a row that exists.
__device__ __forceinline__ void epi_apply(const Params& p, int row, int nb0, float (&sum)[BN / 2]) {
  if (row >= p.M || nb0 >= p.N) return;
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j)
      if (nb0 + j < p.N) sum[j] += __ldg(&p.bias[nb0 + j]);
  }
  if (p.epilogue == TL_EPI_RELU) {
#pragma unroll
    for (int j = 0; j < BN / 2; ++j) sum[j] = fmaxf(0.f, sum[j]);
  }
  if (p.mask) {
    const float* mrow = p.mask + (int64_t)row * p.ldm + nb0;
    if (nb0 + BN / 2 <= p.N && (p.ldm % 4 == 0) && (((uintptr_t)p.mask & 15) == 0)) {
#pragma unroll
      for (int j = 0; j < BN / 8; ++j) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(mrow) + j);
        sum[4 * j] = __fmul_rn(sum[4 * j], q.x > 0.f ? 1.f : 0.f);
        sum[4 * j + 1] = __fmul_rn(sum[4 * j + 1], q.y > 0.f ? 1.f : 0.f);
        sum[4 * j + 2] = __fmul_rn(sum[4 * j + 2], q.z > 0.f ? 1.f : 0.f);
        sum[4 * j + 3] = __fmul_rn(sum[4 * j + 3], q.w > 0.f ? 1.f : 0.f);
      }
    } else {
#pragma unroll
      for (int j = 0; j < BN / 2; ++j)
        if (nb0 + j < p.N) sum[j] = __fmul_rn(sum[j], mrow[j] > 0.f ? 1.f : 0.f);
    }
  }
}

// A warp's 32 rows x BN/2 columns (lane = row) leave in 32-column slabs:
// each lane writes its row of the slab into the warp's staging tile (16-byte
// chunk j of row r at chunk j ^ (r & 7): the tensor map's 128-byte swizzle,
// and no bank conflicts), then lane 0 stores the tile with TMA.  Rows past M
// and columns past N are clipped by the tensor map; slabs that start past
// them are skipped.  With `split` >= 0 the map is the 3-D split-K partial
// buffer [split][M][N].
__device__ __forceinline__ void tma_store_rows(const CUtensorMap* map, uint32_t stg, int lane,
                                               int row0, int nb0, int M, int N, int split,
                                               const float (&sum)[BN / 2]) {
  if (row0 >= M) return;
#pragma unroll
  for (int s = 0; s < BN / 64; ++s) {
    const int c0 = nb0 + 32 * s;
    if (c0 >= N) break;
    if (lane == 0) bulk_wait_read();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t a = stg + (uint32_t)lane * 128u + ((uint32_t)(j ^ (lane & 7)) << 4);
      st_shared_v4(a, sum[32 * s + 4 * j], sum[32 * s + 4 * j + 1], sum[32 * s + 4 * j + 2],
                   sum[32 * s + 4 * j + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (split >= 0)
        tma_store_3d(map, stg, c0, row0, split);
      else
        tma_store_2d(map, stg, c0, row0);
      bulk_commit();
    }
  }
}

__device__ __forceinline__ void mma2_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma2_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate = 1u) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at this shared offset in both CTAs of the pair once
// the leader's MMAs issued so far have completed
__device__ __forceinline__ void mma2_commit_both(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}"
      ::"r"(bar)
      : "memory");
}

// Dynamic tile scheduling with cluster launch control (sm_100): one thread
// asks the hardware to cancel the launch of a cluster that has not started
// yet; the 16-byte answer is written to the same shared-memory offset in
// both CTAs of the pair and completes each CTA's mbarrier there.  When the
// cancel succeeded, this cluster computes the cancelled cluster's tiles.
constexpr int CLC_SLOTS = 4;  // answers in flight before one must be consumed
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes"
      ".multicast::cluster::all.b128 [%0], [%1];" ::"r"(resp),
      "r"(bar)
      : "memory");
}
// blockIdx.x of the first CTA of the cancelled cluster, or -1 when the
// answer says no cluster was left to cancel
__device__ __forceinline__ int clc_first_ctaid_x(uint32_t resp) {
  int x;
  asm volatile(
      "{\n\t.reg .b128 r;\n\t.reg .pred p;\n\t"
      "ld.shared.b128 r, [%1];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "mov.s32 %0, -1;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n\t}"
      : "=r"(x)
      : "r"(resp)
      : "memory");
  return x;
}

// Answer r (the group after a cluster's r-th group): wait for it in this
// CTA, read it and (arrive) tell the leader's clc_empty it was read.  Returns
// the next group, -1 when no cluster was left to cancel, -2 when the wait
// gave up.
__device__ __forceinline__ int clc_next_group(int r, uint64_t* clc_full, bool arrive) {
  const uint32_t q = (uint32_t)(r % CLC_SLOTS);
  const uint32_t full0 = smem_u32(clc_full);
  if (!mbar_wait(full0 + 8u * q, (uint32_t)(r / CLC_SLOTS) & 1u)) return -2;
  // layout: clc_full[CLC_SLOTS], clc_empty[CLC_SLOTS], answers[CLC_SLOTS][16 B]
  const int x = clc_first_ctaid_x(full0 + 16u * CLC_SLOTS + 16u * q);
  if (arrive) mbar_arrive_cluster(mapa_shared(full0 + 8u * CLC_SLOTS, 0) + 8u * q);
  return x < 0 ? -1 : (x >> 1);
}

template <int A_MN, int B_MN>
__host__ __device__ constexpr uint32_t idesc2_tf32() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)A_MN << 15) | ((uint32_t)B_MN << 16) |
         ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}
template <int A_MN, int B_MN>
__host__ __device__ constexpr uint32_t idesc2_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)A_MN << 15) | ((uint32_t)B_MN << 16) |
         ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

template <int TA, int TB, int SCHEME>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmAx,
                    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmBx,
                    const __grid_constant__ CUtensorMap tmC, Params p) {
  constexpr bool PAIR = SCHEME != kScheme3xTF32;  // bf16 pair tiles
  constexpr bool X3 = Ring2<SCHEME>::X3;          // pair tiles only, no fp32 tiles
  constexpr int NST = Ring2<SCHEME>::kStages, SBYTES = Ring2<SCHEME>::kBytes;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* stage_out = smem + NST * SBYTES;  // [EPI_WARPS][STG_TILE], 1024-aligned
  uint64_t* bars = (uint64_t*)(stage_out + STG_BYTES);
  uint64_t* full = bars;                // [NST] loads of both CTAs -> leader's MMA
  uint64_t* empty = bars + NST;         // [NST] MMA -> each CTA's producer
  uint64_t* acc_full = bars + 2 * NST;  // [2] MMA -> each CTA's epilogue
  uint64_t* acc_free = acc_full + 2;        // [2] both CTAs' epilogues -> leader's MMA
  uint64_t* clc_full = acc_free + 2;        // [CLC_SLOTS] scheduling answer arrived (each CTA)
  uint64_t* clc_empty = clc_full + CLC_SLOTS;  // [CLC_SLOTS] answer read by every role (leader)
  unsigned char* clc_resp = (unsigned char*)(clc_empty + CLC_SLOTS);  // [CLC_SLOTS][16 B]
  uint32_t* tmem_slot = (uint32_t*)(clc_resp + 16 * CLC_SLOTS);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tiles come in groups of p.tpc consecutive global indices (tile2_of): group
  // c is cluster c's launch; this cluster starts with its own group and, with
  // p.clc, goes on with the groups of the clusters it cancels.
  const int n_tiles = (p.N + 255) / 256, m_tiles = (p.M + 255) / 256;
  const int nk_all = (p.K + BK - 1) / BK;
  const int total = p.splits * m_tiles * n_tiles;
  const int cid = (int)(blockIdx.x >> 1);
  // every role that reads a scheduling answer arrives once on the leader's
  // clc_empty: both producers, the MMA thread, both CTAs' epilogue warps
  constexpr uint32_t kClcReaders = 3 + 2 * EPI_WARPS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_free[b]), 2 * EPI_WARPS);
    }
    for (int q = 0; q < CLC_SLOTS; ++q) {
      mbar_init(smem_u32(&clc_full[q]), 1);
      mbar_init(smem_u32(&clc_empty[q]), kClcReaders);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  cluster_sync_all();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // The stage ring and the two accumulators run on across the cluster's
  // tiles: k-block `it` (counted over all its tiles) uses stage it % NST,
  // chunk `cg` accumulator cg & 1, so the loads and MMAs of the next tile
  // proceed while the epilogue stores the previous one.
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);  // the leader's full[0]
      bool ok = true;
      int it = 0;
      for (int grp = cid, r = 0; ok; ++r) {
      const int g0 = grp * p.tpc, ntl = min(p.tpc, total - g0);
      for (int t = 0; t < ntl && ok; ++t) {
        const Tile2 tt = tile2_of(p, g0 + t, m_tiles, n_tiles, nk_all);
        const int m0 = tt.m0 + 128 * (int)rank;  // this CTA's rows of A
        const int nb = tt.n0 + HB * (int)rank;   // this CTA's rows of B (N)
        for (int kb = 0; kb < tt.nk; ++kb, ++it) {
          const int s = it % NST;
          const uint32_t ph = (it / NST) & 1;
          if (it >= NST && !mbar_wait(smem_u32(&empty[s]), ph ^ 1)) {
            ok = false;
            break;
          }
          unsigned char* st = smem + s * SBYTES;
          const uint32_t s0 = smem_u32(st);
          // X3 stage: A pair, B pair; otherwise A, A pair (or lo), B, B pair (or lo)
          const uint32_t sA = s0, sAx = X3 ? s0 : s0 + A_TILE;
          const uint32_t sB = sAx + A_TILE, sBx = X3 ? s0 + A_TILE : sB + B_HALF;
          const uint32_t fb = full0 + 8u * (uint32_t)s;
          if (leader) mbar_expect_tx(smem_u32(&full[s]), 2 * SBYTES);
          const int k0 = (tt.kb0 + kb) * BK;
          if (X3) {
            // no fp32 tiles
          } else if (TA == 0) {
            tma_load_2d_pair(sA, &tmA, fb, k0, m0);
            if (!PAIR) tma_load_2d_pair(sAx, &tmAx, fb, k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 32; ++c) {
              tma_load_2d_pair(sA + c * 4096, &tmA, fb, m0 + 32 * c, k0);
              if (!PAIR) tma_load_2d_pair(sAx + c * 4096, &tmAx, fb, m0 + 32 * c, k0);
            }
          }
          if (X3) {
            // no fp32 tiles
          } else if (TB == 1) {
            tma_load_2d_pair(sB, &tmB, fb, k0, nb);
            if (!PAIR) tma_load_2d_pair(sBx, &tmBx, fb, k0, nb);
          } else {
#pragma unroll
            for (int c = 0; c < HB / 32; ++c) {
              tma_load_2d_pair(sB + c * 4096, &tmB, fb, nb + 32 * c, k0);
              if (!PAIR) tma_load_2d_pair(sBx + c * 4096, &tmBx, fb, nb + 32 * c, k0);
            }
          }
          if (PAIR) {
            if (TA == 0) {
              tma_load_2d_pair(sAx, &tmAx, fb, 2 * k0, m0);
            } else {
#pragma unroll
              for (int c = 0; c < BM / 64; ++c)
                tma_load_2d_pair(sAx + c * PAIR_MN_CHUNK, &tmAx, fb, m0 + 64 * c, 2 * k0);
            }
            if (TB == 1) {
              tma_load_2d_pair(sBx, &tmBx, fb, 2 * k0, nb);
            } else {
#pragma unroll
              for (int c = 0; c < HB / 64; ++c)
                tma_load_2d_pair(sBx + c * PAIR_MN_CHUNK, &tmBx, fb, nb + 64 * c, 2 * k0);
            }
          }
        }
      }
      if (!ok || !p.clc) break;
      // every load of this group is issued: ask for the next group (the
      // leader), expect this CTA's copy of the answer, then read it
      {
        const int q = r % CLC_SLOTS;
        mbar_expect_tx(smem_u32(&clc_full[q]), 16);
        if (leader) {
          if (r >= CLC_SLOTS &&
              !mbar_wait(smem_u32(&clc_empty[q]), (uint32_t)(r / CLC_SLOTS - 1) & 1u)) {
            ok = false;
            break;
          }
          clc_try_cancel(smem_u32(clc_resp + 16 * q), smem_u32(&clc_full[q]));
        }
      }
      grp = clc_next_group(r, clc_full, true);
      if (grp < 0) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA (leader)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc2_tf32<TA, TB ? 0 : 1>();
      bool ok = true;
      int it = 0, cg = 0;
      for (int grp = cid, r = 0; ok; ++r) {
      const int g0 = grp * p.tpc, ntl = min(p.tpc, total - g0);
      for (int t = 0; t < ntl && ok; ++t) {
        const Tile2 tt = tile2_of(p, g0 + t, m_tiles, n_tiles, nk_all);
        const int nchunks = (tt.nk + KC - 1) / KC;
        for (int c = 0; c < nchunks && ok; ++c, ++cg) {
          const int b = cg & 1;
          const uint32_t acc = tmem + (uint32_t)(b * BN);
          if (cg >= 2 && !mbar_wait(smem_u32(&acc_free[b]), ((cg >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          fence_after();
          const int kb_end = min(tt.nk, (c + 1) * KC);
          for (int kb = c * KC; kb < kb_end; ++kb, ++it) {
            const int s = it % NST;
            const uint32_t ph = (it / NST) & 1;
            if (!mbar_wait(smem_u32(&full[s]), ph)) {
              ok = false;
              break;
            }
            fence_after();
            unsigned char* st = smem + s * SBYTES;
            const uint32_t s0 = smem_u32(st);
            const uint32_t sA = s0, sAx = X3 ? s0 : s0 + A_TILE;
            const uint32_t sB = sAx + A_TILE, sBx = X3 ? s0 + A_TILE : sB + B_HALF;
            if constexpr (X3) {
              // values x values: the A pair's first half (k-steps 0, 1) with
              // the B pair's second half (k-steps 2, 3; B pairs hold lows first)
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
                mma2_bf16(acc, TA ? mn16_desc(sAx, k) : kmajor_desc(sAx, k),
                          TB ? kmajor_desc(sBx, k + 2) : mn16_desc(sBx, k + 2),
                          idesc2_bf16<TA, TB ? 0 : 1>(), first);
              }
            } else if constexpr (PAIR) {
#pragma unroll
              for (int k = 0; k < BK / 8; ++k) {
                const uint64_t a = TA ? mnmajor_desc(sA, k) : kmajor_desc(sA, k);
                const uint64_t bh = TB ? kmajor_desc(sB, k) : mnmajor_desc(sB, k);
                const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
                mma2_tf32(acc, a, bh, idesc, first);
              }
            }
            if constexpr (PAIR) {
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma2_bf16(acc, TA ? mn16_desc(sAx, k) : kmajor_desc(sAx, k),
                          TB ? kmajor_desc(sBx, k) : mn16_desc(sBx, k), idesc2_bf16<TA, TB ? 0 : 1>());
            } else {
#pragma unroll
              for (int k = 0; k < BK / 8; ++k) {
                const uint64_t a = TA ? mnmajor_desc(sA, k) : kmajor_desc(sA, k);
                const uint64_t al = TA ? mnmajor_desc(sAx, k) : kmajor_desc(sAx, k);
                const uint64_t bh = TB ? kmajor_desc(sB, k) : mnmajor_desc(sB, k);
                const uint64_t bl = TB ? kmajor_desc(sBx, k) : mnmajor_desc(sBx, k);
                const uint32_t first = (kb == c * KC && k == 0) ? 0u : 1u;
                mma2_tf32(acc, a, bh, idesc, first);
                mma2_tf32(acc, a, bl, idesc, 1u);
                mma2_tf32(acc, al, bh, idesc, 1u);
              }
            }
            mma2_commit_both(smem_u32(&empty[s]));  // frees stage s in both CTAs
          }
          mma2_commit_both(smem_u32(&acc_full[b]));  // chunk ready in both CTAs
        }
      }
      if (!ok || !p.clc) break;
      grp = clc_next_group(r, clc_full, true);
      if (grp < 0) break;
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- epilogue
    const int e = warp - 2;
    const int quarter = warp & 3;
    const int half = e >= 4 ? 1 : 0;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t free0 = mapa_shared(smem_u32(&acc_free[0]), 0);  // the leader's acc_free[0]
    const uint32_t tbase = tmem + lane_base + (uint32_t)(half * (BN / 2));
    float sum[BN / 2];
    bool ok = true;
    int cg = 0;
    for (int grp = cid, r = 0; ok; ++r) {
    const int g0 = grp * p.tpc, ntl = min(p.tpc, total - g0);
    for (int g = g0; g < g0 + ntl && ok; ++g) {
      // only the chunk count is needed while the tile drains (the registers
      // hold the row's partial sums); its position is derived for the store
      const int nchunks = (tile2_of(p, g, m_tiles, n_tiles, nk_all).nk + KC - 1) / KC;
#pragma unroll
      for (int j = 0; j < BN / 2; ++j) sum[j] = 0.f;
      for (int c = 0; c < nchunks; ++c, ++cg) {
        const int b = cg & 1;
        if (!mbar_wait(smem_u32(&acc_full[b]), (cg >> 1) & 1)) {
          ok = false;
          break;
        }
        fence_after();
        __syncwarp();
        const uint32_t base = tbase + (uint32_t)(b * BN);
        if constexpr (kDrain16) {
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            float v[16];
            tmem_ld16(base + q * 16, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) sum[q * 16 + j] = __fadd_rn(sum[q * 16 + j], v[j]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < BN / 64; ++q) {
            float v[32];
            tmem_ld32(base + q * 32, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) sum[q * 32 + j] = __fadd_rn(sum[q * 32 + j], v[j]);
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(free0 + 8u * (uint32_t)b);
      }
      ok = __all_sync(0xffffffffu, ok);  // the slab stores below are warp-wide
      if (ok) {
        const Tile2 tt = tile2_of(p, g, m_tiles, n_tiles, nk_all);
        const int row = tt.m0 + 128 * (int)rank + quarter * 32 + lane;
        const int nb0 = tt.n0 + half * (BN / 2);
        if (p.tma_store) {
          if (p.splits == 1) epi_apply(p, row, nb0, sum);
          tma_store_rows(&tmC, smem_u32(stage_out + e * STG_TILE), lane, row - lane, nb0, p.M, p.N,
                         p.splits > 1 ? tt.split : -1, sum);
        } else if (p.splits > 1) {
          store_partial(p, tt.split, row, nb0, sum);
        } else {
          store_row(p, row, nb0, sum);
        }
      }
    }
    if (!ok || !p.clc) break;
    // every lane reads the answer; lane 0 reports the warp's read
    grp = clc_next_group(r, clc_full, lane == 0);
    __syncwarp();
    if (grp < 0) break;
    }
    // the staging tiles stay allocated until every TMA store has read them
    if (p.tma_store && lane == 0) bulk_wait_all();
    __syncwarp();
  }
  fence_before();
  cluster_sync_all();  // neither CTA releases TMEM or exits while the pair is still working
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                 : "memory");
  }
}

// Split-K fold: C = epilogue(sum over splits of the partial sums, in split
// order), four columns per thread when N is a multiple of 4.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(Params p) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t mn = (int64_t)p.M * p.N;
  if (p.N % 4 == 0 && p.ldc % 4 == 0 && (((uintptr_t)p.C & 15) == 0)) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn / 4; i += stride) {
      float4 v = __ldcs(reinterpret_cast<const float4*>(p.partial) + i);
      for (int s = 1; s < p.splits; ++s) {
        const float4 q = __ldcs(reinterpret_cast<const float4*>(p.partial + (int64_t)s * mn) + i);
        v.x += q.x; v.y += q.y; v.z += q.z; v.w += q.w;
      }
      const int64_t e = 4 * i, row = e / p.N, col = e - row * p.N;
      float o[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (p.bias) o[c] += p.bias[col + c];
        if (p.epilogue == TL_EPI_RELU) o[c] = fmaxf(0.f, o[c]);
        if (p.mask) o[c] = __fmul_rn(o[c], p.mask[row * p.ldm + col + c] > 0.f ? 1.f : 0.f);
      }
      float4* c4 = reinterpret_cast<float4*>(p.C + row * p.ldc + col);
      if (p.accumulate) {
        const float4 q = *c4;
        o[0] = q.x + o[0]; o[1] = q.y + o[1]; o[2] = q.z + o[2]; o[3] = q.w + o[3];
      }
      *c4 = make_float4(o[0], o[1], o[2], o[3]);
    }
  } else {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < mn; e += stride) {
      float v = p.partial[e];
      for (int s = 1; s < p.splits; ++s) v += p.partial[(int64_t)s * mn + e];
      const int64_t row = e / p.N, col = e - row * p.N;
      if (p.bias) v += p.bias[col];
      if (p.epilogue == TL_EPI_RELU) v = fmaxf(0.f, v);
      if (p.mask) v = __fmul_rn(v, p.mask[row * p.ldm + col] > 0.f ? 1.f : 0.f);
      float* c = p.C + row * p.ldc + col;
      *c = p.accumulate ? *c + v : v;
    }
  }
}

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// hi = rna_tf32(x), lo = rna_tf32(x - hi): both exactly representable in
// TF32, so the product does not depend on how the tensor core narrows fp32.
__global__ void __launch_bounds__(256) split_hilo_kernel(const float* __restrict__ src,
                                                         float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float x = src[i];
    float h = tf32_rna(x);
    hi[i] = h;
    lo[i] = tf32_rna(x - h);
  }
}

// lo = x - trunc_tf32(x), exact in fp32
__global__ void __launch_bounds__(256) split_lo_kernel(const float* __restrict__ src,
                                                       float* __restrict__ dst, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n4 = n >> 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 x = ld_stream4(src + 4 * i);
    float4 y;
    y.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    y.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    y.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    y.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    reinterpret_cast<float4*>(dst)[i] = y;
  }
  for (int64_t i = 4 * n4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = src[i] - __uint_as_float(__float_as_uint(src[i]) & 0xFFFFE000u);
}

// The low part a pair matrix stores beside bf16(x): for the TF32+bf16 scheme
// (lo_mode 0) x - trunc_tf32(x), the part the TF32 product misses; for the
// BF16X3 scheme (lo_mode 1) x - bf16(x), the part the bf16 value misses.
// Both differences are exact in fp32.
__device__ __forceinline__ float lo_of(float x, int lo_mode) {
  return lo_mode ? x - __bfloat162float(__float2bfloat16_rn(x))
                 : x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
}

// Pair matrix of a K-major operand X[r][k] (row stride ld): row r of P holds,
// per 32-deep k-block j, 32 bf16 of one kind then 32 of the other at columns
// 64j..64j+63 -- bf16(x) first for an A operand, bf16(lo) first for B
// (lo_first).  Columns for k >= K are zero.  Rows r are grid-strided, the 4-k
// groups of a row are spread over the threads.
__global__ void __launch_bounds__(256) pair_rows_kernel(const float* __restrict__ X, int64_t ld,
                                                        int64_t R, int64_t K, int64_t kp,
                                                        int lo_first, int lo_mode,
                                                        __nv_bfloat16* __restrict__ P) {
  const bool vec = (ld % 4 == 0) && (((uintptr_t)X & 15) == 0);
  const int64_t nq = kp >> 2;
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    const float* src = X + r * ld;
    __nv_bfloat16* dst = P + r * 2 * kp;
    for (int64_t q = threadIdx.x; q < nq; q += blockDim.x) {
      const int64_t k = 4 * q;
      float x[4];
      if (vec && k + 3 < K) {
        const float4 v = ld_stream4(src + k);
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = (k + i < K) ? src[k + i] : 0.f;
      }
      const uint2 hv = make_uint2(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]));
      const uint2 lv = make_uint2(pack_bf16(lo_of(x[0], lo_mode), lo_of(x[1], lo_mode)),
                                  pack_bf16(lo_of(x[2], lo_mode), lo_of(x[3], lo_mode)));
      __nv_bfloat16* o = dst + 64 * (k >> 5) + (k & 31);
      *reinterpret_cast<uint2*>(o) = lo_first ? lv : hv;
      *reinterpret_cast<uint2*>(o + 32) = lo_first ? hv : lv;
    }
  }
}

// Pair matrix of an MN-major operand, kept MN-major (X stored [K][R], row
// stride ld): pair row 64j+i holds bf16 of X[32j+i][0..R) and pair row
// 64j+32+i bf16 of lo(X[32j+i][...]) -- the other way round when lo_first --
// in rows of rp (R rounded up to 8) elements.  Rows for k >= K and columns
// r >= R are zero.  A streaming map: each thread converts 8 consecutive r of
// one k row.
__global__ void __launch_bounds__(256) pair_mn_kernel(const float* __restrict__ X, int64_t ld,
                                                      int64_t K, int64_t R, int64_t rp, int64_t kp,
                                                      int lo_first, int lo_mode,
                                                      __nv_bfloat16* __restrict__ P) {
  const bool vec = (ld % 4 == 0) && (((uintptr_t)X & 15) == 0);
  const int64_t ng = rp >> 3;
  for (int64_t k = blockIdx.x; k < kp; k += gridDim.x) {
    const float* src = X + k * ld;
    __nv_bfloat16* vrow = P + (64 * (k >> 5) + (k & 31)) * rp;
    __nv_bfloat16* lrow = vrow + 32 * rp;
    for (int64_t g = threadIdx.x; g < ng; g += blockDim.x) {
      const int64_t r = 8 * g;
      float x[8];
      if (k < K && vec && r + 7 < R) {
        const float4 a = ld_stream4(src + r), b = ld_stream4(src + r + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = (k < K && r + i < R) ? src[r + i] : 0.f;
      }
      const uint4 hv = make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]),
                                  pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
      const uint4 lv = make_uint4(pack_bf16(lo_of(x[0], lo_mode), lo_of(x[1], lo_mode)),
                                  pack_bf16(lo_of(x[2], lo_mode), lo_of(x[3], lo_mode)),
                                  pack_bf16(lo_of(x[4], lo_mode), lo_of(x[5], lo_mode)),
                                  pack_bf16(lo_of(x[6], lo_mode), lo_of(x[7], lo_mode)));
      *reinterpret_cast<uint4*>(vrow + r) = lo_first ? lv : hv;
      *reinterpret_cast<uint4*>(lrow + r) = lo_first ? hv : lv;
    }
  }
}

// Both pair layouts of X [R][C] (row stride ld) from one read: the K-major
// pair (X as [rows = MN][cols = K]: P[r][64j + i], k = c = 32j + i) and the
// MN-major pair (X as [rows = K][cols = MN]: rows 64j + i / 64j + 32 + i for
// k = r = 32j + i, columns c < rp = ceil8(C)).  Either output may be null;
// lo_first selects the B-operand ordering.  Padding (c >= C up to ceil32(C),
// r >= R up to ceil32(R)) is written as zeros.
__global__ void __launch_bounds__(256) pair_both_kernel(const float* __restrict__ X, int64_t ld,
                                                        int64_t R, int64_t C,
                                                        __nv_bfloat16* __restrict__ pk, int k_lo_first,
                                                        __nv_bfloat16* __restrict__ pm, int m_lo_first,
                                                        int lo_mode) {
  const bool vec = (ld % 4 == 0) && (((uintptr_t)X & 15) == 0);
  const int64_t kpc = (C + 31) / 32 * 32;         // K-major row: 2 * kpc bf16
  const int64_t rp = (C + 7) / 8 * 8;             // MN-major row length
  const int64_t r_end = pm ? (R + 31) / 32 * 32 : R;
  const int64_t c_end = pk ? kpc : rp;
  for (int64_t r = blockIdx.x; r < r_end; r += gridDim.x) {
    const float* src = X + r * ld;
    __nv_bfloat16* kv = pk ? pk + r * 2 * kpc : nullptr;
    __nv_bfloat16* mv = pm ? pm + (64 * (r >> 5) + (r & 31)) * rp : nullptr;
    for (int64_t c = 8 * (int64_t)threadIdx.x; c < c_end; c += 8 * (int64_t)blockDim.x) {
      float x[8];
      if (r < R && vec && c + 7 < C) {
        const float4 a = ld_stream4(src + c), b = ld_stream4(src + c + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = (r < R && c + i < C) ? src[c + i] : 0.f;
      }
      const uint4 hv = make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]),
                                  pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
      const uint4 lv = make_uint4(pack_bf16(lo_of(x[0], lo_mode), lo_of(x[1], lo_mode)),
                                  pack_bf16(lo_of(x[2], lo_mode), lo_of(x[3], lo_mode)),
                                  pack_bf16(lo_of(x[4], lo_mode), lo_of(x[5], lo_mode)),
                                  pack_bf16(lo_of(x[6], lo_mode), lo_of(x[7], lo_mode)));
      if (kv && r < R) {
        __nv_bfloat16* o = kv + 64 * (c >> 5) + (c & 31);
        *reinterpret_cast<uint4*>(o) = k_lo_first ? lv : hv;
        *reinterpret_cast<uint4*>(o + 32) = k_lo_first ? hv : lv;
      }
      if (mv && c < rp) {
        *reinterpret_cast<uint4*>(mv + c) = m_lo_first ? lv : hv;
        *reinterpret_cast<uint4*>(mv + 32 * rp + c) = m_lo_first ? hv : lv;
      }
    }
  }
}

// pair_both_kernel that also sums the columns of X (the bias gradient
// db = sum over rows of dY, autograd.py:619-646) from the same read: each
// block accumulates, in double, the columns of its threads over the rows it
// converts (rows blockIdx.x + k * gridDim.x) and writes them as one row of
// `part` ([gridDim.x][C] doubles); colsum_finish_kernel adds those rows.
// J: column steps of 2048 per thread (c_end <= 2048 * J); SUM false: the
// pairs alone (pair_prepare's kernel for up to 8192 columns: the unrolled
// column steps keep every step's loads of a row in flight together).
template <int J, bool SUM>
__global__ void __launch_bounds__(256) pair_colsum_kernel(const float* __restrict__ X, int64_t ld,
                                                          int64_t R, int64_t C,
                                                          __nv_bfloat16* __restrict__ pk,
                                                          int k_lo_first,
                                                          __nv_bfloat16* __restrict__ pm,
                                                          int m_lo_first, int lo_mode,
                                                          double* __restrict__ part) {
  const bool vec = (ld % 4 == 0) && (((uintptr_t)X & 15) == 0);
  const int64_t kpc = (C + 31) / 32 * 32;
  const int64_t rp = (C + 7) / 8 * 8;
  const int64_t r_end = pm ? (R + 31) / 32 * 32 : R;
  const int64_t c_end = pk ? kpc : rp;
  double acc[J][8];
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[j][i] = 0.0;
  for (int64_t r = blockIdx.x; r < r_end; r += gridDim.x) {
    const float* src = X + r * ld;
    __nv_bfloat16* kv = pk ? pk + r * 2 * kpc : nullptr;
    __nv_bfloat16* mv = pm ? pm + (64 * (r >> 5) + (r & 31)) * rp : nullptr;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int64_t c = 8 * (int64_t)threadIdx.x + 2048 * (int64_t)j;
      if (c >= c_end) continue;
      float x[8];
      if (r < R && vec && c + 7 < C) {
        const float4 a = ld_stream4(src + c), b = ld_stream4(src + c + 4);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = (r < R && c + i < C) ? src[c + i] : 0.f;
      }
      if constexpr (SUM) {
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[j][i] += (double)x[i];  // padding adds zeros
      }
      const uint4 hv = make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]),
                                  pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
      const uint4 lv = make_uint4(pack_bf16(lo_of(x[0], lo_mode), lo_of(x[1], lo_mode)),
                                  pack_bf16(lo_of(x[2], lo_mode), lo_of(x[3], lo_mode)),
                                  pack_bf16(lo_of(x[4], lo_mode), lo_of(x[5], lo_mode)),
                                  pack_bf16(lo_of(x[6], lo_mode), lo_of(x[7], lo_mode)));
      if (kv && r < R) {
        __nv_bfloat16* o = kv + 64 * (c >> 5) + (c & 31);
        *reinterpret_cast<uint4*>(o) = k_lo_first ? lv : hv;
        *reinterpret_cast<uint4*>(o + 32) = k_lo_first ? hv : lv;
      }
      if (mv && c < rp) {
        *reinterpret_cast<uint4*>(mv + c) = m_lo_first ? lv : hv;
        *reinterpret_cast<uint4*>(mv + 32 * rp + c) = m_lo_first ? hv : lv;
      }
    }
  }
  if constexpr (!SUM) return;
  double* prow = part + (int64_t)blockIdx.x * C;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int64_t c = 8 * (int64_t)threadIdx.x + 2048 * (int64_t)j;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (c + i < C) prow[c + i] = acc[j][i];
  }
}

// out[c] = sum of part[b][c] over b < G, in double, in a fixed order (warp w
// adds rows w, w + 32, ... in turn; then warps 0..31 in turn): 32 columns per
// block, one per lane.
__global__ void __launch_bounds__(1024) colsum_finish_kernel(const double* __restrict__ part,
                                                             int64_t G, int64_t C,
                                                             float* __restrict__ out) {
  __shared__ double sh[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  double s = 0.0;
  if (c < C) {
    int64_t b = w;
    for (; b + 96 < G; b += 128) {  // four rows in flight, added in row order
      const double v0 = part[b * C + c], v1 = part[(b + 32) * C + c];
      const double v2 = part[(b + 64) * C + c], v3 = part[(b + 96) * C + c];
      s += v0; s += v1; s += v2; s += v3;
    }
    for (; b < G; b += 32) s += part[b * C + c];
  }
  sh[w][lane] = s;
  __syncthreads();
  if (w == 0 && c < C) {
    double t = sh[0][lane];
    for (int k = 1; k < 32; ++k) t += sh[k][lane];
    out[c] = (float)t;
  }
}

// ------------------------------------------------------------- host side ---
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled g_encode = nullptr;
std::once_flag g_encode_once;
std::mutex g_ws_mu;
struct Workspace {
  float* ptr = nullptr;
  size_t floats = 0;
};
Workspace g_ws[64];
Workspace g_ws_partial[64];  // split-K partial sums
std::vector<float*> g_retired;  // kept alive: captured graphs may still point at them

bool load_encode() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = (PFN_encodeTiled)fn;
  });
  return g_encode != nullptr;
}

// 2-D fp32 tensor map over a row-major [rows][cols] matrix with leading dim ld.
// K-major tiles use the 128-byte swizzle; MN-major tiles its 32-byte-atom form.
bool make_map(CUtensorMap* m, const float* base, int64_t rows, int64_t cols, int64_t ld,
              uint32_t box_inner, uint32_t box_outer, bool mn_major) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D bf16 tensor map over a pair matrix [rows][2*kp]: 64-wide boxes (128 B),
// 128-byte swizzle, K-major.
// 3-D fp32 tensor map over split-K partial sums [splits][M][N]: 32 x 32 x 1
// boxes, 128-byte swizzle (the epilogue's staging layout).
bool make_partial_map(CUtensorMap* m, const float* base, int64_t splits, int64_t M, int64_t N) {
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)splits};
  cuuint64_t strides[2] = {(cuuint64_t)N * 4, (cuuint64_t)(M * N) * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_pair_map(CUtensorMap* m, const __nv_bfloat16* base, int64_t rows, int64_t kp,
                   uint32_t box_outer) {
  cuuint64_t dims[2] = {(cuuint64_t)(2 * kp), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(2 * kp) * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D bf16 tensor map over an MN-major pair matrix [2*kp][rp]: 64 x 64 boxes
// (128 B rows), 128-byte swizzle.
bool make_pair_map_mn(CUtensorMap* m, const __nv_bfloat16* base, int64_t rp, int64_t kp) {
  cuuint64_t dims[2] = {(cuuint64_t)rp, (cuuint64_t)(2 * kp)};
  cuuint64_t strides[1] = {(cuuint64_t)rp * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Split workspace, grown on demand outside stream capture and never freed
// (graphs captured earlier may still reference an older buffer).
int workspace(size_t floats, float** out, cudaStream_t st, Workspace* slots = g_ws) {
  int dev = 0;
  TL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return TL_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace& w = slots[dev];
  if (w.floats < floats) {
    cudaStreamCaptureStatus cs;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return TL_ERR_UNSUPPORTED;
    size_t want = floats + floats / 4;
    float* p = nullptr;
    TL_CUDA_TRY(cudaMalloc(&p, want * 4));
    if (w.ptr) g_retired.push_back(w.ptr);
    w.ptr = p;
    w.floats = want;
  }
  *out = w.ptr;
  return TL_OK;
}

int g_split_mode = 0;  // 0: raw operand is hi (lo pre-pass); 1: hi and lo both rounded
int g_scheme = kSchemeBF16X3;
int g_cta_pair = 1;  // 256 x 256 CTA-pair tiles when the product has more than one row tile
int g_tiles_per_cluster = 4;  // upper bound on the tiles one CTA pair computes in turn
// CTA-pair tile schedule: 0 static groups of tiles_per_cluster tiles, one per
// cluster launch; 1 dynamic: one tile per cluster launch, and every running
// cluster takes the tiles of clusters not launched yet (cluster launch
// control), so an SM pair computes tiles back to back until none are left;
// 2 (default) dynamic where it measured faster (use_dynamic)
int g_tile_dynamic = 2;
// CTA-pair epilogue: 1 (default) TMA stores from shared memory where the
// output allows a tensor map, 0 every lane stores its own row
int g_tma_store = 1;

// Tiles per cluster for a CTA-pair launch of `tiles` tiles: each cluster
// launch pays a prologue (barrier set-up, TMEM allocation, pipeline fill) and
// an exposed epilogue (the tile store); a cluster that computes several
// tiles in turn overlaps both with the MMAs of its next tile.  Used only
// while the launch keeps at least four waves of clusters (so the hardware
// scheduler still balances them) and its last wave is no emptier than with
// one tile per cluster (wave efficiency within 1%).
int tiles_per_cluster(int64_t tiles) {
  const int64_t slots = sm_count() / 2;
  if (slots < 1) return 1;
  auto eff = [&](int64_t clusters) {
    const int64_t waves = (clusters + slots - 1) / slots;
    return (double)clusters / (double)(waves * slots);
  };
  const double base = eff(tiles);
  for (int t = g_tiles_per_cluster; t >= 2; --t) {
    const int64_t clusters = (tiles + t - 1) / t;
    if (clusters >= 4 * slots && eff(clusters) >= base - 0.01) return t;
  }
  return 1;
}

// The automatic schedule.  Measured on one B200 (BF16X3, CUDA events):
// dynamic against static 65536x4096x1024 +6%, 8192x4096x1024 +18%,
// 8192x4096x4096 +2.4% (launches static leaves at one tile per cluster, or
// with short tiles), 65536x4096x4096 -0.5% (four tiles per cluster already).
bool use_dynamic(int64_t work, int64_t K) {
  if (g_tile_dynamic != 2) return g_tile_dynamic == 1;
  return tiles_per_cluster(work) == 1 || K <= 1024;
}

// K splits for the CTA-pair kernel: a product of only a few waves of cluster
// tiles leaves most SM pairs idle in its last wave (e.g. 256 tiles on 74
// pairs: 3.46 waves, 86% busy).  Split K so that tiles x splits fill whole
// waves (>= 95%), keeping at least 8 k-blocks (256 of K) per split.
int split_count(int64_t clusters, int64_t nk) {
  const int64_t slots = sm_count() / 2;
  if (slots < 1 || clusters >= 8 * slots) return 1;
  auto eff = [&](int64_t s) {
    const int64_t work = clusters * s, waves = (work + slots - 1) / slots;
    return (double)work / (double)(waves * slots);
  };
  if (eff(1) >= 0.95) return 1;
  for (int s = 2; s <= 8; ++s)
    if (nk / s >= 8 && eff(s) >= 0.95) return s;
  return 1;
}

// Launch the single-CTA or the CTA-pair kernel over prepared tensor maps.
template <int TA, int TB, int SCHEME>
int run_tiles(bool two, const CUtensorMap& ma, const CUtensorMap& max_, const CUtensorMap& mb,
              const CUtensorMap& mbx, const Params& p, int64_t M, int64_t N, cudaStream_t st) {
  if (two) {
    auto kern = gemm_tc2_kernel<TA, TB, SCHEME>;
    TL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES));
    const int64_t clusters = ((M + 255) / 256) * ((N + 255) / 256);
    const int splits = split_count(clusters, (p.K + BK - 1) / BK);
    if (2 * clusters * splits > INT32_MAX) return TL_ERR_UNSUPPORTED;
    Params q = p;
    q.splits = splits;
    q.clc = use_dynamic(clusters * splits, p.K) ? 1 : 0;
    q.tpc = q.clc ? 1 : tiles_per_cluster(clusters * splits);
    const int64_t launched = (clusters * splits + q.tpc - 1) / q.tpc;  // clusters launched
    if (splits > 1) {
      float* part = nullptr;
      TL_TRY(workspace((size_t)splits * M * N, &part, st, g_ws_partial));
      q.partial = part;
    }
    // results through shared memory and TMA stores where the output's layout
    // allows a tensor map (16-byte aligned base and rows); accumulate keeps
    // the read-modify-write stores
    CUtensorMap mc;
    memset(&mc, 0, sizeof(mc));
    if (g_tma_store && !q.accumulate) {
      if (splits > 1)
        q.tma_store = (N % 4 == 0) && make_partial_map(&mc, q.partial, splits, M, N) ? 1 : 0;
      else
        q.tma_store = (q.ldc % 4 == 0) && ((((uintptr_t)q.C) & 15) == 0) &&
                      make_map(&mc, q.C, M, N, q.ldc, 32, 32, false) ? 1 : 0;
    }
    kern<<<(unsigned)(2 * launched), THREADS, SMEM2_BYTES, st>>>(ma, max_, mb, mbx, mc, q);
    if (splits > 1) {
      TL_TRY(after_launch());
      const int64_t units = (N % 4 == 0) ? M * N / 4 : M * N;
      const int64_t cap = 8LL * sm_count();
      splitk_reduce_kernel<<<(unsigned)((units + 255) / 256 < cap ? (units + 255) / 256 : cap), 256, 0,
                             st>>>(q);
    }
  } else {
    auto kern = gemm_tc_kernel<TA, TB, SCHEME>;
    TL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
    kern<<<grid, THREADS, SMEM_BYTES, st>>>(ma, max_, mb, mbx, p);
  }
  return after_launch();
}

unsigned split_grid(size_t n) {
  unsigned g = (unsigned)((n / 4 + 255) / 256);
  unsigned cap = 8u * sm_count();
  return g < 1 ? 1 : (g < cap ? g : cap);
}

unsigned pair_grid(int64_t units) {
  const int64_t cap = 8LL * sm_count();
  return (unsigned)(units < 1 ? 1 : (units < cap ? units : cap));
}

template <int TA, int TB>
int launch_pair(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B,
                int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate, int epilogue,
                const float* mask, int64_t ldm, const void* a_pre, const void* b_pre,
                cudaStream_t st) {
  const int64_t kp = (K + 31) / 32 * 32;
  const int64_t mp = (M + 7) / 8 * 8, np_ = (N + 7) / 8 * 8;  // MN-major pair row lengths
  const bool x3 = g_scheme == kSchemeBF16X3;
  const int lo_mode = x3 ? 1 : 0;
  // K-major pairs: [M][2kp]; MN-major pairs: [2kp][mp] (bf16, 4 bytes per element pair);
  // a pair the caller computed already (a_pre / b_pre) is used as it is
  const size_t a_bytes = a_pre ? 0 : ((size_t)(TA ? mp : M) * kp * 4 + 1023) / 1024 * 1024;
  const size_t b_bytes = b_pre ? 0 : ((size_t)(TB ? N : np_) * kp * 4 + 1023) / 1024 * 1024;
  float* ws = nullptr;
  if (a_bytes + b_bytes) TL_TRY(workspace((a_bytes + b_bytes) / 4, &ws, st));
  const __nv_bfloat16* ap = reinterpret_cast<const __nv_bfloat16*>(a_pre);
  const __nv_bfloat16* bp = reinterpret_cast<const __nv_bfloat16*>(b_pre);
  if (!a_pre) {
    __nv_bfloat16* w = reinterpret_cast<__nv_bfloat16*>(ws);
    if (TA == 0)
      pair_rows_kernel<<<pair_grid(M), 256, 0, st>>>(A, lda, M, K, kp, 0, lo_mode, w);
    else
      pair_mn_kernel<<<pair_grid(kp), 256, 0, st>>>(A, lda, K, M, mp, kp, 0, lo_mode, w);
    TL_TRY(after_launch());
    ap = w;
  }
  if (!b_pre) {
    __nv_bfloat16* w = reinterpret_cast<__nv_bfloat16*>((char*)ws + a_bytes);
    if (TB == 1)
      pair_rows_kernel<<<pair_grid(N), 256, 0, st>>>(B, ldb, N, K, kp, 1, lo_mode, w);
    else
      pair_mn_kernel<<<pair_grid(kp), 256, 0, st>>>(B, ldb, K, N, np_, kp, 1, lo_mode, w);
    TL_TRY(after_launch());
    bp = w;
  }

  const int64_t a_rows = TA ? K : M, a_cols = TA ? M : K;
  const int64_t b_rows = TB ? N : K, b_cols = TB ? K : N;
  const bool two = g_cta_pair && M > BM;
  const uint32_t b_box = two ? HB : BN;  // B rows a CTA loads per k-block (K-major B)
  CUtensorMap ma, map_, mb, mbp;
  if (!make_map(&ma, A, a_rows, a_cols, lda, 32, TA ? 32 : BM, TA == 1) ||
      !make_map(&mb, B, b_rows, b_cols, ldb, 32, TB ? b_box : 32, TB == 0) ||
      !(TA ? make_pair_map_mn(&map_, ap, mp, kp) : make_pair_map(&map_, ap, M, kp, BM)) ||
      !(TB ? make_pair_map(&mbp, bp, N, kp, b_box) : make_pair_map_mn(&mbp, bp, np_, kp)))
    return TL_ERR_UNSUPPORTED;
  Params p{(int)M, (int)N, (int)K, C, ldc, bias, accumulate, epilogue, mask, ldm, 1, nullptr};
  if (x3) return run_tiles<TA, TB, kSchemeBF16X3>(two, ma, map_, mb, mbp, p, M, N, st);
  return run_tiles<TA, TB, kSchemeTF32BF16>(two, ma, map_, mb, mbp, p, M, N, st);
}

template <int TA, int TB>
int launch(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
           float* C, int64_t ldc, const float* bias, int accumulate, int epilogue, const float* mask,
           int64_t ldm, const void* a_pre, const void* b_pre, cudaStream_t st) {
  if (!load_encode()) return TL_ERR_UNSUPPORTED;
  if ((g_scheme == kSchemeTF32BF16 || g_scheme == kSchemeBF16X3) && g_split_mode == 0)
    return launch_pair<TA, TB>(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate, epilogue, mask,
                               ldm, a_pre, b_pre, st);
  const int64_t a_rows = TA ? K : M, a_cols = TA ? M : K;
  const int64_t b_rows = TB ? N : K, b_cols = TB ? K : N;
  // the elements a row-major [rows][cols] matrix with leading dim ld spans
  const size_t a_n = (size_t)(a_rows - 1) * lda + a_cols;
  const size_t b_n = (size_t)(b_rows - 1) * ldb + b_cols;
  const size_t a_pad = (a_n + 63) / 64 * 64, b_pad = (b_n + 63) / 64 * 64;
  const bool explicit_hi = g_split_mode == 1;
  float* ws = nullptr;
  TL_TRY(workspace((explicit_hi ? 2 : 1) * (a_pad + b_pad), &ws, st));
  const float *a_hi = A, *b_hi = B;
  float *a_lo, *b_lo;
  if (explicit_hi) {
    float* ah = ws;
    a_lo = ws + a_pad;
    float* bh = a_lo + a_pad;
    b_lo = bh + b_pad;
    split_hilo_kernel<<<split_grid(a_n), 256, 0, st>>>(A, ah, a_lo, (int64_t)a_n);
    TL_TRY(after_launch());
    split_hilo_kernel<<<split_grid(b_n), 256, 0, st>>>(B, bh, b_lo, (int64_t)b_n);
    TL_TRY(after_launch());
    a_hi = ah;
    b_hi = bh;
  } else {
    a_lo = ws;
    b_lo = ws + a_pad;
    split_lo_kernel<<<split_grid(a_n), 256, 0, st>>>(A, a_lo, (int64_t)a_n);
    TL_TRY(after_launch());
    split_lo_kernel<<<split_grid(b_n), 256, 0, st>>>(B, b_lo, (int64_t)b_n);
    TL_TRY(after_launch());
  }

  CUtensorMap ma, mal, mb, mbl;
  const bool two = g_cta_pair && M > BM;
  const uint32_t a_inner = 32, a_outer = TA ? 32 : BM;
  const uint32_t b_inner = 32, b_outer = TB ? (two ? HB : BN) : 32;
  const bool a_mn = TA == 1, b_mn = TB == 0;
  if (!make_map(&ma, a_hi, a_rows, a_cols, lda, a_inner, a_outer, a_mn) ||
      !make_map(&mal, a_lo, a_rows, a_cols, lda, a_inner, a_outer, a_mn) ||
      !make_map(&mb, b_hi, b_rows, b_cols, ldb, b_inner, b_outer, b_mn) ||
      !make_map(&mbl, b_lo, b_rows, b_cols, ldb, b_inner, b_outer, b_mn))
    return TL_ERR_UNSUPPORTED;
  Params p{(int)M, (int)N, (int)K, C, ldc, bias, accumulate, epilogue, mask, ldm, 1, nullptr};
  return run_tiles<TA, TB, kScheme3xTF32>(two, ma, mal, mb, mbl, p, M, N, st);
}

}  // namespace

bool gemm_tc_ok(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                const float* B, int64_t ldb, const float* C, int64_t ldc) {
  (void)C;
  (void)ldc;
  if (!load_encode()) return false;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return false;
  if (M < 64 || N < 32 || K < 32) return false;          // small products: CUDA cores
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  if (lda % 4 || ldb % 4) return false;                  // TMA strides: multiples of 16 B
  if (((uintptr_t)A & 15) || ((uintptr_t)B & 15)) return false;
  const int64_t a_cols = ta ? M : K, b_cols = tb ? K : N;
  if (lda < a_cols || ldb < b_cols) return false;
  return true;
}

int gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
            const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate,
            int epilogue, const float* mask, int64_t ldm, const void* a_pair, const void* b_pair,
            cudaStream_t st) {
#define TL_TC(a, b) \
  launch<a, b>(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate, epilogue, mask, ldm, a_pair, b_pair, st)
  if (!ta && !tb) return TL_TC(0, 0);
  if (!ta && tb) return TL_TC(0, 1);
  if (ta && !tb) return TL_TC(1, 0);
  return TL_TC(1, 1);
#undef TL_TC
}

bool gemm_uses_pairs(int ta, int tb, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb) {
  if ((g_scheme != kSchemeTF32BF16 && g_scheme != kSchemeBF16X3) || g_split_mode != 0) return false;
  if (M < 64 || N < 32 || K < 32 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return false;
  if (lda % 4 || ldb % 4) return false;
  return lda >= (ta ? M : K) && ldb >= (tb ? K : N);
}

int64_t pair_bytes(int64_t rows, int64_t cols, int layout) {
  if (rows <= 0 || cols <= 0) return -1;
  if (layout == 0) return rows * ((cols + 31) / 32 * 32) * 4;            // K-major
  if (layout == 1) return ((rows + 31) / 32 * 32) * ((cols + 7) / 8 * 8) * 4;  // MN-major
  return -1;
}

// Blocks of the pair pre-pass for rows x cols (and so rows of the column-sum
// partials it writes).
int64_t pair_grid(int64_t rows, bool mnmajor) {
  const int64_t r_end = mnmajor ? (rows + 31) / 32 * 32 : rows;
  const int64_t cap = 8LL * sm_count();
  return r_end < cap ? r_end : cap;
}

int pair_prepare(const float* X, int64_t ld, int64_t rows, int64_t cols, void* kmajor,
                 int k_lo_first, void* mnmajor, int m_lo_first, cudaStream_t st) {
  const int64_t c_end = kmajor ? (cols + 31) / 32 * 32 : (cols + 7) / 8 * 8;
  if (c_end <= 4 * 2048) {
    auto* pk = reinterpret_cast<__nv_bfloat16*>(kmajor);
    auto* pm = reinterpret_cast<__nv_bfloat16*>(mnmajor);
    const int lo = g_scheme == kSchemeBF16X3 ? 1 : 0;
    const int64_t g = pair_grid(rows, mnmajor != nullptr);
    auto launch = [&](auto kern) -> int {
      int per_sm = 0;
      TL_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0));
      const int64_t gg = std::min<int64_t>(g, (int64_t)std::max(per_sm, 1) * sm_count());
      kern<<<(unsigned)gg, 256, 0, st>>>(X, ld, rows, cols, pk, k_lo_first, pm, m_lo_first, lo,
                                         nullptr);
      return after_launch();
    };
    if (c_end <= 2048) return launch(pair_colsum_kernel<1, false>);
    if (c_end <= 4096) return launch(pair_colsum_kernel<2, false>);
    return launch(pair_colsum_kernel<4, false>);
  }
  const int64_t r_end = mnmajor ? (rows + 31) / 32 * 32 : rows;
  const int64_t cap = 8LL * sm_count();
  pair_both_kernel<<<(unsigned)(r_end < cap ? r_end : cap), 256, 0, st>>>(
      X, ld, rows, cols, reinterpret_cast<__nv_bfloat16*>(kmajor), k_lo_first,
      reinterpret_cast<__nv_bfloat16*>(mnmajor), m_lo_first, g_scheme == kSchemeBF16X3 ? 1 : 0);
  return after_launch();
}

size_t pair_colsum_scratch_bytes(int64_t rows, int64_t cols) {
  return (size_t)pair_grid(rows, true) * (size_t)cols * sizeof(double);
}

int pair_prepare_colsum(const float* X, int64_t ld, int64_t rows, int64_t cols, void* kmajor,
                        int k_lo_first, void* mnmajor, int m_lo_first, float* colsum,
                        void* scratch, size_t scratch_bytes, cudaStream_t st) {
  const int64_t g = pair_grid(rows, mnmajor != nullptr);
  const int64_t c_end = kmajor ? (cols + 31) / 32 * 32 : (cols + 7) / 8 * 8;
  if ((size_t)g * (size_t)cols * sizeof(double) > scratch_bytes) return TL_ERR_INVALID_ARG;
  if (c_end > 4 * 2048) return TL_ERR_UNSUPPORTED;
  double* part = static_cast<double*>(scratch);
  auto* pk = reinterpret_cast<__nv_bfloat16*>(kmajor);
  auto* pm = reinterpret_cast<__nv_bfloat16*>(mnmajor);
  const int lo = g_scheme == kSchemeBF16X3 ? 1 : 0;
  // one wave of resident blocks (the double sums take registers: fewer
  // blocks fit an SM than pair_prepare's eight), each converting every
  // g-th row
  auto launch = [&](auto kern) -> int {
    int per_sm = 0;
    TL_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0));
    const int64_t gg = std::min<int64_t>(g, (int64_t)std::max(per_sm, 1) * sm_count());
    kern<<<(unsigned)gg, 256, 0, st>>>(X, ld, rows, cols, pk, k_lo_first, pm, m_lo_first, lo, part);
    TL_TRY(after_launch());
    colsum_finish_kernel<<<(unsigned)((cols + 31) / 32), 1024, 0, st>>>(part, gg, cols, colsum);
    return after_launch();
  };
  if (c_end <= 2048) return launch(pair_colsum_kernel<1, true>);
  if (c_end <= 4096) return launch(pair_colsum_kernel<2, true>);
  return launch(pair_colsum_kernel<4, true>);
}

// The launch run_tiles makes for an M x N x K product on the tensor cores
// (host-side: the same split_count and tiles_per_cluster decisions).
int gemm_tc_plan(int64_t M, int64_t N, int64_t K, int* out) {
  if (M <= 0 || N <= 0 || K <= 0 || !out) return TL_ERR_INVALID_ARG;
  const bool two = g_cta_pair && M > BM;
  if (!two) {
    out[0] = 0;
    out[1] = 1;
    out[2] = 1;
    out[3] = (int)(((N + BN - 1) / BN) * ((M + BM - 1) / BM));
    return TL_OK;
  }
  const int64_t clusters = ((M + 255) / 256) * ((N + 255) / 256);
  const int splits = split_count(clusters, (K + BK - 1) / BK);
  if (2 * clusters * splits > INT32_MAX) return TL_ERR_UNSUPPORTED;
  const bool dyn = use_dynamic(clusters * splits, K);
  const int tpc = dyn ? 1 : tiles_per_cluster(clusters * splits);
  out[0] = dyn ? 2 : 1;
  out[1] = splits;
  out[2] = tpc;
  out[3] = (int)((clusters * splits + tpc - 1) / tpc);
  return TL_OK;
}

void gemm_set_split_mode(int mode) { g_split_mode = mode; }

int gemm_set_cta_pair(int enable) {
  const int prev = g_cta_pair;
  g_cta_pair = enable ? 1 : 0;
  return prev;
}

int gemm_set_tma_store(int mode) {
  const int prev = g_tma_store;
  g_tma_store = mode ? 1 : 0;
  return prev;
}

int gemm_set_tile_dynamic(int mode) {
  const int prev = g_tile_dynamic;
  g_tile_dynamic = mode;
  return prev;
}

int gemm_set_scheme(int scheme) {
  if (scheme != kScheme3xTF32 && scheme != kSchemeTF32BF16 && scheme != kSchemeBF16X3) return -1;
  const int prev = g_scheme;
  g_scheme = scheme;
  return prev;
}

}  // namespace tl

extern "C" int tl_device_error(int* code, int reset) {
  int v = 0;
  TL_CUDA_TRY(cudaMemcpyFromSymbol(&v, tl::g_device_error, sizeof(int)));
  if (code) *code = v;
  if (reset && v) {
    int z = 0;
    TL_CUDA_TRY(cudaMemcpyToSymbol(tl::g_device_error, &z, sizeof(int)));
  }
  return TL_OK;
}
