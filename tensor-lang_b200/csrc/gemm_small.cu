// Skinny fp32 GEMMs: one dimension of at most 32.
//
// A classifier head such as linear(a2[B,4096], W3[4096,10]) and its VJPs
// (autograd.py:619-646) are products with N = 10 or K = 10.  Tensor-core
// tiles waste 92% of the work on them, and a 128x128 CUDA-core tile wastes
// as much; all three are bound by the bytes of the large operand.  Each
// kernel here streams the large operand once with coalesced loads and keeps
// the narrow operand in shared memory:
//
//   nn  C[M,N]  = A[M,K]   @ B[K,N]    N <= 32   one warp per row, K split
//                                                  across lanes, warp reduce
//   tn  C[M,N]  = A[K,M]^T @ B[K,N]    N <= 32   one thread per column m,
//                                                  K split into chunks whose
//                                                  partials are combined in a
//                                                  fixed order (deterministic)
//   nt  C[M,N]  = A[M,K]   @ B[N,K]^T  K <= 32   one thread per column n,
//                                                  B row in registers
//
// All accumulate in fp32 with FMA; epilogue: + bias[n], relu, relu mask
// (v * (mask[m, n] > 0)), accumulate.
#include <mutex>
#include <vector>

#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int SMALL = 32;

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// relu-mask epilogue (tl_gemm_masked): v * (mask[m, n] > 0), as the relu VJP
__device__ __forceinline__ float mask_of(float v, const float* mask, int64_t ldm, int64_t m,
                                         int64_t n) {
  return mask ? __fmul_rn(v, mask[m * ldm + n] > 0.f ? 1.f : 0.f) : v;
}

__device__ __forceinline__ float epi(float v, const float* bias, int64_t n, int relu) {
  if (bias) v += bias[n];
  if (relu) v = fmaxf(0.f, v);
  return v;
}

// ------------------------------------------------------------------- nn ---
// Block: 8 warps; B is staged in shared memory in K chunks of KCH rows
// (padded rows of NB+1 floats: conflict-free reads); each warp owns RPW rows.
template <int NB, int RPW>
__global__ void __launch_bounds__(256) small_nn_kernel(int64_t M, int N, int64_t K,
                                                       const float* __restrict__ A, int64_t lda,
                                                       const float* __restrict__ B, int64_t ldb,
                                                       float* __restrict__ C, int64_t ldc,
                                                       const float* __restrict__ bias,
                                                       int accumulate, int relu, const float* __restrict__ mask, int64_t ldm) {
  constexpr int KCH = NB <= 16 ? 512 : 256;  // <= 34 KB of static shared memory
  __shared__ float Bs[KCH][NB + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t m_base = ((int64_t)blockIdx.x * 8 + warp) * RPW;
  float acc[RPW][NB];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;

  for (int64_t k0 = 0; k0 < K; k0 += KCH) {
    const int kc = (int)(K - k0 < KCH ? K - k0 : KCH);
    __syncthreads();
    for (int i = threadIdx.x; i < kc * NB; i += blockDim.x) {
      int kk = i / NB, n = i % NB;
      Bs[kk][n] = (n < N) ? B[(k0 + kk) * ldb + n] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t m = m_base + r;
      if (m >= M) break;
      const float* a = A + m * lda + k0;
#pragma unroll 4
      for (int kk = lane; kk < kc; kk += 32) {
        const float av = a[kk];
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[r][n] = fmaf(av, Bs[kk][n], acc[r][n]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t m = m_base + r;
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      float v = warp_sum(acc[r][n]);
      if (lane == n && n < N && m < M) {
        float* c = C + m * ldc + n;
        float o = mask_of(epi(v, bias, n, relu), mask, ldm, m, n);
        *c = accumulate ? *c + o : o;
      }
    }
  }
}

// ------------------------------------------------------------------- tn ---
// grid (ceil(M/256), chunks): each thread owns column m and a K chunk; the
// chunk's partial C[m, 0:NB] goes to the workspace; the last chunk block of a
// column stripe folds the partials in chunk order.
template <int NB>
__global__ void __launch_bounds__(256) small_tn_kernel(int64_t M, int N, int64_t K, int64_t chunk,
                                                       const float* __restrict__ A, int64_t lda,
                                                       const float* __restrict__ B, int64_t ldb,
                                                       float* __restrict__ C, int64_t ldc,
                                                       const float* __restrict__ bias,
                                                       int accumulate, int relu, const float* __restrict__ mask, int64_t ldm,
                                                       unsigned* counters, float* partials) {
  constexpr int KT = 256;
  __shared__ float Bs[KT][NB];
  const int64_t m = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t k_begin = (int64_t)blockIdx.y * chunk;
  const int64_t k_end = K < k_begin + chunk ? K : k_begin + chunk;
  float acc[NB];
#pragma unroll
  for (int n = 0; n < NB; ++n) acc[n] = 0.f;
  for (int64_t k0 = k_begin; k0 < k_end; k0 += KT) {
    const int kt = (int)(k_end - k0 < KT ? k_end - k0 : KT);
    __syncthreads();
    for (int i = threadIdx.x; i < kt * NB; i += blockDim.x) {
      int kk = i / NB, n = i % NB;
      Bs[kk][n] = (n < N) ? B[(k0 + kk) * ldb + n] : 0.f;
    }
    __syncthreads();
    if (m < M) {
      const float* a = A + k0 * lda + m;
#pragma unroll 4
      for (int kk = 0; kk < kt; ++kk) {
        const float av = a[(int64_t)kk * lda];
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[n] = fmaf(av, Bs[kk][n], acc[n]);
      }
    }
  }
  float* part = partials + ((size_t)blockIdx.y * M) * NB;
  if (m < M) {
#pragma unroll
    for (int n = 0; n < NB; ++n) part[(size_t)m * NB + n] = acc[n];
  }
  __threadfence();
  __shared__ unsigned last;
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&counters[blockIdx.x], 1u) == gridDim.y - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (m < M) {
    float tot[NB];
#pragma unroll
    for (int n = 0; n < NB; ++n) tot[n] = 0.f;
    for (unsigned y = 0; y < gridDim.y; ++y) {
      const float* p = partials + ((size_t)y * M + m) * NB;
#pragma unroll
      for (int n = 0; n < NB; ++n) tot[n] += __ldcg(p + n);
    }
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      if (n < N) {
        float* c = C + m * ldc + n;
        float o = mask_of(epi(tot[n], bias, n, relu), mask, ldm, m, n);
        *c = accumulate ? *c + o : o;
      }
    }
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

// ------------------------------------------------------------------- nt ---
// C[m, n] = sum_k A[m,k] B[n,k], K <= 32: block = 256 columns n x ROWS rows m;
// thread keeps B[n, 0:K] in registers, rows of A staged in shared memory.
template <int KB>
__global__ void __launch_bounds__(256) small_nt_kernel(int64_t M, int64_t N, int K,
                                                       const float* __restrict__ A, int64_t lda,
                                                       const float* __restrict__ B, int64_t ldb,
                                                       float* __restrict__ C, int64_t ldc,
                                                       const float* __restrict__ bias,
                                                       int accumulate, int relu, const float* __restrict__ mask, int64_t ldm, int rows) {
  extern __shared__ float As[];  // [rows][KB]
  const int64_t n = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t m0 = (int64_t)blockIdx.y * rows;
  const int mr = (int)(M - m0 < rows ? M - m0 : rows);
  for (int i = threadIdx.x; i < mr * KB; i += blockDim.x) {
    int r = i / KB, k = i % KB;
    As[i] = (k < K) ? A[(m0 + r) * lda + k] : 0.f;
  }
  float b[KB];
#pragma unroll
  for (int k = 0; k < KB; ++k) b[k] = (n < N && k < K) ? B[n * ldb + k] : 0.f;
  const float bn = (bias && n < N) ? bias[n] : 0.f;
  __syncthreads();
  if (n >= N) return;
  for (int r = 0; r < mr; ++r) {
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < KB; ++k) v = fmaf(As[r * KB + k], b[k], v);
    v += bn;
    if (relu) v = fmaxf(0.f, v);
    v = mask_of(v, mask, ldm, m0 + r, n);
    float* c = C + (m0 + r) * ldc + n;
    *c = accumulate ? *c + v : v;
  }
}

// ----------------------------------------------------------------- nn4 ---
// nn with 128-bit loads: lane l reads A[m, k0+4(l+32j) .. +3] for RPW rows at
// once, and B is staged transposed, [NB][KCH+4], so that one 128-bit shared
// load of B serves RPW rows (4*RPW FMAs per load).  Needs K and lda
// multiples of 4 and a 16-byte aligned A.  Rows past M read row 0 (in
// bounds) and are not stored.
template <int NB, int RPW>
__global__ void __launch_bounds__(256, 2) small_nn4_kernel(int64_t M, int N, int64_t K,
                                                           const float* __restrict__ A, int64_t lda,
                                                           const float* __restrict__ B, int64_t ldb,
                                                           float* __restrict__ C, int64_t ldc,
                                                           const float* __restrict__ bias,
                                                           int accumulate, int relu, const float* __restrict__ mask, int64_t ldm) {
  constexpr int KCH = NB <= 16 ? 512 : 256, LDT = KCH + 4;
  __shared__ __align__(16) float Bt[NB * LDT];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t m_base = ((int64_t)blockIdx.x * 8 + warp) * RPW;
  const float* arow[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) arow[r] = A + (m_base + r < M ? m_base + r : 0) * lda;
  float acc[RPW][NB];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;

  for (int64_t k0 = 0; k0 < K; k0 += KCH) {
    const int kc = (int)(K - k0 < KCH ? K - k0 : KCH);
    __syncthreads();
    for (int i = threadIdx.x; i < kc * NB; i += blockDim.x) {
      const int kk = i / NB, n = i - kk * NB;
      Bt[n * LDT + kk] = (n < N) ? B[(k0 + kk) * ldb + n] : 0.f;
    }
    __syncthreads();
    const int nq = kc >> 2;
#pragma unroll 2
    for (int q = lane; q < nq; q += 32) {
      float4 a[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) a[r] = ld_stream4(arow[r] + k0 + 4 * q);
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float4 b = *reinterpret_cast<const float4*>(&Bt[n * LDT + 4 * q]);
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          acc[r][n] = fmaf(a[r].w, b.w, fmaf(a[r].z, b.z, fmaf(a[r].y, b.y, fmaf(a[r].x, b.x, acc[r][n]))));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t m = m_base + r;
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const float v = warp_sum(acc[r][n]);
      if (lane == n && n < N && m < M) {
        float* c = C + m * ldc + n;
        const float o = mask_of(epi(v, bias, n, relu), mask, ldm, m, n);
        *c = accumulate ? *c + o : o;
      }
    }
  }
}

// ---------------------------------------------------------------- nn4p ---
// nn4 with all of B^T resident in shared memory ([NB][K+4], staged once per
// block): a persistent grid of one 512-thread block per SM walks 64-row
// groups (12 warps x RPW rows), so B is read from global memory once per SM
// instead of once per row group.  Needs NB*(K+4)*4 bytes of shared memory.
// 12 warps: up to 170 registers a thread, 12 loads of 16 bytes in flight each.
// (Per float4 of A the kernel issues NB/4 shared loads and 4*NB FMAs per row;
// with N = 10 that is about half of HBM speed at 4 instructions a clock.)
constexpr int kNnpWarps = 12;
template <int NB, int RPW>
__global__ void __launch_bounds__(32 * kNnpWarps, 1) small_nn4p_kernel(int64_t M, int N, int64_t K,
                                                            const float* __restrict__ A, int64_t lda,
                                                            const float* __restrict__ B, int64_t ldb,
                                                            float* __restrict__ C, int64_t ldc,
                                                            const float* __restrict__ bias,
                                                            int accumulate, int relu, const float* __restrict__ mask, int64_t ldm) {
  extern __shared__ __align__(16) float Btp[];
  const int64_t ldt = K + 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (ldb == N && (((uintptr_t)B & 15) == 0) && (K * N) % 4 == 0) {
    const int64_t n4 = K * N / 4;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(B)[i];
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t e = 4 * i + c, kk = e / N, n = e - kk * N;
        Btp[n * ldt + kk] = vv[c];
      }
    }
    for (int64_t i = threadIdx.x; i < (int64_t)(NB - N) * K; i += blockDim.x) {
      const int64_t n = N + i / K, kk = i % K;
      Btp[n * ldt + kk] = 0.f;
    }
  } else {
    for (int64_t i = threadIdx.x; i < K * NB; i += blockDim.x) {
      const int64_t kk = i / NB, n = i - kk * NB;
      Btp[n * ldt + kk] = (n < N) ? B[kk * ldb + n] : 0.f;
    }
  }
  __syncthreads();
  const int64_t groups = (M + kNnpWarps * RPW - 1) / (kNnpWarps * RPW);
  const int nq = (int)(K >> 2);
  for (int64_t g = blockIdx.x; g < groups; g += gridDim.x) {
    const int64_t m_base = (g * kNnpWarps + warp) * RPW;
    const float* arow[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) arow[r] = A + (m_base + r < M ? m_base + r : 0) * lda;
    float acc[RPW][NB];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;
#pragma unroll 3
    for (int q = lane; q < nq; q += 32) {  // 3 trips unrolled: 12 loads of 16 B in flight a lane
      float4 a[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) a[r] = ld_stream4(arow[r] + 4 * q);
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float4 b = *reinterpret_cast<const float4*>(&Btp[n * ldt + 4 * q]);
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          acc[r][n] = fmaf(a[r].w, b.w, fmaf(a[r].z, b.z, fmaf(a[r].y, b.y, fmaf(a[r].x, b.x, acc[r][n]))));
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t m = m_base + r;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float v = warp_sum(acc[r][n]);
        if (lane == n && n < N && m < M) {
          float* c = C + m * ldc + n;
          const float o = mask_of(epi(v, bias, n, relu), mask, ldm, m, n);
          *c = accumulate ? *c + o : o;
        }
      }
    }
  }
}

// ----------------------------------------------------------------- tn4 ---
// tn with 128-bit loads: a block owns 128 columns m (lane l: m0+4l..+3) and a
// K chunk; its 8 warps take every 8th row k of the chunk.  The warps' sums
// fold through shared memory in a fixed tree (4+4, 2+2, 1+1); warp 0 writes
// the chunk partial and the stripe's last block folds the chunks in order.
// Needs M and lda multiples of 4, a 16-byte aligned A and NB <= 16.
template <int NB>
__global__ void __launch_bounds__(256, 2) small_tn4_kernel(int64_t M, int N, int64_t K, int64_t chunk,
                                                           const float* __restrict__ A, int64_t lda,
                                                           const float* __restrict__ B, int64_t ldb,
                                                           float* __restrict__ C, int64_t ldc,
                                                           const float* __restrict__ bias,
                                                           int accumulate, int relu, const float* __restrict__ mask, int64_t ldm,
                                                           unsigned* counters, float* partials) {
  constexpr int KT = NB <= 12 ? 512 : 256;
  __shared__ __align__(16) float Bs[KT * NB];
  __shared__ float fold[2][4 * NB][32];
  __shared__ unsigned last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t m = (int64_t)blockIdx.x * 128 + 4 * lane;
  const bool mv = m < M;
  const int64_t k_begin = (int64_t)blockIdx.y * chunk;
  const int64_t k_end = K < k_begin + chunk ? K : k_begin + chunk;
  float acc[4][NB];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int n = 0; n < NB; ++n) acc[c][n] = 0.f;

  for (int64_t k0 = k_begin; k0 < k_end; k0 += KT) {
    const int kt = (int)(k_end - k0 < KT ? k_end - k0 : KT);
    __syncthreads();
    if (ldb == N && (kt * N) % 4 == 0 && ((((uintptr_t)(B + k0 * ldb)) & 15) == 0)) {
      // the stage's rows are one contiguous run: 128-bit loads, all in
      // flight, scattered into the NB-wide rows (pad columns zeroed)
      const float4* src = reinterpret_cast<const float4*>(B + k0 * ldb);
      for (int i = threadIdx.x; i < kt * N / 4; i += blockDim.x) {
        const float4 v = src[i];
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int e = 4 * i + c, kk = e / N;
          Bs[kk * NB + (e - kk * N)] = vv[c];
        }
      }
      if (N < NB)
        for (int i = threadIdx.x; i < kt * (NB - N); i += blockDim.x) {
          const int kk = i / (NB - N);
          Bs[kk * NB + N + (i - kk * (NB - N))] = 0.f;
        }
    } else {
#pragma unroll 4
      for (int i = threadIdx.x; i < kt * NB; i += blockDim.x) {
        const int kk = i / NB, n = i - kk * NB;
        Bs[i] = (n < N) ? B[(k0 + kk) * ldb + n] : 0.f;
      }
    }
    __syncthreads();
    if (mv) {
#pragma unroll 8
      for (int kk = warp; kk < kt; kk += 8) {
        const float4 a = ld_stream4(A + (k0 + kk) * lda + m);
#pragma unroll
        for (int q = 0; q < NB / 4; ++q) {
          const float4 b = *reinterpret_cast<const float4*>(&Bs[kk * NB + 4 * q]);
          const float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[0][4 * q + i] = fmaf(a.x, bb[i], acc[0][4 * q + i]);
            acc[1][4 * q + i] = fmaf(a.y, bb[i], acc[1][4 * q + i]);
            acc[2][4 * q + i] = fmaf(a.z, bb[i], acc[2][4 * q + i]);
            acc[3][4 * q + i] = fmaf(a.w, bb[i], acc[3][4 * q + i]);
          }
        }
      }
    }
  }
  // fixed-order tree over the 8 warps (w += w + s for s = 4, 2, 1), through a
  // two-warp buffer: warps 4,5 then 6,7 for s = 4
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int s = step < 2 ? 4 : (step == 2 ? 2 : 1);
    const int lo = step == 1 ? 2 : 0;      // receiving warps lo, lo+1 (s = 4)
    __syncthreads();
    const int src = warp - s;
    const bool sends = (s == 4) ? (src == lo || src == lo + 1) : (warp >= s && warp < 2 * s);
    if (sends) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int n = 0; n < NB; ++n) fold[src - lo][c * NB + n][lane] = acc[c][n];
    }
    __syncthreads();
    const bool takes = (s == 4) ? (warp == lo || warp == lo + 1) : (warp < s);
    if (takes) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int n = 0; n < NB; ++n) acc[c][n] += fold[warp - lo][c * NB + n][lane];
    }
  }
  if (warp == 0 && mv) {
    float* part = partials + ((size_t)blockIdx.y * M + m) * NB;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int n = 0; n < NB; ++n) part[c * NB + n] = acc[c][n];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&counters[blockIdx.x], 1u) == gridDim.y - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int64_t mb = (int64_t)blockIdx.x * 128;
  for (int o = threadIdx.x; o < 128 * NB; o += blockDim.x) {
    const int col = o / NB, n = o - col * NB;
    const int64_t mm = mb + col;
    if (mm >= M || n >= N) continue;
    float tot = 0.f;
    for (unsigned y = 0; y < gridDim.y; ++y) tot += __ldcg(&partials[((size_t)y * M + mm) * NB + n]);
    float* c = C + mm * ldc + n;
    const float v = mask_of(epi(tot, bias, n, relu), mask, ldm, mm, n);
    *c = accumulate ? *c + v : v;
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

// ----------------------------------------------------------------- nt4 ---
// nt with 128-bit stores: a thread owns 4 consecutive columns n and keeps
// their B rows in registers; rows of A are staged in shared memory and read
// as 128-bit broadcasts.  Per output the k order is the nt kernel's.  Needs
// N and ldc multiples of 4, a 16-byte aligned C and KB <= 16.
template <int KB>
__global__ void __launch_bounds__(256) small_nt4_kernel(int64_t M, int64_t N, int K,
                                                        const float* __restrict__ A, int64_t lda,
                                                        const float* __restrict__ B, int64_t ldb,
                                                        float* __restrict__ C, int64_t ldc,
                                                        const float* __restrict__ bias,
                                                        int accumulate, int relu, const float* __restrict__ mask, int64_t ldm, int rows) {
  extern __shared__ __align__(16) float As4[];  // [rows][KB]
  const int64_t n = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
  const int64_t m0 = (int64_t)blockIdx.y * rows;
  const int mr = (int)(M - m0 < rows ? M - m0 : rows);
  for (int i = threadIdx.x; i < mr * KB; i += blockDim.x) {
    const int r = i / KB, k = i - r * KB;
    As4[i] = (k < K) ? A[(m0 + r) * lda + k] : 0.f;
  }
  float b[4][KB];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int k = 0; k < KB; ++k) b[c][k] = (n + c < N && k < K) ? B[(n + c) * ldb + k] : 0.f;
  float bn[4] = {0.f, 0.f, 0.f, 0.f};
  if (bias && n < N) {
#pragma unroll
    for (int c = 0; c < 4; ++c) bn[c] = bias[n + c];
  }
  __syncthreads();
  if (n >= N) return;
  const bool mask4 = mask && (ldm % 4 == 0) && ((((uintptr_t)mask) & 15) == 0);
  if (!mask4) {  // no mask operand: one row at a time keeps the registers (occupancy) low
    for (int r = 0; r < mr; ++r) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < KB / 4; ++q) {
        const float4 a = *reinterpret_cast<const float4*>(&As4[r * KB + 4 * q]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[c] = fmaf(a.x, b[c][4 * q], v[c]);
          v[c] = fmaf(a.y, b[c][4 * q + 1], v[c]);
          v[c] = fmaf(a.z, b[c][4 * q + 2], v[c]);
          v[c] = fmaf(a.w, b[c][4 * q + 3], v[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        v[c] += bn[c];
        if (relu) v[c] = fmaxf(0.f, v[c]);
        if (mask) v[c] = mask_of(v[c], mask, ldm, m0 + r, n + c);
      }
      float4* c4 = reinterpret_cast<float4*>(C + (m0 + r) * ldc + n);
      float4 o = make_float4(v[0], v[1], v[2], v[3]);
      if (accumulate) {
        const float4 q = *c4;
        o.x = q.x + o.x; o.y = q.y + o.y; o.z = q.z + o.z; o.w = q.w + o.w;
      }
      *c4 = o;
    }
    return;
  }
  // with a mask: rows in groups of 4, the group's mask vectors loaded before
  // any of its rows is computed, so 4 loads of 16 bytes are in flight a thread
  for (int r0 = 0; r0 < mr; r0 += 4) {
    float4 mk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      mk[i] = (r0 + i < mr) ? __ldg(reinterpret_cast<const float4*>(mask + (m0 + r0 + i) * ldm + n))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + i;
      if (r >= mr) break;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < KB / 4; ++q) {
        const float4 a = *reinterpret_cast<const float4*>(&As4[r * KB + 4 * q]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[c] = fmaf(a.x, b[c][4 * q], v[c]);
          v[c] = fmaf(a.y, b[c][4 * q + 1], v[c]);
          v[c] = fmaf(a.z, b[c][4 * q + 2], v[c]);
          v[c] = fmaf(a.w, b[c][4 * q + 3], v[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        v[c] += bn[c];
        if (relu) v[c] = fmaxf(0.f, v[c]);
      }
      v[0] = __fmul_rn(v[0], mk[i].x > 0.f ? 1.f : 0.f);
      v[1] = __fmul_rn(v[1], mk[i].y > 0.f ? 1.f : 0.f);
      v[2] = __fmul_rn(v[2], mk[i].z > 0.f ? 1.f : 0.f);
      v[3] = __fmul_rn(v[3], mk[i].w > 0.f ? 1.f : 0.f);
      float4* c4 = reinterpret_cast<float4*>(C + (m0 + r) * ldc + n);
      float4 o = make_float4(v[0], v[1], v[2], v[3]);
      if (accumulate) {
        const float4 q = *c4;
        o.x = q.x + o.x; o.y = q.y + o.y; o.z = q.z + o.z; o.w = q.w + o.w;
      }
      *c4 = o;
    }
  }
}

// workspace for tn partials and counters (grown outside capture, never freed)
std::mutex g_small_mu;
struct SmallWs {
  void* ptr = nullptr;
  size_t bytes = 0;
};
SmallWs g_small_ws[64];
std::vector<void*>* g_small_retired = nullptr;

int small_workspace(size_t bytes, void** out, cudaStream_t st) {
  int dev = 0;
  TL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return TL_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_small_mu);
  SmallWs& w = g_small_ws[dev];
  if (w.bytes < bytes) {
    cudaStreamCaptureStatus cs;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
      return TL_ERR_UNSUPPORTED;
    size_t want = bytes + bytes / 4 + 4096;
    void* p = nullptr;
    TL_CUDA_TRY(cudaMalloc(&p, want));
    TL_CUDA_TRY(cudaMemset(p, 0, 4096));  // counters start at zero; kernels reset them
    if (w.ptr) {
      if (!g_small_retired) g_small_retired = new std::vector<void*>();
      g_small_retired->push_back(w.ptr);
    }
    w.ptr = p;
    w.bytes = want;
  }
  *out = w.ptr;
  return TL_OK;
}

template <template <int> class F, typename... Args>
int dispatch_nb(int n, Args... args) {
  if (n <= 4) return F<4>::run(args...);
  if (n <= 8) return F<8>::run(args...);
  if (n <= 12) return F<12>::run(args...);
  if (n <= 16) return F<16>::run(args...);
  if (n <= 24) return F<24>::run(args...);
  return F<32>::run(args...);
}

template <int NB>
struct RunNN {
  static int run(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu, const float* mask, int64_t ldm,
                 cudaStream_t st) {
    constexpr int RPW = NB <= 12 ? 4 : 2;   // nn4 / nn kernels (8 warps a block)
    constexpr int RPWP = RPW;               // persistent nn4p (12 warps a block)
    const int64_t blocks = (M + 8 * RPW - 1) / (8 * RPW);
    if (blocks > INT32_MAX) return TL_ERR_UNSUPPORTED;
    if (K % 4 == 0 && lda % 4 == 0 && aligned16(A)) {
      if constexpr (NB <= 16) {
        const size_t smem = (size_t)NB * (K + 4) * 4;
        if (smem <= 200 * 1024) {
          auto kern = small_nn4p_kernel<NB, RPWP>;
          TL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
          const int64_t groups = (M + kNnpWarps * RPWP - 1) / (kNnpWarps * RPWP);
          const unsigned grid = (unsigned)(groups < sm_count() ? groups : sm_count());
          kern<<<grid, 32 * kNnpWarps, smem, st>>>(M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm);
          return after_launch();
        }
      }
      small_nn4_kernel<NB, RPW><<<(unsigned)blocks, 256, 0, st>>>(M, N, K, A, lda, B, ldb, C, ldc,
                                                                  bias, acc, relu, mask, ldm);
      return after_launch();
    }
    small_nn_kernel<NB, RPW><<<(unsigned)blocks, 256, 0, st>>>(M, N, K, A, lda, B, ldb, C, ldc,
                                                                bias, acc, relu, mask, ldm);
    return after_launch();
  }
};

template <int NB>
struct RunTN {
  static int run(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu, const float* mask, int64_t ldm,
                 cudaStream_t st) {
    if constexpr (NB <= 16) {
      if (M % 4 == 0 && lda % 4 == 0 && aligned16(A)) return run4(M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm, st);
    }
    const unsigned gx = (unsigned)((M + 255) / 256);
    if (gx > 1024) return TL_ERR_UNSUPPORTED;
    int64_t want = (4LL * sm_count() + gx - 1) / gx;
    int64_t maxy = (K + 255) / 256;
    if (want > maxy) want = maxy;
    if (want < 1) want = 1;
    const int64_t chunk = ((K + want - 1) / want + 255) / 256 * 256;
    const unsigned gy = (unsigned)((K + chunk - 1) / chunk);
    void* ws = nullptr;
    TL_TRY(small_workspace(4096 + (size_t)gy * M * NB * 4, &ws, st));
    small_tn_kernel<NB><<<dim3(gx, gy), 256, 0, st>>>(M, N, K, chunk, A, lda, B, ldb, C, ldc, bias,
                                                       acc, relu, mask, ldm, (unsigned*)ws,
                                                       (float*)((char*)ws + 4096));
    return after_launch();
  }
  static int run4(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* B,
                  int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu, const float* mask, int64_t ldm,
                  cudaStream_t st) {
    const unsigned gx = (unsigned)((M + 127) / 128);
    if (gx > 1024) return TL_ERR_UNSUPPORTED;
    // at most one wave of two resident blocks per SM; chunks of whole 512-row stages
    int64_t want = 2LL * sm_count() / gx;
    const int64_t maxy = (K + 511) / 512;
    if (want > maxy) want = maxy;
    if (want < 1) want = 1;
    const int64_t chunk = ((K + want - 1) / want + 511) / 512 * 512;
    const unsigned gy = (unsigned)((K + chunk - 1) / chunk);
    void* ws = nullptr;
    TL_TRY(small_workspace(4096 + (size_t)gy * M * NB * 4, &ws, st));
    small_tn4_kernel<NB><<<dim3(gx, gy), 256, 0, st>>>(M, N, K, chunk, A, lda, B, ldb, C, ldc, bias,
                                                        acc, relu, mask, ldm, (unsigned*)ws,
                                                        (float*)((char*)ws + 4096));
    return after_launch();
  }
};

template <int KB>
struct RunNT {
  static int run(int64_t M, int64_t N, int K, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu, const float* mask, int64_t ldm,
                 cudaStream_t st) {
    const int rows = 64;
    if constexpr (KB <= 16) {
      const int64_t gy4 = (M + rows - 1) / rows;
      if (N % 4 == 0 && ldc % 4 == 0 && aligned16(C) && gy4 <= 65535) {
        const unsigned gx4 = (unsigned)((N + 1023) / 1024);
        small_nt4_kernel<KB><<<dim3(gx4, (unsigned)gy4), 256, rows * KB * 4, st>>>(
            M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm, rows);
        return after_launch();
      }
    }
    const unsigned gx = (unsigned)((N + 255) / 256);
    const int64_t gy = (M + rows - 1) / rows;
    if (gy > 65535) return small_nt_launch_wide(M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm, st);
    small_nt_kernel<KB><<<dim3(gx, (unsigned)gy), 256, rows * KB * 4, st>>>(
        M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm, rows);
    return after_launch();
  }
  // very tall outputs: more rows per block so the grid's y extent fits
  static int small_nt_launch_wide(int64_t M, int64_t N, int K, const float* A, int64_t lda,
                                  const float* B, int64_t ldb, float* C, int64_t ldc,
                                  const float* bias, int acc, int relu, const float* mask, int64_t ldm, cudaStream_t st) {
    const int64_t rows = (M + 65534) / 65535;
    if (rows * KB * 4 > 48 * 1024) return TL_ERR_UNSUPPORTED;
    const unsigned gx = (unsigned)((N + 255) / 256);
    const unsigned gy = (unsigned)((M + rows - 1) / rows);
    small_nt_kernel<KB><<<dim3(gx, gy), 256, (size_t)rows * KB * 4, st>>>(
        M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, mask, ldm, (int)rows);
    return after_launch();
  }
};

}  // namespace

// Returns TL_ERR_UNSUPPORTED when no skinny kernel applies.
int gemm_small(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
               const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
               int accumulate, int epilogue, const float* mask, int64_t ldm, cudaStream_t st) {
  const int relu = epilogue == TL_EPI_RELU;
  if (N <= SMALL && !ta && !tb)
    return dispatch_nb<RunNN>((int)N, M, (int)N, K, A, lda, B, ldb, C, ldc, bias, accumulate, relu,
                              mask, ldm, st);
  if (N <= SMALL && ta && !tb)
    return dispatch_nb<RunTN>((int)N, M, (int)N, K, A, lda, B, ldb, C, ldc, bias, accumulate, relu,
                              mask, ldm, st);
  if (K <= SMALL && !ta && tb)
    return dispatch_nb<RunNT>((int)K, M, N, (int)K, A, lda, B, ldb, C, ldc, bias, accumulate, relu,
                              mask, ldm, st);
  return TL_ERR_UNSUPPORTED;
}

// Products this small keep the tiled kernel, whose per-output k order is
// sequential like the reference's (tiny programs compare with atol 1e-8).
bool gemm_small_ok(int ta, int tb, int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (N <= SMALL && !tb && M * K >= (1 << 16)) return true;   // nn and tn
  if (K <= SMALL && !ta && tb && M * N >= (1 << 16)) return true;  // nt
  return false;
}

}  // namespace tl
