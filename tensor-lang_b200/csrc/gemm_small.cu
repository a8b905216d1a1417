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
// All accumulate in fp32 with FMA; epilogue: + bias[n], relu, accumulate.
#include <mutex>
#include <vector>

#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int SMALL = 32;

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
                                                       int accumulate, int relu) {
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
        float o = epi(v, bias, n, relu);
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
                                                       int accumulate, int relu,
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
        float o = epi(tot[n], bias, n, relu);
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
                                                       int accumulate, int relu, int rows) {
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
    float* c = C + (m0 + r) * ldc + n;
    *c = accumulate ? *c + v : v;
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
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu,
                 cudaStream_t st) {
    constexpr int RPW = NB <= 12 ? 4 : 2;
    const int64_t blocks = (M + 8 * RPW - 1) / (8 * RPW);
    if (blocks > INT32_MAX) return TL_ERR_UNSUPPORTED;
    small_nn_kernel<NB, RPW><<<(unsigned)blocks, 256, 0, st>>>(M, N, K, A, lda, B, ldb, C, ldc,
                                                                bias, acc, relu);
    return after_launch();
  }
};

template <int NB>
struct RunTN {
  static int run(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu,
                 cudaStream_t st) {
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
                                                       acc, relu, (unsigned*)ws,
                                                       (float*)((char*)ws + 4096));
    return after_launch();
  }
};

template <int KB>
struct RunNT {
  static int run(int64_t M, int64_t N, int K, const float* A, int64_t lda, const float* B,
                 int64_t ldb, float* C, int64_t ldc, const float* bias, int acc, int relu,
                 cudaStream_t st) {
    const int rows = 64;
    const unsigned gx = (unsigned)((N + 255) / 256);
    const int64_t gy = (M + rows - 1) / rows;
    if (gy > 65535) return small_nt_launch_wide(M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, st);
    small_nt_kernel<KB><<<dim3(gx, (unsigned)gy), 256, rows * KB * 4, st>>>(
        M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, rows);
    return after_launch();
  }
  // very tall outputs: more rows per block so the grid's y extent fits
  static int small_nt_launch_wide(int64_t M, int64_t N, int K, const float* A, int64_t lda,
                                  const float* B, int64_t ldb, float* C, int64_t ldc,
                                  const float* bias, int acc, int relu, cudaStream_t st) {
    const int64_t rows = (M + 65534) / 65535;
    if (rows * KB * 4 > 48 * 1024) return TL_ERR_UNSUPPORTED;
    const unsigned gx = (unsigned)((N + 255) / 256);
    const unsigned gy = (unsigned)((M + rows - 1) / rows);
    small_nt_kernel<KB><<<dim3(gx, gy), 256, (size_t)rows * KB * 4, st>>>(
        M, N, K, A, lda, B, ldb, C, ldc, bias, acc, relu, (int)rows);
    return after_launch();
  }
};

}  // namespace

// Returns TL_ERR_UNSUPPORTED when no skinny kernel applies.
int gemm_small(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
               const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
               int accumulate, int epilogue, cudaStream_t st) {
  const int relu = epilogue == TL_EPI_RELU;
  if (N <= SMALL && !ta && !tb)
    return dispatch_nb<RunNN>((int)N, M, (int)N, K, A, lda, B, ldb, C, ldc, bias, accumulate, relu, st);
  if (N <= SMALL && ta && !tb)
    return dispatch_nb<RunTN>((int)N, M, (int)N, K, A, lda, B, ldb, C, ldc, bias, accumulate, relu, st);
  if (K <= SMALL && !ta && tb)
    return dispatch_nb<RunNT>((int)K, M, N, (int)K, A, lda, B, ldb, C, ldc, bias, accumulate, relu, st);
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
