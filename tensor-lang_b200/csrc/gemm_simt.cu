// Tiled float32 GEMM on the CUDA cores.
//
// This is the path for products the tensor-core kernel does not take
// (leading dimensions that are not a multiple of 4 floats, tiny or skinny
// shapes such as the 10-wide output layer) and the fp32 cross-check of the
// tensor-core path.  It replaces the reference's one-thread-per-output
// matmul (kernel_generator.py:501-525) and linear (:1584-1661) kernels,
// which have no data reuse.
//
// 128x128 block tile, 8-deep k slices double-buffered in shared memory,
// 8x8 outputs per thread (two 4x4 quadrants, 64 apart, so shared-memory
// reads are conflict-free float4s), fp32 FMA accumulation.
#include "tl_common.cuh"

namespace tl {

int gemm_tc(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
            const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate,
            int epilogue, const float* mask, int64_t ldm, const void* a_pair, const void* b_pair,
            cudaStream_t st);
bool gemm_uses_pairs(int ta, int tb, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb);
int gemm_tc_plan(int64_t M, int64_t N, int64_t K, int* out);
int64_t pair_bytes(int64_t rows, int64_t cols, int layout);
int pair_prepare(const float* X, int64_t ld, int64_t rows, int64_t cols, void* kmajor,
                 int k_lo_first, void* mnmajor, int m_lo_first, cudaStream_t st);
size_t pair_colsum_scratch_bytes(int64_t rows, int64_t cols);
int pair_prepare_colsum(const float* X, int64_t ld, int64_t rows, int64_t cols, void* kmajor,
                        int k_lo_first, void* mnmajor, int m_lo_first, float* colsum,
                        void* scratch, size_t scratch_bytes, cudaStream_t st);
bool gemm_tc_ok(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                const float* B, int64_t ldb, const float* C, int64_t ldc);
void gemm_set_split_mode(int mode);
int gemm_set_scheme(int scheme);
int gemm_set_cta_pair(int enable);
int gemm_set_tile_dynamic(int enable);
int gemm_set_tma_store(int mode);
int gemm_small(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
               const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
               int accumulate, int epilogue, const float* mask, int64_t ldm, cudaStream_t st);
bool gemm_small_ok(int ta, int tb, int64_t M, int64_t N, int64_t K);

namespace {

constexpr int BM = 128, BN = 128, BK = 8;
bool g_force_simt = false;

template <int TA, int TB>
__global__ void __launch_bounds__(256) sgemm_kernel(int64_t M, int64_t N, int64_t K,
                                                    const float* __restrict__ A, int64_t lda,
                                                    const float* __restrict__ B, int64_t ldb,
                                                    float* __restrict__ C, int64_t ldc,
                                                    const float* __restrict__ bias, int accumulate,
                                                    int epilogue, const float* __restrict__ mask,
                                                    int64_t ldm) {
  __shared__ __align__(16) float As[2][BK][BM + 4];
  __shared__ __align__(16) float Bs[2][BK][BN + 4];
  const int t = threadIdx.x;
  const int tx = t & 15, ty = t >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  float ra[4], rb[4];
  // global -> register staging of one k-slice
  auto load_slice = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t m, k;
      if (TA) {  // A stored [K][M]: contiguous along m
        k = k0 + (t >> 5);
        m = m0 + (t & 31) * 4 + i;
        ra[i] = (m < M && k < K) ? A[k * lda + m] : 0.f;
      } else {  // A stored [M][K]: contiguous along k
        m = m0 + (t >> 1);
        k = k0 + (t & 1) * 4 + i;
        ra[i] = (m < M && k < K) ? A[m * lda + k] : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t n, k;
      if (TB) {  // B stored [N][K]: contiguous along k
        n = n0 + (t >> 1);
        k = k0 + (t & 1) * 4 + i;
        rb[i] = (n < N && k < K) ? B[n * ldb + k] : 0.f;
      } else {  // B stored [K][N]: contiguous along n
        k = k0 + (t >> 5);
        n = n0 + (t & 31) * 4 + i;
        rb[i] = (n < N && k < K) ? B[k * ldb + n] : 0.f;
      }
    }
  };
  auto store_slice = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (TA) As[buf][t >> 5][(t & 31) * 4 + i] = ra[i];
      else As[buf][(t & 1) * 4 + i][t >> 1] = ra[i];
      if (TB) Bs[buf][(t & 1) * 4 + i][t >> 1] = rb[i];
      else Bs[buf][t >> 5][(t & 31) * 4 + i] = rb[i];
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int64_t nk = (K + BK - 1) / BK;
  load_slice(0);
  store_slice(0);
  __syncthreads();
  for (int64_t kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) load_slice((kt + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][64 + tx * 4]);
      float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < nk) {
      store_slice(cur ^ 1);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int64_t m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= N) continue;
      float v = acc[i][j];
      if (bias) v += bias[n];
      if (epilogue == TL_EPI_RELU) v = fmaxf(0.f, v);
      if (mask) v = __fmul_rn(v, mask[m * ldm + n] > 0.f ? 1.f : 0.f);
      float* c = C + m * ldc + n;
      *c = accumulate ? *c + v : v;
    }
  }
}

}  // namespace

int gemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
              const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias,
              int accumulate, int epilogue, const float* mask, int64_t ldm, cudaStream_t st) {
  dim3 grid(ceil_div_u(N, BN), ceil_div_u(M, BM));
  if (grid.y > 65535) return TL_ERR_UNSUPPORTED;
#define TL_SG(a, b) \
  sgemm_kernel<a, b><<<grid, 256, 0, st>>>(M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate, epilogue, \
                                           mask, ldm)
  if (!ta && !tb) TL_SG(0, 0);
  else if (!ta && tb) TL_SG(0, 1);
  else if (ta && !tb) TL_SG(1, 0);
  else TL_SG(1, 1);
#undef TL_SG
  return after_launch();
}

}  // namespace tl

extern "C" {

int tl_gemm_pairs(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, const float* A,
                  int64_t lda, const void* a_pair, const float* B, int64_t ldb, const void* b_pair,
                  float* C, int64_t ldc, const float* bias, int accumulate, int epilogue,
                  const float* mask, int64_t ldm, void* stream) {
  if (M <= 0 || N <= 0 || !C) return TL_ERR_INVALID_ARG;
  if (K > 0 && (!A || !B)) return TL_ERR_INVALID_ARG;
  if (mask && ldm < N) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  if (!tl::g_force_simt && tl::gemm_tc_ok(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc))
    return tl::gemm_tc(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate,
                       epilogue, mask, ldm, a_pair, b_pair, st);
  if (K > 0 && tl::gemm_small_ok(trans_a, trans_b, M, N, K)) {
    int s = tl::gemm_small(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate,
                           epilogue, mask, ldm, st);
    if (s != TL_ERR_UNSUPPORTED) return s;
  }
  return tl::gemm_simt(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate,
                       epilogue, mask, ldm, st);
}

int tl_gemm_masked(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, const float* A,
                   int64_t lda, const float* B, int64_t ldb, float* C, int64_t ldc,
                   const float* bias, int accumulate, int epilogue, const float* mask,
                   int64_t ldm, void* stream) {
  return tl_gemm_pairs(trans_a, trans_b, M, N, K, A, lda, nullptr, B, ldb, nullptr, C, ldc, bias,
                       accumulate, epilogue, mask, ldm, stream);
}

int tl_gemm_uses_pairs(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, int64_t lda,
                       int64_t ldb) {
  return (!tl::g_force_simt && tl::gemm_uses_pairs(trans_a, trans_b, M, N, K, lda, ldb)) ? 1 : 0;
}

int64_t tl_gemm_pair_bytes(int64_t rows, int64_t cols, int layout) {
  return tl::pair_bytes(rows, cols, layout);
}

int tl_gemm_pair_prepare(const float* X, int64_t ld, int64_t rows, int64_t cols, void* kmajor,
                         int kmajor_lo_first, void* mnmajor, int mnmajor_lo_first, void* stream) {
  if (!X || rows <= 0 || cols <= 0 || ld < cols || (!kmajor && !mnmajor)) return TL_ERR_INVALID_ARG;
  if ((((uintptr_t)kmajor) & 15) || (((uintptr_t)mnmajor) & 15)) return TL_ERR_INVALID_ARG;
  return tl::pair_prepare(X, ld, rows, cols, kmajor, kmajor_lo_first, mnmajor, mnmajor_lo_first,
                          tl::stream_or_default(stream));
}

size_t tl_gemm_pair_colsum_scratch_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return tl::pair_colsum_scratch_bytes(rows, cols);
}

int tl_gemm_pair_prepare_colsum(const float* X, int64_t ld, int64_t rows, int64_t cols,
                                void* kmajor, int kmajor_lo_first, void* mnmajor,
                                int mnmajor_lo_first, float* colsum, void* scratch,
                                size_t scratch_bytes, void* stream) {
  if (!X || !colsum || !scratch || rows <= 0 || cols <= 0 || ld < cols || (!kmajor && !mnmajor))
    return TL_ERR_INVALID_ARG;
  if ((((uintptr_t)kmajor) & 15) || (((uintptr_t)mnmajor) & 15) || (((uintptr_t)scratch) & 7))
    return TL_ERR_INVALID_ARG;
  return tl::pair_prepare_colsum(X, ld, rows, cols, kmajor, kmajor_lo_first, mnmajor,
                                 mnmajor_lo_first, colsum, scratch, scratch_bytes,
                                 tl::stream_or_default(stream));
}

int tl_gemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
            const float* B, int64_t ldb, float* C, int64_t ldc, const float* bias, int accumulate,
            int epilogue, void* stream) {
  return tl_gemm_masked(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc, bias, accumulate,
                        epilogue, nullptr, 0, stream);
}

int tl_gemm_path(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, const float* A,
                 int64_t lda, const float* B, int64_t ldb, const float* C, int64_t ldc) {
  if (!tl::g_force_simt && tl::gemm_tc_ok(trans_a, trans_b, M, N, K, A, lda, B, ldb, C, ldc))
    return 0;
  return 1;
}

int tl_gemm_tc_plan(int64_t M, int64_t N, int64_t K, int* plan) {
  return tl::gemm_tc_plan(M, N, K, plan);
}

int tl_gemm_force_simt(int force) {
  if (force < 0 || force > 2) return TL_ERR_INVALID_ARG;
  tl::g_force_simt = force == 1;
  tl::gemm_set_split_mode(force == 2 ? 1 : 0);
  return TL_OK;
}

int tl_gemm_set_cta_pair(int enable, int* previous) {
  if (enable != 0 && enable != 1) return TL_ERR_INVALID_ARG;
  const int prev = tl::gemm_set_cta_pair(enable);
  if (previous) *previous = prev;
  return TL_OK;
}

int tl_gemm_set_tile_schedule(int dynamic, int* previous) {
  if (dynamic < 0 || dynamic > 2) return TL_ERR_INVALID_ARG;
  const int prev = tl::gemm_set_tile_dynamic(dynamic);
  if (previous) *previous = prev;
  return TL_OK;
}

int tl_gemm_set_store_path(int tma, int* previous) {
  if (tma < 0 || tma > 1) return TL_ERR_INVALID_ARG;
  const int prev = tl::gemm_set_tma_store(tma);
  if (previous) *previous = prev;
  return TL_OK;
}

int tl_gemm_set_scheme(int scheme, int* previous) {
  const int prev = tl::gemm_set_scheme(scheme);
  if (prev < 0) return TL_ERR_INVALID_ARG;
  if (previous) *previous = prev;
  return TL_OK;
}

}  // extern "C"
