// The classifier head of a training step in one pass over its input.
//
// A linear layer with a few outputs followed by a row softmax and
// cross_entropy (kernel_generator.py:1584-1661, :564-640, :1816-1885), and
// the backward of that chain (autograd.py:691-704 then :563-580, and the
// linear VJP :619-646 with the relu mask of the layer below, autograd.py:
// 540-544), run unfused as five kernels that each stream the [M, K] input or
// the [M, N] logits: the skinny forward product, softmax, the chained
// cross_entropy/softmax VJP, the skinny dX product with its relu-mask
// epilogue.  Here one warp takes RPW rows at a time and does all of it:
//
//   z  = A @ W + b                      (A [M, K] read once from DRAM)
//   p  = softmax(z)                     per row, in registers
//   dp = (p - t) / divisor * up         (the cross_entropy VJP)
//   dz = dp * p - p * sum(dp * p)       (the softmax VJP)
//   dx = (dz @ W^T) * (mask > 0)        (the mask is the layer's relu output)
//
// The loss itself stays with the loss kernel (it reads p).  Every value is
// computed in exactly the order of the unfused kernels -- the forward
// product's per-lane k order and warp fold (small_nn4p_kernel), softmax_rows_warp's
// fold, softmax_bwd_warp's double fold, small_nt4_kernel's per-column chain
// over the zero-padded classes and its bias and mask steps -- so the fused
// step is bit-identical to the unfused one.
#include <math.h>

#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int kHeadWarps = 12;

template <int NB, int RPW>
__global__ void __launch_bounds__(32 * kHeadWarps, 1)
    head_ce_kernel(int64_t M, int N, int64_t K, const float* __restrict__ A, int64_t lda,
                   const float* __restrict__ W, int64_t ldw, const float* __restrict__ bias,
                   const float* __restrict__ tgt, int onehot, const float* __restrict__ upstream,
                   float divisor, float* __restrict__ z, float* __restrict__ p,
                   float* __restrict__ dp, float* __restrict__ dz, float* __restrict__ dx,
                   int64_t lddx, const float* __restrict__ mask, int64_t ldm) {
  extern __shared__ __align__(16) float Wt[];  // W^T, [NB][K + 4], classes past N zero
  const int64_t ldt = K + 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // stage W^T (the forward product's B operand, as small_nn4p_kernel stages it)
  if (ldw == N && (((uintptr_t)W & 15) == 0) && (K * N) % 4 == 0) {
    const int64_t n4 = K * N / 4;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(W)[i];
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t e = 4 * i + c, kk = e / N, n = e - kk * N;
        Wt[n * ldt + kk] = vv[c];
      }
    }
    for (int64_t i = threadIdx.x; i < (int64_t)(NB - N) * K; i += blockDim.x) {
      const int64_t n = N + i / K, kk = i % K;
      Wt[n * ldt + kk] = 0.f;
    }
  } else {
    for (int64_t i = threadIdx.x; i < K * NB; i += blockDim.x) {
      const int64_t kk = i / NB, n = i - kk * NB;
      Wt[n * ldt + kk] = (n < N) ? W[kk * ldw + n] : 0.f;
    }
  }
  __syncthreads();
  const float up = upstream ? upstream[0] : 1.0f;
  const int64_t groups = (M + kHeadWarps * RPW - 1) / (kHeadWarps * RPW);
  const int nq = (int)(K >> 2);
  for (int64_t g = blockIdx.x; g < groups; g += gridDim.x) {
    const int64_t m_base = (g * kHeadWarps + warp) * RPW;
    const float* arow[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) arow[r] = A + (m_base + r < M ? m_base + r : 0) * lda;

    // ---- z = A @ W + b: small_nn4p_kernel's per-lane order and warp fold
    float acc[RPW][NB];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int n = 0; n < NB; ++n) acc[r][n] = 0.f;
#pragma unroll 3
    for (int q = lane; q < nq; q += 32) {
      float4 a[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) a[r] = ld_stream4(arow[r] + 4 * q);
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float4 b = *reinterpret_cast<const float4*>(&Wt[n * ldt + 4 * q]);
#pragma unroll
        for (int r = 0; r < RPW; ++r)
          acc[r][n] = fmaf(a[r].w, b.w, fmaf(a[r].z, b.z, fmaf(a[r].y, b.y, fmaf(a[r].x, b.x, acc[r][n]))));
      }
    }
    // each lane keeps the logit of class `lane` of its rows
    float zl[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      zl[r] = 0.f;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        float v = warp_sum(acc[r][n]);
        if (bias && n < N) v += bias[n];
        if (lane == n) zl[r] = v;
      }
    }

    // ---- softmax, the cross_entropy VJP and the softmax VJP, per row
    float dzl[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t m = m_base + r;
      const bool in = lane < N;
      // softmax_rows_warp
      float v = in ? zl[r] : -INFINITY;
      float mx = fmaxf(-INFINITY, v);
      mx = warp_max(mx);
      v = in ? expf(v - mx) : 0.f;
      float s = 0.f;
      s += v;
      s = warp_sum(s);
      const float pv = in ? v / s : 0.f;
      // softmax_bwd_warp<true>
      float t = 0.f;
      if (in && m < M) {
        if (onehot) {
          t = tgt[m * N + lane];
        } else {
          const int cls = max(0, min((int)tgt[m], N - 1));
          t = lane == cls ? 1.0f : 0.0f;
        }
      }
      const float gv = in ? (pv - t) / divisor * up : 0.f;
      const float gs = in ? gv * pv : 0.f;
      double dacc = 0.0;
      dacc += (double)gs;
      const float tot = (float)warp_sum(dacc);
      const float rr = gs - pv * tot;
      dzl[r] = in ? rr : 0.f;
      if (in && m < M) {
        if (z) z[m * N + lane] = zl[r];
        if (p) p[m * N + lane] = pv;
        if (dp) dp[m * N + lane] = gv;
        if (dz) dz[m * N + lane] = rr;
      }
    }

    // ---- dx = (dz @ W^T) * (mask > 0): small_nt4_kernel's chain over the
    // zero-padded classes, its (zero) bias add and its mask step
    float dzv[RPW][NB];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
#pragma unroll
      for (int n = 0; n < NB; ++n) dzv[r][n] = __shfl_sync(0xffffffffu, dzl[r], n);
    // the mask vectors of U column steps are loaded before any of them is
    // used, so U * RPW loads of 16 bytes are in flight a lane
    constexpr int U = RPW <= 2 ? 4 : 2;
    for (int q0 = lane; q0 < nq; q0 += 32 * U) {
      float4 mk[U][RPW];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const int q = q0 + 32 * u;
          const int64_t m = m_base + r;
          mk[u][r] = (q < nq && m < M)
                         ? __ldg(reinterpret_cast<const float4*>(mask + m * ldm + 4 * q))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int q = q0 + 32 * u;
        if (q >= nq) break;
        float4 w[NB];
#pragma unroll
        for (int n = 0; n < NB; ++n) w[n] = *reinterpret_cast<const float4*>(&Wt[n * ldt + 4 * q]);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
          const int64_t m = m_base + r;
          if (m >= M) break;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int n = 0; n < NB; ++n) {
            v[0] = fmaf(dzv[r][n], w[n].x, v[0]);
            v[1] = fmaf(dzv[r][n], w[n].y, v[1]);
            v[2] = fmaf(dzv[r][n], w[n].z, v[2]);
            v[3] = fmaf(dzv[r][n], w[n].w, v[3]);
          }
          const float4 k4 = mk[u][r];
          v[0] = __fmul_rn(__fadd_rn(v[0], 0.f), k4.x > 0.f ? 1.f : 0.f);
          v[1] = __fmul_rn(__fadd_rn(v[1], 0.f), k4.y > 0.f ? 1.f : 0.f);
          v[2] = __fmul_rn(__fadd_rn(v[2], 0.f), k4.z > 0.f ? 1.f : 0.f);
          v[3] = __fmul_rn(__fadd_rn(v[3], 0.f), k4.w > 0.f ? 1.f : 0.f);
          *reinterpret_cast<float4*>(dx + m * lddx + 4 * q) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  }
}

bool aligned16(const void* q) { return ((uintptr_t)q & 15) == 0; }

template <int NB>
int launch_head(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* W,
                int64_t ldw, const float* bias, const float* tgt, int onehot, const float* upstream,
                float divisor, float* z, float* p, float* dp, float* dz, float* dx, int64_t lddx,
                const float* mask, int64_t ldm, cudaStream_t st) {
  const size_t smem = (size_t)NB * (K + 4) * 4;
  // four rows a warp while that keeps the blocks' group counts even;
  // two on shorter batches (the last round of groups is then half as long)
  const int64_t sms = sm_count();
  const bool four = NB <= 12 && (M + 4 * kHeadWarps - 1) / (4 * kHeadWarps) >= 4 * sms;
  if (four) {
    auto kern = head_ce_kernel<NB, NB <= 12 ? 4 : 2>;
    TL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t groups = (M + 4 * kHeadWarps - 1) / (4 * kHeadWarps);
    kern<<<(unsigned)(groups < sms ? groups : sms), 32 * kHeadWarps, smem, st>>>(
        M, N, K, A, lda, W, ldw, bias, tgt, onehot, upstream, divisor, z, p, dp, dz, dx, lddx, mask, ldm);
  } else {
    auto kern = head_ce_kernel<NB, 2>;
    TL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t groups = (M + 2 * kHeadWarps - 1) / (2 * kHeadWarps);
    kern<<<(unsigned)(groups < sms ? groups : sms), 32 * kHeadWarps, smem, st>>>(
        M, N, K, A, lda, W, ldw, bias, tgt, onehot, upstream, divisor, z, p, dp, dz, dx, lddx, mask, ldm);
  }
  return after_launch();
}

}  // namespace

// Whether tl_head_ce can run this shape with results bit-identical to the
// unfused kernels: the shapes on which tl_gemm takes small_nn4p_kernel for
// the forward product and small_nt4_kernel for dX.
int head_ce_ok(int64_t M, int N, int64_t K, const float* A, int64_t lda, const float* dx,
               int64_t lddx) {
  if (M <= 0 || N <= 0 || N > 16 || K <= 0 || K % 4 || lda % 4 || !aligned16(A)) return 0;
  if (M * K < (1 << 16)) return 0;  // tl_gemm keeps its tiled kernel on these
  const int nb = N <= 4 ? 4 : N <= 8 ? 8 : N <= 12 ? 12 : 16;
  if ((size_t)nb * (K + 4) * 4 > 200 * 1024) return 0;
  if (K % 4 || lddx % 4 || (dx && !aligned16(dx)) || (M + 63) / 64 > 65535) return 0;
  return 1;
}

}  // namespace tl

extern "C" {

int tl_head_ce_ok(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* dx,
                  int64_t lddx) {
  return tl::head_ce_ok(M, (int)N, K, A, lda, dx, lddx);
}

int tl_head_ce(const float* A, int64_t lda, const float* W, int64_t ldw, const float* bias,
               const float* target, int onehot, const float* upstream, float divisor, float* z,
               float* p, float* dp, float* dz, float* dx, int64_t lddx, const float* mask,
               int64_t ldm, int64_t M, int64_t N, int64_t K, void* stream) {
  if (!A || !W || !target || !dx || !mask || divisor == 0.f) return TL_ERR_INVALID_ARG;
  if (!tl::head_ce_ok(M, (int)N, K, A, lda, dx, lddx)) return TL_ERR_UNSUPPORTED;
  if (ldw < N || ldm % 4 || !tl::aligned16(mask)) return TL_ERR_UNSUPPORTED;
  cudaStream_t st = tl::stream_or_default(stream);
  const int n = (int)N;
  if (n <= 4)
    return tl::launch_head<4>(M, n, K, A, lda, W, ldw, bias, target, onehot, upstream, divisor, z, p,
                              dp, dz, dx, lddx, mask, ldm, st);
  if (n <= 8)
    return tl::launch_head<8>(M, n, K, A, lda, W, ldw, bias, target, onehot, upstream, divisor, z, p,
                              dp, dz, dx, lddx, mask, ldm, st);
  if (n <= 12)
    return tl::launch_head<12>(M, n, K, A, lda, W, ldw, bias, target, onehot, upstream, divisor, z,
                               p, dp, dz, dx, lddx, mask, ldm, st);
  return tl::launch_head<16>(M, n, K, A, lda, W, ldw, bias, target, onehot, upstream, divisor, z, p,
                             dp, dz, dx, lddx, mask, ldm, st);
}

}  // extern "C"
