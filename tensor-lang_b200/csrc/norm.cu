// Softmax, layer/instance/batch normalisation, losses and their reverse-mode
// kernels.
//
// Replaces softmax (kernel_generator.py:564-640), layer_norm (:1667-1810),
// instance_norm (:2017-2061), batch_norm (:1978-2011), cross_entropy
// (:1816-1885), mse_loss (:1891-1943), and moves the matching VJPs of
// tensorlang/autograd.py (softmax :563-580, layer_norm :649-674,
// mse :677-688, cross_entropy :691-704) from NumPy on the host to the device.
//
// The reference runs one thread per row with three sequential passes over
// global memory.  Here rows up to 256 wide are one warp each (values in
// registers); wider rows are one block each with the row staged once in
// shared memory, so every element is read from HBM once and written once.
// Row statistics accumulate in float64.
#include <cfloat>

#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int kWarpCols = 256;        // rows up to this width: one warp per row
constexpr int kWarpPer = kWarpCols / 32;
constexpr int64_t kSmemRowMax = 48 * 1024;  // widest row staged in shared memory (floats)
constexpr size_t kCounterBytes = 4096;      // same scratch convention as reduce.cu

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// ------------------------------------------------------------- softmax ----
__global__ void __launch_bounds__(256) softmax_rows_warp(const float* __restrict__ in,
                                                         float* __restrict__ out, int64_t rows,
                                                         int cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* p = in + row * cols;
  float v[kWarpPer];
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    v[k] = c < cols ? p[c] : -INFINITY;
    m = fmaxf(m, v[k]);
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    v[k] = c < cols ? expf(v[k] - m) : 0.f;
    s += v[k];
  }
  s = warp_sum(s);
  float* q = out + row * cols;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    if (c < cols) q[c] = v[k] / s;
  }
}

// One block per row, the row staged in dynamic shared memory.
__global__ void __launch_bounds__(256) softmax_rows_block(const float* __restrict__ in,
                                                          float* __restrict__ out, int64_t cols,
                                                          int vec) {
  extern __shared__ float row_s[];
  __shared__ float shm[8];
  __shared__ double shd[8];
  const int64_t row = blockIdx.x;
  const float* p = in + row * cols;
  float m = -INFINITY;
  if (vec) {
    for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      float4 a = ld_stream4(p + 4 * i);
      reinterpret_cast<float4*>(row_s)[i] = a;
      m = fmaxf(fmaxf(fmaxf(m, a.x), fmaxf(a.y, a.z)), a.w);
    }
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
      float a = p[i];
      row_s[i] = a;
      m = fmaxf(m, a);
    }
  }
  m = block_max(m, shm);
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float e = expf(row_s[i] - m);
    row_s[i] = e;
    s += (double)e;
  }
  const float tot = (float)block_sum(s, shd);
  float* q = out + row * cols;
  if (vec) {
    for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      float4 e = reinterpret_cast<float4*>(row_s)[i];
      st_stream4(q + 4 * i, make_float4(e.x / tot, e.y / tot, e.z / tot, e.w / tot));
    }
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) q[i] = row_s[i] / tot;
  }
}

// Register-resident rows: 128 threads per row, each holding VPT float4s
// (rows up to 512*VPT wide, a multiple of 4).  One HBM read and one write per
// element, no shared-memory staging, two block reductions per row.
constexpr int RT = 128;  // threads per row

__device__ __forceinline__ float block128_max(float v, float* sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  v = fmaxf(fmaxf(sh[0], sh[1]), fmaxf(sh[2], sh[3]));
  return v;
}
__device__ __forceinline__ double block128_sum(double v, double* sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  return (sh[0] + sh[1]) + (sh[2] + sh[3]);
}

template <int VPT>
__global__ void __launch_bounds__(RT) softmax_rows_reg(const float* __restrict__ in,
                                                       float* __restrict__ out, int64_t cols) {
  __shared__ float shm[4];
  __shared__ double shd[4];
  const float* p = in + (int64_t)blockIdx.x * cols;
  const int n4 = (int)(cols >> 2);
  float4 x[VPT];
  float m = -INFINITY;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    x[v] = i < n4 ? ld_stream4(p + 4 * i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    m = fmaxf(fmaxf(fmaxf(m, x[v].x), fmaxf(x[v].y, x[v].z)), x[v].w);
  }
  m = block128_max(m, shm);
  double s = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    if (i < n4) {
      x[v].x = expf(x[v].x - m); x[v].y = expf(x[v].y - m);
      x[v].z = expf(x[v].z - m); x[v].w = expf(x[v].w - m);
      s += (double)((x[v].x + x[v].y) + (x[v].z + x[v].w));
    }
  }
  const float tot = (float)block128_sum(s, shd);
  float* q = out + (int64_t)blockIdx.x * cols;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    if (i < n4)
      st_stream4(q + 4 * i, make_float4(x[v].x / tot, x[v].y / tot, x[v].z / tot, x[v].w / tot));
  }
}

template <int VPT>
__global__ void __launch_bounds__(RT) layer_norm_rows_reg(const float* __restrict__ in,
                                                          float* __restrict__ out, int64_t cols,
                                                          float eps) {
  __shared__ double shd[2][4];
  const float* p = in + (int64_t)blockIdx.x * cols;
  const int n4 = (int)(cols >> 2);
  float4 x[VPT];
  double s = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    x[v] = i < n4 ? ld_stream4(p + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (double)x[v].x; s += (double)x[v].y; s += (double)x[v].z; s += (double)x[v].w;
  }
  const float mean = (float)(block128_sum(s, shd[0]) / (double)cols);
  double ss = 0.0;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    if (i < n4) {
      x[v].x -= mean; x[v].y -= mean; x[v].z -= mean; x[v].w -= mean;
      ss += (double)x[v].x * x[v].x; ss += (double)x[v].y * x[v].y;
      ss += (double)x[v].z * x[v].z; ss += (double)x[v].w * x[v].w;
    }
  }
  const float var = (float)(block128_sum(ss, shd[1]) / (double)cols);
  const float sd = sqrtf(var + eps);
  float* q = out + (int64_t)blockIdx.x * cols;
#pragma unroll
  for (int v = 0; v < VPT; ++v) {
    const int i = threadIdx.x + v * RT;
    if (i < n4) st_stream4(q + 4 * i, make_float4(x[v].x / sd, x[v].y / sd, x[v].z / sd, x[v].w / sd));
  }
}

// VPT choice for a row of `cols` floats (cols % 4 == 0): 0 when too wide
int rows_vpt(int64_t cols) {
  const int64_t n4 = cols / 4;
  for (int v : {1, 2, 4, 8, 16})
    if (n4 <= (int64_t)v * RT) return v;
  return 0;
}

// Rows too wide for shared memory: three passes over global memory.
__global__ void __launch_bounds__(256) softmax_rows_global(const float* __restrict__ in,
                                                           float* __restrict__ out, int64_t cols) {
  __shared__ float shm[8];
  __shared__ double shd[8];
  const float* p = in + (int64_t)blockIdx.x * cols;
  float m = -INFINITY;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, p[i]);
  m = block_max(m, shm);
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) s += (double)expf(p[i] - m);
  const float tot = (float)block_sum(s, shd);
  float* q = out + (int64_t)blockIdx.x * cols;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) q[i] = expf(p[i] - m) / tot;
}

// ----------------------------------------------------------- layer norm ---
__global__ void __launch_bounds__(256) layer_norm_rows_warp(const float* __restrict__ in,
                                                            float* __restrict__ out, int64_t rows,
                                                            int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* p = in + row * cols;
  float v[kWarpPer];
  double s = 0.0;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    v[k] = c < cols ? p[c] : 0.f;
    s += (double)v[k];
  }
  const float mean = (float)(warp_sum(s) / (double)cols);
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    v[k] = v[k] - mean;
    if (c < cols) ss += (double)v[k] * (double)v[k];
  }
  const float var = (float)(warp_sum(ss) / (double)cols);
  const float sd = sqrtf(var + eps);
  float* q = out + row * cols;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    if (c < cols) q[c] = v[k] / sd;
  }
}

__global__ void __launch_bounds__(256) layer_norm_rows_block(const float* __restrict__ in,
                                                             float* __restrict__ out, int64_t cols,
                                                             float eps, int vec, int staged) {
  extern __shared__ float row_s[];
  __shared__ double shd[8];
  const int64_t row = blockIdx.x;
  const float* p = in + row * cols;
  const float* src = staged ? row_s : p;
  double s = 0.0;
  if (staged && vec) {
    for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      float4 a = ld_stream4(p + 4 * i);
      reinterpret_cast<float4*>(row_s)[i] = a;
      s += (double)a.x; s += (double)a.y; s += (double)a.z; s += (double)a.w;
    }
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
      float a = p[i];
      if (staged) row_s[i] = a;
      s += (double)a;
    }
  }
  const float mean = (float)(block_sum(s, shd) / (double)cols);
  double ss = 0.0;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float d = src[i] - mean;
    ss += (double)d * (double)d;
  }
  const float var = (float)(block_sum(ss, shd) / (double)cols);
  const float sd = sqrtf(var + eps);
  float* q = out + row * cols;
  if (staged && vec) {
    for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
      float4 a = reinterpret_cast<const float4*>(row_s)[i];
      st_stream4(q + 4 * i, make_float4((a.x - mean) / sd, (a.y - mean) / sd,
                                        (a.z - mean) / sd, (a.w - mean) / sd));
    }
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) q[i] = (src[i] - mean) / sd;
  }
}

// Column statistics (sum, sum of squares in float64) with the same chunked
// fixed-order combine as the axis-0 reductions; the last chunk writes
// mean[c] and sd[c] = sqrt(var + eps).
__global__ void __launch_bounds__(256) col_stats_kernel(const float* __restrict__ in, int64_t rows,
                                                        int64_t cols, int64_t chunk, float eps,
                                                        unsigned* counters, double* partials,
                                                        float* mean_out, float* sd_out) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = c < cols;
  const int64_t r0 = (int64_t)blockIdx.y * chunk;
  int64_t r1 = r0 + chunk;
  if (r1 > rows) r1 = rows;
  double s = 0.0, ss = 0.0;
  if (active) {
    for (int64_t r = r0; r < r1; ++r) {
      double x = (double)in[r * cols + c];
      s += x;
      ss += x * x;
    }
    partials[2 * ((size_t)blockIdx.y * cols + c)] = s;
    partials[2 * ((size_t)blockIdx.y * cols + c) + 1] = ss;
  }
  __threadfence();
  __shared__ unsigned is_last;
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(&counters[blockIdx.x], 1u) == gridDim.y - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (active) {
    double ts = 0.0, tss = 0.0;
    for (unsigned y = 0; y < gridDim.y; ++y) {
      ts += __ldcg(&partials[2 * ((size_t)y * cols + c)]);
      tss += __ldcg(&partials[2 * ((size_t)y * cols + c) + 1]);
    }
    double mu = ts / (double)rows;
    double var = tss / (double)rows - mu * mu;
    if (var < 0.0) var = 0.0;
    mean_out[c] = (float)mu;
    sd_out[c] = sqrtf((float)var + eps);
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

// out[r,c] = (x[r,c] - mean[c]) / sd[c]
__global__ void __launch_bounds__(256) col_normalize_kernel(const float* __restrict__ in,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ sd,
                                                            float* __restrict__ out, int64_t n,
                                                            int64_t cols) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t c = i % cols;
    out[i] = (in[i] - mean[c]) / sd[c];
  }
}

// batch_norm with running statistics: (x - rm[c]) / sqrtf(rv[c] + eps)
__global__ void __launch_bounds__(256) batch_norm_kernel(const float* __restrict__ in,
                                                         const float* __restrict__ rm,
                                                         const float* __restrict__ rv,
                                                         float* __restrict__ out, int64_t n,
                                                         int64_t cols, float eps) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t c = i % cols;
    out[i] = (in[i] - rm[c]) / sqrtf(rv[c] + eps);
  }
}

// --------------------------------------------------------------- losses ---
// Scalar loss = (sum over items of f(item)) / divisor, float64 accumulation,
// fixed-order combine by the last block.
template <int KIND>  // 0 mse, 1 CE class-index, 2 CE one-hot
__global__ void __launch_bounds__(256) loss_kernel(const float* __restrict__ a,
                                                   const float* __restrict__ b,
                                                   float* __restrict__ out, int64_t items,
                                                   int64_t classes, unsigned* counter,
                                                   double* partials) {
  __shared__ double shd[8];
  __shared__ unsigned is_last;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  double acc = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
    if constexpr (KIND == 0) {
      float d = a[i] - b[i];
      acc += (double)(d * d);
    } else {
      float p;
      if constexpr (KIND == 1) {
        int c = (int)b[i];
        c = max(0, min(c, (int)classes - 1));
        p = a[i * classes + c];
      } else {
        p = 0.f;
        for (int64_t c = 0; c < classes; ++c) p += b[i * classes + c] * a[i * classes + c];
      }
      p = fmaxf(p, 1e-7f);
      p = fminf(p, 1.0f - 1e-7f);
      acc += (double)(-logf(p));
    }
  }
  double blk = block_sum(acc, shd);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = blk;
    __threadfence();
    is_last = (atomicAdd(counter, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last || threadIdx.x != 0) return;
  __threadfence();
  double t = 0.0;
  for (unsigned k = 0; k < gridDim.x; ++k) t += __ldcg(&partials[k]);
  out[0] = (float)t / (float)items;
  *counter = 0u;
}

unsigned loss_blocks(int64_t items) {
  int64_t b = (items + 255) / 256;
  int64_t cap = 4LL * sm_count();
  if (cap > 1024) cap = 1024;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

// -------------------------------------------------- reverse-mode kernels ---
// softmax VJP: dx = g*s - s*sum(g*s)   (autograd.py:563-580)
// CE+softmax: gp = (p - t)/divisor*up; dz = gp*p - p*sum(gp*p)
template <bool CE>
__global__ void __launch_bounds__(256) softmax_bwd_warp(const float* __restrict__ s,
                                                        const float* __restrict__ g,
                                                        const float* __restrict__ tgt, int onehot,
                                                        const float* __restrict__ upstream,
                                                        float divisor, float* __restrict__ dp,
                                                        float* __restrict__ dx, int64_t rows,
                                                        int cols, int accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float up = (CE && upstream) ? upstream[0] : 1.0f;
  int cls = -1;
  if (CE && !onehot) cls = max(0, min((int)tgt[row], cols - 1));
  float sv[kWarpPer], gs[kWarpPer];
  double acc = 0.0;
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    sv[k] = 0.f;
    gs[k] = 0.f;
    if (c < cols) {
      sv[k] = s[row * cols + c];
      float gv;
      if constexpr (CE) {
        float t = onehot ? tgt[row * cols + c] : (c == cls ? 1.0f : 0.0f);
        gv = (sv[k] - t) / divisor * up;
        if (dp) dp[row * cols + c] = gv;
      } else {
        gv = g[row * cols + c];
      }
      gs[k] = gv * sv[k];
      acc += (double)gs[k];
    }
  }
  const float tot = (float)warp_sum(acc);
#pragma unroll
  for (int k = 0; k < kWarpPer; ++k) {
    int c = lane + 32 * k;
    if (c < cols) {
      float r = gs[k] - sv[k] * tot;
      float* o = dx + row * cols + c;
      *o = accumulate ? *o + r : r;
    }
  }
}

template <bool CE>
__global__ void __launch_bounds__(256) softmax_bwd_block(const float* __restrict__ s,
                                                         const float* __restrict__ g,
                                                         const float* __restrict__ tgt, int onehot,
                                                         const float* __restrict__ upstream,
                                                         float divisor, float* __restrict__ dp,
                                                         float* __restrict__ dx, int64_t cols,
                                                         int accumulate) {
  __shared__ double shd[8];
  const int64_t row = blockIdx.x;
  const float up = (CE && upstream) ? upstream[0] : 1.0f;
  int64_t cls = -1;
  if (CE && !onehot) {
    cls = (int64_t)tgt[row];
    cls = cls < 0 ? 0 : (cls > cols - 1 ? cols - 1 : cls);
  }
  auto grad_at = [&](int64_t c, float sv) -> float {
    if constexpr (CE) {
      float t = onehot ? tgt[row * cols + c] : (c == cls ? 1.0f : 0.0f);
      return (sv - t) / divisor * up;
    } else {
      return g[row * cols + c];
    }
  };
  double acc = 0.0;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float sv = s[row * cols + c];
    float gv = grad_at(c, sv);
    if (CE && dp) dp[row * cols + c] = gv;
    acc += (double)(gv * sv);
  }
  const float tot = (float)block_sum(acc, shd);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float sv = s[row * cols + c];
    float gv = grad_at(c, sv);
    float r = gv * sv - sv * tot;
    float* o = dx + row * cols + c;
    *o = accumulate ? *o + r : r;
  }
}

// layer_norm VJP along rows (autograd.py:649-674)
__global__ void __launch_bounds__(256) layer_norm_bwd_block(const float* __restrict__ x,
                                                            const float* __restrict__ g,
                                                            float* __restrict__ dx, int64_t cols,
                                                            float eps, int accumulate) {
  __shared__ double shd[8];
  const int64_t row = blockIdx.x;
  const float* xp = x + row * cols;
  const float* gp = g + row * cols;
  double s = 0.0;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s += (double)xp[c];
  const double mean = block_sum(s, shd) / (double)cols;
  double v = 0.0, sgd = 0.0, sg = 0.0, sd_ = 0.0;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    double d = (double)xp[c] - mean;
    v += d * d;
    sgd += (double)gp[c] * d;
    sg += (double)gp[c];
    sd_ += d;
  }
  const double var = block_sum(v, shd) / (double)cols;
  const double sum_gd = block_sum(sgd, shd);
  const double sum_g = block_sum(sg, shd);
  const double sum_d = block_sum(sd_, shd);
  const double ve = var + (double)eps;
  const double stdv = sqrt(ve);
  const double n = (double)cols;
  const double gvar = sum_gd * -0.5 * pow(ve, -1.5);
  const double gmean = -sum_g / stdv + gvar * (-2.0 * sum_d) / n;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    double d = (double)xp[c] - mean;
    float r = (float)((double)gp[c] / stdv + gvar * 2.0 * d / n + gmean / n);
    float* o = dx + row * cols + c;
    *o = accumulate ? *o + r : r;
  }
}

}  // namespace
}  // namespace tl

extern "C" {

int tl_softmax_rows(const float* in, float* out, int64_t rows, int64_t cols, void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  const int vpt = (cols % 4 == 0 && tl::aligned16(in) && tl::aligned16(out)) ? tl::rows_vpt(cols) : 0;
  if (cols <= tl::kWarpCols) {
    tl::softmax_rows_warp<<<tl::ceil_div_u(rows, 8), 256, 0, st>>>(in, out, rows, (int)cols);
  } else if (vpt && rows <= INT32_MAX) {
    switch (vpt) {
      case 1: tl::softmax_rows_reg<1><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols); break;
      case 2: tl::softmax_rows_reg<2><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols); break;
      case 4: tl::softmax_rows_reg<4><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols); break;
      case 8: tl::softmax_rows_reg<8><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols); break;
      default: tl::softmax_rows_reg<16><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols); break;
    }
  } else if (cols <= tl::kSmemRowMax) {
    size_t smem = (size_t)cols * 4;
    if (smem > 48 * 1024)
      TL_CUDA_TRY(cudaFuncSetAttribute(tl::softmax_rows_block,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int vec = (cols % 4 == 0) && tl::aligned16(in) && tl::aligned16(out);
    tl::softmax_rows_block<<<(unsigned)rows, 256, smem, st>>>(in, out, cols, vec);
  } else {
    tl::softmax_rows_global<<<(unsigned)rows, 256, 0, st>>>(in, out, cols);
  }
  return tl::after_launch();
}

size_t tl_norm_cols_scratch_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  int64_t gx = (cols + 255) / 256;
  int64_t want = (4LL * 148 + gx - 1) / gx;
  if (want > rows) want = rows;
  if (want > 1024) want = 1024;
  if (want < 1) want = 1;
  return tl::kCounterBytes + (size_t)want * cols * 16 + (size_t)cols * 8 + 256;
}

int tl_layer_norm_rows(const float* in, float* out, int64_t rows, int64_t cols, float eps,
                       void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  const int vpt = (cols % 4 == 0 && tl::aligned16(in) && tl::aligned16(out)) ? tl::rows_vpt(cols) : 0;
  if (cols <= tl::kWarpCols) {
    tl::layer_norm_rows_warp<<<tl::ceil_div_u(rows, 8), 256, 0, st>>>(in, out, rows, (int)cols, eps);
  } else if (vpt && rows <= INT32_MAX) {
    switch (vpt) {
      case 1: tl::layer_norm_rows_reg<1><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols, eps); break;
      case 2: tl::layer_norm_rows_reg<2><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols, eps); break;
      case 4: tl::layer_norm_rows_reg<4><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols, eps); break;
      case 8: tl::layer_norm_rows_reg<8><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols, eps); break;
      default: tl::layer_norm_rows_reg<16><<<(unsigned)rows, tl::RT, 0, st>>>(in, out, cols, eps); break;
    }
  } else {
    int staged = cols <= tl::kSmemRowMax;
    size_t smem = staged ? (size_t)cols * 4 : 0;
    if (smem > 48 * 1024)
      TL_CUDA_TRY(cudaFuncSetAttribute(tl::layer_norm_rows_block,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int vec = (cols % 4 == 0) && tl::aligned16(in) && tl::aligned16(out);
    tl::layer_norm_rows_block<<<(unsigned)rows, 256, smem, st>>>(in, out, cols, eps, vec, staged);
  }
  return tl::after_launch();
}

int tl_layer_norm_cols(const float* in, float* out, int64_t rows, int64_t cols, float eps,
                       void* scratch, void* stream) {
  if (!in || !out || !scratch || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  int64_t gx = (cols + 255) / 256;
  if (gx > (int64_t)(tl::kCounterBytes / 4)) return TL_ERR_UNSUPPORTED;
  int64_t want = (4LL * 148 + gx - 1) / gx;
  if (want > rows) want = rows;
  if (want > 1024) want = 1024;
  if (want < 1) want = 1;
  int64_t chunk = (rows + want - 1) / want;
  unsigned gy = (unsigned)((rows + chunk - 1) / chunk);
  unsigned* counters = (unsigned*)scratch;
  double* partials = (double*)((char*)scratch + tl::kCounterBytes);
  float* mean = (float*)(partials + (size_t)want * cols * 2);
  float* sd = mean + cols;
  tl::col_stats_kernel<<<dim3((unsigned)gx, gy), 256, 0, st>>>(in, rows, cols, chunk, eps, counters,
                                                                partials, mean, sd);
  TL_TRY(tl::after_launch());
  int64_t n = rows * cols;
  unsigned grid = tl::ceil_div_u(n, 256);
  if (grid > 8u * tl::sm_count()) grid = 8u * tl::sm_count();
  tl::col_normalize_kernel<<<grid, 256, 0, st>>>(in, mean, sd, out, n, cols);
  return tl::after_launch();
}

int tl_batch_norm(const float* in, const float* running_mean, const float* running_var, float* out,
                  int64_t rows, int64_t cols, float eps, void* stream) {
  if (!in || !out || !running_mean || !running_var || rows <= 0 || cols <= 0)
    return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  int64_t n = rows * cols;
  unsigned grid = tl::ceil_div_u(n, 256);
  if (grid > 8u * tl::sm_count()) grid = 8u * tl::sm_count();
  tl::batch_norm_kernel<<<grid, 256, 0, st>>>(in, running_mean, running_var, out, n, cols, eps);
  return tl::after_launch();
}

size_t tl_loss_scratch_bytes(int64_t n) {
  (void)n;
  return tl::kCounterBytes + 1024 * 8;
}

int tl_mse_loss(const float* pred, const float* target, float* out, int64_t n, void* scratch,
                void* stream) {
  if (!pred || !target || !out || !scratch || n <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  unsigned* counter = (unsigned*)scratch;
  double* partials = (double*)((char*)scratch + tl::kCounterBytes);
  tl::loss_kernel<0><<<tl::loss_blocks(n), 256, 0, st>>>(pred, target, out, n, 1, counter, partials);
  return tl::after_launch();
}

int tl_cross_entropy(const float* probs, const float* target, float* out, int64_t batch,
                     int64_t classes, int onehot, void* scratch, void* stream) {
  if (!probs || !target || !out || !scratch || batch <= 0 || classes <= 0)
    return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  unsigned* counter = (unsigned*)scratch;
  double* partials = (double*)((char*)scratch + tl::kCounterBytes);
  if (onehot)
    tl::loss_kernel<2><<<tl::loss_blocks(batch), 256, 0, st>>>(probs, target, out, batch, classes,
                                                                counter, partials);
  else
    tl::loss_kernel<1><<<tl::loss_blocks(batch), 256, 0, st>>>(probs, target, out, batch, classes,
                                                                counter, partials);
  return tl::after_launch();
}

int tl_softmax_backward_rows(const float* s, const float* g, float* dx, int64_t rows, int64_t cols,
                             int accumulate, void* stream) {
  if (!s || !g || !dx || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  if (cols <= tl::kWarpCols)
    tl::softmax_bwd_warp<false><<<tl::ceil_div_u(rows, 8), 256, 0, st>>>(
        s, g, nullptr, 0, nullptr, 1.f, nullptr, dx, rows, (int)cols, accumulate);
  else
    tl::softmax_bwd_block<false><<<(unsigned)rows, 256, 0, st>>>(s, g, nullptr, 0, nullptr, 1.f,
                                                                  nullptr, dx, cols, accumulate);
  return tl::after_launch();
}

int tl_ce_softmax_backward(const float* p, const float* target, int onehot, const float* upstream,
                           float divisor, float* dp, float* dz, int64_t rows, int64_t cols,
                           int accumulate, void* stream) {
  if (!p || !target || !dz || rows <= 0 || cols <= 0 || divisor == 0.f) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  if (cols <= tl::kWarpCols)
    tl::softmax_bwd_warp<true><<<tl::ceil_div_u(rows, 8), 256, 0, st>>>(
        p, nullptr, target, onehot, upstream, divisor, dp, dz, rows, (int)cols, accumulate);
  else
    tl::softmax_bwd_block<true><<<(unsigned)rows, 256, 0, st>>>(p, nullptr, target, onehot, upstream,
                                                                 divisor, dp, dz, cols, accumulate);
  return tl::after_launch();
}

int tl_layer_norm_backward_rows(const float* x, const float* g, float* dx, int64_t rows,
                                int64_t cols, float eps, int accumulate, void* stream) {
  if (!x || !g || !dx || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  tl::layer_norm_bwd_block<<<(unsigned)rows, 256, 0, st>>>(x, g, dx, cols, eps, accumulate);
  return tl::after_launch();
}

}  // extern "C"
