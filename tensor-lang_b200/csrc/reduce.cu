// Axis and full reductions: sum / mean / max / min / argmax / argmin.
//
// Replaces the reference's sum (kernel_generator.py:784-882), mean (:888-989),
// max (:1246-1345), min (:1352-1453), argmax (:1459-1542), argmin (:1549-1578).
// The reference runs one thread per output row/column with a sequential
// float32 loop (uncoalesced for axis 1) and atomics for full reductions.
// Here: axis 1 is one warp per row with 128-bit loads; axis 0 is column
// stripes of 128-bit loads split into row chunks whose partials are combined
// in a fixed order by the last chunk to finish; full reductions are
// grid-stride blocks combined the same way.  Sums accumulate in float64 and
// round once, so results do not depend on launch shape; argmax/argmin keep the
// first index of the extreme value (the reference's strict `>`/`<` scan).
#include <cfloat>
#include <climits>

#include "tl_common.cuh"

namespace tl {
namespace {

constexpr int kAssumedSms = 148;      // planning constant for chunk counts
constexpr int kFullMaxBlocks = 2048;  // upper bound of full-reduction blocks
constexpr int kFullBlocksPerSm = 4;   // launch bounds keep 4 blocks of 256 resident per SM
// Every scratch buffer starts with a fixed counter region; partials follow it,
// so reductions of different kinds may share one scratch buffer in stream order.
// completion counters ahead of the partials: one per column stripe, enough
// for 131072 columns on the one-column-per-lane path (32 columns a stripe)
constexpr size_t kCounterBytes = 16384;
constexpr unsigned kMaxColBlocks = kCounterBytes / 4;

struct ArgVal {
  float v;
  int64_t i;  // INT64_MAX marks "no element seen"
};

template <bool LARGEST>
__device__ __forceinline__ bool arg_better(float vo, int64_t io, float v, int64_t i) {
  if (io == INT64_MAX) return false;
  if (i == INT64_MAX) return true;
  if (LARGEST ? (vo > v) : (vo < v)) return true;
  return vo == v && io < i;
}

template <bool LARGEST>
__device__ __forceinline__ void arg_take(float& v, int64_t& i, float x, int64_t ix) {
  if (i == INT64_MAX || (LARGEST ? (x > v) : (x < v))) {
    v = x;
    i = ix;
  }
}

template <bool LARGEST>
__device__ __forceinline__ void warp_arg(float& v, int64_t& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float vo = __shfl_xor_sync(0xffffffffu, v, o);
    int64_t io = __shfl_xor_sync(0xffffffffu, i, o);
    if (arg_better<LARGEST>(vo, io, v, i)) {
      v = vo;
      i = io;
    }
  }
}

// ------------------------------------------------------------ axis = 1 ----
template <int OP, bool VEC>
__global__ void __launch_bounds__(256) reduce_rows_kernel(const float* __restrict__ in,
                                                          float* __restrict__ out, int64_t rows,
                                                          int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* p = in + row * cols;
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
    double s = 0.0;
    if constexpr (VEC) {
      const int64_t n4 = cols >> 2;
      int64_t i = lane;
      for (; i + 96 < n4; i += 128) {
        float4 a = ld_stream4(p + 4 * i), b = ld_stream4(p + 4 * (i + 32));
        float4 c = ld_stream4(p + 4 * (i + 64)), d = ld_stream4(p + 4 * (i + 96));
        s += (double)a.x; s += (double)a.y; s += (double)a.z; s += (double)a.w;
        s += (double)b.x; s += (double)b.y; s += (double)b.z; s += (double)b.w;
        s += (double)c.x; s += (double)c.y; s += (double)c.z; s += (double)c.w;
        s += (double)d.x; s += (double)d.y; s += (double)d.z; s += (double)d.w;
      }
      for (; i < n4; i += 32) {
        float4 a = ld_stream4(p + 4 * i);
        s += (double)a.x; s += (double)a.y; s += (double)a.z; s += (double)a.w;
      }
    } else {
      for (int64_t i = lane; i < cols; i += 32) s += (double)p[i];
    }
    s = warp_sum(s);
    if (lane == 0) out[row] = (OP == TL_RED_MEAN) ? (float)(s / (double)cols) : (float)s;
  } else if constexpr (OP == TL_RED_MAX || OP == TL_RED_MIN) {
    float m = (OP == TL_RED_MAX) ? -INFINITY : INFINITY;
    if constexpr (VEC) {
      const int64_t n4 = cols >> 2;
      for (int64_t i = lane; i < n4; i += 32) {
        float4 a = ld_stream4(p + 4 * i);
        if (OP == TL_RED_MAX) m = fmaxf(fmaxf(fmaxf(m, a.x), fmaxf(a.y, a.z)), a.w);
        else m = fminf(fminf(fminf(m, a.x), fminf(a.y, a.z)), a.w);
      }
    } else {
      for (int64_t i = lane; i < cols; i += 32)
        m = (OP == TL_RED_MAX) ? fmaxf(m, p[i]) : fminf(m, p[i]);
    }
    m = (OP == TL_RED_MAX) ? warp_max(m) : warp_min(m);
    if (lane == 0) out[row] = m;
  } else {
    constexpr bool L = (OP == TL_RED_ARGMAX);
    float v = 0.f;
    int64_t ix = INT64_MAX;
    if constexpr (VEC) {
      const int64_t n4 = cols >> 2;
      for (int64_t i = lane; i < n4; i += 32) {
        float4 a = ld_stream4(p + 4 * i);
        arg_take<L>(v, ix, a.x, 4 * i);
        arg_take<L>(v, ix, a.y, 4 * i + 1);
        arg_take<L>(v, ix, a.z, 4 * i + 2);
        arg_take<L>(v, ix, a.w, 4 * i + 3);
      }
    } else {
      for (int64_t i = lane; i < cols; i += 32) arg_take<L>(v, ix, p[i], i);
    }
    warp_arg<L>(v, ix);
    if (lane == 0) out[row] = (float)ix;
  }
}

// ------------------------------------------------------------ axis = 0 ----
// A block owns a stripe of 32*VEC columns (lane l: columns 4l..4l+3 when
// VEC = 4) and a chunk of rows; its 8 warps take every 8th row of the chunk
// (4 rows in flight per trip) and fold their results through shared memory
// in warp order.  Each block writes one partial per column; the last block of
// a stripe folds the chunks' partials in chunk order.  Both folds are fixed-
// order, so results do not depend on timing.
constexpr int kColBlocksPerSm = 4;  // launch bounds below keep 4 resident

struct ColPlan {
  int vec;      // 4: float4 per lane, else 1
  unsigned gx;  // column stripes
  unsigned gy;  // row chunks
  int64_t chunk;
};

ColPlan col_plan(int64_t rows, int64_t cols, bool vec_ok) {
  ColPlan p;
  p.vec = vec_ok ? 4 : 1;
  p.gx = ceil_div_u(cols, 32LL * p.vec);
  // one resident wave: kColBlocksPerSm blocks of 256 threads on every SM
  int64_t want = (int64_t)kColBlocksPerSm * kAssumedSms / p.gx;  // rounded down: no second wave
  int64_t maxy = (rows + 63) / 64;  // at least 64 rows per chunk
  if (want > maxy) want = maxy;
  if (want > 256) want = 256;
  if (want < 1) want = 1;
  p.chunk = (rows + want - 1) / want;
  p.gy = (unsigned)((rows + p.chunk - 1) / p.chunk);
  return p;
}

size_t col_partial_bytes(int op) { return (op == TL_RED_ARGMAX || op == TL_RED_ARGMIN) ? 16 : 8; }

template <int OP>
struct ColAcc {
  double s;
  float m;
  int64_t i;
};

template <int OP>
__device__ __forceinline__ void col_init(ColAcc<OP>& a) {
  a.s = 0.0;
  a.m = (OP == TL_RED_MAX) ? -INFINITY : INFINITY;
  a.i = INT64_MAX;
}
template <int OP>
__device__ __forceinline__ void col_add(ColAcc<OP>& a, float x, int64_t r) {
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) a.s += (double)x;
  else if constexpr (OP == TL_RED_MAX) a.m = fmaxf(a.m, x);
  else if constexpr (OP == TL_RED_MIN) a.m = fminf(a.m, x);
  else arg_take<OP == TL_RED_ARGMAX>(a.m, a.i, x, r);
}
template <int OP>
__device__ __forceinline__ void col_merge(ColAcc<OP>& a, const ColAcc<OP>& b) {
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) a.s += b.s;
  else if constexpr (OP == TL_RED_MAX) a.m = fmaxf(a.m, b.m);
  else if constexpr (OP == TL_RED_MIN) a.m = fminf(a.m, b.m);
  else if (arg_better<OP == TL_RED_ARGMAX>(b.m, b.i, a.m, a.i)) { a.m = b.m; a.i = b.i; }
}
template <int OP>
__device__ __forceinline__ void col_store(void* partials, size_t off, const ColAcc<OP>& a) {
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) ((double*)partials)[off] = a.s;
  else if constexpr (OP == TL_RED_MAX || OP == TL_RED_MIN) ((float*)partials)[2 * off] = a.m;
  else {
    ((float*)partials)[4 * off] = a.m;
    ((int64_t*)partials)[2 * off + 1] = a.i;
  }
}
template <int OP>
__device__ __forceinline__ ColAcc<OP> col_load(const void* partials, size_t off) {
  ColAcc<OP> a;
  col_init(a);
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) a.s = __ldcg(&((const double*)partials)[off]);
  else if constexpr (OP == TL_RED_MAX || OP == TL_RED_MIN) a.m = __ldcg(&((const float*)partials)[2 * off]);
  else {
    a.m = __ldcg(&((const float*)partials)[4 * off]);
    a.i = __ldcg(&((const int64_t*)partials)[2 * off + 1]);
  }
  return a;
}

template <int OP, int VEC>
__global__ void __launch_bounds__(256, kColBlocksPerSm) reduce_cols_kernel(const float* __restrict__ in,
                                                          float* __restrict__ out, int64_t rows,
                                                          int64_t cols, int64_t chunk,
                                                          unsigned* counters, void* partials) {
  __shared__ ColAcc<OP> sh[8][32 * VEC];
  __shared__ unsigned is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = (int64_t)blockIdx.x * 32 * VEC + (int64_t)lane * VEC;
  const bool active = c0 < cols;
  const int64_t r_begin = (int64_t)blockIdx.y * chunk;
  const int64_t r_end = r_begin + chunk < rows ? r_begin + chunk : rows;

  ColAcc<OP> acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) col_init(acc[k]);
  if (active) {
    int64_t r = r_begin + warp;
    for (; r + 24 < r_end; r += 32) {  // 4 rows in flight per trip
      float x[4][VEC];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float* p = in + (r + 8 * q) * cols + c0;
        if constexpr (VEC == 4) {
          float4 a = ld_stream4(p);
          x[q][0] = a.x; x[q][1] = a.y; x[q][2] = a.z; x[q][3] = a.w;
        } else {
          x[q][0] = *p;
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < VEC; ++k) col_add(acc[k], x[q][k], r + 8 * q);
    }
    for (; r < r_end; r += 8) {
      const float* p = in + r * cols + c0;
      if constexpr (VEC == 4) {
        float4 a = ld_stream4(p);
        col_add(acc[0], a.x, r); col_add(acc[1], a.y, r); col_add(acc[2], a.z, r); col_add(acc[3], a.w, r);
      } else {
        col_add(acc[0], *p, r);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VEC; ++k) sh[warp][lane * VEC + k] = acc[k];
  __syncthreads();
  // fold the 8 warps (warp order) and write this chunk's partial
  for (int j = threadIdx.x; j < 32 * VEC; j += blockDim.x) {
    const int64_t c = (int64_t)blockIdx.x * 32 * VEC + j;
    if (c >= cols) continue;
    ColAcc<OP> t = sh[0][j];
    for (int w = 1; w < 8; ++w) col_merge(t, sh[w][j]);
    col_store(partials, (size_t)blockIdx.y * cols + c, t);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(&counters[blockIdx.x], 1u) == gridDim.y - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int j = threadIdx.x; j < 32 * VEC; j += blockDim.x) {
    const int64_t c = (int64_t)blockIdx.x * 32 * VEC + j;
    if (c >= cols) continue;
    ColAcc<OP> t;
    col_init(t);
    unsigned y = 0;
    for (; y + 3 < gridDim.y; y += 4) {  // 4 partial loads in flight
      ColAcc<OP> a = col_load<OP>(partials, (size_t)y * cols + c);
      ColAcc<OP> b = col_load<OP>(partials, (size_t)(y + 1) * cols + c);
      ColAcc<OP> d = col_load<OP>(partials, (size_t)(y + 2) * cols + c);
      ColAcc<OP> e = col_load<OP>(partials, (size_t)(y + 3) * cols + c);
      col_merge(t, a); col_merge(t, b); col_merge(t, d); col_merge(t, e);
    }
    for (; y < gridDim.y; ++y) col_merge(t, col_load<OP>(partials, (size_t)y * cols + c));
    if constexpr (OP == TL_RED_SUM) out[c] = (float)t.s;
    else if constexpr (OP == TL_RED_MEAN) out[c] = (float)(t.s / (double)rows);
    else if constexpr (OP == TL_RED_ARGMAX || OP == TL_RED_ARGMIN) out[c] = (float)t.i;
    else out[c] = t.m;
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;
}

// ------------------------------------------------------------ axis = None -
template <int OP, bool VEC>
__global__ void __launch_bounds__(256, kFullBlocksPerSm) reduce_full_kernel(const float* __restrict__ in,
                                                          float* __restrict__ out, int64_t n,
                                                          unsigned* counter, void* partials) {
  constexpr bool ARG = (OP == TL_RED_ARGMAX || OP == TL_RED_ARGMIN);
  constexpr bool L = (OP == TL_RED_ARGMAX);
  __shared__ double sh_d[8];
  __shared__ float sh_f[8];
  __shared__ int64_t sh_i[8];
  __shared__ unsigned is_last;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;

  double s = 0.0;
  float m = (OP == TL_RED_MAX) ? -INFINITY : INFINITY;
  int64_t ix = INT64_MAX;
  if constexpr (VEC) {
    const int64_t n4 = n >> 2;
    int64_t i = tid;
    if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
      // 4 loads in flight, 4 independent accumulation chains
      double s1 = 0.0, s2 = 0.0, s3 = 0.0;
#pragma unroll 1
      for (; i + 3 * stride < n4; i += 4 * stride) {
        float4 a = ld_stream4(in + 4 * i), b = ld_stream4(in + 4 * (i + stride));
        float4 c = ld_stream4(in + 4 * (i + 2 * stride)), d = ld_stream4(in + 4 * (i + 3 * stride));
        s += (double)a.x; s += (double)a.y; s += (double)a.z; s += (double)a.w;
        s1 += (double)b.x; s1 += (double)b.y; s1 += (double)b.z; s1 += (double)b.w;
        s2 += (double)c.x; s2 += (double)c.y; s2 += (double)c.z; s2 += (double)c.w;
        s3 += (double)d.x; s3 += (double)d.y; s3 += (double)d.z; s3 += (double)d.w;
      }
      s = (s + s1) + (s2 + s3);
    } else if constexpr (OP == TL_RED_MAX || OP == TL_RED_MIN) {
#pragma unroll 1
      for (; i + 3 * stride < n4; i += 4 * stride) {
        float4 a = ld_stream4(in + 4 * i), b = ld_stream4(in + 4 * (i + stride));
        float4 c = ld_stream4(in + 4 * (i + 2 * stride)), d = ld_stream4(in + 4 * (i + 3 * stride));
        if constexpr (OP == TL_RED_MAX) {
          const float ab = fmaxf(fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w)), fmaxf(fmaxf(b.x, b.y), fmaxf(b.z, b.w)));
          const float cd = fmaxf(fmaxf(fmaxf(c.x, c.y), fmaxf(c.z, c.w)), fmaxf(fmaxf(d.x, d.y), fmaxf(d.z, d.w)));
          m = fmaxf(m, fmaxf(ab, cd));
        } else {
          const float ab = fminf(fminf(fminf(a.x, a.y), fminf(a.z, a.w)), fminf(fminf(b.x, b.y), fminf(b.z, b.w)));
          const float cd = fminf(fminf(fminf(c.x, c.y), fminf(c.z, c.w)), fminf(fminf(d.x, d.y), fminf(d.z, d.w)));
          m = fminf(m, fminf(ab, cd));
        }
      }
    }
    for (; i < n4; i += stride) {
      float4 a = ld_stream4(in + 4 * i);
      if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
        s += (double)a.x; s += (double)a.y; s += (double)a.z; s += (double)a.w;
      } else if constexpr (OP == TL_RED_MAX) {
        m = fmaxf(fmaxf(fmaxf(m, a.x), fmaxf(a.y, a.z)), a.w);
      } else if constexpr (OP == TL_RED_MIN) {
        m = fminf(fminf(fminf(m, a.x), fminf(a.y, a.z)), a.w);
      } else {
        arg_take<L>(m, ix, a.x, 4 * i);
        arg_take<L>(m, ix, a.y, 4 * i + 1);
        arg_take<L>(m, ix, a.z, 4 * i + 2);
        arg_take<L>(m, ix, a.w, 4 * i + 3);
      }
    }
  } else {
    for (int64_t i = tid; i < n; i += stride) {
      float x = in[i];
      if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) s += (double)x;
      else if constexpr (OP == TL_RED_MAX) m = fmaxf(m, x);
      else if constexpr (OP == TL_RED_MIN) m = fminf(m, x);
      else arg_take<L>(m, ix, x, i);
    }
  }
  // block combine (fixed order over warps)
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
    s = warp_sum(s);
    if (lane == 0) sh_d[wid] = s;
  } else if constexpr (ARG) {
    warp_arg<L>(m, ix);
    if (lane == 0) { sh_f[wid] = m; sh_i[wid] = ix; }
  } else {
    m = (OP == TL_RED_MAX) ? warp_max(m) : warp_min(m);
    if (lane == 0) sh_f[wid] = m;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
      double t = 0.0;
      for (int w = 0; w < nw; ++w) t += sh_d[w];
      ((double*)partials)[blockIdx.x] = t;
    } else if constexpr (ARG) {
      float tv = sh_f[0];
      int64_t ti = sh_i[0];
      for (int w = 1; w < nw; ++w)
        if (arg_better<L>(sh_f[w], sh_i[w], tv, ti)) { tv = sh_f[w]; ti = sh_i[w]; }
      ((float*)partials)[4 * blockIdx.x] = tv;
      ((int64_t*)partials)[2 * blockIdx.x + 1] = ti;
    } else {
      float t = sh_f[0];
      for (int w = 1; w < nw; ++w) t = (OP == TL_RED_MAX) ? fmaxf(t, sh_f[w]) : fminf(t, sh_f[w]);
      ((float*)partials)[2 * blockIdx.x] = t;
    }
    __threadfence();
    is_last = (atomicAdd(counter, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if constexpr (OP == TL_RED_SUM || OP == TL_RED_MEAN) {
    // each thread folds a fixed strided subset, then a fixed-order block fold
    double t = 0.0;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) t += __ldcg(&((double*)partials)[b]);
    t = warp_sum(t);
    if (lane == 0) sh_d[wid] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
      double tt = 0.0;
      for (int w = 0; w < nw; ++w) tt += sh_d[w];
      out[0] = (OP == TL_RED_MEAN) ? (float)(tt / (double)n) : (float)tt;
      *counter = 0u;
    }
    return;
  }
  if constexpr (ARG) {
    float tv = 0.f;
    int64_t ti = INT64_MAX;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
      float pv = __ldcg(&((float*)partials)[4 * b]);
      int64_t pi = __ldcg(&((int64_t*)partials)[2 * b + 1]);
      if (arg_better<L>(pv, pi, tv, ti)) { tv = pv; ti = pi; }
    }
    warp_arg<L>(tv, ti);
    if (lane == 0) { sh_f[wid] = tv; sh_i[wid] = ti; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 0; w < nw; ++w)
        if (arg_better<L>(sh_f[w], sh_i[w], tv, ti)) { tv = sh_f[w]; ti = sh_i[w]; }
      out[0] = (float)ti;
      *counter = 0u;
    }
  } else {
    float t = (OP == TL_RED_MAX) ? -INFINITY : INFINITY;
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
      float pv = __ldcg(&((float*)partials)[2 * b]);
      t = (OP == TL_RED_MAX) ? fmaxf(t, pv) : fminf(t, pv);
    }
    t = (OP == TL_RED_MAX) ? warp_max(t) : warp_min(t);
    if (lane == 0) sh_f[wid] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 0; w < nw; ++w) t = (OP == TL_RED_MAX) ? fmaxf(t, sh_f[w]) : fminf(t, sh_f[w]);
      out[0] = t;
      *counter = 0u;
    }
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <int OP>
int launch_rows(const float* in, float* out, int64_t rows, int64_t cols, cudaStream_t st) {
  const unsigned grid = ceil_div_u(rows, 8);
  if (cols % 4 == 0 && aligned16(in))
    reduce_rows_kernel<OP, true><<<grid, 256, 0, st>>>(in, out, rows, cols);
  else
    reduce_rows_kernel<OP, false><<<grid, 256, 0, st>>>(in, out, rows, cols);
  return after_launch();
}

template <int OP>
int launch_cols(const float* in, float* out, int64_t rows, int64_t cols, void* scratch,
                cudaStream_t st) {
  const bool vec = (cols % 4 == 0) && aligned16(in);
  ColPlan p = col_plan(rows, cols, vec);
  if (p.gx > kMaxColBlocks) return TL_ERR_UNSUPPORTED;
  unsigned* counters = (unsigned*)scratch;
  void* partials = (char*)scratch + kCounterBytes;
  dim3 grid(p.gx, p.gy);
  if (vec)
    reduce_cols_kernel<OP, 4><<<grid, 256, 0, st>>>(in, out, rows, cols, p.chunk, counters, partials);
  else
    reduce_cols_kernel<OP, 1><<<grid, 256, 0, st>>>(in, out, rows, cols, p.chunk, counters, partials);
  return after_launch();
}

unsigned full_blocks(int64_t n) {
  int64_t b = (n + 4LL * 256 - 1) / (4LL * 256);
  int64_t cap = (int64_t)kFullBlocksPerSm * sm_count();  // exactly one resident wave
  if (cap > kFullMaxBlocks) cap = kFullMaxBlocks;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

template <int OP>
int launch_full(const float* in, float* out, int64_t n, void* scratch, cudaStream_t st) {
  unsigned* counter = (unsigned*)scratch;
  void* partials = (char*)scratch + kCounterBytes;
  const unsigned grid = full_blocks(n);
  if (n % 4 == 0 && aligned16(in))
    reduce_full_kernel<OP, true><<<grid, 256, 0, st>>>(in, out, n, counter, partials);
  else
    reduce_full_kernel<OP, false><<<grid, 256, 0, st>>>(in, out, n, counter, partials);
  return after_launch();
}

#define TL_DISPATCH_OP(op, F, ...)                          \
  switch (op) {                                             \
    case TL_RED_SUM: return F<TL_RED_SUM>(__VA_ARGS__);     \
    case TL_RED_MEAN: return F<TL_RED_MEAN>(__VA_ARGS__);   \
    case TL_RED_MAX: return F<TL_RED_MAX>(__VA_ARGS__);     \
    case TL_RED_MIN: return F<TL_RED_MIN>(__VA_ARGS__);     \
    case TL_RED_ARGMAX: return F<TL_RED_ARGMAX>(__VA_ARGS__); \
    case TL_RED_ARGMIN: return F<TL_RED_ARGMIN>(__VA_ARGS__); \
    default: return TL_ERR_INVALID_ARG;                     \
  }

}  // namespace
}  // namespace tl

extern "C" {

int tl_reduce_rows(int op, const float* in, float* out, int64_t rows, int64_t cols, void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  TL_DISPATCH_OP(op, tl::launch_rows, in, out, rows, cols, st);
}

size_t tl_reduce_cols_scratch_bytes(int op, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  tl::ColPlan p = tl::col_plan(rows, cols, cols % 4 == 0);
  tl::ColPlan q = tl::col_plan(rows, cols, false);
  unsigned gy = p.gy > q.gy ? p.gy : q.gy;
  return tl::kCounterBytes + (size_t)gy * (size_t)cols * tl::col_partial_bytes(op);
}

int tl_reduce_cols(int op, const float* in, float* out, int64_t rows, int64_t cols, void* scratch,
                   void* stream) {
  if (!in || !out || !scratch || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  TL_DISPATCH_OP(op, tl::launch_cols, in, out, rows, cols, scratch, st);
}

size_t tl_reduce_full_scratch_bytes(int op, int64_t n) {
  (void)op;
  (void)n;
  return tl::kCounterBytes + (size_t)tl::kFullMaxBlocks * 16;
}

int tl_reduce_full(int op, const float* in, float* out, int64_t n, void* scratch, void* stream) {
  if (!in || !out || !scratch || n <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  TL_DISPATCH_OP(op, tl::launch_full, in, out, n, scratch, st);
}

}  // extern "C"

// ===================================================== no-allocation variant
// Column reduction whose scratch is a file-scope device array instead of a
// caller-provided buffer, for callers that cannot allocate device memory
// (for example a plugin running inside a host framework that owns every
// device allocation, or a fixed-budget path that must not allocate while it
// runs).  The array is part of the module: every GPU that loads this library
// holds it until process exit.  Every call shares it, so calls whose kernels
// overlap on the GPU race; serialise them on one stream.
namespace tl {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress with the device current.  It is looked up on every
// call (cheap once the module is loaded), so it stays right after the
// device's context is reset and the module reloaded.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  TL_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
  *out = p;
  return TL_OK;
}

template <int OP>
int launch_cols_noalloc(const float* in, float* out, int64_t rows, int64_t cols, cudaStream_t st) {
  const bool vec = (cols % 4 == 0) && aligned16(in);
  ColPlan p = col_plan(rows, cols, vec);
  if (p.gx > kMaxColBlocks) return TL_ERR_UNSUPPORTED;  // as tl_reduce_cols
  // fewer row chunks, so that the partials fit in the static array
  const size_t per_chunk = (size_t)cols * col_partial_bytes(OP);
  const size_t fit = (kNoAllocScratchBytes - kCounterBytes) / per_chunk;
  if (fit < 1) return TL_ERR_INVALID_ARG;
  if (p.gy > fit) {
    p.chunk = (rows + (int64_t)fit - 1) / (int64_t)fit;
    p.gy = (unsigned)((rows + p.chunk - 1) / p.chunk);
  }
  void* base = nullptr;
  TL_TRY(noalloc_scratch(&base));
  // the completion counters must start at zero; the partials need no clearing
  TL_CUDA_TRY(cudaMemsetAsync(base, 0, (size_t)p.gx * sizeof(unsigned), st));
  unsigned* counters = (unsigned*)base;
  void* partials = (char*)base + kCounterBytes;
  dim3 grid(p.gx, p.gy);
  if (vec)
    reduce_cols_kernel<OP, 4><<<grid, 256, 0, st>>>(in, out, rows, cols, p.chunk, counters, partials);
  else
    reduce_cols_kernel<OP, 1><<<grid, 256, 0, st>>>(in, out, rows, cols, p.chunk, counters, partials);
  return after_launch();
}

}  // namespace
}  // namespace tl

extern "C" int tl_reduce_cols_noalloc(int op, const float* in, float* out, int64_t rows,
                                      int64_t cols, void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  if (op < TL_RED_SUM || op > TL_RED_ARGMIN) return TL_ERR_INVALID_ARG;
  // widest row whose single-chunk partials still fit in the static array
  const int64_t max_cols =
      (int64_t)((tl::kNoAllocScratchBytes - tl::kCounterBytes) / tl::col_partial_bytes(op));
  if (cols > max_cols) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  TL_DISPATCH_OP(op, tl::launch_cols_noalloc, in, out, rows, cols, st);
}
