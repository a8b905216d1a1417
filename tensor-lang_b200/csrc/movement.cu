// Data movement: transpose, slice, concat.
//
// Replaces transpose (kernel_generator.py:1949-1972, a naive uncoalesced
// 16x16 kernel), slice (:1112-1240) and concat along axis 0 (:2092-2132).
// Transpose goes through 32x32 shared-memory tiles (padded against bank
// conflicts) so both the read and the write are coalesced; slice is a pitched
// copy; concat of row-major tensors along axis 0 is two contiguous copies.
#include "tl_common.cuh"

namespace tl {
namespace {

__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ in,
                                                        float* __restrict__ out, int64_t rows,
                                                        int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t bx = (int64_t)blockIdx.x * 32, by = (int64_t)blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    int64_t r = by + ty + k, c = bx + tx;
    if (r < rows && c < cols) tile[ty + k][tx] = in[r * cols + c];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    int64_t r = bx + ty + k, c = by + tx;  // out is [cols, rows]
    if (r < cols && c < rows) out[r * rows + c] = tile[tx][ty + k];
  }
}

}  // namespace
}  // namespace tl

extern "C" {

int tl_transpose2d(const float* in, float* out, int64_t rows, int64_t cols, void* stream) {
  if (!in || !out || rows <= 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  if ((rows + 31) / 32 > 65535) return TL_ERR_UNSUPPORTED;
  cudaStream_t st = tl::stream_or_default(stream);
  dim3 grid(tl::ceil_div_u(cols, 32), tl::ceil_div_u(rows, 32));
  tl::transpose_kernel<<<grid, 256, 0, st>>>(in, out, rows, cols);
  return tl::after_launch();
}

int tl_slice2d(const float* in, float* out, int64_t in_cols, int64_t row_start, int64_t col_start,
               int64_t out_rows, int64_t out_cols, void* stream) {
  if (!in || !out || in_cols <= 0 || row_start < 0 || col_start < 0) return TL_ERR_INVALID_ARG;
  if (out_rows <= 0 || out_cols <= 0) return TL_OK;
  cudaStream_t st = tl::stream_or_default(stream);
  TL_CUDA_TRY(cudaMemcpy2DAsync(out, (size_t)out_cols * 4, in + row_start * in_cols + col_start,
                                (size_t)in_cols * 4, (size_t)out_cols * 4, (size_t)out_rows,
                                cudaMemcpyDeviceToDevice, st));
  return TL_OK;
}

int tl_concat_rows(const float* a, const float* b, float* out, int64_t rows_a, int64_t rows_b,
                   int64_t cols, void* stream) {
  if (!a || !b || !out || rows_a < 0 || rows_b < 0 || cols <= 0) return TL_ERR_INVALID_ARG;
  cudaStream_t st = tl::stream_or_default(stream);
  if (rows_a)
    TL_CUDA_TRY(cudaMemcpyAsync(out, a, (size_t)rows_a * cols * 4, cudaMemcpyDeviceToDevice, st));
  if (rows_b)
    TL_CUDA_TRY(cudaMemcpyAsync(out + rows_a * cols, b, (size_t)rows_b * cols * 4,
                                cudaMemcpyDeviceToDevice, st));
  return TL_OK;
}

}  // extern "C"
