// LoRA merge: W[rowmap[i], :] = bf16( f32(W0[rowmap[i], :]) + scale * (B A)[i, :] )
//
// The reference applies an adapter at run time after every adapted linear,
// out += scale * B (A x)  (lora_apply, iris_lora.c:43; hooks
// iris_transformer_flux.c:2429-2532, :3818, :3909).  Since the product is
// linear in x, W x + scale * B (A x) = (W + scale * B A) x: the backend folds
// each adapter into its resident bf16 weight once, so a step with a LoRA costs
// exactly what a step without one costs.  This kernel is that fold.
//
//   B    f32 [nrows, rank]  the adapter's up matrix, rows already in the
//                            device weight's row order (gate/up interleave,
//                            tensor-parallel shard)
//   A    f32 [rank, cols]   the down matrix, columns in the device order
//   rowmap int [nrows]      device row of B's row i
//   W0 / W bf16 [*, ld]     original and live weight (may alias)
//
// Tile 64 rows x 128 columns per 256-thread block, rank consumed in chunks of
// 32 through shared memory; each thread owns 4 rows x 8 contiguous columns, so
// its weight loads and stores are 16-byte vectors and a warp covers two
// 256-byte row segments.  The weight traffic (read W0, write W: 4 bytes per
// element) is the roofline for ranks up to ~32; the rank-r product is
// 2r FLOPs per element on the FP32 pipes.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int LM_ROWS = 64;
constexpr int LM_COLS = 128;
constexpr int LM_KC = 32;

__global__ void __launch_bounds__(256)
lora_merge_kernel(uint16_t* __restrict__ w, const uint16_t* __restrict__ w0, int ld,
                  const float* __restrict__ B, const float* __restrict__ A,
                  const int* __restrict__ rowmap, int nrows, int cols, int rank, float scale) {
  __shared__ float Bs[LM_ROWS][LM_KC + 1];
  __shared__ __align__(16) float As[LM_KC][LM_COLS];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;  // 16 column groups x 16 row groups
  const int row0 = blockIdx.y * LM_ROWS, col0 = blockIdx.x * LM_COLS;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < rank; k0 += LM_KC) {
    // B chunk: 64 x 32 (8 per thread), zero outside [nrows, rank)
    for (int e = tid; e < LM_ROWS * LM_KC; e += 256) {
      int r = e / LM_KC, k = e % LM_KC;
      int gr = row0 + r, gk = k0 + k;
      Bs[r][k] = (gr < nrows && gk < rank) ? B[(size_t)gr * rank + gk] : 0.f;
    }
    // A chunk: 32 x 128 (16 per thread), zero outside [rank, cols)
    for (int e = tid; e < LM_KC * LM_COLS; e += 256) {
      int k = e / LM_COLS, c = e % LM_COLS;
      int gk = k0 + k, gc = col0 + c;
      As[k][c] = (gk < rank && gc < cols) ? A[(size_t)gk * cols + gc] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < LM_KC; k++) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[k][tx * 8]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[k][tx * 8 + 4]);
      float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        float b = Bs[ty * 4 + i][k];
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = fmaf(b, a[j], acc[i][j]);
      }
    }
    __syncthreads();
  }

  const int c = col0 + tx * 8;
  if (c >= cols) return;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int r = row0 + ty * 4 + i;
    if (r >= nrows) break;
    size_t off = (size_t)rowmap[r] * ld + c;
    uint4 v = *reinterpret_cast<const uint4*>(w0 + off);
    uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float lo = __uint_as_float(u[j] << 16) + scale * acc[i][2 * j];
      float hi = __uint_as_float(u[j] & 0xFFFF0000u) + scale * acc[i][2 * j + 1];
      __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
      u[j] = *reinterpret_cast<uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(w + off) = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

}  // namespace

extern "C" cudaError_t iris_launch_lora_merge(void* w, const void* w0, int ld, const float* B,
                                              const float* A, const int* rowmap, int nrows, int cols,
                                              int rank, float scale, cudaStream_t stream) {
  if (nrows <= 0 || cols <= 0) return cudaSuccess;
  if (rank <= 0 || (cols & 7) || (ld & 7) || ld < cols) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(w0)) & 15) return cudaErrorInvalidValue;
  dim3 grid((cols + LM_COLS - 1) / LM_COLS, (nrows + LM_ROWS - 1) / LM_ROWS);
  if (grid.y > 65535) return cudaErrorInvalidValue;
  lora_merge_kernel<<<grid, 256, 0, stream>>>(static_cast<uint16_t*>(w), static_cast<const uint16_t*>(w0),
                                              ld, B, A, rowmap, nrows, cols, rank, scale);
  return cudaGetLastError();
}
