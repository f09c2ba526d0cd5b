// LoRA fold on the tensor cores:
//   W[drow[i], :] = bf16( W0[drow[i], :] + scale * (B A)[bsrc[i], :] )
//
// The reference applies an adapter at run time after every adapted linear,
// out += scale * B (A x)  (lora_apply, iris_lora.c:43; hooks
// iris_transformer_flux.c:2429-2532, :3818, :3909).  Since the product is
// linear in x, W x + scale * B (A x) = (W + scale * B A) x: the backend folds
// each adapter into its resident bf16 weight once, so a step with a LoRA costs
// exactly what a step without one costs.
//
// The rank-r product B A is a GEMM with K = r: two small prep kernels gather
// the adapter's operands straight from the file's bytes (bf16, f16 or f32) into
// K-major bf16 tiles, padded to K = 64 —
//   Bp [n, Kp]     row i = B's row bsrc[i] (the device row order: gate/up
//                  interleave, tensor-parallel shard)
//   At [cols, Kp]  row c = A's column acol(c)
// — and the tcgen05 GEMM (gemm.cu) runs with its IRIS_EPI_LORA_FOLD
// epilogue, which reads the base row from W0, adds scale * acc and stores the
// bf16 result.  bf16 adapters are exact operands.  f16 / f32 adapters are split
// into bf16 hi + lo parts, K = 4r: Bh·Ah + Bh·Al + Bl·Ah + Bl·Al — exact for f16
// (11 significant bits fit in hi + lo), 16 of f32's 24 bits otherwise.  With K
// this short the GEMM is bound by the weight traffic, 2 bytes read + 2 written
// per element.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "iris_kernels.h"

namespace {

__device__ __forceinline__ float lora_load(const void* p, size_t i, int dtype) {
  if (dtype == IRIS_LORA_BF16) return __uint_as_float((uint32_t) static_cast<const uint16_t*>(p)[i] << 16);
  if (dtype == IRIS_LORA_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

// K column k of an operand row with rank-r entries x(0..r-1): unsplit, k < r
// holds bf16(x_k); split, part = k / r holds the bf16 hi or lo part of
// x_{k mod r} (B parts hi, hi, lo, lo against A parts hi, lo, hi, lo).
__device__ __forceinline__ uint16_t lora_part(float x, bool lo_part) {
  const uint16_t hi = bf16_bits(x);
  if (!lo_part) return hi;
  return bf16_bits(x - __uint_as_float((uint32_t)hi << 16));
}

// one K-major operand row of kp bf16 values: value k from x(part, k mod r)
// via `get`, written as 16-byte stores
template <typename Get>
__device__ __forceinline__ void lora_row(uint16_t* __restrict__ row, int kp, int rank, int nparts, Get get) {
  uint4* d = reinterpret_cast<uint4*>(row);
  for (int k8 = 0; k8 < kp; k8 += 8) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint32_t h[2];
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int k = k8 + 2 * q + e, part = k / rank;
        h[e] = part < nparts ? get(part, k - part * rank) : 0u;
      }
      w[q] = h[0] | (h[1] << 16);
    }
    d[k8 >> 3] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Bp row i <- B row bsrc[i]; one thread per row (B parts: hi, hi, lo, lo)
__global__ void lora_prep_b_kernel(uint16_t* __restrict__ dst, int kp, const void* __restrict__ B, int dtype,
                                   int rank, const int* __restrict__ bsrc, int n, int split) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const size_t src = (size_t)__ldg(bsrc + i) * rank;
  lora_row(dst + (size_t)i * kp, kp, rank, split ? 4 : 1, [&](int part, int kk) -> uint32_t {
    return lora_part(lora_load(B, src + kk, dtype), split && part >= 2);
  });
}

// At row c <- A column acol(c); one thread per column, so that the threads of
// a warp read consecutive columns of A (A parts: hi, lo, hi, lo)
__global__ void lora_prep_a_kernel(uint16_t* __restrict__ dst, int kp, const void* __restrict__ A, int dtype,
                                   int rank, int in_dim, int cols, int seg, int off0, int off1, int split) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int sc = c < seg ? off0 + c : off1 + (c - seg);
  lora_row(dst + (size_t)c * kp, kp, rank, split ? 4 : 1, [&](int part, int kk) -> uint32_t {
    return lora_part(lora_load(A, (size_t)kk * in_dim + sc, dtype), split && (part & 1));
  });
}

}  // namespace

extern "C" size_t iris_lora_fold_scratch_bytes(int nrows, int cols, int rank, int split) {
  const int K = split ? 4 * rank : rank;
  const size_t kp = (size_t)((K + 63) / 64) * 64;
  return ((size_t)nrows + (size_t)cols) * kp * 2 + 256;
}

extern "C" cudaError_t iris_launch_lora_fold(const IrisLoraFold* f, void* scratch, size_t scratch_bytes,
                                             int* status, int num_sms, cudaStream_t stream, int* launches) {
  if (launches) *launches = 0;
  if (!f || f->nrows <= 0 || f->cols <= 0) return cudaSuccess;
  if (f->rank <= 0 || f->cols % 128 || f->ld % 8 || f->ld < f->cols || f->in_dim <= 0) return cudaErrorInvalidValue;
  if (f->b_dtype < 0 || f->b_dtype > 2 || f->a_dtype < 0 || f->a_dtype > 2) return cudaErrorInvalidValue;
  if (f->acol_seg < 0 || f->acol_seg > f->cols) return cudaErrorInvalidValue;
  if (((uintptr_t)f->w | (uintptr_t)f->w0) & 15) return cudaErrorInvalidValue;
  const int split = (f->b_dtype != IRIS_LORA_BF16 || f->a_dtype != IRIS_LORA_BF16) ? 1 : 0;
  const int K = split ? 4 * f->rank : f->rank;
  const int kp = (K + 63) / 64 * 64;
  if (iris_lora_fold_scratch_bytes(f->nrows, f->cols, f->rank, split) > scratch_bytes) return cudaErrorInvalidValue;
  uint16_t* bp = reinterpret_cast<uint16_t*>((reinterpret_cast<uintptr_t>(scratch) + 127) & ~uintptr_t(127));
  uint16_t* at = bp + (size_t)f->nrows * kp;  // nrows * kp * 2 bytes: a multiple of 128
  lora_prep_b_kernel<<<(f->nrows + 127) / 128, 128, 0, stream>>>(bp, kp, f->B, f->b_dtype, f->rank, f->bsrc,
                                                                  f->nrows, split);
  lora_prep_a_kernel<<<(f->cols + 127) / 128, 128, 0, stream>>>(at, kp, f->A, f->a_dtype, f->rank, f->in_dim,
                                                                f->cols, f->acol_seg, f->acol_off0, f->acol_off1,
                                                                split);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  IrisGemmParams p;
  memset(&p, 0, sizeof(p));
  if (iris_make_tmap_bf16(&p.tmap_a, bp, f->nrows, kp, kp, 128) ||
      iris_make_tmap_bf16(&p.tmap_b[0], at, f->cols, kp, kp, 128))
    return cudaErrorInvalidValue;
  p.ngroups = 1;
  p.row0[0] = 0;
  p.rows[0] = f->nrows;
  p.N = f->cols;
  p.K = kp;
  p.bn = f->cols % 256 == 0 ? 256 : 128;
  p.mode = IRIS_EPI_LORA_FOLD;
  p.out = f->w;
  p.ldo = f->ld;
  p.fold_rows = f->drow;
  p.fold_w0 = f->w0;
  p.fold_scale = f->scale;
  p.status = status;
  p.splitk = 1;
  int n = 0;
  e = iris_launch_gemm_ex(&p, num_sms, stream, &n);
  if (launches) *launches = 2 + n;
  return e;
}
