// Elementwise and row kernels behind the f32 half of the op-level iris_gpu_*
// surface (iris_metal.h:353-566), which the reference's Z-Image GPU block
// (iris_transformer_zimage.c:934-1190) and the f32 fallbacks of its Flux
// single block (iris_transformer_flux.c:2637-3040) call.  The fused model
// path never uses them.  All are HBM-bound one-pass kernels.
//
//   layernorm_mod_f32  iris_gpu_adaln_norm         (1 + scale) * LN(x) + shift
//   head_rmsnorm_f32   iris_gpu_qk_rms_norm        per-head RMSNorm, in place
//   rope_pairs         iris_gpu_rope_* (f32, bf16) consecutive-pair rotation
//                      from [rows, table_ld] cos/sin tables (pair values
//                      duplicated, as the reference builds them)
//   silu_mul_f32, gated_add_f32, add_f32, add_bf16
#include "iris_kernels.h"

#include <cuda_bf16.h>
#include <stdint.h>

namespace {

inline int blocks_for(long n, int threads) {
  long b = (n + threads - 1) / threads;
  if (b > 148L * 32) b = 148L * 32;
  return (int)(b < 1 ? 1 : b);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  return warp_sum(l < 8 ? red[l] : 0.f);
}

// One 256-thread block per row; two passes over the row (mean, then the
// centred sum of squares) as apply_adaln does, eps inside the square root.
__global__ void __launch_bounds__(256)
layernorm_mod_f32_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ shift,
                         const float* __restrict__ scale, int cols, float eps) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * cols;
  float* o = out + (size_t)blockIdx.x * cols;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += 256) s += xr[c];
  const float mean = block_sum256(s, red) / (float)cols;
  float q = 0.f;
  for (int c = threadIdx.x; c < cols; c += 256) {
    const float d = xr[c] - mean;
    q += d * d;
  }
  const float rstd = 1.0f / sqrtf(block_sum256(q, red) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += 256)
    o[c] = (1.0f + scale[c]) * ((xr[c] - mean) * rstd) + shift[c];
}

// One warp per (row, head) of 128 values: x = x * rsqrt(mean(x^2) + eps) * w.
__global__ void __launch_bounds__(256)
head_rmsnorm_f32_kernel(float* __restrict__ x, int rows, int heads, const float* __restrict__ w, float eps) {
  const long item = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (long)rows * heads) return;
  float4* p = reinterpret_cast<float4*>(x + item * 128) + lane;
  float4 v = *p;
  const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
  const float r = 1.0f / sqrtf(ss / 128.0f + eps);
  const float4 g = reinterpret_cast<const float4*>(w)[lane];
  v.x *= r * g.x;
  v.y *= r * g.y;
  v.z *= r * g.z;
  v.w *= r * g.w;
  *p = v;
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ void from_f(float& d, float v) { d = v; }
__device__ __forceinline__ void from_f(__nv_bfloat16& d, float v) { d = __float2bfloat16_rn(v); }

// Rows [0, rows) of x [rows, heads * hd]; pair i of every head rotates by the
// table entry at column 2i of its row: (a, b) -> (a c - b s, b c + a s).
template <typename T>
__global__ void rope_pairs_kernel(T* __restrict__ x, int rows, int heads, int hd, const float* __restrict__ cs,
                                  const float* __restrict__ sn, int table_ld) {
  const int half = hd >> 1;
  const long n = (long)rows * heads * half;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int p = (int)(i % half);
    const long rh = i / half;
    const int row = (int)(rh / heads);
    T* e = x + rh * hd + 2 * p;
    const float c = cs[(size_t)row * table_ld + 2 * p], s = sn[(size_t)row * table_ld + 2 * p];
    const float a = to_f(e[0]), b = to_f(e[1]);
    from_f(e[0], a * c - b * s);
    from_f(e[1], b * c + a * s);
  }
}

__global__ void silu_mul_f32_kernel(float* __restrict__ g, const float* __restrict__ u, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float a = g[i];
    g[i] = a / (1.0f + __expf(-a)) * u[i];
  }
}

__global__ void gated_add_f32_kernel(float* __restrict__ out, const float* __restrict__ gate,
                                     const float* __restrict__ proj, int cols, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] += gate[i % cols] * proj[i];
}

__global__ void add_f32_kernel(float* out, const float* a, const float* b, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = a[i] + b[i];
}

__global__ void add_bf16_kernel(__nv_bfloat16* out, const __nv_bfloat16* a, const __nv_bfloat16* b, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(__bfloat162float(a[i]) + __bfloat162float(b[i]));
}

}  // namespace

extern "C" cudaError_t iris_launch_layernorm_mod_f32(float* out, const float* x, const float* shift,
                                                     const float* scale, int rows, int cols, float eps,
                                                     cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  layernorm_mod_f32_kernel<<<rows, 256, 0, stream>>>(out, x, shift, scale, cols, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_head_rmsnorm_f32(float* x, int rows, int heads, const float* w, float eps,
                                                    cudaStream_t stream) {
  const long items = (long)rows * heads;
  if (items <= 0) return cudaSuccess;
  if (reinterpret_cast<uintptr_t>(x) & 15 || reinterpret_cast<uintptr_t>(w) & 15) return cudaErrorInvalidValue;
  head_rmsnorm_f32_kernel<<<(int)((items + 7) / 8), 256, 0, stream>>>(x, rows, heads, w, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_rope_pairs(void* x, int bf16, int rows, int heads, int hd, const float* cs,
                                              const float* sn, int table_ld, cudaStream_t stream) {
  const long n = (long)rows * heads * (hd / 2);
  if (n <= 0) return cudaSuccess;
  if (hd & 1) return cudaErrorInvalidValue;
  if (bf16)
    rope_pairs_kernel<__nv_bfloat16><<<blocks_for(n, 256), 256, 0, stream>>>(
        static_cast<__nv_bfloat16*>(x), rows, heads, hd, cs, sn, table_ld);
  else
    rope_pairs_kernel<float><<<blocks_for(n, 256), 256, 0, stream>>>(static_cast<float*>(x), rows, heads, hd, cs,
                                                                      sn, table_ld);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_silu_mul_f32(float* gate, const float* up, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  silu_mul_f32_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(gate, up, n);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_gated_add_f32(float* out, const float* gate, const float* proj, int rows,
                                                 int cols, cudaStream_t stream) {
  const long n = (long)rows * cols;
  if (n <= 0) return cudaSuccess;
  gated_add_f32_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(out, gate, proj, cols, n);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_add_f32(float* out, const float* a, const float* b, long n,
                                           cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  add_f32_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(out, a, b, n);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_add_bf16(void* out, const void* a, const void* b, long n,
                                            cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  add_bf16_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(out),
                                                          static_cast<const __nv_bfloat16*>(a),
                                                          static_cast<const __nv_bfloat16*>(b), n);
  return cudaGetLastError();
}
