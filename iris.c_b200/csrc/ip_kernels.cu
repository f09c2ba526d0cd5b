// IP-Adapter kernels (reference: iris_ip_adapter.c; hooks
// iris_transformer_flux.c:2355-2365, :2440-2446, :2607-2612, :3848-3855, :3921-3926).
//
// Once per conditioning image (f32, the reference's precision, so the
// per-image embeddings and per-block K/V match it to f32 rounding):
//   ip_sgemm          C = A B^T or A B (+ bias): perceiver projections, FiLM,
//                     per-block ip_embeds @ stacked[block]
//   ip_colnorm        per-dimension standardisation over the token axis + affine
//   ip_layernorm      per-row LayerNorm (biased variance, eps 1e-5)
//   ip_film_tokens    token = q * (1 + scale) + shift
//   ip_mha            small multi-head cross-attention (perceiver: T queries)
//   ip_scale_rows     hybrid group gate on V rows
// Per step and adapted block (the image rows of the sequence):
//   ip_unrope         post-RoPE bf16 Q of the block -> the pre-RoPE Q the adapter
//                     attends with (the inverse rotation of each pair)
//   (tcgen05 attention over the adapter's T keys, attention_tc.cu)
//   ip_add            hidden += scale[block] * O  (scale read from device memory,
//                     so a per-step schedule needs no new graph)
// SREF: axpy_dev (temb += flag * CSD delta), silu_f32 (the CSD modulation MLP).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "iris_kernels.h"
#include "rope.cuh"

namespace {

constexpr int SG_T = 64;   // 64 x 64 output tile, 256 threads, 4 x 4 per thread
constexpr int SG_K = 16;

__global__ void __launch_bounds__(256)
ip_sgemm_kernel(const float* __restrict__ A, int lda, const float* __restrict__ B, int ldb, int transB,
                const float* __restrict__ bias, float* __restrict__ C, int ldc, int M, int N, int K, long sA,
                long sB, long sC) {
  __shared__ float As[SG_K][SG_T + 1];
  __shared__ float Bs[SG_K][SG_T + 1];
  A += sA * blockIdx.z;  // batch: one (A, B, C) triple per z
  B += sB * blockIdx.z;
  C += sC * blockIdx.z;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * SG_T, n0 = blockIdx.x * SG_T;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += SG_K) {
    for (int e = threadIdx.x; e < SG_T * SG_K; e += 256) {
      const int r = e / SG_K, k = e % SG_K;
      const int gm = m0 + r, gk = k0 + k;
      As[k][r] = (gm < M && gk < K) ? A[(size_t)gm * lda + gk] : 0.f;
      const int gn = n0 + r;
      float b = 0.f;
      if (gn < N && gk < K) b = transB ? B[(size_t)gn * ldb + gk] : B[(size_t)gk * ldb + gn];
      Bs[k][r] = b;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SG_K; k++) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = Bs[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int n = n0 + tx * 4 + j;
      if (n < N) C[(size_t)m * ldc + n] = acc[i][j] + (bias ? bias[n] : 0.f);
    }
  }
}

// out[t, d] = (x[t, d] - mean_d) / sqrt(var_d + eps) * g[d] + b[d], statistics over t
__global__ void ip_colnorm_kernel(const float* __restrict__ x, int n, int S, const float* __restrict__ g,
                                  const float* __restrict__ b, float* __restrict__ out) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= S) return;
  float mean = 0.f;
  for (int t = 0; t < n; t++) mean += x[(size_t)t * S + d];
  mean /= (float)n;
  float var = 0.f;
  for (int t = 0; t < n; t++) {
    const float e = x[(size_t)t * S + d] - mean;
    var += e * e;
  }
  var /= (float)n;
  const float inv = 1.0f / sqrtf(var + 1e-5f);
  for (int t = 0; t < n; t++) out[(size_t)t * S + d] = (x[(size_t)t * S + d] - mean) * inv * g[d] + b[d];
}

__device__ __forceinline__ float block_sum256(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) s += red[i];
  __syncthreads();
  return s;
}

// in place, one block per row
__global__ void __launch_bounds__(256)
ip_layernorm_kernel(float* __restrict__ x, int H, const float* __restrict__ w, const float* __restrict__ b) {
  __shared__ float red[8];
  float* r = x + (size_t)blockIdx.x * H;
  float s = 0.f;
  for (int d = threadIdx.x; d < H; d += 256) s += r[d];
  const float mean = block_sum256(s, red) / (float)H;
  float q = 0.f;
  for (int d = threadIdx.x; d < H; d += 256) {
    const float e = r[d] - mean;
    q += e * e;
  }
  const float inv = 1.0f / sqrtf(block_sum256(q, red) / (float)H + 1e-5f);
  for (int d = threadIdx.x; d < H; d += 256) r[d] = (r[d] - mean) * inv * w[d] + b[d];
}

__global__ void ip_film_tokens_kernel(const float* __restrict__ q, const float* __restrict__ film, int T, int H,
                                      float* __restrict__ out) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * H) return;
  const int d = (int)(i % H);
  out[i] = q[i] * (1.0f + film[d]) + film[H + d];
}

// out[t, h*hd : (h+1)*hd] = softmax(q_t,h . K_h^T / sqrt(hd)) V_h ; one block per (t, h)
__global__ void __launch_bounds__(256)
ip_mha_kernel(const float* __restrict__ Q, const float* __restrict__ K, const float* __restrict__ V, int n, int H,
              int hd, float* __restrict__ out) {
  extern __shared__ float sm[];  // scores [n] then q [hd]
  __shared__ float red[8];
  const int t = blockIdx.x, h = blockIdx.y;
  float* sc = sm;
  float* qs = sm + n;
  for (int d = threadIdx.x; d < hd; d += 256) qs[d] = Q[(size_t)t * H + h * hd + d];
  __syncthreads();
  const float scale = 1.0f / sqrtf((float)hd);
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < n; j += 256) {
    const float* kr = K + (size_t)j * H + h * hd;
    float s = 0.f;
    for (int d = 0; d < hd; d++) s = fmaf(qs[d], kr[d], s);
    s *= scale;
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int i = 1; i < 8; i++) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float s = 0.f;
  for (int j = threadIdx.x; j < n; j += 256) {
    const float p = expf(sc[j] - mx);
    sc[j] = p;
    s += p;
  }
  const float inv = 1.0f / block_sum256(s, red);  // includes the barrier that publishes sc
  for (int d = threadIdx.x; d < hd; d += 256) {
    float o = 0.f;
    for (int j = 0; j < n; j++) o = fmaf(sc[j], V[(size_t)j * H + h * hd + d], o);
    out[(size_t)t * H + h * hd + d] = o * inv;
  }
}

__global__ void ip_scale_rows_kernel(float* __restrict__ x, int rows, int H, int row_split, float s0, float s1) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)rows * H) return;
  x[i] *= (i / H) < row_split ? s0 : s1;
}

// q_pre = R^-1 q: each rotated pair (x0 c - x1 s, x1 c + x0 s) back to (x0, x1),
// with c, s evaluated from the row's position ids as the QKV epilogue does;
// grid (pairs / 256, rows): one thread per pair of one row
__global__ void ip_unrope_kernel(const __nv_bfloat16* __restrict__ q, int ldq, const uint16_t* __restrict__ pos,
                                 const IrisRopeSpec* __restrict__ spec, int H, __nv_bfloat16* __restrict__ out) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
  if (p >= H / 2) return;
  const int pr = p & 63;  // pair index inside its 128-wide head
  const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(q + (size_t)r * ldq + 2 * p);
  const float y0 = __bfloat162float(v.x), y1 = __bfloat162float(v.y);
  const int ax = (int)((__ldg(spec->axis_bits + pr / 16) >> (2 * (pr % 16))) & 3u);
  const uint32_t ps = iris::rope_axis_pos(iris::rope_load_pos(pos, r), ax);
  float c = 1.0f, s = 0.0f;
  if (ps != 0) iris::rope_cos_sin(ps, __ldg(spec->freq + pr), c, s);
  *reinterpret_cast<__nv_bfloat162*>(out + (size_t)r * H + 2 * p) =
      __floats2bfloat162_rn(y0 * c + y1 * s, y1 * c - y0 * s);
}

// grid (H / 4 / 256, rows): 4 columns per thread
__global__ void ip_add_kernel(float* __restrict__ hidden, int ldh, const __nv_bfloat16* __restrict__ o, int H,
                              const float* __restrict__ scale) {
  const int c4 = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
  if (c4 >= H / 4) return;
  const float s = __ldg(scale);
  const uint2 u = *reinterpret_cast<const uint2*>(o + (size_t)r * H + 4 * c4);
  float4* h = reinterpret_cast<float4*>(hidden + (size_t)r * ldh) + c4;
  float4 v = *h;
  v.x += s * __uint_as_float(u.x << 16);
  v.y += s * __uint_as_float(u.x & 0xFFFF0000u);
  v.z += s * __uint_as_float(u.y << 16);
  v.w += s * __uint_as_float(u.y & 0xFFFF0000u);
  *h = v;
}

// y += (*a) * x  (SREF: the CSD temb delta, gated per forward by a device flag)
__global__ void axpy_dev_kernel(float* __restrict__ y, const float* __restrict__ x, const float* __restrict__ a,
                                int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] += __ldg(a) * x[i];
}

__global__ void silu_f32_kernel(float* __restrict__ x, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = x[i] / (1.0f + expf(-x[i]));
}

inline unsigned blocks_for(long n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

extern "C" {

cudaError_t iris_launch_ip_sgemm(const float* A, int lda, const float* B, int ldb, int transB, const float* bias,
                                 float* C, int ldc, int M, int N, int K, cudaStream_t stream) {
  return iris_launch_ip_sgemm_batched(A, lda, 0, B, ldb, 0, transB, bias, C, ldc, 0, M, N, K, 1, stream);
}

cudaError_t iris_launch_ip_sgemm_batched(const float* A, int lda, long sA, const float* B, int ldb, long sB,
                                         int transB, const float* bias, float* C, int ldc, long sC, int M, int N,
                                         int K, int batch, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || batch <= 0) return cudaSuccess;
  if (K <= 0 || batch > 65535) return cudaErrorInvalidValue;
  dim3 grid((N + SG_T - 1) / SG_T, (M + SG_T - 1) / SG_T, batch);
  ip_sgemm_kernel<<<grid, 256, 0, stream>>>(A, lda, B, ldb, transB, bias, C, ldc, M, N, K, sA, sB, sC);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_colnorm(const float* x, int n, int S, const float* g, const float* b, float* out,
                                   cudaStream_t stream) {
  if (n <= 0 || S <= 0) return cudaSuccess;
  ip_colnorm_kernel<<<blocks_for(S, 128), 128, 0, stream>>>(x, n, S, g, b, out);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_layernorm(float* x, int rows, int H, const float* w, const float* b, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  ip_layernorm_kernel<<<rows, 256, 0, stream>>>(x, H, w, b);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_film_tokens(const float* q, const float* film, int T, int H, float* out,
                                       cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  ip_film_tokens_kernel<<<blocks_for((long)T * H, 256), 256, 0, stream>>>(q, film, T, H, out);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_mha(const float* Q, const float* K, const float* V, int T, int n, int H, int heads,
                               float* out, cudaStream_t stream) {
  if (T <= 0 || n <= 0) return cudaSuccess;
  if (heads <= 0 || H % heads) return cudaErrorInvalidValue;
  const int hd = H / heads;
  const size_t smem = (size_t)(n + hd) * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(ip_mha_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  ip_mha_kernel<<<dim3(T, heads), 256, smem, stream>>>(Q, K, V, n, H, hd, out);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_scale_rows(float* x, int rows, int H, int row_split, float s0, float s1,
                                      cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  ip_scale_rows_kernel<<<blocks_for((long)rows * H, 256), 256, 0, stream>>>(x, rows, H, row_split, s0, s1);
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_unrope(const void* q, int ldq, const uint16_t* pos, const IrisRopeSpec* spec, int rows,
                                  int H, void* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if ((H & 127) || (ldq & 1) || rows > 65535 || !pos || !spec) return cudaErrorInvalidValue;
  ip_unrope_kernel<<<dim3(blocks_for(H / 2, 256), rows), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, pos, spec, H, static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

cudaError_t iris_launch_ip_add(float* hidden, int ldh, const void* o, int rows, int H, const float* scale,
                               cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if ((H & 3) || (ldh & 3) || rows > 65535) return cudaErrorInvalidValue;
  ip_add_kernel<<<dim3(blocks_for(H / 4, 256), rows), 256, 0, stream>>>(hidden, ldh,
                                                                        static_cast<const __nv_bfloat16*>(o), H,
                                                                        scale);
  return cudaGetLastError();
}

cudaError_t iris_launch_axpy_dev(float* y, const float* x, const float* a, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  axpy_dev_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(y, x, a, n);
  return cudaGetLastError();
}

cudaError_t iris_launch_silu_f32(float* x, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  silu_f32_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(x, n);
  return cudaGetLastError();
}

}  // extern "C"
