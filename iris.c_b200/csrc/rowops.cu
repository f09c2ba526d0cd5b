// Row-wise and elementwise kernels of the DiT step (everything that is not a
// GEMM or attention).  All are HBM-bound: each reads its inputs once with
// 16-byte vector accesses and writes its outputs once.
//
//   adaln            apply_adaln           iris_transformer_flux.c:1391-1460
//   gemv             modulation / time-embedding linears (:1366, :4059-4069,
//                    :3787-3797, :4270-4281; zimage.c:563-585, :798-808)
//   timestep_sincos  get_timestep_embedding  iris_transformer_flux.c:1349
//   nchw_to_tokens   NCHW -> NLC transpose   iris_transformer_flux.c:3986-3993
//   euler            iris_axpy / CFG combine iris_sample.c:359, :768-771
//   head_rmsnorm_rope apply_qk_norm + apply_rope_2d (:1464, :1026) for the
//                    op-level iris_gpu_* surface
//   rmsnorm          zi_rms_norm             iris_transformer_zimage.c:657
#include "iris_kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// block-wide sum for 256 threads
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// ------------------------------------------------------------------ adaLN
// One 256-thread block per row; the row (cols <= 8192) is held in registers
// between the mean pass, the variance pass and the output pass.
constexpr int ADALN_MAXV = 8;  // float4 per thread

__global__ void __launch_bounds__(256)
adaln_kernel(const float* __restrict__ x, int ldx, __nv_bfloat16* __restrict__ out, int ldout,
             int cols, const float* __restrict__ shift0, const float* __restrict__ scale0,
             const float* __restrict__ shift1, const float* __restrict__ scale1, int split,
             float eps) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  iris::grid_dep_wait();
  iris::grid_dep_launch();
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * ldx);
  const int nv = cols >> 2;
  float4 v[ADALN_MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; i++) {
    int c = threadIdx.x + i * 256;
    if (c < nv) {
      v[i] = xr[c];
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  const float mean = block_sum(s, red) / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; i++) {
    int c = threadIdx.x + i * 256;
    if (c < nv) {
      float a = v[i].x - mean, b = v[i].y - mean, cc = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (cc * cc + d * d);
    }
  }
  const float var = block_sum(q, red) / (float)cols;
  const float rstd = 1.0f / sqrtf(var + eps);
  const bool g1 = row >= split;
  const float4* sh = reinterpret_cast<const float4*>(g1 ? shift1 : shift0);
  const float4* sc = reinterpret_cast<const float4*>(g1 ? scale1 : scale0);
  uint2* o = reinterpret_cast<uint2*>(out + (size_t)row * ldout);
#pragma unroll
  for (int i = 0; i < ADALN_MAXV; i++) {
    int c = threadIdx.x + i * 256;
    if (c < nv) {
      float4 a = __ldg(sh + c), b = __ldg(sc + c);
      float y0 = (1.0f + b.x) * ((v[i].x - mean) * rstd) + a.x;
      float y1 = (1.0f + b.y) * ((v[i].y - mean) * rstd) + a.y;
      float y2 = (1.0f + b.z) * ((v[i].z - mean) * rstd) + a.z;
      float y3 = (1.0f + b.w) * ((v[i].w - mean) * rstd) + a.w;
      o[c] = make_uint2(pack2(y0, y1), pack2(y2, y3));
    }
  }
}

// Warp-per-row variant for rows of NV*128 floats (H = 3072 / 4096): the whole
// row sits in registers (NV float4 per lane), both reductions are warp
// shuffles (no shared memory or block barriers), and every load of the row is
// issued before the first reduction, so each warp keeps NV*512 bytes in
// flight.  One-warp blocks: the register budget allows ~11 such warps per SM,
// so a 1536-row launch runs as a single wave.  Same two-pass mean / variance
// as the block kernel above.
template <int NV>
__global__ void __launch_bounds__(32)
adaln_warp_kernel(float* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ delta, int ld_delta,
                  __nv_bfloat16* __restrict__ out, int ldout, int rows,
                  const float* __restrict__ shift0, const float* __restrict__ scale0,
                  const float* __restrict__ shift1, const float* __restrict__ scale1, int split, float eps) {
  const int row = blockIdx.x;
  const int lane = threadIdx.x;
  if (row >= rows) return;
  iris::grid_dep_wait();
  iris::grid_dep_launch();
  constexpr int cols = NV * 128;
  float4* xr = reinterpret_cast<float4*>(x + (size_t)row * ldx);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) v[i] = xr[lane + 32 * i];
  if (delta) {  // pending tensor-parallel residual update, folded in here
    const uint2* dr = reinterpret_cast<const uint2*>(delta + (size_t)row * ld_delta);
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const uint2 d = dr[lane + 32 * i];
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&d.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&d.y));
      v[i].x += a.x;
      v[i].y += a.y;
      v[i].z += b.x;
      v[i].w += b.y;
      xr[lane + 32 * i] = v[i];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; i++) {
    float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b * b) + (c * c + d * d);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = 1.0f / sqrtf(q / (float)cols + eps);
  const bool g1 = row >= split;
  const float4* sh = reinterpret_cast<const float4*>(g1 ? shift1 : shift0);
  const float4* sc = reinterpret_cast<const float4*>(g1 ? scale1 : scale0);
  uint2* o = reinterpret_cast<uint2*>(out + (size_t)row * ldout);
#pragma unroll
  for (int i = 0; i < NV; i++) {
    const int c = lane + 32 * i;
    float4 a = __ldg(sh + c), b = __ldg(sc + c);
    float y0 = (1.0f + b.x) * ((v[i].x - mean) * rstd) + a.x;
    float y1 = (1.0f + b.y) * ((v[i].y - mean) * rstd) + a.y;
    float y2 = (1.0f + b.z) * ((v[i].z - mean) * rstd) + a.z;
    float y3 = (1.0f + b.w) * ((v[i].w - mean) * rstd) + a.w;
    o[c] = make_uint2(pack2(y0, y1), pack2(y2, y3));
  }
}

__global__ void add_bf16_rows_kernel(float* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ d, int ldd,
                                     int cols) {
  const int row = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (c >= cols) return;
  float4* xp = reinterpret_cast<float4*>(x + (size_t)row * ldx + c);
  const uint2 dv = *reinterpret_cast<const uint2*>(d + (size_t)row * ldd + c);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dv.y));
  float4 v = *xp;
  v.x += a.x;
  v.y += a.y;
  v.z += b.x;
  v.w += b.y;
  *xp = v;
}

// Tensor-parallel adaLN (see IrisAdalnTpArgs): one warp per owned row, the
// partial updates of every rank summed in rank order (exact f32 sums, the
// same order on every rank), the bf16 output row stored into every rank's
// xmod buffer over NVLink, then one xmod-arrival signal per launch.
template <int NV>
__global__ void __launch_bounds__(32) adaln_tp_kernel(const __grid_constant__ IrisAdalnTpArgs a) {
  const int i = blockIdx.x, lane = threadIdx.x;
  const int row = a.row0 + i;
  bool ok = true;
  if (a.has_part) {
    if (lane == 0) ok = iris::tp_wait(a.tp, IRIS_TP_PART, IRIS_TP_BASE_PART, a.part_index, a.status);
    ok = __shfl_sync(0xffffffffu, ok, 0);
  }
  if (ok && i < a.rows && row >= a.row_lo) {
    constexpr int cols = NV * 128;
    float4* xr = reinterpret_cast<float4*>(a.x + (size_t)row * a.H);
    float4 v[NV];
#pragma unroll
    for (int q = 0; q < NV; q++) v[q] = xr[lane + 32 * q];
    if (a.has_part) {
      for (int s = 0; s < a.tp.size; s++) {
        const float4* pr = reinterpret_cast<const float4*>(a.recv + ((size_t)s * a.chunk + i) * a.H);
#pragma unroll
        for (int q = 0; q < NV; q++) {
          const float4 d = pr[lane + 32 * q];
          v[q].x += d.x;
          v[q].y += d.y;
          v[q].z += d.z;
          v[q].w += d.w;
        }
      }
#pragma unroll
      for (int q = 0; q < NV; q++) xr[lane + 32 * q] = v[q];
    }
    if (a.xmod[0]) {
      float sum = 0.f;
#pragma unroll
      for (int q = 0; q < NV; q++) sum += (v[q].x + v[q].y) + (v[q].z + v[q].w);
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float mean = sum / (float)cols;
      float sq = 0.f;
#pragma unroll
      for (int q = 0; q < NV; q++) {
        float b0 = v[q].x - mean, b1 = v[q].y - mean, b2 = v[q].z - mean, b3 = v[q].w - mean;
        sq += (b0 * b0 + b1 * b1) + (b2 * b2 + b3 * b3);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      const float rstd = 1.0f / sqrtf(sq / (float)cols + a.eps);
      const bool g1 = row >= a.split;
      const float4* sh = reinterpret_cast<const float4*>(g1 ? a.shift1 : a.shift0);
      const float4* sc = reinterpret_cast<const float4*>(g1 ? a.scale1 : a.scale0);
#pragma unroll
      for (int q = 0; q < NV; q++) {
        const int c = lane + 32 * q;
        const float4 s4 = __ldg(sh + c), k4 = __ldg(sc + c);
        const uint2 o = make_uint2(pack2((1.0f + k4.x) * ((v[q].x - mean) * rstd) + s4.x,
                                         (1.0f + k4.y) * ((v[q].y - mean) * rstd) + s4.y),
                                   pack2((1.0f + k4.z) * ((v[q].z - mean) * rstd) + s4.z,
                                         (1.0f + k4.w) * ((v[q].w - mean) * rstd) + s4.w));
        for (int p = 0; p < a.tp.size; p++)
          reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.xmod[p]) + (size_t)row * a.H)[c] = o;
      }
    }
  }
  if (a.xmod[0]) {
    __syncwarp();
    if (lane == 0) iris::tp_signal(a.tp, IRIS_TP_DONE_ADALN, IRIS_TP_X, gridDim.x);
  }
}

__global__ void tp_barrier_kernel(const __grid_constant__ IrisTpParams tp, int* status) {
  unsigned* own = tp.flags[tp.rank];
  iris::fence_acq_rel_sys();
  for (int p = 0; p < tp.size; p++) iris::red_release_sys_add(tp.flags[p] + IRIS_TP_BAR + tp.rank, 1u);
  if (iris::tp_wait(tp, IRIS_TP_BAR, IRIS_TP_BASE_BAR, 1u, status)) own[IRIS_TP_BASE_BAR] += 1u;
}

__global__ void tp_advance_kernel(unsigned* flags, unsigned parts, unsigned xs) {
  flags[IRIS_TP_BASE_PART] += parts;
  flags[IRIS_TP_BASE_X] += xs;
}

// ------------------------------------------------------------------ GEMV
// One warp per output row; x (after the optional SiLU) is staged in shared
// memory; W rows are read with 16-byte loads.
__global__ void __launch_bounds__(256)
gemv_kernel(const __nv_bfloat16* __restrict__ w, const float* __restrict__ x,
            const float* __restrict__ bias, float* __restrict__ y, int n, int k, int act_in,
            int act_out) {
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    float v = x[i];
    xs[i] = act_in ? silu_f(v) : v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= n) return;
  const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)row * k);
  float acc = 0.f;
  for (int c = lane; c < (k >> 3); c += 32) {
    uint4 u = __ldg(wr + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float* xv = xs + c * 8;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      float2 f = __bfloat1622float2(h[e]);
      acc += f.x * xv[2 * e] + f.y * xv[2 * e + 1];
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    if (bias) acc += bias[row];
    y[row] = act_out ? silu_f(acc) : acc;
  }
}

// ------------------------------------------------------------------ timestep embedding
__global__ void timestep_sincos_kernel(const float* __restrict__ t_dev, float t_scale,
                                       float* __restrict__ out, int dim) {
  int half = dim >> 1;
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= half) return;
  float t = t_dev[0] * t_scale;
  float freq = expf(-logf(10000.0f) * (float)i / (float)half);
  float a = t * freq;
  out[i] = cosf(a);
  out[i + half] = sinf(a);
}

// ------------------------------------------------------------------ layout transforms
__global__ void nchw_to_tokens_kernel(const float* __restrict__ x, int c, int n,
                                      __nv_bfloat16* __restrict__ out, int ldo) {
  __shared__ float tile[32][33];
  int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    int ch = c0 + r, p = p0 + tx;
    tile[r][tx] = (ch < c && p < n) ? x[(size_t)ch * n + p] : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    int p = p0 + r, ch = c0 + tx;
    if (p < n && ch < c) out[(size_t)p * ldo + ch] = __float2bfloat16_rn(tile[tx][r]);
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ out,
                                   long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = __float2bfloat16_rn(x[i]);
}

__global__ void f16_to_bf16_kernel(const __half* __restrict__ x, __nv_bfloat16* __restrict__ out, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = __float2bfloat16_rn(__half2float(x[i]));
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ out,
                                   long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = __bfloat162float(x[i]);
}

__global__ void euler_kernel(float* __restrict__ z, const float* __restrict__ v,
                             const float* __restrict__ vu, float g, float dt, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    float vel = vu ? vu[i] + g * (v[i] - vu[i]) : v[i];
    z[i] += dt * vel;
  }
}

// ------------------------------------------------------------------ seeded RNG
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float hash_normal(uint64_t seed, uint64_t sid, uint64_t i) {
  uint64_t h = mix64(seed * 0x9e3779b97f4a7c15ull + mix64(sid + 0x632be59bd9b4e019ull) + i);
  uint64_t h2 = mix64(h ^ 0xd1b54a32d192ed03ull);
  float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  float u2 = (float)(h2 >> 40) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void randn_bf16_kernel(__nv_bfloat16* out, long n, uint64_t seed, uint64_t sid,
                                  float mean, float std) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = __float2bfloat16_rn(mean + std * hash_normal(seed, sid, i));
}

__global__ void randn_f32_kernel(float* out, long n, uint64_t seed, uint64_t sid, float mean,
                                 float std) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = mean + std * hash_normal(seed, sid, i);
}

// ------------------------------------------------------------------ op-level helpers
// In-place per-head RMSNorm (w may be NULL: no norm) and pair RoPE (cos may be
// NULL: no rotation) on bf16 [rows, ld]; one warp per (row, head), 4 elements per lane.
__global__ void head_rmsnorm_rope_kernel(__nv_bfloat16* x, int ld, int rows, int heads,
                                         const float* __restrict__ w, float eps,
                                         const float* __restrict__ rc,
                                         const float* __restrict__ rs) {
  int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (gw >= rows * heads) return;
  int row = gw / heads, h = gw - row * heads;
  uint2* p = reinterpret_cast<uint2*>(x + (size_t)row * ld + h * 128) + lane;
  uint2 u = *p;
  float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
  float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
  float v[4] = {a.x, a.y, b.x, b.y};
  if (w) {
    float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    float r = 1.0f / sqrtf(ss / 128.0f + eps);
#pragma unroll
    for (int e = 0; e < 4; e++) v[e] = v[e] * r * w[lane * 4 + e];
  }
  if (rc) {
#pragma unroll
    for (int pr = 0; pr < 2; pr++) {
      float c = rc[(size_t)row * 64 + lane * 2 + pr], s = rs[(size_t)row * 64 + lane * 2 + pr];
      float x0 = v[2 * pr], x1 = v[2 * pr + 1];
      v[2 * pr] = x0 * c - x1 * s;
      v[2 * pr + 1] = x1 * c + x0 * s;
    }
  }
  *p = make_uint2(pack2(v[0], v[1]), pack2(v[2], v[3]));
}

__global__ void silu_mul_bf16_kernel(__nv_bfloat16* gate, const __nv_bfloat16* up, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    float g = __bfloat162float(gate[i]);
    gate[i] = __float2bfloat16_rn(silu_f(g) * __bfloat162float(up[i]));
  }
}

__global__ void gated_add_bf16_kernel(__nv_bfloat16* out, const __nv_bfloat16* gate,
                                      const __nv_bfloat16* proj, int rows, int cols) {
  long n = (long)rows * cols;
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    int c = (int)(i % cols);
    float o = __bfloat162float(out[i]) + __bfloat162float(gate[c]) * __bfloat162float(proj[i]);
    out[i] = __float2bfloat16_rn(o);
  }
}

// out = x * rsqrt(mean(x^2) + eps) * w [* mul]; one block per row
__global__ void __launch_bounds__(256)
rmsnorm_kernel(const float* __restrict__ x, int ldx, const float* __restrict__ w,
               float* __restrict__ out_f32, __nv_bfloat16* __restrict__ out_bf16, int ldout,
               int cols, float eps, const float* __restrict__ mul) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  const float* xr = x + (size_t)row * ldx;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += 256) s += xr[c] * xr[c];
  float r = 1.0f / sqrtf(block_sum(s, red) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += 256) {
    float y = xr[c] * r * w[c];
    if (mul) y *= mul[c];
    if (out_f32) out_f32[(size_t)row * ldout + c] = y;
    if (out_bf16) out_bf16[(size_t)row * ldout + c] = __float2bfloat16_rn(y);
  }
}

// Warp-per-row RMSNorm for rows of NV*128 floats (Z-Image D = 3840, caption
// 2560): the row in registers, one shuffle reduction, 16-byte loads and
// 8-byte bf16 stores.  Same arithmetic as rmsnorm_kernel.
template <int NV>
__global__ void __launch_bounds__(32)
rmsnorm_warp_kernel(const float* __restrict__ x, int ldx, const float* __restrict__ w, float* __restrict__ out_f32,
                    __nv_bfloat16* __restrict__ out_bf16, int ldout, float eps, const float* __restrict__ mul) {
  const int row = blockIdx.x, lane = threadIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * ldx);
  float4 v[NV];
#pragma unroll
  for (int q = 0; q < NV; q++) v[q] = xr[lane + 32 * q];
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < NV; q++) s += (v[q].x * v[q].x + v[q].y * v[q].y) + (v[q].z * v[q].z + v[q].w * v[q].w);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float r = 1.0f / sqrtf(s / (float)(NV * 128) + eps);
#pragma unroll
  for (int q = 0; q < NV; q++) {
    const int c = lane + 32 * q;
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w) + c);
    float4 y = make_float4(v[q].x * r * ww.x, v[q].y * r * ww.y, v[q].z * r * ww.z, v[q].w * r * ww.w);
    if (mul) {
      const float4 m = __ldg(reinterpret_cast<const float4*>(mul) + c);
      y.x *= m.x;
      y.y *= m.y;
      y.z *= m.z;
      y.w *= m.w;
    }
    if (out_f32) reinterpret_cast<float4*>(out_f32 + (size_t)row * ldout)[c] = y;
    if (out_bf16)
      reinterpret_cast<uint2*>(out_bf16 + (size_t)row * ldout)[c] = make_uint2(pack2(y.x, y.y), pack2(y.z, y.w));
  }
}

__global__ void copy_rows_bf16_kernel(uint16_t* dst, int ldd, const uint16_t* src, int lds,
                                      int rows, int cols) {
  long n = (long)rows * cols;
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    long r = i / cols, c = i - r * cols;
    dst[r * ldd + c] = src[r * lds + c];
  }
}

// dst [2F, cols] row r: block b = r / 256, w = r % 256 takes gate row b*128+w
// (w < 128) or up row F + b*128 + w-128 of src [2F, cols] = [gate; up].
__global__ void interleave_gate_up_kernel(uint4* dst, const uint4* src, int F, int cols8) {
  int r = blockIdx.x;
  int b = r >> 8, w = r & 255;
  int sr = (w < 128) ? (b * 128 + w) : (F + b * 128 + (w - 128));
  for (int c = threadIdx.x; c < cols8; c += blockDim.x)
    dst[(size_t)r * cols8 + c] = src[(size_t)sr * cols8 + c];
}

// ------------------------------------------------------------------ Z-Image
// x[r] += gate * RMSNorm(y[r]) * w   (gate NULL = 1): the post-norm gated
// residual of zi_block_forward (iris_transformer_zimage.c:831-835, :845-849).
__global__ void __launch_bounds__(256)
resid_rmsnorm_gate_kernel(float* __restrict__ x, int ldx, const float* __restrict__ y, int ldy,
                          const float* __restrict__ w, const float* __restrict__ gate, int cols,
                          float eps) {
  __shared__ float red[8];
  const int row = blockIdx.x;
  const float* yr = y + (size_t)row * ldy;
  float* xr = x + (size_t)row * ldx;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += 256) s += yr[c] * yr[c];
  const float r = 1.0f / sqrtf(block_sum(s, red) / (float)cols + eps);
  for (int c = threadIdx.x; c < cols; c += 256) {
    float v = yr[c] * r * w[c];
    xr[c] += gate ? gate[c] * v : v;
  }
}

// per block of 4*dim modulation values: [1+scale_msa | tanh(gate_msa) | 1+scale_mlp | tanh(gate_mlp)]
// (zi_block_forward :812-818)
__global__ void zi_mod_transform_kernel(float* m, int dim, long n) {
  long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  long stride = (long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    int part = (int)((i / dim) & 3);
    m[i] = (part & 1) ? tanhf(m[i]) : 1.0f + m[i];
  }
}

// latent [C, H, W] f32 -> tokens [H/ps * W/ps, ps*ps*C] bf16 in (ph, pw, c) order (zi_patchify :1634)
__global__ void patchify_kernel(const float* __restrict__ lat, int c, int H, int W, int ps,
                                __nv_bfloat16* __restrict__ out, int ldo) {
  const int wt = W / ps;
  const int pf = ps * ps * c;
  const int tok = blockIdx.x;
  const int ty = tok / wt, tx = tok - ty * wt;
  for (int j = threadIdx.x; j < pf; j += blockDim.x) {
    int ch = j % c, pp = j / c, pw = pp % ps, ph = pp / ps;
    out[(size_t)tok * ldo + j] = __float2bfloat16_rn(lat[((size_t)ch * H + ty * ps + ph) * W + tx * ps + pw]);
  }
}

// tokens f32 [n, ldt] (first ps*ps*C columns) -> latent [C, H, W] (zi_unpatchify :1663)
__global__ void unpatchify_kernel(const float* __restrict__ tok, int ldt, int c, int H, int W, int ps,
                                  float* __restrict__ lat) {
  const int wt = W / ps;
  const int pf = ps * ps * c;
  const int t = blockIdx.x;
  const int ty = t / wt, tx = t - ty * wt;
  for (int j = threadIdx.x; j < pf; j += blockDim.x) {
    int ch = j % c, pp = j / c, pw = pp % ps, ph = pp / ps;
    lat[((size_t)ch * H + ty * ps + ph) * W + tx * ps + pw] = tok[(size_t)t * ldt + j];
  }
}

// rows [0, n) of dst (row stride ld) = vec [cols]
__global__ void fill_rows_f32_kernel(float* dst, int ld, const float* __restrict__ vec, int n, int cols) {
  for (int r = blockIdx.x; r < n; r += gridDim.x)
    for (int c = threadIdx.x; c < cols; c += blockDim.x) dst[(size_t)r * ld + c] = vec[c];
}

inline int grid_for(long n, int threads) {
  long b = (n + threads - 1) / threads;
  if (b > 148 * 16) b = 148 * 16;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

extern "C" {

cudaError_t iris_launch_adaln(const float* x, int ldx, void* out, int ldout, int rows, int cols,
                              const float* shift0, const float* scale0, const float* shift1,
                              const float* scale1, int split, float eps, cudaStream_t stream) {
  return iris_launch_adaln_delta(const_cast<float*>(x), ldx, nullptr, 0, out, ldout, rows, cols, shift0, scale0,
                                 shift1, scale1, split, eps, stream);
}

cudaError_t iris_launch_adaln_tp(const IrisAdalnTpArgs* a, cudaStream_t stream) {
  if (a->chunk <= 0) return cudaSuccess;
  if (a->H == 3072)
    adaln_tp_kernel<24><<<a->chunk, 32, 0, stream>>>(*a);
  else if (a->H == 4096)
    adaln_tp_kernel<32><<<a->chunk, 32, 0, stream>>>(*a);
  else if (a->H == 1024)
    adaln_tp_kernel<8><<<a->chunk, 32, 0, stream>>>(*a);
  else if (a->H == 2048)
    adaln_tp_kernel<16><<<a->chunk, 32, 0, stream>>>(*a);
  else if (a->H == 512)
    adaln_tp_kernel<4><<<a->chunk, 32, 0, stream>>>(*a);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t iris_launch_tp_barrier(const IrisTpParams* tp, int* status, cudaStream_t stream) {
  tp_barrier_kernel<<<1, 1, 0, stream>>>(*tp, status);
  return cudaGetLastError();
}

cudaError_t iris_launch_tp_advance(unsigned* flags, unsigned parts, unsigned xs, cudaStream_t stream) {
  tp_advance_kernel<<<1, 1, 0, stream>>>(flags, parts, xs);
  return cudaGetLastError();
}

cudaError_t iris_launch_add_bf16_rows(float* x, int ldx, const void* delta, int ld_delta, int rows, int cols,
                                      cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if ((cols & 3) || (ldx & 3) || (ld_delta & 3)) return cudaErrorInvalidValue;
  add_bf16_rows_kernel<<<dim3((cols / 4 + 255) / 256, rows), 256, 0, stream>>>(
      x, ldx, static_cast<const __nv_bfloat16*>(delta), ld_delta, cols);
  return cudaGetLastError();
}

cudaError_t iris_launch_adaln_delta(float* x, int ldx, const void* delta_v, int ld_delta, void* out, int ldout,
                                    int rows, int cols, const float* shift0, const float* scale0,
                                    const float* shift1, const float* scale1, int split, float eps,
                                    cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if ((cols & 3) || cols > 256 * 4 * ADALN_MAXV || (ldx & 3) || (ldout & 3) || (ld_delta & 3))
    return cudaErrorInvalidValue;
  const __nv_bfloat16* delta = static_cast<const __nv_bfloat16*>(delta_v);
  if (delta && cols != 3072 && cols != 4096) {
    cudaError_t e = iris_launch_add_bf16_rows(x, ldx, delta, ld_delta, rows, cols, stream);
    if (e != cudaSuccess) return e;
    delta = nullptr;
  }
  if (cols == 3072 || cols == 4096) {
    const float* sh1 = shift1 ? shift1 : shift0;
    const float* sc1 = scale1 ? scale1 : scale0;
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
    return iris::launch_overlapped(cols == 3072 ? adaln_warp_kernel<24> : adaln_warp_kernel<32>, dim3(rows),
                                   dim3(32), 0, stream, x, ldx, delta, ld_delta, o, ldout, rows, shift0, scale0, sh1,
                                   sc1, split, eps);
  }
  return iris::launch_overlapped(adaln_kernel, dim3(rows), dim3(256), 0, stream, (const float*)x, ldx,
                                 static_cast<__nv_bfloat16*>(out), ldout, cols, shift0, scale0,
                                 shift1 ? shift1 : shift0, scale1 ? scale1 : scale0, split, eps);
}

cudaError_t iris_launch_gemv(const void* w, const float* x, const float* bias, float* y, int n,
                             int k, int act_in, int act_out, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (k & 7) return cudaErrorInvalidValue;
  size_t sm = (size_t)k * sizeof(float);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sm);
    if (e != cudaSuccess) return e;
  }
  gemv_kernel<<<(n + 7) / 8, 256, sm, stream>>>(static_cast<const __nv_bfloat16*>(w), x, bias, y,
                                               n, k, act_in, act_out);
  return cudaGetLastError();
}

cudaError_t iris_launch_timestep_sincos(const float* t_dev, float t_scale, float* out, int dim,
                                        cudaStream_t stream) {
  timestep_sincos_kernel<<<(dim / 2 + 127) / 128, 128, 0, stream>>>(t_dev, t_scale, out, dim);
  return cudaGetLastError();
}

cudaError_t iris_launch_nchw_to_tokens(const float* x, int c, int n, void* out, int ldo,
                                       cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  dim3 grid((n + 31) / 32, (c + 31) / 32);
  nchw_to_tokens_kernel<<<grid, dim3(32, 8), 0, stream>>>(x, c, n, static_cast<__nv_bfloat16*>(out),
                                                           ldo);
  return cudaGetLastError();
}

cudaError_t iris_launch_f32_to_bf16(const float* x, void* out, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  f32_to_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(x, static_cast<__nv_bfloat16*>(out), n);
  return cudaGetLastError();
}

cudaError_t iris_launch_f16_to_bf16(const void* x, void* out, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  f16_to_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const __half*>(x),
                                                           static_cast<__nv_bfloat16*>(out), n);
  return cudaGetLastError();
}

cudaError_t iris_launch_bf16_to_f32(const void* x, float* out, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  bf16_to_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                           out, n);
  return cudaGetLastError();
}

cudaError_t iris_launch_euler(float* z, const float* v, const float* v_uncond, float guidance,
                              float dt, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  euler_kernel<<<grid_for(n, 256), 256, 0, stream>>>(z, v, v_uncond, guidance, dt, n);
  return cudaGetLastError();
}

cudaError_t iris_launch_randn_bf16(void* out, long n, uint64_t seed, uint64_t sid, float mean,
                                   float std, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  randn_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(out), n, seed,
                                                          sid, mean, std);
  return cudaGetLastError();
}

cudaError_t iris_launch_randn_f32(float* out, long n, uint64_t seed, uint64_t sid, float mean,
                                  float std, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  randn_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(out, n, seed, sid, mean, std);
  return cudaGetLastError();
}

cudaError_t iris_launch_head_rmsnorm_rope(void* x, int ld, int rows, int heads, const float* w,
                                          float eps, const float* rope_cos, const float* rope_sin,
                                          cudaStream_t stream) {
  long warps = (long)rows * heads;
  if (warps <= 0) return cudaSuccess;
  if (ld & 3) return cudaErrorInvalidValue;
  head_rmsnorm_rope_kernel<<<(int)((warps + 7) / 8), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(x), ld, rows, heads, w, eps, rope_cos, rope_sin);
  return cudaGetLastError();
}

cudaError_t iris_launch_silu_mul_bf16(void* gate, const void* up, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  silu_mul_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up), n);
  return cudaGetLastError();
}

cudaError_t iris_launch_gated_add_bf16(void* out, const void* gate, const void* proj, int rows,
                                       int cols, cudaStream_t stream) {
  long n = (long)rows * cols;
  if (n <= 0) return cudaSuccess;
  gated_add_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gate),
      static_cast<const __nv_bfloat16*>(proj), rows, cols);
  return cudaGetLastError();
}

cudaError_t iris_launch_rmsnorm(const float* x, int ldx, const float* w, float* out_f32,
                                void* out_bf16, int ldout, int rows, int cols, float eps,
                                const float* mul, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(out_bf16);
  const bool vec = (cols % 128 == 0) && !(ldx & 3) && !(ldout & 3);
  if (vec && cols == 3840)
    rmsnorm_warp_kernel<30><<<rows, 32, 0, stream>>>(x, ldx, w, out_f32, ob, ldout, eps, mul);
  else if (vec && cols == 2560)
    rmsnorm_warp_kernel<20><<<rows, 32, 0, stream>>>(x, ldx, w, out_f32, ob, ldout, eps, mul);
  else if (vec && cols == 3072)
    rmsnorm_warp_kernel<24><<<rows, 32, 0, stream>>>(x, ldx, w, out_f32, ob, ldout, eps, mul);
  else
    rmsnorm_kernel<<<rows, 256, 0, stream>>>(x, ldx, w, out_f32, ob, ldout, cols, eps, mul);
  return cudaGetLastError();
}

cudaError_t iris_launch_resid_rmsnorm_gate(float* x, int ldx, const float* y, int ldy, const float* w,
                                           const float* gate, int rows, int cols, float eps,
                                           cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  resid_rmsnorm_gate_kernel<<<rows, 256, 0, stream>>>(x, ldx, y, ldy, w, gate, cols, eps);
  return cudaGetLastError();
}

cudaError_t iris_launch_zi_mod_transform(float* m, int dim, long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  zi_mod_transform_kernel<<<grid_for(n, 256), 256, 0, stream>>>(m, dim, n);
  return cudaGetLastError();
}

cudaError_t iris_launch_patchify(const float* lat, int c, int H, int W, int ps, void* out, int ldo,
                                 cudaStream_t stream) {
  int n = (H / ps) * (W / ps);
  if (n <= 0) return cudaSuccess;
  patchify_kernel<<<n, 128, 0, stream>>>(lat, c, H, W, ps, static_cast<__nv_bfloat16*>(out), ldo);
  return cudaGetLastError();
}

cudaError_t iris_launch_unpatchify(const float* tok, int ldt, int c, int H, int W, int ps, float* lat,
                                   cudaStream_t stream) {
  int n = (H / ps) * (W / ps);
  if (n <= 0) return cudaSuccess;
  unpatchify_kernel<<<n, 128, 0, stream>>>(tok, ldt, c, H, W, ps, lat);
  return cudaGetLastError();
}

cudaError_t iris_launch_fill_rows_f32(float* dst, int ld, const float* vec, int n, int cols,
                                      cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_rows_f32_kernel<<<n < 1024 ? n : 1024, 256, 0, stream>>>(dst, ld, vec, n, cols);
  return cudaGetLastError();
}

cudaError_t iris_launch_interleave_gate_up(void* dst, const void* src, int F, int cols,
                                           cudaStream_t stream) {
  if (F <= 0) return cudaSuccess;
  if ((F & 127) || (cols & 7)) return cudaErrorInvalidValue;
  interleave_gate_up_kernel<<<2 * F, 128, 0, stream>>>(static_cast<uint4*>(dst),
                                                       static_cast<const uint4*>(src), F, cols / 8);
  return cudaGetLastError();
}

cudaError_t iris_launch_copy_rows_bf16(void* dst, int ldd, const void* src, int lds, int rows,
                                       int cols, cudaStream_t stream) {
  long n = (long)rows * cols;
  if (n <= 0) return cudaSuccess;
  copy_rows_bf16_kernel<<<grid_for(n, 256), 256, 0, stream>>>(
      static_cast<uint16_t*>(dst), ldd, static_cast<const uint16_t*>(src), lds, rows, cols);
  return cudaGetLastError();
}

}  // extern "C"
