// Row kernels of the Qwen3 text encoder (iris_qwen3.c): token embedding
// lookup and the per-head Q/K RMSNorm + split-half RoPE between the QKV
// projection and attention.  The projections, the attention and the MLP run
// on the tcgen05 GEMM and attention kernels.
#include "iris_kernels.h"

#include <cuda_bf16.h>

namespace {

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// x[s, :] = table[ids[s], :] (bf16 -> f32); ids outside [0, vocab) give zeros
// (qwen3_forward, iris_qwen3.c:1079-1090).  8 columns per thread.
__global__ void embed_rows_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table, int vocab,
                                  int H, float* __restrict__ x) {
  const int s = blockIdx.x;
  const int id = ids[s];
  const bool ok = id >= 0 && id < vocab;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (ok) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(table + (long)id * H + c));
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
      const float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
      a = make_float4(f0.x, f0.y, f1.x, f1.y);
      b = make_float4(f2.x, f2.y, f3.x, f3.y);
    }
    float4* d = reinterpret_cast<float4*>(x + (long)s * H + c);
    d[0] = a;
    d[1] = b;
  }
}

// One warp per (row, head) of the f32 QKV projection [S, ld] (Q heads, then
// K heads, then V heads of 128 columns).  Q and K: RMSNorm over the head
// (qwen3_head_rms_norm, iris_qwen3.c:213) then the split-half rotation of
// pairs (i, i + 64) with cos/sin [S, 64] (apply_rope, :277); V is copied.
// Lane l holds columns 2l, 2l + 1 and their partners 2l + 64, 2l + 65.
__global__ void qk_norm_rope_half_kernel(const float* __restrict__ qkv, int ld, int S, int nh, int nkv,
                                         const float* __restrict__ qw, const float* __restrict__ kw,
                                         const float* __restrict__ cosb, const float* __restrict__ sinb, float eps,
                                         __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                                         __nv_bfloat16* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const long wid = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nhead = nh + 2 * nkv;
  if (wid >= (long)S * nhead) return;
  const int s = (int)(wid / nhead), hh = (int)(wid - (long)s * nhead);
  const float* src = qkv + (long)s * ld + hh * 128;
  const float2 lo = *reinterpret_cast<const float2*>(src + 2 * lane);
  const float2 hi = *reinterpret_cast<const float2*>(src + 64 + 2 * lane);
  if (hh >= nh + nkv) {  // value head: bf16 copy
    __nv_bfloat16* dst = v + (long)s * nkv * 128 + (hh - nh - nkv) * 128;
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack2(lo.x, lo.y);
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack2(hi.x, hi.y);
    return;
  }
  const bool isq = hh < nh;
  const float* w = isq ? qw : kw;
  float ss = lo.x * lo.x + lo.y * lo.y + hi.x * hi.x + hi.y * hi.y;
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = 1.0f / sqrtf(ss / 128.0f + eps);
  const float x0a = lo.x * r * w[2 * lane], x0b = lo.y * r * w[2 * lane + 1];
  const float x1a = hi.x * r * w[64 + 2 * lane], x1b = hi.y * r * w[64 + 2 * lane + 1];
  const float2 c = *reinterpret_cast<const float2*>(cosb + (long)s * 64 + 2 * lane);
  const float2 sn = *reinterpret_cast<const float2*>(sinb + (long)s * 64 + 2 * lane);
  __nv_bfloat16* dst = isq ? q + (long)s * nh * 128 + hh * 128 : k + (long)s * nkv * 128 + (hh - nh) * 128;
  *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack2(x0a * c.x - x1a * sn.x, x0b * c.y - x1b * sn.y);
  *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack2(x0a * sn.x + x1a * c.x, x0b * sn.y + x1b * c.y);
}

}  // namespace

extern "C" cudaError_t iris_launch_embed_rows(const int* ids, int S, const void* table, int vocab, int H, float* x,
                                              cudaStream_t stream) {
  if (S <= 0) return cudaSuccess;
  if (H % 8) return cudaErrorInvalidValue;
  embed_rows_kernel<<<S, 128, 0, stream>>>(ids, reinterpret_cast<const __nv_bfloat16*>(table), vocab, H, x);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_qk_norm_rope_half(const float* qkv, int ld, int S, int nh, int nkv,
                                                     const float* qw, const float* kw, const float* cosb,
                                                     const float* sinb, float eps, void* q, void* k, void* v,
                                                     cudaStream_t stream) {
  if (S <= 0) return cudaSuccess;
  const long warps = (long)S * (nh + 2 * nkv);
  qk_norm_rope_half_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, stream>>>(
      qkv, ld, S, nh, nkv, qw, kw, cosb, sinb, eps, reinterpret_cast<__nv_bfloat16*>(q),
      reinterpret_cast<__nv_bfloat16*>(k), reinterpret_cast<__nv_bfloat16*>(v));
  return cudaGetLastError();
}
