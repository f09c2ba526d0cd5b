// Fused multi-head attention, O = softmax(Q K^T * scale) V, head_dim 128.
//
// Replaces the reference's attention paths: the BLAS per-head
// sgemm -> softmax -> sgemm threads (mha_forward / joint_attention,
// iris_transformer_flux.c:1789-2022), the generic flash attention
// (iris_flash_attention, iris_kernels.c:943-1048) and Z-Image's masked
// scalar attention (zi_attention, iris_transformer_zimage.c:689-762).
// Joint text+image attention needs no special case: the hidden state is kept
// as one [TXT, IMG] sequence, so K/V are already concatenated in that order.
//
// One CTA = 128 query rows of one head (8 warps x 16 rows); keys stream in
// tiles of 64 through a cp.async double buffer; scores stay in registers
// with an online (running max / running sum) softmax in f32; P is re-used
// directly as the A operand of the P.V product.  Shared-memory rows are 256
// bytes with a 16-byte-chunk XOR swizzle so ldmatrix is conflict-free.
#include "iris_kernels.h"

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

namespace {

constexpr int HD = 128;
constexpr int BQ = 128;
constexpr int BKV = 64;
constexpr int NT = 256;
constexpr int SMEM_Q = BQ * HD * 2;    // 32 KB
constexpr int SMEM_KV = BKV * HD * 2;  // 16 KB per tile
constexpr int SMEM_TOTAL = SMEM_Q + 4 * SMEM_KV;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of 16B chunk `c` (0..15) of row `r` in a swizzled [rows][128] bf16 tile
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load rows [row0, row0+nrows) x 128 bf16 of head `col0` into a swizzled tile.
__device__ __forceinline__ void load_tile(uint8_t* sm, const __nv_bfloat16* g, int ld, int row0,
                                          int nrows, int total_rows, int col0) {
  uint32_t base = smem_u32(sm);
  for (int i = threadIdx.x; i < nrows * 16; i += NT) {
    int r = i >> 4, c = i & 15;
    int gr = row0 + r;
    bool ok = gr < total_rows;
    const __nv_bfloat16* src = g + (size_t)(ok ? gr : 0) * ld + col0 + c * 8;
    cp_async16(base + swz(r, c), src, ok);
  }
}

__global__ void __launch_bounds__(NT, 1)
attention_kernel(const __nv_bfloat16* __restrict__ Q, int ldq, const __nv_bfloat16* __restrict__ K,
                 const __nv_bfloat16* __restrict__ V, int ldk, __nv_bfloat16* __restrict__ O,
                 int ldo, int sq, int sk, float scale_log2, const uint8_t* __restrict__ kmask) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + SMEM_Q, smem + SMEM_Q + SMEM_KV};
  uint8_t* sV[2] = {smem + SMEM_Q + 2 * SMEM_KV, smem + SMEM_Q + 3 * SMEM_KV};

  const int head = blockIdx.y;
  const int q0 = blockIdx.x * BQ;
  const int col0 = head * HD;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;   // row within 8
  const int cq = lane & 3;   // column pair

  load_tile(sQ, Q, ldq, q0, BQ, sq, col0);
  load_tile(sK[0], K, ldk, 0, BKV, sk, col0);
  load_tile(sV[0], V, ldk, 0, BKV, sk, col0);
  cp_async_commit();

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  const int ntiles = (sk + BKV - 1) / BKV;
  const uint32_t q_base = smem_u32(sQ);
  const int qrow_ld = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);  // ldmatrix row (A)
  const int qchunk_hi = lane >> 4;                                      // 0/1: k 0-7 / 8-15

  for (int j = 0; j < ntiles; j++) {
    if (j + 1 < ntiles) {
      load_tile(sK[(j + 1) & 1], K, ldk, (j + 1) * BKV, BKV, sk, col0);
      load_tile(sV[(j + 1) & 1], V, ldk, (j + 1) * BKV, BKV, sk, col0);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    const uint32_t k_base = smem_u32(sK[j & 1]);
    const uint32_t v_base = smem_u32(sV[j & 1]);

    // ---- S = Q K^T  (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(q_base + swz(qrow_ld, kk * 2 + qchunk_hi), a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        int krow = nt * 8 + (lane & 7) + 8 * (lane >> 4);
        int kch = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(k_base + swz(krow, kch), b0, b1, b2, b3);
        mma16816(s[nt], a0, a1, a2, a3, b0, b1);
        mma16816(s[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }

    // ---- scale, mask, online softmax (rows g and g+8 of this warp's 16)
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
#pragma unroll
      for (int e = 0; e < 2; e++) {
        int key = j * BKV + nt * 8 + cq * 2 + e;
        float v0 = s[nt][e] * scale_log2, v1 = s[nt][2 + e] * scale_log2;
        if (key >= sk) {
          v0 = -INFINITY;
          v1 = -INFINITY;
        } else if (kmask && !kmask[key]) {
          v0 = -1e9f * 1.4426950408889634f;
          v1 = v0;
        }
        s[nt][e] = v0;
        s[nt][2 + e] = v1;
        tmax0 = fmaxf(tmax0, v0);
        tmax1 = fmaxf(tmax1, v1);
      }
    }
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 1));
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 2));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 1));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 2));
    float mn0 = fmaxf(m0, tmax0), mn1 = fmaxf(m1, tmax1);
    float alpha0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mn0);
    float alpha1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      s[nt][0] = exp2f(s[nt][0] - mn0);
      s[nt][1] = exp2f(s[nt][1] - mn0);
      s[nt][2] = exp2f(s[nt][2] - mn1);
      s[nt][3] = exp2f(s[nt][3] - mn1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * alpha0 + rs0;
    l1 = l1 * alpha1 + rs1;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      o[i][0] *= alpha0;
      o[i][1] *= alpha0;
      o[i][2] *= alpha1;
      o[i][3] *= alpha1;
    }

    // ---- O += P V   (P from the S accumulators, 4 k-steps of 16 keys)
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
      uint32_t a0 = pack2(s[2 * ks][0], s[2 * ks][1]);
      uint32_t a1 = pack2(s[2 * ks][2], s[2 * ks][3]);
      uint32_t a2 = pack2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      uint32_t a3 = pack2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
      int vrow = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(v_base + swz(vrow, dt + (lane >> 4)), b0, b1, b2, b3);
        mma16816(o[dt], a0, a1, a2, a3, b0, b1);
        mma16816(o[dt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // tile (j & 1) is refilled by the prefetch of iteration j+1
  }

  // ---- normalise, stage through shared memory, coalesced 16-byte stores
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  int r0 = warp * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int dt = 0; dt < 16; dt++) {
    int chunk = dt;  // 8 d per d-tile = one 16B chunk
    uint32_t off = (uint32_t)(cq * 4);
    *reinterpret_cast<uint32_t*>(sQ + swz(r0, chunk) + off) = pack2(o[dt][0] * inv0, o[dt][1] * inv0);
    *reinterpret_cast<uint32_t*>(sQ + swz(r1, chunk) + off) = pack2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < BQ * 16; i += NT) {
    int r = i >> 4, c = i & 15;
    int gr = q0 + r;
    if (gr < sq) {
      uint4 val = *reinterpret_cast<const uint4*>(sQ + swz(r, c));
      *reinterpret_cast<uint4*>(O + (size_t)gr * ldo + col0 + c * 8) = val;
    }
  }
}

}  // namespace

static bool g_attn_attr = false;

extern "C" cudaError_t iris_attention_init(void) {
  if (g_attn_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_TOTAL);
  if (e == cudaSuccess) g_attn_attr = true;
  return e;
}

extern "C" cudaError_t iris_launch_attention_mma(const void* q, int ldq, const void* k, const void* v,
                                             int ldk, void* o, int ldo, int sq, int sk, int heads,
                                             float scale, const uint8_t* key_mask,
                                             cudaStream_t stream) {
  if (!g_attn_attr) {
    cudaError_t e = iris_attention_init();
    if (e != cudaSuccess) return e;
  }
  if (sq <= 0 || sk <= 0 || heads <= 0) return cudaSuccess;
  if ((ldq | ldk | ldo) & 7) return cudaErrorInvalidValue;
  dim3 grid((sq + BQ - 1) / BQ, heads);
  attention_kernel<<<grid, NT, SMEM_TOTAL, stream>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v), ldk, static_cast<__nv_bfloat16*>(o), ldo, sq, sk,
      scale * 1.4426950408889634f, key_mask);
  return cudaGetLastError();
}
