// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   O = softmax(Q K^T * scale) V      per head, head_dim 128, bf16 in/out
//
// Replaces the reference's attention paths (mha_forward / joint_attention,
// iris_transformer_flux.c:1789-2022; iris_flash_attention,
// iris_kernels.c:943-1048; the masked zi_attention,
// iris_transformer_zimage.c:689-762).
//
// One CTA = 128 query rows of one head; keys stream in tiles of 128.
//   warp 0      TMA producer: Q once, then K_j and V_j into two-stage rings
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_j = Q K_j^T       -> TMEM columns [128 (j&1), +128)  (f32)
//                 O  += P_{j-1} V_{j-1} -> TMEM columns [256, 384)         (f32)
//               S_{j+1} is computed while the softmax warps work on S_j.
//   warps 2..5  softmax: thread = query row (TMEM lane), so row max and row
//               sum need no shuffles; P_j (bf16) goes to one of two
//               128B-swizzled shared tiles (A operand of the P.V MMA), so the
//               softmax of tile j overlaps P_{j-1} V_{j-1} and S_{j+1}.
//               Lazy rescaling: a row keeps its reference max until a tile's
//               max exceeds it by more than 2^8, so the O correction in TMEM
//               (tcgen05.ld / st, after P_{j-1} V_{j-1} is done) is rare; O
//               and l always share the same reference, so the result is
//               exact.  Epilogue: O / l -> bf16 -> global.
// V is consumed as an MN-major B operand straight from its [keys, d] layout.
// Every wait is bounded (see ptx.cuh).
#include "iris_kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int HD = 128;
constexpr int BOX = 128 * 64 * 2;   // one 64-column swizzle box of a 128-row tile: 16 KB
constexpr int TILE = 2 * BOX;       // 128 x 128 bf16 tile
constexpr int OFF_Q = 0;
constexpr int OFF_K = TILE;          // 2 stages
constexpr int OFF_V = 3 * TILE;      // 2 stages
constexpr int OFF_P = 5 * TILE;      // 2 buffers
constexpr int OFF_BAR = 7 * TILE;
constexpr int SMEM_BYTES = 7 * TILE + 256 + 1024;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P values stay <= 256
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;

#define IRIS_DEV_ERR_ATTN_PRODUCER 0x201
#define IRIS_DEV_ERR_ATTN_MMA 0x202
#define IRIS_DEV_ERR_ATTN_SOFTMAX 0x203
#define IRIS_DEV_ERR_ATTN_DRAIN 0x204

struct AttnBars {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t pv_done[2];  // P_j V_j done, by P buffer j & 1
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

struct AttnParams {
  CUtensorMap tq, tk, tv;
  __nv_bfloat16* o;
  int ldo;
  int sq, sk;
  float scale_log2;
  const uint8_t* kmask;
  int* status;
};

int* g_attn_status = nullptr;

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(NUM_THREADS, 1) attn_tc_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnBars* bars = reinterpret_cast<AttnBars*>(smem + OFF_BAR);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * BQ;
  const int col0 = head * HD;
  const int n = (p.sk + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    iris::mbar_init(&bars->q_full, 1);
    for (int s = 0; s < 2; s++) {
      iris::mbar_init(&bars->k_full[s], 1);
      iris::mbar_init(&bars->k_empty[s], 1);
      iris::mbar_init(&bars->v_full[s], 1);
      iris::mbar_init(&bars->v_empty[s], 1);
      iris::mbar_init(&bars->s_full[s], 1);
    }
    iris::mbar_init(&bars->p_full, 128);
    iris::mbar_init(&bars->pv_done[0], 1);
    iris::mbar_init(&bars->pv_done[1], 1);
    iris::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    iris::fence_mbar_init();
    iris::tma_prefetch_desc(&p.tq);
    iris::tma_prefetch_desc(&p.tk);
    iris::tma_prefetch_desc(&p.tv);
  }
  if (warp == 1) iris::tmem_alloc(&bars->tmem_base, TMEM_COLS);
  iris::tc_fence_before();
  __syncthreads();
  iris::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    iris::mbar_arrive_expect_tx(&bars->q_full, TILE);
    iris::tma_load_2d(smem + OFF_Q, &p.tq, &bars->q_full, col0, q0);
    iris::tma_load_2d(smem + OFF_Q + BOX, &p.tq, &bars->q_full, col0 + 64, q0);
    int issued = 0;  // K/V tiles issued (each arms k_full and v_full of its stage)
    bool ok = true;
    for (int j = 0; j < n && ok; j++) {
      int s = j & 1;
      uint32_t u = (uint32_t)(j >> 1);
      if (!iris::mbar_wait(&bars->k_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER)) {
        ok = false;
        break;
      }
      iris::mbar_arrive_expect_tx(&bars->k_full[s], TILE);
      iris::tma_load_2d(smem + OFF_K + s * TILE, &p.tk, &bars->k_full[s], col0, j * BKV);
      iris::tma_load_2d(smem + OFF_K + s * TILE + BOX, &p.tk, &bars->k_full[s], col0 + 64, j * BKV);
      if (!iris::mbar_wait(&bars->v_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER)) {
        ok = false;
        // K_j was issued without its V_j: drain it below through k_full
        volatile int no_abort = 0;
        iris::mbar_wait(&bars->k_full[s], u & 1, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
        break;
      }
      iris::mbar_arrive_expect_tx(&bars->v_full[s], TILE);
      iris::tma_load_2d(smem + OFF_V + s * TILE, &p.tv, &bars->v_full[s], 0 + col0, j * BKV);
      iris::tma_load_2d(smem + OFF_V + s * TILE + BOX, &p.tv, &bars->v_full[s], col0 + 64, j * BKV);
      issued = j + 1;
    }
    if (!ok) {
      // wait (bounded) for the copies still in flight before the CTA exits
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->q_full, 0, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
      for (int j = issued - 2 < 0 ? 0 : issued - 2; j < issued; j++) {
        uint32_t u = (uint32_t)(j >> 1);
        iris::mbar_wait(&bars->k_full[j & 1], u & 1, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
        iris::mbar_wait(&bars->v_full[j & 1], u & 1, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_s = iris::umma_idesc_bf16_f32(BQ, BKV);
    const uint32_t idesc_o = iris::umma_idesc_bf16_f32_bmn(BQ, HD);
    const uint32_t qa = iris::smem_u32(smem + OFF_Q);
    const uint32_t pa = iris::smem_u32(smem + OFF_P);
    bool ok = iris::mbar_wait(&bars->q_full, 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA);
    iris::tc_fence_after();
    for (int j = 0; j <= n && ok; j++) {
      if (j < n) {
        int s = j & 1;
        uint32_t u = (uint32_t)(j >> 1);
        if (!iris::mbar_wait(&bars->k_full[s], u & 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        const uint32_t kb = iris::smem_u32(smem + OFF_K + s * TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
          uint32_t off = (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32);
          iris::umma_bf16(tmem + s * 128, iris::umma_desc_k_sw128(qa + off),
                          iris::umma_desc_k_sw128(kb + off), idesc_s, kk > 0);
        }
        iris::umma_commit(&bars->k_empty[s]);
        iris::umma_commit(&bars->s_full[s]);
      }
      if (j > 0) {
        int jj = j - 1, s = jj & 1;
        uint32_t u = (uint32_t)(jj >> 1);
        if (!iris::mbar_wait(&bars->p_full, (uint32_t)(jj & 1), abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA) ||
            !iris::mbar_wait(&bars->v_full[s], u & 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        const uint32_t vb = iris::smem_u32(smem + OFF_V + s * TILE);
        const uint32_t pb = pa + (uint32_t)(s * TILE);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; kk++) {
          // A: P rows, 16 keys = 32 bytes inside a 64-key swizzle box
          uint64_t adesc = iris::umma_desc_k_sw128(pb + (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32));
          // B: V [keys, d] MN-major; 16 keys = 2 atoms of 8 rows (2048 B);
          // the two 64-wide d chunks are BOX apart, 8-key groups 1024 B apart
          uint64_t bdesc = iris::umma_desc_mn_sw128(vb + (uint32_t)(kk * 2048), BOX, 1024);
          iris::umma_bf16(tmem + 256, adesc, bdesc, idesc_o, (jj > 0 || kk > 0));
        }
        iris::umma_commit(&bars->v_empty[s]);
        iris::umma_commit(&bars->pv_done[s]);
      }
    }
    if (!ok) {
      iris::umma_commit(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;  // reference max (scaled, log2 units) and row sum
    bool ok = true;
    for (int j = 0; j < n && ok; j++) {
      const int b = j & 1;
      if (!iris::mbar_wait(&bars->s_full[b], (uint32_t)((j >> 1) & 1), abort_flag, p.status,
                           IRIS_DEV_ERR_ATTN_SOFTMAX)) {
        ok = false;
        break;
      }
      iris::tc_fence_after();
      float s[BKV];
      iris::tmem_ld64(tmem + b * 128 + lane_off, s);
      iris::tmem_ld64(tmem + b * 128 + lane_off + 64, s + 64);
      const int kbase = j * BKV;
      // full tiles stay raw (scale folded into the exponent's FMA); ragged or
      // masked tiles are scaled here so that padding can be set in log2 units
      float sc = p.scale_log2, tmax = -INFINITY;
      if (kbase + BKV <= p.sk && !p.kmask) {
#pragma unroll
        for (int i = 0; i < BKV; i++) tmax = fmaxf(tmax, s[i]);
        tmax *= sc;
      } else {
#pragma unroll
        for (int i = 0; i < BKV; i++) {
          int key = kbase + i;
          float v = s[i] * p.scale_log2;
          if (key >= p.sk) v = -INFINITY;
          else if (p.kmask && !p.kmask[key]) v = -1e9f * LOG2E;
          s[i] = v;
          tmax = fmaxf(tmax, v);
        }
        sc = 1.0f;
      }
      const bool grow = tmax > m + RESCALE_THRESHOLD;
      const float m_new = grow ? tmax : m;
      const float alpha = (grow && m != -INFINITY) ? iris::ex2_approx(m - m_new) : (grow ? 0.f : 1.f);
      // O holds P_0..P_{j-1} V: correct it once P_{j-1} V_{j-1} is in (warp-uniform:
      // tcgen05.ld / st are collective)
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        if (!iris::mbar_wait(&bars->pv_done[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), abort_flag, p.status,
                             IRIS_DEV_ERR_ATTN_SOFTMAX)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          float o[32];
          iris::tmem_ld32(tmem + 256 + lane_off + 32 * c, o);
#pragma unroll
          for (int e = 0; e < 32; e++) o[e] *= alpha;
          iris::tmem_st32(tmem + 256 + lane_off + 32 * c, o);
        }
      }
      m = m_new;
      const float nm = (m == -INFINITY) ? 0.f : -m;
      // P buffer b was last read by P_{j-2} V_{j-2}
      if (j >= 2 && !iris::mbar_wait(&bars->pv_done[b], (uint32_t)(((j - 2) >> 1) & 1), abort_flag, p.status,
                                     IRIS_DEV_ERR_ATTN_SOFTMAX)) {
        ok = false;
        break;
      }
      uint8_t* prow = smem + OFF_P + b * TILE + r * 128;
      float rs = 0.f;
#pragma unroll
      for (int c16 = 0; c16 < 16; c16++) {  // 8 keys = one 16-byte chunk
        float e[8];
#pragma unroll
        for (int t = 0; t < 8; t++) {
          e[t] = iris::ex2_approx(fmaf(s[c16 * 8 + t], sc, nm));
          rs += e[t];
        }
        uint4 w;
        w.x = pack_bf16(e[0], e[1]);
        w.y = pack_bf16(e[2], e[3]);
        w.z = pack_bf16(e[4], e[5]);
        w.w = pack_bf16(e[6], e[7]);
        int box = c16 >> 3, ch = c16 & 7;
        *reinterpret_cast<uint4*>(prow + box * BOX + ((ch ^ (r & 7)) << 4)) = w;
      }
      l = l * alpha + rs;
      iris::fence_proxy_async_smem();
      iris::tc_fence_before();
      iris::mbar_arrive(&bars->p_full);
    }
    // the last commit covers every earlier MMA of this CTA
    if (ok && n > 0 &&
        iris::mbar_wait(&bars->pv_done[(n - 1) & 1], (uint32_t)(((n - 1) >> 1) & 1), abort_flag, p.status,
                        IRIS_DEV_ERR_ATTN_SOFTMAX)) {
      iris::tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      const int row = q0 + r;
      __nv_bfloat16* dst = p.o + (size_t)row * p.ldo + col0;
#pragma unroll 1
      for (int c = 0; c < 4; c++) {
        float o[32];
        iris::tmem_ld32(tmem + 256 + lane_off + 32 * c, o);
        if (row < p.sq) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            uint4 w;
            w.x = pack_bf16(o[8 * q + 0] * inv, o[8 * q + 1] * inv);
            w.y = pack_bf16(o[8 * q + 2] * inv, o[8 * q + 3] * inv);
            w.z = pack_bf16(o[8 * q + 4] * inv, o[8 * q + 5] * inv);
            w.w = pack_bf16(o[8 * q + 6] * inv, o[8 * q + 7] * inv);
            d4[q] = w;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc(tmem, TMEM_COLS);
  }
}

bool g_attn_tc_attr = false;

}  // namespace

extern "C" void iris_attention_set_status(int* status) { g_attn_status = status; }

extern "C" cudaError_t iris_attention_tc_init(void) {
  if (g_attn_tc_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess) g_attn_tc_attr = true;
  return e;
}

extern "C" cudaError_t iris_launch_attention_tc(const void* q, int ldq, const void* k, const void* v, int ldk,
                                                void* o, int ldo, int sq, int sk, int heads, float scale,
                                                const uint8_t* key_mask, cudaStream_t stream) {
  if (sq <= 0 || sk <= 0 || heads <= 0) return cudaSuccess;
  if ((ldq | ldk | ldo) & 7) return cudaErrorInvalidValue;
  if (!g_attn_tc_attr) {
    cudaError_t e = iris_attention_tc_init();
    if (e != cudaSuccess) return e;
  }
  AttnParams p;
  memset(&p, 0, sizeof(p));
  if (iris_make_tmap_bf16(&p.tq, q, (uint64_t)sq, (uint64_t)heads * HD, (uint64_t)ldq, BQ) ||
      iris_make_tmap_bf16(&p.tk, k, (uint64_t)sk, (uint64_t)heads * HD, (uint64_t)ldk, BKV) ||
      iris_make_tmap_bf16(&p.tv, v, (uint64_t)sk, (uint64_t)heads * HD, (uint64_t)ldk, BKV))
    return cudaErrorInvalidValue;
  p.o = static_cast<__nv_bfloat16*>(o);
  p.ldo = ldo;
  p.sq = sq;
  p.sk = sk;
  p.scale_log2 = scale * LOG2E;
  p.kmask = key_mask;
  p.status = g_attn_status;
  dim3 grid((sq + BQ - 1) / BQ, heads);
  attn_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(p);
  return cudaGetLastError();
}

// Attention entry point: the tcgen05 kernel above; IRIS_ATTN=mma selects the
// mma.sync kernel of attention.cu instead (kept for A/B measurements).
extern "C" cudaError_t iris_launch_attention(const void* q, int ldq, const void* k, const void* v, int ldk,
                                             void* o, int ldo, int sq, int sk, int heads, float scale,
                                             const uint8_t* key_mask, cudaStream_t stream) {
  static int use_mma = -1;
  if (use_mma < 0) {
    const char* e = getenv("IRIS_ATTN");
    use_mma = (e && strcmp(e, "mma") == 0) ? 1 : 0;
  }
  if (use_mma)
    return iris_launch_attention_mma(q, ldq, k, v, ldk, o, ldo, sq, sk, heads, scale, key_mask, stream);
  return iris_launch_attention_tc(q, ldq, k, v, ldk, o, ldo, sq, sk, heads, scale, key_mask, stream);
}
