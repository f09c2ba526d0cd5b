// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   O = softmax(Q K^T * scale) V      per head, head_dim 128, bf16 in/out
//
// Replaces the reference's attention paths (mha_forward / joint_attention,
// iris_transformer_flux.c:1789-2022; iris_flash_attention,
// iris_kernels.c:943-1048; the masked zi_attention,
// iris_transformer_zimage.c:689-762).
//
// One CTA = two 128-row query tiles (Q0, Q1) of one head; both read the same
// K/V tiles of 128 keys, which stream through two-stage TMA rings.
//   warp 0      TMA producer
//   warp 1      TMEM owner + single-thread MMA issuer.  TMEM columns:
//                 [0,128) S0 / P0   [128,256) S1 / P1   [256,384) O0   [384,512) O1
//               Per key tile j, in issue order (the tensor pipe runs them in
//               order, so an MMA never overtakes the one before it):
//                 O0 += P0_j V_j,  S0_{j+1} = Q0 K_{j+1}^T,
//                 O1 += P1_j V_j,  S1_{j+1} = Q1 K_{j+1}^T
//               so the softmax of one query tile overlaps the MMAs of the other.
//   warps 2..5  softmax of Q0, warps 6..9 softmax of Q1: thread = query row
//               (TMEM lane), so row max and row sum need no shuffles.  S_j is
//               read from TMEM, P_j = 2^(S_j - m) goes back as bf16 over the
//               first 64 columns of the same S buffer and is the TMEM A
//               operand of P_j V_j (V is an MN-major B operand straight from
//               its [keys, d] layout).  Lazy rescaling: a row keeps its
//               reference max m until a tile's max exceeds it by more than
//               2^8; only then is O (already final for tiles < j, since the
//               commit that signals S_j covers P_{j-1} V_{j-1}) scaled in TMEM.
//               O and l always share the same m, so the result is exact.
//               Epilogue: O / l -> bf16 -> shared memory (the idle K / V
//               rings) -> global, whole rows per store instruction.
// Every wait is bounded (see ptx.cuh).
#include "iris_kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int BQ = 128;             // rows per query tile; a CTA holds two
constexpr int BKV = 128;
constexpr int HD = 128;
constexpr int BOX = 128 * 64 * 2;   // one 64-column swizzle box of a 128-row tile: 16 KB
constexpr int TILE = 2 * BOX;       // 128 x 128 bf16 tile
constexpr int OFF_Q = 0;            // 2 query tiles
constexpr int KST = 2;              // K ring stages
constexpr int VST = 3;              // V ring stages (V_j is released half a key tile after K_j)
constexpr int OFF_K = 2 * TILE;
constexpr int OFF_V = OFF_K + KST * TILE;
constexpr int OFF_BAR = OFF_V + VST * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr int NUM_THREADS = 320;
constexpr int TMEM_COLS = 512;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: a new reference max moves P by >= 2^8
// A tile whose row sum against the current reference stays <= 2^16 has every
// P <= 2^16, which bf16 P and the f32 O / l accumulators take as they are;
// only larger sums send the row's warp to the exact max / rescale path.
constexpr float FAST_SUM_LIMIT = 65536.0f;
// epilogue staging of one softmax warp's 32 output rows (128 bf16 + 16 bytes of padding each)
constexpr int O_STAGE_LD = 128 * 2 + 16;
constexpr int O_STAGE_BYTES = 32 * O_STAGE_LD;
#define IRIS_DEV_ERR_ATTN_PRODUCER 0x201
#define IRIS_DEV_ERR_ATTN_MMA 0x202
#define IRIS_DEV_ERR_ATTN_SOFTMAX 0x203
#define IRIS_DEV_ERR_ATTN_DRAIN 0x204

struct AttnBars {
  uint64_t q_full;
  uint64_t k_full[KST], k_empty[KST];
  uint64_t v_full[VST], v_empty[VST];
  uint64_t s_full[2];  // per query tile: S_j written (and every earlier MMA done)
  uint64_t p_full[2];  // per query tile: P_j in TMEM (128 arrivals)
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int nkv;  // key tiles this CTA visits (live_key_tiles)
};

struct AttnParams {
  CUtensorMap tq, tk, tv;
  __nv_bfloat16* o;
  int ldo;
  int sq, sk;
  float scale_log2;
  const uint8_t* kmask;
  int causal;     // key j of query row i masked when j > i (masked instantiation only)
  int kv_group;   // query heads per key/value head (grouped-query attention)
  int one_tile;   // single-CTA kernel: one 128-row query tile per CTA instead of two
  int* status;
};

int* g_attn_status = nullptr;

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two keys of a full tile in one go, on Blackwell's paired f32 ops:
//   x = s * scale + nm (fma.f32x2), e = 2^x (SFU), row-sum accumulator += e
//   (add.f32x2), P pair -> bf16x2: 5 instructions for 2 keys.  The softmax
//   is bound by instruction issue, not by one pipe, so every one counts.
__device__ __forceinline__ uint32_t exp_pair(float s0, float s1, uint64_t sc2, uint64_t nm2, uint64_t& acc) {
  uint32_t pw;
  asm("{\n\t.reg .b64 sv, xv, ev;\n\t.reg .f32 x0, x1, e0, e1;\n\t"
      "mov.b64 sv, {%2, %3};\n\t"
      "fma.rn.f32x2 xv, sv, %4, %5;\n\t"
      "mov.b64 {x0, x1}, xv;\n\t"
      "ex2.approx.ftz.f32 e0, x0;\n\t"
      "ex2.approx.ftz.f32 e1, x1;\n\t"
      "mov.b64 ev, {e0, e1};\n\t"
      "add.rn.f32x2 %1, %1, ev;\n\t"
      "cvt.rn.bf16x2.f32 %0, e1, e0;\n\t}"
      : "=r"(pw), "+l"(acc)
      : "f"(s0), "f"(s1), "l"(sc2), "l"(nm2));
  return pw;
}

__device__ __forceinline__ uint64_t f32x2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float sum_f32x2(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return a + b;
}

// Softmax and epilogue of one 128-row query tile t (warps of one warpgroup):
// per key tile, S_t from TMEM -> P_t (bf16) back into TMEM, running row sum and
// lazy reference max; at the end O_t / l -> bf16 rows [row0, row0 + 128).
// kPair: the P-ready barrier lives in the even CTA of a pair (one arrival per
// warp through its cluster address), otherwise in this CTA (128 arrivals).
// kMasked: a key mask exists (a separate instantiation, so the unmasked
// softmax carries no mask test).
template <bool kPair, bool kMasked>
__device__ __forceinline__ void softmax_role(const AttnParams& p, uint32_t tmem, int t, int warp, int lane,
                                             uint64_t* s_full, uint64_t* p_full, uint32_t p_full_cluster,
                                             uint64_t* o_done, volatile int* abort_flag, int row0, int col0,
                                             int n, uint8_t* ostage) {
  const int quarter = warp & 3;
  const int r = quarter * 32 + lane;  // query row within the tile = TMEM lane
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const uint32_t s_addr = tmem + lane_off + t * 128;
  const uint32_t o_addr = tmem + lane_off + 256 + t * 128;
  float m = -INFINITY, l = 0.f;  // reference max (scaled, log2 units) and row sum
  bool ok = true;
  // S row -> scaled logits (log2 units): padding keys -inf, masked keys
  // -1e9 (in natural-log units, as the reference's masked softmax)
  const int qrow = row0 + r;
  auto logit = [&](float sv, int key, bool full) -> float {
    if (full) return sv * p.scale_log2;
    if (key >= p.sk) return -INFINITY;
    if (kMasked && p.kmask && !p.kmask[key]) return -1e9f * LOG2E;
    if (kMasked && p.causal && key > qrow) return -1e9f * LOG2E;
    return sv * p.scale_log2;
  };
  // A tile with masked or padding keys is rewritten in place once
  // (mask_tile) and then takes the full-tile path instead of testing every
  // key in each pass: a masked key's S becomes masked_s, whose logit is -1e9
  // in natural-log units (the value above), a padding key's -inf.  Every
  // masked key of a row carries the same logit, so a row without a kept key
  // still spreads uniformly over them.  kw: the tile's kept-key bits, the
  // same for every row (word e bit l = key 4l + e).
  const float masked_s = -1e9f * LOG2E / p.scale_log2;
  auto mask_tile = [&](int kbase, const uint32_t* kw) {
    const int lim_c = (kMasked && p.causal) ? qrow - kbase : BKV;  // causal: keys past this row's own
    const int lim_s = p.sk - kbase;                                  // padding from here on
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
      float sv[32];
      iris::tmem_ld32(s_addr + 32 * c, sv);
      uint32_t kc[4];  // the chunk's 32 keys: word e bit l = key 32c + 4l + e
#pragma unroll
      for (int e = 0; e < 4; e++) kc[e] = kw[e] >> (8 * c);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const int kk = 32 * c + i;
        const bool kept = ((kc[i & 3] >> (i >> 2)) & 1u) && kk <= lim_c;
        sv[i] = kk >= lim_s ? -INFINITY : (kept ? sv[i] : masked_s);
      }
      iris::tmem_st32(s_addr + 32 * c, sv);
    }
  };
  // exponentials of 64 keys (half h of the tile) against reference max -nm
  // -> 32 packed bf16 words; returns the largest exponent argument
  auto half_exps = [&](int h, int kbase, bool full, float nm, uint32_t* pw, float* rsum) -> float {
    float sv[64];
    iris::tmem_ld64(s_addr + 64 * h, sv);
    float xm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    if (full) {
      const uint64_t sc2 = f32x2(p.scale_log2, p.scale_log2), nm2 = f32x2(nm, nm);
      uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < 32; i++) pw[i] = exp_pair(sv[2 * i], sv[2 * i + 1], sc2, nm2, acc[i & 3]);
#pragma unroll
      for (int i = 0; i < 4; i++) rsum[i] += sum_f32x2(acc[i]);
      return -INFINITY;  // the caller checks the row sum instead
    }
#pragma unroll
    for (int c = 0; c < 8; c++) {
      float e[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = c * 8 + u;
        const float x = full ? fmaf(sv[i], p.scale_log2, nm) : logit(sv[i], kbase + 64 * h + i, false) + nm;
        xm[u & 3] = fmaxf(xm[u & 3], x);
        e[u] = iris::ex2_approx(x);
        rsum[u] += e[u];
      }
#pragma unroll
      for (int u = 0; u < 4; u++) pw[c * 4 + u] = pack_bf16(e[2 * u], e[2 * u + 1]);
    }
    return fmaxf(fmaxf(xm[0], xm[1]), fmaxf(xm[2], xm[3]));
  };
  for (int j = 0; j < n; j++) {
    if (!iris::mbar_wait(s_full, (uint32_t)(j & 1), abort_flag, p.status, IRIS_DEV_ERR_ATTN_SOFTMAX)) {
      ok = false;
      break;
    }
    iris::tc_fence_after();
    const int kbase = j * BKV;
    bool full = kbase + BKV <= p.sk;
    // causal: a key tile reaching past the tile's first query row is masked per element
    if (kMasked && p.causal && kbase + BKV - 1 > row0) full = false;
    if (kMasked && full && p.kmask) {  // a masked sequence: tiles without padding keys still take the fast path
      const uint32_t m4 = reinterpret_cast<const uint32_t*>(p.kmask + kbase)[lane];
      full = __all_sync(0xffffffffu, m4 == 0x01010101u);
    }
    if (kMasked && !full) {
      // A tile every key of which is masked for every row of the query tile
      // (entirely after the diagonal, or all padding) contributes exp(-1e9 - m)
      // = 0 once a row has seen a real key (m > -1e8): P = 0, l and O unchanged.
      // (A row whose keys are all masked keeps the exact path: the reference's
      // softmax then spreads uniformly over its masked keys.)
      bool dead = p.causal && kbase > row0 + BQ - 1;
      if (!dead && p.kmask) {
        uint32_t m4 = 0;
        const int k4 = kbase + 4 * lane;
        if (k4 + 3 < p.sk) m4 = reinterpret_cast<const uint32_t*>(p.kmask + kbase)[lane];
        else
          for (int e = 0; e < 4; e++) m4 |= (k4 + e < p.sk) ? (uint32_t)p.kmask[k4 + e] << (8 * e) : 0u;
        dead = __all_sync(0xffffffffu, m4 == 0u);
      }
      if (__all_sync(0xffffffffu, dead && m > -1e8f)) {
        uint32_t z[BKV / 2];
#pragma unroll
        for (int i = 0; i < BKV / 2; i++) z[i] = 0u;
        iris::tmem_st64(s_addr, z);  // P_j = 0 over the first 64 columns of S_j
        iris::tc_fence_before();
        if (kPair) {
          __syncwarp();
          if (lane == 0) iris::mbar_arrive_cluster(p_full_cluster);
        } else {
          iris::mbar_arrive(p_full);
        }
        continue;
      }
    }
    if (kMasked && !full) {
      uint32_t m4 = 0x01010101u;  // this lane's 4 keys, one byte each (non-zero = kept)
      if (kMasked && p.kmask) {
        const int k4 = kbase + 4 * lane;
        m4 = 0;
        if (k4 + 3 < p.sk) m4 = reinterpret_cast<const uint32_t*>(p.kmask + kbase)[lane];
        else
          for (int e = 0; e < 4; e++) m4 |= (k4 + e < p.sk) ? (uint32_t)p.kmask[k4 + e] << (8 * e) : 0u;
      }
      uint32_t kw[4];
#pragma unroll
      for (int e = 0; e < 4; e++) kw[e] = __ballot_sync(0xffffffffu, (m4 >> (8 * e)) & 0xffu);
      mask_tile(kbase, kw);
      full = true;
    }
    uint32_t pw[BKV / 2];
    float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float alpha = 1.f;
    // fast path: P against the current reference max; it stands unless a
    // logit exceeds it by more than the threshold (m = -inf: first tile)
    bool redo = true;
    if (m != -INFINITY) {
      const float nm = -m;
      const float x0 = half_exps(0, kbase, full, nm, pw, rsum);
      const float x1 = half_exps(1, kbase, full, nm, pw + 32, rsum);
      const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
      // (a NaN sum also redoes: !(rs <= limit))
      redo = __any_sync(0xffffffffu, fmaxf(x0, x1) > RESCALE_THRESHOLD || !(rs <= FAST_SUM_LIMIT));
    }
    if (redo) {
      // slow path (warp-uniform): row max of the tile, new reference, O
      // correction, P again
      float tm[8];
#pragma unroll
      for (int i = 0; i < 8; i++) tm[i] = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float sv[64];
        iris::tmem_ld64(s_addr + 64 * h, sv);
#pragma unroll
        for (int i = 0; i < 64; i++) tm[i & 7] = fmaxf(tm[i & 7], logit(sv[i], kbase + 64 * h + i, full));
      }
      const float tmax = fmaxf(fmaxf(fmaxf(tm[0], tm[1]), fmaxf(tm[2], tm[3])),
                               fmaxf(fmaxf(tm[4], tm[5]), fmaxf(tm[6], tm[7])));
      const bool grow = tmax > m + RESCALE_THRESHOLD;
      const float m_new = grow ? tmax : m;
      alpha = (grow && m != -INFINITY) ? iris::ex2_approx(m - m_new) : (grow ? 0.f : 1.f);
      // O = P_0..P_{j-1} V is final here (the commit behind s_full covers
      // P_{j-1} V_{j-1})
      if (j > 0) {
#pragma unroll 1
        for (int c = 0; c < 4; c++) {
          float o[32];
          iris::tmem_ld32(o_addr + 32 * c, o);
#pragma unroll
          for (int e = 0; e < 32; e++) o[e] *= alpha;
          iris::tmem_st32(o_addr + 32 * c, o);
        }
      }
      m = m_new;
      const float nm = (m == -INFINITY) ? 0.f : -m;
#pragma unroll
      for (int i = 0; i < 8; i++) rsum[i] = 0.f;
      half_exps(0, kbase, full, nm, pw, rsum);
      half_exps(1, kbase, full, nm, pw + 32, rsum);
    }
    iris::tmem_st64(s_addr, pw);  // P_j over the first 64 columns of S_j
    const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
    l = l * alpha + rs;
    iris::tc_fence_before();
    if (kPair) {
      // the even CTA's MMA thread waits for both CTAs' P: one arrival per warp
      __syncwarp();
      if (lane == 0) iris::mbar_arrive_cluster(p_full_cluster);
    } else {
      iris::mbar_arrive(p_full);
    }
  }
  if (ok && n > 0 && iris::mbar_wait(o_done, 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_SOFTMAX)) {
    iris::tc_fence_after();
    const float inv = l > 0.f ? 1.0f / l : 0.f;
    // O / l of this warp's 32 rows goes through shared memory (the K / V rings,
    // idle once every MMA is done; rows 272 bytes apart so that a 16-byte
    // store of each lane spreads over the banks), then leaves as whole rows:
    // each global store instruction writes two rows' 256 contiguous bytes.
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
      float o[32];
      iris::tmem_ld32(o_addr + 32 * c, o);
      uint4* d4 = reinterpret_cast<uint4*>(ostage + lane * O_STAGE_LD + c * 64);
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
    __syncwarp();
    const int wrow = row0 + (warp & 3) * 32;  // the warp's first row
#pragma unroll 4
    for (int k = 0; k < 16; k++) {
      const int rr = 2 * k + (lane >> 4), cb = (lane & 15) * 16;
      const uint4 val = *reinterpret_cast<const uint4*>(ostage + rr * O_STAGE_LD + cb);
      if (wrow + rr < p.sq)
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.o + (size_t)(wrow + rr) * p.ldo + col0) + cb) = val;
    }
    __syncwarp();
  }
}

// Key tiles a CTA (or CTA pair) whose query rows are [row_first, row_last]
// visits; one warp computes it.  Tiles after the last key the mask keeps,
// and under the causal mask tiles after row_last, are masked for every row:
// once a row has seen a kept key such a tile adds exactly nothing (P = 0, the
// dead-tile path of the softmax), so the loops end before them.  A row that
// sees no kept key at all (a causal row before the first kept key, or a mask
// that keeps none) takes the exact path over every key tile, so a CTA holding
// one visits them all.  Mask bytes are read four at a time from 4-byte
// aligned offsets, as the softmax reads them.
template <bool kMasked>
__device__ int live_key_tiles(const AttnParams& p, int row_first, int row_last, int lane) {
  const int n = (p.sk + BKV - 1) / BKV;
  if (!kMasked) return n;
  int first = 0, last = p.sk - 1;
  if (p.kmask) {
    int lo = 0x7fffffff, hi = -1;
    for (int k = 4 * lane; k < p.sk; k += 128) {
      uint32_t m4 = 0;
      if (k + 3 < p.sk) m4 = *reinterpret_cast<const uint32_t*>(p.kmask + k);
      else
        for (int e = 0; e < 4; e++) m4 |= (k + e < p.sk) ? (uint32_t)p.kmask[k + e] << (8 * e) : 0u;
      if (m4) {
        lo = min(lo, k + (__ffs(m4) - 1) / 8);
        hi = max(hi, k + (31 - __clz(m4)) / 8);
      }
    }
    for (int o = 16; o; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (hi < 0) return n;
    first = lo;
    last = hi;
  }
  if (p.causal) {
    if (row_first < first) return n;
    last = min(last, row_last);
  }
  return min(n, last / BKV + 1);
}

template <bool kMasked>
__global__ void __launch_bounds__(NUM_THREADS, 1) attn_tc_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnBars* bars = reinterpret_cast<AttnBars*>(smem + OFF_BAR);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * (p.one_tile ? BQ : 2 * BQ);
  const bool has1 = !p.one_tile && q0 + BQ < p.sq;  // second query tile holds rows
  const int col0 = head * HD;
  const int kvcol0 = (head / p.kv_group) * HD;

  // Set-up before the wait for the previous kernel (a CTA that starts during
  // its tail allocates and initialises meanwhile); the masked instantiation
  // reads the key mask first, which the previous kernel may write.
  if (kMasked) iris::grid_dep_wait();
  if (warp == 2) {
    const int nkv = live_key_tiles<kMasked>(p, q0, min(p.sq, q0 + (has1 ? 2 : 1) * BQ) - 1, lane);
    if (lane == 0) bars->nkv = nkv;
  }
  if (threadIdx.x == 0) {
    iris::mbar_init(&bars->q_full, 1);
    for (int s = 0; s < KST; s++) {
      iris::mbar_init(&bars->k_full[s], 1);
      iris::mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < VST; s++) {
      iris::mbar_init(&bars->v_full[s], 1);
      iris::mbar_init(&bars->v_empty[s], 1);
    }
    for (int s = 0; s < 2; s++) {
      iris::mbar_init(&bars->s_full[s], 1);
      iris::mbar_init(&bars->p_full[s], 128);
    }
    iris::mbar_init(&bars->o_done, 1);
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
  if (!kMasked) iris::grid_dep_wait();  // Q, K and V come from the previous kernel
  const uint32_t tmem = bars->tmem_base;
  iris::grid_dep_launch();  // after this CTA's TMEM allocation
  const int n = bars->nkv;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    iris::mbar_arrive_expect_tx(&bars->q_full, (has1 ? 2 : 1) * TILE);
    for (int t = 0; t < (has1 ? 2 : 1); t++) {
      iris::tma_load_2d(smem + OFF_Q + t * TILE, &p.tq, &bars->q_full, col0, q0 + t * BQ);
      iris::tma_load_2d(smem + OFF_Q + t * TILE + BOX, &p.tq, &bars->q_full, col0 + 64, q0 + t * BQ);
    }
    // Loads in the order their stages are released: K_{j+KST} once Q1 K_j^T
    // is done, V_{j+VST} once P1_j V_j is done (the tensor pipe finishes
    // P1_{j-1} V_{j-1} before Q1 K_j^T before P1_j V_j), so no wait of this
    // single thread holds back a load whose stage is already free.
    int nk = 0, nv = 0;  // tiles issued
    bool ok = true;
    auto load_k = [&]() -> bool {
      const int s = nk % KST;
      const uint32_t u = (uint32_t)(nk / KST);
      if (!iris::mbar_wait(&bars->k_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER))
        return false;
      iris::mbar_arrive_expect_tx(&bars->k_full[s], TILE);
      iris::tma_load_2d(smem + OFF_K + s * TILE, &p.tk, &bars->k_full[s], kvcol0, nk * BKV);
      iris::tma_load_2d(smem + OFF_K + s * TILE + BOX, &p.tk, &bars->k_full[s], kvcol0 + 64, nk * BKV);
      nk++;
      return true;
    };
    auto load_v = [&]() -> bool {
      const int s = nv % VST;
      const uint32_t u = (uint32_t)(nv / VST);
      if (!iris::mbar_wait(&bars->v_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER))
        return false;
      iris::mbar_arrive_expect_tx(&bars->v_full[s], TILE);
      iris::tma_load_2d(smem + OFF_V + s * TILE, &p.tv, &bars->v_full[s], kvcol0, nv * BKV);
      iris::tma_load_2d(smem + OFF_V + s * TILE + BOX, &p.tv, &bars->v_full[s], kvcol0 + 64, nv * BKV);
      nv++;
      return true;
    };
    while (ok && nk < (n < KST ? n : KST)) ok = load_k();
    while (ok && nv < (n < VST ? n : VST)) ok = load_v();
    while (ok && (nk < n || nv < n)) {
      if (nk < n) ok = load_k();
      if (ok && nv < n) ok = load_v();
    }
    if (!ok) {
      // wait (bounded) for the copies still in flight before the CTA exits
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->q_full, 0, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
      for (int j = nk - KST < 0 ? 0 : nk - KST; j < nk; j++)
        iris::mbar_wait(&bars->k_full[j % KST], (uint32_t)((j / KST) & 1), &no_abort, p.status,
                        IRIS_DEV_ERR_ATTN_DRAIN);
      for (int j = nv - VST < 0 ? 0 : nv - VST; j < nv; j++)
        iris::mbar_wait(&bars->v_full[j % VST], (uint32_t)((j / VST) & 1), &no_abort, p.status,
                        IRIS_DEV_ERR_ATTN_DRAIN);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_s = iris::umma_idesc_bf16_f32(BQ, BKV);
    const uint32_t idesc_o = iris::umma_idesc_bf16_f32_bmn(BQ, HD);
    const int nq = has1 ? 2 : 1;
    auto qk = [&](int t, int j) {  // S_t = Q_t K_j^T
      const uint32_t qa = iris::smem_u32(smem + OFF_Q + t * TILE);
      const uint32_t kb = iris::smem_u32(smem + OFF_K + (j % KST) * TILE);
#pragma unroll
      for (int kk = 0; kk < HD / 16; kk++) {
        uint32_t off = (uint32_t)((kk >> 2) * BOX + (kk & 3) * 32);
        iris::umma_bf16(tmem + t * 128, iris::umma_desc_k_sw128(qa + off), iris::umma_desc_k_sw128(kb + off),
                        idesc_s, kk > 0);
      }
    };
    auto pv = [&](int t, int j) {  // O_t += P_t V_j, P_t from TMEM
      const uint32_t vb = iris::smem_u32(smem + OFF_V + (j % VST) * TILE);
#pragma unroll
      for (int kk = 0; kk < BKV / 16; kk++) {
        // B: V [keys, d] MN-major; 16 keys = 2 atoms of 8 rows (2048 B);
        // the two 64-wide d chunks are BOX apart, 8-key groups 1024 B apart
        uint64_t bdesc = iris::umma_desc_mn_sw128(vb + (uint32_t)(kk * 2048), BOX, 1024);
        iris::umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, bdesc, idesc_o, (j > 0 || kk > 0));
      }
    };
    bool ok = iris::mbar_wait(&bars->q_full, 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA) &&
              iris::mbar_wait(&bars->k_full[0], 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA);
    if (ok) {
      iris::tc_fence_after();
      for (int t = 0; t < nq; t++) {
        qk(t, 0);
        iris::umma_commit(&bars->s_full[t]);
      }
      iris::umma_commit(&bars->k_empty[0]);
    }
    for (int j = 0; j < n && ok; j++) {
      const bool more = j + 1 < n;
      if (!iris::mbar_wait(&bars->v_full[j % VST], (uint32_t)((j / VST) & 1), abort_flag, p.status,
                           IRIS_DEV_ERR_ATTN_MMA)) {
        ok = false;
        break;
      }
      for (int t = 0; t < nq; t++) {
        if (!iris::mbar_wait(&bars->p_full[t], (uint32_t)(j & 1), abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        pv(t, j);
        if (more) {
          // K_{j+1} is first needed here, after P0_j V_j went in
          if (t == 0 && !iris::mbar_wait(&bars->k_full[(j + 1) % KST], (uint32_t)(((j + 1) / KST) & 1), abort_flag,
                                         p.status, IRIS_DEV_ERR_ATTN_MMA)) {
            ok = false;
            break;
          }
          iris::tc_fence_after();
          qk(t, j + 1);
          iris::umma_commit(&bars->s_full[t]);
        }
      }
      if (!ok) break;
      iris::umma_commit(&bars->v_empty[j % VST]);
      if (more) iris::umma_commit(&bars->k_empty[(j + 1) % KST]);
    }
    if (ok) {
      iris::umma_commit(&bars->o_done);
    } else {
      iris::umma_commit(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
    }
  } else if (warp >= 2 && (warp < 6 || has1)) {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >= 6 ? 1 : 0;  // query tile
    softmax_role<false, kMasked>(p, tmem, t, warp, lane, &bars->s_full[t], &bars->p_full[t], 0u, &bars->o_done, abort_flag,
                        q0 + t * BQ, col0, n, smem + OFF_K + (warp - 2) * O_STAGE_BYTES);
  }

  __syncthreads();
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, cta_group::2).  The pair holds four query
// tiles (two per CTA); every MMA is M = 256 over the pair: S_t = Q_t K_j^T
// takes query tile t of both CTAs and a key tile whose 128 keys are split
// 64 / 64 between the CTAs' shared memory; O_t += P_t V_j takes both CTAs'
// P_t from their TMEM and V_j's 128 head dimensions split 64 / 64.  Per CTA
// and K step the tensor cores read 6 KB (S) or 2 KB (O) of shared memory
// instead of 8 KB / 4 KB, which is what bounded the single-CTA kernel, and
// every K/V byte crosses L2 once per 256 query rows.  The even CTA's thread 32
// issues all MMAs; softmax and epilogue run in both CTAs as above.
constexpr int HALF = TILE / 2;  // 16 KB: a 64-key K half (two 64x64 boxes) or a 128-key x 64-dim V half
constexpr int PK_ST = 4;
constexpr int PV_ST = 4;
constexpr int P_OFF_K = 2 * TILE;
constexpr int P_OFF_V = P_OFF_K + PK_ST * HALF;
constexpr int P_OFF_BAR = P_OFF_V + PV_ST * HALF;
constexpr int P_SMEM_BYTES = P_OFF_BAR + 512 + 1024;

struct PairBars {
  uint64_t q_full;                           // even CTA: both CTAs' query tiles (2 arrivals + bytes)
  uint64_t k_full[PK_ST], k_empty[PK_ST];    // full: even CTA (2 arrivals + bytes); empty: each CTA
  uint64_t v_full[PV_ST], v_empty[PV_ST];
  uint64_t s_full[2];                        // each CTA
  uint64_t p_full[2];                        // even CTA: 8 warp arrivals (4 per CTA)
  uint64_t o_done;                           // each CTA
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int nkv;                                   // key tiles the pair visits (live_key_tiles)
};

static_assert(sizeof(AttnBars) <= 256 && sizeof(PairBars) <= 512, "barrier blocks fit their reserved shared bytes");
static_assert(8 * O_STAGE_BYTES <= (KST + VST) * TILE && 8 * O_STAGE_BYTES <= (PK_ST + PV_ST) * HALF,
              "the epilogue staging of eight softmax warps fits the K / V rings");

template <bool kMasked>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
attn_pair_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + P_OFF_BAR);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const uint32_t rank = iris::cluster_ctarank();
  const int q0 = (blockIdx.x >> 1) * (4 * BQ) + (int)rank * (2 * BQ);  // this CTA's two query tiles
  const int col0 = head * HD;
  const int kvcol0 = (head / p.kv_group) * HD;

  // Set-up before the wait for the previous kernel (a CTA that starts during
  // its tail allocates and initialises meanwhile); the masked instantiation
  // reads the key mask first, which the previous kernel may write.
  if (kMasked) iris::grid_dep_wait();
  if (warp == 2) {  // both CTAs of the pair: the same rows, the same count
    const int r0 = (blockIdx.x >> 1) * (4 * BQ);
    const int nkv = live_key_tiles<kMasked>(p, r0, min(p.sq, r0 + 4 * BQ) - 1, lane);
    if (lane == 0) bars->nkv = nkv;
  }
  if (threadIdx.x == 0) {
    iris::mbar_init(&bars->q_full, 2);
    for (int s = 0; s < PK_ST; s++) {
      iris::mbar_init(&bars->k_full[s], 2);
      iris::mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < PV_ST; s++) {
      iris::mbar_init(&bars->v_full[s], 2);
      iris::mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < 2; t++) {
      iris::mbar_init(&bars->s_full[t], 1);
      iris::mbar_init(&bars->p_full[t], 8);
    }
    iris::mbar_init(&bars->o_done, 1);
    iris::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    iris::fence_mbar_init();
    iris::tma_prefetch_desc(&p.tq);
    iris::tma_prefetch_desc(&p.tk);
    iris::tma_prefetch_desc(&p.tv);
  }
  if (warp == 1) iris::tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
  iris::tc_fence_before();
  __syncthreads();
  iris::cluster_sync();  // both CTAs' barriers exist before any remote arrive
  iris::tc_fence_after();
  if (!kMasked) iris::grid_dep_wait();  // Q, K and V come from the previous kernel
  const uint32_t tmem = bars->tmem_base;
  iris::grid_dep_launch();  // after this CTA's TMEM allocation
  const int n = bars->nkv;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const uint32_t qf = iris::mapa_shared(&bars->q_full, 0);
    iris::mbar_arrive_expect_tx_cluster(qf, 2 * TILE);
    for (int t = 0; t < 2; t++) {
      iris::tma_load_2d_pair(smem + t * TILE, &p.tq, qf, col0, q0 + t * BQ);
      iris::tma_load_2d_pair(smem + t * TILE + BOX, &p.tq, qf, col0 + 64, q0 + t * BQ);
    }
    int nk = 0, nv = 0;
    bool ok = true;
    auto load_k = [&]() -> bool {  // this CTA's 64 keys of key tile nk, both head-dim halves
      const int s = nk % PK_ST;
      const uint32_t u = (uint32_t)(nk / PK_ST);
      if (!iris::mbar_wait(&bars->k_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER))
        return false;
      const uint32_t kf = iris::mapa_shared(&bars->k_full[s], 0);
      iris::mbar_arrive_expect_tx_cluster(kf, HALF);
      const int krow = nk * BKV + 64 * (int)rank;
      iris::tma_load_2d_pair(smem + P_OFF_K + s * HALF, &p.tk, kf, kvcol0, krow);
      iris::tma_load_2d_pair(smem + P_OFF_K + s * HALF + HALF / 2, &p.tk, kf, kvcol0 + 64, krow);
      nk++;
      return true;
    };
    auto load_v = [&]() -> bool {  // this CTA's 64 head dims of value tile nv, all 128 keys
      const int s = nv % PV_ST;
      const uint32_t u = (uint32_t)(nv / PV_ST);
      if (!iris::mbar_wait(&bars->v_empty[s], (u & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_ATTN_PRODUCER))
        return false;
      const uint32_t vf = iris::mapa_shared(&bars->v_full[s], 0);
      iris::mbar_arrive_expect_tx_cluster(vf, HALF);
      iris::tma_load_2d_pair(smem + P_OFF_V + s * HALF, &p.tv, vf, kvcol0 + 64 * (int)rank, nv * BKV);
      nv++;
      return true;
    };
    while (ok && nk < (n < PK_ST ? n : PK_ST)) ok = load_k();
    while (ok && nv < (n < PV_ST ? n : PV_ST)) ok = load_v();
    while (ok && (nk < n || nv < n)) {
      if (nk < n) ok = load_k();
      if (ok && nv < n) ok = load_v();
    }
    if (!ok) {
      // the stage barriers live in the even CTA: give copies still in flight
      // (microseconds) time to land before this CTA can exit
      const uint64_t t0 = iris::globaltimer();
      while (iris::globaltimer() - t0 < 50000ull) {
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    const uint32_t idesc_s = iris::umma_idesc_bf16_f32(2 * BQ, BKV);
    const uint32_t idesc_o = iris::umma_idesc_bf16_f32_bmn(2 * BQ, HD);
    auto qk = [&](int t, int j) {  // S_t = Q_t K_j^T over the pair
      const uint32_t qa = iris::smem_u32(smem + t * TILE);
      const uint32_t kb = iris::smem_u32(smem + P_OFF_K + (j % PK_ST) * HALF);
#pragma unroll
      for (int kk = 0; kk < HD / 16; kk++) {
        const uint32_t in = (uint32_t)((kk & 3) * 32);
        iris::umma_bf16_pair(tmem + t * 128, iris::umma_desc_k_sw128(qa + (kk >> 2) * BOX + in),
                             iris::umma_desc_k_sw128(kb + (kk >> 2) * (HALF / 2) + in), idesc_s, kk > 0);
      }
    };
    auto pv = [&](int t, int j) {  // O_t += P_t V_j over the pair, P_t from TMEM
      const uint32_t vb = iris::smem_u32(smem + P_OFF_V + (j % PV_ST) * HALF);
#pragma unroll
      for (int kk = 0; kk < BKV / 16; kk++) {
        // B: this CTA's 64 head dims of V [keys, d] MN-major; 16 keys = 2048 B
        const uint64_t bdesc = iris::umma_desc_mn_sw128(vb + (uint32_t)(kk * 2048), BOX, 1024);
        iris::umma_bf16_pair_ts(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, bdesc, idesc_o, (j > 0 || kk > 0));
      }
    };
    bool ok = iris::mbar_wait(&bars->q_full, 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA) &&
              iris::mbar_wait(&bars->k_full[0], 0, abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA);
    if (ok) {
      iris::tc_fence_after();
      for (int t = 0; t < 2; t++) {
        qk(t, 0);
        iris::umma_commit_pair(&bars->s_full[t]);
      }
      iris::umma_commit_pair(&bars->k_empty[0]);
    }
    for (int j = 0; j < n && ok; j++) {
      const bool more = j + 1 < n;
      if (!iris::mbar_wait(&bars->v_full[j % PV_ST], (uint32_t)((j / PV_ST) & 1), abort_flag, p.status,
                           IRIS_DEV_ERR_ATTN_MMA)) {
        ok = false;
        break;
      }
      for (int t = 0; t < 2; t++) {
        if (!iris::mbar_wait(&bars->p_full[t], (uint32_t)(j & 1), abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        pv(t, j);
        if (more) {
          if (t == 0 && !iris::mbar_wait(&bars->k_full[(j + 1) % PK_ST], (uint32_t)(((j + 1) / PK_ST) & 1),
                                         abort_flag, p.status, IRIS_DEV_ERR_ATTN_MMA)) {
            ok = false;
            break;
          }
          iris::tc_fence_after();
          qk(t, j + 1);
          iris::umma_commit_pair(&bars->s_full[t]);
        }
      }
      if (!ok) break;
      iris::umma_commit_pair(&bars->v_empty[j % PV_ST]);
      if (more) iris::umma_commit_pair(&bars->k_empty[(j + 1) % PK_ST]);
    }
    if (ok) {
      iris::umma_commit_pair(&bars->o_done);
    } else {
      iris::umma_commit_pair(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_ATTN_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    const int t = warp >= 6 ? 1 : 0;
    softmax_role<true, kMasked>(p, tmem, t, warp, lane, &bars->s_full[t], nullptr, iris::mapa_shared(&bars->p_full[t], 0),
                       &bars->o_done, abort_flag, q0 + t * BQ, col0, n, smem + P_OFF_K + (warp - 2) * O_STAGE_BYTES);
  }

  __syncthreads();
  iris::cluster_sync();  // no CTA leaves while the pair MMA may still read its shared memory / TMEM
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Short sequences (at most 128 queries and 128 keys: a 64x64 image with a
// short prompt, a short text-encoder prompt).  There the tcgen05 kernels'
// fixed chain (TMEM allocation, TMA round trips, one key tile through
// S -> P -> O and the epilogue) costs several times the arithmetic.  This
// kernel takes 16 query rows of one head per CTA on the FMA pipe, in f32: K
// (transposed) and V staged in shared memory, two rows per warp; a lane owns
// keys lane + 32i of the scores and head dimensions 4 lane .. 4 lane + 3 of
// the output.  Masked keys take the logit -1e9 (natural-log units) as in the
// tensor-core kernels.
constexpr int SM_WARPS = 8;
constexpr int SM_RPW = 2;                    // query rows per warp
constexpr int SM_ROWS = SM_WARPS * SM_RPW;  // query rows per CTA
constexpr int SM_KEYS = 128;
constexpr int SM_SMEM = HD * SM_KEYS * 2 + SM_KEYS * HD * 2 + SM_ROWS * HD * 4 + SM_ROWS * SM_KEYS * 4;

struct SmallAttnArgs {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16* o;
  int ldq, ldk, ldo, sq, sk, kv_group, causal;
  float scale_log2;
  const uint8_t* kmask;
};

__global__ void __launch_bounds__(SM_WARPS * 32) attn_small_kernel(const __grid_constant__ SmallAttnArgs a) {
  constexpr int NT = SM_WARPS * 32;
  constexpr int VPT = SM_KEYS * (HD / 8) / NT;         // V chunks per thread
  constexpr int QPT = (SM_ROWS * (HD / 8) + NT - 1) / NT;  // Q chunks per thread
  extern __shared__ __align__(16) uint8_t sm_raw[];
  __nv_bfloat16* kt = reinterpret_cast<__nv_bfloat16*>(sm_raw);  // [HD][SM_KEYS]
  __nv_bfloat16* vs = kt + HD * SM_KEYS;                          // [SM_KEYS][HD]
  float* qs = reinterpret_cast<float*>(vs + SM_KEYS * HD);        // [SM_ROWS][HD]
  float* ps = qs + SM_ROWS * HD;                                  // [SM_ROWS][SM_KEYS]
  const int head = blockIdx.y, kvh = head / a.kv_group;
  const int r0 = blockIdx.x * SM_ROWS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  iris::grid_dep_wait();
  // every global load of the CTA's K, V and Q in flight before the first
  // shared-memory store (one L2 round trip)
  const int key = tid & (SM_KEYS - 1), dh = (tid >> 7) * (HD / 2);  // K: one key, half its dimensions
  uint4 kr[HD / 16], vr[VPT], qr[QPT];
  if (key < a.sk) {
    const __nv_bfloat16* src = a.k + (size_t)key * a.ldk + kvh * HD + dh;
#pragma unroll
    for (int c = 0; c < HD / 16; c++) kr[c] = *reinterpret_cast<const uint4*>(src + 8 * c);
  }
#pragma unroll
  for (int j = 0; j < VPT; j++) {  // V rows, 16-byte chunks
    const int i = tid + j * NT, vk = i >> 4, c = (i & 15) * 8;
    if (vk < a.sk) vr[j] = *reinterpret_cast<const uint4*>(a.v + (size_t)vk * a.ldk + kvh * HD + c);
  }
#pragma unroll
  for (int j = 0; j < QPT; j++) {  // Q rows, 16-byte chunks
    const int i = tid + j * NT, row = r0 + (i >> 4), c = (i & 15) * 8;
    if (i < SM_ROWS * (HD / 8) && row < a.sq)
      qr[j] = *reinterpret_cast<const uint4*>(a.q + (size_t)row * a.ldq + head * HD + c);
  }
  if (key < a.sk) {
#pragma unroll
    for (int c = 0; c < HD / 16; c++) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&kr[c]);
#pragma unroll
      for (int i = 0; i < 8; i++) kt[(dh + 8 * c + i) * SM_KEYS + key] = e[i];
    }
  }
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    const int i = tid + j * NT, vk = i >> 4, c = (i & 15) * 8;
    if (vk < a.sk) *reinterpret_cast<uint4*>(vs + vk * HD + c) = vr[j];
    else if (vk < ((a.sk + 3) & ~3)) *reinterpret_cast<uint4*>(vs + vk * HD + c) = make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int j = 0; j < QPT; j++) {  // Q as f32, zeros past sq
    const int i = tid + j * NT, r = i >> 4, c = (i & 15) * 8;
    if (i >= SM_ROWS * (HD / 8)) continue;
    float* d = qs + r * HD + c;
    if (r0 + r < a.sq) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&qr[j]);
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const float2 f = __bfloat1622float2(h[t]);
        d[2 * t] = f.x;
        d[2 * t + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; t++) d[t] = 0.f;
    }
  }
  __syncthreads();
  iris::grid_dep_launch();
  const int ra = SM_RPW * warp;  // this warp's first row within the CTA
  float sc[SM_RPW][4];
#pragma unroll
  for (int r = 0; r < SM_RPW; r++)
#pragma unroll
    for (int i = 0; i < 4; i++) sc[r][i] = 0.f;
#pragma unroll 2
  for (int d0 = 0; d0 < HD; d0 += 4) {
    float qv[SM_RPW][4];
#pragma unroll
    for (int r = 0; r < SM_RPW; r++) {
      const float4 q4 = *reinterpret_cast<const float4*>(qs + (ra + r) * HD + d0);
      qv[r][0] = q4.x;
      qv[r][1] = q4.y;
      qv[r][2] = q4.z;
      qv[r][3] = q4.w;
    }
#pragma unroll
    for (int dd = 0; dd < 4; dd++) {
      const uint2 u = *reinterpret_cast<const uint2*>(kt + (d0 + dd) * SM_KEYS + 4 * lane);  // keys 4 lane ..
      const float2 ka = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 kb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      const float kv[4] = {ka.x, ka.y, kb.x, kb.y};
#pragma unroll
      for (int r = 0; r < SM_RPW; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) sc[r][i] = fmaf(qv[r][dd], kv[i], sc[r][i]);
    }
  }
  float inv[SM_RPW];
#pragma unroll
  for (int r = 0; r < SM_RPW; r++) {
    const int row = r0 + ra + r;
    float x[4], m = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int key = 4 * lane + i;
      if (key >= a.sk) x[i] = -INFINITY;
      else if ((a.kmask && !a.kmask[key]) || (a.causal && key > row)) x[i] = -1e9f * LOG2E;
      else x[i] = sc[r][i] * a.scale_log2;
      m = fmaxf(m, x[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float e[4], l = 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      e[i] = exp2f(x[i] - m);
      l += e[i];
    }
    *reinterpret_cast<float4*>(ps + (ra + r) * SM_KEYS + 4 * lane) = make_float4(e[0], e[1], e[2], e[3]);
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    inv[r] = 1.0f / l;
  }
  __syncwarp();  // the warp reads back its own rows of P
  float acc[SM_RPW][4];
#pragma unroll
  for (int r = 0; r < SM_RPW; r++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[r][i] = 0.f;
  const int sk4 = (a.sk + 3) & ~3;  // keys past sk: P = 0 and V rows of zeros
#pragma unroll 2
  for (int k0 = 0; k0 < sk4; k0 += 4) {
    float pv[SM_RPW][4];
#pragma unroll
    for (int r = 0; r < SM_RPW; r++) {
      const float4 p4 = *reinterpret_cast<const float4*>(ps + (ra + r) * SM_KEYS + k0);
      pv[r][0] = p4.x;
      pv[r][1] = p4.y;
      pv[r][2] = p4.z;
      pv[r][3] = p4.w;
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint2 u = *reinterpret_cast<const uint2*>(vs + (k0 + kk) * HD + 4 * lane);
      const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 vb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      const float vv[4] = {va.x, va.y, vb.x, vb.y};
#pragma unroll
      for (int r = 0; r < SM_RPW; r++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[r][i] = fmaf(pv[r][kk], vv[i], acc[r][i]);
    }
  }
#pragma unroll
  for (int r = 0; r < SM_RPW; r++) {
    const int row = r0 + ra + r;
    if (row < a.sq)
      *reinterpret_cast<uint2*>(a.o + (size_t)row * a.ldo + head * HD + 4 * lane) =
          make_uint2(pack_bf16(acc[r][0] * inv[r], acc[r][1] * inv[r]),
                     pack_bf16(acc[r][2] * inv[r], acc[r][3] * inv[r]));
  }
}

bool g_attn_tc_attr = false;

}  // namespace

extern "C" void iris_attention_set_status(int* status) { g_attn_status = status; }

extern "C" cudaError_t iris_attention_tc_init(void) {
  if (g_attn_tc_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SM_SMEM);
  if (e == cudaSuccess) g_attn_tc_attr = true;
  return e;
}

extern "C" cudaError_t iris_launch_attention_tc(const void* q, int ldq, const void* k, const void* v, int ldk,
                                                void* o, int ldo, int sq, int sk, int heads, float scale,
                                                const uint8_t* key_mask, cudaStream_t stream) {
  return iris_launch_attention_gqa(q, ldq, k, v, ldk, o, ldo, sq, sk, heads, 1, 0, scale, key_mask, stream);
}

extern "C" cudaError_t iris_launch_attention_gqa(const void* q, int ldq, const void* k, const void* v, int ldk,
                                                 void* o, int ldo, int sq, int sk, int heads, int kv_group,
                                                 int causal, float scale, const uint8_t* key_mask,
                                                 cudaStream_t stream) {
  if (sq <= 0 || sk <= 0 || heads <= 0) return cudaSuccess;
  if (kv_group < 1 || heads % kv_group) return cudaErrorInvalidValue;
  if ((ldq | ldk | ldo) & 7) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(key_mask) & 3) return cudaErrorInvalidValue;  // read four bytes at a time
  if (!g_attn_tc_attr) {
    cudaError_t e = iris_attention_tc_init();
    if (e != cudaSuccess) return e;
  }
  if (sq <= SM_KEYS && sk <= SM_KEYS) {  // short sequences: the FMA-pipe kernel above
    SmallAttnArgs a;
    a.q = static_cast<const __nv_bfloat16*>(q);
    a.k = static_cast<const __nv_bfloat16*>(k);
    a.v = static_cast<const __nv_bfloat16*>(v);
    a.o = static_cast<__nv_bfloat16*>(o);
    a.ldq = ldq;
    a.ldk = ldk;
    a.ldo = ldo;
    a.sq = sq;
    a.sk = sk;
    a.kv_group = kv_group;
    a.causal = causal;
    a.scale_log2 = scale * LOG2E;
    a.kmask = key_mask;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(o)) & 15)
      return cudaErrorInvalidValue;
    return iris::launch_overlapped(attn_small_kernel, dim3((sq + SM_ROWS - 1) / SM_ROWS, heads), dim3(SM_WARPS * 32),
                                   SM_SMEM, stream, a);
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms = n;
  }
  // Pairs take four 128-row query tiles each.  A short sequence (a 512-token
  // prompt) would leave most SMs idle with pairs: one query tile per CTA on
  // the single-CTA kernel then spreads the work over four times the CTAs and
  // shortens each CTA's chain of key tiles.
  const long pair_ctas = 2L * ((sq + 4 * BQ - 1) / (4 * BQ)) * heads;
  const int one_tile = pair_ctas <= sms / 2;
  const int single = one_tile;
  AttnParams p;
  memset(&p, 0, sizeof(p));
  // the pair kernel loads 64-key halves of each key tile
  if (iris_make_tmap_bf16(&p.tq, q, (uint64_t)sq, (uint64_t)heads * HD, (uint64_t)ldq, BQ) ||
      iris_make_tmap_bf16(&p.tk, k, (uint64_t)sk, (uint64_t)(heads / kv_group) * HD, (uint64_t)ldk,
                          single ? BKV : 64) ||
      iris_make_tmap_bf16(&p.tv, v, (uint64_t)sk, (uint64_t)(heads / kv_group) * HD, (uint64_t)ldk, BKV))
    return cudaErrorInvalidValue;
  p.o = static_cast<__nv_bfloat16*>(o);
  p.ldo = ldo;
  p.sq = sq;
  p.sk = sk;
  p.scale_log2 = scale * LOG2E;
  p.kmask = key_mask;
  p.causal = causal;
  p.kv_group = kv_group;
  p.one_tile = one_tile;
  p.status = g_attn_status;
  const bool masked = key_mask != nullptr || causal;
  if (single) {
    const int rows = one_tile ? BQ : 2 * BQ;
    dim3 grid((sq + rows - 1) / rows, heads);
    return iris::launch_overlapped(masked ? attn_tc_kernel<true> : attn_tc_kernel<false>, grid, dim3(NUM_THREADS),
                                   SMEM_BYTES, stream, p);
  }
  dim3 grid(2 * ((sq + 4 * BQ - 1) / (4 * BQ)), heads);
  return iris::launch_overlapped(masked ? attn_pair_kernel<true> : attn_pair_kernel<false>, grid, dim3(NUM_THREADS),
                                 P_SMEM_BYTES, stream, p);
}

// Attention entry point (the tcgen05 kernels above).
extern "C" cudaError_t iris_launch_attention(const void* q, int ldq, const void* k, const void* v, int ldk,
                                             void* o, int ldo, int sq, int sk, int heads, float scale,
                                             const uint8_t* key_mask, cudaStream_t stream) {
  return iris_launch_attention_tc(q, ldq, k, v, ldk, o, ldo, sq, sk, heads, scale, key_mask, stream);
}
