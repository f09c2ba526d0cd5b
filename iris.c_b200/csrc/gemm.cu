// Persistent tcgen05 GEMM for the DiT linears, with the block epilogues fused.
//
//   C[M, N] = A[M, K] * W[N, K]^T     (bf16 operands, f32 accumulation in TMEM)
//
// Replaces the reference's per-linear sgemm calls (iris_linear_nobias /
// iris_linear_nobias_bf16, iris_kernels.c:220-336; LINEAR_BF16_OR_F32,
// iris_transformer_flux.c:121) together with the elementwise passes that
// follow them: QK-RMSNorm + RoPE (:1464, :1026), SiLU-gate * up (:2299),
// gate * proj + residual (:136) and the split/concat copies of the single
// block (:3833-3840, :3896-3902).
//
// CTA layout (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile 128x64 and W tile bn x 64 per stage
//   warp 1      TMEM owner + MMA issuer (one thread): 4 x UMMA 128xbnx16 per stage
//   warps 2..5  epilogue: TMEM -> registers -> fused math -> global
// Two TMEM accumulators (2 x 256 columns) let the epilogue of tile i overlap
// the main loop of tile i+1.  Tiles are ordered M-fastest so the CTAs that
// run concurrently share one weight column band in L2.
#include "iris_kernels.h"
#include "ptx.cuh"
#include "rope.cuh"

#include <cuda_bf16.h>
#include <stdlib.h>
#include <string.h>

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int STAGES = 4;                   // with 128-row A tiles
constexpr int MAX_STAGES = 5;               // with A tiles of at most 80 rows
constexpr int SMEM_LIMIT = 232448;          // dynamic shared memory a CTA may opt into
constexpr int A_BYTES = BM * BK * 2;        // 16 KB
constexpr int B_BYTES_MAX = 256 * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES_MAX;
constexpr int NUM_THREADS = 192;          // single-CTA kernel: producer, MMA, 4 epilogue warps
constexpr int EPI_WARPS2 = 8;             // CTA-pair kernel: two epilogue warps per TMEM lane quarter
constexpr int NUM_THREADS2 = 64 + 32 * EPI_WARPS2;
constexpr int TMEM_COLS = 512;
// f32 epilogue staging: 32 rows x (32 + 4) floats per epilogue warp, so that
// 16-byte shared accesses run in conflict-free 8-lane phases
constexpr int EPI_LD = 36;
constexpr int EPI_WARP_BYTES = 32 * EPI_LD * 4;
constexpr int EPI_BYTES = 4 * EPI_WARP_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*barriers*/ + EPI_BYTES + 1024 /*align slack*/;

struct Bars {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tile_coords(const IrisGemmParams& p, int t, int mt0, int mtot,
                                            int& g, int& m_local, int& n0) {
  int nt = t / mtot;
  int mt = t - nt * mtot;
  g = (mt < mt0) ? 0 : 1;
  m_local = g ? mt - mt0 : mt;
  n0 = nt * p.bn;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// x * sigmoid(x) with the fast divide (a reciprocal and a multiply, within 2
// ulp: far below the bf16 rounding of the result).  For x below about -88,
// 1 + e^-x is infinite or beyond 2^126 and the quotient is 0, the limit.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Store 32 f32 values (cols j0..j0+31 of a chunk) as bf16 to dst (16B aligned).
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    uint4 u;
    u.x = pack_bf16(v[8 * i + 0], v[8 * i + 1]);
    u.y = pack_bf16(v[8 * i + 2], v[8 * i + 3]);
    u.z = pack_bf16(v[8 * i + 4], v[8 * i + 5]);
    u.w = pack_bf16(v[8 * i + 6], v[8 * i + 7]);
    d[i] = u;
  }
}

// Epilogue for NC consecutive 128-column chunks (heads) of one row that belong
// to the Q/K/V region (NC = 2 only when both are Q or K heads).  TMEM loads
// are warp-collective and always executed by all 32 lanes; only the
// global-memory traffic is predicated on `valid`.  The pair rotation is
// evaluated in registers: the row's four position ids (one 8-byte load) and,
// per 32-column block, the 16 pairs' frequencies, axes and K scales (the same
// for every row: L1 broadcasts) give cos / sin of pos * freq
// (iris::rope_cos_sin; position 0 gives exactly cos 1, sin 0, the identity, as
// the reference's tables hold).  A block's 16 evaluations have no branch
// between them, so they overlap each other and the block's TMEM load, and
// serve every head of the row; a block is skipped as a whole when every row of
// the warp has position 0 on all of its axes (text rows have only L, image
// rows T = 0 and L = 0) and no band scale.  The norm weights come from L1 too.
template <int NC>
__device__ __forceinline__ void epi_qkv_chunks(const IrisGemmParams& p, uint32_t taddr, int g, int row, bool valid,
                                               int col0) {
  int which[NC];
  __nv_bfloat16* dst[NC];
  const float* nw[NC];
  float r[NC];
  bool kscale[NC];
  const bool qk = col0 / p.H < 2;  // (all NC chunks are Q / K heads, or NC = 1)
  const bool rope = qk && p.rope_pos != nullptr && valid;
  iris::RopePos pos = {{0u, 0u, 0u, 0u}};
  if (rope) pos = iris::rope_load_pos(p.rope_pos, row);
  bool anyk = false;
#pragma unroll
  for (int h = 0; h < NC; h++) {
    const int c0 = col0 + 128 * h;
    which[h] = c0 / p.H;
    const int cin = c0 - which[h] * p.H;
    dst[h] = reinterpret_cast<__nv_bfloat16*>(which[h] == 0 ? p.q : which[h] == 1 ? p.k : p.v) +
             (size_t)row * p.ldqkv + cin;
    // K of the rows a launch marks takes the band scale (SREF, single blocks)
    kscale[h] = which[h] == 1 && p.rope_k_row0 > 0 && row >= p.rope_k_row0;
    anyk |= kscale[h];
    r[h] = 1.0f;
    nw[h] = nullptr;
    if (which[h] < 2) {
      // pass 1: sum of squares over the 128-wide head (TMEM is re-read in pass 2
      // rather than keeping 128 values live in registers)
      nw[h] = (which[h] == 0) ? p.qnorm[g] : p.knorm[g];
      float ss = 0.f;
#pragma unroll 1
      for (int j = 0; j < 4; j++) {
        float v[32];
        iris::tmem_ld32(taddr + 128 * h + 32 * j, v);
#pragma unroll
        for (int e = 0; e < 32; e++) ss += v[e] * v[e];
      }
      r[h] = rsqrtf(ss * (1.0f / 128.0f) + p.eps);
    }
  }
#pragma unroll 1
  for (int j = 0; j < 4; j++) {
    float rc[16], rs[16];  // this row's cos / sin of the block's 16 pairs
    bool rot = false;      // some row of the warp has a non-zero position on an axis of this block
    if (qk && p.rope_pos) {
      const uint32_t am = __ldg(p.rope_spec->axis_mask + j);
      bool nz = anyk;
#pragma unroll
      for (int a = 0; a < 4; a++) nz |= ((am >> a) & 1u) && pos.v[a] != 0u;
      rot = __any_sync(0xffffffffu, rope && nz);
    }
    if (rot && rope) {
      const float4* f4 = reinterpret_cast<const float4*>(p.rope_spec->freq + 16 * j);
      const uint32_t axb = __ldg(p.rope_spec->axis_bits + j);
#pragma unroll
      for (int q4 = 0; q4 < 4; q4++) {
        const float4 f = __ldg(f4 + q4);
        const float fq[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int e = 4 * q4 + u;
          iris::rope_cos_sin(iris::rope_axis_pos(pos, (int)((axb >> (2 * e)) & 3u)), fq[u], rc[e], rs[e]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < NC; h++) {
      float v[32];
      iris::tmem_ld32(taddr + 128 * h + 32 * j, v);
      if (!valid) continue;
      if (which[h] < 2) {
        const float4* w4 = reinterpret_cast<const float4*>(nw[h] + 32 * j);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float4 w = __ldg(w4 + e);
          v[4 * e + 0] = v[4 * e + 0] * r[h] * w.x;
          v[4 * e + 1] = v[4 * e + 1] * r[h] * w.y;
          v[4 * e + 2] = v[4 * e + 2] * r[h] * w.z;
          v[4 * e + 3] = v[4 * e + 3] * r[h] * w.w;
        }
        if (rot && rope) {
#pragma unroll
          for (int e = 0; e < 16; e++) {
            const float f = kscale[h] ? __ldg(p.rope_spec->kscale + 16 * j + e) : 1.0f;
            const float c = rc[e] * f, sn = rs[e] * f;
            const float x0 = v[2 * e], x1 = v[2 * e + 1];
            v[2 * e] = x0 * c - x1 * sn;
            v[2 * e + 1] = x1 * c + x0 * sn;
          }
        }
      }
      store_bf16x32(dst[h] + 32 * j, v);
    }
  }
}

// Epilogue for a 256-column tile laid out as [gate 128 | up 128].
__device__ __forceinline__ void epi_swiglu_tile(const IrisGemmParams& p, uint32_t taddr, int row,
                                                bool valid, int n0, int j0 = 0, int j1 = 4) {
  int f0 = (n0 - p.swiglu_base) >> 1;
  __nv_bfloat16* dst =
      reinterpret_cast<__nv_bfloat16*>(p.mlp_out) + (size_t)row * p.ld_mlp + p.mlp_col0 + f0;
#pragma unroll 1
  for (int j = j0; j < j1; j++) {
    float gv[32], uv[32];
    iris::tmem_ld32x2(taddr + 32 * j, taddr + 128 + 32 * j, gv, uv);
#pragma unroll
    for (int e = 0; e < 32; e++) gv[e] = silu_f(gv[e]) * uv[e];
    if (valid) store_bf16x32(dst + 32 * j, gv);
  }
}

// ---------------------------------------------------------------- tensor parallelism
// IRIS_EPI_TP_SCATTER: gate * acc of a 32 x 32 block straight into the
// owning ranks' receive buffers (peer memory), transposed through the warp's
// staging tile so that each store covers 4 rows x 128 contiguous bytes.
__device__ __forceinline__ void epi_scatter_block(const IrisGemmParams& p, int g, float* stage, const float* v,
                                                  int lane, int row_first, int rows_valid, int c) {
  float4* st = reinterpret_cast<float4*>(stage + lane * EPI_LD);
#pragma unroll
  for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int rr = lane >> 3, c4 = (lane & 7) * 4;
  const float4 gg = __ldg(reinterpret_cast<const float4*>(p.gate[g] + c + c4));
  const int chunk = p.tp.chunk;
#pragma unroll
  for (int it = 0; it < 8; it++) {
    const int r = it * 4 + rr;
    if (r < rows_valid) {
      const int row = row_first + r, o = row / chunk;
      const float4 a = *reinterpret_cast<const float4*>(stage + r * EPI_LD + c4);
      float* d = p.tp.recv[o] + ((size_t)p.tp.rank * chunk + (row - o * chunk)) * p.N + c + c4;
      *reinterpret_cast<float4*>(d) = make_float4(gg.x * a.x, gg.y * a.y, gg.z * a.z, gg.w * a.w);
    }
  }
  __syncwarp();
}

// f32 outputs (plain store or gated residual update) of a 32-row x 32-column
// block: lane i holds row row_first + i in v.  The block is transposed through
// this warp's shared staging tile so that every global access covers 4 rows x
// 128 contiguous bytes (one thread per row would touch 32 rows per access).
__device__ __forceinline__ void epi_f32_block(const IrisGemmParams& p, int g, float* stage, const float* v,
                                              int lane, int row_first, int rows_valid, int c, float* out_base,
                                              int ldo, bool resid) {
  float4* st = reinterpret_cast<float4*>(stage + lane * EPI_LD);
#pragma unroll
  for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int rr = lane >> 3, c4 = (lane & 7) * 4;
  float* base = out_base + (size_t)(row_first + rr) * ldo + c + c4;
  const size_t step = (size_t)4 * ldo;  // 4 rows per pass
  // all residual loads in flight before the first store
  float4 h[8];
#pragma unroll
  for (int it = 0; it < 8; it++) {
    h[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (resid && !p.resid_store && it * 4 + rr < rows_valid)
      h[it] = __ldcg(reinterpret_cast<const float4*>(base + it * step));
  }
  const float4 gg = resid ? __ldg(reinterpret_cast<const float4*>(p.gate[g] + c + c4)) : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
  for (int it = 0; it < 8; it++) {
    const int r = it * 4 + rr;
    const float4 a = *reinterpret_cast<const float4*>(stage + r * EPI_LD + c4);
    float4 o = h[it];
    o.x += gg.x * a.x;
    o.y += gg.y * a.y;
    o.z += gg.z * a.z;
    o.w += gg.w * a.w;
    if (r < rows_valid) *reinterpret_cast<float4*>(base + it * step) = o;
  }
  __syncwarp();  // the stage is rewritten by the next block
}

// IRIS_EPI_LORA_FOLD, 32-column blocks j0..j1-1 of a 128-column chunk:
// out = bf16(w0 + scale * acc) at each row's target row.  The warp's 32 x 32
// accumulator block is transposed through its shared staging tile so that
// four lanes cover one row's 64 contiguous bytes (every base-weight and output
// sector fully used, 8 rows per access), and the base values of all the
// chunk's blocks are loaded before the first accumulator block is read.
__device__ __forceinline__ void epi_fold_chunk(const IrisGemmParams& p, uint32_t taddr, int row, bool valid,
                                               int col0, int j0, int j1, float* stage, int lane) {
  const int my_drow = valid ? __ldg(p.fold_rows + row) : -1;
  const int rr = lane >> 2, c8 = (lane & 3) * 8;
  int dr[4];
#pragma unroll
  for (int it = 0; it < 4; it++) dr[it] = __shfl_sync(0xffffffffu, my_drow, it * 8 + rr);
  const __nv_bfloat16* w0 = static_cast<const __nv_bfloat16*>(p.fold_w0);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
  uint4 base[16];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if (j < j0 || j >= j1) continue;
#pragma unroll
    for (int it = 0; it < 4; it++)
      if (dr[it] >= 0)
        base[4 * j + it] = *reinterpret_cast<const uint4*>(w0 + (size_t)dr[it] * p.ldo + col0 + 32 * j + c8);
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    if (j < j0 || j >= j1) continue;
    float v[32];
    iris::tmem_ld32(taddr + 32 * j, v);  // warp-collective: every lane
    float4* st = reinterpret_cast<float4*>(stage + lane * EPI_LD);
#pragma unroll
    for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 4; it++) {
      if (dr[it] < 0) continue;
      const float* a = stage + (it * 8 + rr) * EPI_LD + c8;
      const float4 a0 = *reinterpret_cast<const float4*>(a), a1 = *reinterpret_cast<const float4*>(a + 4);
      const float acc[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint4 b = base[4 * j + it];
      const uint32_t u[4] = {b.x, b.y, b.z, b.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float lo = __uint_as_float(u[q] << 16) + p.fold_scale * acc[2 * q];
        const float hi = __uint_as_float(u[q] & 0xFFFF0000u) + p.fold_scale * acc[2 * q + 1];
        o[q] = pack_bf16(lo, hi);
      }
      *reinterpret_cast<uint4*>(out + (size_t)dr[it] * p.ldo + col0 + 32 * j + c8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncwarp();  // the stage is rewritten by the next block
  }
}

__device__ __forceinline__ void epi_plain_chunk(const IrisGemmParams& p, uint32_t taddr, int g,
                                                int row, int row_local, bool valid, int col0, float* stage,
                                                int lane, int rows_valid, int split, int j0 = 0, int j1 = 4) {
#pragma unroll 1
  for (int j = j0; j < j1; j++) {
    float v[32];
    iris::tmem_ld32(taddr + 32 * j, v);
    int c = col0 + 32 * j;
    if (p.mode == IRIS_EPI_TP_SCATTER) {
      epi_scatter_block(p, g, stage, v, lane, row - lane, rows_valid, c);
      continue;
    }
    if (p.splitk > 1) {
      // raw partial of this K range -> workspace slice `split` (reduced later)
      const size_t span = (size_t)(p.ngroups > 1 ? p.row0[1] + p.rows[1] : p.row0[0] + p.rows[0]);
      epi_f32_block(p, g, stage, v, lane, row - lane, rows_valid, c, p.ws + (size_t)split * span * p.N, p.N,
                    false);
      continue;
    }
    if (p.mode == IRIS_EPI_RESID_GATE || p.mode == IRIS_EPI_F32) {
      if (p.bias) {
#pragma unroll
        for (int e = 0; e < 32; e++) v[e] += __ldg(p.bias + c + e);
      }
      // warp-collective: every lane takes part, rows_valid masks the stores
      epi_f32_block(p, g, stage, v, lane, row - lane, rows_valid, c, reinterpret_cast<float*>(p.out), p.ldo,
                    p.mode == IRIS_EPI_RESID_GATE);
      continue;
    }
    if (!valid) continue;
    if (p.bias) {
#pragma unroll
      for (int e = 0; e < 32; e++) v[e] += __ldg(p.bias + c + e);
    }
    if (p.mode == IRIS_EPI_BF16 || p.mode == IRIS_EPI_GATE_BF16) {
      if (p.mode == IRIS_EPI_GATE_BF16) {
        const float4* gp = reinterpret_cast<const float4*>(p.gate[g] + c);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float4 gg = __ldg(gp + e);
          v[4 * e] *= gg.x;
          v[4 * e + 1] *= gg.y;
          v[4 * e + 2] *= gg.z;
          v[4 * e + 3] *= gg.w;
        }
      }
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + c, v);
    } else if (p.mode == IRIS_EPI_F32) {
      float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + c);
#pragma unroll
      for (int e = 0; e < 8; e++) d[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    } else if (p.mode == IRIS_EPI_F32_NCHW) {
      float* d = reinterpret_cast<float*>(p.out) + row_local;
#pragma unroll
      for (int e = 0; e < 32; e++) d[(size_t)(c + e) * p.nchw_rows] = v[e];
    } else {  // IRIS_EPI_RESID_GATE
      float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + c);
      const float4* gp = reinterpret_cast<const float4*>(p.gate[g] + c);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        float4 h = p.resid_store ? make_float4(0.f, 0.f, 0.f, 0.f) : d[e], gg = __ldg(gp + e);
        h.x += gg.x * v[4 * e];
        h.y += gg.y * v[4 * e + 1];
        h.z += gg.z * v[4 * e + 2];
        h.w += gg.w * v[4 * e + 3];
        d[e] = h;
      }
    }
  }
}

// Gated-residual epilogues read the residual rows of their tile: each
// epilogue thread asks L2 for its row's slice of the tile one main loop ahead
// (the weights streaming through L2 would otherwise leave it a DRAM miss
// right when the tensor pipe waits for the accumulator).
__device__ __forceinline__ void prefetch_resid_row(const IrisGemmParams& p, int g, int row_local, int n0) {
  if (p.mode == IRIS_EPI_LORA_FOLD) {  // the base weight row segment the fold reads
    if (row_local >= p.rows[g]) return;
    const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(p.fold_w0) +
                             (size_t)__ldg(p.fold_rows + p.row0[g] + row_local) * p.ldo + n0;
    const int bytes = min(p.bn, p.N - n0) * 2;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w), "r"(bytes) : "memory");
    return;
  }
  if (p.mode != IRIS_EPI_RESID_GATE || p.resid_store || row_local >= p.rows[g]) return;
  const float* a = reinterpret_cast<const float*>(p.out) + (size_t)(p.row0[g] + row_local) * p.ldo + n0;
  const int bytes = min(p.bn, p.N - n0) * 4;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(bytes) : "memory");
}

// Epilogue of one accumulator tile for this thread's row (all modes); the
// warp's 32 rows start at row - lane, rows_valid of them are real.  With two
// epilogue warps per lane quarter (halves = 2), warp `half` takes the
// 128-column chunk `half` of a 256-wide tile, or half of the 32-column blocks
// of a 128-wide one (a Q/K head's RMSNorm needs its whole chunk in one warp).
// kFold: the IRIS_EPI_LORA_FOLD instantiation of the kernels (its epilogue
// keeps a whole base-weight chunk in registers; compiled apart so that the
// other epilogues keep their register allocation).
template <bool kFold>
__device__ __forceinline__ void epi_tile(const IrisGemmParams& p, uint32_t taddr, int g, int row, int row_local,
                                         bool valid, int n0, float* stage, int lane, int rows_valid,
                                         int split = 0, int half = 0, int halves = 1) {
  if constexpr (kFold) {
    const int nchunks = p.bn / 128;
    for (int c = 0; c < nchunks; c++) {
      const int col0 = n0 + c * 128;
      if (col0 >= p.N) break;
      if (halves == 2 && nchunks == 2 && c != half) continue;
      if (halves == 2 && nchunks == 1)
        epi_fold_chunk(p, taddr + c * 128, row, valid, col0, 2 * half, 2 * half + 2, stage, lane);
      else epi_fold_chunk(p, taddr + c * 128, row, valid, col0, 0, 4, stage, lane);
    }
    return;
  }
  bool swiglu_tile = (p.mode == IRIS_EPI_SWIGLU) || (p.mode == IRIS_EPI_SINGLE && n0 >= p.swiglu_base);
  if (swiglu_tile) {
    if (halves == 2) epi_swiglu_tile(p, taddr, row, valid, n0, 2 * half, 2 * half + 2);
    else epi_swiglu_tile(p, taddr, row, valid, n0);
  } else {
    const int nchunks = p.bn / 128;
    for (int c = 0; c < nchunks; c++) {
      int col0 = n0 + c * 128;
      if (col0 >= p.N) break;
      const bool qkv = p.mode == IRIS_EPI_QKV || p.mode == IRIS_EPI_SINGLE;
      if (halves == 2 && nchunks == 2 && c != half) continue;
      if (qkv) {
        if (halves == 2 && nchunks == 1 && half) continue;
        // one warp holding both heads of a Q/K tile: their rotation is evaluated once
        if (halves == 1 && nchunks == 2 && c == 0 && col0 + 256 <= 2 * p.H && col0 + 256 <= p.N) {
          epi_qkv_chunks<2>(p, taddr, g, row, valid, col0);
          break;
        }
        epi_qkv_chunks<1>(p, taddr + c * 128, g, row, valid, col0);
      } else if (halves == 2 && nchunks == 1) {
        epi_plain_chunk(p, taddr + c * 128, g, row, row_local, valid, col0, stage, lane, rows_valid, split,
                        2 * half, 2 * half + 2);
      } else {
        epi_plain_chunk(p, taddr + c * 128, g, row, row_local, valid, col0, stage, lane, rows_valid, split);
      }
    }
  }
}

template <bool kFold>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ IrisGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // Stages of A (a_box rows; with fewer than 128 the tensor cores' reads of
  // rows a_box..127 fall into the stage's B tile: rows no epilogue stores)
  // and B (up to 256 rows); their number is set by the host to fill shared memory.
  const int nst = p.nstages > 0 ? p.nstages : STAGES;
  const uint32_t a_bytes = (uint32_t)(p.a_box ? p.a_box : BM) * BK * 2;
  const uint32_t stage_bytes = a_bytes + B_BYTES_MAX;
  Bars* bars = reinterpret_cast<Bars*>(smem + nst * stage_bytes);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int mt0 = (p.rows[0] + BM - 1) / BM;
  const int mt1 = p.ngroups > 1 ? (p.rows[1] + BM - 1) / BM : 0;
  const int mtot = mt0 + mt1;
  const int ntiles_n = (p.N + p.bn - 1) / p.bn;
  const int nsplit = p.splitk > 1 ? p.splitk : 1;
  const int total = mtot * ntiles_n * nsplit;  // work units: (tile, K split)
  const int num_kb = (p.K + BK - 1) / BK;
  const uint32_t b_bytes = (uint32_t)p.bn * BK * 2;
  const uint32_t idesc = iris::umma_idesc_bf16_f32(BM, p.bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; s++) {
      iris::mbar_init(&bars->full[s], 1);
      iris::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      iris::mbar_init(&bars->tfull[b], 1);
      iris::mbar_init(&bars->tempty[b], 128);
    }
    iris::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    iris::fence_mbar_init();
    iris::tma_prefetch_desc(&p.tmap_a);
    iris::tma_prefetch_desc(&p.tmap_b[0]);
    if (p.ngroups > 1) iris::tma_prefetch_desc(&p.tmap_b[1]);
  }
  if (warp == 1) iris::tmem_alloc(&bars->tmem_base, TMEM_COLS);
  iris::tc_fence_before();
  __syncthreads();
  iris::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // The prologue above overlapped the previous kernel's tail; so do the
  // weight loads of the first stages when B is a resident weight.
  const int pre = (p.b_static && p.tp.size <= 1 && blockIdx.x < total && !kFold)
                      ? min(nst, (blockIdx.x % nsplit + 1) * num_kb / nsplit - (blockIdx.x % nsplit) * num_kb / nsplit)
                      : 0;
  if (warp == 0 && lane == 0 && pre > 0) {
    int g, ml, n0;
    tile_coords(p, blockIdx.x / nsplit, mt0, mtot, g, ml, n0);
    const int kb0 = (blockIdx.x % nsplit) * num_kb / nsplit;
    for (int s = 0; s < pre; s++) {
      iris::mbar_arrive_expect_tx(&bars->full[s], a_bytes + b_bytes);
      for (int h = 0; h < p.bn / 128; h++)
        iris::tma_load_2d(smem + s * stage_bytes + a_bytes + h * (128 * BK * 2), &p.tmap_b[g], &bars->full[s],
                          (kb0 + s) * BK, n0 + 128 * h);
    }
  }
  iris::grid_dep_wait();
  if (!kFold) iris::grid_dep_launch();  // a fold rewrites weights: nothing may start early after it

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    long issued = 0;
    bool ok = true;
    if (p.tp.size > 1 && p.tp.wait_x) {  // A rows written by peer GPUs: wait for all of them
      ok = iris::tp_wait(p.tp, IRIS_TP_X, IRIS_TP_BASE_X, p.tp.wait_x, p.status);
      if (!ok) *abort_flag = 1;
      iris::fence_proxy_async_global();
    }
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      int g, ml, n0;
      tile_coords(p, u / nsplit, mt0, mtot, g, ml, n0);
      int arow = p.row0[g] + ml * BM;
      const int sp = u % nsplit, kb0 = sp * num_kb / nsplit, kb1 = (sp + 1) * num_kb / nsplit;
      for (int kb = kb0; kb < kb1; kb++) {
        if (!iris::mbar_wait(&bars->empty[stage], phase ^ 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_PRODUCER)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * stage_bytes;
        uint8_t* sb = sa + a_bytes;
        const bool b_done = issued < pre;  // the first unit's early weight stages
        if (!b_done) iris::mbar_arrive_expect_tx(&bars->full[stage], a_bytes + b_bytes);
        iris::tma_load_2d(sa, &p.tmap_a, &bars->full[stage], kb * BK, arow);
        for (int h = 0; h < p.bn / 128 && !b_done; h++)  // weight tensor maps have 128-row boxes
          iris::tma_load_2d(sb + h * (128 * BK * 2), &p.tmap_b[g], &bars->full[stage], kb * BK, n0 + 128 * h);
        issued++;
        if (++stage == nst) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {
      // Drain: wait (bounded) for the copies this thread issued last, so no
      // TMA write lands in shared memory after the CTA exits.
      long n = issued < nst ? issued : nst;
      int s = stage;
      uint32_t ph = phase;
      for (long i = 0; i < n; i++) {
        if (--s < 0) { s = nst - 1; ph ^= 1; }
        volatile int no_abort = 0;
        iris::mbar_wait(&bars->full[s], ph, &no_abort, p.status, IRIS_DEV_ERR_GEMM_DRAIN);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x, it++) {
      int buf = it & 1;
      uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tempty[buf], (use & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_MMA)) {
        ok = false;
        break;
      }
      iris::tc_fence_after();
      uint32_t d_tmem = tmem_base + buf * 256;
      const int sp = u % nsplit, kb0 = sp * num_kb / nsplit, kb1 = (sp + 1) * num_kb / nsplit;
      for (int kb = kb0; kb < kb1; kb++) {
        if (!iris::mbar_wait(&bars->full[stage], phase, abort_flag, p.status, IRIS_DEV_ERR_GEMM_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        uint32_t sa = iris::smem_u32(smem + stage * stage_bytes);
        uint32_t sb = sa + a_bytes;
        uint64_t adesc = iris::umma_desc_k_sw128(sa);
        uint64_t bdesc = iris::umma_desc_k_sw128(sb);
#pragma unroll
        for (int kk = 0; kk < BK / 16; kk++) {
          // +32 bytes along K inside the 128B swizzle atom = +2 in the >>4 address field
          iris::umma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb != kb0 || kk != 0));
        }
        iris::umma_commit(&bars->empty[stage]);
        if (++stage == nst) { stage = 0; phase ^= 1; }
      }
      if (ok) iris::umma_commit(&bars->tfull[buf]);
    }
    if (!ok) {
      iris::umma_commit(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_GEMM_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    // f32 staging (only the epilogues that stage get it from the host)
    float* stage = reinterpret_cast<float*>(smem + nst * stage_bytes + 1024 + (warp - 2) * EPI_WARP_BYTES);
    int it = 0;
    if (blockIdx.x < total && nsplit == 1) {
      int g, ml, n0;
      tile_coords(p, blockIdx.x, mt0, mtot, g, ml, n0);
      prefetch_resid_row(p, g, ml * BM + quarter * 32 + lane, n0);
    }
    for (int u = blockIdx.x; u < total; u += gridDim.x, it++) {
      int buf = it & 1;
      uint32_t use = (uint32_t)(it >> 1);
      if (u + (int)gridDim.x < total && nsplit == 1) {
        int g2, ml2, n02;
        tile_coords(p, u + gridDim.x, mt0, mtot, g2, ml2, n02);
        prefetch_resid_row(p, g2, ml2 * BM + quarter * 32 + lane, n02);
      }
      if (!iris::mbar_wait(&bars->tfull[buf], use & 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_EPILOGUE)) break;
      iris::tc_fence_after();
      int g, ml, n0;
      tile_coords(p, u / nsplit, mt0, mtot, g, ml, n0);
      int row_local = ml * BM + quarter * 32 + lane;
      bool valid = row_local < p.rows[g];
      int row = p.row0[g] + row_local;
      uint32_t taddr = tmem_base + buf * 256 + ((uint32_t)(quarter * 32) << 16);
      const int rows_valid = min(32, max(0, p.rows[g] - (row_local - lane)));
      epi_tile<kFold>(p, taddr, g, row, row_local, valid, n0, stage, lane, rows_valid, u % nsplit);
      iris::tc_fence_before();
      iris::mbar_arrive(&bars->tempty[buf]);
    }
    if (p.mode == IRIS_EPI_TP_SCATTER) {
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps' stores are issued
      if (warp == 2 && lane == 0) iris::tp_signal(p.tp, IRIS_TP_DONE_GEMM, IRIS_TP_PART, gridDim.x);
    }
  }

  __syncthreads();
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, cta_group::2): one MMA of M = 256, N = 256
// per K step, issued by the even CTA over both CTAs' shared memory.  Each CTA
// loads its own 128 rows of A and its own 128-row half of the weight tile, so
// per CTA and K step the tensor cores read 8 KB of shared memory instead of
// 12 KB and the weights cross L2 once per 256 rows instead of per 128.  Each
// CTA's TMEM holds the accumulator of its own 128 rows; both epilogues run as
// in the single-CTA kernel.
constexpr int BM2 = 256;
constexpr int STAGES2 = 5;
constexpr int STAGE2_BYTES = A_BYTES + 128 * BK * 2;  // 32 KB
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + EPI_WARPS2 * EPI_WARP_BYTES + 1024;
// IRIS_EPI_LORA_FOLD instantiation: 2 stages, and per epilogue warp a landing
// buffer for the next tile's base-weight block (32 rows x 128 columns bf16)
constexpr int FOLD_STAGES2 = 2;
constexpr int FOLD_LANDING_BYTES = 32 * 128 * 2;
constexpr int FOLD_SMEM2_BYTES = FOLD_STAGES2 * STAGE2_BYTES + 1024 + EPI_WARPS2 * EPI_WARP_BYTES +
                                 EPI_WARPS2 * FOLD_LANDING_BYTES + 1024;

struct Bars2 {
  uint64_t full[STAGES2];   // even CTA: both CTAs' tiles of the stage landed (2 arrivals + bytes)
  uint64_t empty[STAGES2];  // each CTA: the pair MMA released the stage
  uint64_t tfull[2];        // each CTA: accumulator ready
  uint64_t tempty[2];       // even CTA: both epilogues drained the accumulator (8 warp arrivals)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Fold epilogue of one pair-kernel warp (rows quarter*32.. of this CTA's 128,
// column half `half` of each 256-wide tile).  The base-weight block of the
// next tile is copied into this warp's landing buffer (cp.async, 16 bytes per
// lane and piece) while the current tile is combined, so every SM keeps
// 8 x 8 KB of base-weight reads in flight.  The pieces are laid out so that
// each lane reads back exactly the slots it copied: no cross-lane hazard.
__device__ __forceinline__ void fold_issue(const IrisGemmParams& p, uint4* landing, int t, int mt0, int mtot,
                                           uint32_t rank, int quarter, int half, int lane, int* dr) {
  int g, ml, n0;
  tile_coords(p, t, mt0, mtot, g, ml, n0);
  const int row_local = ml * BM2 + 128 * (int)rank + quarter * 32 + lane;
  const int my = row_local < p.rows[g] ? __ldg(p.fold_rows + p.row0[g] + row_local) : -1;
  const int rr = lane >> 2, c8 = (lane & 3) * 8, col0 = n0 + half * 128;
#pragma unroll
  for (int it = 0; it < 4; it++) dr[it] = __shfl_sync(0xffffffffu, my, it * 8 + rr);
  const __nv_bfloat16* w0 = static_cast<const __nv_bfloat16*>(p.fold_w0);
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int it = 0; it < 4; it++)
      if (dr[it] >= 0) {
        const void* src = w0 + (size_t)dr[it] * p.ldo + col0 + 32 * j + c8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(iris::smem_u32(landing + (4 * j + it) * 32 + lane)),
                     "l"(src) : "memory");
      }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void fold_epilogue_pair(const IrisGemmParams& p, uint64_t* tfull, uint32_t tempty_c0,
                                                   uint32_t tempty_c1, volatile int* abort_flag, uint32_t tmem_base,
                                                   float* stage, uint4* landing, int pair, int npairs, int total,
                                                   int mt0, int mtot, uint32_t rank, int quarter, int half,
                                                   int lane) {
  int dr[4], drn[4];
  if (pair < total) fold_issue(p, landing, pair, mt0, mtot, rank, quarter, half, lane, drn);
  const int rr = lane >> 2, c8 = (lane & 3) * 8;
  int it = 0;
  for (int t = pair; t < total; t += npairs, it++) {
    const int buf = it & 1;
    const uint32_t use = (uint32_t)(it >> 1);
    if (!iris::mbar_wait(&tfull[buf], use & 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_EPILOGUE)) break;
    iris::tc_fence_after();
    // this tile's base block: landed copies -> registers, then the next tile's copies
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    uint4 base[16];
#pragma unroll
    for (int q = 0; q < 16; q++) base[q] = landing[q * 32 + lane];
#pragma unroll
    for (int q = 0; q < 4; q++) dr[q] = drn[q];
    if (t + 2 * npairs < total) {  // the tile after next: its base rows into L2
      int g2, ml2, n02;
      tile_coords(p, t + 2 * npairs, mt0, mtot, g2, ml2, n02);
      if (half == 0) prefetch_resid_row(p, g2, ml2 * BM2 + 128 * (int)rank + quarter * 32 + lane, n02);
    }
    if (t + npairs < total) fold_issue(p, landing, t + npairs, mt0, mtot, rank, quarter, half, lane, drn);
    int g, ml, n0;
    tile_coords(p, t, mt0, mtot, g, ml, n0);
    const int col0 = n0 + half * 128;
    const uint32_t taddr = tmem_base + buf * 256 + ((uint32_t)(quarter * 32) << 16) + half * 128;
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float v[32];
      iris::tmem_ld32(taddr + 32 * j, v);
      float4* st = reinterpret_cast<float4*>(stage + lane * EPI_LD);
#pragma unroll
      for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      __syncwarp();
#pragma unroll
      for (int r = 0; r < 4; r++) {
        if (dr[r] < 0) continue;
        const float* a = stage + (r * 8 + rr) * EPI_LD + c8;
        const float4 a0 = *reinterpret_cast<const float4*>(a), a1 = *reinterpret_cast<const float4*>(a + 4);
        const float acc[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint4 b = base[4 * j + r];
        const uint32_t u[4] = {b.x, b.y, b.z, b.w};
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float lo = __uint_as_float(u[q] << 16) + p.fold_scale * acc[2 * q];
          const float hi = __uint_as_float(u[q] & 0xFFFF0000u) + p.fold_scale * acc[2 * q + 1];
          o[q] = pack_bf16(lo, hi);
        }
        *reinterpret_cast<uint4*>(out + (size_t)dr[r] * p.ldo + col0 + 32 * j + c8) =
            make_uint4(o[0], o[1], o[2], o[3]);
      }
      __syncwarp();  // the stage is rewritten by the next block
    }
    iris::tc_fence_before();
    __syncwarp();
    if (lane == 0) iris::mbar_arrive_cluster(buf ? tempty_c1 : tempty_c0);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // no copy lands after the CTA has moved on
}

template <bool kFold>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS2, 1)
gemm_tc2_kernel(const __grid_constant__ IrisGemmParams p) {
  // the fold's K is one block: two stages free the shared memory for its
  // base-weight landing buffers
  constexpr int kStages = kFold ? FOLD_STAGES2 : STAGES2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars2* bars = reinterpret_cast<Bars2*>(smem + kStages * STAGE2_BYTES);
  volatile int* abort_flag = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = iris::cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  const int mt0 = (p.rows[0] + BM2 - 1) / BM2;
  const int mt1 = p.ngroups > 1 ? (p.rows[1] + BM2 - 1) / BM2 : 0;
  const int mtot = mt0 + mt1;
  const int ntiles_n = (p.N + p.bn - 1) / p.bn;
  const int total = mtot * ntiles_n;
  const int num_kb = (p.K + BK - 1) / BK;
  const uint32_t idesc = iris::umma_idesc_bf16_f32(BM2, 256);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      iris::mbar_init(&bars->full[s], 2);
      iris::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      iris::mbar_init(&bars->tfull[b], 1);
      iris::mbar_init(&bars->tempty[b], 2 * EPI_WARPS2);
    }
    iris::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    iris::fence_mbar_init();
    iris::tma_prefetch_desc(&p.tmap_a);
    iris::tma_prefetch_desc(&p.tmap_b[0]);
    if (p.ngroups > 1) iris::tma_prefetch_desc(&p.tmap_b[1]);
  }
  if (warp == 1) iris::tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
  iris::tc_fence_before();
  __syncthreads();
  iris::cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  iris::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  // The prologue above overlapped the previous kernel's tail; so do the
  // weight loads of the first stages when B is a resident weight.
  const int pre = (p.b_static && p.tp.size <= 1 && pair < total && !kFold) ? min(kStages, num_kb) : 0;
  if (warp == 0 && lane == 0 && pre > 0) {
    int g, ml, n0;
    tile_coords(p, pair, mt0, mtot, g, ml, n0);
    for (int s = 0; s < pre; s++) {
      const uint32_t full_c = iris::mapa_shared(&bars->full[s], 0);
      iris::mbar_arrive_expect_tx_cluster(full_c, STAGE2_BYTES);
      iris::tma_load_2d_pair(smem + s * STAGE2_BYTES + A_BYTES, &p.tmap_b[g], full_c, s * BK, n0 + 128 * (int)rank);
    }
  }
  iris::grid_dep_wait();
  if (!kFold) iris::grid_dep_launch();  // a fold rewrites weights: nothing may start early after it

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true, issued_any = pre > 0;
    if (p.tp.size > 1 && p.tp.wait_x) {  // A rows written by peer GPUs: wait for all of them
      ok = iris::tp_wait(p.tp, IRIS_TP_X, IRIS_TP_BASE_X, p.tp.wait_x, p.status);
      if (!ok) *abort_flag = 1;
      iris::fence_proxy_async_global();
    }
    for (int t = pair; t < total && ok; t += npairs) {
      int g, ml, n0;
      tile_coords(p, t, mt0, mtot, g, ml, n0);
      const int arow = p.row0[g] + ml * BM2 + 128 * (int)rank;
      const int brow = n0 + 128 * (int)rank;
      for (int kb = 0; kb < num_kb; kb++) {
        if (!iris::mbar_wait(&bars->empty[stage], phase ^ 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_PRODUCER)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * STAGE2_BYTES;
        uint8_t* sb = sa + A_BYTES;
        const uint32_t full_c = iris::mapa_shared(&bars->full[stage], 0);
        const bool b_done = t == pair && kb < pre;  // the first tile's early weight stages
        if (!b_done) iris::mbar_arrive_expect_tx_cluster(full_c, STAGE2_BYTES);
        iris::tma_load_2d_pair(sa, &p.tmap_a, full_c, kb * BK, arow);
        if (!b_done) iris::tma_load_2d_pair(sb, &p.tmap_b[g], full_c, kb * BK, brow);
        issued_any = true;
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && issued_any) {
      // the stage barriers live in the even CTA: give copies still in flight
      // (microseconds) time to land before this CTA can exit
      const uint64_t t0 = iris::globaltimer();
      while (iris::globaltimer() - t0 < 50000ull) {
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------ MMA issuer (even CTA)
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs, it++) {
      int buf = it & 1;
      uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tempty[buf], (use & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_MMA)) {
        ok = false;
        break;
      }
      iris::tc_fence_after();
      uint32_t d_tmem = tmem_base + buf * 256;
      for (int kb = 0; kb < num_kb; kb++) {
        if (!iris::mbar_wait(&bars->full[stage], phase, abort_flag, p.status, IRIS_DEV_ERR_GEMM_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        uint32_t sa = iris::smem_u32(smem + stage * STAGE2_BYTES);
        uint32_t sb = sa + A_BYTES;
        uint64_t adesc = iris::umma_desc_k_sw128(sa);
        uint64_t bdesc = iris::umma_desc_k_sw128(sb);
#pragma unroll
        for (int kk = 0; kk < BK / 16; kk++)
          iris::umma_bf16_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
        iris::umma_commit_pair(&bars->empty[stage]);
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (ok) iris::umma_commit_pair(&bars->tfull[buf]);
    }
    if (!ok) {
      iris::umma_commit_pair(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_GEMM_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue (both CTAs, 8 warps)
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = ew >> 2;      // which half of the tile's columns
    float* stage = reinterpret_cast<float*>(smem + kStages * STAGE2_BYTES + 1024 + ew * EPI_WARP_BYTES);
    const uint32_t tempty_c0 = iris::mapa_shared(&bars->tempty[0], 0);
    const uint32_t tempty_c1 = iris::mapa_shared(&bars->tempty[1], 0);
    int it = 0;
    if constexpr (kFold) {
      uint4* landing = reinterpret_cast<uint4*>(smem + kStages * STAGE2_BYTES + 1024 +
                                                EPI_WARPS2 * EPI_WARP_BYTES + ew * FOLD_LANDING_BYTES);
      fold_epilogue_pair(p, bars->tfull, tempty_c0, tempty_c1, abort_flag, tmem_base, stage, landing, pair, npairs,
                         total, mt0, mtot, rank, quarter, half, lane);
    } else {
    if (pair < total && half == 0) {
      int g, ml, n0;
      tile_coords(p, pair, mt0, mtot, g, ml, n0);
      prefetch_resid_row(p, g, ml * BM2 + 128 * (int)rank + quarter * 32 + lane, n0);
    }
    for (int t = pair; t < total; t += npairs, it++) {
      int buf = it & 1;
      uint32_t use = (uint32_t)(it >> 1);
      if (t + npairs < total && half == 0) {
        int g2, ml2, n02;
        tile_coords(p, t + npairs, mt0, mtot, g2, ml2, n02);
        prefetch_resid_row(p, g2, ml2 * BM2 + 128 * (int)rank + quarter * 32 + lane, n02);
      }
      if (!iris::mbar_wait(&bars->tfull[buf], use & 1, abort_flag, p.status, IRIS_DEV_ERR_GEMM_EPILOGUE)) break;
      iris::tc_fence_after();
      int g, ml, n0;
      tile_coords(p, t, mt0, mtot, g, ml, n0);
      int row_local = ml * BM2 + 128 * (int)rank + quarter * 32 + lane;
      bool valid = row_local < p.rows[g];
      int row = p.row0[g] + row_local;
      uint32_t taddr = tmem_base + buf * 256 + ((uint32_t)(quarter * 32) << 16);
      const int rows_valid = min(32, max(0, p.rows[g] - (row_local - lane)));
      epi_tile<kFold>(p, taddr, g, row, row_local, valid, n0, stage, lane, rows_valid, 0, half, 2);
      iris::tc_fence_before();
      __syncwarp();
      if (lane == 0) iris::mbar_arrive_cluster(buf ? tempty_c1 : tempty_c0);
    }
    }
    if (p.mode == IRIS_EPI_TP_SCATTER) {
      asm volatile("bar.sync 1, %0;" ::"r"(32 * EPI_WARPS2) : "memory");  // every epilogue warp's stores are issued
      if (ew == 0 && lane == 0) iris::tp_signal(p.tp, IRIS_TP_DONE_GEMM, IRIS_TP_PART, gridDim.x);
    }
  }

  __syncthreads();
  iris::cluster_sync();  // no CTA leaves while the pair MMA may still read its shared memory
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Split-K reduction: out = epilogue(sum of the K-range partials) for every
// real row (fixed summation order, so results do not depend on scheduling).
__global__ void splitk_reduce_kernel(const __grid_constant__ IrisGemmParams p, int span) {
  const int row = blockIdx.y;
  const int g = (p.ngroups > 1 && row >= p.row0[1]) ? 1 : 0;
  const int local = row - p.row0[g];
  if (local < 0 || local >= p.rows[g]) return;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (c >= p.N) return;
  iris::grid_dep_wait();
  iris::grid_dep_launch();
  const size_t slice = (size_t)span * p.N;
  const float* w = p.ws + (size_t)row * p.N + c;
  // partials requested 8 at a time (one L2 round trip per batch instead of
  // one per split), added in split order
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < p.splitk; s0 += 8) {
    float4 part[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (s0 + i < p.splitk) part[i] = __ldcg(reinterpret_cast<const float4*>(w + (s0 + i) * slice));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (s0 + i >= p.splitk) break;
      if (s0 + i == 0) {
        acc = part[0];
      } else {
        acc.x += part[i].x;
        acc.y += part[i].y;
        acc.z += part[i].z;
        acc.w += part[i].w;
      }
    }
  }
  if (p.bias) {
    const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + c));
    acc.x += b.x;
    acc.y += b.y;
    acc.z += b.z;
    acc.w += b.w;
  }
  if (p.mode == IRIS_EPI_RESID_GATE) {
    float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + c);
    const float4 gg = __ldg(reinterpret_cast<const float4*>(p.gate[g] + c));
    float4 h = p.resid_store ? make_float4(0.f, 0.f, 0.f, 0.f) : *d;
    h.x += gg.x * acc.x;
    h.y += gg.y * acc.y;
    h.z += gg.z * acc.z;
    h.w += gg.w * acc.w;
    *d = h;
  } else if (p.mode == IRIS_EPI_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + c) = acc;
  } else {  // IRIS_EPI_BF16
    uint2 o = make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + c) = o;
  }
}

// Split-K reduction of a gated residual update fused with the adaLN that
// reads the updated rows next: one CTA per row, a thread per 4 columns.  The
// row's new residual is stored as the plain reduction would store it, then
// LayerNorm (mean, then the variance around it, eps inside the root) and the
// row group's modulation give the next GEMM's bf16 operand.
__global__ void __launch_bounds__(1024) splitk_reduce_ln_kernel(const __grid_constant__ IrisGemmParams p) {
  const int row = blockIdx.x;
  const int g = (p.ngroups > 1 && row >= p.row0[1]) ? 1 : 0;
  const int local = row - p.row0[g];
  if (local < 0 || local >= p.rows[g]) return;  // the whole CTA
  const int c = threadIdx.x * 4;
  const int span = p.ngroups > 1 ? p.row0[1] + p.rows[1] : p.row0[0] + p.rows[0];
  iris::grid_dep_wait();
  iris::grid_dep_launch();
  const size_t slice = (size_t)span * p.N;
  const float* w = p.ws + (size_t)row * p.N + c;
  float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)row * p.ldo + c);
  const float4 gg = __ldg(reinterpret_cast<const float4*>(p.gate[g] + c));
  float4 h = *d;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < p.splitk; s0 += 8) {
    float4 part[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (s0 + i < p.splitk) part[i] = __ldcg(reinterpret_cast<const float4*>(w + (s0 + i) * slice));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (s0 + i >= p.splitk) break;
      if (s0 + i == 0) {
        acc = part[0];
      } else {
        acc.x += part[i].x;
        acc.y += part[i].y;
        acc.z += part[i].z;
        acc.w += part[i].w;
      }
    }
  }
  if (p.bias) {
    const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + c));
    acc.x += b.x;
    acc.y += b.y;
    acc.z += b.z;
    acc.w += b.w;
  }
  h.x += gg.x * acc.x;
  h.y += gg.y * acc.y;
  h.z += gg.z * acc.z;
  h.w += gg.w * acc.w;
  *d = h;
  __shared__ float red[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  auto block_sum = [&](float v) -> float {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();  // red is reused
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
  };
  const float mean = block_sum((h.x + h.y) + (h.z + h.w)) / (float)p.N;
  const float a0 = h.x - mean, a1 = h.y - mean, a2 = h.z - mean, a3 = h.w - mean;
  const float var = block_sum((a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3)) / (float)p.N;
  const float rstd = 1.0f / sqrtf(var + p.ln_eps);
  const int gl = row >= p.ln_split ? 1 : 0;
  const float4 sh = __ldg(reinterpret_cast<const float4*>(p.ln_shift[gl] + c));
  const float4 sc = __ldg(reinterpret_cast<const float4*>(p.ln_scale[gl] + c));
  const float y0 = (1.0f + sc.x) * (a0 * rstd) + sh.x, y1 = (1.0f + sc.y) * (a1 * rstd) + sh.y;
  const float y2 = (1.0f + sc.z) * (a2 * rstd) + sh.z, y3 = (1.0f + sc.w) * (a3 * rstd) + sh.w;
  *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.ln_out) + (size_t)row * p.ln_ld + c) =
      make_uint2(pack_bf16(y0, y1), pack_bf16(y2, y3));
}

}  // namespace

extern "C" int iris_make_tmap_bf16(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols,
                                   uint64_t ld, uint32_t box_rows) {
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                               const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                               const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f)
      return -1;
    fn = reinterpret_cast<EncodeFn>(f);
  }
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * 2) & 15) || box_rows == 0 || box_rows > 256)
    return -2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  // 128-row boxes at most: a 256-row weight tile is loaded as two boxes (the
  // swizzled layout of two stacked 128-row boxes equals one 256-row box)
  cuuint32_t box[2] = {64, box_rows > 128 ? 128u : box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

static bool g_gemm_attr = false;
static int g_max_pairs = 0;  // CTA pairs that can be resident at once

extern "C" cudaError_t iris_gemm_init(void) {
  if (g_gemm_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_LIMIT);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc2_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc2_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FOLD_SMEM2_BYTES);
  if (e == cudaSuccess) {
    // clusters are placed within GPCs: ask how many pairs fit at once rather
    // than assuming SMs / 2 (a persistent grid larger than that would run its
    // last pairs after the others)
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS2, 1, 1);
    cfg.dynamicSmemBytes = SMEM2_BYTES;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, gemm_tc2_kernel<false>, &cfg);
    g_max_pairs = (e == cudaSuccess && n > 0) ? n : 0;
    e = cudaSuccess;
    cudaGetLastError();
  }
  if (e == cudaSuccess) g_gemm_attr = true;
  return e;
}

extern "C" cudaError_t iris_launch_gemm(const IrisGemmParams* p, int num_sms, cudaStream_t stream) {
  return iris_launch_gemm_ex(p, num_sms, stream, nullptr);
}

// Launch plan of a GEMM: the CTA-pair kernel, or the single-CTA kernel with
// `splitk` K splits (1: none).
struct GemmPlan {
  bool pair;
  long grid;
  int splitk;
};

static GemmPlan gemm_plan(const IrisGemmParams* p, int num_sms) {
  GemmPlan g = {false, 0, 1};
  const int rows = p->rows[0] + (p->ngroups > 1 ? p->rows[1] : 0);
  const bool linear = p->mode == IRIS_EPI_BF16 || p->mode == IRIS_EPI_F32 || p->mode == IRIS_EPI_RESID_GATE;
  if (p->bn == 256 && rows >= 512 && g_max_pairs > 0) {
    int mt = (p->rows[0] + BM2 - 1) / BM2 + (p->ngroups > 1 ? (p->rows[1] + BM2 - 1) / BM2 : 0);
    long total = (long)mt * ((p->N + 255) / 256);
    long cap = g_max_pairs < num_sms / 2 ? g_max_pairs : num_sms / 2;
    // a pair grid under half the pairs leaves SMs idle: a linear epilogue with a
    // workspace goes to the single-CTA kernel below, which splits K instead
    const bool split_instead = p->ws && linear && 2 * total < cap && p->K / BK >= 8;
    if (!split_instead) {
      g.pair = true;
      g.grid = 2 * (total < cap ? total : cap);
      return g;
    }
  }
  int mt = (p->rows[0] + BM - 1) / BM + (p->ngroups > 1 ? (p->rows[1] + BM - 1) / BM : 0);
  long tiles = (long)mt * ((p->N + p->bn - 1) / p->bn);
  // Few output tiles (a short sequence): split K so that enough CTAs stream
  // the weights, when the caller gave a workspace and the epilogue is linear.
  const int num_kb = (p->K + BK - 1) / BK;
  const int span = p->ngroups > 1 ? p->row0[1] + p->rows[1] : p->row0[0] + p->rows[0];
  if (p->ws && tiles > 0 && tiles < num_sms / 2 && num_kb >= 8 && linear) {
    long s = num_sms / tiles;
    if (s > num_kb / 4) s = num_kb / 4;
    const long fit = (long)(p->ws_bytes / ((size_t)span * p->N * sizeof(float)));
    if (s > fit) s = fit;
    if (s >= 2) g.splitk = (int)s;
  }
  const long total = tiles * g.splitk;
  g.grid = total < num_sms ? total : num_sms;
  return g;
}

extern "C" int iris_gemm_splits(const IrisGemmParams* p, int num_sms) {
  if (!g_gemm_attr && iris_gemm_init() != cudaSuccess) return 1;
  return gemm_plan(p, num_sms).splitk;
}


extern "C" cudaError_t iris_launch_gemm_ex(const IrisGemmParams* p, int num_sms, cudaStream_t stream,
                                           int* launches) {
  if (launches) *launches = 1;
  if (!g_gemm_attr) {
    cudaError_t e = iris_gemm_init();
    if (e != cudaSuccess) return e;
  }
  if (p->bn != 128 && p->bn != 256) return cudaErrorInvalidValue;
  if (p->K % BK != 0 || p->N % 128 != 0) return cudaErrorInvalidValue;
  // A tensor-parallel launch waits on peer GPUs: it starts only after the
  // previous kernel has finished, as an ordinary launch does.
  const bool overlap = p->tp.size <= 1;
  const GemmPlan plan = gemm_plan(p, num_sms);
  if (plan.pair) {
    if (p->ln_out) return cudaErrorInvalidValue;  // the adaLN is applied by split-K reductions only
    if (p->mode == IRIS_EPI_LORA_FOLD)
      gemm_tc2_kernel<true><<<(int)plan.grid, NUM_THREADS2, FOLD_SMEM2_BYTES, stream>>>(*p);
    else if (overlap)
      return iris::launch_overlapped(gemm_tc2_kernel<false>, dim3((unsigned)plan.grid), dim3(NUM_THREADS2),
                                     SMEM2_BYTES, stream, *p);
    else
      gemm_tc2_kernel<false><<<(int)plan.grid, NUM_THREADS2, SMEM2_BYTES, stream>>>(*p);
    return cudaGetLastError();
  }
  if (plan.grid <= 0) return cudaSuccess;
  IrisGemmParams q = *p;
  q.splitk = plan.splitk;
  const int span = p->ngroups > 1 ? p->row0[1] + p->rows[1] : p->row0[0] + p->rows[0];
  const int grid = (int)plan.grid;
  // A stages of a_box rows (every tile's rows must lie inside the box), and
  // as many stages as shared memory holds next to the f32 staging of the
  // epilogues that use it
  if (p->a_box) {
    if (p->a_box % 8 || p->a_box > BM || p->mode == IRIS_EPI_LORA_FOLD || p->rows[0] > p->a_box ||
        (p->ngroups > 1 && p->rows[1] > p->a_box))
      return cudaErrorInvalidValue;
  }
  const bool staging = p->mode == IRIS_EPI_RESID_GATE || p->mode == IRIS_EPI_F32 ||
                       p->mode == IRIS_EPI_TP_SCATTER || q.splitk > 1;
  const size_t stage_bytes = (size_t)(p->a_box ? p->a_box : BM) * BK * 2 + B_BYTES_MAX;
  const size_t fixed = 1024 /*barriers*/ + (staging ? EPI_BYTES : 0) + 1024 /*align slack*/;
  q.nstages = (int)((SMEM_LIMIT - fixed) / stage_bytes);
  if (q.nstages > MAX_STAGES) q.nstages = MAX_STAGES;
  const size_t smem = (size_t)q.nstages * stage_bytes + fixed;
  // the reduction applies the next adaLN when asked to (one CTA per row)
  const bool ln = q.splitk > 1 && p->ln_out && p->mode == IRIS_EPI_RESID_GATE && !p->resid_store &&
                  p->N % 128 == 0 && p->N <= 4 * 1024;
  if (p->ln_out && !ln) return cudaErrorInvalidValue;  // the caller relies on the adaLN being applied
  cudaError_t e;
  if (q.mode == IRIS_EPI_LORA_FOLD) {
    q.nstages = STAGES;
    gemm_tc_kernel<true><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(q);
    e = cudaGetLastError();
  } else if (overlap) {
    e = iris::launch_overlapped(gemm_tc_kernel<false>, dim3(grid), dim3(NUM_THREADS), smem, stream, q);
  } else {
    gemm_tc_kernel<false><<<grid, NUM_THREADS, smem, stream>>>(q);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess || q.splitk == 1) return e;
  if (launches) *launches = 2;
  if (ln)
    return iris::launch_overlapped(splitk_reduce_ln_kernel, dim3(span), dim3(p->N / 4), 0, stream, q);
  return iris::launch_overlapped(splitk_reduce_kernel, dim3((p->N / 4 + 255) / 256, span), dim3(256), 0, stream,
                                 q, span);
}

