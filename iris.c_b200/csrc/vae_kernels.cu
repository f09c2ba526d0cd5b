// Autoencoder decoder kernels: the convolutions as implicit GEMMs on the
// tcgen05 tensor cores, GroupNorm, and the small data-movement steps around
// them.  Replaces the reference's CPU decoder passes (iris_vae_decode,
// iris_vae.c:835-990: iris_conv2d im2col + sgemm, iris_group_norm, swish,
// iris_upsample_nearest, iris_unpatchify) and its Metal equivalents
// (iris_gpu_conv2d_f32 / group_norm_f32 / swish_f32 / upsample_nearest_2x_f32,
// iris_metal.h:520-565).
//
// Activations are NHWC ("pixel rows" of channels): a 3x3 convolution is then
// a GEMM whose K index runs over (tap, input channel), and the A tile of one
// (tap, 64-channel block) is a single 3-D TMA box {64 channels, bw, bh pixels}
// of the input at the tap's offset.  Pixels outside the image read as zeros
// (TMA out-of-bounds fill), which is exactly the convolution's zero padding,
// so no padded copy of any activation exists.
#include "iris_kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <string.h>

#define IRIS_DEV_ERR_CONV_PRODUCER 0x401
#define IRIS_DEV_ERR_CONV_MMA 0x402
#define IRIS_DEV_ERR_CONV_EPILOGUE 0x403
#define IRIS_DEV_ERR_CONV_DRAIN 0x404

namespace {

constexpr int CBM = 128;                    // output pixels per CTA tile
constexpr int CBK = 64;                     // input channels per K block
constexpr int CA_BYTES = CBM * CBK * 2;     // 16 KB
constexpr int C_EPI_WARPS = 8;               // two per TMEM lane quarter, splitting the columns
constexpr int CNUM_THREADS = 64 + 32 * C_EPI_WARPS;
constexpr int CTMEM_COLS = 512;
constexpr int C_EPI_LD = 36;
constexpr int C_EPI_WARP_BYTES = 32 * C_EPI_LD * 4;
// per epilogue warp: 32 groups x {sum, sum of squares} (f64)
constexpr int C_GN_BYTES = C_EPI_WARPS * 32 * 2 * 8;
// single CTA: 3 stages of A 16 KB + B (bn <= 256 rows) 32 KB; CTA pair: each
// CTA holds half of B, 5 stages of A 16 KB + B 16 KB
template <bool kPair>
struct ConvCfg {
  static constexpr int STAGES = kPair ? 5 : 3;
  static constexpr int STAGE_BYTES = kPair ? CA_BYTES + 128 * CBK * 2 : CA_BYTES + 256 * CBK * 2;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + C_EPI_WARPS * C_EPI_WARP_BYTES + C_GN_BYTES + 1024;
};

struct ConvBars {
  uint64_t full[6];
  uint64_t empty[6];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int32_t c,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(iris::smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(iris::smem_u32(bar)), "r"(c), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load into this CTA's shared memory, completion signalled on the
// even CTA's mbarrier (cta_group::2; no multicast).
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster,
                                                 int32_t c, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(iris::smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct TileCoord {
  int x0, y0, n0;
};

// Work unit u -> this CTA's 128-pixel box (x0, y0) and first output channel.
// A CTA pair's unit covers bw x 2bh pixels, the odd CTA the lower half.
__device__ __forceinline__ TileCoord conv_tile(const IrisConvParams& p, int u, int tiles_x, int ntiles, int rows,
                                               int rank) {
  const int mt = u / ntiles, nt = u - mt * ntiles;
  const int ty = mt / tiles_x, tx = mt - ty * tiles_x;
  return TileCoord{tx * p.bw, ty * rows * p.bh + rank * p.bh, nt * p.bn};
}

// Pixel offsets (or -1 outside the image) of the 8 tile rows it * 4 + (lane >> 3)
// of a 32-row quarter starting at tile row row_base, the rows this lane
// stores in conv_store_block.
__device__ __forceinline__ void conv_rows(const IrisConvParams& p, const TileCoord& tc, int row_base, int lane,
                                          long* pix) {
  const int rr = lane >> 3;
#pragma unroll
  for (int it = 0; it < 8; it++) {
    const int r = row_base + it * 4 + rr;
    const int px = tc.x0 + (r & (p.bw - 1)), py = tc.y0 + (r >> p.bw_log2);
    pix[it] = (px < p.W && py < p.H) ? (long)py * p.W + px : -1;
  }
}

// NHWC store of a 32-pixel x 32-channel block: lane i holds pixel row i of
// the tile quarter in v.  Transposed through the warp's staging tile so that
// each store instruction covers 4 pixels x 32 channels (8 lanes per pixel).
// gs / gq return this lane's sum and sum of squares of its stored values.
__device__ __forceinline__ void conv_store_block(const IrisConvParams& p, float* stage, const float* v, int lane,
                                                 const long* pix, int c, float& gs, float& gq) {
  float4* st = reinterpret_cast<float4*>(stage + lane * C_EPI_LD);
#pragma unroll
  for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int rr = lane >> 3, c4 = (lane & 7) * 4;
  const int cc = c + c4;
  const bool cok = cc < p.cout;
  const float4 bb = cok ? __ldg(reinterpret_cast<const float4*>(p.bias + cc)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 h[8];
#pragma unroll
  for (int it = 0; it < 8; it++) {
    h[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.resid && cok && pix[it] >= 0)
      h[it] = __ldcg(reinterpret_cast<const float4*>(p.resid + pix[it] * p.cout + cc));
  }
  gs = 0.f;
  gq = 0.f;
#pragma unroll
  for (int it = 0; it < 8; it++) {
    if (!cok || pix[it] < 0) continue;
    const float4 a = *reinterpret_cast<const float4*>(stage + (it * 4 + rr) * C_EPI_LD + c4);
    float4 o = make_float4(a.x + bb.x + h[it].x, a.y + bb.y + h[it].y, a.z + bb.z + h[it].z, a.w + bb.w + h[it].w);
    gs += (o.x + o.y) + (o.z + o.w);
    gq += (o.x * o.x + o.y * o.y) + (o.z * o.z + o.w * o.w);
    if (p.mode == IRIS_CONV_F32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + pix[it] * p.cout + cc) = o;
    } else {  // IRIS_CONV_BF16
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + pix[it] * p.cout + cc) =
          make_uint2(pack2(o.x, o.y), pack2(o.z, o.w));
    }
  }
  __syncwarp();  // the stage is rewritten by the next block
}

// Persistent convolution kernel.  192 threads: warp 0 TMA producer, warp 1
// TMEM owner + MMA issuer, warps 2-5 epilogue; two TMEM accumulators so the
// epilogue of one unit overlaps the main loop of the next.  kPair: clusters
// of 2 CTAs share one M = 256 MMA (cta_group::2) issued by the even CTA; each
// CTA loads its own 128-pixel A box and half of the weight tile, so a CTA
// reads half as much weight data per MMA as a single-CTA tile of the same N.
template <bool kPair>
__global__ void __launch_bounds__(CNUM_THREADS, 1) conv_kernel(const __grid_constant__ IrisConvParams p) {
  using Cfg = ConvCfg<kPair>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  ConvBars* bars = reinterpret_cast<ConvBars*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? iris::cluster_ctarank() : 0;
  const int unit0 = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int nunits = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int rows = kPair ? 2 : 1;  // 128-pixel boxes stacked per unit

  const int tiles_x = (p.W + p.bw - 1) / p.bw, tiles_y = (p.H + rows * p.bh - 1) / (rows * p.bh);
  const int ntiles = p.cout_pad / p.bn;
  const int total = tiles_x * tiles_y * ntiles;
  const int cb0 = p.cin0 / CBK;
  const int nkb0 = p.taps0 * cb0;
  const int nkb = nkb0 + p.cin1 / CBK;
  const int bload = kPair ? p.bn / 2 : p.bn;           // weight rows this CTA loads per stage
  const int brows = bload < 128 ? bload : 128;          // rows per weight box
  const uint32_t stage_tx = (uint32_t)(CA_BYTES + bload * CBK * 2);
  // Each CTA (pair) starts its K loop at a different K block: every CTA of a
  // launch with one output-channel tile reads the same weights, and in
  // lockstep they would all hit the same L2 lines at once.  The rotation is a
  // function of the unit slot only, so results are deterministic.
  const int krot = (int)(((long)unit0 * nkb) / nunits);
  const uint32_t idesc = iris::umma_idesc_bf16_f32(kPair ? 256 : CBM, p.bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; s++) {
      iris::mbar_init(&bars->full[s], kPair ? 2 : 1);
      iris::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      iris::mbar_init(&bars->tfull[b], 1);
      iris::mbar_init(&bars->tempty[b], kPair ? 2 * C_EPI_WARPS : 32 * C_EPI_WARPS);
    }
    iris::mbar_init(&bars->drain, 1);
    bars->abort = 0;
    iris::fence_mbar_init();
    iris::tma_prefetch_desc(&p.tmap_a[0]);
    if (p.cin1) iris::tma_prefetch_desc(&p.tmap_a[1]);
    iris::tma_prefetch_desc(kPair ? &p.tmap_b_half : &p.tmap_b);
  }
  if (warp == 1) {
    if (kPair) iris::tmem_alloc_pair(&bars->tmem_base, CTMEM_COLS);
    else iris::tmem_alloc(&bars->tmem_base, CTMEM_COLS);
  }
  iris::tc_fence_before();
  __syncthreads();
  if (kPair) iris::cluster_sync();  // both CTAs' barriers exist before any remote arrive
  iris::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    long issued = 0;
    bool ok = true;
    const CUtensorMap* tmb = kPair ? &p.tmap_b_half : &p.tmap_b;
    for (int u = unit0; u < total && ok; u += nunits) {
      const TileCoord tc = conv_tile(p, u, tiles_x, ntiles, rows, (int)rank);
      const int b0 = tc.n0 + (int)rank * bload;
      for (int j = 0; j < nkb; j++) {
        const int kb = j + krot < nkb ? j + krot : j + krot - nkb;
        if (!iris::mbar_wait(&bars->empty[stage], phase ^ 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_PRODUCER)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
        uint8_t* sb = sa + CA_BYTES;
        int ca, xa, ya;
        const CUtensorMap* tma;
        if (kb < nkb0) {
          const int tap = kb / cb0, cblk = kb - tap * cb0;
          const int dx = p.taps0 == 9 ? tap % 3 - 1 : 0, dy = p.taps0 == 9 ? tap / 3 - 1 : 0;
          tma = &p.tmap_a[0];
          ca = cblk * CBK;
          xa = tc.x0 + dx;
          ya = tc.y0 + dy;
        } else {
          tma = &p.tmap_a[1];
          ca = (kb - nkb0) * CBK;
          xa = tc.x0;
          ya = tc.y0;
        }
        if (kPair) {
          const uint32_t full_c = iris::mapa_shared(&bars->full[stage], 0);
          iris::mbar_arrive_expect_tx_cluster(full_c, stage_tx);
          tma_load_3d_pair(sa, tma, full_c, ca, xa, ya);
          for (int r = 0; r < bload; r += brows)
            iris::tma_load_2d_pair(sb + r * (CBK * 2), tmb, full_c, kb * CBK, b0 + r);
        } else {
          iris::mbar_arrive_expect_tx(&bars->full[stage], stage_tx);
          tma_load_3d(sa, tma, &bars->full[stage], ca, xa, ya);
          for (int r = 0; r < bload; r += brows)
            iris::tma_load_2d(sb + r * (CBK * 2), tmb, &bars->full[stage], kb * CBK, b0 + r);
        }
        issued++;
        if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok && issued) {
      if (kPair) {
        // the stage barriers live in the even CTA: give copies still in
        // flight (microseconds) time to land before this CTA can exit
        const uint64_t t0 = iris::globaltimer();
        while (iris::globaltimer() - t0 < 50000ull) {
        }
      } else {
        // bounded drain of the copies still in flight before the CTA exits
        long n = issued < Cfg::STAGES ? issued : Cfg::STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (long i = 0; i < n; i++) {
          if (--s < 0) { s = Cfg::STAGES - 1; ph ^= 1; }
          volatile int no_abort = 0;
          iris::mbar_wait(&bars->full[s], ph, &no_abort, p.status, IRIS_DEV_ERR_CONV_DRAIN);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------ MMA issuer (the even CTA of a pair)
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int u = unit0; u < total && ok; u += nunits, it++) {
      const int buf = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tempty[buf], (use & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_MMA)) {
        ok = false;
        break;
      }
      iris::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * 256;
      for (int kb = 0; kb < nkb; kb++) {  // (stage order; the K block itself is rotated by the producer)
        if (!iris::mbar_wait(&bars->full[stage], phase, abort_flag, p.status, IRIS_DEV_ERR_CONV_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        const uint32_t sa = iris::smem_u32(smem + stage * Cfg::STAGE_BYTES);
        const uint64_t adesc = iris::umma_desc_k_sw128(sa);
        const uint64_t bdesc = iris::umma_desc_k_sw128(sa + CA_BYTES);
#pragma unroll
        for (int kk = 0; kk < CBK / 16; kk++) {
          if (kPair) iris::umma_bf16_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          else iris::umma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
        }
        if (kPair) iris::umma_commit_pair(&bars->empty[stage]);
        else iris::umma_commit(&bars->empty[stage]);
        if (++stage == Cfg::STAGES) { stage = 0; phase ^= 1; }
      }
      if (ok) {
        if (kPair) iris::umma_commit_pair(&bars->tfull[buf]);
        else iris::umma_commit(&bars->tfull[buf]);
      }
    }
    if (!ok) {
      if (kPair) iris::umma_commit_pair(&bars->drain);
      else iris::umma_commit(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_CONV_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue (every CTA, its own 128 pixels)
    // 8 warps: warp w reads TMEM lane quarter w % 4 and every other
    // 32-column block of the tile, starting at block (w - 2) / 4
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int half = ew >> 2;
    float* stage = reinterpret_cast<float*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 + ew * C_EPI_WARP_BYTES);
    // GroupNorm statistics of this warp's outputs, accumulated over its tiles
    // in tile order (one writer lane per group: deterministic)
    double* gacc0 = reinterpret_cast<double*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 +
                                              C_EPI_WARPS * C_EPI_WARP_BYTES);
    double* gacc = gacc0 + ew * 64;
    gacc[2 * lane] = 0.0;
    gacc[2 * lane + 1] = 0.0;
    __syncwarp();
    const int lpg = p.gn_cg / 4;  // lanes (4 channels each) per group inside a 32-channel block
    const int nblk = p.bn >= 32 ? p.bn / 32 : 1;
    const uint32_t tempty_c0 = kPair ? iris::mapa_shared(&bars->tempty[0], 0) : 0;
    const uint32_t tempty_c1 = kPair ? iris::mapa_shared(&bars->tempty[1], 0) : 0;
    int it = 0;
    for (int u = unit0; u < total; u += nunits, it++) {
      const int buf = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tfull[buf], use & 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_EPILOGUE)) break;
      iris::tc_fence_after();
      const TileCoord tc = conv_tile(p, u, tiles_x, ntiles, rows, (int)rank);
      const uint32_t taddr = tmem_base + buf * 256 + ((uint32_t)(quarter * 32) << 16);
      if (p.mode == IRIS_CONV_F32_NCHW) {
        // few output channels (the RGB projection): one pixel per lane,
        // channel planes, consecutive lanes -> consecutive pixels
        if (half == 0) {
          float v[32];
          iris::tmem_ld32(taddr, v);
          const int r = quarter * 32 + lane;
          const int px = tc.x0 + (r & (p.bw - 1)), py = tc.y0 + (r >> p.bw_log2);
          if (px < p.W && py < p.H) {
            const long hw = (long)p.H * p.W, pix = (long)py * p.W + px;
#pragma unroll
            for (int c = 0; c < 32; c++)
              if (c < p.cout) reinterpret_cast<float*>(p.out)[c * hw + pix] = v[c] + __ldg(p.bias + c);
          }
        }
      } else {
        long pix[8];
        conv_rows(p, tc, quarter * 32, lane, pix);
        for (int b = half; b < nblk; b += 2) {
          const int c = 32 * b;
          float v[32];
          iris::tmem_ld32(taddr + c, v);
          float gs, gq;
          conv_store_block(p, stage, v, lane, pix, tc.n0 + c, gs, gq);
          if (p.gn_part && tc.n0 + c < p.cout) {
            // lanes l, l ^ 8, l ^ 16, l ^ 24 hold the same 4 channels of other pixels
            gs += __shfl_xor_sync(0xffffffffu, gs, 8);
            gq += __shfl_xor_sync(0xffffffffu, gq, 8);
            gs += __shfl_xor_sync(0xffffffffu, gs, 16);
            gq += __shfl_xor_sync(0xffffffffu, gq, 16);
            for (int m = 1; m < lpg; m <<= 1) {
              gs += __shfl_xor_sync(0xffffffffu, gs, m);
              gq += __shfl_xor_sync(0xffffffffu, gq, m);
            }
            if (lane < 8 && lane % lpg == 0) {
              const int g = (tc.n0 + c + 4 * lane) / p.gn_cg;
              gacc[2 * g] += (double)gs;
              gacc[2 * g + 1] += (double)gq;
            }
          }
        }
      }
      iris::tc_fence_before();
      if (kPair) {
        __syncwarp();
        if (lane == 0) iris::mbar_arrive_cluster(buf ? tempty_c1 : tempty_c0);
      } else {
        iris::mbar_arrive(&bars->tempty[buf]);
      }
    }
    if (p.gn_part) {  // one partial slot per CTA: the epilogue warps' sums in warp order
      asm volatile("bar.sync 1, %0;" ::"r"(32 * C_EPI_WARPS) : "memory");
      if (ew == 0) {
        double a = 0.0, b = 0.0;
        for (int w = 0; w < C_EPI_WARPS; w++) {
          a += gacc0[w * 64 + 2 * lane];
          b += gacc0[w * 64 + 2 * lane + 1];
        }
        double* dst = p.gn_part + (long)blockIdx.x * 64;
        dst[2 * lane] = a;
        dst[2 * lane + 1] = b;
      }
    }
  }

  __syncthreads();
  if (kPair) iris::cluster_sync();  // no CTA leaves while the pair MMA may still read its shared memory
  if (warp == 1) {
    iris::tc_fence_after();
    if (kPair) iris::tmem_dealloc_pair(tmem_base, CTMEM_COLS);
    else iris::tmem_dealloc(tmem_base, CTMEM_COLS);
  }
}

// ---------------------------------------------------------------- GroupNorm
// Partial statistics of 32 channel groups over an NHWC f32 tensor [P, C] (for
// inputs that no convolution epilogue summed): per-thread float64 sums of a
// fixed float4 column, a fixed-order block reduction, one 64-double slot per
// block in the convolution's gn_part layout (gn_finalize_kernel reduces them).
constexpr int GN_THREADS = 256;

__global__ void __launch_bounds__(GN_THREADS) gn_stats_kernel(const float* __restrict__ x, long P, int C,
                                                              double* part) {
  __shared__ double sh_s[GN_THREADS], sh_q[GN_THREADS];
  const int nq = C / 4, ppi = GN_THREADS / nq;
  const int q = threadIdx.x % nq, pl = threadIdx.x / nq;
  double s = 0.0, ss = 0.0;
  for (long pix = (long)blockIdx.x * ppi + pl; pix < P; pix += (long)gridDim.x * ppi) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(x + pix * C) + q);
    s += (double)((v.x + v.y) + (v.z + v.w));
    ss += (double)((v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w));
  }
  sh_s[threadIdx.x] = s;
  sh_q[threadIdx.x] = ss;
  __syncthreads();
  const int qpg = C / 32 / 4;  // float4 columns per group
  if (threadIdx.x < 32) {
    const int g = threadIdx.x;
    double a = 0.0, b = 0.0;
    for (int r = 0; r < ppi; r++)
      for (int k = 0; k < qpg; k++) {
        a += sh_s[r * nq + g * qpg + k];
        b += sh_q[r * nq + g * qpg + k];
      }
    part[(long)blockIdx.x * 64 + 2 * g] = a;
    part[(long)blockIdx.x * 64 + 2 * g + 1] = b;
  }
}

// NHWC f32 [P, C] -> bf16, optionally 2x nearest-neighbour upsampled (the
// output then has 2H x 2W pixels; W = input width).  8 channels per thread.
__global__ void nhwc_to_bf16_kernel(const float* __restrict__ x, long P, int C, int W, int up2,
                                    __nv_bfloat16* __restrict__ out) {
  const int n8 = C / 8;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * n8) return;
  const long pix = i / n8;
  const int c = (int)(i - pix * n8) * 8;
  const float4* src = reinterpret_cast<const float4*>(x + pix * C + c);
  const float4 a = __ldg(src), b = __ldg(src + 1);
  const uint4 o = make_uint4(pack2(a.x, a.y), pack2(a.z, a.w), pack2(b.x, b.y), pack2(b.z, b.w));
  if (!up2) {
    *reinterpret_cast<uint4*>(out + pix * C + c) = o;
  } else {
    const long py = pix / W, px = pix - py * W, W2 = 2L * W;
#pragma unroll
    for (int a2 = 0; a2 < 2; a2++)
#pragma unroll
      for (int b2 = 0; b2 < 2; b2++)
        *reinterpret_cast<uint4*>(out + ((2 * py + a2) * W2 + 2 * px + b2) * C + c) = o;
  }
}

// GroupNorm from the convolution's partial sums: warp g reduces group g's
// nparts partials in a fixed order (float64), then writes the per-channel
// affine form of the normalisation, y = x * ab[c] + ab[C + c] with
// ab[c] = gamma[c] / sqrt(var + eps), ab[C + c] = beta[c] - mean * ab[c].
__global__ void __launch_bounds__(1024) gn_finalize_kernel(const double* __restrict__ part, int nparts, int C,
                                                           const float* __restrict__ gamma,
                                                           const float* __restrict__ beta, float eps, long count,
                                                           float* __restrict__ ab) {
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double a = 0.0, b = 0.0;
#pragma unroll 4
  for (int i = lane; i < nparts; i += 32) {
    const double2 v = __ldcg(reinterpret_cast<const double2*>(part + (long)i * 64 + 2 * g));
    a += v.x;
    b += v.y;
  }
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const double mean = a / (double)count;
  double var = b / (double)count - mean * mean;
  if (var < 0.0) var = 0.0;
  const float rstd = 1.0f / sqrtf((float)var + eps);
  const int cg = C / 32;
  for (int c = g * cg + lane; c < (g + 1) * cg; c += 32) {
    const float sc = rstd * gamma[c];
    ab[c] = sc;
    ab[C + c] = beta[c] - (float)mean * sc;
  }
}

// NHWC f32 [P, C] -> bf16 x * ab[c] + ab[C + c] (SiLU optional); raw (optional)
// receives the un-normalised bf16 copy (a resnet shortcut's input).  8 channels
// per thread.
__global__ void gn_affine_kernel(const float* __restrict__ x, long P, int C, const float* __restrict__ ab, int silu,
                                 __nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ raw) {
  const int n8 = C / 8;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * n8) return;
  const long pix = i / n8;
  const int c = (int)(i - pix * n8) * 8;
  const float4* src = reinterpret_cast<const float4*>(x + pix * C + c);
  const float4 a = __ldg(src), b = __ldg(src + 1);
  const float4 s0 = __ldg(reinterpret_cast<const float4*>(ab + c)), s1 = __ldg(reinterpret_cast<const float4*>(ab + c + 4));
  const float4 t0 = __ldg(reinterpret_cast<const float4*>(ab + C + c)),
               t1 = __ldg(reinterpret_cast<const float4*>(ab + C + c + 4));
  const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  const float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; e++) {
    v[e] = fmaf(xv[e], sv[e], tv[e]);
    if (silu) v[e] = __fdividef(v[e], 1.0f + __expf(-v[e]));
  }
  *reinterpret_cast<uint4*>(out + pix * C + c) =
      make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
  if (raw)
    *reinterpret_cast<uint4*>(raw + pix * C + c) =
        make_uint4(pack2(xv[0], xv[1]), pack2(xv[2], xv[3]), pack2(xv[4], xv[5]), pack2(xv[6], xv[7]));
}

// Latent [4z, h, w] (NCHW, after the transformer's 2x2 patchify) -> denormalised,
// unpatchified [2h, 2w, z] pixels, optional post-quant 1x1 conv in f32,
// stored as bf16 pixel rows of 64 channels (channels >= z zero).
__global__ void vae_latent_prep_kernel(const float* __restrict__ lat, int z, int h, int w,
                                       const float* bn_mean, const float* bn_std, float scaling, float shift,
                                       const float* pq_w, const float* pq_b, __nv_bfloat16* __restrict__ out) {
  const int W2 = 2 * w;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= 4 * h * w) return;
  const int oh = idx / W2, ow = idx - oh * W2;
  const int ph = oh >> 1, pi = oh & 1, pw = ow >> 1, pj = ow & 1;
  float v[32];
  for (int c = 0; c < z; c++) {
    const int ic = c * 4 + pi * 2 + pj;
    float t = lat[(long)ic * h * w + ph * w + pw];
    t = bn_std ? t * bn_std[ic] + bn_mean[ic] : t / scaling + shift;
    v[c] = t;
  }
  float y[32];
  for (int c = 0; c < z; c++) {
    if (pq_w) {
      float acc = 0.f;
      for (int k = 0; k < z; k++) acc += pq_w[c * z + k] * v[k];
      y[c] = acc + pq_b[c];
    } else {
      y[c] = v[c];
    }
  }
  __nv_bfloat16* o = out + (long)idx * 64;
  for (int c = 0; c < 64; c += 2)
    *reinterpret_cast<uint32_t*>(o + c) = pack2(c < z ? y[c] : 0.f, c + 1 < z ? y[c + 1] : 0.f);
}

// Row softmax of f32 scores [rows, ld] over the first n columns, scaled;
// bf16 probabilities out [rows, ld] with columns n .. ld-1 zero.
__global__ void __launch_bounds__(256) vae_softmax_kernel(const float* __restrict__ s, int ld, int n, float scale,
                                                          __nv_bfloat16* __restrict__ out) {
  __shared__ float red[8];
  const float* row = s + (long)blockIdx.x * ld;
  __nv_bfloat16* orow = out + (long)blockIdx.x * ld;
  const int t = threadIdx.x, lane = t & 31, wp = t >> 5;
  float m = -INFINITY;
  for (int j = t; j < n; j += 256) m = fmaxf(m, row[j]);
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[wp] = m;
  __syncthreads();
  m = red[0];
  for (int k = 1; k < 8; k++) m = fmaxf(m, red[k]);
  __syncthreads();
  float sum = 0.f;
  for (int j = t; j < n; j += 256) sum += __expf((row[j] - m) * scale);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[wp] = sum;
  __syncthreads();
  sum = 0.f;
  for (int k = 0; k < 8; k++) sum += red[k];
  const float inv = 1.0f / sum;
  for (int j = t; j < ld; j += 256)
    orow[j] = __float2bfloat16_rn(j < n ? __expf((row[j] - m) * scale) * inv : 0.f);
}

// RGB planes f32 [3, P] in [-1, 1] -> interleaved uint8 [P, 3] with the
// reference's rounding: (v + 1) * 0.5 * 255, clamped to [0, 255], + 0.5, truncated.
__global__ void vae_rgb8_kernel(const float* __restrict__ x, long P, uint8_t* __restrict__ out) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 3 * P) return;
  const long pix = i / 3;
  const int c = (int)(i - pix * 3);
  float v = (x[c * P + pix] + 1.0f) * 0.5f;
  v = v * 255.0f;
  v = fminf(fmaxf(v, 0.0f), 255.0f);
  out[i] = (uint8_t)(v + 0.5f);
}

}  // namespace

extern "C" int iris_make_tmap_nhwc_bf16(CUtensorMap* m, const void* ptr, int H, int W, int C, int bw, int bh) {
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f)
      return -1;
    fn = reinterpret_cast<EncodeFn>(f);
  }
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || C % 64 || bw * bh != CBM || bw > 256 || bh > 256 || H < 1 ||
      W < 1)
    return -2;
  cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H};
  cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)bw, (cuuint32_t)bh};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

static bool g_conv_attr = false;
static int g_conv_pairs = 0;  // CTA pairs that can be resident at once

extern "C" cudaError_t iris_conv_init(void) {
  if (g_conv_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(conv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       ConvCfg<false>::SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(conv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ConvCfg<true>::SMEM_BYTES);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(conv_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
  cfg.blockDim = dim3(CNUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = ConvCfg<true>::SMEM_BYTES;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, conv_kernel<true>, &cfg) == cudaSuccess && n > 0) g_conv_pairs = n;
  cudaGetLastError();
  g_conv_attr = true;
  return cudaSuccess;
}

// Units of work and CTAs of a launch: pair launches use 2-CTA clusters over
// units of 2 x 128 pixels, when p->pair is set and pairs can be resident.
static long conv_units(const IrisConvParams* p, int pair) {
  const int rows = pair ? 2 : 1;
  return (long)((p->W + p->bw - 1) / p->bw) * ((p->H + rows * p->bh - 1) / (rows * p->bh)) * (p->cout_pad / p->bn);
}

extern "C" int iris_conv_grid(const IrisConvParams* p, int num_sms) {
  if (p->pair && g_conv_pairs > 0) {
    const long units = conv_units(p, 1);
    long cap = g_conv_pairs < num_sms / 2 ? g_conv_pairs : num_sms / 2;
    return (int)(2 * (units < cap ? units : cap));
  }
  const long tiles = conv_units(p, 0);
  return (int)(tiles < num_sms ? tiles : num_sms);
}

extern "C" int iris_conv_pairs_available(void) { return g_conv_pairs; }

extern "C" cudaError_t iris_launch_conv(const IrisConvParams* p, int num_sms, cudaStream_t stream) {
  if (!g_conv_attr) {
    cudaError_t e = iris_conv_init();
    if (e != cudaSuccess) return e;
  }
  const int bn = p->bn;
  if (!(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256) || p->cout_pad % bn || p->cout > p->cout_pad ||
      p->cin0 % CBK || p->cin0 <= 0 || p->cin1 % CBK || (p->taps0 != 9 && p->taps0 != 1) ||
      p->bw * p->bh != CBM || (p->bw & (p->bw - 1)) || (1 << p->bw_log2) != p->bw || p->H < 1 || p->W < 1)
    return cudaErrorInvalidValue;
  if (p->mode == IRIS_CONV_F32_NCHW ? p->cout > 32 : p->cout % 4 != 0) return cudaErrorInvalidValue;
  if (p->gn_part && (p->mode == IRIS_CONV_F32_NCHW || p->cout % 32 || p->cout / p->gn_cg != 32 ||
                     (p->gn_cg != 4 && p->gn_cg != 8 && p->gn_cg != 16)))
    return cudaErrorInvalidValue;
  const int grid = iris_conv_grid(p, num_sms);
  if (p->pair && g_conv_pairs > 0) {
    if (bn != 128 && bn != 256) return cudaErrorInvalidValue;  // M = 256 MMA: N in {128, 256} here
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(CNUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = ConvCfg<true>::SMEM_BYTES;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv_kernel<true>, *p);
  }
  conv_kernel<false><<<grid, CNUM_THREADS, ConvCfg<false>::SMEM_BYTES, stream>>>(*p);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_gn_stats(const float* x, long P, int C, double* part, int nblocks,
                                            cudaStream_t stream) {
  if (C % 128 || C > 1024 || nblocks < 1) return cudaErrorInvalidValue;
  gn_stats_kernel<<<nblocks, GN_THREADS, 0, stream>>>(x, P, C, part);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_nhwc_to_bf16(const float* x, long P, int C, int W, int up2, void* out,
                                                cudaStream_t stream) {
  if (C % 8) return cudaErrorInvalidValue;
  const long n = P * (C / 8);
  if (n == 0) return cudaSuccess;
  nhwc_to_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, P, C, W, up2,
                                                                      reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_vae_latent_prep(const float* lat, int z, int h, int w, const float* bn_mean,
                                                   const float* bn_std, float scaling, float shift,
                                                   const float* pq_w, const float* pq_b, void* out,
                                                   cudaStream_t stream) {
  if (z < 1 || z > 32 || (!bn_std && scaling == 0.0f)) return cudaErrorInvalidValue;
  const int n = 4 * h * w;
  vae_latent_prep_kernel<<<(n + 127) / 128, 128, 0, stream>>>(lat, z, h, w, bn_mean, bn_std, scaling, shift, pq_w,
                                                              pq_b, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_vae_softmax(const float* s, int rows, int ld, int n, float scale, void* out,
                                               cudaStream_t stream) {
  if (rows < 1 || n < 1 || n > ld) return cudaErrorInvalidValue;
  vae_softmax_kernel<<<rows, 256, 0, stream>>>(s, ld, n, scale, reinterpret_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_vae_rgb8(const float* x, long P, uint8_t* out, cudaStream_t stream) {
  const long n = 3 * P;
  vae_rgb8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, P, out);
  return cudaGetLastError();
}


extern "C" cudaError_t iris_launch_gn_finalize(const double* part, int nparts, int C, const float* gamma,
                                               const float* beta, float eps, long count, float* ab,
                                               cudaStream_t stream) {
  if (C % 32 || C / 32 > 32 || nparts < 1) return cudaErrorInvalidValue;
  gn_finalize_kernel<<<1, 1024, 0, stream>>>(part, nparts, C, gamma, beta, eps, count, ab);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_gn_affine(const float* x, long P, int C, const float* ab, int silu, void* out,
                                             void* raw, cudaStream_t stream) {
  if (C % 8) return cudaErrorInvalidValue;
  const long n = P * (C / 8);
  if (n == 0) return cudaSuccess;
  gn_affine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, P, C, ab, silu,
                                                                   reinterpret_cast<__nv_bfloat16*>(out),
                                                                   reinterpret_cast<__nv_bfloat16*>(raw));
  return cudaGetLastError();
}

