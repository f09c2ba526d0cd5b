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

constexpr int CBM = 128;                    // output pixels per tile
constexpr int CBK = 64;                     // input channels per K block
constexpr int CSTAGES = 4;
constexpr int CA_BYTES = CBM * CBK * 2;     // 16 KB
constexpr int CB_BYTES_MAX = 256 * CBK * 2; // 32 KB
constexpr int CSTAGE_BYTES = CA_BYTES + CB_BYTES_MAX;
constexpr int CNUM_THREADS = 192;
constexpr int CTMEM_COLS = 512;
constexpr int C_EPI_LD = 36;
constexpr int C_EPI_WARP_BYTES = 32 * C_EPI_LD * 4;
constexpr int C_SMEM_BYTES = CSTAGES * CSTAGE_BYTES + 1024 + 4 * C_EPI_WARP_BYTES + 1024;

struct ConvBars {
  uint64_t full[CSTAGES];
  uint64_t empty[CSTAGES];
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

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct TileCoord {
  int x0, y0, n0;
};

__device__ __forceinline__ TileCoord conv_tile(const IrisConvParams& p, int u, int tiles_x, int ntiles) {
  const int mt = u / ntiles, nt = u - mt * ntiles;
  const int ty = mt / tiles_x, tx = mt - ty * tiles_x;
  return TileCoord{tx * p.bw, ty * p.bh, nt * p.bn};
}

// NHWC store of a 32-pixel x 32-channel block: lane i holds pixel row i of
// the tile quarter in v.  Transposed through the warp's staging tile so that
// each store instruction covers 4 pixels x 32 channels (8 lanes per pixel).
__device__ __forceinline__ void conv_store_block(const IrisConvParams& p, float* stage, const float* v, int lane,
                                                 int row_base, const TileCoord& tc, int c) {
  float4* st = reinterpret_cast<float4*>(stage + lane * C_EPI_LD);
#pragma unroll
  for (int q = 0; q < 8; q++) st[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int rr = lane >> 3, c4 = (lane & 7) * 4;
  const int cc = c + c4;
  const bool cok = cc < p.cout;
  const float4 bb = cok ? __ldg(reinterpret_cast<const float4*>(p.bias + cc)) : make_float4(0.f, 0.f, 0.f, 0.f);
  long pix[8];
  float4 h[8];
#pragma unroll
  for (int it = 0; it < 8; it++) {
    const int r = row_base + it * 4 + rr;  // pixel row inside the 128-pixel tile
    const int px = tc.x0 + r % p.bw, py = tc.y0 + r / p.bw;
    pix[it] = (cok && px < p.W && py < p.H) ? (long)py * p.W + px : -1;
    h[it] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.resid && pix[it] >= 0) h[it] = __ldcg(reinterpret_cast<const float4*>(p.resid + pix[it] * p.cout + cc));
  }
#pragma unroll
  for (int it = 0; it < 8; it++) {
    if (pix[it] < 0) continue;
    const float4 a = *reinterpret_cast<const float4*>(stage + (it * 4 + rr) * C_EPI_LD + c4);
    float4 o = make_float4(a.x + bb.x + h[it].x, a.y + bb.y + h[it].y, a.z + bb.z + h[it].z, a.w + bb.w + h[it].w);
    if (p.mode == IRIS_CONV_F32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + pix[it] * p.cout + cc) = o;
    } else {  // IRIS_CONV_BF16
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + pix[it] * p.cout + cc) =
          make_uint2(pack2(o.x, o.y), pack2(o.z, o.w));
    }
  }
  __syncwarp();  // the stage is rewritten by the next block
}

__global__ void __launch_bounds__(CNUM_THREADS, 1) conv_tc_kernel(const __grid_constant__ IrisConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  ConvBars* bars = reinterpret_cast<ConvBars*>(smem + CSTAGES * CSTAGE_BYTES);
  volatile int* abort_flag = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int tiles_x = (p.W + p.bw - 1) / p.bw, tiles_y = (p.H + p.bh - 1) / p.bh;
  const int ntiles = p.cout_pad / p.bn;
  const int total = tiles_x * tiles_y * ntiles;
  const int cb0 = p.cin0 / CBK;
  const int nkb0 = p.taps0 * cb0;
  const int nkb = nkb0 + p.cin1 / CBK;
  const int brows = p.bn < 128 ? p.bn : 128;
  const uint32_t b_bytes = (uint32_t)p.bn * CBK * 2;
  const uint32_t idesc = iris::umma_idesc_bf16_f32(CBM, p.bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < CSTAGES; s++) {
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
    iris::tma_prefetch_desc(&p.tmap_a[0]);
    if (p.cin1) iris::tma_prefetch_desc(&p.tmap_a[1]);
    iris::tma_prefetch_desc(&p.tmap_b);
  }
  if (warp == 1) iris::tmem_alloc(&bars->tmem_base, CTMEM_COLS);
  iris::tc_fence_before();
  __syncthreads();
  iris::tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------ TMA producer
    int stage = 0;
    uint32_t phase = 0;
    long issued = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
      const TileCoord tc = conv_tile(p, u, tiles_x, ntiles);
      for (int kb = 0; kb < nkb; kb++) {
        if (!iris::mbar_wait(&bars->empty[stage], phase ^ 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_PRODUCER)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * CSTAGE_BYTES;
        uint8_t* sb = sa + CA_BYTES;
        iris::mbar_arrive_expect_tx(&bars->full[stage], CA_BYTES + b_bytes);
        if (kb < nkb0) {
          const int tap = kb / cb0, cblk = kb - tap * cb0;
          const int dx = p.taps0 == 9 ? tap % 3 - 1 : 0, dy = p.taps0 == 9 ? tap / 3 - 1 : 0;
          tma_load_3d(sa, &p.tmap_a[0], &bars->full[stage], cblk * CBK, tc.x0 + dx, tc.y0 + dy);
        } else {
          tma_load_3d(sa, &p.tmap_a[1], &bars->full[stage], (kb - nkb0) * CBK, tc.x0, tc.y0);
        }
        for (int r = 0; r < p.bn; r += brows)
          iris::tma_load_2d(sb + r * (CBK * 2), &p.tmap_b, &bars->full[stage], kb * CBK, tc.n0 + r);
        issued++;
        if (++stage == CSTAGES) { stage = 0; phase ^= 1; }
      }
    }
    if (!ok) {
      // bounded drain of the copies still in flight before the CTA exits
      long n = issued < CSTAGES ? issued : CSTAGES;
      int s = stage;
      uint32_t ph = phase;
      for (long i = 0; i < n; i++) {
        if (--s < 0) { s = CSTAGES - 1; ph ^= 1; }
        volatile int no_abort = 0;
        iris::mbar_wait(&bars->full[s], ph, &no_abort, p.status, IRIS_DEV_ERR_CONV_DRAIN);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x, it++) {
      const int buf = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tempty[buf], (use & 1) ^ 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_MMA)) {
        ok = false;
        break;
      }
      iris::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * 256;
      for (int kb = 0; kb < nkb; kb++) {
        if (!iris::mbar_wait(&bars->full[stage], phase, abort_flag, p.status, IRIS_DEV_ERR_CONV_MMA)) {
          ok = false;
          break;
        }
        iris::tc_fence_after();
        const uint32_t sa = iris::smem_u32(smem + stage * CSTAGE_BYTES);
        const uint64_t adesc = iris::umma_desc_k_sw128(sa);
        const uint64_t bdesc = iris::umma_desc_k_sw128(sa + CA_BYTES);
#pragma unroll
        for (int kk = 0; kk < CBK / 16; kk++)
          iris::umma_bf16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb != 0 || kk != 0));
        iris::umma_commit(&bars->empty[stage]);
        if (++stage == CSTAGES) { stage = 0; phase ^= 1; }
      }
      if (ok) iris::umma_commit(&bars->tfull[buf]);
    }
    if (!ok) {
      iris::umma_commit(&bars->drain);
      volatile int no_abort = 0;
      iris::mbar_wait(&bars->drain, 0, &no_abort, p.status, IRIS_DEV_ERR_CONV_DRAIN);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    float* stage = reinterpret_cast<float*>(smem + CSTAGES * CSTAGE_BYTES + 1024 + (warp - 2) * C_EPI_WARP_BYTES);
    int it = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, it++) {
      const int buf = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      if (!iris::mbar_wait(&bars->tfull[buf], use & 1, abort_flag, p.status, IRIS_DEV_ERR_CONV_EPILOGUE)) break;
      iris::tc_fence_after();
      const TileCoord tc = conv_tile(p, u, tiles_x, ntiles);
      const uint32_t taddr = tmem_base + buf * 256 + ((uint32_t)(quarter * 32) << 16);
      if (p.mode == IRIS_CONV_F32_NCHW) {
        // few output channels (the RGB projection): one pixel per lane,
        // channel planes, consecutive lanes -> consecutive pixels
        float v[32];
        iris::tmem_ld32(taddr, v);
        const int r = quarter * 32 + lane;
        const int px = tc.x0 + r % p.bw, py = tc.y0 + r / p.bw;
        if (px < p.W && py < p.H) {
          const long hw = (long)p.H * p.W, pix = (long)py * p.W + px;
#pragma unroll
          for (int c = 0; c < 32; c++)
            if (c < p.cout) reinterpret_cast<float*>(p.out)[c * hw + pix] = v[c] + __ldg(p.bias + c);
        }
      } else {
        for (int c = 0; c < p.bn; c += 32) {
          float v[32];
          iris::tmem_ld32(taddr + c, v);
          conv_store_block(p, stage, v, lane, quarter * 32, tc, tc.n0 + c);
        }
      }
      iris::tc_fence_before();
      iris::mbar_arrive(&bars->tempty[buf]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    iris::tc_fence_after();
    iris::tmem_dealloc(tmem_base, CTMEM_COLS);
  }
}

// ---------------------------------------------------------------- GroupNorm
// Statistics of 32 channel groups over an NHWC f32 tensor [P, C]: per-thread
// float64 sums of a fixed float4 column, a fixed-order block reduction into
// per-block partials, and the last block to finish sums the partials in block
// order (deterministic) into {mean, 1 / sqrt(var + eps)} per group.
constexpr int GN_THREADS = 256;

__global__ void __launch_bounds__(GN_THREADS) gn_stats_kernel(const float* __restrict__ x, long P, int C,
                                                              double* part, unsigned* counter, float* stats,
                                                              float eps) {
  __shared__ double sh_s[GN_THREADS], sh_q[GN_THREADS];
  __shared__ bool last;
  const int nq = C / 4, ppi = GN_THREADS / nq;
  const int q = threadIdx.x % nq, pl = threadIdx.x / nq;
  double s = 0.0, ss = 0.0;
  if (pl < ppi) {
    for (long pix = (long)blockIdx.x * ppi + pl; pix < P; pix += (long)gridDim.x * ppi) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(x + pix * C) + q);
      s += (double)((v.x + v.y) + (v.z + v.w));
      ss += (double)((v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w));
    }
  }
  sh_s[threadIdx.x] = s;
  sh_q[threadIdx.x] = ss;
  __syncthreads();
  const int cg = C / 32, qpg = cg / 4;  // float4 columns per group
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
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x < 32) {
    const int g = threadIdx.x;
    double a = 0.0, b = 0.0;
    for (unsigned blk = 0; blk < gridDim.x; blk++) {
      a += __ldcg(part + (long)blk * 64 + 2 * g);
      b += __ldcg(part + (long)blk * 64 + 2 * g + 1);
    }
    const double n = (double)P * cg;
    const double mean = a / n;
    double var = b / n - mean * mean;
    if (var < 0.0) var = 0.0;
    stats[2 * g] = (float)mean;
    stats[2 * g + 1] = 1.0f / sqrtf((float)var + eps);
  }
  if (threadIdx.x == 0) *counter = 0;  // ready for the next launch (graph replays)
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }

// NHWC f32 [P, C] -> bf16, optionally GroupNorm-normalised (stats != NULL,
// per-channel gamma/beta), SiLU, and 2x nearest-neighbour upsampled (the
// output then has 2H x 2W pixels).  Each thread converts 8 channels.
__global__ void nhwc_to_bf16_kernel(const float* __restrict__ x, long P, int C, int W, const float* stats,
                                    const float* __restrict__ gamma, const float* __restrict__ beta, int silu,
                                    int up2, __nv_bfloat16* __restrict__ out) {
  const int n8 = C / 8;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * n8) return;
  const long pix = i / n8;
  const int c = (int)(i - pix * n8) * 8;
  const float4* src = reinterpret_cast<const float4*>(x + pix * C + c);
  const float4 a = __ldg(src), b = __ldg(src + 1);
  float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  if (stats) {
    const int cg = C / 32;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int g = (c + e) / cg;
      v[e] = (v[e] - __ldg(stats + 2 * g)) * __ldg(stats + 2 * g + 1) * __ldg(gamma + c + e) + __ldg(beta + c + e);
    }
  }
  if (silu) {
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = silu_f(v[e]);
  }
  const uint4 o = make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
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

extern "C" cudaError_t iris_conv_init(void) {
  if (g_conv_attr) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C_SMEM_BYTES);
  if (e == cudaSuccess) g_conv_attr = true;
  return e;
}

extern "C" cudaError_t iris_launch_conv(const IrisConvParams* p, int num_sms, cudaStream_t stream) {
  if (!g_conv_attr) {
    cudaError_t e = iris_conv_init();
    if (e != cudaSuccess) return e;
  }
  const int bn = p->bn;
  if (!(bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256) || p->cout_pad % bn || p->cout > p->cout_pad ||
      p->cin0 % CBK || p->cin0 <= 0 || p->cin1 % CBK || (p->taps0 != 9 && p->taps0 != 1) ||
      p->bw * p->bh != CBM || p->H < 1 || p->W < 1)
    return cudaErrorInvalidValue;
  if (p->mode == IRIS_CONV_F32_NCHW ? p->cout > 32 : p->cout % 4 != 0) return cudaErrorInvalidValue;
  const long tiles = (long)((p->W + p->bw - 1) / p->bw) * ((p->H + p->bh - 1) / p->bh) * (p->cout_pad / bn);
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  conv_tc_kernel<<<grid, CNUM_THREADS, C_SMEM_BYTES, stream>>>(*p);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_gn_stats(const float* x, long P, int C, double* part, int nblocks,
                                            unsigned* counter, float* stats, float eps, cudaStream_t stream) {
  if (C % 128 || C > 1024 || nblocks < 1) return cudaErrorInvalidValue;
  gn_stats_kernel<<<nblocks, GN_THREADS, 0, stream>>>(x, P, C, part, counter, stats, eps);
  return cudaGetLastError();
}

extern "C" cudaError_t iris_launch_nhwc_to_bf16(const float* x, long P, int C, int W, const float* stats,
                                                const float* gamma, const float* beta, int silu, int up2, void* out,
                                                cudaStream_t stream) {
  if (C % 32) return cudaErrorInvalidValue;
  const long n = P * (C / 8);
  if (n == 0) return cudaSuccess;
  nhwc_to_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      x, P, C, W, stats, gamma, beta, silu, up2, reinterpret_cast<__nv_bfloat16*>(out));
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
