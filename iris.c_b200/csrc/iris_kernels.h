/*
 * Internal C interface between the C host code of the iris CUDA backend and
 * its sm_100a kernels (.cu files).  Plain C: pointers, sizes and CUtensorMap
 * descriptors, no C++ types.  Every launcher enqueues work on `stream` and
 * returns a cudaError_t value (0 = success).
 */
#ifndef IRIS_KERNELS_CUDA_H
#define IRIS_KERNELS_CUDA_H

#include <cuda.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ GEMM
 * C[M, N] = A[M, K] * B[N, K]^T with bf16 operands (both K-major, row-major
 * in memory) and f32 accumulation in TMEM, followed by one of the fused
 * epilogues below.  Rows of A are split into up to two groups (the text and
 * image streams of a double block), each with its own weight matrix B and
 * epilogue vectors; groups share N and K. */
enum {
    IRIS_EPI_BF16 = 0,        /* out bf16 [row, ldo] (+ bias[col])                         */
    IRIS_EPI_F32 = 1,         /* out f32  [row, ldo] (+ bias[col])                         */
    IRIS_EPI_F32_NCHW = 2,    /* out f32 [col, nchw_rows] (channel-major, + bias)          */
    IRIS_EPI_RESID_GATE = 3,  /* f32 out[row, col] += gate[g][col] * acc                   */
    IRIS_EPI_QKV = 4,         /* cols [0,H) Q, [H,2H) K, [2H,3H) V; per-head RMSNorm on Q/K
                                 then pair RoPE evaluated in registers from the row's
                                 position ids (rope_pos, rope_spec); bf16 stores            */
    IRIS_EPI_SWIGLU = 5,      /* 256-col tiles hold [gate 128 | up 128] of 128 features:
                                 mlp_out[row, mlp_col0 + f] = SiLU(gate) * up (bf16)       */
    IRIS_EPI_GATE_BF16 = 7,   /* out bf16 [row, ldo] = gate[g][col] * acc (tensor-parallel
                                 partial of a gated residual update)                      */
    IRIS_EPI_TP_SCATTER = 8,  /* f32 gate[g][col] * acc -> the owning rank's receive slot
                                 tp.recv[row / chunk][tp.rank] over NVLink, then a
                                 partial-arrival signal to every rank                     */
    IRIS_EPI_SINGLE = 6,      /* cols < 3H as IRIS_EPI_QKV, cols >= 3H as IRIS_EPI_SWIGLU   */
    IRIS_EPI_LORA_FOLD = 9,   /* bf16 out[fold_rows[row], col] = bf16(fold_w0[same] +
                                 fold_scale * acc): a low-rank update folded into a weight */
};

/* Tensor-parallel exchange over NVLink peer memory (size > 1).  Rows of the
 * sequence are owned in chunks of `chunk` rows by rank row / chunk.  Each
 * rank's flag block (uint32 words, in symmetric memory):
 *   [0, 8)   partial-update arrivals, by sender rank
 *   [8, 16)  adaLN-output (xmod) arrivals, by sender rank
 *   16, 17   CTA completion counters of the signalling GEMM / adaLN launch
 *   18, 19   sync bases: partial / xmod syncs completed before this call
 *   [20, 28) call-start barrier arrivals by sender, 28 its base (a call's
 *            first writes into peer memory wait until every rank has
 *            finished its previous call)
 * A signalling launch adds 1 to slot [sender] of every rank's block once all
 * its CTAs' stores are out (system-scope release); a waiting launch polls
 * its own block until every sender's slot reaches base + index.        */
#define IRIS_TP_MAX 8
#define IRIS_TP_PART 0
#define IRIS_TP_X 8
#define IRIS_TP_DONE_GEMM 16
#define IRIS_TP_DONE_ADALN 17
#define IRIS_TP_BASE_PART 18
#define IRIS_TP_BASE_X 19
#define IRIS_TP_BAR 20        /* [20, 28): call-start barrier arrivals, by sender */
#define IRIS_TP_BASE_BAR 28
/* Rotary embedding of one model, per rotation pair p (64 pairs of a 128-wide
 * head; pair p rotates columns 2p, 2p + 1): angle = pos[axis(p)] * freq[p], with
 * pos the row's position id on that axis, freq[p] = 1 / theta^(2i / axis_dim)
 * computed on the host exactly as the reference does; axis(p) = bits 2(p % 16)
 * and up of axis_bits[p / 16].  kscale[p] multiplies cos and sin of K on the
 * rows a launch marks (SREF band control; 1 elsewhere). */
typedef struct {
    float freq[64];
    float kscale[64];
    uint32_t axis_bits[4];
    uint32_t axis_mask[4];    /* per 16-pair block: bit a set if a pair of it uses axis a */
} IrisRopeSpec;

static inline void iris_rope_set_axis(IrisRopeSpec *s, int pair, int axis) {
    s->axis_bits[pair / 16] = (s->axis_bits[pair / 16] & ~(3u << (2 * (pair % 16)))) |
                              ((uint32_t)axis << (2 * (pair % 16)));
    s->axis_mask[pair / 16] |= 1u << axis;
}

typedef struct {
    int size, rank;           /* size > 1 enables the peer-memory paths          */
    int chunk;                /* rows owned per rank                              */
    float *recv[IRIS_TP_MAX]; /* rank p's partial receive buffer [size][chunk][N] (peer-mapped) */
    unsigned *flags[IRIS_TP_MAX];  /* rank p's flag block (peer-mapped; [rank] = own) */
    unsigned wait_x;          /* GEMM: xmod sync index to wait for before loading A (0 = none) */
} IrisTpParams;

typedef struct {
    CUtensorMap tmap_a;       /* A: box {64, 128} rows, 128B swizzle                  */
    CUtensorMap tmap_b[2];    /* B per group: box {64, bn} rows, 128B swizzle          */
    int ngroups;
    int row0[2];              /* first row of each group in A and row-indexed outputs  */
    int rows[2];              /* rows per group                                        */
    int N, K;
    int bn;                   /* 128 or 256 */
    int mode;
    void *out;                /* BF16/F32/NCHW/RESID destination                       */
    int ldo;                  /* elements */
    int nchw_rows;            /* IRIS_EPI_F32_NCHW: channel stride                      */
    const float *bias;        /* optional [N]                                          */
    const float *gate[2];     /* RESID: per group [N]                                  */
    int resid_store;          /* RESID: out = gate*acc instead of out += gate*acc      */
    const float *qnorm[2];    /* QKV: per group [128]                                  */
    const float *knorm[2];
    const uint16_t *rope_pos; /* QKV: [rows_total][4] position ids by absolute row
                                 (NULL = no RoPE)                                       */
    const IrisRopeSpec *rope_spec;  /* QKV: frequency / axis / K scale per rotation pair */
    int rope_k_row0;          /* QKV: K of rows >= this (when > 0) takes kscale         */
    void *q, *k, *v;          /* QKV destinations (bf16) with row stride ldqkv         */
    int ldqkv;
    int H;                    /* width of Q, K and V blocks (heads * 128)              */
    float eps;
    void *mlp_out;            /* SWIGLU destination (bf16)                             */
    int ld_mlp;
    int mlp_col0;
    int swiglu_base;          /* first column of the gate/up region in N              */
    int *status;              /* device status word for bounded-wait failures         */
    /* optional split-K workspace (f32) for launches with few output tiles: the
       K range is split over CTAs, partial tiles go to ws [split][row][N] and a
       reduction pass applies the epilogue (BF16, F32 and RESID_GATE modes) */
    float *ws;
    size_t ws_bytes;
    int splitk;               /* set by iris_launch_gemm                              */
    int a_box;                /* rows of tmap_a's box when under 128 (a multiple of 8, at
                                 least every group's row count): smaller A stages, so
                                 more of them in flight; 0 = 128                       */
    int nstages;              /* set by iris_launch_gemm                              */
    /* optional, RESID_GATE launches that split over K (iris_gemm_splits > 1):
       the reduction also applies the next adaLN to each finished row,
       ln_out[r] = bf16((1 + ln_scale[g]) * LayerNorm(out[r]) + ln_shift[g]),
       g = (r >= ln_split) -- what iris_launch_adaln would do next           */
    void *ln_out;
    int ln_ld;
    int ln_split;
    const float *ln_shift[2], *ln_scale[2];
    float ln_eps;
    int b_static;             /* B is a resident weight that no kernel of the stream
                                 writes: its first stages may load before the
                                 previous kernel has finished                         */
    IrisTpParams tp;          /* IRIS_EPI_TP_SCATTER destination and xmod wait        */
    const int *fold_rows;     /* IRIS_EPI_LORA_FOLD: output row of each A row          */
    const void *fold_w0;      /* IRIS_EPI_LORA_FOLD: base weight (bf16, row stride ldo) */
    float fold_scale;
} IrisGemmParams;

/* Encodes a 2-D bf16 tensor map over a row-major [rows, cols] matrix with
 * row stride ld (elements) and box {64, box_rows}, 128-byte swizzle. */
int iris_make_tmap_bf16(CUtensorMap *m, const void *ptr, uint64_t rows, uint64_t cols,
                        uint64_t ld, uint32_t box_rows);

cudaError_t iris_launch_gemm(const IrisGemmParams *p, int num_sms, cudaStream_t stream);
/* The number of K splits iris_launch_gemm would use for p (1: none). */
int iris_gemm_splits(const IrisGemmParams *p, int num_sms);
/* as iris_launch_gemm; *launches = kernels queued (2 when a split-K
 * reduction pass follows the GEMM) */
cudaError_t iris_launch_gemm_ex(const IrisGemmParams *p, int num_sms, cudaStream_t stream, int *launches);

/* one-time kernel attribute setup (dynamic shared memory limits); called at
 * library init so that nothing but launches happens during graph capture */
cudaError_t iris_gemm_init(void);

/* ------------------------------------------------------------------ attention
 * O = softmax(Q K^T * scale) V for every head, bf16 in/out, f32 softmax.
 * Q [sq, ldq], K/V [sk, ldk] with head h at columns h*128 .. h*128+127.
 * key_mask (optional, [sk], 1 = valid) sets masked scores to -1e9 exactly as
 * the Z-Image reference does. */
cudaError_t iris_launch_attention(const void *q, int ldq, const void *k, const void *v, int ldk,
                                  void *o, int ldo, int sq, int sk, int heads, float scale,
                                  const uint8_t *key_mask, cudaStream_t stream);
/* the tcgen05/TMEM implementation behind it */
cudaError_t iris_launch_attention_tc(const void *q, int ldq, const void *k, const void *v, int ldk,
                                     void *o, int ldo, int sq, int sk, int heads, float scale,
                                     const uint8_t *key_mask, cudaStream_t stream);
cudaError_t iris_attention_tc_init(void);
/* tcgen05 attention with grouped-query heads (query head h reads key/value
 * head h / kv_group; K and V hold heads / kv_group heads) and an optional
 * causal mask (key j > query i scores -1e9, as the reference's encoder
 * attention does) */
cudaError_t iris_launch_attention_gqa(const void *q, int ldq, const void *k, const void *v, int ldk, void *o,
                                      int ldo, int sq, int sk, int heads, int kv_group, int causal, float scale,
                                      const uint8_t *key_mask, cudaStream_t stream);
void iris_attention_set_status(int *status);

/* ------------------------------------------------------------------ row kernels */
/* out_bf16[r] = (1 + scale_g) * LayerNorm(x[r]) + shift_g, g = (r >= split) */
/* as iris_launch_adaln, first adding a pending bf16 residual update to x
 * (x += delta, written back) when delta is not NULL */
cudaError_t iris_launch_adaln_delta(float *x, int ldx, const void *delta, int ld_delta, void *out, int ldout,
                                    int rows, int cols, const float *shift0, const float *scale0,
                                    const float *shift1, const float *scale1, int split, float eps,
                                    cudaStream_t stream);
/* Tensor-parallel adaLN over this rank's rows (one warp per row).
 * Rows [row0, row0 + rows) of x belong to this rank; rows below row_lo are
 * skipped.  If has_part, first waits for the partial updates of partial sync
 * `part_index` from every rank and adds them (rank order) from recv
 * [size][chunk][H] into x.  If xmod[0] is not NULL, then applies adaLN (shift/
 * scale per row group, split = first row of group 1) and stores the bf16 row
 * into xmod[p] of every rank p (peer memory), then signals xmod arrival. */
typedef struct {
    float *x;
    int row0, rows, row_lo, chunk, H;
    const float *recv;
    int has_part;
    unsigned part_index;
    void *xmod[IRIS_TP_MAX];
    const float *shift0, *scale0, *shift1, *scale1;
    int split;
    float eps;
    IrisTpParams tp;
    int *status;
} IrisAdalnTpArgs;
cudaError_t iris_launch_adaln_tp(const IrisAdalnTpArgs *a, cudaStream_t stream);
/* call-start barrier over all ranks (one thread; bounded wait) */
cudaError_t iris_launch_tp_barrier(const IrisTpParams *tp, int *status, cudaStream_t stream);
/* advance this rank's sync bases by the syncs one call queued */
cudaError_t iris_launch_tp_advance(unsigned *flags, unsigned parts, unsigned xs, cudaStream_t stream);
/* x[row, col] += delta[row, col] (f32 += bf16) */
cudaError_t iris_launch_add_bf16_rows(float *x, int ldx, const void *delta, int ld_delta, int rows, int cols,
                                      cudaStream_t stream);
cudaError_t iris_launch_adaln(const float *x, int ldx, void *out, int ldout, int rows, int cols,
                              const float *shift0, const float *scale0, const float *shift1,
                              const float *scale1, int split, float eps, cudaStream_t stream);
/* y[n] = act_out(sum_k W[n,k] * act_in(x[k]) + b[n]); W bf16 [N, K]; act 0 none, 1 SiLU */
cudaError_t iris_launch_gemv(const void *w, const float *x, const float *bias, float *y, int n,
                             int k, int act_in, int act_out, cudaStream_t stream);
/* out[i] = [cos(t*1000*f_i), sin(...)] with f_i = exp(-ln(1e4) i/half), t read from *t_dev */
cudaError_t iris_launch_timestep_sincos(const float *t_dev, float t_scale, float *out, int dim,
                                        cudaStream_t stream);
/* NCHW f32 [C, n] -> row-major bf16 [n, C] at row stride ldo */
cudaError_t iris_launch_nchw_to_tokens(const float *x, int c, int n, void *out, int ldo,
                                       cudaStream_t stream);
cudaError_t iris_launch_f32_to_bf16(const float *x, void *out, long n, cudaStream_t stream);
cudaError_t iris_launch_bf16_to_f32(const void *x, float *out, long n, cudaStream_t stream);
cudaError_t iris_launch_f16_to_bf16(const void *x, void *out, long n, cudaStream_t stream);
/* z += dt * v ; or with CFG: z += dt * (vu + g (vc - vu)) */
cudaError_t iris_launch_euler(float *z, const float *v, const float *v_uncond, float guidance,
                              float dt, long n, cudaStream_t stream);
/* seeded N(0, std) bf16 fill (counter-based hash RNG; used for random-init models) */
cudaError_t iris_launch_randn_bf16(void *out, long n, uint64_t seed, uint64_t stream_id,
                                   float mean, float std, cudaStream_t stream);
cudaError_t iris_launch_randn_f32(float *out, long n, uint64_t seed, uint64_t stream_id,
                                  float mean, float std, cudaStream_t stream);

/* op-level helpers (iris_gpu_* surface) */
cudaError_t iris_launch_head_rmsnorm_rope(void *x, int ld, int rows, int heads, const float *w,
                                          float eps, const float *rope_cos,
                                          const float *rope_sin, cudaStream_t stream);
cudaError_t iris_launch_silu_mul_bf16(void *gate, const void *up, long n, cudaStream_t stream);
cudaError_t iris_launch_gated_add_bf16(void *out, const void *gate, const void *proj, int rows,
                                       int cols, cudaStream_t stream);
cudaError_t iris_launch_rmsnorm(const float *x, int ldx, const float *w, float *out_f32,
                                void *out_bf16, int ldout, int rows, int cols, float eps,
                                const float *mul, cudaStream_t stream);
/* Z-Image row kernels */
cudaError_t iris_launch_resid_rmsnorm_gate(float *x, int ldx, const float *y, int ldy, const float *w,
                                           const float *gate, int rows, int cols, float eps,
                                           cudaStream_t stream);
cudaError_t iris_launch_zi_mod_transform(float *m, int dim, long n, cudaStream_t stream);
cudaError_t iris_launch_patchify(const float *lat, int c, int H, int W, int ps, void *out, int ldo,
                                 cudaStream_t stream);
cudaError_t iris_launch_unpatchify(const float *tok, int ldt, int c, int H, int W, int ps, float *lat,
                                   cudaStream_t stream);
cudaError_t iris_launch_fill_rows_f32(float *dst, int ld, const float *vec, int n, int cols,
                                      cudaStream_t stream);
/* [gate; up] (2F rows) -> 256-row blocks of [gate 128 | up 128] (GEMM SwiGLU layout) */
cudaError_t iris_launch_interleave_gate_up(void *dst, const void *src, int F, int cols,
                                           cudaStream_t stream);
cudaError_t iris_launch_copy_rows_bf16(void *dst, int ldd, const void *src, int lds, int rows,
                                       int cols, cudaStream_t stream);
/* LoRA fold (lora_kernels.cu): w[drow[i], 0:cols] = bf16(w0[drow[i], 0:cols] +
 * scale * (B A)[bsrc[i], acol(0:cols)]) for i < nrows, on the tcgen05 GEMM.
 * B [*, rank] and A [rank, in_dim] are the adapter's matrices as stored
 * (IRIS_LORA_BF16 / F16 / F32); acol(c) = c < acol_seg ? acol_off0 + c :
 * acol_off1 + (c - acol_seg).  cols % 128 == 0, ld % 8 == 0, w / w0
 * 16-byte aligned (may alias).  Scratch: iris_lora_fold_scratch_bytes. */
#define IRIS_LORA_BF16 0
#define IRIS_LORA_F16 1
#define IRIS_LORA_F32 2
typedef struct {
    void *w;
    const void *w0;
    int ld, cols, nrows;
    const void *B;
    int b_dtype, rank;
    const int *bsrc, *drow;     /* device [nrows] */
    const void *A;
    int a_dtype, in_dim;
    int acol_seg, acol_off0, acol_off1;
    float scale;
} IrisLoraFold;
size_t iris_lora_fold_scratch_bytes(int nrows, int cols, int rank, int split);
/* prep kernels + one GEMM; *launches = kernels queued */
cudaError_t iris_launch_lora_fold(const IrisLoraFold *f, void *scratch, size_t scratch_bytes, int *status,
                                  int num_sms, cudaStream_t stream, int *launches);

/* ------------------------------------------------------------------ IP-Adapter (ip_kernels.cu) */
/* f32 C[M, N] = A[M, K] (B[N, K])^T (transB) or A B[K, N], + bias[N] */
cudaError_t iris_launch_ip_sgemm(const float *A, int lda, const float *B, int ldb, int transB, const float *bias,
                                 float *C, int ldc, int M, int N, int K, cudaStream_t stream);
/* the same for `batch` problems, operand z at A + z*sA, B + z*sB, C + z*sC */
cudaError_t iris_launch_ip_sgemm_batched(const float *A, int lda, long sA, const float *B, int ldb, long sB,
                                         int transB, const float *bias, float *C, int ldc, long sC, int M, int N,
                                         int K, int batch, cudaStream_t stream);
cudaError_t iris_launch_ip_colnorm(const float *x, int n, int S, const float *g, const float *b, float *out,
                                   cudaStream_t stream);
cudaError_t iris_launch_ip_layernorm(float *x, int rows, int H, const float *w, const float *b, cudaStream_t stream);
cudaError_t iris_launch_ip_film_tokens(const float *q, const float *film, int T, int H, float *out,
                                       cudaStream_t stream);
cudaError_t iris_launch_ip_mha(const float *Q, const float *K, const float *V, int T, int n, int H, int heads,
                               float *out, cudaStream_t stream);
cudaError_t iris_launch_ip_scale_rows(float *x, int rows, int H, int row_split, float s0, float s1,
                                      cudaStream_t stream);
/* bf16 q [rows, ldq] after the pair RoPE of position ids pos [rows][4] and spec
 * -> bf16 [rows, H] before it */
cudaError_t iris_launch_ip_unrope(const void *q, int ldq, const uint16_t *pos, const IrisRopeSpec *spec,
                                  int rows, int H, void *out, cudaStream_t stream);
/* f32 hidden[rows, ldh] += *scale * bf16 o[rows, H] */
cudaError_t iris_launch_ip_add(float *hidden, int ldh, const void *o, int rows, int H, const float *scale,
                               cudaStream_t stream);

/* y[n] += (*a) * x[n], a in device memory; in-place SiLU */
cudaError_t iris_launch_axpy_dev(float *y, const float *x, const float *a, int n, cudaStream_t stream);
cudaError_t iris_launch_silu_f32(float *x, int n, cudaStream_t stream);

/* ------------------------------------------------------------------ text encoder (Qwen3) */
/* x[s] = f32 of table[ids[s]] (bf16 [vocab, H]); ids outside [0, vocab) -> zeros */
cudaError_t iris_launch_embed_rows(const int *ids, int S, const void *table, int vocab, int H, float *x,
                                   cudaStream_t stream);
/* f32 QKV projection [S, ld] (nh Q heads, nkv K heads, nkv V heads of 128) ->
 * bf16 q [S, nh*128], k / v [S, nkv*128]: per-head RMSNorm (qw / kw) and
 * split-half RoPE (cos/sin [S, 64]) on Q and K */
cudaError_t iris_launch_qk_norm_rope_half(const float *qkv, int ld, int S, int nh, int nkv, const float *qw,
                                          const float *kw, const float *cosb, const float *sinb, float eps, void *q,
                                          void *k, void *v, cudaStream_t stream);

/* ------------------------------------------------------------------ autoencoder decoder
 * Stride-1 convolution with zero padding as an implicit GEMM on the tensor
 * cores.  Activations are NHWC bf16 [H, W, C]; output pixel p, channel n:
 *   out[p, n] = bias[n] (+ resid[p, n]) + sum over K of A(p, k) W[n, k]
 * where K runs over segment 0 (taps0 = 9: the 3x3 taps (dy, dx) row-major,
 * each over cin0 channels of tmap_a[0] at the shifted pixel; taps0 = 1: the
 * pixel itself) and then segment 1 (cin1 channels of tmap_a[1] at the pixel:
 * a fused 1x1 shortcut convolution).  W is bf16 [cout_pad, K] row-major,
 * K = taps0 * cin0 + cin1.  Tiles: 128 pixels (a bw x bh block, bw * bh =
 * 128) x bn output channels. */
enum {
    IRIS_CONV_F32 = 0,        /* out f32 NHWC [H * W, cout]                               */
    IRIS_CONV_BF16 = 1,       /* out bf16 NHWC [H * W, cout]                              */
    IRIS_CONV_F32_NCHW = 2,   /* out f32 channel planes [cout, H * W] (cout <= 32)        */
};
typedef struct {
    CUtensorMap tmap_a[2];    /* NHWC bf16 activations: 3-D {C, W, H}, box {64, bw, bh}    */
    CUtensorMap tmap_b;       /* weights: 2-D [cout_pad, K], box {64, min(bn, 128)}        */
    CUtensorMap tmap_b_half;  /* the same weights, box {64, bn / 2} (CTA-pair launches)    */
    int pair;                 /* 1: CTA-pair kernel (bn 128 or 256; 256-pixel units)       */
    int H, W;
    int bw, bh;               /* bw a power of two */
    int bw_log2;
    int taps0;                /* 9 or 1 */
    int cin0, cin1;           /* multiples of 64; cin1 = 0: no second segment */
    int cout, cout_pad, bn;   /* bn in {16, 32, 64, 128, 256}; cout_pad % bn == 0 */
    int mode;
    void *out;
    const float *bias;        /* [cout_pad] */
    const float *resid;       /* optional f32 NHWC [H * W, cout]; may be `out` (F32 mode) */
    double *gn_part;          /* optional: GroupNorm partial sums of the outputs, one slot of
                                 64 doubles (32 groups x {sum, sum of squares}) per CTA;
                                 iris_conv_grid slots                               */
    int gn_cg;                /* channels per group (cout / 32: 4, 8 or 16)        */
    int *status;
} IrisConvParams;
/* 3-D tensor map over an NHWC bf16 tensor [H, W, C] (C % 64 == 0), box {64, bw, bh} */
int iris_make_tmap_nhwc_bf16(CUtensorMap *m, const void *ptr, int H, int W, int C, int bw, int bh);
cudaError_t iris_conv_init(void);
cudaError_t iris_launch_conv(const IrisConvParams *p, int num_sms, cudaStream_t stream);
/* CTAs iris_launch_conv starts for p */
int iris_conv_grid(const IrisConvParams *p, int num_sms);
/* CTA pairs of the pair kernel that fit on the device at once (0: none) */
int iris_conv_pairs_available(void);
/* GroupNorm (32 groups) of a convolution's output from its gn_part partials
 * (nparts slots, count = pixels * C / 32 values per group): per-channel affine
 * ab[c] = gamma[c] * rstd_g, ab[C + c] = beta[c] - mean_g * ab[c] */
cudaError_t iris_launch_gn_finalize(const double *part, int nparts, int C, const float *gamma, const float *beta,
                                    float eps, long count, float *ab, cudaStream_t stream);
/* NHWC f32 [P, C] -> bf16 x * ab[c] + ab[C + c] (+ SiLU); raw (optional) gets the plain bf16 copy */
cudaError_t iris_launch_gn_affine(const float *x, long P, int C, const float *ab, int silu, void *out, void *raw,
                                  cudaStream_t stream);
/* GroupNorm partial sums (32 groups) of NHWC f32 [P, C] when no convolution
 * epilogue produced them: one slot of 64 doubles per block (gn_part layout) */
cudaError_t iris_launch_gn_stats(const float *x, long P, int C, double *part, int nblocks, cudaStream_t stream);
/* NHWC f32 [P, C] -> bf16, optionally 2x nearest upsampled (W = input width; output [2H, 2W, C]) */
cudaError_t iris_launch_nhwc_to_bf16(const float *x, long P, int C, int W, int up2, void *out, cudaStream_t stream);
/* latent [4z, h, w] -> denormalised (bn_std/bn_mean, else x / scaling + shift),
 * unpatchified, optional f32 post-quant 1x1 conv -> bf16 NHWC [2h, 2w, 64] */
cudaError_t iris_launch_vae_latent_prep(const float *lat, int z, int h, int w, const float *bn_mean,
                                        const float *bn_std, float scaling, float shift, const float *pq_w,
                                        const float *pq_b, void *out, cudaStream_t stream);
/* rows of f32 scores [rows, ld]: bf16 softmax(scale * s) over the first n columns, zeros after */
cudaError_t iris_launch_vae_softmax(const float *s, int rows, int ld, int n, float scale, void *out,
                                    cudaStream_t stream);
/* f32 planes [3, P] -> uint8 [P, 3] (reference rounding) */
cudaError_t iris_launch_vae_rgb8(const float *x, long P, uint8_t *out, cudaStream_t stream);

/* f32 row kernels of the op-level surface (compat_kernels.cu) */
/* out = (1 + scale) * LayerNorm(x) + shift, rows of `cols` f32, eps inside the sqrt */
cudaError_t iris_launch_layernorm_mod_f32(float *out, const float *x, const float *shift, const float *scale,
                                          int rows, int cols, float eps, cudaStream_t stream);
/* per-head (128) RMSNorm of f32 [rows, heads * 128] in place; x and w 16-byte aligned */
cudaError_t iris_launch_head_rmsnorm_f32(float *x, int rows, int heads, const float *w, float eps,
                                         cudaStream_t stream);
/* consecutive-pair RoPE in place on [rows, heads * hd] (bf16 != 0: bf16 data) from
 * [rows, table_ld] cos/sin tables, pair i using column 2i */
cudaError_t iris_launch_rope_pairs(void *x, int bf16, int rows, int heads, int hd, const float *cs,
                                   const float *sn, int table_ld, cudaStream_t stream);
cudaError_t iris_launch_silu_mul_f32(float *gate, const float *up, long n, cudaStream_t stream);
/* out[r, c] += gate[c] * proj[r, c] */
cudaError_t iris_launch_gated_add_f32(float *out, const float *gate, const float *proj, int rows, int cols,
                                      cudaStream_t stream);
cudaError_t iris_launch_add_f32(float *out, const float *a, const float *b, long n, cudaStream_t stream);
cudaError_t iris_launch_add_bf16(void *out, const void *a, const void *b, long n, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif
