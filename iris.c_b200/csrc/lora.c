/*
 * LoRA adapters for the Flux transformer, folded into the resident bf16
 * weights on the GPU.
 *
 * Reference: iris_lora.c — format detection :87-114, XLabs :240, Kohya :281,
 * Diffusers :342, BFL :423 loaders, lora_load :504; iris_load_lora /
 * iris_unload_lora (iris.c:460-481, iris.h:163-168); hooks in the blocks
 * (iris_transformer_flux.c:2429-2487 q/k/v after the projection and before
 * QK-norm, :2529-2532 output projections, :3818 single linear1, :3909 single
 * linear2), each `out += scale * B (A x)` (lora_apply, iris_lora.c:43).
 *
 * The reference keeps the adapters beside the model and pays two thin GEMMs
 * after every adapted linear on every step (and leaves its GPU path while a
 * LoRA is active).  Here `W x + scale * B (A x) = (W + scale * B A) x` is used
 * once at load time: each adapter is folded into the weight rows it adapts
 * (lora_kernels.cu), so a LoRA step runs the same graph at the same speed as a
 * step without one.  The weights an adapter touched are kept as they were
 * loaded, so a new adapter, a new scale or an unload starts again from the base
 * model (no drift from repeated fold/unfold).
 *
 * Adapter shapes follow the reference: A (`down` / `lora_A`) [rank, in],
 * B (`up` / `lora_B`) [out, rank].  A fused Q|K|V up matrix [3H, rank] shares
 * one A (load_adapter_split_qkv, iris_lora.c:184); here it stays one adapter
 * over the stacked Q|K|V rows of the device weight.  The device weights differ
 * from the reference layout in two ways the fold maps through: the single
 * block's gate/up rows are interleaved in 128-row blocks (SwiGLU epilogue
 * layout), and a tensor-parallel rank holds only its heads' Q/K/V rows, its
 * MLP columns' gate/up rows, and the matching input columns of the output
 * projections.
 *
 * Stricter than the reference: every adapter's shapes are checked against the
 * model (the reference does not check the single-block or fused-QKV input
 * widths, iris_lora.c:191, :327), and a B whose second dimension is not the
 * rank is skipped.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "flux_internal.h"

/* which resident weight an adapter folds into */
enum { TGT_QKV = 0, TGT_PROJ = 1, TGT_L1 = 2, TGT_L2 = 3 };

typedef struct {
    int tgt, block, stream;  /* stream (double blocks): 1 image, 0 text */
    int row_off;             /* first reference row of the target this B covers */
    int rank, in_dim, out_dim;
    const st_tensor_t *ta, *tb;  /* A [rank, in_dim], B [out_dim, rank] in the open file */
    size_t a_off, b_off;     /* their bytes in the device copy of the file's tensors */
} lora_ad_t;

typedef struct {
    uint16_t *live, *orig;
    size_t numel;
} lora_saved_t;

struct iris_flux_lora {
    int adapters;
    float scale;
    int nsaved, cap;
    lora_saved_t *saved;
    double merge_ms, merge_bytes;
};

/* safetensors dtype -> the fold kernels' operand type (-1: unsupported) */
static int fold_dtype(st_dtype_t d) {
    return d == ST_BF16 ? IRIS_LORA_BF16 : d == ST_F16 ? IRIS_LORA_F16 : d == ST_F32 ? IRIS_LORA_F32 : -1;
}

typedef enum { FMT_UNKNOWN = 0, FMT_XLABS, FMT_KOHYA, FMT_DIFFUSERS, FMT_BFL } lora_fmt_t;

/* first tensor name that identifies a format decides it, in the reference's
 * order of tests (detect_format, iris_lora.c:95-113) */
static lora_fmt_t detect_format(const st_model_t *st) {
    for (int i = 0; i < st->ntensors; i++) {
        const char *n = st->tensors[i].name;
        if (strstr(n, "processor.")) return FMT_XLABS;
        if (strstr(n, "lora_unet_")) return FMT_KOHYA;
        if (strstr(n, "transformer.transformer_blocks") || strstr(n, "transformer.single_transformer_blocks") ||
            strstr(n, "transformer.x_embedder"))
            return FMT_DIFFUSERS;
        if (strstr(n, "diffusion_model.double_blocks.") || strstr(n, "base_model.model.double_blocks."))
            return FMT_BFL;
    }
    return FMT_UNKNOWN;
}

typedef struct {
    lora_ad_t *v;
    int n, cap;
} ad_list_t;

static void ads_free(ad_list_t *l) {
    free(l->v);
    memset(l, 0, sizeof(*l));
}

/* Record one (down, up) pair.  Returns 1 when added, 0 when absent or skipped,
 * < 0 on an allocation failure.  exp_in / exp_out: the shapes the target needs. */
static int add_adapter(ad_list_t *l, const st_model_t *st, const char *down_key, const char *up_key,
                       int tgt, int block, int stream, int row_off, int exp_in, int exp_out) {
    const st_tensor_t *dn = st_find(st, down_key), *up = st_find(st, up_key);
    if (!dn || !up || dn->ndim != 2 || up->ndim != 2) return 0;
    int rank = (int)dn->shape[0], in = (int)dn->shape[1], out = (int)up->shape[0];
    if (fold_dtype(dn->dtype) < 0 || fold_dtype(up->dtype) < 0 ||
        dn->nbytes != (size_t)rank * in * (dn->dtype == ST_F32 ? 4 : 2) ||
        up->nbytes != (size_t)out * rank * (up->dtype == ST_F32 ? 4 : 2)) {
        fprintf(stderr, "iris_cuda LoRA: skipping %s: unsupported data type or size\n", down_key);
        return 0;
    }
    if (rank <= 0 || up->shape[1] != rank || in != exp_in || out != exp_out) {
        fprintf(stderr, "iris_cuda LoRA: skipping %s: A [%lld, %lld], B [%lld, %lld], expected in %d, out %d\n",
                down_key, (long long)dn->shape[0], (long long)dn->shape[1], (long long)up->shape[0],
                (long long)up->shape[1], exp_in, exp_out);
        return 0;
    }
    if (l->n == l->cap) {
        int nc = l->cap ? 2 * l->cap : 64;
        lora_ad_t *nv = (lora_ad_t *)realloc(l->v, (size_t)nc * sizeof(*nv));
        if (!nv) return IRIS_CUDA_ERR_OOM;
        l->v = nv;
        l->cap = nc;
    }
    lora_ad_t *a = &l->v[l->n];
    memset(a, 0, sizeof(*a));
    a->tgt = tgt; a->block = block; a->stream = stream; a->row_off = row_off;
    a->rank = rank; a->in_dim = in; a->out_dim = out;
    a->ta = dn;
    a->tb = up;
    l->n++;
    return 1;
}

#define ADD(dk, uk, tgt, blk, s, off, in, out)                                         \
    do {                                                                               \
        int r_ = add_adapter(l, st, dk, uk, tgt, blk, s, off, in, out);                \
        if (r_ < 0) return r_;                                                         \
    } while (0)

/* The key names of each format (iris_lora.c:240-486).  Double blocks: stream 1
 * is the image stream, 0 the text stream. */
static int collect(ad_list_t *l, const st_model_t *st, lora_fmt_t fmt, int nd, int ns, int H, int F) {
    char dk[320], uk[320];
    const int L1 = 3 * H + 2 * F, L2in = H + F;
    if (fmt == FMT_XLABS) {
        for (int i = 0; i < nd; i++)
            for (int s = 1; s >= 0; s--) {
                int n = s ? 1 : 2;  /* lora1 = image, lora2 = text */
                snprintf(dk, sizeof(dk), "double_blocks.%d.processor.qkv_lora%d.down.weight", i, n);
                snprintf(uk, sizeof(uk), "double_blocks.%d.processor.qkv_lora%d.up.weight", i, n);
                ADD(dk, uk, TGT_QKV, i, s, 0, H, 3 * H);
                snprintf(dk, sizeof(dk), "double_blocks.%d.processor.proj_lora%d.down.weight", i, n);
                snprintf(uk, sizeof(uk), "double_blocks.%d.processor.proj_lora%d.up.weight", i, n);
                ADD(dk, uk, TGT_PROJ, i, s, 0, H, H);
            }
        return 0;
    }
    if (fmt == FMT_KOHYA || fmt == FMT_BFL) {
        const char *pre = "diffusion_model";
        if (fmt == FMT_BFL)
            for (int t = 0; t < st->ntensors; t++)
                if (strstr(st->tensors[t].name, "base_model.model.double_blocks.")) { pre = "base_model.model"; break; }
        for (int i = 0; i < nd; i++)
            for (int s = 1; s >= 0; s--) {
                const char *sn = s ? "img" : "txt";
                for (int pj = 0; pj < 2; pj++) {
                    const char *what = pj ? "proj" : "qkv";
                    if (fmt == FMT_KOHYA) {
                        snprintf(dk, sizeof(dk), "lora_unet_double_blocks_%d_%s_attn_%s.lora_down.weight", i, sn, what);
                        snprintf(uk, sizeof(uk), "lora_unet_double_blocks_%d_%s_attn_%s.lora_up.weight", i, sn, what);
                    } else {
                        snprintf(dk, sizeof(dk), "%s.double_blocks.%d.%s_attn.%s.lora_A.weight", pre, i, sn, what);
                        snprintf(uk, sizeof(uk), "%s.double_blocks.%d.%s_attn.%s.lora_B.weight", pre, i, sn, what);
                    }
                    ADD(dk, uk, pj ? TGT_PROJ : TGT_QKV, i, s, 0, H, pj ? H : 3 * H);
                }
            }
        for (int i = 0; i < ns; i++)
            for (int k = 1; k <= 2; k++) {
                if (fmt == FMT_KOHYA) {
                    snprintf(dk, sizeof(dk), "lora_unet_single_blocks_%d_linear%d.lora_down.weight", i, k);
                    snprintf(uk, sizeof(uk), "lora_unet_single_blocks_%d_linear%d.lora_up.weight", i, k);
                } else {
                    snprintf(dk, sizeof(dk), "%s.single_blocks.%d.linear%d.lora_A.weight", pre, i, k);
                    snprintf(uk, sizeof(uk), "%s.single_blocks.%d.linear%d.lora_B.weight", pre, i, k);
                }
                ADD(dk, uk, k == 1 ? TGT_L1 : TGT_L2, i, 0, 0, k == 1 ? H : L2in, k == 1 ? L1 : H);
            }
        return 0;
    }
    /* Diffusers: separate Q/K/V per stream, the single block's fused
     * to_qkv_mlp_proj / to_out (proj_out as the fallback name of to_out) */
    static const char *const names[2][4] = {{"add_q_proj", "add_k_proj", "add_v_proj", "to_add_out"},
                                            {"to_q", "to_k", "to_v", "to_out.0"}};
    for (int i = 0; i < nd; i++)
        for (int s = 1; s >= 0; s--)
            for (int j = 0; j < 4; j++) {
                snprintf(dk, sizeof(dk), "transformer.transformer_blocks.%d.attn.%s.lora_A.weight", i, names[s][j]);
                snprintf(uk, sizeof(uk), "transformer.transformer_blocks.%d.attn.%s.lora_B.weight", i, names[s][j]);
                if (j < 3) ADD(dk, uk, TGT_QKV, i, s, j * H, H, H);
                else ADD(dk, uk, TGT_PROJ, i, s, 0, H, H);
            }
    for (int i = 0; i < ns; i++) {
        snprintf(dk, sizeof(dk), "transformer.single_transformer_blocks.%d.attn.to_qkv_mlp_proj.lora_A.weight", i);
        snprintf(uk, sizeof(uk), "transformer.single_transformer_blocks.%d.attn.to_qkv_mlp_proj.lora_B.weight", i);
        ADD(dk, uk, TGT_L1, i, 0, 0, H, L1);
        snprintf(dk, sizeof(dk), "transformer.single_transformer_blocks.%d.attn.to_out.lora_A.weight", i);
        snprintf(uk, sizeof(uk), "transformer.single_transformer_blocks.%d.attn.to_out.lora_B.weight", i);
        int before = l->n;
        ADD(dk, uk, TGT_L2, i, 0, 0, L2in, H);
        if (l->n == before) {
            snprintf(dk, sizeof(dk), "transformer.single_transformer_blocks.%d.proj_out.lora_A.weight", i);
            snprintf(uk, sizeof(uk), "transformer.single_transformer_blocks.%d.proj_out.lora_B.weight", i);
            ADD(dk, uk, TGT_L2, i, 0, 0, L2in, H);
        }
    }
    return 0;
}
#undef ADD

/* ---------------------------------------------------------------- layout map */

/* device weight (pointer, rows, columns) of an adapter's target on this rank */
static uint16_t *target_weight(const iris_cuda_flux_t *tf, const lora_ad_t *a, int *rows, int *cols) {
    const int H = tf->H, Hl = tf->Hl, Fl = tf->Fl;
    switch (a->tgt) {
    case TGT_QKV: *rows = 3 * Hl; *cols = H; return tf->dbl[a->block].w_qkv[a->stream];
    case TGT_PROJ: *rows = H; *cols = Hl; return tf->dbl[a->block].w_out[a->stream];
    case TGT_L1: *rows = 3 * Hl + 2 * Fl; *cols = H; return tf->sgl[a->block].w_fused;
    default: *rows = H; *cols = Hl + Fl; return tf->sgl[a->block].w_out;
    }
}

/* Device row of reference row R of the target, -1 when another rank owns it.
 * Q|K|V rows: head rows [h0, h0+Hl) of each third.  Single-block gate/up rows
 * (after 3H): this rank's MLP columns [f0, f0+Fl), interleaved as 128 gate
 * rows then the same 128 features' up rows. */
static int device_row(const iris_cuda_flux_t *tf, int tgt, int R) {
    const int H = tf->H, F = tf->F, Hl = tf->Hl, Fl = tf->Fl;
    const int h0 = tf->tp_rank * Hl, f0 = tf->tp_rank * Fl;
    if (tgt == TGT_PROJ || tgt == TGT_L2) return R;
    if (R < 3 * H) {
        int j = R / H, hr = R % H;
        return (hr >= h0 && hr < h0 + Hl) ? j * Hl + hr - h0 : -1;
    }
    int m = R - 3 * H, up = m >= F, fc = up ? m - F : m;
    if (fc < f0 || fc >= f0 + Fl) return -1;
    int l = fc - f0;
    return 3 * Hl + (l / 128) * 256 + up * 128 + l % 128;
}

/* reference input column of device column c */
static int ref_col(const iris_cuda_flux_t *tf, int tgt, int c) {
    const int H = tf->H, Hl = tf->Hl, Fl = tf->Fl;
    const int h0 = tf->tp_rank * Hl, f0 = tf->tp_rank * Fl;
    if (tgt == TGT_QKV || tgt == TGT_L1) return c;
    if (c < Hl) return h0 + c;
    return H + f0 + (c - Hl);  /* TGT_L2: MLP half of [attention | MLP] */
}

/* ---------------------------------------------------------------- state */

static int copy_d2d(void *dst, const void *src, size_t bytes, const char *what) {
    return iris_cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, g_rt.stream), what);
}

/* the saved copy of a live weight, or NULL */
static lora_saved_t *find_saved(struct iris_flux_lora *L, const uint16_t *live) {
    for (int i = 0; i < L->nsaved; i++)
        if (L->saved[i].live == live) return &L->saved[i];
    return NULL;
}

/* Save a live weight (still the base model's) the first time an adapter
 * targets it. */
static lora_saved_t *save_weight(struct iris_flux_lora *L, uint16_t *live, size_t numel) {
    if (L->nsaved == L->cap) {
        int nc = L->cap ? 2 * L->cap : 32;
        lora_saved_t *nv = (lora_saved_t *)realloc(L->saved, (size_t)nc * sizeof(*nv));
        if (!nv) return NULL;
        L->saved = nv;
        L->cap = nc;
    }
    uint16_t *o = (uint16_t *)iris_dmalloc(numel * 2);
    if (!o) return NULL;
    if (copy_d2d(o, live, numel * 2, "LoRA save")) {
        iris_dfree(o);
        return NULL;
    }
    lora_saved_t *sv = &L->saved[L->nsaved++];
    sv->live = live;
    sv->orig = o;
    sv->numel = numel;
    return sv;
}

static int restore_all(struct iris_flux_lora *L) {
    for (int i = 0; i < L->nsaved; i++) {
        int rc = copy_d2d(L->saved[i].live, L->saved[i].orig, L->saved[i].numel * 2, "LoRA restore");
        if (rc) return rc;
    }
    return 0;
}

void iris_flux_lora_release(iris_cuda_flux_t *tf) {
    if (!tf || !tf->lora) return;
    struct iris_flux_lora *L = tf->lora;
    iris_stream_drain();
    for (int i = 0; i < L->nsaved; i++) iris_dfree(L->saved[i].orig);
    free(L->saved);
    free(L);
    tf->lora = NULL;
}

/* Device rows this rank holds of an adapter's B: raw row bsrc[i] -> row drow[i]
 * of the target weight.  Returns the count. */
static int adapter_rows(const iris_cuda_flux_t *tf, const lora_ad_t *a, int rows, int *bsrc, int *drow) {
    int n = 0;
    for (int r = 0; r < a->out_dim; r++) {
        int d = device_row(tf, a->tgt, a->row_off + r);
        if (d < 0 || d >= rows) continue;
        bsrc[n] = r;
        drow[n] = d;
        n++;
    }
    return n;
}

/* Fold every adapter into the live weights.  Device work, in stream order:
 *  1. the adapters' A / B bytes, as stored in the file, in one device buffer;
 *  2. for each target weight: first use -> save the base copy; a weight the
 *     previous adapter changed and the new one does not cover entirely ->
 *     restore it from the base copy;
 *  3. per adapter: prep kernels + the tcgen05 GEMM with the fold epilogue
 *     (reads the base rows, writes the live rows). */
static int fold(iris_cuda_flux_t *tf, struct iris_flux_lora *L, ad_list_t *ads, const st_model_t *st,
                float scale) {
    int rc = 0, max_rows = 0;
    size_t raw_bytes = 0, scratch = 0;
    for (int i = 0; i < ads->n; i++) {
        lora_ad_t *a = &ads->v[i];
        int rows, cols;
        target_weight(tf, a, &rows, &cols);
        if (a->out_dim > max_rows) max_rows = a->out_dim;
        a->a_off = raw_bytes;
        raw_bytes += (a->ta->nbytes + 255) & ~(size_t)255;
        a->b_off = raw_bytes;
        raw_bytes += (a->tb->nbytes + 255) & ~(size_t)255;
        const int split = a->ta->dtype != ST_BF16 || a->tb->dtype != ST_BF16;
        size_t sb = iris_lora_fold_scratch_bytes(a->out_dim, cols, a->rank, split);
        if (sb > scratch) scratch = sb;
    }
    int *hmap = (int *)malloc((size_t)ads->n * 2 * max_rows * sizeof(int));
    int *nrow = (int *)calloc((size_t)ads->n, sizeof(int));
    uint8_t *raw = (uint8_t *)iris_dmalloc(raw_bytes + scratch + (size_t)ads->n * 2 * max_rows * sizeof(int) + 512);
    cudaEvent_t e0 = NULL, e1 = NULL;
    double bytes = 0;
    if (!hmap || !nrow || !raw) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "LoRA staging"); goto out; }
    uint8_t *dscratch = raw + ((raw_bytes + 255) & ~(size_t)255);
    int *dmap = (int *)(dscratch + ((scratch + 255) & ~(size_t)255));
    /* row maps (host) */
    for (int i = 0; i < ads->n; i++) {
        int rows, cols;
        target_weight(tf, &ads->v[i], &rows, &cols);
        int *bs = hmap + (size_t)i * 2 * max_rows;
        nrow[i] = adapter_rows(tf, &ads->v[i], rows, bs, bs + max_rows);
    }
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    /* 1. uploads (stream-ordered copies straight from the mapped file) */
    for (int i = 0; i < ads->n && !rc; i++) {
        const lora_ad_t *a = &ads->v[i];
        const uint8_t *base = (const uint8_t *)st->maps[a->ta->file] + st->data_start[a->ta->file];
        rc = iris_cuda_check(cudaMemcpyAsync(raw + a->a_off, base + a->ta->offset, a->ta->nbytes,
                                             cudaMemcpyHostToDevice, g_rt.stream), "LoRA upload");
        base = (const uint8_t *)st->maps[a->tb->file] + st->data_start[a->tb->file];
        if (!rc)
            rc = iris_cuda_check(cudaMemcpyAsync(raw + a->b_off, base + a->tb->offset, a->tb->nbytes,
                                                 cudaMemcpyHostToDevice, g_rt.stream), "LoRA upload");
    }
    if (!rc)
        rc = iris_cuda_check(cudaMemcpyAsync(dmap, hmap, (size_t)ads->n * 2 * max_rows * sizeof(int),
                                             cudaMemcpyHostToDevice, g_rt.stream), "LoRA upload");
    if (!rc) rc = iris_stream_drain();  /* the pageable sources must stay valid until copied */
    if (rc) goto out;
    cudaEventRecord(e0, g_rt.stream);
    /* 2. base copies: save on first use, restore what the new adapter does not rewrite */
    for (int i = 0; i < ads->n; i++) {
        int rows, cols;
        uint16_t *live = target_weight(tf, &ads->v[i], &rows, &cols);
        if (!find_saved(L, live)) {
            if (!save_weight(L, live, (size_t)rows * cols)) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "LoRA base copy"); goto out; }
            bytes += 4.0 * rows * cols;
        }
    }
    for (int s = 0; s < L->nsaved; s++) {
        long covered = 0;
        for (int i = 0; i < ads->n; i++) {
            int rows, cols;
            if (target_weight(tf, &ads->v[i], &rows, &cols) == L->saved[s].live) covered += (long)nrow[i] * cols;
        }
        if ((size_t)covered != L->saved[s].numel) {
            if ((rc = copy_d2d(L->saved[s].live, L->saved[s].orig, L->saved[s].numel * 2, "LoRA restore"))) goto out;
            bytes += 4.0 * L->saved[s].numel;
        }
    }
    /* 3. folds */
    const int H = tf->H, Hl = tf->Hl, h0 = tf->tp_rank * tf->Hl, f0 = tf->tp_rank * tf->Fl;
    for (int i = 0; i < ads->n; i++) {
        const lora_ad_t *a = &ads->v[i];
        if (!nrow[i]) continue;
        int rows, cols;
        IrisLoraFold f;
        memset(&f, 0, sizeof(f));
        f.w = target_weight(tf, a, &rows, &cols);
        f.w0 = find_saved(L, (uint16_t *)f.w)->orig;
        f.ld = cols;
        f.cols = cols;
        f.nrows = nrow[i];
        f.B = raw + a->b_off;
        f.b_dtype = fold_dtype(a->tb->dtype);
        f.rank = a->rank;
        f.bsrc = dmap + (size_t)i * 2 * max_rows;
        f.drow = f.bsrc + max_rows;
        f.A = raw + a->a_off;
        f.a_dtype = fold_dtype(a->ta->dtype);
        f.in_dim = a->in_dim;
        /* device column c of the target reads A's column acol(c) */
        f.acol_seg = (a->tgt == TGT_L2) ? Hl : cols;
        f.acol_off0 = (a->tgt == TGT_PROJ || a->tgt == TGT_L2) ? h0 : 0;
        f.acol_off1 = H + f0;
        f.scale = scale;
        int n = 0;
        rc = iris_cuda_check(iris_launch_lora_fold(&f, dscratch, scratch, g_rt.d_status, g_rt.num_sms, g_rt.stream,
                                                   &n), "LoRA fold");
        iris_count_launch((uint64_t)n);
        if (rc) goto out;
        bytes += 4.0 * nrow[i] * cols + (double)a->ta->nbytes + (double)a->tb->nbytes;
    }
    cudaEventRecord(e1, g_rt.stream);
    if ((rc = iris_cuda_check(cudaEventSynchronize(e1), "LoRA fold"))) goto out;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    L->merge_ms = ms;
    L->merge_bytes = bytes;
out:
    iris_stream_drain();
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    iris_dfree(raw);
    free(hmap);
    free(nrow);
    return rc;
}

int iris_cuda_flux_load_lora(iris_cuda_flux_t *tf, const char *path, float scale) {
    if (!tf || !path || !*path) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (scale != scale) return iris_fail(IRIS_CUDA_ERR_ARG, "LoRA scale is NaN");
    st_model_t st;
    if (st_open_file(&st, path) != 0) return iris_fail(IRIS_CUDA_ERR_IO, "cannot open LoRA %s", path);
    lora_fmt_t fmt = detect_format(&st);
    if (fmt == FMT_UNKNOWN) {
        st_close(&st);
        return iris_fail(IRIS_CUDA_ERR_IO, "unknown LoRA format in %s", path);
    }
    ad_list_t ads;
    memset(&ads, 0, sizeof(ads));
    int rc = collect(&ads, &st, fmt, tf->cfg.n_double, tf->cfg.n_single, tf->H, tf->F);
    if (rc) { st_close(&st); ads_free(&ads); return iris_fail(rc, "LoRA: out of host memory"); }
    if (!ads.n) {
        /* like lora_load (iris_lora.c:578): nothing usable leaves the current state */
        st_close(&st);
        ads_free(&ads);
        return iris_fail(IRIS_CUDA_ERR_ARG, "LoRA %s: no adapters match this model", path);
    }
    if (!tf->lora) {
        tf->lora = (struct iris_flux_lora *)calloc(1, sizeof(*tf->lora));
        if (!tf->lora) { st_close(&st); ads_free(&ads); return iris_fail(IRIS_CUDA_ERR_OOM, "LoRA state"); }
    }
    struct iris_flux_lora *L = tf->lora;
    L->adapters = 0;
    L->merge_ms = 0;
    L->merge_bytes = 0;
    if (scale == 0.0f) rc = restore_all(L);  /* strength 0: the base model exactly */
    else rc = fold(tf, L, &ads, &st, scale);
    if (!rc) {
        L->adapters = ads.n;
        L->scale = scale;
    } else {
        restore_all(L);  /* never leave a half-folded model */
    }
    iris_stream_drain();
    st_close(&st);
    ads_free(&ads);
    return rc;
}

int iris_cuda_lora_probe(const char *path, int n_double, int n_single, int hidden, int mlp, int *per_kind) {
    if (!path || n_double < 0 || n_single < 0 || hidden <= 0 || mlp <= 0)
        return iris_fail(IRIS_CUDA_ERR_ARG, "bad argument");
    st_model_t st;
    if (st_open_file(&st, path) != 0) return iris_fail(IRIS_CUDA_ERR_IO, "cannot open LoRA %s", path);
    lora_fmt_t fmt = detect_format(&st);
    if (fmt == FMT_UNKNOWN) {
        st_close(&st);
        return iris_fail(IRIS_CUDA_ERR_IO, "unknown LoRA format in %s", path);
    }
    ad_list_t ads;
    memset(&ads, 0, sizeof(ads));
    int rc = collect(&ads, &st, fmt, n_double, n_single, hidden, mlp);
    st_close(&st);
    if (rc) { ads_free(&ads); return iris_fail(rc, "LoRA: out of host memory"); }
    if (per_kind) {
        memset(per_kind, 0, 5 * sizeof(int));
        per_kind[0] = (int)fmt;
        for (int i = 0; i < ads.n; i++) per_kind[1 + ads.v[i].tgt]++;
    }
    int n = ads.n;
    ads_free(&ads);
    return n;
}

int iris_cuda_flux_unload_lora(iris_cuda_flux_t *tf) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!tf->lora) return 0;
    int rc = restore_all(tf->lora);
    if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "LoRA restore");
    iris_flux_lora_release(tf);
    return rc;
}

int iris_cuda_flux_lora_adapters(const iris_cuda_flux_t *tf) {
    return (tf && tf->lora) ? tf->lora->adapters : 0;
}

int iris_cuda_flux_lora_stats(const iris_cuda_flux_t *tf, double *fold_ms, double *fold_bytes) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (fold_ms) *fold_ms = tf->lora ? tf->lora->merge_ms : 0.0;
    if (fold_bytes) *fold_bytes = tf->lora ? tf->lora->merge_bytes : 0.0;
    return 0;
}
