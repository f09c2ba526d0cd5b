/*
 * Z-Image (S3-DiT) transformer on B200, on the same kernels as Flux.
 *
 * Reference: iris_transformer_zimage.c — forward :1696-1980, block :790-858,
 * attention :689, FFN :764, final layer :1581, patchify :1634, RoPE :595-650,
 * loader :2024-2427; sampler iris_sample.c:412.
 *
 * Layout: hidden f32 [S, D] in [IMG (padded to 32) | CAP (padded to 32)] order
 * for the whole step (the order of the reference's unified sequence,
 * :1905-1907).  The noise refiners run on the image row range and the context
 * refiners on the caption row range of the same buffer (each with its own
 * attention), so no concatenation copy is needed.  Padding keys are masked in
 * the attention kernel (-1e9, :734-741).
 *
 * Per block: RMSNorm x (1 + scale) -> fused QKV GEMM with per-head RMSNorm +
 * 3-axis RoPE epilogue -> masked attention -> out-projection GEMM (f32) ->
 * x += tanh(gate) * RMSNorm(out) -> RMSNorm x (1 + scale) -> [w1 | w3] GEMM
 * with SiLU(w1 x) * (w3 x) epilogue -> w2 GEMM (f32) -> x += tanh(gate) *
 * RMSNorm(out).  Unmodulated (context refiner) blocks use scale 1, gate 1.
 * All modulation vectors of a step come from one GEMV.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "iris_internal.h"

#define ZI_MULTI 32
#define ZI_EPS 1e-5f

typedef struct {
    uint16_t *w_qkv, *w_out, *w13, *w2;
    float *qn, *kn, *n1, *n2, *fn1, *fn2;
    int mod_index; /* -1 = unmodulated */
    CUtensorMap tm_qkv, tm_out, tm13, tm2;
} zi_blk_t;

typedef struct {
    int valid;
    int lat_h, lat_w, cap_seq;
    int n_img, n_cap, ni, nc, S;
    float *hidden, *tmp, *lat_in, *out, *cap_f32, *tok_out;
    uint16_t *rope_pos;        /* [S][4] RoPE position ids (T, H, W; the 4th unused) */
    IrisRopeSpec *rope_spec;   /* per rotation pair: frequency and axis */
    uint16_t *xmod, *q, *k, *v, *attn, *mlp, *tok_img, *cap_bf16;
    uint8_t *mask;
    CUtensorMap tm_xmod, tm_attn, tm_mlp, tm_tok_img, tm_cap;
    cudaGraph_t graph;
    cudaGraphExec_t gexec;
    int graph_ok;
    uint64_t graph_kernels;
} zi_plan_t;

struct iris_cuda_zimage {
    iris_cuda_zimage_config_t cfg;
    int D, F, A, pf, NH;
    uint16_t *w_t0, *w_t2, *w_cap, *w_x, *w_mods, *w_fada, *w_final;
    float *b_t0, *b_t2, *cap_norm, *b_cap, *b_x, *x_pad, *cap_pad, *b_mods, *b_fada, *b_final, *zeros;
    CUtensorMap tm_cap, tm_x, tm_final;
    zi_blk_t *noise, *ctx, *layers;
    int n_mod;
    size_t weight_bytes;
    float *t_dev, *sincos, *temb_h, *temb, *mods, *fscale;
    zi_plan_t plan;
};

/* ------------------------------------------------------------------ load */
static uint16_t *zalloc_w(iris_cuda_zimage_t *z, size_t n) {
    uint16_t *p = (uint16_t *)iris_dmalloc(n * 2);
    if (p) z->weight_bytes += n * 2;
    return p;
}

static int zi_check_cfg(const iris_cuda_zimage_config_t *c) {
    if (c->dim % 256 || c->dim != c->heads * 128)
        return iris_fail(IRIS_CUDA_ERR_ARG, "dim must be heads*128 and a multiple of 256");
    if (c->axes_dims[0] + c->axes_dims[1] + c->axes_dims[2] != 128 || (c->axes_dims[0] & 1) ||
        (c->axes_dims[1] & 1) || (c->axes_dims[2] & 1))
        return iris_fail(IRIS_CUDA_ERR_ARG, "axes_dims must be even and sum to 128");
    if (c->ffn_dim % 128 || c->cap_feat_dim % 64 || c->adaln_dim % 8 || c->t_mid % 8)
        return iris_fail(IRIS_CUDA_ERR_ARG, "unsupported ffn/cap/adaln/t_mid width");
    if (c->patch_size * c->patch_size * c->in_channels > 128 ||
        (c->patch_size * c->patch_size * c->in_channels) % 64)
        return iris_fail(IRIS_CUDA_ERR_ARG, "patch features must be 64 or 128");
    return 0;
}

static int load_block(iris_cuda_zimage_t *z, iris_wsrc_t *ws, zi_blk_t *b, const char *prefix,
                      int modulated, uint16_t *tmp) {
    int D = z->D, F = z->F, rc = 0;
    char nm[256];
#define ZCHK(x) do { if ((rc = (x)) != 0) return rc; } while (0)
#define ZW(p, n) do { if (!((p) = zalloc_w(z, (n)))) return IRIS_CUDA_ERR_OOM; } while (0)
#define ZF(p, n) do { if (!((p) = (float *)iris_dmalloc((n) * 4))) return IRIS_CUDA_ERR_OOM; } while (0)
    ZW(b->w_qkv, (size_t)3 * D * D);
    ZW(b->w_out, (size_t)D * D);
    ZW(b->w13, (size_t)2 * F * D);
    ZW(b->w2, (size_t)D * F);
    ZF(b->qn, 128); ZF(b->kn, 128); ZF(b->n1, D); ZF(b->n2, D); ZF(b->fn1, D); ZF(b->fn2, D);
    static const char *qkv[3] = {"attention.to_q", "attention.to_k", "attention.to_v"};
    for (int j = 0; j < 3; j++) {
        snprintf(nm, sizeof(nm), "%s.%s.weight", prefix, qkv[j]);
        ZCHK(iris_wsrc_get(ws, nm, (size_t)D * D, b->w_qkv + (size_t)j * D * D));
    }
    snprintf(nm, sizeof(nm), "%s.attention.to_out.0.weight", prefix);
    ZCHK(iris_wsrc_get(ws, nm, (size_t)D * D, b->w_out));
    /* [w1 (gate); w3 (up)] -> interleaved 128-row blocks for the SwiGLU epilogue */
    snprintf(nm, sizeof(nm), "%s.feed_forward.w1.weight", prefix);
    ZCHK(iris_wsrc_get(ws, nm, (size_t)F * D, tmp));
    snprintf(nm, sizeof(nm), "%s.feed_forward.w3.weight", prefix);
    ZCHK(iris_wsrc_get(ws, nm, (size_t)F * D, tmp + (size_t)F * D));
    iris_count_launch(1);
    ZCHK(iris_cuda_check(iris_launch_interleave_gate_up(b->w13, tmp, F, D, g_rt.stream), nm));
    snprintf(nm, sizeof(nm), "%s.feed_forward.w2.weight", prefix);
    ZCHK(iris_wsrc_get(ws, nm, (size_t)D * F, b->w2));
    uint16_t *t2 = tmp + (size_t)2 * F * D; /* small-tensor slot after the FFN staging */
    struct { const char *n; float *dst; int len; } small[6] = {
        {"attention.norm_q", b->qn, 128}, {"attention.norm_k", b->kn, 128},
        {"attention_norm1", b->n1, D},    {"attention_norm2", b->n2, D},
        {"ffn_norm1", b->fn1, D},         {"ffn_norm2", b->fn2, D}};
    for (int j = 0; j < 6; j++) {
        snprintf(nm, sizeof(nm), "%s.%s.weight", prefix, small[j].n);
        ZCHK(iris_wsrc_get_f32(ws, nm, (size_t)small[j].len, small[j].dst, t2 + (size_t)j * D));
    }
    if (modulated) {
        int mi = b->mod_index;
        snprintf(nm, sizeof(nm), "%s.adaLN_modulation.0.weight", prefix);
        ZCHK(iris_wsrc_get(ws, nm, (size_t)4 * D * z->A, z->w_mods + (size_t)mi * 4 * D * z->A));
        snprintf(nm, sizeof(nm), "%s.adaLN_modulation.0.bias", prefix);
        ZCHK(iris_wsrc_get_f32(ws, nm, (size_t)4 * D, z->b_mods + (size_t)mi * 4 * D, t2 + (size_t)6 * D));
    }
    ZCHK(iris_mk_tmap(&b->tm_qkv, b->w_qkv, 3 * D, D, D, 256));
    ZCHK(iris_mk_tmap(&b->tm_out, b->w_out, D, D, D, 256));
    ZCHK(iris_mk_tmap(&b->tm13, b->w13, 2 * F, D, D, 256));
    ZCHK(iris_mk_tmap(&b->tm2, b->w2, D, F, F, 256));
    /* the staging slots are reused by the next block: finish these uploads */
    return iris_cuda_check(cudaStreamSynchronize(g_rt.stream), prefix);
#undef ZCHK
#undef ZW
#undef ZF
}

static void zi_plan_free(zi_plan_t *P);

void iris_cuda_zimage_free(iris_cuda_zimage_t *z) {
    if (!z) return;
    cudaStreamSynchronize(g_rt.stream);
    zi_plan_free(&z->plan);
    zi_blk_t *sets[3] = {z->noise, z->ctx, z->layers};
    int counts[3] = {z->cfg.n_refiner, z->cfg.n_refiner, z->cfg.n_layers};
    for (int s = 0; s < 3; s++) {
        if (!sets[s]) continue;
        for (int i = 0; i < counts[s]; i++) {
            zi_blk_t *b = &sets[s][i];
            iris_dfree(b->w_qkv); iris_dfree(b->w_out); iris_dfree(b->w13); iris_dfree(b->w2);
            iris_dfree(b->qn); iris_dfree(b->kn); iris_dfree(b->n1); iris_dfree(b->n2);
            iris_dfree(b->fn1); iris_dfree(b->fn2);
        }
        free(sets[s]);
    }
    uint16_t *ws[] = {z->w_t0, z->w_t2, z->w_cap, z->w_x, z->w_mods, z->w_fada, z->w_final};
    for (size_t i = 0; i < sizeof(ws) / sizeof(ws[0]); i++) iris_dfree(ws[i]);
    float *fs[] = {z->b_t0, z->b_t2, z->cap_norm, z->b_cap, z->b_x, z->x_pad, z->cap_pad, z->b_mods,
                   z->b_fada, z->b_final, z->zeros, z->t_dev, z->sincos, z->temb_h, z->temb, z->mods,
                   z->fscale};
    for (size_t i = 0; i < sizeof(fs) / sizeof(fs[0]); i++) iris_dfree(fs[i]);
    free(z);
}

static int load_all(iris_cuda_zimage_t *z, iris_wsrc_t *ws) {
    const int D = z->D, F = z->F, A = z->A, ps = z->cfg.patch_size, pf = z->pf;
    const int cap = z->cfg.cap_feat_dim, tm = z->cfg.t_mid;
    int rc = 0;
    char nm[256];
    size_t tmp_n = (size_t)2 * F * D + (size_t)8 * D + 4 * (size_t)D + (size_t)cap + 1024;
    uint16_t *tmp = (uint16_t *)iris_dmalloc(tmp_n * 2);
    if (!tmp) return IRIS_CUDA_ERR_OOM;
    uint16_t *t2 = tmp + (size_t)2 * F * D;
    z->n_mod = z->cfg.n_refiner + z->cfg.n_layers; /* modulated: noise refiners + main layers */
#define CHK(x) do { if ((rc = (x)) != 0) goto done; } while (0)
#define AW(p, n) do { if (!((p) = zalloc_w(z, (n)))) { rc = IRIS_CUDA_ERR_OOM; goto done; } } while (0)
#define AF(p, n) do { if (!((p) = (float *)iris_dmalloc((size_t)(n) * 4))) { rc = IRIS_CUDA_ERR_OOM; goto done; } } while (0)
    AW(z->w_t0, (size_t)tm * 256); AF(z->b_t0, tm);
    AW(z->w_t2, (size_t)A * tm); AF(z->b_t2, A);
    AW(z->w_cap, (size_t)D * cap); AF(z->b_cap, D); AF(z->cap_norm, cap);
    AW(z->w_x, (size_t)D * pf); AF(z->b_x, D);
    AF(z->x_pad, D); AF(z->cap_pad, D);
    AW(z->w_mods, (size_t)(z->n_mod > 0 ? z->n_mod : 1) * 4 * D * A);
    AF(z->b_mods, (size_t)(z->n_mod > 0 ? z->n_mod : 1) * 4 * D);
    AW(z->w_fada, (size_t)D * A); AF(z->b_fada, D);
    AW(z->w_final, (size_t)128 * D); AF(z->b_final, 128);
    AF(z->zeros, D);
    CHK(iris_cuda_check(cudaMemsetAsync(z->w_final, 0, (size_t)128 * D * 2, g_rt.stream), "final"));
    CHK(iris_cuda_check(cudaMemsetAsync(z->b_final, 0, 128 * 4, g_rt.stream), "final"));
    CHK(iris_cuda_check(cudaMemsetAsync(z->zeros, 0, (size_t)D * 4, g_rt.stream), "zeros"));

    CHK(iris_wsrc_get(ws, "t_embedder.mlp.0.weight", (size_t)tm * 256, z->w_t0));
    CHK(iris_wsrc_get_f32(ws, "t_embedder.mlp.0.bias", tm, z->b_t0, t2));
    CHK(iris_wsrc_get(ws, "t_embedder.mlp.2.weight", (size_t)A * tm, z->w_t2));
    CHK(iris_wsrc_get_f32(ws, "t_embedder.mlp.2.bias", A, z->b_t2, t2 + 1024));
    CHK(iris_wsrc_get_f32(ws, "cap_embedder.0.weight", cap, z->cap_norm, t2 + 2048));
    CHK(iris_wsrc_get(ws, "cap_embedder.1.weight", (size_t)D * cap, z->w_cap));
    CHK(iris_wsrc_get_f32(ws, "cap_embedder.1.bias", D, z->b_cap, t2 + 2048 + cap));
    snprintf(nm, sizeof(nm), "all_x_embedder.%d-1.weight", ps);
    CHK(iris_wsrc_get(ws, nm, (size_t)D * pf, z->w_x));
    snprintf(nm, sizeof(nm), "all_x_embedder.%d-1.bias", ps);
    CHK(iris_wsrc_get_f32(ws, nm, D, z->b_x, t2 + 2048 + cap + D));
    CHK(iris_wsrc_get_f32(ws, "x_pad_token", D, z->x_pad, t2 + 2048 + cap + 2 * D));
    CHK(iris_wsrc_get_f32(ws, "cap_pad_token", D, z->cap_pad, t2 + 2048 + cap + 3 * D));
    snprintf(nm, sizeof(nm), "all_final_layer.%d-1.adaLN_modulation.1.weight", ps);
    CHK(iris_wsrc_get(ws, nm, (size_t)D * A, z->w_fada));
    snprintf(nm, sizeof(nm), "all_final_layer.%d-1.adaLN_modulation.1.bias", ps);
    CHK(iris_wsrc_get_f32(ws, nm, D, z->b_fada, t2 + 2048 + cap + 4 * D));
    snprintf(nm, sizeof(nm), "all_final_layer.%d-1.linear.weight", ps);
    CHK(iris_wsrc_get(ws, nm, (size_t)pf * D, z->w_final));
    snprintf(nm, sizeof(nm), "all_final_layer.%d-1.linear.bias", ps);
    CHK(iris_wsrc_get_f32(ws, nm, pf, z->b_final, t2 + 2048 + cap + 5 * D));
    CHK(iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "embedders"));
    CHK(iris_mk_tmap(&z->tm_cap, z->w_cap, D, cap, cap, 256));
    CHK(iris_mk_tmap(&z->tm_x, z->w_x, D, pf, pf, 256));
    CHK(iris_mk_tmap(&z->tm_final, z->w_final, 128, D, D, 128));

    z->noise = (zi_blk_t *)calloc((size_t)(z->cfg.n_refiner > 0 ? z->cfg.n_refiner : 1), sizeof(zi_blk_t));
    z->ctx = (zi_blk_t *)calloc((size_t)(z->cfg.n_refiner > 0 ? z->cfg.n_refiner : 1), sizeof(zi_blk_t));
    z->layers = (zi_blk_t *)calloc((size_t)(z->cfg.n_layers > 0 ? z->cfg.n_layers : 1), sizeof(zi_blk_t));
    if (!z->noise || !z->ctx || !z->layers) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "block tables"); goto done; }
    {
        int mi = 0;
        for (int i = 0; i < z->cfg.n_refiner; i++) {
            snprintf(nm, sizeof(nm), "noise_refiner.%d", i);
            z->noise[i].mod_index = mi++;
            CHK(load_block(z, ws, &z->noise[i], nm, 1, tmp));
        }
        for (int i = 0; i < z->cfg.n_refiner; i++) {
            snprintf(nm, sizeof(nm), "context_refiner.%d", i);
            z->ctx[i].mod_index = -1;
            CHK(load_block(z, ws, &z->ctx[i], nm, 0, tmp));
        }
        for (int i = 0; i < z->cfg.n_layers; i++) {
            snprintf(nm, sizeof(nm), "layers.%d", i);
            z->layers[i].mod_index = mi++;
            CHK(load_block(z, ws, &z->layers[i], nm, 1, tmp));
        }
    }
    AF(z->t_dev, 4); AF(z->sincos, 256); AF(z->temb_h, tm); AF(z->temb, A);
    AF(z->mods, (size_t)(z->n_mod > 0 ? z->n_mod : 1) * 4 * D); AF(z->fscale, D);
#undef CHK
#undef AW
#undef AF
done:
    cudaStreamSynchronize(g_rt.stream);
    iris_dfree(tmp);
    return rc;
}

static iris_cuda_zimage_t *zi_new(const iris_cuda_zimage_config_t *cfg) {
    if (zi_check_cfg(cfg)) return NULL;
    iris_cuda_zimage_t *z = (iris_cuda_zimage_t *)calloc(1, sizeof(*z));
    if (!z) { iris_fail(IRIS_CUDA_ERR_OOM, "model struct"); return NULL; }
    z->cfg = *cfg;
    z->D = cfg->dim;
    z->F = cfg->ffn_dim;
    z->A = cfg->adaln_dim;
    z->NH = cfg->heads;
    z->pf = cfg->patch_size * cfg->patch_size * cfg->in_channels;
    return z;
}

/* config.json keys and defaults of the reference's Z-Image autodetection
 * (iris.c:300-330); ffn and t-MLP widths from the weight shapes (:2270-2290). */
static void zi_parse_config(const char *model_dir, const st_model_t *st, iris_cuda_zimage_config_t *c) {
    c->dim = 3840; c->n_layers = 30; c->n_refiner = 2; c->cap_feat_dim = 2560; c->in_channels = 16;
    c->patch_size = 2; c->rope_theta = 256.0f;
    c->axes_dims[0] = 32; c->axes_dims[1] = 48; c->axes_dims[2] = 48;
    char path[1200];
    snprintf(path, sizeof(path), "%s/transformer/config.json", model_dir);
    FILE *f = fopen(path, "rb");
    if (f) {
        char buf[8192];
        size_t n = fread(buf, 1, sizeof(buf) - 1, f);
        fclose(f);
        buf[n] = 0;
        double v;
        if (json_get_number(buf, "dim", &v) == 0 && v > 0) c->dim = (int)v;
        if (json_get_number(buf, "n_layers", &v) == 0 && v >= 0) c->n_layers = (int)v;
        if (json_get_number(buf, "n_refiner_layers", &v) == 0 && v >= 0) c->n_refiner = (int)v;
        if (json_get_number(buf, "cap_feat_dim", &v) == 0 && v > 0) c->cap_feat_dim = (int)v;
        if (json_get_number(buf, "in_channels", &v) == 0 && v > 0) c->in_channels = (int)v;
        if (json_get_number(buf, "patch_size", &v) == 0 && v > 0) c->patch_size = (int)v;
        if (json_get_number(buf, "rope_theta", &v) == 0 && v > 0) c->rope_theta = (float)v;
        const char *p = strstr(buf, "\"axes_dims\"");
        if (p && (p = strchr(p, '['))) {
            for (int i = 0; i < 3 && p; i++) {
                char *end;
                long a = strtol(p + 1, &end, 10);
                if (end == p + 1) break;
                c->axes_dims[i] = (int)a;
                p = strchr(end, ',');
            }
        }
    }
    c->heads = c->dim / 128;
    c->adaln_dim = c->dim < 256 ? c->dim : 256;
    c->ffn_dim = (8 * c->dim / 3 + 255) / 256 * 256;
    c->t_mid = 1024;
    const st_tensor_t *t = st_find(st, "layers.0.feed_forward.w1.weight");
    if (!t) t = st_find(st, "noise_refiner.0.feed_forward.w1.weight");
    if (t && t->ndim >= 1) c->ffn_dim = (int)t->shape[0];
    t = st_find(st, "t_embedder.mlp.0.weight");
    if (t && t->ndim >= 1) c->t_mid = (int)t->shape[0];
}

iris_cuda_zimage_t *iris_cuda_zimage_load(const char *model_dir) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    char tdir[1200];
    snprintf(tdir, sizeof(tdir), "%s/transformer", model_dir);
    if (st_open_dir(&ws.st, tdir) != 0) {
        iris_fail(IRIS_CUDA_ERR_IO, "cannot open safetensors in %s", tdir);
        return NULL;
    }
    iris_cuda_zimage_config_t cfg;
    zi_parse_config(model_dir, &ws.st, &cfg);
    iris_cuda_zimage_t *z = zi_new(&cfg);
    int rc = z ? load_all(z, &ws) : IRIS_CUDA_ERR_ARG;
    st_close(&ws.st);
    iris_wsrc_free(&ws);
    if (rc) { iris_cuda_zimage_free(z); return NULL; }
    return z;
}

iris_cuda_zimage_t *iris_cuda_zimage_random(const iris_cuda_zimage_config_t *cfg, uint64_t seed,
                                            float std, int norm_unit) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_cuda_zimage_t *z = zi_new(cfg);
    if (!z) return NULL;
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    ws.random = 1;
    ws.seed = seed;
    ws.std = std;
    ws.norm_unit = norm_unit;
    if (load_all(z, &ws)) { iris_cuda_zimage_free(z); return NULL; }
    return z;
}

int iris_cuda_zimage_get_config(const iris_cuda_zimage_t *z, iris_cuda_zimage_config_t *out) {
    if (!z || !out) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    *out = z->cfg;
    return 0;
}

size_t iris_cuda_zimage_weight_bytes(const iris_cuda_zimage_t *z) { return z ? z->weight_bytes : 0; }

/* ------------------------------------------------------------------ plan */
static void zi_plan_free(zi_plan_t *P) {
    if (P->graph_ok) {
        cudaGraphExecDestroy(P->gexec);
        cudaGraphDestroy(P->graph);
    }
    void *ps[] = {P->hidden, P->tmp, P->lat_in, P->out, P->cap_f32, P->rope_pos, P->rope_spec, P->tok_out,
                  P->xmod, P->q, P->k, P->v, P->attn, P->mlp, P->tok_img, P->cap_bf16, P->mask};
    for (size_t i = 0; i < sizeof(ps) / sizeof(ps[0]); i++) iris_dfree(ps[i]);
    memset(P, 0, sizeof(*P));
}

/* RoPE position ids per token -- image rows (cap_padded + 1, y, x), image
 * padding (0, 0, 0), caption rows (1 + s, 0, 0) -- and the per-pair spec,
 * freq = 1/theta^(2i/d) per axis (pairs of axis 0 first, then 1, then 2),
 * from which the QKV epilogue evaluates the rotation in registers.  A position
 * outside [0, 1024) is left unrotated by the reference, so it is stored as 0,
 * the identity (zi_precompute_rope :595, zi_apply_rope :620, position ids
 * :1832-1862). */
static void zi_fill_rope(const iris_cuda_zimage_t *z, const zi_plan_t *P, uint16_t *pos, IrisRopeSpec *spec,
                         uint8_t *mask) {
    const int *ax = z->cfg.axes_dims;
    const int wt = P->lat_w / z->cfg.patch_size;
    int pair = 0;
    memset(spec, 0, sizeof(*spec));
    for (int a = 0; a < 3; a++)
        for (int i = 0; i < ax[a] / 2; i++, pair++) {
            spec->freq[pair] = 1.0f / powf(z->cfg.rope_theta, (float)(2 * i) / (float)ax[a]);
            iris_rope_set_axis(spec, pair, a);
            spec->kscale[pair] = 1.0f;
        }
    for (int row = 0; row < P->S; row++) {
        int p3[3] = {0, 0, 0};
        int valid;
        if (row < P->ni) {
            valid = row < P->n_img;
            if (valid) { p3[0] = P->nc + 1; p3[1] = row / wt; p3[2] = row % wt; }
        } else {
            int s = row - P->ni;
            valid = s < P->n_cap;
            p3[0] = 1 + s;
        }
        mask[row] = (uint8_t)valid;
        uint16_t *p = pos + (size_t)row * 4;
        for (int a = 0; a < 3; a++) p[a] = (uint16_t)((p3[a] >= 0 && p3[a] < 1024) ? p3[a] : 0);
        p[3] = 0;
    }
}

static int zi_plan_ensure(iris_cuda_zimage_t *z, int lat_h, int lat_w, int cap_seq) {
    zi_plan_t *P = &z->plan;
    const int ps = z->cfg.patch_size;
    if (lat_h <= 0 || lat_w <= 0 || lat_h % ps || lat_w % ps || cap_seq <= 0)
        return iris_fail(IRIS_CUDA_ERR_ARG, "latent %dx%d must be a positive multiple of the patch size; "
                         "caption must be non-empty", lat_h, lat_w);
    if (P->valid && P->lat_h == lat_h && P->lat_w == lat_w && P->cap_seq == cap_seq) return 0;
    cudaStreamSynchronize(g_rt.stream);
    zi_plan_free(P);
    const int D = z->D, F = z->F, cap = z->cfg.cap_feat_dim, cin = z->cfg.in_channels;
    P->lat_h = lat_h; P->lat_w = lat_w; P->cap_seq = cap_seq;
    P->n_img = (lat_h / ps) * (lat_w / ps);
    P->n_cap = cap_seq;
    P->ni = P->n_img + (ZI_MULTI - P->n_img % ZI_MULTI) % ZI_MULTI;
    P->nc = P->n_cap + (ZI_MULTI - P->n_cap % ZI_MULTI) % ZI_MULTI;
    const int S = P->S = P->ni + P->nc;
    size_t sD = (size_t)S * D;
#define PA(p, bytes) do { if (!((p) = iris_dmalloc(bytes))) goto oom; } while (0)
    PA(P->hidden, sD * 4);
    PA(P->tmp, sD * 4);
    PA(P->lat_in, (size_t)cin * lat_h * lat_w * 4);
    PA(P->out, (size_t)cin * lat_h * lat_w * 4);
    PA(P->cap_f32, (size_t)P->nc * cap * 4);
    PA(P->rope_pos, (size_t)S * 4 * sizeof(uint16_t));
    PA(P->rope_spec, sizeof(IrisRopeSpec));
    PA(P->tok_out, (size_t)P->n_img * 128 * 4);
    PA(P->xmod, sD * 2);
    PA(P->q, sD * 2);
    PA(P->k, sD * 2);
    PA(P->v, sD * 2);
    PA(P->attn, sD * 2);
    PA(P->mlp, (size_t)S * F * 2);
    PA(P->tok_img, (size_t)P->ni * z->pf * 2);
    PA(P->cap_bf16, (size_t)P->nc * cap * 2);
    PA(P->mask, (size_t)S);
#undef PA
    /* padding rows of the embedder inputs stay zero (their embeddings are replaced by pad tokens) */
    cudaMemsetAsync(P->tok_img, 0, (size_t)P->ni * z->pf * 2, g_rt.stream);
    cudaMemsetAsync(P->cap_bf16, 0, (size_t)P->nc * cap * 2, g_rt.stream);
    if (iris_mk_tmap(&P->tm_xmod, P->xmod, S, D, D, 128) || iris_mk_tmap(&P->tm_attn, P->attn, S, D, D, 128) ||
        iris_mk_tmap(&P->tm_mlp, P->mlp, S, F, F, 128) ||
        iris_mk_tmap(&P->tm_tok_img, P->tok_img, P->ni, z->pf, z->pf, 128) ||
        iris_mk_tmap(&P->tm_cap, P->cap_bf16, P->nc, cap, cap, 128)) {
        zi_plan_free(P);
        return IRIS_CUDA_ERR_CUDA;
    }
    {
        uint16_t *pos = (uint16_t *)malloc((size_t)S * 4 * sizeof(uint16_t));
        uint8_t *mk = (uint8_t *)malloc((size_t)S);
        IrisRopeSpec spec;
        if (!pos || !mk) { free(pos); free(mk); goto oom; }
        zi_fill_rope(z, P, pos, &spec, mk);
        int rc = iris_h2d(P->rope_pos, pos, (size_t)S * 4 * sizeof(uint16_t)) ||
                 iris_h2d(P->rope_spec, &spec, sizeof(spec)) || iris_h2d(P->mask, mk, (size_t)S);
        free(pos); free(mk);
        if (rc) { zi_plan_free(P); return IRIS_CUDA_ERR_CUDA; }
    }
    P->valid = 1;
    return 0;
oom:
    zi_plan_free(P);
    return iris_fail(IRIS_CUDA_ERR_OOM, "Z-Image activation buffers for S=%d", S);
}

/* ------------------------------------------------------------------ forward */
typedef struct {
    int rc;
    uint64_t kernels;
} zenq_t;

static void zq(zenq_t *E, cudaError_t e, const char *what) {
    E->kernels++;
    if (!E->rc && e != cudaSuccess) E->rc = iris_cuda_check(e, what);
}

static void zgemm(zenq_t *E, const CUtensorMap *ta, const CUtensorMap *tb, int row0, int rows, int N,
                  int K, int mode, IrisGemmParams *p, const char *what) {
    p->tmap_a = *ta;
    p->tmap_b[0] = *tb;
    p->ngroups = 1;
    p->row0[0] = row0;
    p->rows[0] = rows;
    p->N = N;
    p->K = K;
    p->mode = mode;
    if (!p->bn) p->bn = 256;
    p->status = g_rt.d_status;
    p->b_static = 1;  /* B: a resident weight */
    zq(E, iris_launch_gemm(p, g_rt.num_sms, g_rt.stream), what);
}

/* one block on hidden rows [r0, r0 + len) */
static void zi_enq_block(iris_cuda_zimage_t *z, const zi_blk_t *b, int r0, int len, int masked, zenq_t *E) {
    zi_plan_t *P = &z->plan;
    cudaStream_t st = g_rt.stream;
    const int D = z->D, F = z->F;
    const float *mod = b->mod_index >= 0 ? z->mods + (size_t)b->mod_index * 4 * D : NULL;
    IrisGemmParams gp;
    float *hid = P->hidden + (size_t)r0 * D;
    zq(E, iris_launch_rmsnorm(hid, D, b->n1, NULL, P->xmod + (size_t)r0 * D, D, len, D, ZI_EPS,
                              mod ? mod : NULL, st), "zi_norm1");
    memset(&gp, 0, sizeof(gp));
    gp.qnorm[0] = b->qn; gp.knorm[0] = b->kn;
    gp.rope_pos = P->rope_pos; gp.rope_spec = P->rope_spec;
    gp.q = P->q; gp.k = P->k; gp.v = P->v; gp.ldqkv = D; gp.H = D; gp.eps = ZI_EPS;
    zgemm(E, &P->tm_xmod, &b->tm_qkv, r0, len, 3 * D, D, IRIS_EPI_QKV, &gp, "zi_qkv");
    size_t o = (size_t)r0 * D;
    zq(E, iris_launch_attention(P->q + o, D, P->k + o, P->v + o, D, P->attn + o, D, len, len, z->NH,
                                1.0f / sqrtf(128.0f), masked ? P->mask + r0 : NULL, st), "zi_attn");
    memset(&gp, 0, sizeof(gp));
    gp.out = P->tmp; gp.ldo = D;
    zgemm(E, &P->tm_attn, &b->tm_out, r0, len, D, D, IRIS_EPI_F32, &gp, "zi_out");
    zq(E, iris_launch_resid_rmsnorm_gate(hid, D, P->tmp + o, D, b->n2, mod ? mod + D : NULL, len, D, ZI_EPS, st),
       "zi_resid1");
    zq(E, iris_launch_rmsnorm(hid, D, b->fn1, NULL, P->xmod + o, D, len, D, ZI_EPS, mod ? mod + 2 * D : NULL, st),
       "zi_norm2");
    memset(&gp, 0, sizeof(gp));
    gp.mlp_out = P->mlp; gp.ld_mlp = F; gp.mlp_col0 = 0; gp.swiglu_base = 0;
    zgemm(E, &P->tm_xmod, &b->tm13, r0, len, 2 * F, D, IRIS_EPI_SWIGLU, &gp, "zi_w13");
    memset(&gp, 0, sizeof(gp));
    gp.out = P->tmp; gp.ldo = D;
    zgemm(E, &P->tm_mlp, &b->tm2, r0, len, D, F, IRIS_EPI_F32, &gp, "zi_w2");
    zq(E, iris_launch_resid_rmsnorm_gate(hid, D, P->tmp + o, D, b->fn2, mod ? mod + 3 * D : NULL, len, D, ZI_EPS, st),
       "zi_resid2");
}

static int zi_enqueue_forward(iris_cuda_zimage_t *z, zenq_t *E) {
    zi_plan_t *P = &z->plan;
    cudaStream_t st = g_rt.stream;
    const int D = z->D, A = z->A, tm = z->cfg.t_mid, cap = z->cfg.cap_feat_dim, ps = z->cfg.patch_size;
    IrisGemmParams gp;
    /* timestep embedding, all block modulations (1 + scale, tanh gate) and the final scale */
    zq(E, iris_launch_timestep_sincos(z->t_dev, 1000.0f, z->sincos, 256, st), "zi_sincos");
    zq(E, iris_launch_gemv(z->w_t0, z->sincos, z->b_t0, z->temb_h, tm, 256, 0, 1, st), "zi_t0");
    zq(E, iris_launch_gemv(z->w_t2, z->temb_h, z->b_t2, z->temb, A, tm, 0, 0, st), "zi_t2");
    if (z->n_mod > 0) {
        zq(E, iris_launch_gemv(z->w_mods, z->temb, z->b_mods, z->mods, z->n_mod * 4 * D, A, 0, 0, st), "zi_mods");
        zq(E, iris_launch_zi_mod_transform(z->mods, D, (long)z->n_mod * 4 * D, st), "zi_mod_tf");
    }
    zq(E, iris_launch_gemv(z->w_fada, z->temb, z->b_fada, z->fscale, D, A, 1, 0, st), "zi_fscale");
    /* embedders: patch tokens and caption features, padding rows -> pad tokens */
    zq(E, iris_launch_patchify(P->lat_in, z->cfg.in_channels, P->lat_h, P->lat_w, ps, P->tok_img, z->pf, st),
       "zi_patchify");
    memset(&gp, 0, sizeof(gp));
    gp.out = P->hidden; gp.ldo = D; gp.bias = z->b_x;
    zgemm(E, &P->tm_tok_img, &z->tm_x, 0, P->ni, D, z->pf, IRIS_EPI_F32, &gp, "zi_x_emb");
    zq(E, iris_launch_fill_rows_f32(P->hidden + (size_t)P->n_img * D, D, z->x_pad, P->ni - P->n_img, D, st),
       "zi_x_pad");
    zq(E, iris_launch_rmsnorm(P->cap_f32, cap, z->cap_norm, NULL, P->cap_bf16, cap, P->n_cap, cap, ZI_EPS, NULL, st),
       "zi_cap_norm");
    memset(&gp, 0, sizeof(gp));
    gp.out = P->hidden + (size_t)P->ni * D; gp.ldo = D; gp.bias = z->b_cap;
    zgemm(E, &P->tm_cap, &z->tm_cap, 0, P->nc, D, cap, IRIS_EPI_F32, &gp, "zi_cap_emb");
    zq(E, iris_launch_fill_rows_f32(P->hidden + (size_t)(P->ni + P->n_cap) * D, D, z->cap_pad,
                                    P->nc - P->n_cap, D, st), "zi_cap_pad");
    /* refiners on their own row ranges, then the main layers over the whole sequence */
    int img_masked = P->ni != P->n_img, cap_masked = P->nc != P->n_cap;
    for (int i = 0; i < z->cfg.n_refiner; i++) zi_enq_block(z, &z->noise[i], 0, P->ni, img_masked, E);
    for (int i = 0; i < z->cfg.n_refiner; i++) zi_enq_block(z, &z->ctx[i], P->ni, P->nc, cap_masked, E);
    for (int i = 0; i < z->cfg.n_layers; i++)
        zi_enq_block(z, &z->layers[i], 0, P->S, img_masked || cap_masked, E);
    /* final layer on the real image rows: LayerNorm (eps 1e-6) x (1 + scale), linear + bias */
    zq(E, iris_launch_adaln(P->hidden, D, P->xmod, D, P->n_img, D, z->zeros, z->fscale, NULL, NULL,
                            P->n_img, 1e-6f, st), "zi_final_norm");
    memset(&gp, 0, sizeof(gp));
    gp.out = P->tok_out; gp.ldo = 128; gp.bias = z->b_final; gp.bn = 128;
    zgemm(E, &P->tm_xmod, &z->tm_final, 0, P->n_img, 128, D, IRIS_EPI_F32, &gp, "zi_final");
    zq(E, iris_launch_unpatchify(P->tok_out, 128, z->cfg.in_channels, P->lat_h, P->lat_w, ps, P->out, st),
       "zi_unpatchify");
    return E->rc;
}

static int zi_run_forward(iris_cuda_zimage_t *z) {
    zi_plan_t *P = &z->plan;
    if (iris_fault("launch")) return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected launch failure");
    if (!P->graph_ok) {
        zenq_t E = {0, 0};
        cudaError_t e = cudaStreamBeginCapture(g_rt.stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return iris_cuda_check(e, "begin capture");
        int rc = zi_enqueue_forward(z, &E);
        cudaGraph_t g = NULL;
        e = cudaStreamEndCapture(g_rt.stream, &g);
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        if (e != cudaSuccess) return iris_cuda_check(e, "end capture");
        e = cudaGraphInstantiate(&P->gexec, g, 0);
        if (e != cudaSuccess) { cudaGraphDestroy(g); return iris_cuda_check(e, "graph instantiate"); }
        P->graph = g;
        P->graph_ok = 1;
        P->graph_kernels = E.kernels;
    }
    iris_count_launch(P->graph_kernels);
    return iris_cuda_check(cudaGraphLaunch(P->gexec, g_rt.stream), "graph launch");
}

static int zi_inputs(iris_cuda_zimage_t *z, const float *lat, int h, int w, const float *cap, int cap_seq,
                     enum cudaMemcpyKind kind) {
    int rc = zi_plan_ensure(z, h, w, cap_seq);
    if (rc) return rc;
    zi_plan_t *P = &z->plan;
    if (lat && lat != P->lat_in &&
        (rc = iris_cuda_check(cudaMemcpyAsync(P->lat_in, lat, (size_t)z->cfg.in_channels * h * w * 4, kind,
                                              g_rt.stream), "latent")))
        return rc;
    if (cap && (rc = iris_cuda_check(cudaMemcpyAsync(P->cap_f32, cap, (size_t)cap_seq * z->cfg.cap_feat_dim * 4,
                                                     kind, g_rt.stream), "caption")))
        return rc;
    return 0;
}

float *iris_cuda_zi_transformer_forward(iris_cuda_zimage_t *z, const float *latent, int latent_h,
                                        int latent_w, float timestep, const float *cap_feats, int cap_seq) {
    if (!z || !latent || !cap_feats) { iris_fail(IRIS_CUDA_ERR_ARG, "null argument"); return NULL; }
    int rc = zi_inputs(z, latent, latent_h, latent_w, cap_feats, cap_seq, cudaMemcpyHostToDevice);
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(z->t_dev, &timestep, 4, cudaMemcpyHostToDevice, g_rt.stream), "t");
    if (!rc) rc = zi_run_forward(z);
    size_t n = (size_t)z->cfg.in_channels * latent_h * latent_w;
    float *out = rc ? NULL : (float *)malloc(n * 4);
    if (!rc && !out) rc = iris_fail(IRIS_CUDA_ERR_OOM, "output");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, z->plan.out, n * 4, cudaMemcpyDeviceToHost, g_rt.stream), "out");
    if (!rc) rc = iris_cuda_synchronize();
    if (rc) { free(out); return NULL; }
    return out;
}

/* Euler loop on resident buffers: t = 1 - sigma, z += (s_{n+1} - s_n) * (-v)
 * (iris_sample_euler_zimage, iris_sample.c:412-480). */
static int zi_euler_core(iris_cuda_zimage_t *z, const float *schedule, int steps) {
    zi_plan_t *P = &z->plan;
    size_t n = (size_t)z->cfg.in_channels * P->lat_h * P->lat_w;
    float *ts = (float *)malloc((size_t)steps * sizeof(float));
    if (!ts) return iris_fail(IRIS_CUDA_ERR_OOM, "timesteps");
    for (int s = 0; s < steps; s++) ts[s] = 1.0f - schedule[s];
    float *d_ts = (float *)iris_dmalloc((size_t)steps * 4);
    int rc = d_ts ? 0 : IRIS_CUDA_ERR_OOM;
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(d_ts, ts, (size_t)steps * 4, cudaMemcpyHostToDevice, g_rt.stream), "t");
    for (int s = 0; s < steps && !rc; s++) {
        rc = iris_cuda_check(cudaMemcpyAsync(z->t_dev, d_ts + s, 4, cudaMemcpyDeviceToDevice, g_rt.stream), "t");
        if (!rc) rc = zi_run_forward(z);
        if (!rc) {
            iris_count_launch(1);
            rc = iris_cuda_check(iris_launch_euler(P->lat_in, P->out, NULL, 1.0f, -(schedule[s + 1] - schedule[s]),
                                                   (long)n, g_rt.stream), "euler");
        }
    }
    cudaStreamSynchronize(g_rt.stream);
    iris_dfree(d_ts);
    free(ts);
    return rc;
}

float *iris_cuda_sample_euler_zimage(iris_cuda_zimage_t *z, const float *zin, int batch, int channels, int h,
                                     int w, int patch_size, const float *cap_feats, int cap_seq,
                                     const float *schedule, int num_steps, void (*progress_callback)(int, int)) {
    (void)progress_callback;
    if (!z || !zin || !cap_feats || !schedule) { iris_fail(IRIS_CUDA_ERR_ARG, "null argument"); return NULL; }
    if (batch != 1 || channels != z->cfg.in_channels || patch_size != z->cfg.patch_size || num_steps <= 0) {
        iris_fail(IRIS_CUDA_ERR_ARG, "batch 1, the model's channels and patch size, steps > 0 required");
        return NULL;
    }
    int rc = zi_inputs(z, zin, h, w, cap_feats, cap_seq, cudaMemcpyHostToDevice);
    if (!rc) rc = zi_euler_core(z, schedule, num_steps);
    size_t n = (size_t)channels * h * w;
    float *out = rc ? NULL : (float *)malloc(n * 4);
    if (!rc && !out) rc = iris_fail(IRIS_CUDA_ERR_OOM, "output");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, z->plan.lat_in, n * 4, cudaMemcpyDeviceToHost, g_rt.stream), "z");
    if (!rc) rc = iris_cuda_synchronize();
    if (rc) { free(out); return NULL; }
    return out;
}

int iris_cuda_sample_euler_zimage_dev(iris_cuda_zimage_t *z, float *d_z, int h, int w, const float *d_cap,
                                      int cap_seq, const float *schedule, int num_steps) {
    if (!z || !d_z || !d_cap || !schedule || num_steps <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "bad argument");
    int rc = zi_inputs(z, d_z, h, w, d_cap, cap_seq, cudaMemcpyDeviceToDevice);
    if (!rc) rc = zi_euler_core(z, schedule, num_steps);
    if (rc) return rc;
    return iris_cuda_check(cudaMemcpyAsync(d_z, z->plan.lat_in, (size_t)z->cfg.in_channels * h * w * 4,
                                           cudaMemcpyDeviceToDevice, g_rt.stream), "z");
}
