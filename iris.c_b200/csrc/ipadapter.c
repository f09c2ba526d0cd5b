/*
 * IP-Adapter for the Flux transformer on the GPU.
 *
 * Reference: iris_ip_adapter.c (bundle loader :113, perceive :331, get_kv :366,
 * inject :386, schedule :401-433), iris_load_ip_adapter / iris_set_ip_schedule /
 * iris_unload_ip_adapter (iris.c:520-640), the hooks in the blocks
 * (iris_transformer_flux.c:2355-2365, :2440-2446, :2607-2612, :3848-3855,
 * :3921-3926) and the samplers' per-step iris_transformer_set_ip_step
 * (iris_sample.c:351, :751).
 *
 * Attach time (once per conditioning image, f32 like the reference): the
 * bundle's weights are dequantised (bf16 / f16 / f32, int8 rows times their
 * scale) and uploaded, the perceiver (SigLIP cross-attention, CSD FiLM, or the
 * hybrid of both) turns the features into ip_embeds [T, H], and every adapted
 * block's k = ip_embeds @ Wk[b], v = ip_embeds @ Wv[b] (hybrid: V groups gated)
 * is computed and kept in bf16 [2][nb][T][H] (20 MB for Klein-4B, T = 64).  The
 * reference recomputes k / v inside every block of every step; here they are
 * constants of the attachment.
 *
 * Per step and block (flux.c): the block's post-RoPE image Q is rotated back
 * to the pre-RoPE Q the adapter was trained on (ip_kernels.cu), attends to the
 * block's T adapter tokens on the tcgen05 attention kernel, and the result,
 * times ip_scale[block] * schedule multiplier (a device array, so a schedule
 * changes no graph), is added to the image rows of the hidden state after the
 * block.  Tensor parallelism is not supported with an adapter.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "flux_internal.h"

/* ------------------------------------------------------------ meta.json */
/* the reference's cfg_find_value / cfg_int / cfg_bool (iris_config_parse.h) */
static const char *meta_value(const char *json, const char *key) {
    char q[128];
    size_t kl = strlen(key);
    if (kl + 3 >= sizeof(q)) return NULL;
    snprintf(q, sizeof(q), "\"%s\"", key);
    const char *p = strstr(json, q);
    if (!p) return NULL;
    p = strchr(p + kl + 2, ':');
    return p ? p + 1 : NULL;
}
static int meta_int(const char *json, const char *key, int dflt) {
    const char *v = meta_value(json, key);
    return v ? atoi(v) : dflt;
}
static int meta_bool(const char *json, const char *key, int dflt) {
    const char *v = meta_value(json, key);
    if (!v) return dflt;
    while (*v == ' ' || *v == '\t' || *v == '\n' || *v == '\r') v++;
    if (!strncmp(v, "true", 4)) return 1;
    if (!strncmp(v, "false", 5)) return 0;
    return dflt;
}
static void meta_str(const char *json, const char *key, char *out, size_t cap) {
    const char *c = meta_value(json, key);
    if (!c) return;
    while (*c == ' ' || *c == '"') c++;
    snprintf(out, cap, "%s", c);
    char *e = strchr(out, '"');
    if (e) *e = 0;
}

/* ------------------------------------------------------------ tensors */
/* f32 copy of a bundle tensor on the device (NULL when absent or malformed);
 * int8 tensors are dequantised with "<name>.scale", one entry per row
 * (load_tensor_f32, iris_ip_adapter.c:80) */
static float *dev_tensor(iris_wsrc_t *ws, const char *name, size_t *numel_out) {
    const st_model_t *st = &ws->st;
    const st_tensor_t *t = st_find(st, name);
    if (!t) return NULL;
    size_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= (size_t)t->shape[i];
    if (t->dtype == ST_BF16 && t->nbytes == n * 2) {
        /* the bulk of a bundle: the pipelined file upload, widened to f32 on the device */
        float *d = (float *)iris_dmalloc(n * sizeof(float));
        uint16_t *tmp = (uint16_t *)iris_dmalloc(n * 2);
        int rc = (!d || !tmp) ? IRIS_CUDA_ERR_OOM : iris_wsrc_get(ws, name, n, tmp);
        if (!rc) rc = iris_cuda_check(iris_launch_bf16_to_f32(tmp, d, (long)n, g_rt.stream), name);
        if (!rc) rc = iris_stream_drain();
        iris_dfree(tmp);
        if (rc) { iris_dfree(d); return NULL; }
        if (numel_out) *numel_out = n;
        return d;
    }
    float *h = (float *)malloc(n * sizeof(float) + 4);
    if (!h) return NULL;
    int ok = 0;
    if (t->dtype == ST_I8) {
        char sname[320];
        snprintf(sname, sizeof(sname), "%s.scale", name);
        const st_tensor_t *ts = st_find(st, sname);
        const int8_t *q = (const int8_t *)st_raw(st, t);
        size_t cols = t->ndim > 0 ? (size_t)t->shape[t->ndim - 1] : n;
        size_t rows = cols ? n / cols : 0;
        size_t sn = 1;
        if (ts) for (int i = 0; i < ts->ndim; i++) sn *= (size_t)ts->shape[i];
        float *sc = ts && sn == rows && t->nbytes == n ? (float *)malloc(rows * sizeof(float) + 4) : NULL;
        if (sc && q && st_read_f32(st, ts, sc, rows) == 0) {
            for (size_t r = 0; r < rows; r++)
                for (size_t c = 0; c < cols; c++) h[r * cols + c] = (float)q[r * cols + c] * sc[r];
            ok = 1;
        }
        free(sc);
    } else {
        ok = st_read_f32(st, t, h, n) == 0;
    }
    float *d = NULL;
    if (ok && (d = (float *)iris_dmalloc(n * sizeof(float))) && iris_h2d(d, h, n * sizeof(float))) {
        iris_dfree(d);
        d = NULL;
    }
    free(h);
    if (d && numel_out) *numel_out = n;
    return d;
}

typedef struct {
    int nb, nd, ns, H, T, S, pheads, csd_dim, style_only;
    char mode[16], quant[16];
    float *qtok, *nw, *nbias, *fw, *fb, *wq, *wk, *wv, *wo, *in_g, *in_b;  /* perceiver / csd */
    float *cq, *cfw, *cfb, *cnw, *cnb, *gate;                              /* hybrid csd half */
    float *ipk, *ipv, *ipscale;                                            /* stacked per block */
} ip_bundle_t;

static void bundle_free(ip_bundle_t *b) {
    float *ps[] = {b->qtok, b->nw, b->nbias, b->fw, b->fb, b->wq, b->wk, b->wv, b->wo, b->in_g, b->in_b,
                   b->cq, b->cfw, b->cfb, b->cnw, b->cnb, b->gate, b->ipk, b->ipv, b->ipscale};
    for (size_t i = 0; i < sizeof(ps) / sizeof(ps[0]); i++) iris_dfree(ps[i]);
    memset(b, 0, sizeof(*b));
}

static int bundle_load(ip_bundle_t *b, const char *dir) {
    memset(b, 0, sizeof(*b));
    char path[1200], meta[4096];
    snprintf(path, sizeof(path), "%s/adapter_meta.json", dir);
    FILE *f = fopen(path, "rb");
    if (!f) return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: cannot open %s", path);
    size_t mn = fread(meta, 1, sizeof(meta) - 1, f);
    fclose(f);
    meta[mn] = 0;
    b->nb = meta_int(meta, "num_blocks", 0);
    b->nd = meta_int(meta, "num_double_blocks", 0);
    b->ns = meta_int(meta, "num_single_blocks", 0);
    b->H = meta_int(meta, "hidden_dim", 0);
    b->T = meta_int(meta, "num_image_tokens", 0);
    b->S = meta_int(meta, "siglip_dim", 0);
    b->pheads = meta_int(meta, "perceiver_heads", 0);
    b->style_only = meta_bool(meta, "style_only", 0);
    snprintf(b->mode, sizeof(b->mode), "siglip");
    meta_str(meta, "cond_mode", b->mode, sizeof(b->mode));
    b->csd_dim = meta_int(meta, "csd_dim", 768);
    meta_str(meta, "quant", b->quant, sizeof(b->quant));
    if (b->H <= 0 || b->nb <= 0 || b->T <= 0) return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: bad meta in %s", dir);
    if (b->pheads <= 0 || b->H % b->pheads) b->pheads = b->H / 128;  /* legacy bundles */
    const int csd = !strcmp(b->mode, "csd"), hybrid = !strcmp(b->mode, "hybrid");
    if (!csd && !hybrid && strcmp(b->mode, "siglip"))
        return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: unknown cond_mode %s", b->mode);
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    snprintf(path, sizeof(path), "%s/adapter_weights.safetensors", dir);
    if (st_open_file(&ws.st, path)) return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: cannot open %s", path);
    iris_wsrc_t *st = &ws;
    b->qtok = dev_tensor(st, "perceiver.query_tokens", NULL);
    b->nw = dev_tensor(st, "perceiver.norm_weight", NULL);
    b->nbias = dev_tensor(st, "perceiver.norm_bias", NULL);
    if (csd) {
        b->fw = dev_tensor(st, "perceiver.film_weight", NULL);
        b->fb = dev_tensor(st, "perceiver.film_bias", NULL);
    } else {
        b->wq = dev_tensor(st, "perceiver.query_proj", NULL);
        b->wk = dev_tensor(st, "perceiver.key_proj", NULL);
        b->wv = dev_tensor(st, "perceiver.value_proj", NULL);
        b->wo = dev_tensor(st, "perceiver.out_proj", NULL);
        b->in_g = dev_tensor(st, "perceiver.in_gamma", NULL);
        b->in_b = dev_tensor(st, "perceiver.in_beta", NULL);
    }
    if (hybrid) {
        b->cq = dev_tensor(st, "csd.query_tokens", NULL);
        b->cfw = dev_tensor(st, "csd.film_weight", NULL);
        b->cfb = dev_tensor(st, "csd.film_bias", NULL);
        b->cnw = dev_tensor(st, "csd.norm_weight", NULL);
        b->cnb = dev_tensor(st, "csd.norm_bias", NULL);
        b->gate = dev_tensor(st, "group_gate", NULL);
    }
    size_t nk = 0, nv = 0, ns = 0;
    b->ipk = dev_tensor(st, "ip_k_stacked", &nk);
    b->ipv = dev_tensor(st, "ip_v_stacked", &nv);
    b->ipscale = dev_tensor(&ws, "ip_scale", &ns);
    iris_wsrc_free(&ws);
    st_close(&ws.st);
    int ok = b->qtok && b->nw && b->nbias && b->ipk && b->ipv && b->ipscale;
    ok = ok && (csd ? (b->fw && b->fb) : (b->wq && b->wk && b->wv && b->wo));
    if (hybrid) ok = ok && b->cq && b->cfw && b->cfb && b->cnw && b->cnb;
    const size_t HH = (size_t)b->H * b->H;
    ok = ok && nk == (size_t)b->nb * HH && nv == nk && ns == (size_t)b->nb;
    if (!ok) {
        bundle_free(b);
        return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: missing or malformed tensors in %s", dir);
    }
    return 0;
}

/* ------------------------------------------------------------ perceive */
#define ICK(x) do { if ((rc = iris_cuda_check((x), "IP-Adapter"))) goto out; } while (0)

/* FiLM: out[T, H] = LayerNorm(qtok * (1 + scale) + shift), [scale; shift] = fw csd + fb */
static int csd_film(const ip_bundle_t *b, const float *d_csd, int T, const float *qtok, const float *fw,
                    const float *fb, const float *nw, const float *nbias, float *out) {
    int rc = 0;
    const int H = b->H;
    cudaStream_t st = g_rt.stream;
    float *film = (float *)iris_dmalloc((size_t)2 * H * sizeof(float));
    if (!film) return IRIS_CUDA_ERR_OOM;
    ICK(iris_launch_ip_sgemm(d_csd, b->csd_dim, fw, b->csd_dim, 1, fb, film, 2 * H, 1, 2 * H, b->csd_dim, st));
    ICK(iris_launch_ip_film_tokens(qtok, film, T, H, out, st));
    ICK(iris_launch_ip_layernorm(out, T, H, nw, nbias, st));
    iris_count_launch(3);
out:
    iris_stream_drain();
    iris_dfree(film);
    return rc;
}

/* SigLIP PerceiverResampler over n feature rows -> out[T, H] */
static int siglip_perceive(const ip_bundle_t *b, const float *d_feat, int n, int T, float *out) {
    int rc = 0;
    const int H = b->H, S = b->S;
    cudaStream_t st = g_rt.stream;
    float *xin = (float *)iris_dmalloc((size_t)n * S * sizeof(float));
    float *Q = (float *)iris_dmalloc((size_t)T * H * sizeof(float));
    float *K = (float *)iris_dmalloc((size_t)n * H * sizeof(float));
    float *V = (float *)iris_dmalloc((size_t)n * H * sizeof(float));
    float *att = (float *)iris_dmalloc((size_t)T * H * sizeof(float));
    if (!xin || !Q || !K || !V || !att) { rc = IRIS_CUDA_ERR_OOM; goto out; }
    const float *x = d_feat;
    if (b->in_g && b->in_b) {
        ICK(iris_launch_ip_colnorm(d_feat, n, S, b->in_g, b->in_b, xin, st));
        x = xin;
    }
    ICK(iris_launch_ip_sgemm(b->qtok, H, b->wq, H, 1, NULL, Q, H, T, H, H, st));
    ICK(iris_launch_ip_sgemm(x, S, b->wk, S, 1, NULL, K, H, n, H, S, st));
    ICK(iris_launch_ip_sgemm(x, S, b->wv, S, 1, NULL, V, H, n, H, S, st));
    ICK(iris_launch_ip_mha(Q, K, V, T, n, H, b->pheads, att, st));
    ICK(iris_launch_ip_sgemm(att, H, b->wo, H, 1, NULL, out, H, T, H, H, st));
    ICK(iris_launch_ip_layernorm(out, T, H, b->nw, b->nbias, st));
    iris_count_launch(7);
out:
    iris_stream_drain();
    iris_dfree(xin); iris_dfree(Q); iris_dfree(K); iris_dfree(V); iris_dfree(att);
    return rc;
}

/* iris_ip_adapter_perceive (:331): features as iris_load_ip_adapter reads them
 * (siglip [n, S]; csd one [csd_dim] vector; hybrid [n, S] with the CSD vector,
 * zero-padded, as the last row) -> embeds [T, H] */
static int perceive(const ip_bundle_t *b, const float *d_feat, int n, float *embeds) {
    if (!strcmp(b->mode, "csd")) return csd_film(b, d_feat, b->T, b->qtok, b->fw, b->fb, b->nw, b->nbias, embeds);
    if (!strcmp(b->mode, "hybrid")) {
        const int half = b->T / 2;
        if (n < 2) return iris_fail(IRIS_CUDA_ERR_ARG, "IP-Adapter: hybrid features need SigLIP rows + CSD row");
        int rc = siglip_perceive(b, d_feat, n - 1, half, embeds);
        if (!rc) rc = csd_film(b, d_feat + (size_t)(n - 1) * b->S, half, b->cq, b->cfw, b->cfb, b->cnw, b->cnb,
                               embeds + (size_t)half * b->H);
        return rc;
    }
    return siglip_perceive(b, d_feat, n, b->T, embeds);
}

/* ------------------------------------------------------------ state */
void iris_flux_ip_release(iris_cuda_flux_t *tf) {
    if (!tf || !tf->ip) return;
    iris_stream_drain();
    struct iris_flux_ip *ip = tf->ip;
    iris_dfree(ip->kv);
    iris_dfree(ip->d_scale);
    iris_dfree(ip->embeds);
    free(ip->h_scale);
    free(ip->h_cur);
    free(ip);
    tf->ip = NULL;
}

static int upload_scales(struct iris_flux_ip *ip) {
    for (int b = 0; b < ip->nb; b++) ip->h_cur[b] = ip->h_scale[b] * ip->mult;
    return iris_h2d(ip->d_scale, ip->h_cur, (size_t)ip->nb * sizeof(float));
}

int iris_cuda_flux_load_ip_adapter_mem(iris_cuda_flux_t *tf, const char *bundle_dir, const float *features,
                                       int n_rows, float scale_mult) {
    if (!tf || !bundle_dir || !features || n_rows <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (tf->tp > 1) return iris_fail(IRIS_CUDA_ERR_ARG, "IP-Adapter with tensor parallelism is not supported");
    ip_bundle_t b;
    int rc = bundle_load(&b, bundle_dir);
    if (rc) return rc;
    float *feat = NULL, *emb = NULL, *kf = NULL, *vf = NULL;
    struct iris_flux_ip *ip = NULL;
    const int H = b.H, T = b.T;
    if (H != tf->H || b.nb != tf->cfg.n_double + tf->cfg.n_single || b.nd != tf->cfg.n_double) {
        rc = iris_fail(IRIS_CUDA_ERR_ARG, "IP-Adapter: bundle mismatch (hidden %d vs %d, blocks %d+%d vs %d+%d)", H,
                       tf->H, b.nd, b.nb - b.nd, tf->cfg.n_double, tf->cfg.n_single);
        goto out;
    }
    const int csd = !strcmp(b.mode, "csd");
    const int row = csd ? b.csd_dim : b.S;
    if (row <= 0) { rc = iris_fail(IRIS_CUDA_ERR_ARG, "IP-Adapter: feature width 0"); goto out; }
    if (csd && n_rows != 1)
        fprintf(stderr, "iris_cuda IP-Adapter: CSD features have %d vectors; using the first.\n", n_rows);
    const int n = csd ? 1 : n_rows;
    feat = (float *)iris_dmalloc((size_t)n * row * sizeof(float));
    emb = (float *)iris_dmalloc((size_t)T * H * sizeof(float));
    kf = (float *)iris_dmalloc((size_t)b.nb * T * H * sizeof(float));
    vf = (float *)iris_dmalloc((size_t)b.nb * T * H * sizeof(float));
    ip = (struct iris_flux_ip *)calloc(1, sizeof(*ip));
    if (!feat || !emb || !kf || !vf || !ip) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "IP-Adapter"); goto out; }
    if ((rc = iris_h2d(feat, features, (size_t)n * row * sizeof(float)))) goto out;
    if ((rc = perceive(&b, feat, n, emb))) goto out;
    ip->nb = b.nb;
    ip->nd = b.nd;
    ip->T = T;
    ip->mult = 1.0f;
    ip->kv = (uint16_t *)iris_dmalloc((size_t)b.nb * 2 * T * H * 2);
    ip->d_scale = (float *)iris_dmalloc((size_t)b.nb * sizeof(float));
    ip->h_scale = (float *)malloc((size_t)b.nb * sizeof(float));
    ip->h_cur = (float *)malloc((size_t)b.nb * sizeof(float));
    float *hg = b.gate ? (float *)malloc((size_t)b.nb * 2 * sizeof(float)) : NULL;
    if (!ip->kv || !ip->d_scale || !ip->h_scale || !ip->h_cur || (b.gate && !hg)) {
        free(hg);
        rc = iris_fail(IRIS_CUDA_ERR_OOM, "IP-Adapter");
        goto out;
    }
    rc = iris_cuda_check(cudaMemcpyAsync(ip->h_scale, b.ipscale, (size_t)b.nb * sizeof(float),
                                         cudaMemcpyDeviceToHost, g_rt.stream), "IP scale");
    if (!rc && hg)
        rc = iris_cuda_check(cudaMemcpyAsync(hg, b.gate, (size_t)b.nb * 2 * sizeof(float), cudaMemcpyDeviceToHost,
                                             g_rt.stream), "IP gate");
    if (!rc) rc = iris_stream_drain();
    for (int i = 0; i < b.nb; i++) ip->h_scale[i] *= scale_mult;
    /* every block at once: k[b] = embeds @ Wk[b], v[b] = embeds @ Wv[b] (einsum btd,de->te,
       iris_ip_adapter.c:366), f32, then the hybrid gate on V and bf16 [2][nb][T][H] */
    const long THl = (long)T * H, HHl = (long)H * H;
    if (!rc) rc = iris_cuda_check(iris_launch_ip_sgemm_batched(emb, H, 0, b.ipk, H, HHl, 0, NULL, kf, H, THl, T, H, H,
                                                               b.nb, g_rt.stream), "k");
    if (!rc) rc = iris_cuda_check(iris_launch_ip_sgemm_batched(emb, H, 0, b.ipv, H, HHl, 0, NULL, vf, H, THl, T, H, H,
                                                               b.nb, g_rt.stream), "v");
    for (int i = 0; !rc && hg && i < b.nb; i++)
        rc = iris_cuda_check(iris_launch_ip_scale_rows(vf + (size_t)i * THl, T, H, T / 2, hg[2 * i], hg[2 * i + 1],
                                                       g_rt.stream), "gate");
    if (!rc) rc = iris_cuda_check(iris_launch_f32_to_bf16(kf, ip->kv, (long)b.nb * THl, g_rt.stream), "k bf16");
    if (!rc) rc = iris_cuda_check(iris_launch_f32_to_bf16(vf, ip->kv + (size_t)b.nb * THl, (long)b.nb * THl,
                                                          g_rt.stream), "v bf16");
    iris_count_launch(4 + (hg ? b.nb : 0));
    free(hg);
    if (!rc) rc = upload_scales(ip);
    if (rc) goto out;
    /* replace any adapter attached before; plans are rebuilt with the hooks */
    iris_flux_ip_release(tf);
    ip->embeds = emb;
    emb = NULL;
    tf->ip = ip;
    ip = NULL;
    iris_flux_invalidate_plan(tf);
out:
    iris_stream_drain();
    if (ip) {
        iris_dfree(ip->kv); iris_dfree(ip->d_scale);
        free(ip->h_scale); free(ip->h_cur); free(ip);
    }
    iris_dfree(feat); iris_dfree(emb); iris_dfree(kf); iris_dfree(vf);
    bundle_free(&b);
    return rc;
}

int iris_cuda_flux_load_ip_adapter(iris_cuda_flux_t *tf, const char *bundle_dir, const char *features_path,
                                   float scale_mult) {
    if (!tf || !bundle_dir || !features_path) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    /* the row width the features file is cut into: the meta's csd_dim or siglip_dim */
    char path[1200], meta[4096];
    snprintf(path, sizeof(path), "%s/adapter_meta.json", bundle_dir);
    FILE *f = fopen(path, "rb");
    if (!f) return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: cannot open %s", path);
    size_t mn = fread(meta, 1, sizeof(meta) - 1, f);
    fclose(f);
    meta[mn] = 0;
    char mode[16] = "siglip";
    meta_str(meta, "cond_mode", mode, sizeof(mode));
    const int row = !strcmp(mode, "csd") ? meta_int(meta, "csd_dim", 768) : meta_int(meta, "siglip_dim", 0);
    f = fopen(features_path, "rb");
    if (!f) return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: cannot open features file %s", features_path);
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    if (row <= 0 || sz <= 0 || sz % ((long)row * 4)) {
        fclose(f);
        return iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: features size %ld is not a multiple of %d f32 rows", sz, row);
    }
    float *h = (float *)malloc((size_t)sz);
    size_t got = h ? fread(h, 1, (size_t)sz, f) : 0;
    fclose(f);
    int rc = got == (size_t)sz ? iris_cuda_flux_load_ip_adapter_mem(tf, bundle_dir, h, (int)(sz / (row * 4)), scale_mult)
                               : iris_fail(IRIS_CUDA_ERR_IO, "IP-Adapter: failed to read features");
    free(h);
    return rc;
}

int iris_cuda_flux_unload_ip_adapter(iris_cuda_flux_t *tf) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!tf->ip) return 0;
    iris_flux_ip_release(tf);
    iris_flux_invalidate_plan(tf);
    return 0;
}

int iris_cuda_flux_set_ip_schedule(iris_cuda_flux_t *tf, const char *spec) {
    if (!tf || !tf->ip) return iris_fail(IRIS_CUDA_ERR_ARG, "no IP-Adapter attached");
    struct iris_flux_ip *ip = tf->ip;
    /* iris_ip_adapter_set_schedule (:401): reset first, so a bad spec leaves "none" */
    ip->sched_kind = 0;
    ip->sched_param = 0.0f;
    ip->mult = 1.0f;
    int rc = 0;
    if (spec && *spec && strcmp(spec, "none")) {
        float fr = 0.0f;
        if (sscanf(spec, "late:%f", &fr) == 1) ip->sched_kind = 1;
        else if (sscanf(spec, "early:%f", &fr) == 1) ip->sched_kind = 2;
        else rc = iris_fail(IRIS_CUDA_ERR_ARG, "ip-schedule: bad spec '%s' (want none|late:F|early:F)", spec);
        if (!rc && (!isfinite(fr) || fr < 0.0f || fr > 1.0f)) {
            ip->sched_kind = 0;
            rc = iris_fail(IRIS_CUDA_ERR_ARG, "ip-schedule: fraction %.3f out of [0,1]", (double)fr);
        }
        if (!rc) ip->sched_param = fr;
    }
    int rc2 = upload_scales(ip);
    return rc ? rc : rc2;
}

int iris_cuda_flux_set_ip_step(iris_cuda_flux_t *tf, int step, int num_steps) {
    if (!tf || !tf->ip) return 0;
    struct iris_flux_ip *ip = tf->ip;
    float m = 1.0f;
    if (ip->sched_kind && num_steps > 0) {
        /* step fraction 0 at the first (noisiest) step, 1 at the last (:424) */
        float frac = num_steps > 1 ? (float)step / (float)(num_steps - 1) : 1.0f;
        m = ip->sched_kind == 1 ? (frac >= ip->sched_param ? 1.0f : 0.0f) : (frac < ip->sched_param ? 1.0f : 0.0f);
    }
    if (m == ip->mult) return 0;
    ip->mult = m;
    return upload_scales(ip);
}

int iris_cuda_flux_ip_embeds(const iris_cuda_flux_t *tf, float *out, int cap) {
    if (!tf || !tf->ip || !out) return iris_fail(IRIS_CUDA_ERR_ARG, "no IP-Adapter attached");
    const int n = tf->ip->T * tf->H;
    if (cap < n) return iris_fail(IRIS_CUDA_ERR_ARG, "buffer too small (%d < %d)", cap, n);
    int rc = iris_cuda_check(cudaMemcpyAsync(out, tf->ip->embeds, (size_t)n * 4, cudaMemcpyDeviceToHost, g_rt.stream),
                             "ip embeds");
    if (!rc) rc = iris_stream_drain();
    return rc ? rc : n;
}
