/*
 * Autoencoder decoder on the GPU: latent -> RGB image, the step after the
 * denoising loop.  Replaces iris_vae_decode (iris_vae.c:835-990) and its
 * loader iris_vae_load_safetensors_ex (iris_vae.c:1227-1385).
 *
 * Layout: every activation is NHWC (pixel rows of channels).  The residual
 * stream between resnet blocks stays f32; the inputs of the convolutions
 * (GroupNorm + SiLU outputs, the upsampled tensor, the shortcut input) are
 * bf16.  Convolutions run as implicit GEMMs (vae.cu) with their bias, the
 * residual add and the 1x1 shortcut convolution fused; the mid-block
 * attention (one head of 512 channels over the H*W latent pixels) runs as
 * tensor-core GEMMs around an f32 row softmax.  One decode of a given size
 * is captured once into a CUDA graph and replayed.
 */
#include "iris_internal.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define VAE_BASE 128
#define VAE_MID 512
#define VAE_GN_BLOCKS 592            /* GroupNorm statistics-pass blocks (max) */
#define VAE_GN_SLOTS 1024            /* GroupNorm partial slots: >= SMs and >= VAE_GN_BLOCKS */
#define VAE_MAX_MID_PIXELS 65536     /* 2x2-unpatchified latent pixels (4 MP images) */

static const int k_mult[4] = {1, 2, 4, 4};  /* iris_vae.c:1236 */

typedef struct {
    uint16_t *w;     /* bf16 [cout_pad, k] */
    float *b;        /* [cout_pad] (conv bias + shortcut bias) */
    CUtensorMap tm;      /* weight boxes of min(bn, 128) rows */
    CUtensorMap tm64;    /* weight boxes of 64 rows (CTA-pair tiles of N = 128) */
    int taps0, cin0, cin1, cout, cout_pad, bn, k;
    int cin_real;    /* segment-0 channels before padding to 64 */
} vconv_t;

typedef struct {
    float *g, *b;
} vgn_t;

typedef struct {
    int cin, cout;
    vgn_t n1, n2;
    vconv_t c1, c2;  /* c2 carries the 1x1 shortcut as its second K segment */
} vres_t;

typedef struct {
    int valid, lh, lw;
    int H[4], W[4];  /* level l: H[3] = 2 lh (after unpatchify), H[l - 1] = 2 H[l] */
    int P3p;         /* mid-level pixels rounded up to 128 (attention GEMM extents) */
    float *lat;
    uint16_t *xin;
    float *X, *T;
    uint16_t *Hb, *Xb;
    uint16_t *hA, *qk, *vT, *Pm, *O;
    float *S;
    double *part;    /* GroupNorm partial sums of the last convolution (or stats pass) */
    int gn_nparts;   /* slots in part */
    float *ab;       /* per-channel GroupNorm affine [2 * 512] */
    float *rgb;
    uint8_t *rgb8;
    cudaGraph_t graph;
    cudaGraphExec_t gexec;
    int graph_ok;
    uint64_t graph_kernels;
} vplan_t;

struct iris_cuda_vae {
    int z, lat_ch;
    float eps, scaling, shift;
    float *bn_mean, *bn_std, *pq_w, *pq_b;
    vconv_t conv_in, upc[3], conv_out;
    vres_t mid[2], up[12];
    vgn_t attn_gn, out_gn;
    uint16_t *w_qk, *w_v, *w_o;
    float *b_qk, *b_v, *b_o, *ones;
    vplan_t plan;
    size_t weight_bytes;
    void *allocs[256];
    int nallocs;
};

/* ------------------------------------------------------------------ loading */
static void *vae_alloc(iris_cuda_vae_t *v, size_t bytes) {
    if (v->nallocs >= (int)(sizeof(v->allocs) / sizeof(v->allocs[0]))) return NULL;
    void *p = iris_dmalloc(bytes);
    if (p) v->allocs[v->nallocs++] = p;
    return p;
}

static void *vae_upload(iris_cuda_vae_t *v, const void *host, size_t bytes) {
    void *d = vae_alloc(v, bytes);
    if (!d) return NULL;
    if (iris_h2d(d, host, bytes)) return NULL;
    v->weight_bytes += bytes;
    return d;
}

/* Where the weights come from: a safetensors file, or (st == NULL) a seeded
 * host RNG for benchmarks: convolution / projection weights N(0, 1/fan_in),
 * norm scales 1 + N(0, 0.1), biases N(0, 0.02), latent statistics mean
 * N(0, 0.5) and variance 1 + |N(0, 0.2)|. */
typedef struct {
    const st_model_t *st;
    uint64_t seed;
} vsrc_t;

static uint64_t splitmix(uint64_t *x) {
    uint64_t z = (*x += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static float rand_normal(uint64_t *x) {  /* Box-Muller on two 24-bit uniforms */
    const float u1 = ((float)(splitmix(x) >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)(splitmix(x) >> 40) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
}

static int ends_with(const char *s, const char *suf) {
    size_t a = strlen(s), b = strlen(suf);
    return a >= b && strcmp(s + a - b, suf) == 0;
}

/* f32 host copy of tensor `name` with `numel` elements (NULL if absent or
 * mis-sized); fan_in scales random projection weights */
static float *read_host(const vsrc_t *src, const char *name, size_t numel, int fan_in) {
    if (src->st) {
        const st_tensor_t *t = st_find(src->st, name);
        if (!t) return NULL;
        float *h = (float *)malloc(numel * sizeof(float));
        if (!h) return NULL;
        if (st_read_f32(src->st, t, h, numel)) { free(h); return NULL; }
        return h;
    }
    float *h = (float *)malloc(numel * sizeof(float));
    if (!h) return NULL;
    uint64_t x = src->seed * 0x2545F4914F6CDD1Dull ^ (uint64_t)iris_crc32(name);
    const int is_bias = ends_with(name, ".bias");
    const int is_norm = !is_bias && (strstr(name, "norm") != NULL);
    for (size_t i = 0; i < numel; i++) {
        const float g = rand_normal(&x);
        if (strcmp(name, "bn.running_mean") == 0) h[i] = 0.5f * g;
        else if (strcmp(name, "bn.running_var") == 0) h[i] = 1.0f + fabsf(0.2f * g);
        else if (is_bias) h[i] = 0.02f * g;
        else if (is_norm) h[i] = 1.0f + 0.1f * g;
        else h[i] = g / sqrtf((float)(fan_in > 0 ? fan_in : 1));
    }
    return h;
}

static int has_tensor(const vsrc_t *src, const char *name) { return src->st ? st_find(src->st, name) != NULL : 1; }

static int missing(const char *name) { return iris_fail(IRIS_CUDA_ERR_IO, "VAE tensor %s missing or mis-sized", name); }

static int load_vec(iris_cuda_vae_t *v, const vsrc_t *st, const char *name, int n, int fan_in, float **dst) {
    float *h = read_host(st, name, (size_t)n, fan_in);
    if (!h) return missing(name);
    *dst = (float *)vae_upload(v, h, (size_t)n * 4);
    free(h);
    return *dst ? 0 : iris_fail(IRIS_CUDA_ERR_OOM, "VAE upload");
}

static int load_gn(iris_cuda_vae_t *v, const vsrc_t *st, const char *prefix, int c, vgn_t *gn) {
    char n[300];
    snprintf(n, sizeof(n), "%s.weight", prefix);
    int rc = load_vec(v, st, n, c, 0, &gn->g);
    snprintf(n, sizeof(n), "%s.bias", prefix);
    return rc ? rc : load_vec(v, st, n, c, 0, &gn->b);
}

/* Convolution `prefix` (OIHW [cout, cin, k, k], k = 3 if taps == 9 else 1)
 * repacked as the GEMM operand [cout_pad, taps * cin_pad (+ skip_cin)]
 * with K ordered (tap, channel); an optional 1x1 shortcut `skip` ([cout,
 * skip_cin]) appended as extra K columns, its bias added to the conv bias. */
static int load_conv(iris_cuda_vae_t *v, const vsrc_t *st, const char *prefix, int cin, int cin_pad, int cout,
                     int taps, const char *skip, int skip_cin, int bn, vconv_t *cv) {
    char n[300];
    const int cout_pad = (cout + bn - 1) / bn * bn;
    const int k = taps * cin_pad + (skip ? skip_cin : 0);
    snprintf(n, sizeof(n), "%s.weight", prefix);
    float *w = read_host(st, n, (size_t)cout * cin * taps, cin * taps);
    if (!w) return missing(n);
    snprintf(n, sizeof(n), "%s.bias", prefix);
    float *b = read_host(st, n, (size_t)cout, 0);
    if (!b) { free(w); return missing(n); }
    float *ws = NULL, *bs = NULL;
    if (skip) {
        snprintf(n, sizeof(n), "%s.weight", skip);
        ws = read_host(st, n, (size_t)cout * skip_cin, skip_cin);
        snprintf(n, sizeof(n), "%s.bias", skip);
        bs = read_host(st, n, (size_t)cout, 0);
        if (!ws || !bs) { free(w); free(b); free(ws); free(bs); return missing(n); }
    }
    uint16_t *m = (uint16_t *)calloc((size_t)cout_pad * k, sizeof(uint16_t));
    float *bias = (float *)calloc((size_t)cout_pad, sizeof(float));
    int rc = 0;
    if (!m || !bias) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE weight staging");
    for (int o = 0; !rc && o < cout; o++) {
        for (int c = 0; c < cin; c++)
            for (int t = 0; t < taps; t++)  /* OIHW: weight[o][c][ky][kx], t = ky * 3 + kx */
                m[(size_t)o * k + (size_t)t * cin_pad + c] = f32_to_bf16_bits(w[((size_t)o * cin + c) * taps + t]);
        if (skip)
            for (int c = 0; c < skip_cin; c++)
                m[(size_t)o * k + (size_t)taps * cin_pad + c] = f32_to_bf16_bits(ws[(size_t)o * skip_cin + c]);
        bias[o] = b[o] + (skip ? bs[o] : 0.0f);
    }
    if (!rc) {
        cv->w = (uint16_t *)vae_upload(v, m, (size_t)cout_pad * k * 2);
        cv->b = (float *)vae_upload(v, bias, (size_t)cout_pad * 4);
        if (!cv->w || !cv->b) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE upload");
    }
    if (!rc && (iris_make_tmap_bf16(&cv->tm, cv->w, (uint64_t)cout_pad, (uint64_t)k, (uint64_t)k,
                                    (uint32_t)(bn < 128 ? bn : 128)) ||
                iris_make_tmap_bf16(&cv->tm64, cv->w, (uint64_t)cout_pad, (uint64_t)k, (uint64_t)k, 64)))
        rc = iris_fail(IRIS_CUDA_ERR_CUDA, "VAE weight tensor map");
    cv->taps0 = taps;
    cv->cin_real = cin;
    cv->cin0 = cin_pad;
    cv->cin1 = skip ? skip_cin : 0;
    cv->cout = cout;
    cv->cout_pad = cout_pad;
    cv->bn = bn;
    cv->k = k;
    free(w); free(b); free(ws); free(bs); free(m); free(bias);
    return rc;
}

static int conv_bn(int cout) { return cout >= 256 ? 256 : cout >= 128 ? 128 : 16; }

static int load_res(iris_cuda_vae_t *v, const vsrc_t *st, const char *prefix, int cin, int cout, vres_t *r) {
    char n[300], n2[300];
    r->cin = cin;
    r->cout = cout;
    int rc;
    snprintf(n, sizeof(n), "%s.norm1", prefix);
    if ((rc = load_gn(v, st, n, cin, &r->n1))) return rc;
    snprintf(n, sizeof(n), "%s.norm2", prefix);
    if ((rc = load_gn(v, st, n, cout, &r->n2))) return rc;
    snprintf(n, sizeof(n), "%s.conv1", prefix);
    if ((rc = load_conv(v, st, n, cin, cin, cout, 9, NULL, 0, conv_bn(cout), &r->c1))) return rc;
    snprintf(n, sizeof(n), "%s.conv2", prefix);
    snprintf(n2, sizeof(n2), "%s.conv_shortcut", prefix);
    return load_conv(v, st, n, cout, cout, cout, 9, cin != cout ? n2 : NULL, cin, conv_bn(cout), &r->c2);
}

/* [c, c] (or [c, c, 1, 1]) projections of the mid-block attention */
static int load_attn(iris_cuda_vae_t *v, const vsrc_t *st, const char *prefix) {
    const int c = VAE_MID;
    char n[300];
    const char *names[4] = {"to_q", "to_k", "to_v", "to_out.0"};
    float *w[4] = {0}, *b[4] = {0};
    int rc = 0;
    for (int i = 0; i < 4 && !rc; i++) {
        snprintf(n, sizeof(n), "%s.%s.weight", prefix, names[i]);
        if (!(w[i] = read_host(st, n, (size_t)c * c, c))) rc = missing(n);
        snprintf(n, sizeof(n), "%s.%s.bias", prefix, names[i]);
        if (!rc && !(b[i] = read_host(st, n, (size_t)c, 0))) rc = missing(n);
    }
    uint16_t *m = rc ? NULL : (uint16_t *)malloc((size_t)2 * c * c * 2);
    float *bb = rc ? NULL : (float *)malloc((size_t)2 * c * 4);
    float *ones = rc ? NULL : (float *)malloc((size_t)c * 4);
    if (!rc && (!m || !bb || !ones)) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE staging");
    if (!rc) {
        for (size_t i = 0; i < (size_t)c * c; i++) {
            m[i] = f32_to_bf16_bits(w[0][i]);
            m[(size_t)c * c + i] = f32_to_bf16_bits(w[1][i]);
        }
        memcpy(bb, b[0], (size_t)c * 4);
        memcpy(bb + c, b[1], (size_t)c * 4);
        v->w_qk = (uint16_t *)vae_upload(v, m, (size_t)2 * c * c * 2);
        v->b_qk = (float *)vae_upload(v, bb, (size_t)2 * c * 4);
        for (size_t i = 0; i < (size_t)c * c; i++) m[i] = f32_to_bf16_bits(w[2][i]);
        v->w_v = (uint16_t *)vae_upload(v, m, (size_t)c * c * 2);
        v->b_v = (float *)vae_upload(v, b[2], (size_t)c * 4);
        for (size_t i = 0; i < (size_t)c * c; i++) m[i] = f32_to_bf16_bits(w[3][i]);
        v->w_o = (uint16_t *)vae_upload(v, m, (size_t)c * c * 2);
        v->b_o = (float *)vae_upload(v, b[3], (size_t)c * 4);
        for (int i = 0; i < c; i++) ones[i] = 1.0f;
        v->ones = (float *)vae_upload(v, ones, (size_t)c * 4);
        if (!v->w_qk || !v->b_qk || !v->w_v || !v->b_v || !v->w_o || !v->b_o || !v->ones)
            rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE upload");
    }
    for (int i = 0; i < 4; i++) { free(w[i]); free(b[i]); }
    free(m); free(bb); free(ones);
    return rc;
}

static int vae_load_all(iris_cuda_vae_t *v, const vsrc_t *st) {
    int rc;
    char n[300];
    const int z = v->z;
    if (!v->scaling) {  /* Flux: batch-norm statistics -> (mean, sqrt(var + eps)) */
        float *mean = read_host(st, "bn.running_mean", (size_t)v->lat_ch, 0);
        float *var = read_host(st, "bn.running_var", (size_t)v->lat_ch, 0);
        float *sd = (float *)malloc((size_t)v->lat_ch * 4);
        rc = 0;
        if (!sd) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE staging");
        /* no statistics in the file: identity (iris_vae.c:1367-1374) */
        for (int i = 0; !rc && i < v->lat_ch; i++) sd[i] = sqrtf((var ? var[i] : 1.0f) + v->eps);
        if (!rc && !mean) {
            mean = (float *)calloc((size_t)v->lat_ch, 4);
            if (!mean) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE staging");
        }
        if (!rc) {
            v->bn_mean = (float *)vae_upload(v, mean, (size_t)v->lat_ch * 4);
            v->bn_std = (float *)vae_upload(v, sd, (size_t)v->lat_ch * 4);
            if (!v->bn_mean || !v->bn_std) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE upload");
        }
        free(mean); free(var); free(sd);
        if (rc) return rc;
    }
    /* present in Flux files only; the random source follows the Flux layout when scaling == 0 */
    if (st->st ? has_tensor(st, "post_quant_conv.weight") : !v->scaling) {
        if ((rc = load_vec(v, st, "post_quant_conv.weight", z * z, z, &v->pq_w))) return rc;
        if ((rc = load_vec(v, st, "post_quant_conv.bias", z, 0, &v->pq_b))) return rc;
    }
    if ((rc = load_conv(v, st, "decoder.conv_in", z, 64, VAE_MID, 9, NULL, 0, 256, &v->conv_in))) return rc;
    if ((rc = load_res(v, st, "decoder.mid_block.resnets.0", VAE_MID, VAE_MID, &v->mid[0]))) return rc;
    if ((rc = load_gn(v, st, "decoder.mid_block.attentions.0.group_norm", VAE_MID, &v->attn_gn))) return rc;
    if ((rc = load_attn(v, st, "decoder.mid_block.attentions.0"))) return rc;
    if ((rc = load_res(v, st, "decoder.mid_block.resnets.1", VAE_MID, VAE_MID, &v->mid[1]))) return rc;
    int bi = 0;
    for (int level = 3; level >= 0; level--) {  /* iris_vae.c:1318-1329 */
        const int ch = VAE_BASE * k_mult[level];
        const int prev = level == 3 ? VAE_MID : VAE_BASE * k_mult[level + 1];
        for (int r = 0; r < 3; r++) {
            snprintf(n, sizeof(n), "decoder.up_blocks.%d.resnets.%d", 3 - level, r);
            if ((rc = load_res(v, st, n, r == 0 ? prev : ch, ch, &v->up[bi++]))) return rc;
        }
    }
    for (int i = 0; i < 3; i++) {
        const int ch = VAE_BASE * k_mult[3 - i];
        snprintf(n, sizeof(n), "decoder.up_blocks.%d.upsamplers.0.conv", i);
        if ((rc = load_conv(v, st, n, ch, ch, ch, 9, NULL, 0, conv_bn(ch), &v->upc[i]))) return rc;
    }
    if ((rc = load_gn(v, st, "decoder.conv_norm_out", VAE_BASE, &v->out_gn))) return rc;
    return load_conv(v, st, "decoder.conv_out", VAE_BASE, VAE_BASE, 3, 9, NULL, 0, 16, &v->conv_out);
}

static void plan_free(vplan_t *P) {
    if (P->graph_ok) {
        cudaGraphExecDestroy(P->gexec);
        cudaGraphDestroy(P->graph);
    }
    void *bufs[] = {P->lat, P->xin, P->X, P->T, P->Hb, P->Xb, P->hA, P->qk, P->vT, P->Pm, P->O,
                    P->S, P->part, P->ab, P->rgb, P->rgb8};
    for (size_t i = 0; i < sizeof(bufs) / sizeof(bufs[0]); i++) iris_dfree(bufs[i]);
    memset(P, 0, sizeof(*P));
}

void iris_cuda_vae_free(iris_cuda_vae_t *v) {
    if (!v) return;
    if (g_rt.initialized) cudaStreamSynchronize(g_rt.stream);
    plan_free(&v->plan);
    for (int i = 0; i < v->nallocs; i++) iris_dfree(v->allocs[i]);
    free(v);
}

static iris_cuda_vae_t *vae_create(const vsrc_t *src, int z, float scaling, float shift) {
    iris_cuda_vae_t *v = (iris_cuda_vae_t *)calloc(1, sizeof(*v));
    if (!v) { iris_fail(IRIS_CUDA_ERR_OOM, "VAE struct"); return NULL; }
    v->z = z;
    v->lat_ch = 4 * z;
    v->scaling = scaling;
    v->shift = shift;
    v->eps = scaling != 0.0f ? 1e-6f : 1e-4f;  /* iris_vae.c:1245 */
    if (vae_load_all(v, src)) { iris_cuda_vae_free(v); return NULL; }
    return v;
}

iris_cuda_vae_t *iris_cuda_vae_load(const char *vae_dir, int z_channels, float scaling, float shift) {
    if (!vae_dir) { iris_fail(IRIS_CUDA_ERR_ARG, "null VAE directory"); return NULL; }
    if (iris_rt_ensure()) return NULL;
    /* config.json overrides, as iris_parse_vae_config (iris_vae_config.h) does */
    int z = z_channels > 0 ? z_channels : 32;
    char path[4200];
    snprintf(path, sizeof(path), "%s/config.json", vae_dir);
    FILE *f = fopen(path, "rb");
    if (f && z_channels <= 0) {
        char buf[8192];
        size_t got = fread(buf, 1, sizeof(buf) - 1, f);
        buf[got] = 0;
        double d;
        if (!json_get_number(buf, "latent_channels", &d) && d > 0) z = (int)d;
        if (!json_get_number(buf, "scaling_factor", &d)) scaling = (float)d;
        if (!json_get_number(buf, "shift_factor", &d)) shift = (float)d;
    }
    if (f) fclose(f);
    if (z < 1 || z > 32) { iris_fail(IRIS_CUDA_ERR_ARG, "latent channels %d (1..32 supported)", z); return NULL; }
    st_model_t st;
    if (st_open_dir(&st, vae_dir)) { iris_fail(IRIS_CUDA_ERR_IO, "cannot open VAE weights in %s", vae_dir); return NULL; }
    vsrc_t src = {&st, 0};
    iris_cuda_vae_t *v = vae_create(&src, z, scaling, shift);
    st_close(&st);
    return v;
}

iris_cuda_vae_t *iris_cuda_vae_random(int z_channels, float scaling, float shift, uint64_t seed) {
    if (iris_rt_ensure()) return NULL;
    if (z_channels < 1 || z_channels > 32) {
        iris_fail(IRIS_CUDA_ERR_ARG, "latent channels %d (1..32 supported)", z_channels);
        return NULL;
    }
    vsrc_t src = {NULL, seed};
    return vae_create(&src, z_channels, scaling, shift);
}

size_t iris_cuda_vae_weight_bytes(const iris_cuda_vae_t *v) { return v ? v->weight_bytes : 0; }

/* ------------------------------------------------------------------ plan */
static int plan_ensure(iris_cuda_vae_t *v, int lh, int lw) {
    vplan_t *P = &v->plan;
    if (P->valid && P->lh == lh && P->lw == lw) return 0;
    plan_free(P);
    P->lh = lh;
    P->lw = lw;
    P->H[3] = 2 * lh;
    P->W[3] = 2 * lw;
    for (int l = 2; l >= 0; l--) {
        P->H[l] = 2 * P->H[l + 1];
        P->W[l] = 2 * P->W[l + 1];
    }
    const size_t p3 = (size_t)P->H[3] * P->W[3], p0 = (size_t)P->H[0] * P->W[0];
    P->P3p = (int)((p3 + 127) / 128 * 128);
    const size_t p3p = (size_t)P->P3p;
    /* largest activation of each buffer over the levels (channels 512/512/256/128) */
    const size_t x_elems = p0 * 256;           /* upsampled conv output entering level 0 */
    const size_t t_elems = p0 * 128;           /* conv1 outputs: P_l * cout_l <= P0 * 128 */
    const size_t hb_elems = p0 * 256;          /* GroupNorm outputs / upsampled input */
    const size_t xb_elems = p0 * 256;          /* shortcut inputs (bf16 copy of a block input) */
    int rc = 0;
#define ALLOC(dst, bytes) \
    do { if (!rc && !((dst) = iris_dmalloc(bytes))) rc = iris_fail(IRIS_CUDA_ERR_OOM, "VAE plan (%zu bytes)", (size_t)(bytes)); } while (0)
    ALLOC(P->lat, (size_t)v->lat_ch * lh * lw * 4);
    ALLOC(P->xin, p3 * 64 * 2);
    ALLOC(P->X, x_elems * 4);
    ALLOC(P->T, t_elems * 4);
    ALLOC(P->Hb, hb_elems * 2);
    ALLOC(P->Xb, xb_elems * 2);
    ALLOC(P->hA, p3p * VAE_MID * 2);
    ALLOC(P->qk, p3p * 2 * VAE_MID * 2);
    ALLOC(P->vT, (size_t)VAE_MID * p3p * 2);
    ALLOC(P->S, p3 * p3p * 4);
    ALLOC(P->Pm, p3 * p3p * 2);
    ALLOC(P->O, p3 * VAE_MID * 2);
    ALLOC(P->part, (size_t)VAE_GN_SLOTS * 64 * sizeof(double));
    ALLOC(P->ab, 2 * VAE_MID * 4);
    ALLOC(P->rgb, 3 * p0 * 4);
    ALLOC(P->rgb8, 3 * p0);
#undef ALLOC
    /* the attention's padding rows (pixels P3 .. P3p - 1) feed GEMM operands: zero once */
    if (!rc) rc = iris_cuda_check(cudaMemsetAsync(P->hA, 0, p3p * VAE_MID * 2, g_rt.stream), "memset");
    if (!rc) rc = iris_cuda_check(cudaMemsetAsync(P->qk, 0, p3p * 2 * VAE_MID * 2, g_rt.stream), "memset");
    if (rc) { plan_free(P); return rc; }
    P->valid = 1;
    return 0;
}

/* ------------------------------------------------------------------ enqueue */
typedef struct {
    int rc;
    uint64_t kernels;
    /* profiling (iris_cuda_vae_profile): an event after every launch */
    iris_cuda_kernel_time_t *prof;
    cudaEvent_t *ev;
    int nprof, maxprof;
} venq_t;

/* account one launch: name, algorithmic FLOPs and HBM bytes for the profile */
static void enq_done(venq_t *E, cudaError_t e, const char *what, double flops, double bytes) {
    if (E->rc) return;
    if (e != cudaSuccess) { E->rc = iris_cuda_check(e, what); return; }
    E->kernels++;
    if (E->prof && E->nprof < E->maxprof) {
        iris_cuda_kernel_time_t *k = &E->prof[E->nprof];
        snprintf(k->name, sizeof(k->name), "%s", what);
        k->flops = flops;
        k->bytes = bytes;
        cudaEventRecord(E->ev[E->nprof + 1], g_rt.stream);
        E->nprof++;
    }
}

static void enq_check(venq_t *E, cudaError_t e, const char *what) { enq_done(E, e, what, 0.0, 0.0); }

static int pow2_at_least(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

/* Tile shape of a convolution launch: single CTA with N = 256 or 128, or a
 * CTA pair (M = 256) with N = 256 or 128, whichever the wave count and the
 * shapes' relative throughputs on B200 (tensor-pipe share reached by each
 * shape; a single CTA at N = 128 is bound by shared-memory reads) predict to
 * finish first. */
static void conv_shape(IrisConvParams *p, const vconv_t *cv) {
    if (cv->bn < 128) return;
    const int sms = g_rt.num_sms;
    const int pairs = iris_conv_pairs_available() < sms / 2 ? iris_conv_pairs_available() : sms / 2;
    const long tx = (p->W + p->bw - 1) / p->bw;
    const long ty1 = (p->H + p->bh - 1) / p->bh, ty2 = (p->H + 2 * p->bh - 1) / (2 * p->bh);
    struct { int pair, bn; double rate; } opt[4] = {{0, 256, 0.80}, {0, 128, 0.55}, {1, 256, 0.78}, {1, 128, 0.62}};
    double best = 1e30;
    for (int i = 0; i < 4; i++) {
        if (opt[i].bn > cv->bn || cv->cout_pad % opt[i].bn) continue;
        if (opt[i].pair && pairs <= 0) continue;
        const long units = tx * (opt[i].pair ? ty2 : ty1) * (cv->cout_pad / opt[i].bn);
        const long slots = opt[i].pair ? pairs : sms;
        const double est = (double)((units + slots - 1) / slots) * opt[i].bn / opt[i].rate;
        if (est < best) {
            best = est;
            p->pair = opt[i].pair;
            p->bn = opt[i].bn;
        }
    }
    p->tmap_b = cv->tm;          /* boxes of min(bn, 128) rows: single CTA, or pair halves of N = 256 */
    if (p->pair) p->tmap_b_half = p->bn == 256 ? cv->tm : cv->tm64;
}

/* conv over an H x W image: segment 0 from in0 (in0_c channels), optional
 * shortcut segment from in1 (in1_c channels) */
static void enq_conv(venq_t *E, iris_cuda_vae_t *v, const vconv_t *cv, const void *in0, int in0_c, const void *in1,
                     int in1_c, int H, int W, int mode, void *out, const float *resid, const vgn_t *gn_next) {
    vplan_t *P = &v->plan;
    if (E->rc) return;
    IrisConvParams p;
    memset(&p, 0, sizeof(p));
    p.bw = pow2_at_least(W) < 128 ? pow2_at_least(W) : 128;
    p.bh = 128 / p.bw;
    while ((1 << p.bw_log2) < p.bw) p.bw_log2++;
    if (iris_make_tmap_nhwc_bf16(&p.tmap_a[0], in0, H, W, in0_c, p.bw, p.bh) ||
        (in1 && iris_make_tmap_nhwc_bf16(&p.tmap_a[1], in1, H, W, in1_c, p.bw, p.bh))) {
        E->rc = iris_fail(IRIS_CUDA_ERR_CUDA, "VAE activation tensor map");
        return;
    }
    p.tmap_b = cv->tm;
    p.H = H;
    p.W = W;
    p.taps0 = cv->taps0;
    p.cin0 = cv->cin0;
    p.cin1 = in1 ? cv->cin1 : 0;
    p.cout = cv->cout;
    p.cout_pad = cv->cout_pad;
    p.bn = cv->bn;
    conv_shape(&p, cv);
    p.mode = mode;
    p.out = out;
    p.bias = cv->b;
    p.resid = resid;
    p.status = g_rt.d_status;
    if (gn_next) {  /* the consuming GroupNorm's partial sums come from this epilogue */
        const int slots = iris_conv_grid(&p, g_rt.num_sms);
        if (slots > VAE_GN_SLOTS) { E->rc = iris_fail(IRIS_CUDA_ERR_ARG, "GroupNorm slots"); return; }
        p.gn_part = P->part;
        p.gn_cg = cv->cout / 32;
        P->gn_nparts = slots;
    }
    const double pix = (double)H * W;
    const double kreal = (double)cv->taps0 * cv->cin_real + p.cin1;
    const double bytes = pix * (cv->cin_real + p.cin1) * 2 + (double)cv->cout * kreal * 2 +
                         pix * cv->cout * (mode == IRIS_CONV_BF16 ? 2 : 4) * (resid ? 2 : 1);
    char name[32];
    snprintf(name, sizeof(name), "conv%s_c%d_%d", cv->taps0 == 9 ? "3x3" : "1x1", cv->cout, H);
    enq_done(E, iris_launch_conv(&p, g_rt.num_sms, g_rt.stream), name, 2.0 * pix * cv->cout * kreal, bytes);
}

/* GroupNorm of x [pix, C] whose partial sums are in P->part (from the
 * convolution that wrote x, or from a statistics pass when stats != 0): the
 * per-channel affine, then the bf16 normalised (and SiLU) copy; raw
 * (optional) gets the plain bf16 x */
static void enq_gn(venq_t *E, iris_cuda_vae_t *v, const float *x, long pix, int C, const vgn_t *gn, int silu,
                   void *out, void *raw, int stats) {
    vplan_t *P = &v->plan;
    if (stats && !E->rc) {
        const long ppi = 256 / (C / 4);
        long nb = (pix + ppi - 1) / ppi;
        if (nb > VAE_GN_BLOCKS) nb = VAE_GN_BLOCKS;
        enq_done(E, iris_launch_gn_stats(x, pix, C, P->part, (int)nb, g_rt.stream), "gn_stats", 0.0,
                 (double)pix * C * 4);
        P->gn_nparts = (int)nb;
    }
    if (!E->rc)
        enq_done(E, iris_launch_gn_finalize(P->part, P->gn_nparts, C, gn->g, gn->b, v->eps, pix * (C / 32), P->ab,
                                            g_rt.stream),
                 "gn_finalize", 0.0, (double)P->gn_nparts * 512);
    if (!E->rc)
        enq_done(E, iris_launch_gn_affine(x, pix, C, P->ab, silu, out, raw, g_rt.stream), "gn_apply", 0.0,
                 (double)pix * C * (raw ? 8 : 6));
}

/* resnet block on P->X (H x W, r->cin channels) -> P->X (r->cout channels);
 * gn_next: the GroupNorm that consumes the block's output (its statistics
 * and affine come from the last convolution), or NULL */
static void enq_res(venq_t *E, iris_cuda_vae_t *v, const vres_t *r, int H, int W, const vgn_t *gn_next) {
    vplan_t *P = &v->plan;
    const long pix = (long)H * W;
    const int skip = r->cin != r->cout;
    enq_gn(E, v, P->X, pix, r->cin, &r->n1, 1, P->Hb, skip ? P->Xb : NULL, 0);
    enq_conv(E, v, &r->c1, P->Hb, r->cin, NULL, 0, H, W, IRIS_CONV_F32, P->T, NULL, &r->n2);
    enq_gn(E, v, P->T, pix, r->cout, &r->n2, 1, P->Hb, NULL, 0);
    enq_conv(E, v, &r->c2, P->Hb, r->cout, skip ? P->Xb : NULL, r->cin, H, W, IRIS_CONV_F32, P->X,
             skip ? NULL : P->X, gn_next);
}

static void enq_gemm(venq_t *E, const void *a, int a_rows, int a_ld, const void *b, int b_rows, int b_ld, int K,
                     int mode, void *out, int ldo, const float *bias, const float *gate) {
    if (E->rc) return;
    IrisGemmParams p;
    memset(&p, 0, sizeof(p));
    const int bn = b_rows % 256 == 0 ? 256 : 128;
    if (iris_make_tmap_bf16(&p.tmap_a, a, (uint64_t)a_rows, (uint64_t)K, (uint64_t)a_ld, 128) ||
        iris_make_tmap_bf16(&p.tmap_b[0], b, (uint64_t)b_rows, (uint64_t)K, (uint64_t)b_ld, (uint32_t)bn)) {
        E->rc = iris_fail(IRIS_CUDA_ERR_CUDA, "VAE attention tensor map");
        return;
    }
    p.ngroups = 1;
    p.row0[0] = 0;
    p.rows[0] = a_rows;
    p.N = b_rows;
    p.K = K;
    p.bn = bn;
    p.mode = mode;
    p.out = out;
    p.ldo = ldo;
    p.bias = bias;
    p.gate[0] = gate;
    p.status = g_rt.d_status;
    int n = 1;
    cudaError_t e = iris_launch_gemm_ex(&p, g_rt.num_sms, g_rt.stream, &n);
    const double by = ((double)a_rows + b_rows) * K * 2 + (double)a_rows * b_rows * (mode == IRIS_EPI_BF16 ? 2 : 4);
    enq_done(E, e, "attn_gemm", 2.0 * a_rows * b_rows * K, by);
    if (!E->rc && n > 1) E->kernels += (uint64_t)(n - 1);
}

/* mid-block attention on P->X [P3, 512], in place (attnblock_forward, iris_vae.c:260) */
static void enq_attn(venq_t *E, iris_cuda_vae_t *v) {
    vplan_t *P = &v->plan;
    const int c = VAE_MID, p3 = P->H[3] * P->W[3], p3p = P->P3p;
    enq_gn(E, v, P->X, p3, c, &v->attn_gn, 0, P->hA, NULL, 0);
    /* [q | k] = h Wqk^T + b  -> bf16 [P3, 1024] */
    enq_gemm(E, P->hA, p3, c, v->w_qk, 2 * c, c, c, IRIS_EPI_BF16, P->qk, 2 * c, v->b_qk, NULL);
    /* V^T = Wv h^T -> bf16 [512, P3p] (its bias is added after P V: the rows of P sum to 1) */
    enq_gemm(E, v->w_v, c, c, P->hA, p3p, c, c, IRIS_EPI_BF16, P->vT, p3p, NULL, NULL);
    /* S = q k^T -> f32 [P3, P3p] */
    enq_gemm(E, P->qk, p3, 2 * c, P->qk + c, p3p, 2 * c, c, IRIS_EPI_F32, P->S, p3p, NULL, NULL);
    if (!E->rc)
        enq_done(E, iris_launch_vae_softmax(P->S, p3, p3p, p3, 1.0f / sqrtf((float)c), P->Pm, g_rt.stream),
                 "attn_softmax", 0.0, (double)p3 * p3p * 6);
    /* O = P V + bv -> bf16 [P3, 512] */
    enq_gemm(E, P->Pm, p3, p3p, P->vT, c, p3p, p3p, IRIS_EPI_BF16, P->O, c, v->b_v, NULL);
    /* x += O Wo^T + bo */
    enq_gemm(E, P->O, p3, c, v->w_o, c, c, c, IRIS_EPI_RESID_GATE, P->X, c, v->b_o, v->ones);
}

static int enqueue_decode(iris_cuda_vae_t *v, venq_t *E) {
    vplan_t *P = &v->plan;
    if (!E->rc)
        enq_check(E, iris_launch_vae_latent_prep(P->lat, v->z, P->lh, P->lw, v->bn_mean, v->bn_std, v->scaling,
                                                 v->shift, v->pq_w, v->pq_b, P->xin, g_rt.stream),
                  "latent prep");
    enq_conv(E, v, &v->conv_in, P->xin, 64, NULL, 0, P->H[3], P->W[3], IRIS_CONV_F32, P->X, NULL, &v->mid[0].n1);
    enq_res(E, v, &v->mid[0], P->H[3], P->W[3], &v->attn_gn);
    enq_attn(E, v);
    /* the attention's output projection (a GEMM) sums no GroupNorm statistics */
    const int p3 = P->H[3] * P->W[3];
    enq_gn(E, v, P->X, p3, VAE_MID, &v->mid[1].n1, 1, P->Hb, NULL, 1);
    {
        const vres_t *r = &v->mid[1];
        enq_conv(E, v, &r->c1, P->Hb, r->cin, NULL, 0, P->H[3], P->W[3], IRIS_CONV_F32, P->T, NULL, &r->n2);
        enq_gn(E, v, P->T, p3, r->cout, &r->n2, 1, P->Hb, NULL, 0);
        enq_conv(E, v, &r->c2, P->Hb, r->cout, NULL, 0, P->H[3], P->W[3], IRIS_CONV_F32, P->X, P->X, &v->up[0].n1);
    }
    int bi = 0;
    for (int level = 3; level >= 0; level--) {
        const int ch = VAE_BASE * k_mult[level];
        for (int r = 0; r < 3; r++, bi++) {
            /* consumer of the block's output: the next block's norm1, nothing
             * before an upsample, the output norm after the last block */
            const vgn_t *next = r < 2 ? &v->up[bi + 1].n1 : level == 0 ? &v->out_gn : NULL;
            enq_res(E, v, &v->up[bi], P->H[level], P->W[level], next);
        }
        if (level > 0) {
            const long pix = (long)P->H[level] * P->W[level];
            if (!E->rc)
                enq_done(E, iris_launch_nhwc_to_bf16(P->X, pix, ch, P->W[level], 1, P->Hb, g_rt.stream), "upsample",
                         0.0, (double)pix * ch * 12);
            enq_conv(E, v, &v->upc[3 - level], P->Hb, ch, NULL, 0, P->H[level - 1], P->W[level - 1], IRIS_CONV_F32,
                     P->X, NULL, &v->up[bi].n1);
        }
    }
    const long p0 = (long)P->H[0] * P->W[0];
    enq_gn(E, v, P->X, p0, VAE_BASE, &v->out_gn, 1, P->Hb, NULL, 0);
    enq_conv(E, v, &v->conv_out, P->Hb, VAE_BASE, NULL, 0, P->H[0], P->W[0], IRIS_CONV_F32_NCHW, P->rgb, NULL, NULL);
    if (!E->rc) enq_check(E, iris_launch_vae_rgb8(P->rgb, p0, P->rgb8, g_rt.stream), "rgb8");
    return E->rc;
}

static int run_decode(iris_cuda_vae_t *v) {
    vplan_t *P = &v->plan;
    if (iris_fault("launch")) return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected launch failure");
    if (!P->graph_ok) {
        static int no_graph = -1;
        if (no_graph < 0) no_graph = getenv("IRIS_CUDA_NO_GRAPH") ? 1 : 0;
        venq_t E = {0};
        if (no_graph) {
            int rc = enqueue_decode(v, &E);
            iris_count_launch(E.kernels);
            return rc;
        }
        cudaError_t e = cudaStreamBeginCapture(g_rt.stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return iris_cuda_check(e, "begin capture");
        int rc = enqueue_decode(v, &E);
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

static int check_args(iris_cuda_vae_t *v, int batch, int lh, int lw) {
    if (!v) return iris_fail(IRIS_CUDA_ERR_ARG, "null VAE");
    if (batch != 1) return iris_fail(IRIS_CUDA_ERR_ARG, "batch %d (1 supported)", batch);
    if (lh < 1 || lw < 1 || (long)4 * lh * lw > VAE_MAX_MID_PIXELS)
        return iris_fail(IRIS_CUDA_ERR_ARG, "latent %dx%d (up to %d latent pixels)", lh, lw, VAE_MAX_MID_PIXELS / 4);
    return 0;
}

int iris_cuda_vae_decode_dev(iris_cuda_vae_t *v, const float *d_latent, int lh, int lw, uint8_t *d_rgb8,
                             float *d_rgb_f32) {
    int rc = check_args(v, 1, lh, lw);
    if (rc) return rc;
    if (!d_latent) return iris_fail(IRIS_CUDA_ERR_ARG, "null latent");
    if ((rc = plan_ensure(v, lh, lw))) return rc;
    vplan_t *P = &v->plan;
    const size_t p0 = (size_t)P->H[0] * P->W[0];
    rc = iris_cuda_check(cudaMemcpyAsync(P->lat, d_latent, (size_t)v->lat_ch * lh * lw * 4,
                                         cudaMemcpyDeviceToDevice, g_rt.stream), "latent copy");
    if (!rc) rc = run_decode(v);
    if (!rc && d_rgb8)
        rc = iris_cuda_check(cudaMemcpyAsync(d_rgb8, P->rgb8, 3 * p0, cudaMemcpyDeviceToDevice, g_rt.stream), "rgb8");
    if (!rc && d_rgb_f32)
        rc = iris_cuda_check(cudaMemcpyAsync(d_rgb_f32, P->rgb, 3 * p0 * 4, cudaMemcpyDeviceToDevice, g_rt.stream),
                             "rgb");
    return rc;
}

/* host latent -> device plan -> decode; out8 / outf (host) receive the results */
static int decode_host(iris_cuda_vae_t *v, const float *latent, int lh, int lw, uint8_t *out8, float *outf) {
    int rc = check_args(v, 1, lh, lw);
    if (rc) return rc;
    if (!latent) return iris_fail(IRIS_CUDA_ERR_ARG, "null latent");
    if ((rc = plan_ensure(v, lh, lw))) return rc;
    vplan_t *P = &v->plan;
    const size_t p0 = (size_t)P->H[0] * P->W[0];
    if (iris_fault("h2d")) return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected h2d failure");
    rc = iris_cuda_check(cudaMemcpyAsync(P->lat, latent, (size_t)v->lat_ch * lh * lw * 4, cudaMemcpyHostToDevice,
                                         g_rt.stream), "h2d");
    if (!rc) rc = run_decode(v);
    if (!rc && out8) rc = iris_cuda_check(cudaMemcpyAsync(out8, P->rgb8, 3 * p0, cudaMemcpyDeviceToHost, g_rt.stream), "d2h");
    if (!rc && outf)
        rc = iris_cuda_check(cudaMemcpyAsync(outf, P->rgb, 3 * p0 * 4, cudaMemcpyDeviceToHost, g_rt.stream), "d2h");
    if (!rc) rc = iris_cuda_synchronize();
    return rc;
}

iris_cuda_image_t *iris_cuda_vae_decode(iris_cuda_vae_t *v, const float *latent, int batch, int lh, int lw) {
    if (check_args(v, batch, lh, lw)) return NULL;
    iris_cuda_image_t *img = (iris_cuda_image_t *)calloc(1, sizeof(*img));
    uint8_t *data = (uint8_t *)malloc((size_t)3 * 256 * lh * lw);
    if (!img || !data) {
        free(img);
        free(data);
        iris_fail(IRIS_CUDA_ERR_OOM, "image");
        return NULL;
    }
    if (decode_host(v, latent, lh, lw, data, NULL)) {
        free(img);
        free(data);
        return NULL;
    }
    img->width = 16 * lw;
    img->height = 16 * lh;
    img->channels = 3;
    img->data = data;
    return img;
}

int iris_cuda_vae_decode_f32(iris_cuda_vae_t *v, const float *latent, int lh, int lw, float *out) {
    if (!out) return iris_fail(IRIS_CUDA_ERR_ARG, "null output");
    return decode_host(v, latent, lh, lw, NULL, out);
}

void iris_cuda_image_free(iris_cuda_image_t *img) {
    if (!img) return;
    free(img->data);
    free(img);
}

uint64_t iris_cuda_vae_graph_kernels(const iris_cuda_vae_t *v) { return v ? v->plan.graph_kernels : 0; }

/* Time every kernel of one decode of the current plan size (no graph; an
 * event after each launch).  Returns the number of entries or a negative
 * status. */
int iris_cuda_vae_profile(iris_cuda_vae_t *v, iris_cuda_kernel_time_t *out, int max_entries) {
    if (!v || !out || max_entries <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!v->plan.valid) return iris_fail(IRIS_CUDA_ERR_ARG, "decode once first (no plan)");
    cudaEvent_t *ev = (cudaEvent_t *)calloc((size_t)max_entries + 1, sizeof(cudaEvent_t));
    if (!ev) return iris_fail(IRIS_CUDA_ERR_OOM, "events");
    int rc = 0, n = 0;
    for (int i = 0; i <= max_entries && !rc; i++) rc = iris_cuda_check(cudaEventCreate(&ev[i]), "event");
    if (!rc) {
        venq_t E = {0};
        E.prof = out;
        E.ev = ev;
        E.maxprof = max_entries;
        cudaEventRecord(ev[0], g_rt.stream);
        rc = enqueue_decode(v, &E);
        iris_count_launch(E.kernels);
        if (!rc) rc = iris_cuda_synchronize();
        for (int i = 0; !rc && i < E.nprof; i++) cudaEventElapsedTime(&out[i].ms, ev[i], ev[i + 1]);
        n = E.nprof;
    }
    for (int i = 0; i <= max_entries; i++)
        if (ev[i]) cudaEventDestroy(ev[i]);
    free(ev);
    return rc ? rc : n;
}
