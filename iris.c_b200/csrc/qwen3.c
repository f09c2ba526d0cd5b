/*
 * Qwen3 text encoder on the GPU: token ids -> the text embeddings the
 * transformer conditions on.  Replaces qwen3_model_load / qwen3_forward /
 * qwen3_set_extraction_mode (iris_qwen3.c:1578, :1072, :1849); tokenisation
 * stays with the caller (the reference's qwen3_tokenize_chat / pad_tokens).
 *
 * Per layer (pre-norm, iris_qwen3.c:496-535): RMSNorm -> one QKV GEMM (f32
 * out) -> per-head Q/K RMSNorm + split-half RoPE (bf16) -> causal grouped-
 * query attention with the padding mask (tcgen05) -> output projection GEMM
 * adding into the f32 hidden state -> RMSNorm -> gate/up GEMM with the SwiGLU
 * epilogue -> down projection GEMM adding into the hidden state.  Flux takes
 * the hidden state after layers 8, 17 and 26 side by side ([S, 3H]); Z-Image
 * the one after layer num_layers - 2 ([S, H]).  Only the layers up to the last
 * extracted one run.  One forward per sequence length is a CUDA graph.
 */
#include "iris_internal.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define Q3_EPS 1e-6f        /* QWEN3_RMS_NORM_EPS */
#define Q3_MAX_SEQ 512      /* QWEN3_MAX_SEQ_LEN: the reference pads every prompt to it */
static const int k_flux_layers[3] = {8, 17, 26};  /* QWEN3_OUTPUT_LAYER_1..3 */

typedef struct {
    uint16_t *w_qkv;   /* [(nh + 2 nkv) * 128, H] */
    uint16_t *w_o;     /* [H, nh * 128] */
    uint16_t *w_gu;    /* [2F, H], gate/up rows interleaved in blocks of 128 */
    uint16_t *w_down;  /* [H, F] */
    float *ln1, *ln2, *qn, *kn;
    CUtensorMap tm_qkv, tm_o, tm_gu, tm_down;
} q3_layer_t;

typedef struct {
    int valid, S;
    int *ids;
    uint8_t *mask;
    float *x, *qkv, *out, *cosb, *sinb;
    float *ws;          /* split-K workspace of the H-wide projections (few output tiles at 512 rows) */
    size_t ws_bytes;
    uint16_t *xn, *q, *k, *v, *attn, *mlp;
    CUtensorMap tm_xn, tm_attn, tm_mlp;
    cudaGraph_t graph;
    cudaGraphExec_t gexec;
    int graph_ok, graph_mode;
    uint64_t graph_kernels;
} q3_plan_t;

struct iris_cuda_qwen3 {
    iris_cuda_qwen3_config_t cfg;
    int mode;              /* 0 Flux, 1 Z-Image extraction */
    int nlayers;           /* layers held on the device */
    uint16_t *embed;       /* [vocab, H] */
    q3_layer_t *layers;
    float *ones;           /* [H] gate of the residual GEMM epilogues */
    q3_plan_t plan;
    size_t weight_bytes;
};

static int q3_qkv_n(const iris_cuda_qwen3_config_t *c) { return (c->heads + 2 * c->kv_heads) * c->head_dim; }

static int last_layer(const iris_cuda_qwen3_t *m) {
    return m->mode ? m->cfg.layers - 2 : k_flux_layers[2];
}

int iris_cuda_qwen3_text_dim(const iris_cuda_qwen3_t *m) {
    return m ? (m->mode ? m->cfg.hidden : 3 * m->cfg.hidden) : 0;
}

static void *q3_dalloc(iris_cuda_qwen3_t *m, size_t bytes) {
    void *p = iris_dmalloc(bytes);
    if (p) m->weight_bytes += bytes;
    return p;
}

/* ------------------------------------------------------------------ loading */
typedef struct {
    iris_wsrc_t *file;      /* NULL: seeded device RNG (the file path shares the
                               pipelined upload of the DiT loaders, weights.c) */
    uint64_t seed;
} q3_src_t;

/* bf16 tensor `name` of numel values to d_dst: from the file, or random
 * N(0, std) (+ mean) from the device RNG keyed by the name */
static int q3_get_bf16(q3_src_t *src, const char *name, size_t numel, uint16_t *d_dst, float mean, float std) {
    if (!src->file) {
        cudaError_t e = iris_launch_randn_bf16(d_dst, (long)numel, src->seed, iris_crc32(name), mean, std, g_rt.stream);
        return iris_cuda_check(e, "randn");
    }
    return iris_wsrc_get(src->file, name, numel, d_dst);
}

/* f32 vector `name` (norm scales) through a bf16 device temp */
static int q3_get_vec(q3_src_t *src, const char *name, int n, float *d_dst, uint16_t *tmp) {
    int rc = q3_get_bf16(src, name, (size_t)n, tmp, src->file ? 0.f : 1.0f, src->file ? 0.f : 0.1f);
    if (!rc) rc = iris_cuda_check(iris_launch_bf16_to_f32(tmp, d_dst, n, g_rt.stream), "bf16 to f32");
    /* tmp is rewritten by the next (host-synchronous) upload */
    if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "bf16 to f32");
    return rc;
}

static int q3_load_layers(iris_cuda_qwen3_t *m, q3_src_t *src) {
    const iris_cuda_qwen3_config_t *c = &m->cfg;
    const int H = c->hidden, F = c->intermediate, qd = c->heads * c->head_dim, kvd = c->kv_heads * c->head_dim;
    const int nq = q3_qkv_n(c);
    char n[256];
    int rc = 0;
    uint16_t *tmp = (uint16_t *)iris_dmalloc((size_t)2 * F * H * 2);
    if (!tmp) return iris_fail(IRIS_CUDA_ERR_OOM, "text encoder staging");
    m->embed = (uint16_t *)q3_dalloc(m, (size_t)c->vocab * H * 2);
    if (!m->embed) rc = iris_fail(IRIS_CUDA_ERR_OOM, "embeddings");
    if (!rc) rc = q3_get_bf16(src, "model.embed_tokens.weight", (size_t)c->vocab * H, m->embed, 0.f, 1.0f);
    for (int i = 0; !rc && i < m->nlayers; i++) {
        q3_layer_t *L = &m->layers[i];
        L->w_qkv = (uint16_t *)q3_dalloc(m, (size_t)nq * H * 2);
        L->w_o = (uint16_t *)q3_dalloc(m, (size_t)H * qd * 2);
        L->w_gu = (uint16_t *)q3_dalloc(m, (size_t)2 * F * H * 2);
        L->w_down = (uint16_t *)q3_dalloc(m, (size_t)H * F * 2);
        L->ln1 = (float *)q3_dalloc(m, (size_t)H * 4);
        L->ln2 = (float *)q3_dalloc(m, (size_t)H * 4);
        L->qn = (float *)q3_dalloc(m, 128 * 4);
        L->kn = (float *)q3_dalloc(m, 128 * 4);
        if (!L->w_qkv || !L->w_o || !L->w_gu || !L->w_down || !L->ln1 || !L->ln2 || !L->qn || !L->kn) {
            rc = iris_fail(IRIS_CUDA_ERR_OOM, "text encoder layer %d", i);
            break;
        }
        const float sdH = 1.0f / sqrtf((float)H), sdQ = 1.0f / sqrtf((float)qd), sdF = 1.0f / sqrtf((float)F);
#define P(fmt) (snprintf(n, sizeof(n), "model.layers.%d." fmt, i), n)
        /* [q; k; v] stacked rows: the QKV projection is one GEMM */
        if (!rc) rc = q3_get_bf16(src, P("self_attn.q_proj.weight"), (size_t)qd * H, L->w_qkv, 0.f, sdH);
        if (!rc) rc = q3_get_bf16(src, P("self_attn.k_proj.weight"), (size_t)kvd * H, L->w_qkv + (size_t)qd * H, 0.f, sdH);
        if (!rc)
            rc = q3_get_bf16(src, P("self_attn.v_proj.weight"), (size_t)kvd * H, L->w_qkv + (size_t)(qd + kvd) * H,
                             0.f, sdH);
        if (!rc) rc = q3_get_bf16(src, P("self_attn.o_proj.weight"), (size_t)H * qd, L->w_o, 0.f, sdQ);
        /* [gate; up] -> 256-row blocks [gate 128 | up 128] (the SwiGLU epilogue's layout) */
        if (!rc) rc = q3_get_bf16(src, P("mlp.gate_proj.weight"), (size_t)F * H, tmp, 0.f, sdH);
        if (!rc) rc = q3_get_bf16(src, P("mlp.up_proj.weight"), (size_t)F * H, tmp + (size_t)F * H, 0.f, sdH);
        if (!rc) rc = iris_cuda_check(iris_launch_interleave_gate_up(L->w_gu, tmp, F, H, g_rt.stream), "interleave");
        if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "interleave");
        if (!rc) rc = q3_get_bf16(src, P("mlp.down_proj.weight"), (size_t)H * F, L->w_down, 0.f, sdF);
        if (!rc) rc = q3_get_vec(src, P("input_layernorm.weight"), H, L->ln1, tmp);
        if (!rc) rc = q3_get_vec(src, P("post_attention_layernorm.weight"), H, L->ln2, tmp);
        if (!rc) rc = q3_get_vec(src, P("self_attn.q_norm.weight"), 128, L->qn, tmp);
        if (!rc) rc = q3_get_vec(src, P("self_attn.k_norm.weight"), 128, L->kn, tmp);
        if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "layer upload");
#undef P
        if (!rc && (iris_make_tmap_bf16(&L->tm_qkv, L->w_qkv, (uint64_t)nq, (uint64_t)H, (uint64_t)H,
                                        nq % 256 ? 128 : 256) ||
                    iris_make_tmap_bf16(&L->tm_o, L->w_o, (uint64_t)H, (uint64_t)qd, (uint64_t)qd,
                                        H % 256 ? 128 : 256) ||
                    iris_make_tmap_bf16(&L->tm_gu, L->w_gu, (uint64_t)2 * F, (uint64_t)H, (uint64_t)H, 256) ||
                    iris_make_tmap_bf16(&L->tm_down, L->w_down, (uint64_t)H, (uint64_t)F, (uint64_t)F,
                                        H % 256 ? 128 : 256)))
            rc = iris_fail(IRIS_CUDA_ERR_CUDA, "text encoder weight tensor map");
    }
    iris_dfree(tmp);
    return rc;
}

static void q3_plan_free(q3_plan_t *P);

void iris_cuda_qwen3_free(iris_cuda_qwen3_t *m) {
    if (!m) return;
    if (g_rt.initialized) cudaStreamSynchronize(g_rt.stream);
    q3_plan_free(&m->plan);
    iris_dfree(m->embed);
    for (int i = 0; m->layers && i < m->nlayers; i++) {
        q3_layer_t *L = &m->layers[i];
        void *b[] = {L->w_qkv, L->w_o, L->w_gu, L->w_down, L->ln1, L->ln2, L->qn, L->kn};
        for (size_t j = 0; j < sizeof(b) / sizeof(b[0]); j++) iris_dfree(b[j]);
    }
    free(m->layers);
    iris_dfree(m->ones);
    free(m);
}

static int q3_check_config(const iris_cuda_qwen3_config_t *c) {
    if (c->hidden <= 0 || c->hidden % 128 || c->intermediate <= 0 || c->intermediate % 128 || c->head_dim != 128 ||
        c->heads <= 0 || c->kv_heads <= 0 || c->heads % c->kv_heads || c->vocab <= 0 || c->layers < 2 ||
        c->rope_theta <= 0.f)
        return iris_fail(IRIS_CUDA_ERR_ARG,
                         "unsupported text encoder shape (hidden %d, intermediate %d, heads %d/%d x %d): hidden and "
                         "intermediate multiples of 128, head_dim 128", c->hidden, c->intermediate, c->heads,
                         c->kv_heads, c->head_dim);
    return 0;
}

static iris_cuda_qwen3_t *q3_create(const iris_cuda_qwen3_config_t *cfg, q3_src_t *src) {
    if (q3_check_config(cfg)) return NULL;
    iris_cuda_qwen3_t *m = (iris_cuda_qwen3_t *)calloc(1, sizeof(*m));
    if (!m) { iris_fail(IRIS_CUDA_ERR_OOM, "text encoder"); return NULL; }
    m->cfg = *cfg;
    /* every layer up to the later of the two extraction points */
    m->nlayers = cfg->layers - 1 > k_flux_layers[2] + 1 ? cfg->layers - 1 : k_flux_layers[2] + 1;
    if (m->nlayers > cfg->layers) m->nlayers = cfg->layers;
    m->layers = (q3_layer_t *)calloc((size_t)m->nlayers, sizeof(q3_layer_t));
    float *ones = (float *)malloc((size_t)cfg->hidden * 4);
    m->ones = (float *)iris_dmalloc((size_t)cfg->hidden * 4);
    int rc = (!m->layers || !ones || !m->ones) ? iris_fail(IRIS_CUDA_ERR_OOM, "text encoder") : 0;
    if (!rc) {
        for (int i = 0; i < cfg->hidden; i++) ones[i] = 1.0f;
        rc = iris_h2d(m->ones, ones, (size_t)cfg->hidden * 4);
    }
    free(ones);
    if (!rc) rc = q3_load_layers(m, src);
    if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "text encoder upload");
    if (rc) { iris_cuda_qwen3_free(m); return NULL; }
    return m;
}

iris_cuda_qwen3_t *iris_cuda_qwen3_load(const char *model_dir) {
    if (!model_dir) { iris_fail(IRIS_CUDA_ERR_ARG, "null model directory"); return NULL; }
    if (iris_rt_ensure()) return NULL;
    /* config.json keys and defaults as parse_qwen3_config / qwen3_set_defaults (iris_qwen3.c:1378-1447) */
    iris_cuda_qwen3_config_t c = {2560, 9728, 32, 8, 128, 151936, 36, 1000000.0f};
    char path[4200];
    snprintf(path, sizeof(path), "%s/config.json", model_dir);
    FILE *f = fopen(path, "rb");
    if (f) {
        char buf[16384];
        size_t got = fread(buf, 1, sizeof(buf) - 1, f);
        buf[got] = 0;
        fclose(f);
        double d;
        if (!json_get_number(buf, "hidden_size", &d) && d > 0) c.hidden = (int)d;
        if (!json_get_number(buf, "intermediate_size", &d) && d > 0) c.intermediate = (int)d;
        if (!json_get_number(buf, "num_attention_heads", &d) && d > 0) c.heads = (int)d;
        if (!json_get_number(buf, "num_key_value_heads", &d) && d > 0) c.kv_heads = (int)d;
        if (!json_get_number(buf, "head_dim", &d) && d > 0) c.head_dim = (int)d;
        if (!json_get_number(buf, "vocab_size", &d) && d > 0) c.vocab = (int)d;
        if (!json_get_number(buf, "num_hidden_layers", &d) && d > 0) c.layers = (int)d;
        if (!json_get_number(buf, "rope_theta", &d) && d > 0) c.rope_theta = (float)d;
    }
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    if (st_open_dir(&ws.st, model_dir)) {
        iris_fail(IRIS_CUDA_ERR_IO, "cannot open text encoder weights in %s", model_dir);
        return NULL;
    }
    q3_src_t src = {&ws, 0};
    iris_cuda_qwen3_t *m = q3_create(&c, &src);
    iris_wsrc_free(&ws);  /* waits for the last uploads */
    st_close(&ws.st);
    return m;
}

iris_cuda_qwen3_t *iris_cuda_qwen3_random(const iris_cuda_qwen3_config_t *cfg, uint64_t seed) {
    if (!cfg) { iris_fail(IRIS_CUDA_ERR_ARG, "null config"); return NULL; }
    if (iris_rt_ensure()) return NULL;
    q3_src_t src = {NULL, seed};
    iris_cuda_qwen3_t *m = q3_create(cfg, &src);
    if (m && iris_cuda_synchronize()) { iris_cuda_qwen3_free(m); return NULL; }
    return m;
}

int iris_cuda_qwen3_get_config(const iris_cuda_qwen3_t *m, iris_cuda_qwen3_config_t *out) {
    if (!m || !out) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    *out = m->cfg;
    return 0;
}

size_t iris_cuda_qwen3_weight_bytes(const iris_cuda_qwen3_t *m) { return m ? m->weight_bytes : 0; }

int iris_cuda_qwen3_set_extraction_mode(iris_cuda_qwen3_t *m, int mode) {
    if (!m || (mode != 0 && mode != 1)) return iris_fail(IRIS_CUDA_ERR_ARG, "extraction mode 0 (Flux) or 1 (Z-Image)");
    if (mode == 0 && m->cfg.layers < k_flux_layers[2] + 1)
        return iris_fail(IRIS_CUDA_ERR_ARG, "Flux extraction needs %d layers", k_flux_layers[2] + 1);
    m->mode = mode;
    return 0;
}

/* ------------------------------------------------------------------ plan */
static void q3_plan_free(q3_plan_t *P) {
    if (P->graph_ok) {
        cudaGraphExecDestroy(P->gexec);
        cudaGraphDestroy(P->graph);
    }
    void *b[] = {P->ids, P->mask, P->x, P->qkv, P->out, P->cosb, P->sinb, P->xn, P->q, P->k, P->v, P->attn, P->mlp,
                 P->ws};
    for (size_t i = 0; i < sizeof(b) / sizeof(b[0]); i++) iris_dfree(b[i]);
    memset(P, 0, sizeof(*P));
}

static int q3_plan_ensure(iris_cuda_qwen3_t *m, int S) {
    q3_plan_t *P = &m->plan;
    if (P->valid && P->S == S) return 0;
    q3_plan_free(P);
    const iris_cuda_qwen3_config_t *c = &m->cfg;
    const size_t H = (size_t)c->hidden, F = (size_t)c->intermediate, qd = (size_t)c->heads * 128,
                 kvd = (size_t)c->kv_heads * 128, nq = (size_t)q3_qkv_n(c);
    int rc = 0;
#define ALLOC(dst, bytes) \
    do { if (!rc && !((dst) = iris_dmalloc(bytes))) rc = iris_fail(IRIS_CUDA_ERR_OOM, "text encoder plan"); } while (0)
    ALLOC(P->ids, (size_t)S * 4);
    ALLOC(P->mask, (size_t)S);
    ALLOC(P->x, S * H * 4);
    ALLOC(P->qkv, S * nq * 4);
    ALLOC(P->out, S * 3 * H * 4);
    ALLOC(P->cosb, (size_t)S * 64 * 4);
    ALLOC(P->sinb, (size_t)S * 64 * 4);
    ALLOC(P->xn, S * H * 2);
    ALLOC(P->q, S * qd * 2);
    ALLOC(P->k, S * kvd * 2);
    ALLOC(P->v, S * kvd * 2);
    ALLOC(P->attn, S * qd * 2);
    ALLOC(P->mlp, S * F * 2);
    P->ws_bytes = (size_t)4 * S * H * 4;  /* up to 4 K splits */
    ALLOC(P->ws, P->ws_bytes);
#undef ALLOC
    if (!rc) {
        /* RoPE tables with the reference's float formulas (compute_rope_freqs, iris_qwen3.c:258-275) */
        float *cs = (float *)malloc((size_t)S * 64 * 4), *sn = (float *)malloc((size_t)S * 64 * 4);
        if (!cs || !sn) rc = iris_fail(IRIS_CUDA_ERR_OOM, "rope tables");
        for (int pos = 0; !rc && pos < S; pos++)
            for (int i = 0; i < 64; i++) {
                const float freq = 1.0f / powf(c->rope_theta, (float)(2 * i) / 128.0f);
                const float angle = pos * freq;
                cs[pos * 64 + i] = cosf(angle);
                sn[pos * 64 + i] = sinf(angle);
            }
        if (!rc) rc = iris_h2d(P->cosb, cs, (size_t)S * 256);
        if (!rc) rc = iris_h2d(P->sinb, sn, (size_t)S * 256);
        free(cs);
        free(sn);
    }
    if (!rc && (iris_make_tmap_bf16(&P->tm_xn, P->xn, (uint64_t)S, H, H, 128) ||
                iris_make_tmap_bf16(&P->tm_attn, P->attn, (uint64_t)S, qd, qd, 128) ||
                iris_make_tmap_bf16(&P->tm_mlp, P->mlp, (uint64_t)S, F, F, 128)))
        rc = iris_fail(IRIS_CUDA_ERR_CUDA, "text encoder activation tensor map");
    if (rc) { q3_plan_free(P); return rc; }
    P->S = S;
    P->valid = 1;
    return 0;
}

/* ------------------------------------------------------------------ enqueue */
typedef struct {
    int rc;
    uint64_t kernels;
    /* profiling (iris_cuda_qwen3_profile): an event after every launch */
    iris_cuda_kernel_time_t *prof;
    cudaEvent_t *ev;
    int nprof, maxprof;
    double flops;  /* algorithmic FLOPs of the next accounted launch */
} q3_enq_t;

static void q3_done(q3_enq_t *E, cudaError_t e, const char *what, int n) {
    if (E->rc) return;
    if (e != cudaSuccess) { E->rc = iris_cuda_check(e, what); return; }
    E->kernels += (uint64_t)n;
    if (E->prof && E->nprof < E->maxprof) {
        iris_cuda_kernel_time_t *k = &E->prof[E->nprof];
        snprintf(k->name, sizeof(k->name), "%s", what);
        k->flops = E->flops;
        k->bytes = 0.0;
        cudaEventRecord(E->ev[E->nprof + 1], g_rt.stream);
        E->nprof++;
    }
    E->flops = 0.0;
}

static void q3_gemm(q3_enq_t *E, const char *name, const CUtensorMap *ta, const CUtensorMap *tb, int M, int N,
                    int K, int mode, void *out, int ldo, const float *gate, void *mlp_out, int ld_mlp, float *ws,
                    size_t ws_bytes) {
    if (E->rc) return;
    IrisGemmParams p;
    memset(&p, 0, sizeof(p));
    p.ws = ws;
    p.ws_bytes = ws_bytes;
    p.tmap_a = *ta;
    p.tmap_b[0] = *tb;
    p.ngroups = 1;
    p.rows[0] = M;
    p.N = N;
    p.K = K;
    p.bn = N % 256 == 0 ? 256 : 128;
    p.b_static = 1;  /* B: a resident weight */
    p.mode = mode;
    p.out = out;
    p.ldo = ldo;
    p.gate[0] = gate;
    p.mlp_out = mlp_out;
    p.ld_mlp = ld_mlp;
    p.status = g_rt.d_status;
    int n = 1;
    cudaError_t e = iris_launch_gemm_ex(&p, g_rt.num_sms, g_rt.stream, &n);
    E->flops = 2.0 * M * N * K;
    q3_done(E, e, name, n);
}

static int q3_enqueue(iris_cuda_qwen3_t *m, q3_enq_t *E) {
    q3_plan_t *P = &m->plan;
    const iris_cuda_qwen3_config_t *c = &m->cfg;
    const int S = P->S, H = c->hidden, F = c->intermediate, qd = c->heads * 128, kvd = c->kv_heads * 128;
    const int nq = q3_qkv_n(c), last = last_layer(m), td = iris_cuda_qwen3_text_dim(m);
    cudaStream_t st = g_rt.stream;
    q3_done(E, iris_launch_embed_rows(P->ids, S, m->embed, c->vocab, H, P->x, st), "embed", 1);
    int slot = 0;
    for (int i = 0; i <= last && !E->rc; i++) {
        const q3_layer_t *L = &m->layers[i];
        q3_done(E, iris_launch_rmsnorm(P->x, H, L->ln1, NULL, P->xn, H, S, H, Q3_EPS, NULL, st), "rmsnorm", 1);
        q3_gemm(E, "qkv", &P->tm_xn, &L->tm_qkv, S, nq, H, IRIS_EPI_F32, P->qkv, nq, NULL, NULL, 0, NULL, 0);
        q3_done(E, iris_launch_qk_norm_rope_half(P->qkv, nq, S, c->heads, c->kv_heads, L->qn, L->kn, P->cosb, P->sinb,
                                                 Q3_EPS, P->q, P->k, P->v, st),
                "qk norm rope", 1);
        E->flops = 2.0 * S * S * qd;  /* causal: half of 4 S^2 d per head */
        q3_done(E, iris_launch_attention_gqa(P->q, qd, P->k, P->v, kvd, P->attn, qd, S, S, c->heads,
                                             c->heads / c->kv_heads, 1, 1.0f / sqrtf(128.0f), P->mask, st),
                "attention", 1);
        q3_gemm(E, "o_proj", &P->tm_attn, &L->tm_o, S, H, qd, IRIS_EPI_RESID_GATE, P->x, H, m->ones, NULL, 0, P->ws, P->ws_bytes);
        q3_done(E, iris_launch_rmsnorm(P->x, H, L->ln2, NULL, P->xn, H, S, H, Q3_EPS, NULL, st), "rmsnorm", 1);
        q3_gemm(E, "gate_up", &P->tm_xn, &L->tm_gu, S, 2 * F, H, IRIS_EPI_SWIGLU, NULL, 0, NULL, P->mlp, F, NULL, 0);
        q3_gemm(E, "down", &P->tm_mlp, &L->tm_down, S, H, F, IRIS_EPI_RESID_GATE, P->x, H, m->ones, NULL, 0, P->ws, P->ws_bytes);
        const int extract = m->mode ? (i == last) : (i == k_flux_layers[0] || i == k_flux_layers[1] || i == k_flux_layers[2]);
        if (extract && !E->rc) {
            q3_done(E, cudaMemcpy2DAsync(P->out + (size_t)slot * H, (size_t)td * 4, P->x, (size_t)H * 4,
                                         (size_t)H * 4, (size_t)S, cudaMemcpyDeviceToDevice, st),
                    "extract", 0);
            slot++;
        }
    }
    return E->rc;
}

static int q3_run(iris_cuda_qwen3_t *m) {
    q3_plan_t *P = &m->plan;
    if (iris_fault("launch")) return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected launch failure");
    if (P->graph_ok && P->graph_mode != m->mode) {
        cudaGraphExecDestroy(P->gexec);
        cudaGraphDestroy(P->graph);
        P->graph_ok = 0;
    }
    if (!P->graph_ok) {
        static int no_graph = -1;
        if (no_graph < 0) no_graph = getenv("IRIS_CUDA_NO_GRAPH") ? 1 : 0;
        q3_enq_t E;
        memset(&E, 0, sizeof(E));
        if (no_graph) {
            int rc = q3_enqueue(m, &E);
            iris_count_launch(E.kernels);
            return rc;
        }
        cudaError_t e = cudaStreamBeginCapture(g_rt.stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return iris_cuda_check(e, "begin capture");
        int rc = q3_enqueue(m, &E);
        cudaGraph_t g = NULL;
        e = cudaStreamEndCapture(g_rt.stream, &g);
        if (rc) { if (g) cudaGraphDestroy(g); return rc; }
        if (e != cudaSuccess) return iris_cuda_check(e, "end capture");
        e = cudaGraphInstantiate(&P->gexec, g, 0);
        if (e != cudaSuccess) { cudaGraphDestroy(g); return iris_cuda_check(e, "graph instantiate"); }
        P->graph = g;
        P->graph_ok = 1;
        P->graph_mode = m->mode;
        P->graph_kernels = E.kernels;
    }
    iris_count_launch(P->graph_kernels);
    return iris_cuda_check(cudaGraphLaunch(P->gexec, g_rt.stream), "graph launch");
}

/* ids / mask host arrays -> plan inputs (mask as bytes for the attention) */
static int q3_inputs(iris_cuda_qwen3_t *m, const int *ids, const int *mask, int S) {
    if (!m || !ids) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (S < 1 || S > Q3_MAX_SEQ) return iris_fail(IRIS_CUDA_ERR_ARG, "sequence length %d (1..%d)", S, Q3_MAX_SEQ);
    int rc = q3_plan_ensure(m, S);
    if (rc) return rc;
    uint8_t mb[Q3_MAX_SEQ];
    for (int i = 0; i < S; i++) mb[i] = mask ? (mask[i] != 0) : 1;
    q3_plan_t *P = &m->plan;
    rc = iris_cuda_check(cudaMemcpyAsync(P->ids, ids, (size_t)S * 4, cudaMemcpyHostToDevice, g_rt.stream), "ids");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(P->mask, mb, (size_t)S, cudaMemcpyHostToDevice, g_rt.stream), "mask");
    /* mb lives on this stack frame: wait for the copy before returning */
    if (!rc) rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "inputs");
    return rc;
}

int iris_cuda_qwen3_forward_dev(iris_cuda_qwen3_t *m, const int *input_ids, const int *attention_mask, int seq_len,
                                float *d_out) {
    if (!d_out) return iris_fail(IRIS_CUDA_ERR_ARG, "null output");
    int rc = q3_inputs(m, input_ids, attention_mask, seq_len);
    if (!rc) rc = q3_run(m);
    if (!rc)
        rc = iris_cuda_check(cudaMemcpyAsync(d_out, m->plan.out, (size_t)seq_len * iris_cuda_qwen3_text_dim(m) * 4,
                                             cudaMemcpyDeviceToDevice, g_rt.stream),
                             "output");
    return rc;
}

float *iris_cuda_qwen3_forward(iris_cuda_qwen3_t *m, const int *input_ids, const int *attention_mask, int seq_len) {
    if (q3_inputs(m, input_ids, attention_mask, seq_len)) return NULL;
    const size_t n = (size_t)seq_len * iris_cuda_qwen3_text_dim(m);
    float *out = (float *)malloc(n * 4);
    if (!out) { iris_fail(IRIS_CUDA_ERR_OOM, "output"); return NULL; }
    int rc = q3_run(m);
    if (!rc) rc = iris_d2h_staged(out, m->plan.out, n * 4, "d2h");
    if (rc) { free(out); return NULL; }
    return out;
}

uint64_t iris_cuda_qwen3_graph_kernels(const iris_cuda_qwen3_t *m) { return m ? m->plan.graph_kernels : 0; }

/* Time every kernel of one forward at the last sequence length (no graph; an
 * event after each launch).  Returns the number of entries or a negative
 * status. */
int iris_cuda_qwen3_profile(iris_cuda_qwen3_t *m, iris_cuda_kernel_time_t *out, int max_entries) {
    if (!m || !out || max_entries <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!m->plan.valid) return iris_fail(IRIS_CUDA_ERR_ARG, "run a forward first (no plan)");
    cudaEvent_t *ev = (cudaEvent_t *)calloc((size_t)max_entries + 1, sizeof(cudaEvent_t));
    if (!ev) return iris_fail(IRIS_CUDA_ERR_OOM, "events");
    int rc = 0, n = 0;
    for (int i = 0; i <= max_entries && !rc; i++) rc = iris_cuda_check(cudaEventCreate(&ev[i]), "event");
    if (!rc) {
        q3_enq_t E;
        memset(&E, 0, sizeof(E));
        E.prof = out;
        E.ev = ev;
        E.maxprof = max_entries;
        cudaEventRecord(ev[0], g_rt.stream);
        rc = q3_enqueue(m, &E);
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
