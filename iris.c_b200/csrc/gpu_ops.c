/*
 * The iris_gpu_* device-tensor surface of iris_metal.h (:155-600),
 * implemented on CUDA with the same names, signatures and failure
 * conventions (NULL / 0 on failure, void ops report through
 * iris_cuda_last_error()).  It lets the reference's bf16 block code
 * (iris_transformer_flux.c:2037-2292, :3243-3751) queue its ops on this
 * backend.  The fused model path (flux.c) does not use these entry points;
 * they exist for callers that drive the transformer op by op.
 *
 * Tensors are device buffers, f32 or bf16 ("f16" in the Metal naming).
 * bf16 weights passed as host pointers are uploaded on first use and cached
 * by address, like the Metal backend's bf16 weight cache (iris_metal.m:1001).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "iris_internal.h"

struct iris_gpu_tensor {
    void *d;
    size_t n;
    int bf16;
    int persistent;
};

static iris_gpu_tensor_t tensor_new(size_t n, int bf16) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_gpu_tensor_t t = (iris_gpu_tensor_t)calloc(1, sizeof(*t));
    if (!t) return NULL;
    t->d = iris_dmalloc(n * (bf16 ? 2 : 4));
    if (!t->d) { free(t); return NULL; }
    t->n = n;
    t->bf16 = bf16;
    return t;
}

iris_gpu_tensor_t iris_gpu_tensor_alloc(size_t n) { return tensor_new(n, 0); }
iris_gpu_tensor_t iris_gpu_tensor_alloc_f16(size_t n) { return tensor_new(n, 1); }

iris_gpu_tensor_t iris_gpu_tensor_alloc_persistent(size_t n) {
    iris_gpu_tensor_t t = tensor_new(n, 0);
    if (t) t->persistent = 1;
    return t;
}

void iris_gpu_tensor_set_persistent(iris_gpu_tensor_t t, int p) {
    if (t) t->persistent = p;
}

iris_gpu_tensor_t iris_gpu_tensor_create(const float *data, size_t n) {
    iris_gpu_tensor_t t = tensor_new(n, 0);
    if (!t) return NULL;
    if (data && iris_cuda_check(cudaMemcpyAsync(t->d, data, n * 4, cudaMemcpyHostToDevice,
                                                g_rt.stream), "tensor_create")) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

/* f32 staging buffer on the device, grown on demand */
static float *scratch_f32(size_t n) {
    static float *buf = NULL;
    static size_t cap = 0;
    if (n > cap) {
        cudaStreamSynchronize(g_rt.stream);
        iris_dfree(buf);
        buf = (float *)iris_dmalloc(n * 4);
        cap = buf ? n : 0;
    }
    return buf;
}

iris_gpu_tensor_t iris_gpu_tensor_create_bf16(const float *data, size_t n) {
    iris_gpu_tensor_t t = tensor_new(n, 1);
    if (!t) return NULL;
    t->persistent = 1;
    if (data) {
        float *s = scratch_f32(n);
        if (!s || iris_cuda_check(cudaMemcpyAsync(s, data, n * 4, cudaMemcpyHostToDevice, g_rt.stream), "h2d") ||
            iris_cuda_check(iris_launch_f32_to_bf16(s, t->d, (long)n, g_rt.stream), "to_bf16")) {
            iris_gpu_tensor_free(t);
            return NULL;
        }
        iris_count_launch(1);
        cudaStreamSynchronize(g_rt.stream);
    }
    return t;
}

void iris_gpu_tensor_read(iris_gpu_tensor_t t, float *out) {
    if (!t || !out) return;
    if (t->bf16) {
        float *s = scratch_f32(t->n);
        if (!s) return;
        iris_count_launch(1);
        if (iris_cuda_check(iris_launch_bf16_to_f32(t->d, s, (long)t->n, g_rt.stream), "to_f32")) return;
        iris_cuda_check(cudaMemcpyAsync(out, s, t->n * 4, cudaMemcpyDeviceToHost, g_rt.stream), "d2h");
    } else {
        iris_cuda_check(cudaMemcpyAsync(out, t->d, t->n * 4, cudaMemcpyDeviceToHost, g_rt.stream), "d2h");
    }
    cudaStreamSynchronize(g_rt.stream);
}

void iris_gpu_tensor_write(iris_gpu_tensor_t t, const float *data) {
    if (!t || !data) return;
    if (t->bf16) {
        float *s = scratch_f32(t->n);
        if (!s) return;
        iris_cuda_check(cudaMemcpyAsync(s, data, t->n * 4, cudaMemcpyHostToDevice, g_rt.stream), "h2d");
        iris_count_launch(1);
        iris_cuda_check(iris_launch_f32_to_bf16(s, t->d, (long)t->n, g_rt.stream), "to_bf16");
        cudaStreamSynchronize(g_rt.stream);
    } else {
        iris_cuda_check(cudaMemcpyAsync(t->d, data, t->n * 4, cudaMemcpyHostToDevice, g_rt.stream), "h2d");
    }
}

void iris_gpu_tensor_free(iris_gpu_tensor_t t) {
    if (!t) return;
    cudaStreamSynchronize(g_rt.stream);
    iris_dfree(t->d);
    free(t);
}

size_t iris_gpu_tensor_size(iris_gpu_tensor_t t) { return t ? t->n : 0; }
int iris_gpu_tensor_is_f16(iris_gpu_tensor_t t) { return t ? t->bf16 : 0; }

iris_gpu_tensor_t iris_gpu_tensor_f32_to_bf16(iris_gpu_tensor_t f) {
    if (!f || f->bf16) return NULL;
    iris_gpu_tensor_t t = tensor_new(f->n, 1);
    if (!t) return NULL;
    iris_count_launch(1);
    if (iris_cuda_check(iris_launch_f32_to_bf16((const float *)f->d, t->d, (long)f->n, g_rt.stream), "to_bf16")) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

iris_gpu_tensor_t iris_gpu_tensor_bf16_to_f32(iris_gpu_tensor_t b) {
    if (!b || !b->bf16) return NULL;
    iris_gpu_tensor_t t = tensor_new(b->n, 0);
    if (!t) return NULL;
    iris_count_launch(1);
    if (iris_cuda_check(iris_launch_bf16_to_f32(b->d, (float *)t->d, (long)b->n, g_rt.stream), "to_f32")) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

int iris_gpu_convert_f32_to_bf16_into(iris_gpu_tensor_t out, iris_gpu_tensor_t in) {
    if (!out || !in || !out->bf16 || in->bf16 || out->n < in->n) return 0;
    iris_count_launch(1);
    return iris_cuda_check(iris_launch_f32_to_bf16((const float *)in->d, out->d, (long)in->n, g_rt.stream),
                           "to_bf16") == 0;
}

int iris_gpu_convert_bf16_to_f32_into(iris_gpu_tensor_t out, iris_gpu_tensor_t in) {
    if (!out || !in || out->bf16 || !in->bf16 || out->n < in->n) return 0;
    iris_count_launch(1);
    return iris_cuda_check(iris_launch_bf16_to_f32(in->d, (float *)out->d, (long)in->n, g_rt.stream),
                           "to_f32") == 0;
}

void iris_gpu_sync(void) {
    if (g_rt.initialized) cudaStreamSynchronize(g_rt.stream);
}
/* Work is queued on one stream in order; batches need no extra encoding. */
void iris_gpu_batch_begin(void) {}
void iris_gpu_batch_end(void) { iris_gpu_sync(); }

/* ------------------------------------------------------------------ weight cache */
typedef struct {
    const uint16_t *host;
    size_t n;
    uint16_t *dev;
    int rows, cols;
    CUtensorMap tm;
} wcache_t;

static wcache_t *g_wc = NULL;
static int g_wc_n = 0, g_wc_cap = 0;

static wcache_t *weight_lookup(const uint16_t *w, int rows, int cols) {
    for (int i = 0; i < g_wc_n; i++)
        if (g_wc[i].host == w && g_wc[i].rows == rows && g_wc[i].cols == cols) return &g_wc[i];
    if (g_wc_n == g_wc_cap) {
        int nc = g_wc_cap ? 2 * g_wc_cap : 256;
        wcache_t *p = (wcache_t *)realloc(g_wc, sizeof(wcache_t) * (size_t)nc);
        if (!p) return NULL;
        g_wc = p;
        g_wc_cap = nc;
    }
    wcache_t *e = &g_wc[g_wc_n];
    memset(e, 0, sizeof(*e));
    e->n = (size_t)rows * cols;
    e->dev = (uint16_t *)iris_dmalloc(e->n * 2);
    if (!e->dev) return NULL;
    if (iris_h2d(e->dev, w, e->n * 2) ||
        iris_make_tmap_bf16(&e->tm, e->dev, (uint64_t)rows, (uint64_t)cols, (uint64_t)cols,
                            (rows % 256 == 0) ? 256 : 128)) {
        iris_dfree(e->dev);
        return NULL;
    }
    e->host = w;
    e->rows = rows;
    e->cols = cols;
    g_wc_n++;
    return e;
}

int iris_gpu_linear_bf16_native_into(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const uint16_t *W,
                                     int seq, int in_dim, int out_dim) {
    if (!out || !x || !W || !x->bf16 || !out->bf16) return 0;
    if (in_dim % 64 || out_dim % 128 || x->n < (size_t)seq * in_dim || out->n < (size_t)seq * out_dim) {
        iris_fail(IRIS_CUDA_ERR_ARG, "linear: unsupported shape %dx%d->%d", seq, in_dim, out_dim);
        return 0;
    }
    wcache_t *wc = weight_lookup(W, out_dim, in_dim);
    if (!wc) return 0;
    IrisGemmParams p;
    memset(&p, 0, sizeof(p));
    if (iris_make_tmap_bf16(&p.tmap_a, x->d, (uint64_t)seq, (uint64_t)in_dim, (uint64_t)in_dim, 128))
        return 0;
    p.tmap_b[0] = wc->tm;
    p.ngroups = 1;
    p.rows[0] = seq;
    p.N = out_dim;
    p.K = in_dim;
    p.bn = (out_dim % 256 == 0) ? 256 : 128;
    p.mode = IRIS_EPI_BF16;
    p.out = out->d;
    p.ldo = out_dim;
    p.status = g_rt.d_status;
    iris_count_launch(1);
    return iris_cuda_check(iris_launch_gemm(&p, g_rt.num_sms, g_rt.stream), "linear") == 0;
}

iris_gpu_tensor_t iris_gpu_linear_bf16_native(iris_gpu_tensor_t x, const uint16_t *W, int seq,
                                              int in_dim, int out_dim) {
    iris_gpu_tensor_t out = tensor_new((size_t)seq * out_dim, 1);
    if (!out) return NULL;
    if (!iris_gpu_linear_bf16_native_into(out, x, W, seq, in_dim, out_dim)) {
        iris_gpu_tensor_free(out);
        return NULL;
    }
    return out;
}

/* ------------------------------------------------------------------ norms / rope */
/* bf16 tensor -> f32 device scratch of its own (small vectors) */
static float *vec_f32(iris_gpu_tensor_t t, size_t n, float *dst) {
    if (!t) return NULL;
    iris_count_launch(1);
    if (t->bf16) {
        if (iris_launch_bf16_to_f32(t->d, dst, (long)n, g_rt.stream) != cudaSuccess) return NULL;
    } else {
        if (cudaMemcpyAsync(dst, t->d, n * 4, cudaMemcpyDeviceToDevice, g_rt.stream) != cudaSuccess)
            return NULL;
    }
    return dst;
}

void iris_gpu_adaln_norm_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t x, iris_gpu_tensor_t shift,
                              iris_gpu_tensor_t scale, int seq, int hidden, float eps) {
    if (!out || !x || !shift || !scale || !out->bf16) return;
    size_t n = (size_t)seq * hidden;
    float *s = scratch_f32(n + 2 * (size_t)hidden);
    if (!s) return;
    float *xf = s, *sh = s + n, *sc = s + n + hidden;
    if (x->bf16) {
        iris_count_launch(1);
        iris_launch_bf16_to_f32(x->d, xf, (long)n, g_rt.stream);
    } else {
        cudaMemcpyAsync(xf, x->d, n * 4, cudaMemcpyDeviceToDevice, g_rt.stream);
    }
    if (!vec_f32(shift, (size_t)hidden, sh) || !vec_f32(scale, (size_t)hidden, sc)) return;
    iris_count_launch(1);
    iris_cuda_check(iris_launch_adaln(xf, hidden, out->d, hidden, seq, hidden, sh, sc, NULL, NULL,
                                      seq, eps, g_rt.stream), "adaln");
}

void iris_gpu_qk_rms_norm_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k, iris_gpu_tensor_t qw,
                               iris_gpu_tensor_t kw, int seq, int heads, int head_dim, float eps) {
    if (!q || !k || head_dim != 128 || !q->bf16 || !k->bf16) return;
    float *s = scratch_f32(256);
    if (!s || !vec_f32(qw, 128, s) || !vec_f32(kw, 128, s + 128)) return;
    iris_count_launch(2);
    iris_cuda_check(iris_launch_head_rmsnorm_rope(q->d, heads * 128, seq, heads, s, eps, NULL, NULL,
                                                  g_rt.stream), "qk_norm");
    iris_cuda_check(iris_launch_head_rmsnorm_rope(k->d, heads * 128, seq, heads, s + 128, eps, NULL,
                                                  NULL, g_rt.stream), "qk_norm");
}

/* Upload [rows, 128] duplicated-pair host tables as a [rows, 64] device table. */
static int upload_rope(float *dc, float *ds, const float *hc, const float *hs, int rows) {
    size_t n = (size_t)rows * 64;
    float *tmp = (float *)malloc(n * 2 * sizeof(float));
    if (!tmp) return -1;
    for (size_t i = 0; i < n; i++) {
        tmp[i] = hc[2 * i];
        tmp[n + i] = hs[2 * i];
    }
    int rc = iris_h2d(dc, tmp, n * 4) || iris_h2d(ds, tmp + n, n * 4);
    free(tmp);
    return rc;
}

void iris_gpu_rope_unified_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *txt_cos,
                                const float *txt_sin, const float *img_cos, const float *img_sin,
                                const float *img_cos_k, const float *img_sin_k, int seq,
                                int img_offset, int heads, int head_dim, int axis_dim) {
    (void)axis_dim;
    if (!q || !k || head_dim != 128 || img_offset < 0 || img_offset > seq) return;
    int n_img = seq - img_offset;
    cudaStreamSynchronize(g_rt.stream);
    float *s = scratch_f32((size_t)seq * 64 * 4);
    if (!s) return;
    float *qc = s, *qs = s + (size_t)seq * 64, *kc = s + (size_t)2 * seq * 64, *ks = s + (size_t)3 * seq * 64;
    if (img_offset && upload_rope(qc, qs, txt_cos, txt_sin, img_offset)) return;
    if (n_img && upload_rope(qc + (size_t)img_offset * 64, qs + (size_t)img_offset * 64, img_cos, img_sin, n_img))
        return;
    const float *kcp = qc, *ksp = qs;
    if (img_cos_k && img_sin_k) {
        cudaMemcpyAsync(kc, qc, (size_t)img_offset * 64 * 4, cudaMemcpyDeviceToDevice, g_rt.stream);
        cudaMemcpyAsync(ks, qs, (size_t)img_offset * 64 * 4, cudaMemcpyDeviceToDevice, g_rt.stream);
        if (n_img && upload_rope(kc + (size_t)img_offset * 64, ks + (size_t)img_offset * 64, img_cos_k,
                                 img_sin_k, n_img))
            return;
        kcp = kc;
        ksp = ks;
    }
    iris_count_launch(2);
    iris_cuda_check(iris_launch_head_rmsnorm_rope(q->d, heads * 128, seq, heads, NULL, 0.f, qc, qs,
                                                  g_rt.stream), "rope");
    iris_cuda_check(iris_launch_head_rmsnorm_rope(k->d, heads * 128, seq, heads, NULL, 0.f, kcp, ksp,
                                                  g_rt.stream), "rope");
    cudaStreamSynchronize(g_rt.stream); /* scratch reuse */
}

void iris_gpu_rope_2d_bf16(iris_gpu_tensor_t x, const float *cos_freq, const float *sin_freq,
                           int seq, int heads, int head_dim, int axis_dim) {
    (void)axis_dim;
    if (!x || head_dim != 128) return;
    cudaStreamSynchronize(g_rt.stream);
    float *s = scratch_f32((size_t)seq * 128);
    if (!s || upload_rope(s, s + (size_t)seq * 64, cos_freq, sin_freq, seq)) return;
    iris_count_launch(1);
    iris_cuda_check(iris_launch_head_rmsnorm_rope(x->d, heads * 128, seq, heads, NULL, 0.f, s,
                                                  s + (size_t)seq * 64, g_rt.stream), "rope");
    cudaStreamSynchronize(g_rt.stream);
}

int iris_gpu_attention_fused_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                  iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads,
                                  int head_dim, float scale) {
    if (!out || !Q || !K || !V || head_dim != 128) return 0;
    if (!(out->bf16 && Q->bf16 && K->bf16 && V->bf16)) return 0;
    int ld = num_heads * 128;
    iris_count_launch(1);
    return iris_cuda_check(iris_launch_attention(Q->d, ld, K->d, V->d, ld, out->d, ld, seq_q, seq_k,
                                                 num_heads, scale, NULL, g_rt.stream), "attention") == 0;
}

void iris_gpu_silu_mul_bf16(iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int n) {
    if (!gate || !up) return;
    iris_count_launch(1);
    iris_cuda_check(iris_launch_silu_mul_bf16(gate->d, up->d, n, g_rt.stream), "silu_mul");
}

void iris_gpu_gated_add_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t gate, iris_gpu_tensor_t proj,
                             int seq, int hidden) {
    if (!out || !gate || !proj) return;
    iris_count_launch(1);
    iris_cuda_check(iris_launch_gated_add_bf16(out->d, gate->d, proj->d, seq, hidden, g_rt.stream),
                    "gated_add");
}

/* ------------------------------------------------------------------ layout copies */
static void copy2d(void *dst, int ldd, const void *src, int lds, int rows, int cols) {
    iris_cuda_check(cudaMemcpy2DAsync(dst, (size_t)ldd * 2, src, (size_t)lds * 2, (size_t)cols * 2,
                                      (size_t)rows, cudaMemcpyDeviceToDevice, g_rt.stream),
                    "copy2d");
}

void iris_gpu_concat_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b,
                              int seq_a, int seq_b, int hidden) {
    if (!out || !a || !b) return;
    copy2d(out->d, hidden, a->d, hidden, seq_a, hidden);
    copy2d((uint16_t *)out->d + (size_t)seq_a * hidden, hidden, b->d, hidden, seq_b, hidden);
}

void iris_gpu_slice_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t in, int seq_out, int hidden,
                             int start) {
    if (!out || !in) return;
    copy2d(out->d, hidden, (const uint16_t *)in->d + (size_t)start * hidden, hidden, seq_out, hidden);
}

void iris_gpu_split_qkv_mlp_bf16(iris_gpu_tensor_t fused, iris_gpu_tensor_t q, iris_gpu_tensor_t k,
                                 iris_gpu_tensor_t v, iris_gpu_tensor_t gate, iris_gpu_tensor_t up,
                                 int seq, int hidden, int mlp) {
    if (!fused || !q || !k || !v || !gate || !up) return;
    int ld = 3 * hidden + 2 * mlp;
    const uint16_t *f = (const uint16_t *)fused->d;
    copy2d(q->d, hidden, f, ld, seq, hidden);
    copy2d(k->d, hidden, f + hidden, ld, seq, hidden);
    copy2d(v->d, hidden, f + 2 * hidden, ld, seq, hidden);
    copy2d(gate->d, mlp, f + 3 * hidden, ld, seq, mlp);
    copy2d(up->d, mlp, f + 3 * hidden + mlp, ld, seq, mlp);
}

void iris_gpu_concat_attn_mlp_bf16(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp,
                                   iris_gpu_tensor_t out, int seq, int hidden, int mlp_hidden) {
    if (!attn || !mlp || !out) return;
    int ld = hidden + mlp_hidden;
    copy2d(out->d, ld, attn->d, hidden, seq, hidden);
    copy2d((uint16_t *)out->d + hidden, ld, mlp->d, mlp_hidden, seq, mlp_hidden);
}
