/*
 * The f32 ops of the iris_gpu_* surface (iris_metal.h:239-266, :353-402,
 * :529-566) and the host-pointer attention entry points (:613-660), which the
 * reference's Z-Image GPU path (iris_transformer_zimage.c:934-1556) and the
 * f32 fallbacks of its Flux blocks (iris_transformer_flux.c:1794-1946,
 * :2637-3040) call.  Same conventions as gpu_ops.c.
 *
 * Linears and attention run on the bf16 tensor cores with f32 accumulation:
 * f32 activations are rounded to bf16 on the way in (f32 host weights once,
 * when they are cached), results are written in f32.  The Metal backend's
 * f32 MPS GEMM keeps f32 operands; on the reference's bf16-valued weights the
 * difference is the rounding of the activations (relative 2^-9 per element).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "gpu_ops_internal.h"

static int is_f32(iris_gpu_tensor_t t, size_t n) { return t && !t->bf16 && t->n >= n; }

/* ------------------------------------------------------------------ linears */
/* out (f32 [seq, out_dim]) = x (f32 or bf16) * W^T (+ b) */
static int linear_into_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const void *W, int w_f32, const float *b,
                           int seq, int in_dim, int out_dim) {
    if (!out || !x || !W) return OP_FAIL("linear: null argument"), 0;
    if (out->bf16 || out->n < (size_t)seq * out_dim || x->n < (size_t)seq * in_dim)
        return OP_FAIL("linear: needs an f32 output of [%d, %d] and an input of [%d, %d]", seq, out_dim, seq,
                       in_dim),
               0;
    const size_t nx = (size_t)seq * in_dim;
    const void *xd = op_dev(x);
    float *od = (float *)op_dev(out);
    if (!xd || !od) return 0;
    void *xb = NULL;
    if (!x->bf16) {
        if (!(xb = op_scratch_get(nx * 2))) return 0;
        iris_count_launch(1);
        if (op_check(iris_launch_f32_to_bf16((const float *)xd, xb, (long)nx, g_rt.stream), "to_bf16")) {
            op_scratch_put(xb, nx * 2);
            return 0;
        }
        xd = xb;
    }
    int ok = op_linear(xd, seq, in_dim, W, w_f32, b, out_dim, od, 1);
    if (xb) op_scratch_put(xb, nx * 2);
    return ok;
}

iris_gpu_tensor_t iris_gpu_linear(iris_gpu_tensor_t x, const float *W, const float *b, int seq_len, int in_dim,
                                  int out_dim) {
    iris_gpu_tensor_t out = op_tensor_new((size_t)seq_len * out_dim, 0);
    if (out && !linear_into_f32(out, x, W, 1, b, seq_len, in_dim, out_dim)) {
        iris_gpu_tensor_free(out);
        return NULL;
    }
    return out;
}

int iris_gpu_linear_bf16_into(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const uint16_t *W_bf16, int seq_len,
                              int in_dim, int out_dim) {
    return linear_into_f32(out, x, W_bf16, 0, NULL, seq_len, in_dim, out_dim);
}

iris_gpu_tensor_t iris_gpu_linear_bf16(iris_gpu_tensor_t x, const uint16_t *W_bf16, int seq_len, int in_dim,
                                       int out_dim) {
    iris_gpu_tensor_t out = op_tensor_new((size_t)seq_len * out_dim, 0);
    if (out && !linear_into_f32(out, x, W_bf16, 0, NULL, seq_len, in_dim, out_dim)) {
        iris_gpu_tensor_free(out);
        return NULL;
    }
    return out;
}

/* ------------------------------------------------------------------ norms */
void iris_gpu_adaln_norm(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const float *shift, const float *scale, int seq,
                         int hidden, float eps) {
    const size_t n = (size_t)seq * hidden;
    if (!is_f32(out, n) || !is_f32(x, n) || !shift || !scale) {
        OP_FAIL("adaln_norm: needs f32 tensors of [%d, %d] and host shift/scale", seq, hidden);
        return;
    }
    const float *sh = op_vec(shift, (size_t)hidden, (size_t)hidden);
    const float *sc = op_vec(scale, (size_t)hidden, (size_t)hidden);
    const float *xd = (const float *)op_dev(x);
    float *od = (float *)op_dev(out);
    if (!sh || !sc || !xd || !od) return;
    iris_count_launch(1);
    op_check(iris_launch_layernorm_mod_f32(od, xd, sh, sc, seq, hidden, eps, g_rt.stream), "adaln_norm");
}

void iris_gpu_rms_norm_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const float *weight, int seq, int hidden,
                           float eps) {
    const size_t n = (size_t)seq * hidden;
    if (!is_f32(out, n) || !is_f32(x, n) || !weight) {
        OP_FAIL("rms_norm_f32: needs f32 tensors of [%d, %d] and a host weight", seq, hidden);
        return;
    }
    const float *w = op_vec(weight, (size_t)hidden, (size_t)hidden);
    const float *xd = (const float *)op_dev(x);
    float *od = (float *)op_dev(out);
    if (!w || !xd || !od) return;
    iris_count_launch(1);
    op_check(iris_launch_rmsnorm(xd, hidden, w, od, NULL, hidden, seq, hidden, eps, NULL, g_rt.stream),
                    "rms_norm");
}

void iris_gpu_qk_rms_norm(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *q_weight, const float *k_weight,
                          int seq, int heads, int head_dim, float eps) {
    const size_t n = (size_t)seq * heads * head_dim;
    if (!is_f32(q, n) || !is_f32(k, n) || !q_weight || !k_weight || head_dim != 128) {
        OP_FAIL("qk_rms_norm: needs f32 q/k with head_dim 128 and host weights");
        return;
    }
    const float *wq = op_vec(q_weight, 128, 128), *wk = op_vec(k_weight, 128, 128);
    float *qd = (float *)op_dev(q), *kd = (float *)op_dev(k);
    if (!wq || !wk || !qd || !kd) return;
    iris_count_launch(2);
    op_check(iris_launch_head_rmsnorm_f32(qd, seq, heads, wq, eps, g_rt.stream), "qk_norm");
    op_check(iris_launch_head_rmsnorm_f32(kd, seq, heads, wk, eps, g_rt.stream), "qk_norm");
}

/* ------------------------------------------------------------------ rope (f32) */
/* rows [r0, r0 + rows) of an f32 [*, heads * hd] tensor rotated by host tables [rows, hd] */
static void rope_f32_rows(iris_gpu_tensor_t x, int r0, int rows, int heads, int hd, const float *cs,
                          const float *sn) {
    if (rows <= 0) return;
    const float *dc = op_table(cs, (size_t)rows * hd), *ds = op_table(sn, (size_t)rows * hd);
    float *xd = (float *)op_dev(x);
    if (!dc || !ds || !xd) return;
    iris_count_launch(1);
    op_check(iris_launch_rope_pairs(xd + (size_t)r0 * heads * hd, 0, rows, heads, hd, dc, ds, hd,
                                           g_rt.stream),
                    "rope");
}

static int rope_f32_check(iris_gpu_tensor_t x, int seq, int heads, int hd) {
    if (!is_f32(x, (size_t)seq * heads * hd) || seq < 0 || heads <= 0 || hd <= 0 || (hd & 1))
        return OP_FAIL("rope: needs an f32 tensor of [%d, %d x %d]", seq, heads, hd), 0;
    return 1;
}

void iris_gpu_rope_single_f32(iris_gpu_tensor_t x, const float *cos_freq, const float *sin_freq, int seq, int heads,
                              int head_dim) {
    if (!rope_f32_check(x, seq, heads, head_dim)) return;
    rope_f32_rows(x, 0, seq, heads, head_dim, cos_freq, sin_freq);
}

void iris_gpu_rope_single_pair_f32(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *cos_freq,
                                   const float *sin_freq, int seq, int heads, int head_dim) {
    if (!rope_f32_check(q, seq, heads, head_dim) || !rope_f32_check(k, seq, heads, head_dim)) return;
    rope_f32_rows(q, 0, seq, heads, head_dim, cos_freq, sin_freq);
    rope_f32_rows(k, 0, seq, heads, head_dim, cos_freq, sin_freq);
}

void iris_gpu_rope_unified(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *txt_cos, const float *txt_sin,
                           const float *img_cos, const float *img_sin, int seq, int img_offset, int heads,
                           int head_dim, int axis_dim) {
    (void)axis_dim;
    if (!rope_f32_check(q, seq, heads, head_dim) || !rope_f32_check(k, seq, heads, head_dim)) return;
    if (img_offset < 0 || img_offset > seq) {
        OP_FAIL("rope_unified: img_offset %d outside [0, %d]", img_offset, seq);
        return;
    }
    iris_gpu_tensor_t t[2] = {q, k};
    for (int i = 0; i < 2; i++) {
        rope_f32_rows(t[i], 0, img_offset, heads, head_dim, txt_cos, txt_sin);
        rope_f32_rows(t[i], img_offset, seq - img_offset, heads, head_dim, img_cos, img_sin);
    }
}

/* ------------------------------------------------------------------ elementwise */
void iris_gpu_silu_mul(iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int n) {
    if (!is_f32(gate, (size_t)n) || !is_f32(up, (size_t)n)) {
        OP_FAIL("silu_mul: needs f32 tensors of %d elements", n);
        return;
    }
    float *g = (float *)op_dev(gate), *u = (float *)op_dev(up);
    if (!g || !u) return;
    iris_count_launch(1);
    op_check(iris_launch_silu_mul_f32(g, u, n, g_rt.stream), "silu_mul");
}

void iris_gpu_gated_add(iris_gpu_tensor_t out, const float *gate, iris_gpu_tensor_t proj, int seq, int hidden) {
    const size_t n = (size_t)seq * hidden;
    if (!is_f32(out, n) || !is_f32(proj, n) || !gate) {
        OP_FAIL("gated_add: needs f32 tensors of [%d, %d] and a host gate", seq, hidden);
        return;
    }
    const float *g = op_vec(gate, (size_t)hidden, (size_t)hidden);
    float *o = (float *)op_dev(out);
    const float *p = (const float *)op_dev(proj);
    if (!g || !o || !p) return;
    iris_count_launch(1);
    op_check(iris_launch_gated_add_f32(o, g, p, seq, hidden, g_rt.stream), "gated_add");
}

void iris_gpu_add_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b, int n) {
    if (!is_f32(out, (size_t)n) || !is_f32(a, (size_t)n) || !is_f32(b, (size_t)n)) {
        OP_FAIL("add_f32: needs f32 tensors of %d elements", n);
        return;
    }
    float *o = (float *)op_dev(out);
    const float *x = (const float *)op_dev(a), *y = (const float *)op_dev(b);
    if (!o || !x || !y) return;
    iris_count_launch(1);
    op_check(iris_launch_add_f32(o, x, y, n, g_rt.stream), "add_f32");
}

/* ------------------------------------------------------------------ attention (f32 interface) */
/* out (f32) = softmax(Q K^T scale) V over f32 tensors [seq, heads * 128]:
 * Q, K, V rounded to bf16, bf16 attention, result widened to f32 */
static int attention_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K, iris_gpu_tensor_t V,
                         int seq_q, int seq_k, int heads, int head_dim, float scale) {
    const int ld = heads * head_dim;
    if (head_dim != 128 || !is_f32(out, (size_t)seq_q * ld) || !is_f32(Q, (size_t)seq_q * ld) ||
        !is_f32(K, (size_t)seq_k * ld) || !is_f32(V, (size_t)seq_k * ld))
        return OP_FAIL("attention: needs f32 tensors with head_dim 128"), 0;
    if (op_attention_bias() != 0.0f)
        return OP_FAIL("attention: the reference-token key bias (SREF strength) is not supported by this backend"),
               0;
    const size_t nq = (size_t)seq_q * ld, nk = (size_t)seq_k * ld;
    const float *qd = (const float *)op_dev(Q), *kd = (const float *)op_dev(K), *vd = (const float *)op_dev(V);
    float *od = (float *)op_dev(out);
    if (!qd || !kd || !vd || !od) return 0;
    char *buf = (char *)op_scratch_get((2 * nq + 2 * nk) * 2);
    if (!buf) return 0;
    void *qb = buf, *kb = buf + nq * 2, *vb = buf + (nq + nk) * 2, *ob = buf + (nq + 2 * nk) * 2;
    iris_count_launch(5);
    int rc = op_check(iris_launch_f32_to_bf16(qd, qb, (long)nq, g_rt.stream), "to_bf16");
    if (!rc) rc = op_check(iris_launch_f32_to_bf16(kd, kb, (long)nk, g_rt.stream), "to_bf16");
    if (!rc) rc = op_check(iris_launch_f32_to_bf16(vd, vb, (long)nk, g_rt.stream), "to_bf16");
    if (!rc)
        rc = op_check(iris_launch_attention(qb, ld, kb, vb, ld, ob, ld, seq_q, seq_k, heads, scale, NULL,
                                                   g_rt.stream),
                             "attention");
    if (!rc) rc = op_check(iris_launch_bf16_to_f32(ob, od, (long)nq, g_rt.stream), "to_f32");
    op_scratch_put(buf, (2 * nq + 2 * nk) * 2);
    return rc == 0;
}

int iris_gpu_attention_fused(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K, iris_gpu_tensor_t V,
                             int seq_q, int seq_k, int num_heads, int head_dim, float scale) {
    return attention_f32(out, Q, K, V, seq_q, seq_k, num_heads, head_dim, scale);
}

int iris_gpu_attention_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K, iris_gpu_tensor_t V,
                            int seq_q, int seq_k, int num_heads, int head_dim, float scale) {
    return attention_f32(out, Q, K, V, seq_q, seq_k, num_heads, head_dim, scale);
}

/* ------------------------------------------------------------------ host-pointer attention */
/* out/Q/K/V host f32 [seq, heads * 128] (iris_metal.h:649): uploaded, run as
 * above, result copied back before returning.  1 on success. */
int iris_metal_attention_fused(float *out, const float *Q, const float *K, const float *V, int seq_q, int seq_k,
                               int num_heads, int head_dim, float scale) {
    if (!out || !Q || !K || !V || head_dim != 128 || seq_q <= 0 || seq_k <= 0 || num_heads <= 0)
        return OP_FAIL("attention_fused (host): bad arguments"), 0;
    const size_t nq = (size_t)seq_q * num_heads * 128, nk = (size_t)seq_k * num_heads * 128;
    iris_gpu_tensor_t q = iris_gpu_tensor_create(Q, nq), k = iris_gpu_tensor_create(K, nk),
                      v = iris_gpu_tensor_create(V, nk), o = iris_gpu_tensor_alloc(nq);
    int ok = q && k && v && o && attention_f32(o, q, k, v, seq_q, seq_k, num_heads, 128, scale);
    if (ok) {
        iris_gpu_tensor_read(o, out);
        ok = cudaGetLastError() == cudaSuccess;
    }
    iris_gpu_tensor_free(q);
    iris_gpu_tensor_free(k);
    iris_gpu_tensor_free(v);
    iris_gpu_tensor_free(o);
    return ok;
}

/* Q, K, V host f32 in [heads, seq, head_dim] layout, out likewise
 * (iris_metal.h:613); each head is a contiguous [seq, 128] matrix, attended
 * as a one-head problem.  scores_scratch is not needed. */
void iris_metal_attention(float *out, const float *Q, const float *K, const float *V, float *scores_scratch,
                          int heads, int seq_q, int seq_k, int head_dim, float scale) {
    (void)scores_scratch;
    if (!out || !Q || !K || !V || head_dim != 128 || heads <= 0 || seq_q <= 0 || seq_k <= 0) {
        OP_FAIL("attention (host): bad arguments");
        return;
    }
    const size_t nq = (size_t)seq_q * 128, nk = (size_t)seq_k * 128;
    for (int h = 0; h < heads; h++)
        if (!iris_metal_attention_fused(out + h * nq, Q + h * nq, K + h * nk, V + h * nk, seq_q, seq_k, 1, 128,
                                        scale))
            return;
}
