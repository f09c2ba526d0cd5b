/*
 * SREF style controls for the Flux transformer on the GPU.
 *
 * Reference: iris_set_sref_csd (iris.c:487) with csd_mod_load / csd_mod_forward
 * (iris_csdmod.c), iris_transformer_set_csd_delta / _set_csd_skip (the delta is
 * added to the timestep embedding before the modulation linears,
 * iris_transformer_flux.c:3972, :4393, :4632; the CFG sampler skips it on the
 * unconditional branch, iris_sample.c:754-758), and iris_transformer_set_sref_bands
 * (:5153) with the K-side band scaling of the reference rows' RoPE in the single
 * blocks (set_kside_krope :1297, band_scale_ref_krope :1272, used at :3872).
 *
 * The CSD modulation MLP (fc1 -> SiLU -> fc2, times the strength) runs once on
 * the device; the delta stays there and one kernel adds it to temb in every
 * forward, gated by a device flag, so the CFG sampler toggles it per branch
 * without a new graph.  The band tables are built with the plan (flux.c) and
 * the single blocks' QKV epilogue rotates K with them.  The reference's
 * attention strength bias (sref_strength) exists only on its Metal path; its
 * CPU path, the parity target, does not apply it.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "flux_internal.h"

static const float k_one = 1.0f, k_zero = 0.0f;

void iris_flux_sref_release(iris_cuda_flux_t *tf) {
    if (!tf) return;
    iris_stream_drain();
    iris_dfree(tf->csd_delta);
    iris_dfree(tf->csd_on);
    tf->csd_delta = tf->csd_on = NULL;
}

int iris_flux_csd_branch(iris_cuda_flux_t *tf, int on) {
    if (!tf || !tf->csd_on) return 0;
    /* a pageable source is staged before the call returns; the copy is ordered on the stream */
    return iris_cuda_check(cudaMemcpyAsync(tf->csd_on, on ? &k_one : &k_zero, 4, cudaMemcpyHostToDevice,
                                           g_rt.stream), "csd flag");
}

float iris_flux_sref_band(const iris_cuda_flux_t *tf, int d) {
    /* s(d) = shf + (slf - shf) * (d / (half - 1))^2, half = 16 (:1276-1280) */
    const float dn = (float)d / 15.0f;
    return tf->sref_shf + (tf->sref_slf - tf->sref_shf) * dn * dn;
}

/* device delta [H] from a host vector (NULL clears) */
static int set_delta_dev(iris_cuda_flux_t *tf, const float *d_delta) {
    const int had = tf->csd_delta != NULL;
    if (!d_delta) {
        iris_flux_sref_release(tf);
        if (had) iris_flux_invalidate_plan(tf);  /* the graph loses the csd_delta node */
        return 0;
    }
    if (!tf->csd_delta) {
        tf->csd_delta = (float *)iris_dmalloc((size_t)tf->H * 4);
        tf->csd_on = (float *)iris_dmalloc(4);
        if (!tf->csd_delta || !tf->csd_on) {
            iris_flux_sref_release(tf);
            return iris_fail(IRIS_CUDA_ERR_OOM, "CSD delta");
        }
    }
    int rc = iris_cuda_check(cudaMemcpyAsync(tf->csd_delta, d_delta, (size_t)tf->H * 4, cudaMemcpyDeviceToDevice,
                                             g_rt.stream), "CSD delta");
    if (!rc) rc = iris_flux_csd_branch(tf, 1);
    if (!rc) rc = iris_stream_drain();
    if (!rc && !had) iris_flux_invalidate_plan(tf);
    return rc;
}

int iris_cuda_flux_set_csd_delta(iris_cuda_flux_t *tf, const float *delta) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!delta) return set_delta_dev(tf, NULL);
    float *d = (float *)iris_dmalloc((size_t)tf->H * 4);
    if (!d) return iris_fail(IRIS_CUDA_ERR_OOM, "CSD delta");
    int rc = iris_h2d(d, delta, (size_t)tf->H * 4);
    if (!rc) rc = set_delta_dev(tf, d);
    iris_dfree(d);
    return rc;
}

int iris_cuda_flux_set_csd_skip(iris_cuda_flux_t *tf, int skip) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    return iris_flux_csd_branch(tf, !skip);
}

int iris_cuda_flux_set_sref_bands(iris_cuda_flux_t *tf, float shf, float slf) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    /* out-of-range values mean "off", as in iris_transformer_set_sref_bands (:5153) */
    const float h = (shf >= 0.0f && shf <= 1.0f) ? shf : 1.0f, l = (slf >= 1.0f) ? slf : 1.0f;
    if (h != tf->sref_shf || l != tf->sref_slf) {
        tf->sref_shf = h;
        tf->sref_slf = l;
        iris_flux_invalidate_plan(tf);  /* the K-side tables belong to the plan */
    }
    return 0;
}

int iris_cuda_flux_set_sref_csd(iris_cuda_flux_t *tf, const char *csdmod_path, const float *csd, int csd_dim,
                                float scale) {
    if (!tf) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!csdmod_path || !*csdmod_path || !csd || scale == 0.0f) return set_delta_dev(tf, NULL);  /* off */
    st_model_t st;
    if (st_open_file(&st, csdmod_path)) return iris_fail(IRIS_CUDA_ERR_IO, "csd_mod: cannot open %s", csdmod_path);
    const st_tensor_t *f1 = st_find(&st, "fc1.weight"), *f2 = st_find(&st, "fc2.weight");
    const st_tensor_t *b1 = st_find(&st, "fc1.bias"), *b2 = st_find(&st, "fc2.bias");
    int rc = 0;
    float *h = NULL, *d = NULL;
    if (!f1 || !f2 || !b1 || !b2 || f1->ndim != 2 || f2->ndim != 2) {
        rc = iris_fail(IRIS_CUDA_ERR_IO, "csd_mod: missing/malformed fc1/fc2 tensors in %s", csdmod_path);
        goto out;
    }
    const int mlp = (int)f1->shape[0], cin = (int)f1->shape[1], hid = (int)f2->shape[0];
    if ((int)f2->shape[1] != mlp || cin != csd_dim || hid != tf->H) {
        rc = iris_fail(IRIS_CUDA_ERR_ARG, "iris_set_sref_csd: dim mismatch (csd %d/%d, hidden %d/%d)", cin, csd_dim,
                       hid, tf->H);
        goto out;
    }
    /* [fc1 w | fc1 b | fc2 w | fc2 b | csd | work | delta] */
    const size_t n1 = (size_t)mlp * cin, n2 = (size_t)hid * mlp;
    const size_t total = n1 + mlp + n2 + hid + cin + mlp + hid;
    h = (float *)malloc((n1 + mlp + n2 + hid) * 4);
    d = (float *)iris_dmalloc(total * 4);
    if (!h || !d) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "csd_mod"); goto out; }
    if (st_read_f32(&st, f1, h, n1) || st_read_f32(&st, b1, h + n1, mlp) || st_read_f32(&st, f2, h + n1 + mlp, n2) ||
        st_read_f32(&st, b2, h + n1 + mlp + n2, hid)) {
        rc = iris_fail(IRIS_CUDA_ERR_IO, "csd_mod: unreadable tensors in %s", csdmod_path);
        goto out;
    }
    float *w1 = d, *bb1 = w1 + n1, *w2 = bb1 + mlp, *bb2 = w2 + n2, *x = bb2 + hid, *work = x + cin, *delta = work + mlp;
    if ((rc = iris_h2d(d, h, (n1 + mlp + n2 + hid) * 4)) || (rc = iris_h2d(x, csd, (size_t)cin * 4))) goto out;
    cudaStream_t s = g_rt.stream;
    /* csd_mod_forward: work = fc1(csd); SiLU; delta = fc2(work); then * strength (iris.c:508-509) */
    rc = iris_cuda_check(iris_launch_ip_sgemm(x, cin, w1, cin, 1, bb1, work, mlp, 1, mlp, cin, s), "csd fc1");
    if (!rc) rc = iris_cuda_check(iris_launch_silu_f32(work, mlp, s), "csd silu");
    if (!rc) rc = iris_cuda_check(iris_launch_ip_sgemm(work, mlp, w2, mlp, 1, bb2, delta, hid, 1, hid, mlp, s), "csd fc2");
    if (!rc) rc = iris_cuda_check(iris_launch_ip_scale_rows(delta, 1, hid, 1, scale, scale, s), "csd scale");
    iris_count_launch(4);
    if (!rc) rc = set_delta_dev(tf, delta);
out:
    iris_stream_drain();
    iris_dfree(d);
    free(h);
    st_close(&st);
    return rc;
}
