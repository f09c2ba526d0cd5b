/*
 * Flux.2 Klein transformer on B200: weights resident in HBM as bf16, one
 * denoising step = one CUDA graph of fused kernels.
 *
 * Reference: iris_transformer_flux.c — loader :5300-5497, forward :3939-4326,
 * double block :2366-2614, single block :3761-3928, multi-reference forward
 * :4579-4840.
 *
 * Data layout in HBM
 *   hidden   f32  [S, H]   S = S_txt + S_img(+refs), rows in [TXT, IMG] order
 *                          for the whole step (the reference concatenates the
 *                          same way before the single blocks, :4110-4114, and
 *                          orders joint-attention K/V [TXT, IMG], :1899-1905)
 *   xmod     bf16 [S, H]   adaLN output = GEMM A operand
 *   q, k, v  bf16 [S, H]   written by the QKV GEMM epilogue after QK-RMSNorm+RoPE
 *   attn     bf16 [S, H]   double-block attention output
 *   mlp      bf16 [S, F]   SiLU(gate)*up (double blocks)
 *   cat      bf16 [S, H+F] single block [attention | SiLU(gate)*up]
 *   rope_pos u16  [S, 4]   RoPE position ids (T, H, W, L) per row; the QKV
 *                          epilogue evaluates cos / sin from them in registers
 * Weights (bf16, [out, in] row-major = K-major GEMM B operands)
 *   double   w_qkv[s] [3H, H] = to_q; to_k; to_v stacked, per stream s
 *            w_in[s]  [2F, H] = ff.linear_in with gate/up interleaved in
 *                              blocks of 128 rows (SwiGLU epilogue layout)
 *   single   w_fused  [3H+2F, H] = Q,K,V rows then interleaved gate/up
 *   w_mod    [17H, H] = double img 6H | double txt 6H | single 3H | final 2H
 *                      (all modulation linears in one GEMV per step)
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "flux_internal.h"

/* ------------------------------------------------------------------ load */
static uint16_t *walloc(iris_cuda_flux_t *tf, size_t numel) {
    uint16_t *p = (uint16_t *)iris_dmalloc(numel * 2);
    if (p) tf->weight_bytes += numel * 2;
    return p;
}

static int check_cfg(const iris_cuda_flux_config_t *c) {
    if (c->head_dim != 128) return iris_fail(IRIS_CUDA_ERR_ARG, "head_dim must be 128");
    if (c->hidden != c->heads * 128) return iris_fail(IRIS_CUDA_ERR_ARG, "hidden != heads*128");
    if (c->hidden % 256) return iris_fail(IRIS_CUDA_ERR_ARG, "hidden must be a multiple of 256");
    if (c->mlp % 128) return iris_fail(IRIS_CUDA_ERR_ARG, "mlp must be a multiple of 128");
    if (c->text_dim % 64 || c->channels % 128)
        return iris_fail(IRIS_CUDA_ERR_ARG, "text_dim %% 64 and channels %% 128 required");
    if (c->hidden > 8192) return iris_fail(IRIS_CUDA_ERR_ARG, "hidden > 8192 unsupported");
    return 0;
}

/* Row block [r0, r0+n) of a row-major [*, cols] device matrix -> dst (contiguous). */
static int copy_rows(uint16_t *dst, const uint16_t *src, size_t r0, size_t n, size_t cols) {
    return iris_cuda_check(cudaMemcpyAsync(dst, src + r0 * cols, n * cols * 2, cudaMemcpyDeviceToDevice,
                                           g_rt.stream), "weight rows");
}

/* Column block [c0, c0+w) of a row-major [rows, lds] device matrix -> dst
 * columns [d0, d0+w) of a row-major [rows, ldd] matrix. */
static int copy_cols(uint16_t *dst, size_t ldd, size_t d0, const uint16_t *src, size_t lds, size_t c0,
                     size_t w, size_t rows) {
    return iris_cuda_check(cudaMemcpy2DAsync(dst + d0, ldd * 2, src + c0, lds * 2, w * 2, rows,
                                             cudaMemcpyDeviceToDevice, g_rt.stream), "weight cols");
}

/* GEMM N-tile width for an output of N columns (256 when it divides N). */
static int bn_for(int N) { return N % 256 == 0 ? 256 : 128; }

/* Load and pack every weight of this rank's tensor-parallel shard (the whole
 * model when tp == 1).  Shard r of tp holds attention heads
 * [r*NH/tp, (r+1)*NH/tp) and MLP columns [r*F/tp, (r+1)*F/tp): the Q/K/V and
 * gate/up rows of those heads/columns, and the matching input columns of the
 * output and down projections.  Embedders, modulation and the final layer are
 * replicated. */
static int load_weights(iris_cuda_flux_t *tf, iris_wsrc_t *ws) {
    const int H = tf->H, F = tf->F, C = tf->C, T = tf->T, Hl = tf->Hl, Fl = tf->Fl;
    const size_t h0 = (size_t)tf->tp_rank * Hl, f0 = (size_t)tf->tp_rank * Fl;
    int rc = 0;
    char nm[256];
    /* tmp: a full source tensor | gate/up staging of the shard | norm staging */
    size_t full_n = (size_t)(3 * H + 2 * F) * H, stage_n = (size_t)2 * Fl * H;
    uint16_t *tmp = (uint16_t *)iris_dmalloc((full_n + stage_n + 512) * 2);
    if (!tmp) return IRIS_CUDA_ERR_OOM;
    uint16_t *stage = tmp + full_n, *ntmp = stage + stage_n;

#define CHK(x) do { if ((rc = (x)) != 0) goto done; } while (0)
#define ALLOC(p, n) do { if (!((p) = walloc(tf, (n)))) { rc = IRIS_CUDA_ERR_OOM; goto done; } } while (0)
    ALLOC(tf->w_x, (size_t)H * C);
    ALLOC(tf->w_ctx, (size_t)H * T);
    ALLOC(tf->w_t1, (size_t)H * 256);
    ALLOC(tf->w_t2, (size_t)H * H);
    ALLOC(tf->w_mod, (size_t)17 * H * H);
    ALLOC(tf->w_proj, (size_t)C * H);
    CHK(iris_wsrc_get(ws, "x_embedder.weight", (size_t)H * C, tf->w_x));
    CHK(iris_wsrc_get(ws, "context_embedder.weight", (size_t)H * T, tf->w_ctx));
    CHK(iris_wsrc_get(ws, "time_guidance_embed.timestep_embedder.linear_1.weight", (size_t)H * 256, tf->w_t1));
    CHK(iris_wsrc_get(ws, "time_guidance_embed.timestep_embedder.linear_2.weight", (size_t)H * H, tf->w_t2));
    CHK(iris_wsrc_get(ws, "double_stream_modulation_img.linear.weight", (size_t)6 * H * H, tf->w_mod));
    CHK(iris_wsrc_get(ws, "double_stream_modulation_txt.linear.weight", (size_t)6 * H * H,
                 tf->w_mod + (size_t)6 * H * H));
    CHK(iris_wsrc_get(ws, "single_stream_modulation.linear.weight", (size_t)3 * H * H,
                 tf->w_mod + (size_t)12 * H * H));
    CHK(iris_wsrc_get(ws, "norm_out.linear.weight", (size_t)2 * H * H, tf->w_mod + (size_t)15 * H * H));
    CHK(iris_wsrc_get(ws, "proj_out.weight", (size_t)C * H, tf->w_proj));
    CHK(iris_mk_tmap(&tf->tm_x, tf->w_x, H, C, C, 256));
    CHK(iris_mk_tmap(&tf->tm_ctx, tf->w_ctx, H, T, T, 256));
    CHK(iris_mk_tmap(&tf->tm_proj, tf->w_proj, C, H, H, 128));

    tf->dbl = (flux_dbl_t *)calloc((size_t)tf->cfg.n_double, sizeof(flux_dbl_t));
    tf->sgl = (flux_sgl_t *)calloc((size_t)tf->cfg.n_single, sizeof(flux_sgl_t));
    if (!tf->dbl || !tf->sgl) { rc = iris_fail(IRIS_CUDA_ERR_OOM, "block tables"); goto done; }

    static const char *qkv_name[2][3] = {{"attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"},
                                         {"attn.to_q", "attn.to_k", "attn.to_v"}};
    static const char *out_name[2] = {"attn.to_add_out", "attn.to_out.0"};
    static const char *ff_name[2] = {"ff_context", "ff"};
    static const char *qn_name[2] = {"attn.norm_added_q", "attn.norm_q"};
    static const char *kn_name[2] = {"attn.norm_added_k", "attn.norm_k"};
    for (int i = 0; i < tf->cfg.n_double; i++) {
        flux_dbl_t *b = &tf->dbl[i];
        for (int s = 0; s < 2; s++) {
            ALLOC(b->w_qkv[s], (size_t)3 * Hl * H);
            ALLOC(b->w_out[s], (size_t)H * Hl);
            ALLOC(b->w_in[s], (size_t)2 * Fl * H);
            ALLOC(b->w_down[s], (size_t)H * Fl);
            b->qn[s] = (float *)iris_dmalloc(128 * 4);
            b->kn[s] = (float *)iris_dmalloc(128 * 4);
            if (!b->qn[s] || !b->kn[s]) { rc = IRIS_CUDA_ERR_OOM; goto done; }
            for (int j = 0; j < 3; j++) {
                snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.weight", i, qkv_name[s][j]);
                CHK(iris_wsrc_get(ws, nm, (size_t)H * H, tmp));
                CHK(copy_rows(b->w_qkv[s] + (size_t)j * Hl * H, tmp, h0, Hl, H));
            }
            snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.weight", i, out_name[s]);
            CHK(iris_wsrc_get(ws, nm, (size_t)H * H, tmp));
            CHK(copy_cols(b->w_out[s], Hl, 0, tmp, H, h0, Hl, H));
            snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.linear_in.weight", i, ff_name[s]);
            CHK(iris_wsrc_get(ws, nm, (size_t)2 * F * H, tmp));
            CHK(copy_rows(stage, tmp, f0, Fl, H));
            CHK(copy_rows(stage + (size_t)Fl * H, tmp, F + f0, Fl, H));
            iris_count_launch(1);
            CHK(iris_cuda_check(iris_launch_interleave_gate_up(b->w_in[s], stage, Fl, H, g_rt.stream), nm));
            snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.linear_out.weight", i, ff_name[s]);
            CHK(iris_wsrc_get(ws, nm, (size_t)H * F, tmp));
            CHK(copy_cols(b->w_down[s], Fl, 0, tmp, F, f0, Fl, H));
            snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.weight", i, qn_name[s]);
            CHK(iris_wsrc_get_f32(ws, nm, 128, b->qn[s], ntmp));
            snprintf(nm, sizeof(nm), "transformer_blocks.%d.%s.weight", i, kn_name[s]);
            CHK(iris_wsrc_get_f32(ws, nm, 128, b->kn[s], ntmp + 128));
            CHK(iris_mk_tmap(&b->tm_qkv[s], b->w_qkv[s], 3 * Hl, H, H, bn_for(3 * Hl)));
            CHK(iris_mk_tmap(&b->tm_out[s], b->w_out[s], H, Hl, Hl, bn_for(H)));
            CHK(iris_mk_tmap(&b->tm_in[s], b->w_in[s], 2 * Fl, H, H, 256));
            CHK(iris_mk_tmap(&b->tm_down[s], b->w_down[s], H, Fl, Fl, bn_for(H)));
        }
    }
    for (int i = 0; i < tf->cfg.n_single; i++) {
        flux_sgl_t *b = &tf->sgl[i];
        ALLOC(b->w_fused, (size_t)(3 * Hl + 2 * Fl) * H);
        ALLOC(b->w_out, (size_t)H * (Hl + Fl));
        b->qn = (float *)iris_dmalloc(128 * 4);
        b->kn = (float *)iris_dmalloc(128 * 4);
        if (!b->qn || !b->kn) { rc = IRIS_CUDA_ERR_OOM; goto done; }
        snprintf(nm, sizeof(nm), "single_transformer_blocks.%d.attn.to_qkv_mlp_proj.weight", i);
        CHK(iris_wsrc_get(ws, nm, full_n, tmp));
        for (int j = 0; j < 3; j++)
            CHK(copy_rows(b->w_fused + (size_t)j * Hl * H, tmp, (size_t)j * H + h0, Hl, H));
        CHK(copy_rows(stage, tmp, (size_t)3 * H + f0, Fl, H));
        CHK(copy_rows(stage + (size_t)Fl * H, tmp, (size_t)3 * H + F + f0, Fl, H));
        iris_count_launch(1);
        CHK(iris_cuda_check(iris_launch_interleave_gate_up(b->w_fused + (size_t)3 * Hl * H, stage, Fl, H,
                                                           g_rt.stream), nm));
        /* linear2 input is [attention H | MLP F]: keep this shard's columns of both */
        snprintf(nm, sizeof(nm), "single_transformer_blocks.%d.attn.to_out.weight", i);
        CHK(iris_wsrc_get(ws, nm, (size_t)H * (H + F), tmp));
        CHK(copy_cols(b->w_out, Hl + Fl, 0, tmp, H + F, h0, Hl, H));
        CHK(copy_cols(b->w_out, Hl + Fl, Hl, tmp, H + F, H + f0, Fl, H));
        snprintf(nm, sizeof(nm), "single_transformer_blocks.%d.attn.norm_q.weight", i);
        CHK(iris_wsrc_get_f32(ws, nm, 128, b->qn, ntmp));
        snprintf(nm, sizeof(nm), "single_transformer_blocks.%d.attn.norm_k.weight", i);
        CHK(iris_wsrc_get_f32(ws, nm, 128, b->kn, ntmp + 128));
        CHK(iris_mk_tmap(&b->tm_fused, b->w_fused, 3 * Hl + 2 * Fl, H, H, 256));
        CHK(iris_mk_tmap(&b->tm_out, b->w_out, H, Hl + Fl, Hl + Fl, bn_for(H)));
    }
    tf->t_dev = (float *)iris_dmalloc(4 * 4);
    tf->sincos = (float *)iris_dmalloc(256 * 4);
    tf->temb_h = (float *)iris_dmalloc((size_t)H * 4);
    tf->temb = (float *)iris_dmalloc((size_t)H * 4);
    tf->mods = (float *)iris_dmalloc((size_t)17 * H * 4);
    if (!tf->t_dev || !tf->sincos || !tf->temb_h || !tf->temb || !tf->mods) {
        rc = IRIS_CUDA_ERR_OOM;
        goto done;
    }
    rc = iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "weight upload");
#undef CHK
#undef ALLOC
done:
    cudaStreamSynchronize(g_rt.stream);
    iris_dfree(tmp);
    return rc;
}

static void plan_free(flux_plan_t *P);

void iris_cuda_flux_free(iris_cuda_flux_t *tf) {
    if (!tf) return;
    iris_stream_drain();
    iris_flux_lora_release(tf);
    iris_flux_ip_release(tf);
    iris_flux_sref_release(tf);
    plan_free(&tf->plan);
    iris_dfree(tf->w_x); iris_dfree(tf->w_ctx); iris_dfree(tf->w_t1); iris_dfree(tf->w_t2);
    iris_dfree(tf->w_mod); iris_dfree(tf->w_proj);
    if (tf->dbl) {
        for (int i = 0; i < tf->cfg.n_double; i++)
            for (int s = 0; s < 2; s++) {
                iris_dfree(tf->dbl[i].w_qkv[s]); iris_dfree(tf->dbl[i].w_out[s]);
                iris_dfree(tf->dbl[i].w_in[s]); iris_dfree(tf->dbl[i].w_down[s]);
                iris_dfree(tf->dbl[i].qn[s]); iris_dfree(tf->dbl[i].kn[s]);
            }
        free(tf->dbl);
    }
    if (tf->sgl) {
        for (int i = 0; i < tf->cfg.n_single; i++) {
            iris_dfree(tf->sgl[i].w_fused); iris_dfree(tf->sgl[i].w_out);
            iris_dfree(tf->sgl[i].qn); iris_dfree(tf->sgl[i].kn);
        }
        free(tf->sgl);
    }
    iris_dfree(tf->t_dev); iris_dfree(tf->sincos); iris_dfree(tf->temb_h);
    iris_dfree(tf->temb); iris_dfree(tf->mods);
    free(tf);
}

static iris_cuda_flux_t *flux_new(const iris_cuda_flux_config_t *cfg, int tp_rank, int tp) {
    if (check_cfg(cfg)) return NULL;
    if (tp < 1 || tp_rank < 0 || tp_rank >= tp) {
        iris_fail(IRIS_CUDA_ERR_ARG, "tensor-parallel rank %d of %d", tp_rank, tp);
        return NULL;
    }
    /* each shard keeps whole heads in pairs (256-column GEMM tiles over Q|K|V
       and an aligned gate/up region) and whole 128-column MLP blocks */
    if (tp > 1 && (cfg->heads % (2 * tp) || cfg->mlp % (128 * tp))) {
        iris_fail(IRIS_CUDA_ERR_ARG, "tp=%d needs heads %% (2*tp) == 0 and mlp %% (128*tp) == 0", tp);
        return NULL;
    }
    iris_cuda_flux_t *tf = (iris_cuda_flux_t *)calloc(1, sizeof(*tf));
    if (!tf) { iris_fail(IRIS_CUDA_ERR_OOM, "model struct"); return NULL; }
    tf->cfg = *cfg;
    tf->H = cfg->hidden;
    tf->F = cfg->mlp;
    tf->C = cfg->channels;
    tf->T = cfg->text_dim;
    tf->NH = cfg->heads;
    tf->tp = tp;
    tf->tp_rank = tp_rank;
    tf->sref_shf = tf->sref_slf = 1.0f;
    tf->NHl = cfg->heads / tp;
    tf->Hl = tf->NHl * 128;
    tf->Fl = cfg->mlp / tp;
    return tf;
}

/* Parse transformer/config.json with the keys and defaults of the reference's
 * parse_transformer_config (iris_transformer_flux.c:395-455, defaults :5309-5320). */
static int parse_config(const char *model_dir, iris_cuda_flux_config_t *c) {
    c->hidden = 3072; c->heads = 24; c->head_dim = 128; c->mlp = 9216;
    c->n_double = 5; c->n_single = 20; c->text_dim = 7680; c->channels = 128;
    c->rope_theta = 2000.0f;
    char path[1200];
    snprintf(path, sizeof(path), "%s/transformer/config.json", model_dir);
    FILE *f = fopen(path, "rb");
    if (!f) return 0;
    char buf[8192];
    size_t n = fread(buf, 1, sizeof(buf) - 1, f);
    fclose(f);
    buf[n] = 0;
    double v, heads = 0, hd = 0;
    if (json_get_number(buf, "num_attention_heads", &v) == 0) heads = v;
    if (json_get_number(buf, "attention_head_dim", &v) == 0) hd = v;
    if (heads <= 0 || hd <= 0) return 0;
    c->heads = (int)heads;
    c->head_dim = (int)hd;
    c->hidden = c->heads * c->head_dim;
    double ratio = 3.0;
    if (json_get_number(buf, "mlp_ratio", &v) == 0 && v > 0) ratio = v;
    c->mlp = (int)(c->hidden * (float)ratio);
    if (json_get_number(buf, "num_layers", &v) == 0 && v > 0) c->n_double = (int)v;
    if (json_get_number(buf, "num_single_layers", &v) == 0 && v > 0) c->n_single = (int)v;
    if (json_get_number(buf, "joint_attention_dim", &v) == 0 && v > 0) c->text_dim = (int)v;
    if (json_get_number(buf, "in_channels", &v) == 0 && v > 0) c->channels = (int)v;
    if (json_get_number(buf, "rope_theta", &v) == 0 && v > 0) c->rope_theta = (float)v;
    return 0;
}

iris_cuda_flux_t *iris_cuda_flux_load(const char *model_dir) {
    return iris_cuda_flux_load_tp(model_dir, 0, 1);
}

iris_cuda_flux_t *iris_cuda_flux_load_tp(const char *model_dir, int tp_rank, int tp_size) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_cuda_flux_config_t cfg;
    parse_config(model_dir, &cfg);
    iris_cuda_flux_t *tf = flux_new(&cfg, tp_rank, tp_size);
    if (!tf) return NULL;
    snprintf(tf->model_dir, sizeof(tf->model_dir), "%s", model_dir);
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    char tdir[1200];
    snprintf(tdir, sizeof(tdir), "%s/transformer", model_dir);
    if (st_open_dir(&ws.st, tdir) != 0) {
        iris_fail(IRIS_CUDA_ERR_IO, "cannot open safetensors in %s", tdir);
        free(tf);
        return NULL;
    }
    int rc = load_weights(tf, &ws);
    st_close(&ws.st);
    iris_wsrc_free(&ws);
    if (rc) { iris_cuda_flux_free(tf); return NULL; }
    return tf;
}

iris_cuda_flux_t *iris_cuda_flux_random(const iris_cuda_flux_config_t *cfg, uint64_t seed,
                                        float std, int norm_unit) {
    return iris_cuda_flux_random_tp(cfg, seed, std, norm_unit, 0, 1);
}

iris_cuda_flux_t *iris_cuda_flux_random_tp(const iris_cuda_flux_config_t *cfg, uint64_t seed,
                                           float std, int norm_unit, int tp_rank, int tp_size) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_cuda_flux_t *tf = flux_new(cfg, tp_rank, tp_size);
    if (!tf) return NULL;
    tf->random = 1;
    tf->seed = seed;
    tf->std = std;
    tf->norm_unit = norm_unit;
    iris_wsrc_t ws;
    memset(&ws, 0, sizeof(ws));
    ws.random = 1;
    ws.seed = seed;
    ws.std = std;
    ws.norm_unit = norm_unit;
    if (load_weights(tf, &ws)) { iris_cuda_flux_free(tf); return NULL; }
    return tf;
}

int iris_cuda_flux_get_config(const iris_cuda_flux_t *tf, iris_cuda_flux_config_t *out) {
    if (!tf || !out) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    *out = tf->cfg;
    return 0;
}

size_t iris_cuda_flux_weight_bytes(const iris_cuda_flux_t *tf) { return tf ? tf->weight_bytes : 0; }

int iris_cuda_flux_read_weight(iris_cuda_flux_t *tf, const char *name, uint16_t *out, size_t numel) {
    if (!tf || !name || !out) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (tf->random) {
        uint16_t *d = (uint16_t *)iris_dmalloc(numel * 2);
        if (!d) return IRIS_CUDA_ERR_OOM;
        iris_wsrc_t ws;
        memset(&ws, 0, sizeof(ws));
        ws.random = 1; ws.seed = tf->seed; ws.std = tf->std; ws.norm_unit = tf->norm_unit;
        int rc = iris_wsrc_get(&ws, name, numel, d);
        if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, d, numel * 2, cudaMemcpyDeviceToHost,
                                                      g_rt.stream), "read weight");
        iris_stream_drain();
        iris_dfree(d);
        return rc;
    }
    st_model_t st;
    char tdir[1200];
    snprintf(tdir, sizeof(tdir), "%s/transformer", tf->model_dir);
    if (st_open_dir(&st, tdir) != 0) return iris_fail(IRIS_CUDA_ERR_IO, "cannot reopen %s", tdir);
    const st_tensor_t *t = st_find(&st, name);
    int rc = t ? st_read_bf16(&st, t, out, numel) : -1;
    st_close(&st);
    return rc ? iris_fail(IRIS_CUDA_ERR_IO, "tensor %s unreadable", name) : 0;
}

/* ------------------------------------------------------------------ plan */
static void plan_free(flux_plan_t *P) {
    if (P->graph_ok) {
        cudaGraphExecDestroy(P->gexec);
        cudaGraphDestroy(P->graph);
    }
    if (P->recv) P->xmod = NULL;  /* tensor-parallel xmod lives in the symmetric arena */
    iris_dfree(P->hidden); iris_dfree(P->lat_in); iris_dfree(P->out); iris_dfree(P->txt_f32);
    iris_dfree(P->rope_pos); iris_dfree(P->rope_spec); iris_dfree(P->xmod); iris_dfree(P->q);
    iris_dfree(P->k); iris_dfree(P->v); iris_dfree(P->attn); iris_dfree(P->mlp);
    iris_dfree(P->cat); iris_dfree(P->tok_img); iris_dfree(P->tok_txt);
    iris_dfree(P->ws);
    iris_dfree(P->ip_q); iris_dfree(P->ip_o);
    memset(P, 0, sizeof(*P));
}

void iris_flux_invalidate_plan(iris_cuda_flux_t *tf) {
    iris_stream_drain();
    plan_free(&tf->plan);
}

/* RoPE position ids per row and the per-pair spec, from which the QKV
 * epilogue evaluates the rotation in registers.  The frequencies are the
 * reference's own f32 values, base_freq[d] = 1/theta^(2d/32) for the T, H, W,
 * L axes (pairs 16a + d of axis a); text rows are (0, 0, 0, i), image rows
 * (T, y, x, 0) with T the reference latent's offset (compute_rope_2d :897,
 * compute_rope_2d_with_t_offset :961, compute_rope_text :1055).  SREF band
 * control scales cos and sin of the H and W pairs of the reference rows'
 * K (band_scale_ref_krope :1272), set up here as kscale + rope_k_row0. */
static int fill_rope(const iris_cuda_flux_t *tf, flux_plan_t *P, uint16_t *pos, IrisRopeSpec *spec) {
    memset(spec, 0, sizeof(*spec));
    for (int d = 0; d < 16; d++) {
        const float f = 1.0f / powf(tf->cfg.rope_theta, (float)(2 * d) / 32.0f);
        for (int a = 0; a < 4; a++) {
            spec->freq[16 * a + d] = f;
            iris_rope_set_axis(spec, 16 * a + d, a);
            spec->kscale[16 * a + d] = (a == 1 || a == 2) ? iris_flux_sref_band(tf, d) : 1.0f;
        }
    }
    int row = 0;
    for (int i = 0; i < P->s_txt; i++, row++) {
        uint16_t *p = pos + (size_t)row * 4;
        p[0] = p[1] = p[2] = 0;
        p[3] = (uint16_t)i;
    }
    for (int r = -1; r < P->num_refs; r++) {
        const int h = r < 0 ? P->img_h : P->ref_h[r], w = r < 0 ? P->img_w : P->ref_w[r];
        const int t = r < 0 ? 0 : P->ref_t[r];
        if (t < 0 || t > 65535) return iris_fail(IRIS_CUDA_ERR_ARG, "reference T offset %d out of range", t);
        for (int y = 0; y < h; y++)
            for (int x = 0; x < w; x++, row++) {
                uint16_t *p = pos + (size_t)row * 4;
                p[0] = (uint16_t)t; p[1] = (uint16_t)y; p[2] = (uint16_t)x; p[3] = 0;
            }
    }
    /* the band scale applies to the reference rows of the single blocks only */
    const int ref0 = P->s_txt + P->n_img;
    P->rope_k_row0 = (P->num_refs > 0 && (tf->sref_shf != 1.0f || tf->sref_slf != 1.0f)) ? ref0 : 0;
    return 0;
}

static int plan_ensure(iris_cuda_flux_t *tf, int s_txt, int img_h, int img_w,
                       const iris_cuda_ref_t *refs, int num_refs) {
    flux_plan_t *P = &tf->plan;
    if (num_refs < 0 || num_refs > MAXREFS) return iris_fail(IRIS_CUDA_ERR_ARG, "num_refs");
    if (s_txt <= 0 || img_h <= 0 || img_w <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "empty input");
    int same = P->valid && P->s_txt == s_txt && P->img_h == img_h && P->img_w == img_w &&
               P->num_refs == num_refs;
    for (int r = 0; same && r < num_refs; r++)
        same = P->ref_h[r] == refs[r].h && P->ref_w[r] == refs[r].w && P->ref_t[r] == refs[r].t_offset;
    if (same) return 0;
    iris_stream_drain();
    plan_free(P);
    int H = tf->H, C = tf->C, T = tf->T, Hl = tf->Hl, Fl = tf->Fl;
    P->s_txt = s_txt; P->img_h = img_h; P->img_w = img_w; P->num_refs = num_refs;
    P->n_img = img_h * img_w;
    P->n_img_total = P->n_img;
    for (int r = 0; r < num_refs; r++) {
        if (refs[r].h <= 0 || refs[r].w <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "empty ref");
        P->ref_h[r] = refs[r].h; P->ref_w[r] = refs[r].w; P->ref_t[r] = refs[r].t_offset;
        P->n_img_total += refs[r].h * refs[r].w;
    }
    int S = P->S = s_txt + P->n_img_total;
    size_t sH = (size_t)S * H, sHl = (size_t)S * Hl;
    const int tp = tf->tp;
    P->chunk = (S + tp - 1) / tp;
#define PA(p, bytes) do { if (!((p) = iris_dmalloc(bytes))) goto oom; } while (0)
    PA(P->hidden, (size_t)P->chunk * tp * H * 4);  /* whole chunks: the row all-gather of run_block */
    PA(P->lat_in, (size_t)C * P->n_img_total * 4);
    PA(P->out, (size_t)C * P->n_img * 4);
    PA(P->txt_f32, (size_t)s_txt * T * 4);
    if (S > 65535 || img_h > 65535 || img_w > 65535) {
        plan_free(P);
        return iris_fail(IRIS_CUDA_ERR_ARG, "sequence of %d rows: RoPE position ids are 16-bit", S);
    }
    PA(P->rope_pos, (size_t)S * 4 * sizeof(uint16_t));
    PA(P->rope_spec, sizeof(IrisRopeSpec));
    if (tp > 1) {
        /* collective: every rank plans the same shape at the same point */
        const size_t recv_b = (size_t)tp * P->chunk * H * 4, xmod_b = sH * 2;
        int rc = iris_comm_sym_init(4096 + recv_b + xmod_b + 1024);
        if (rc) { plan_free(P); return rc; }
        P->flags = (unsigned *)iris_comm_sym_alloc(4096);
        P->recv = (float *)iris_comm_sym_alloc(recv_b);
        P->xmod = (uint16_t *)iris_comm_sym_alloc(xmod_b);
        if (!P->flags || !P->recv || !P->xmod) { plan_free(P); return IRIS_CUDA_ERR_OOM; }
        for (int p = 0; p < tp; p++)  /* every peer's arena must be mapped before a kernel writes to it */
            if (!iris_comm_sym_peer(P->flags, p)) {
                plan_free(P);
                return iris_fail(IRIS_CUDA_ERR_CUDA, "peer %d arena not mapped", p);
            }
    } else {
        PA(P->xmod, sH * 2);
    }
    PA(P->q, sHl * 2);
    PA(P->k, sHl * 2);
    PA(P->v, sHl * 2);
    PA(P->attn, sHl * 2);
    PA(P->mlp, (size_t)S * Fl * 2);
    PA(P->cat, (size_t)S * (Hl + Fl) * 2);
    if (tf->ip) {
        PA(P->ip_q, (size_t)S * H * 2);
        PA(P->ip_o, (size_t)S * H * 2);
    }
    PA(P->tok_img, (size_t)P->n_img_total * C * 2);
    PA(P->tok_txt, (size_t)s_txt * T * 2);
    if (S < 512) {  /* few GEMM tiles: room for 16 K splits of the widest linear */
        P->ws_bytes = (size_t)16 * S * (size_t)(H + tf->F > T ? H + tf->F : T) * 4;
        PA(P->ws, P->ws_bytes);
    } else {
        /* the text embedder alone has few tiles (s_txt rows, K = the text width):
           room for 4 K splits of it; the other linears fill the GPU as they are */
        P->ws_bytes = (size_t)4 * s_txt * H * 4;
        PA(P->ws, P->ws_bytes);
    }
#undef PA
    /* a short sequence fits one box of S rows: smaller A stages, more of them
       in flight while the weights stream */
    P->a_box = S <= 128 ? (S + 7) & ~7 : 0;
    const int ab = P->a_box ? P->a_box : 128;
    if (iris_mk_tmap(&P->tm_xmod, P->xmod, S, H, H, ab) ||
        iris_mk_tmap(&P->tm_attn, P->attn, S, Hl, Hl, ab) ||
        iris_mk_tmap(&P->tm_mlp, P->mlp, S, Fl, Fl, ab) ||
        iris_mk_tmap(&P->tm_cat, P->cat, S, Hl + Fl, Hl + Fl, ab) ||
        iris_mk_tmap(&P->tm_tok_img, P->tok_img, P->n_img_total, C, C, ab) ||
        iris_mk_tmap(&P->tm_tok_txt, P->tok_txt, s_txt, T, T, ab)) {
        plan_free(P);
        return IRIS_CUDA_ERR_CUDA;
    }
    {
        uint16_t *pos = (uint16_t *)malloc((size_t)S * 4 * sizeof(uint16_t));
        IrisRopeSpec spec;
        if (!pos) goto oom;
        int rc = fill_rope(tf, P, pos, &spec);
        if (!rc)
            rc = iris_h2d(P->rope_pos, pos, (size_t)S * 4 * sizeof(uint16_t)) ||
                 iris_h2d(P->rope_spec, &spec, sizeof(spec));
        free(pos);
        if (rc) { plan_free(P); return rc < 0 ? rc : IRIS_CUDA_ERR_CUDA; }
    }
    P->valid = 1;
    return 0;
oom:
    plan_free(P);
    return iris_fail(IRIS_CUDA_ERR_OOM, "activation buffers for S=%d", S);
}

/* ------------------------------------------------------------------ forward */
static void gp_init(IrisGemmParams *p, const flux_plan_t *P, const CUtensorMap *ta, int N, int K, int mode) {
    memset(p, 0, sizeof(*p));
    p->ws = P->ws;  /* split-K workspace of short sequences */
    p->ws_bytes = P->ws_bytes;
    p->tmap_a = *ta;
    p->N = N;
    p->K = K;
    p->mode = mode;
    p->bn = 256;
    p->eps = 1e-6f;
    p->status = g_rt.d_status;
    p->b_static = 1;  /* every B of the forward is a resident weight */
    p->a_box = P->a_box;
}

static void gp_group(IrisGemmParams *p, int g, const CUtensorMap *tb, int row0, int rows) {
    p->tmap_b[g] = *tb;
    p->row0[g] = row0;
    p->rows[g] = rows;
    if (g + 1 > p->ngroups) p->ngroups = g + 1;
}

typedef struct {
    int rc;
    int fuse_ln;  /* a whole forward: a residual GEMM may apply the next block's adaLN */
    uint64_t kernels;
    /* live profiling (iris_cuda_flux_profile): an event after every launch */
    iris_cuda_kernel_time_t *prof;
    cudaEvent_t *ev;
    int nprof, maxprof;
} enq_t;

static void enq_x(enq_t *E, cudaError_t e, const char *what, double flops, double bytes) {
    E->kernels++;
    if (!E->rc && e != cudaSuccess) E->rc = iris_cuda_check(e, what);
    if (E->prof && E->nprof < E->maxprof) {
        iris_cuda_kernel_time_t *k = &E->prof[E->nprof];
        snprintf(k->name, sizeof(k->name), "%s", what);
        k->flops = flops;
        k->bytes = bytes;
        cudaEventRecord(E->ev[E->nprof + 1], g_rt.stream);
        E->nprof++;
    }
}

static void enq(enq_t *E, cudaError_t e, const char *what) { enq_x(E, e, what, 0.0, 0.0); }

static void enq_gemm(enq_t *E, const IrisGemmParams *p, const char *what) {
    double rows = (double)p->rows[0] + (p->ngroups > 1 ? (double)p->rows[1] : 0.0);
    double out_bytes = (p->mode == IRIS_EPI_RESID_GATE) ? 8.0 /* f32 read + write */
                       : (p->mode == IRIS_EPI_F32 || p->mode == IRIS_EPI_F32_NCHW) ? 4.0
                       : (p->mode == IRIS_EPI_SWIGLU) ? 1.0 /* N/2 bf16 outputs */
                       : 2.0;
    if (p->mode == IRIS_EPI_SINGLE) {
        /* 3H bf16 Q/K/V columns + (N-3H)/2 bf16 SwiGLU outputs */
        out_bytes = (3.0 * p->H * 2.0 + (p->N - 3.0 * p->H)) / p->N;
    }
    double bytes = rows * p->K * 2.0 + (double)p->ngroups * p->N * p->K * 2.0 + rows * p->N * out_bytes;
    int launches = 1;
    enq_x(E, iris_launch_gemm_ex(p, g_rt.num_sms, g_rt.stream, &launches), what, 2.0 * rows * p->N * p->K, bytes);
    E->kernels += (uint64_t)(launches - 1);
}

/* Tensor parallelism over NVLink peer memory (no collective library in the
 * forward).  Rows are owned in chunks (rank r: [r*chunk, (r+1)*chunk)).
 *  - an output projection scatters gate * (this shard's partial) of every row
 *    straight into the owning rank's receive buffer (slot = this rank) from
 *    its GEMM epilogue, so the transfer overlaps the remaining tiles, then
 *    signals arrival;
 *  - the next adaLN runs on the owned rows only: it waits for all ranks'
 *    partials, adds them in rank order to the f32 residual stream, normalises
 *    and writes the bf16 row into every rank's xmod, then signals;
 *  - a GEMM that reads xmod waits for every rank's rows before its first load.
 * Sync indices count from per-rank device bases advanced at the end of each
 * call, so a captured forward graph replays correctly. */
static void tp_fill(const iris_cuda_flux_t *tf, IrisTpParams *t, unsigned wait_x) {
    const flux_plan_t *P = &tf->plan;
    memset(t, 0, sizeof(*t));
    if (tf->tp <= 1) return;
    t->size = tf->tp;
    t->rank = tf->tp_rank;
    t->chunk = P->chunk;
    for (int p = 0; p < tf->tp; p++) {
        t->recv[p] = (float *)iris_comm_sym_peer(P->recv, p);
        t->flags[p] = (unsigned *)iris_comm_sym_peer(P->flags, p);
    }
    t->wait_x = wait_x;
}

/* an output projection: gated residual update, or its scattered partial */
static void tp_resid(iris_cuda_flux_t *tf, IrisGemmParams *gp) {
    if (tf->tp <= 1) return;
    gp->mode = IRIS_EPI_TP_SCATTER;
    tp_fill(tf, &gp->tp, 0);
}

static void enq_allreduce(iris_cuda_flux_t *tf, enq_t *E) {
    (void)E;
    if (tf->tp <= 1) return;
    tf->plan.part_i++;  /* the GEMM just queued signals partial sync part_i */
    tf->plan.part_pending = 1;
}

/* a GEMM whose A operand is xmod: wait for every rank's rows */
static void tp_reads_xmod(iris_cuda_flux_t *tf, IrisGemmParams *gp) {
    if (tf->tp > 1) tp_fill(tf, &gp->tp, tf->plan.x_i);
}

/* adaLN of rows [row0, row0 + rows) into xmod (same rows); tensor-parallel:
 * this rank's chunk of them, with the pending partial update folded in */
static cudaError_t adaln_rows(iris_cuda_flux_t *tf, int row0, int rows, const float *sh0, const float *sc0,
                              const float *sh1, const float *sc1, int split) {
    flux_plan_t *P = &tf->plan;
    const int H = tf->H;
    if (tf->tp <= 1)
        return iris_launch_adaln(P->hidden + (size_t)row0 * H, H, P->xmod + (size_t)row0 * H, H, rows, H, sh0,
                                 sc0, sh1, sc1, split - row0, 1e-6f, g_rt.stream);
    IrisAdalnTpArgs a;
    memset(&a, 0, sizeof(a));
    a.x = P->hidden;
    a.row0 = tf->tp_rank * P->chunk;
    a.rows = P->S - a.row0 < P->chunk ? P->S - a.row0 : P->chunk;
    if (a.rows < 0) a.rows = 0;
    a.row_lo = row0;
    a.chunk = P->chunk;
    a.H = H;
    a.recv = P->recv;
    a.has_part = P->part_pending;
    a.part_index = P->part_i;
    for (int p = 0; p < tf->tp; p++) a.xmod[p] = iris_comm_sym_peer(P->xmod, p);
    a.shift0 = sh0; a.scale0 = sc0;
    a.shift1 = sh1 ? sh1 : sh0; a.scale1 = sc1 ? sc1 : sc0;
    a.split = split;
    a.eps = 1e-6f;
    tp_fill(tf, &a.tp, 0);
    a.status = g_rt.d_status;
    P->part_pending = 0;
    P->x_i++;  /* this launch signals xmod sync x_i */
    return iris_launch_adaln_tp(&a, g_rt.stream);
}

/* timestep embedding and every modulation vector of the step */
static void enq_mods(iris_cuda_flux_t *tf, enq_t *E) {
    cudaStream_t st = g_rt.stream;
    const int H = tf->H;
    enq(E, iris_launch_timestep_sincos(tf->t_dev, 1000.0f, tf->sincos, 256, st), "sincos");
    enq(E, iris_launch_gemv(tf->w_t1, tf->sincos, NULL, tf->temb_h, H, 256, 0, 1, st), "t_fc1");
    enq(E, iris_launch_gemv(tf->w_t2, tf->temb_h, NULL, tf->temb, H, H, 0, 0, st), "t_fc2");
    if (tf->csd_delta)  /* SREF CSD modulation: temb += delta unless skipped (:3972) */
        enq(E, iris_launch_axpy_dev(tf->temb, tf->csd_delta, tf->csd_on, H, st), "csd_delta");
    enq_x(E, iris_launch_gemv(tf->w_mod, tf->temb, NULL, tf->mods, 17 * H, H, 1, 0, st), "mods",
          2.0 * 17 * H * (double)H, 2.0 * 17 * H * (double)H);
}

/* input projections: hidden = [txt_in(ctx); img_in(latent tokens)] */
static void enq_embed(iris_cuda_flux_t *tf, enq_t *E) {
    flux_plan_t *P = &tf->plan;
    cudaStream_t st = g_rt.stream;
    const int H = tf->H, C = tf->C, T = tf->T, St = P->s_txt, Si = P->n_img_total;
    IrisGemmParams gp;
    size_t off = 0;
    int row = 0;
    for (int r = -1; r < P->num_refs; r++) {
        int n = r < 0 ? P->n_img : P->ref_h[r] * P->ref_w[r];
        enq(E, iris_launch_nchw_to_tokens(P->lat_in + off, C, n, P->tok_img + (size_t)row * C, C, st),
            "nchw_to_tokens");
        off += (size_t)C * n;
        row += n;
    }
    enq(E, iris_launch_f32_to_bf16(P->txt_f32, P->tok_txt, (long)St * T, st), "txt_bf16");
    gp_init(&gp, P, &P->tm_tok_txt, H, T, IRIS_EPI_F32);
    gp_group(&gp, 0, &tf->tm_ctx, 0, St);
    gp.out = P->hidden;
    gp.ldo = H;
    enq_gemm(E, &gp, "txt_in");
    gp_init(&gp, P, &P->tm_tok_img, H, C, IRIS_EPI_F32);
    gp_group(&gp, 0, &tf->tm_x, 0, Si);
    gp.out = P->hidden + (size_t)St * H;
    gp.ldo = H;
    enq_gemm(E, &gp, "img_in");
}

static void enq_ip(iris_cuda_flux_t *tf, enq_t *E, int blk, int row0, int rows);

/* double-stream block i: group 0 = text rows [0, St), group 1 = image rows */
/* Short sequences run the residual GEMMs split over K; their reduction then
 * also applies the adaLN that reads the updated rows next (one launch fewer
 * per residual update).  Only on one GPU, in a whole forward, and where the
 * next operation on the hidden state is that adaLN (no IP-Adapter update in
 * between). */
static int ip_active(const iris_cuda_flux_t *tf, int blk) {
    return tf->ip && blk < tf->ip->nb && tf->ip->h_scale[blk] != 0.0f;
}

static void fuse_next_adaln(iris_cuda_flux_t *tf, enq_t *E, IrisGemmParams *gp, const float *sh0,
                            const float *sc0, const float *sh1, const float *sc1, int split) {
    flux_plan_t *P = &tf->plan;
    if (!E->fuse_ln || tf->tp > 1 || iris_gemm_splits(gp, g_rt.num_sms) < 2) return;
    gp->ln_out = P->xmod;
    gp->ln_ld = tf->H;
    gp->ln_split = split;
    gp->ln_shift[0] = sh0;
    gp->ln_scale[0] = sc0;
    gp->ln_shift[1] = sh1 ? sh1 : sh0;
    gp->ln_scale[1] = sc1 ? sc1 : sc0;
    gp->ln_eps = 1e-6f;
    P->ln_pending = 1;
}

/* the adaLN about to be enqueued was applied by the previous reduction */
static int adaln_done(flux_plan_t *P) {
    const int d = P->ln_pending;
    P->ln_pending = 0;
    return d;
}

static void enq_double(iris_cuda_flux_t *tf, int i, enq_t *E) {
    flux_plan_t *P = &tf->plan;
    cudaStream_t st = g_rt.stream;
    const int H = tf->H, Hl = tf->Hl, Fl = tf->Fl, NHl = tf->NHl, St = P->s_txt, Si = P->n_img_total,
              S = P->S;
    const float *mi = tf->mods, *mt = tf->mods + (size_t)6 * H;
    flux_dbl_t *b = &tf->dbl[i];
    IrisGemmParams gp;
    if (!adaln_done(P))
        enq_x(E, adaln_rows(tf, 0, S, mt, mt + H, mi, mi + H, St), "adaln1", 0.0, 6.0 * S * (double)H);
    gp_init(&gp, P, &P->tm_xmod, 3 * Hl, H, IRIS_EPI_QKV);
    tp_reads_xmod(tf, &gp);
    gp.bn = bn_for(3 * Hl);
    gp_group(&gp, 0, &b->tm_qkv[0], 0, St);
    gp_group(&gp, 1, &b->tm_qkv[1], St, Si);
    gp.qnorm[0] = b->qn[0]; gp.knorm[0] = b->kn[0];
    gp.qnorm[1] = b->qn[1]; gp.knorm[1] = b->kn[1];
    gp.rope_pos = P->rope_pos; gp.rope_spec = P->rope_spec;
    gp.q = P->q; gp.k = P->k; gp.v = P->v; gp.ldqkv = Hl; gp.H = Hl;
    enq_gemm(E, &gp, "dbl_qkv");
    enq_x(E, iris_launch_attention(P->q, Hl, P->k, P->v, Hl, P->attn, Hl, S, S, NHl,
                                   1.0f / sqrtf(128.0f), NULL, st), "dbl_attn",
          4.0 * S * S * (double)Hl, 8.0 * S * (double)Hl);
    gp_init(&gp, P, &P->tm_attn, H, Hl, IRIS_EPI_RESID_GATE);
    gp_group(&gp, 0, &b->tm_out[0], 0, St);
    gp_group(&gp, 1, &b->tm_out[1], St, Si);
    gp.out = P->hidden; gp.ldo = H;
    gp.gate[0] = mt + 2 * H; gp.gate[1] = mi + 2 * H;
    tp_resid(tf, &gp);
    fuse_next_adaln(tf, E, &gp, mt + 3 * H, mt + 4 * H, mi + 3 * H, mi + 4 * H, St);
    enq_gemm(E, &gp, "dbl_out");
    enq_allreduce(tf, E);
    if (!adaln_done(P))
        enq_x(E, adaln_rows(tf, 0, S, mt + 3 * H, mt + 4 * H, mi + 3 * H, mi + 4 * H, St), "adaln2", 0.0,
              6.0 * S * (double)H);
    gp_init(&gp, P, &P->tm_xmod, 2 * Fl, H, IRIS_EPI_SWIGLU);
    tp_reads_xmod(tf, &gp);
    gp_group(&gp, 0, &b->tm_in[0], 0, St);
    gp_group(&gp, 1, &b->tm_in[1], St, Si);
    gp.mlp_out = P->mlp; gp.ld_mlp = Fl; gp.mlp_col0 = 0; gp.swiglu_base = 0;
    enq_gemm(E, &gp, "dbl_mlp_in");
    gp_init(&gp, P, &P->tm_mlp, H, Fl, IRIS_EPI_RESID_GATE);
    gp_group(&gp, 0, &b->tm_down[0], 0, St);
    gp_group(&gp, 1, &b->tm_down[1], St, Si);
    gp.out = P->hidden; gp.ldo = H;
    gp.gate[0] = mt + 5 * H; gp.gate[1] = mi + 5 * H;
    tp_resid(tf, &gp);
    if (!ip_active(tf, i)) {  /* the next block's adaLN (double blocks share their modulation) */
        const float *ms = tf->mods + (size_t)12 * H;
        if (i + 1 < tf->cfg.n_double) fuse_next_adaln(tf, E, &gp, mt, mt + H, mi, mi + H, St);
        else if (tf->cfg.n_single > 0) fuse_next_adaln(tf, E, &gp, ms, ms + H, NULL, NULL, S);
    }
    enq_gemm(E, &gp, "dbl_mlp_out");
    enq_allreduce(tf, E);
    enq_ip(tf, E, i, St, Si);
}

/* IP-Adapter contribution of adapter block blk to rows [row0, row0 + rows) of
 * the hidden state, after the block (ip_inject_block, iris_transformer_flux.c:2355):
 * the block's post-RoPE Q of those rows rotated back to the pre-RoPE Q, attention
 * over the block's T adapter tokens, hidden += scale[blk] * O.  A block whose
 * static scale is 0 (style-only export) adds nothing, as in the reference. */
static void enq_ip(iris_cuda_flux_t *tf, enq_t *E, int blk, int row0, int rows) {
    struct iris_flux_ip *ip = tf->ip;
    if (!ip || blk >= ip->nb || ip->h_scale[blk] == 0.0f || rows <= 0) return;
    flux_plan_t *P = &tf->plan;
    cudaStream_t st = g_rt.stream;
    const int H = tf->H, T = ip->T;
    const uint16_t *k = ip->kv + (size_t)blk * T * H, *v = ip->kv + (size_t)(ip->nb + blk) * T * H;
    enq(E, iris_launch_ip_unrope(P->q + (size_t)row0 * H, H, P->rope_pos + (size_t)row0 * 4, P->rope_spec, rows,
                                 H, P->ip_q, st), "ip_unrope");
    enq_x(E, iris_launch_attention(P->ip_q, H, k, v, H, P->ip_o, H, rows, T, tf->NH, 1.0f / sqrtf(128.0f), NULL,
                                   st), "ip_attn", 4.0 * rows * T * (double)H, 2.0 * (rows + 2.0 * T) * H * 2.0);
    enq(E, iris_launch_ip_add(P->hidden + (size_t)row0 * H, H, P->ip_o, rows, H, ip->d_scale + blk, st), "ip_add");
}

/* single-stream block i over the whole [TXT, IMG] sequence */
static void enq_single(iris_cuda_flux_t *tf, int i, enq_t *E) {
    flux_plan_t *P = &tf->plan;
    cudaStream_t st = g_rt.stream;
    const int H = tf->H, Hl = tf->Hl, Fl = tf->Fl, NHl = tf->NHl, S = P->S;
    const float *ms = tf->mods + (size_t)12 * H;
    flux_sgl_t *b = &tf->sgl[i];
    IrisGemmParams gp;
    if (!adaln_done(P))
        enq_x(E, adaln_rows(tf, 0, S, ms, ms + H, NULL, NULL, S), "adaln_s", 0.0, 6.0 * S * (double)H);
    gp_init(&gp, P, &P->tm_xmod, 3 * Hl + 2 * Fl, H, IRIS_EPI_SINGLE);
    tp_reads_xmod(tf, &gp);
    gp_group(&gp, 0, &b->tm_fused, 0, S);
    gp.qnorm[0] = b->qn; gp.knorm[0] = b->kn;
    gp.rope_pos = P->rope_pos; gp.rope_spec = P->rope_spec;
    gp.rope_k_row0 = P->rope_k_row0;  /* SREF band control: reference rows' K (:3872) */
    gp.q = P->q; gp.k = P->k; gp.v = P->v; gp.ldqkv = Hl; gp.H = Hl;
    gp.mlp_out = P->cat; gp.ld_mlp = Hl + Fl; gp.mlp_col0 = Hl; gp.swiglu_base = 3 * Hl;
    enq_gemm(E, &gp, "sgl_fused");
    enq_x(E, iris_launch_attention(P->q, Hl, P->k, P->v, Hl, P->cat, Hl + Fl, S, S, NHl,
                                   1.0f / sqrtf(128.0f), NULL, st), "sgl_attn",
          4.0 * S * S * (double)Hl, 8.0 * S * (double)Hl);
    gp_init(&gp, P, &P->tm_cat, H, Hl + Fl, IRIS_EPI_RESID_GATE);
    gp_group(&gp, 0, &b->tm_out, 0, S);
    gp.out = P->hidden; gp.ldo = H;
    gp.gate[0] = ms + 2 * H;
    tp_resid(tf, &gp);
    if (i + 1 < tf->cfg.n_single && !ip_active(tf, tf->cfg.n_double + i))
        fuse_next_adaln(tf, E, &gp, ms, ms + H, NULL, NULL, S);  /* single blocks share their modulation */
    enq_gemm(E, &gp, "sgl_out");
    enq_allreduce(tf, E);
    enq_ip(tf, E, tf->cfg.n_double + i, P->s_txt, S - P->s_txt);
}

/* final layer on the target image rows only (scale first, then shift: :4277-4281) */
static void enq_final(iris_cuda_flux_t *tf, enq_t *E) {
    flux_plan_t *P = &tf->plan;
    const int H = tf->H, C = tf->C, St = P->s_txt;
    const float *mf = tf->mods + (size_t)15 * H;
    IrisGemmParams gp;
    enq(E, adaln_rows(tf, St, P->n_img, mf + H, mf, NULL, NULL, P->S), "adaln_final");
    gp_init(&gp, P, &P->tm_xmod, C, H, IRIS_EPI_F32_NCHW);
    tp_reads_xmod(tf, &gp);
    gp.bn = 128;
    gp_group(&gp, 0, &tf->tm_proj, St, P->n_img);  /* xmod holds the image rows at their own index */
    gp.out = P->out;
    gp.nchw_rows = P->n_img;
    enq_gemm(E, &gp, "proj_out");
}

/* start / end of a call that may exchange over peer memory */
static void tp_begin(iris_cuda_flux_t *tf, enq_t *E) {
    tf->plan.part_i = tf->plan.x_i = 0;
    tf->plan.part_pending = 0;
    if (tf->tp <= 1) return;
    /* no rank writes into a peer's buffers before every rank finished its
       previous call (which may still be reading them) */
    IrisTpParams t;
    tp_fill(tf, &t, 0);
    enq(E, iris_launch_tp_barrier(&t, g_rt.d_status, g_rt.stream), "tp_barrier");
}

static void tp_end(iris_cuda_flux_t *tf, enq_t *E) {
    if (tf->tp <= 1) return;
    enq(E, iris_launch_tp_advance(tf->plan.flags, tf->plan.part_i, tf->plan.x_i, g_rt.stream), "tp_advance");
}

/* Queue one forward over the current plan: reads P->lat_in, P->txt_f32 and
 * tf->t_dev, writes P->out. */
static int enqueue_forward(iris_cuda_flux_t *tf, enq_t *E) {
    E->fuse_ln = 1;
    tf->plan.ln_pending = 0;
    tp_begin(tf, E);
    enq_mods(tf, E);
    enq_embed(tf, E);
    for (int i = 0; i < tf->cfg.n_double; i++) enq_double(tf, i, E);
    for (int i = 0; i < tf->cfg.n_single; i++) enq_single(tf, i, E);
    enq_final(tf, E);
    tp_end(tf, E);
    return E->rc;
}

/* Test hook for per-block parity: run ONE block on a caller-supplied hidden
 * state.  hidden [txt_seq + img_h*img_w, H] f32 host buffer in [TXT, IMG]
 * order, updated in place; the modulation vectors come from timestep t.
 * kind 0 = double block (the reference's double_block_forward, :2366),
 * kind 1 = single block (single_block_forward, :3761). */
int iris_cuda_flux_run_block(iris_cuda_flux_t *tf, int kind, int idx, float *hidden, int txt_seq,
                             int img_h, int img_w, float t) {
    if (!tf || !hidden) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if ((kind == 0 && (idx < 0 || idx >= tf->cfg.n_double)) ||
        (kind == 1 && (idx < 0 || idx >= tf->cfg.n_single)) || kind < 0 || kind > 1)
        return iris_fail(IRIS_CUDA_ERR_ARG, "block index");
    int rc = plan_ensure(tf, txt_seq, img_h, img_w, NULL, 0);
    if (rc) return rc;
    flux_plan_t *P = &tf->plan;
    size_t bytes = (size_t)P->S * tf->H * 4;
    rc = iris_cuda_check(cudaMemcpyAsync(P->hidden, hidden, bytes, cudaMemcpyHostToDevice, g_rt.stream), "h2d");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(tf->t_dev, &t, 4, cudaMemcpyHostToDevice, g_rt.stream), "t");
    if (rc) return rc;
    enq_t E = {0};
    tp_begin(tf, &E);
    enq_mods(tf, &E);
    if (kind == 0) enq_double(tf, idx, &E);
    else enq_single(tf, idx, &E);
    if (tf->tp > 1 && P->part_pending && !E.rc) {
        /* the block's last update (normally folded into the next adaLN): fold it
           into this rank's rows, then gather every rank's rows */
        IrisAdalnTpArgs a;
        memset(&a, 0, sizeof(a));
        a.x = P->hidden;
        a.row0 = tf->tp_rank * P->chunk;
        a.rows = P->S - a.row0 < P->chunk ? P->S - a.row0 : P->chunk;
        if (a.rows < 0) a.rows = 0;
        a.chunk = P->chunk;
        a.H = tf->H;
        a.recv = P->recv;
        a.has_part = 1;
        a.part_index = P->part_i;
        tp_fill(tf, &a.tp, 0);
        a.status = g_rt.d_status;
        enq(&E, iris_launch_adaln_tp(&a, g_rt.stream), "tp_fold");
        if (!E.rc)
            E.rc = iris_comm_allgather_bytes(P->hidden + (size_t)a.row0 * tf->H, P->hidden,
                                             (size_t)P->chunk * tf->H * 4);
    }
    tp_end(tf, &E);
    iris_count_launch(E.kernels);
    if (E.rc) return E.rc;
    rc = iris_cuda_check(cudaMemcpyAsync(hidden, P->hidden, bytes, cudaMemcpyDeviceToHost, g_rt.stream), "d2h");
    if (!rc) rc = iris_cuda_synchronize();
    return rc;
}

/* Live per-kernel timing of one forward over the current plan: the kernels
 * are launched one by one (no graph) with a CUDA event after each, so entry i
 * covers kernel i plus the launch gap before it.  Returns the number of
 * entries written or a negative status. */
int iris_cuda_flux_profile(iris_cuda_flux_t *tf, float timestep, iris_cuda_kernel_time_t *out,
                           int max_entries) {
    if (!tf || !out || max_entries <= 0) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (!tf->plan.valid) return iris_fail(IRIS_CUDA_ERR_ARG, "run a forward first (no plan)");
    cudaEvent_t *ev = (cudaEvent_t *)calloc((size_t)max_entries + 1, sizeof(cudaEvent_t));
    if (!ev) return iris_fail(IRIS_CUDA_ERR_OOM, "events");
    int rc = 0, n = 0;
    for (int i = 0; i <= max_entries && !rc; i++) rc = iris_cuda_check(cudaEventCreate(&ev[i]), "event");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(tf->t_dev, &timestep, 4, cudaMemcpyHostToDevice,
                                                  g_rt.stream), "t");
    if (!rc) {
        enq_t E = {0};
        E.prof = out;
        E.ev = ev;
        E.maxprof = max_entries;
        cudaEventRecord(ev[0], g_rt.stream);
        rc = enqueue_forward(tf, &E);
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

/* Run the forward of the current plan (captured once into a CUDA graph). */
static int run_forward(iris_cuda_flux_t *tf) {
    flux_plan_t *P = &tf->plan;
    if (iris_fault("launch"))
        return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected launch failure");
    if (tf->tp > 1 && (iris_comm_world() != tf->tp || iris_comm_rank() != tf->tp_rank))
        return iris_fail(IRIS_CUDA_ERR_ARG, "shard %d of %d needs a communicator of that rank and size",
                         tf->tp_rank, tf->tp);
    if (!P->graph_ok) {
        static int no_graph = -1;
        if (no_graph < 0) no_graph = getenv("IRIS_CUDA_NO_GRAPH") ? 1 : 0;
        enq_t E = {0};
        if (no_graph) {
            int rc = enqueue_forward(tf, &E);
            iris_count_launch(E.kernels);
            return rc;
        }
        cudaError_t e = cudaStreamBeginCapture(g_rt.stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return iris_cuda_check(e, "begin capture");
        int rc = enqueue_forward(tf, &E);
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

/* shared by the public forward entry points and the samplers */
int iris_flux_plan_and_inputs(iris_cuda_flux_t *tf, const float *d_latent, int img_h, int img_w,
                              const iris_cuda_ref_t *d_refs, int num_refs, const float *d_txt,
                              int txt_seq, enum cudaMemcpyKind kind) {
    int rc = plan_ensure(tf, txt_seq, img_h, img_w, d_refs, num_refs);
    if (rc) return rc;
    flux_plan_t *P = &tf->plan;
    cudaStream_t st = g_rt.stream;
    size_t nC = (size_t)tf->C;
    if (d_latent && d_latent != P->lat_in)
        if ((rc = iris_cuda_check(cudaMemcpyAsync(P->lat_in, d_latent, nC * P->n_img * 4, kind, st),
                                  "latent copy")))
            return rc;
    size_t off = nC * P->n_img;
    for (int r = 0; r < num_refs; r++) {
        size_t n = nC * d_refs[r].h * d_refs[r].w;
        if ((rc = iris_cuda_check(cudaMemcpyAsync(P->lat_in + off, d_refs[r].latent, n * 4, kind, st),
                                  "ref copy")))
            return rc;
        off += n;
    }
    if (d_txt && d_txt != P->txt_f32)
        if ((rc = iris_cuda_check(cudaMemcpyAsync(P->txt_f32, d_txt, (size_t)txt_seq * tf->T * 4,
                                                  kind, st), "txt copy")))
            return rc;
    return 0;
}

float *iris_flux_plan_latent(iris_cuda_flux_t *tf) { return tf->plan.lat_in; }
float *iris_flux_plan_out(iris_cuda_flux_t *tf) { return tf->plan.out; }
float *iris_flux_plan_txt(iris_cuda_flux_t *tf) { return tf->plan.txt_f32; }
float *iris_flux_t_dev(iris_cuda_flux_t *tf) { return tf->t_dev; }
int iris_flux_channels(iris_cuda_flux_t *tf) { return tf->C; }
int iris_flux_text_dim(iris_cuda_flux_t *tf) { return tf->T; }
int iris_flux_tp(iris_cuda_flux_t *tf) { return tf->tp; }

/* set t on the device (async, from a device or pinned source) and run */
int iris_flux_run(iris_cuda_flux_t *tf, const float *t_src, enum cudaMemcpyKind kind) {
    int rc = iris_cuda_check(cudaMemcpyAsync(tf->t_dev, t_src, 4, kind, g_rt.stream), "t copy");
    if (rc) return rc;
    return run_forward(tf);
}

int iris_cuda_flux_forward_dev(iris_cuda_flux_t *tf, const float *d_latent, int img_h, int img_w,
                               const iris_cuda_ref_t *d_refs, int num_refs, const float *d_txt,
                               int txt_seq, float timestep, float *d_out) {
    if (!tf || !d_latent || !d_txt || !d_out) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    int rc = iris_flux_plan_and_inputs(tf, d_latent, img_h, img_w, d_refs, num_refs, d_txt, txt_seq,
                                       cudaMemcpyDeviceToDevice);
    if (rc) return rc;
    /* timestep through a small device scratch slot, ordered on the stream */
    rc = iris_cuda_check(cudaMemcpyAsync(tf->t_dev + 1, &timestep, 4, cudaMemcpyHostToDevice,
                                         g_rt.stream), "t upload");
    if (rc) return rc;
    if ((rc = iris_flux_run(tf, tf->t_dev + 1, cudaMemcpyDeviceToDevice))) return rc;
    return iris_cuda_check(cudaMemcpyAsync(d_out, tf->plan.out,
                                           (size_t)tf->C * img_h * img_w * 4,
                                           cudaMemcpyDeviceToDevice, g_rt.stream), "out copy");
}

static float *forward_host(iris_cuda_flux_t *tf, const float *latent, int h, int w,
                           const iris_cuda_ref_t *refs, int num_refs, const float *txt, int txt_seq,
                           float t) {
    if (!tf || !latent || !txt) { iris_fail(IRIS_CUDA_ERR_ARG, "null argument"); return NULL; }
    if (iris_fault("h2d")) { iris_fail(IRIS_CUDA_ERR_INJECTED, "injected H2D failure"); return NULL; }
    int rc = iris_flux_plan_and_inputs(tf, latent, h, w, refs, num_refs, txt, txt_seq,
                                       cudaMemcpyHostToDevice);
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(tf->t_dev + 1, &t, 4, cudaMemcpyHostToDevice,
                                                  g_rt.stream), "t upload");
    if (!rc) rc = iris_flux_run(tf, tf->t_dev + 1, cudaMemcpyDeviceToDevice);
    size_t n = (size_t)tf->C * h * w;
    float *out = rc ? NULL : (float *)malloc(n * 4);
    if (!rc && !out) rc = iris_fail(IRIS_CUDA_ERR_OOM, "output");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, tf->plan.out, n * 4, cudaMemcpyDeviceToHost,
                                                  g_rt.stream), "out copy");
    if (!rc) rc = iris_cuda_synchronize();
    if (rc) { free(out); return NULL; }
    return out;
}

float *iris_cuda_transformer_forward(iris_cuda_flux_t *tf, const float *img_latent, int img_h,
                                     int img_w, const float *txt_emb, int txt_seq, float timestep) {
    return forward_host(tf, img_latent, img_h, img_w, NULL, 0, txt_emb, txt_seq, timestep);
}

float *iris_cuda_transformer_forward_with_multi_refs(iris_cuda_flux_t *tf, const float *img_latent,
                                                     int img_h, int img_w,
                                                     const iris_cuda_ref_t *refs, int num_refs,
                                                     const float *txt_emb, int txt_seq,
                                                     float timestep) {
    return forward_host(tf, img_latent, img_h, img_w, refs, num_refs, txt_emb, txt_seq, timestep);
}
