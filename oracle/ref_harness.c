/*
 * ORACLE HARNESS — test infrastructure only, never part of the product path.
 *
 * White-box driver for the reference's own CPU implementation of the Flux.2
 * DiT forward (iris.c, built from the unmodified sources under the reference
 * tree by oracle/Makefile).  It #includes the reference's
 * iris_transformer_flux.c so that the file-static block functions can be
 * driven one block at a time, the same technique the reference uses for its
 * VAE unit test (debug/test_vae.c:58).
 *
 * Every entry point is a thin call into reference code:
 *   ref_flux_load            -> iris_transformer_load_safetensors  (iris_transformer_flux.c:5300)
 *   ref_flux_load_mmap       -> iris_transformer_load_safetensors_mmap (:5550)
 *   ref_flux_forward         -> iris_transformer_forward           (iris_transformer_flux.c:3939)
 *   ref_flux_forward_refs    -> iris_transformer_forward_with_multi_refs (:4579)
 *   ref_flux_temb            -> get_timestep_embedding + time_embed_forward (:1349, :1366)
 *   ref_flux_double_block    -> double_block_forward                (:2366)
 *   ref_flux_single_block    -> single_block_forward                (:3761)
 *   ref_flux_rope_img/_txt   -> compute_rope_2d / compute_rope_text (:897, :1055)
 *   ref_flux_set_lora        -> lora_load + iris_transformer_set_lora (iris_lora.c:504, :5131)
 *   ref_lora_get             -> one adapter of lora_load's table     (iris_lora.h:28-49)
 *   ref_ip_perceive/get_kv/inject -> iris_ip_adapter_perceive/_get_kv/_inject (iris_ip_adapter.c:331-386)
 *   ref_flux_set_ip          -> iris_load_ip_adapter minus the file read (iris.c:520)
 *   ref_flux_set_sref_csd/_bands -> iris_set_sref_csd (iris.c:487), iris_transformer_set_sref_bands (:5153)
 *   ref_sample_euler(_cfg)   -> iris_sample_euler / _cfg            (iris_sample.c:313, :717)
 *   ref_init_noise           -> iris_init_noise                     (iris_sample.c:1146)
 *   ref_official_schedule    -> iris_official_schedule              (iris_sample.c:171)
 *   ref_zimage_schedule      -> iris_zimage_schedule                (iris_sample.c:216)
 *   ref_zi_load/forward      -> zi_transformer_load_safetensors / zi_transformer_forward
 *                                                                    (iris_transformer_zimage.c:2164, :1696)
 *   ref_vae_decode           -> iris_vae_load_safetensors_ex + iris_vae_decode
 *                                                                    (iris_vae.c:1227, :835)
 *
 * Build: see oracle/Makefile.  Outputs go to oracle/_ref/ only.
 */
#include "iris_transformer_flux.c"
#include "iris_csdmod.h"

extern float *iris_official_schedule(int num_steps, int image_seq_len);
extern float *iris_zimage_schedule(int num_steps, int image_seq_len);
extern float *iris_init_noise(int batch, int channels, int h, int w, int64_t seed);
extern float *iris_sample_euler(void *transformer, void *text_encoder,
                                float *z, int batch, int channels, int h, int w,
                                const float *text_emb, int text_seq,
                                const float *schedule, int num_steps,
                                void (*progress_callback)(int step, int total));
extern float *iris_sample_euler_cfg(void *transformer, void *text_encoder,
                                    float *z, int batch, int channels, int h, int w,
                                    const float *text_emb_cond, int text_seq_cond,
                                    const float *text_emb_uncond, int text_seq_uncond,
                                    float guidance_scale,
                                    const float *schedule, int num_steps,
                                    void (*progress_callback)(int step, int total));
extern float *iris_sample_euler_zimage(void *transformer,
                                       float *z, int batch, int channels, int h, int w,
                                       int patch_size,
                                       const float *cap_feats, int cap_seq,
                                       const float *schedule, int num_steps,
                                       void (*progress_callback)(int step, int total));
typedef struct zi_transformer zi_transformer_t;
extern zi_transformer_t *zi_transformer_load_safetensors(const char *model_dir,
                                                         int dim, int n_heads,
                                                         int n_layers, int n_refiner,
                                                         int cap_feat_dim, int in_channels,
                                                         int patch_size, float rope_theta,
                                                         const int *axes_dims);
extern void zi_transformer_free(zi_transformer_t *tf);
extern float *zi_transformer_forward(zi_transformer_t *tf, const float *latent,
                                     int latent_h, int latent_w, float timestep,
                                     const float *cap_feats, int cap_seq_len);

void ref_set_threads(int n) {
#ifdef USE_OPENBLAS
    openblas_set_num_threads(n);
#else
    (void)n;
#endif
}

void *ref_flux_load(const char *model_dir) {
    return iris_transformer_load_safetensors(model_dir);
}

/* the CLI's default weight mode (main.c:1250): bf16 block weights stay in the
 * mapped file and are converted to f32 block by block on every step */
void *ref_flux_load_mmap(const char *model_dir) {
    return iris_transformer_load_safetensors_mmap(model_dir);
}

void ref_flux_free(void *tf) { iris_transformer_free((iris_transformer_t *)tf); }

/* cfg[0..9] = hidden, heads, head_dim, mlp, n_double, n_single, text_dim,
 * latent_channels, rope_theta, axis_dim */
void ref_flux_config(void *p, float *cfg) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    cfg[0] = tf->hidden_size; cfg[1] = tf->num_heads; cfg[2] = tf->head_dim;
    cfg[3] = tf->mlp_hidden; cfg[4] = tf->num_double_layers; cfg[5] = tf->num_single_layers;
    cfg[6] = tf->text_dim; cfg[7] = tf->latent_channels; cfg[8] = tf->rope_theta;
    cfg[9] = tf->axis_dim;
}

int ref_flux_forward(void *p, const float *latent, int h, int w,
                     const float *txt, int txt_seq, float t, float *out) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    float *v = iris_transformer_forward(tf, latent, h, w, txt, txt_seq, t);
    if (!v) return -1;
    memcpy(out, v, (size_t)tf->latent_channels * h * w * sizeof(float));
    free(v);
    return 0;
}

/* refs_latent: num_refs latents [C, rh, rw] back to back; t offsets 10*(i+1). */
int ref_flux_forward_refs(void *p, const float *latent, int h, int w,
                          const float *refs_latent, int num_refs, int rh, int rw,
                          const float *txt, int txt_seq, float t, float *out) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    iris_ref_t refs[8];
    if (num_refs > 8) return -2;
    for (int i = 0; i < num_refs; i++) {
        refs[i].latent = refs_latent + (size_t)i * tf->latent_channels * rh * rw;
        refs[i].h = rh; refs[i].w = rw; refs[i].t_offset = 10 * (i + 1);
    }
    float *v = iris_transformer_forward_with_multi_refs(tf, latent, h, w, refs, num_refs,
                                                        txt, txt_seq, t);
    if (!v) return -1;
    memcpy(out, v, (size_t)tf->latent_channels * h * w * sizeof(float));
    free(v);
    return 0;
}

/* LoRA: lora_load (iris_lora.c:504) + iris_transformer_set_lora (:5131), the
 * body of iris_load_lora (iris.c:460).  Returns 0, -1 when nothing loaded. */
int ref_flux_set_lora(void *p, const char *path, float scale) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    lora_state_t *l = lora_load(path, tf->num_double_layers, tf->num_single_layers, tf->hidden_size, scale);
    if (!l) return -1;
    iris_transformer_set_lora(tf, l);
    return 0;
}

void ref_flux_clear_lora(void *p) { iris_transformer_set_lora((iris_transformer_t *)p, NULL); }

/* One adapter of the table lora_load builds: kind 0..9 = double img q, k, v,
 * proj, txt q, k, v, proj, single linear1, linear2.  dims = {rank, in, out};
 * A / B copied when they fit.  Returns 1 present, 0 absent, -1 load failed. */
int ref_lora_get(const char *path, int n_double, int n_single, int hidden, int kind, int block,
                 int *dims, float *A, size_t a_cap, float *B, size_t b_cap) {
    lora_state_t *l = lora_load(path, n_double, n_single, hidden, 1.0f);
    if (!l) return -1;
    lora_adapter_t *tab[10] = {l->double_img_q, l->double_img_k, l->double_img_v, l->double_img_proj,
                               l->double_txt_q, l->double_txt_k, l->double_txt_v, l->double_txt_proj,
                               l->single_linear1, l->single_linear2};
    int rc = 0;
    if (kind >= 0 && kind < 10 && block >= 0 && block < (kind < 8 ? n_double : n_single)) {
        lora_adapter_t *a = &tab[kind][block];
        if (a->lora_A) {
            rc = 1;
            dims[0] = a->rank; dims[1] = a->in_dim; dims[2] = a->out_dim;
            size_t na = (size_t)a->rank * a->in_dim, nb = (size_t)a->out_dim * a->rank;
            if (na <= a_cap) memcpy(A, a->lora_A, na * sizeof(float));
            if (nb <= b_cap) memcpy(B, a->lora_B, nb * sizeof(float));
        }
    }
    lora_free(l);
    return rc;
}

/* IP-Adapter stages (iris_ip_adapter.c): perceive (:331), get_kv (:366),
 * inject (:386) with an optional schedule spec applied at (step, nsteps). */
int ref_ip_perceive(const char *bundle, const float *feats, int n, float *out, int cap) {
    iris_ip_adapter_t *a = iris_ip_adapter_load(bundle);
    if (!a) return -1;
    int need = a->num_image_tokens * a->hidden_dim;
    int rc = need <= cap ? iris_ip_adapter_perceive(a, feats, n, out) : -2;
    iris_ip_adapter_free(a);
    return rc ? rc : need;
}

int ref_ip_get_kv(const char *bundle, int blk, const float *embeds, float *k, float *v) {
    iris_ip_adapter_t *a = iris_ip_adapter_load(bundle);
    if (!a) return -1;
    if (blk < 0 || blk >= a->num_blocks) { iris_ip_adapter_free(a); return -2; }
    iris_ip_adapter_get_kv(a, blk, embeds, k, v);
    iris_ip_adapter_free(a);
    return 0;
}

int ref_ip_inject(const char *bundle, int blk, const float *q, int seq, const float *k, const float *v,
                  float *hidden, const char *sched, int step, int nsteps) {
    iris_ip_adapter_t *a = iris_ip_adapter_load(bundle);
    if (!a) return -1;
    int rc = 0;
    if (sched && iris_ip_adapter_set_schedule(a, sched)) rc = -3;
    if (sched) iris_ip_adapter_set_step(a, step, nsteps);
    if (!rc) iris_ip_adapter_inject(a, blk, q, seq, k, v, hidden);
    iris_ip_adapter_free(a);
    return rc;
}

/* iris_load_ip_adapter (iris.c:520) with the features in memory instead of a
 * file: load, block-count check, ip_scale *= scale_mult, perceive, attach. */
int ref_flux_set_ip(void *p, const char *bundle, const float *feats, int n, float scale_mult) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    iris_ip_adapter_t *ip = iris_ip_adapter_load(bundle);
    if (!ip) return -1;
    if (ip->hidden_dim != tf->hidden_size || ip->num_blocks != tf->num_double_layers + tf->num_single_layers) {
        iris_ip_adapter_free(ip);
        return -2;
    }
    if (scale_mult != 1.0f)
        for (int i = 0; i < ip->num_blocks; i++) ip->ip_scale[i] *= scale_mult;
    float *emb = malloc((size_t)ip->num_image_tokens * ip->hidden_dim * sizeof(float));
    if (!emb || iris_ip_adapter_perceive(ip, feats, n, emb)) {
        free(emb);
        iris_ip_adapter_free(ip);
        return -3;
    }
    return iris_transformer_set_ip_adapter(tf, ip, emb);
}

int ref_flux_set_ip_schedule(void *p, const char *spec) {
    return iris_transformer_set_ip_schedule((iris_transformer_t *)p, spec);
}

void ref_flux_clear_ip(void *p) { iris_transformer_set_ip_adapter((iris_transformer_t *)p, NULL, NULL); }

/* iris_set_sref_csd (iris.c:487) minus the context: csd_mod MLP -> delta * scale
 * -> iris_transformer_set_csd_delta; NULL path / csd or scale 0 clears. */
int ref_flux_set_sref_csd(void *p, const char *csdmod, const float *csd, int csd_dim, float scale) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    if (!csdmod || !*csdmod || !csd || scale == 0.0f) { iris_transformer_set_csd_delta(tf, NULL); return 0; }
    csd_mod_t m;
    if (csd_mod_load(&m, csdmod)) return -1;
    if (m.csd_dim != csd_dim || m.hidden_dim != tf->hidden_size) { csd_mod_free(&m); return -2; }
    float *delta = malloc((size_t)m.hidden_dim * sizeof(float));
    float *work = malloc((size_t)m.mlp_dim * sizeof(float));
    if (!delta || !work) { free(delta); free(work); csd_mod_free(&m); return -3; }
    csd_mod_forward(&m, csd, delta, work);
    for (int i = 0; i < m.hidden_dim; i++) delta[i] *= scale;
    free(work);
    csd_mod_free(&m);
    iris_transformer_set_csd_delta(tf, delta);
    return 0;
}

void ref_flux_set_sref_bands(void *p, float shf, float slf) {
    iris_transformer_set_sref_bands((iris_transformer_t *)p, shf, slf);
}

void ref_flux_temb(void *p, float t, float *t_emb) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    float sincos[256];
    get_timestep_embedding(sincos, t * 1000.0f, tf->time_embed.sincos_dim, 10000.0f);
    time_embed_forward(t_emb, sincos, &tf->time_embed, tf->hidden_size, tf->t_emb_silu);
}

/* Modulation vectors exactly as the forward computes them (:4059-4069, :3787-3797, :4277-4281). */
void ref_flux_mods(void *p, const float *t_emb, float *dbl_img, float *dbl_txt,
                   float *single, float *final_mod) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    int h = tf->hidden_size;
    float *s = malloc((size_t)h * sizeof(float));
    for (int j = 0; j < h; j++) s[j] = t_emb[j] / (1.0f + expf(-t_emb[j]));
    iris_linear_nobias(dbl_img, s, tf->adaln_double_img_weight, 1, h, 6 * h);
    iris_linear_nobias(dbl_txt, s, tf->adaln_double_txt_weight, 1, h, 6 * h);
    iris_linear_nobias(single, s, tf->adaln_single_weight, 1, h, 3 * h);
    iris_linear_nobias(final_mod, s, tf->final_norm_weight, 1, h, 2 * h);
    free(s);
}

void ref_flux_rope_img(void *p, int ph, int pw, float *cos_out, float *sin_out) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    compute_rope_2d(cos_out, sin_out, ph, pw, tf->axis_dim, tf->rope_theta);
}

void ref_flux_rope_txt(void *p, int txt_seq, float *cos_out, float *sin_out) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    compute_rope_text(cos_out, sin_out, txt_seq, tf->axis_dim, tf->rope_theta);
}

int ref_flux_double_block(void *p, int idx, float *img_hidden, float *txt_hidden,
                          const float *img_mod, const float *txt_mod,
                          int ph, int pw, int txt_seq) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    int img_seq = ph * pw;
    if (ensure_work_buffers(tf, img_seq + txt_seq) < 0) return -1;
    if (ensure_attn_scores(tf, img_seq, txt_seq) < 0) return -1;
    float *ic, *is, *tc, *ts;
    get_cached_img_rope(tf, ph, pw, &ic, &is);
    get_cached_txt_rope(tf, txt_seq, &tc, &ts);
    double_block_forward(img_hidden, txt_hidden, &tf->double_blocks[idx], img_mod, txt_mod,
                         ic, is, tc, ts, img_seq, txt_seq, idx, tf);
    return 0;
}

/* hidden: [txt_seq + ph*pw, H] in [TXT, IMG] order. */
int ref_flux_single_block(void *p, int idx, float *hidden, const float *t_emb,
                          int ph, int pw, int txt_seq) {
    iris_transformer_t *tf = (iris_transformer_t *)p;
    int img_seq = ph * pw;
    if (ensure_work_buffers(tf, img_seq + txt_seq) < 0) return -1;
    if (ensure_attn_scores(tf, img_seq, txt_seq) < 0) return -1;
    float *ic, *is, *tc, *ts;
    get_cached_img_rope(tf, ph, pw, &ic, &is);
    get_cached_txt_rope(tf, txt_seq, &tc, &ts);
    tf->sref_krope_cos = NULL;
    tf->sref_krope_sin = NULL;
    single_block_forward(hidden, &tf->single_blocks[idx], t_emb, tf->adaln_single_weight,
                         ic, is, tc, ts, img_seq + txt_seq, txt_seq, idx, tf);
    return 0;
}

int ref_init_noise(int c, int h, int w, int64_t seed, float *out) {
    float *z = iris_init_noise(1, c, h, w, seed);
    if (!z) return -1;
    memcpy(out, z, (size_t)c * h * w * sizeof(float));
    free(z);
    return 0;
}

int ref_official_schedule(int steps, int image_seq_len, float *out) {
    float *s = iris_official_schedule(steps, image_seq_len);
    if (!s) return -1;
    memcpy(out, s, (size_t)(steps + 1) * sizeof(float));
    free(s);
    return 0;
}

int ref_zimage_schedule(int steps, int image_seq_len, float *out) {
    float *s = iris_zimage_schedule(steps, image_seq_len);
    if (!s) return -1;
    memcpy(out, s, (size_t)(steps + 1) * sizeof(float));
    free(s);
    return 0;
}

int ref_sample_euler(void *tf, float *z, int c, int h, int w, const float *txt, int txt_seq,
                     const float *schedule, int steps, float *out) {
    float *r = iris_sample_euler(tf, NULL, z, 1, c, h, w, txt, txt_seq, schedule, steps, NULL);
    if (!r) return -1;
    memcpy(out, r, (size_t)c * h * w * sizeof(float));
    free(r);
    return 0;
}

int ref_sample_euler_cfg(void *tf, float *z, int c, int h, int w,
                         const float *txt_c, int seq_c, const float *txt_u, int seq_u,
                         float g, const float *schedule, int steps, float *out) {
    float *r = iris_sample_euler_cfg(tf, NULL, z, 1, c, h, w, txt_c, seq_c, txt_u, seq_u, g,
                                     schedule, steps, NULL);
    if (!r) return -1;
    memcpy(out, r, (size_t)c * h * w * sizeof(float));
    free(r);
    return 0;
}

/* cfg: dim, n_heads, n_layers, n_refiner, cap_feat_dim, in_channels, patch_size,
 * axes_dims[3]; rope_theta separately (iris.c:309-322 passes these from config.json). */
void *ref_zi_load(const char *model_dir, const int *cfg, float rope_theta) {
    return zi_transformer_load_safetensors(model_dir, cfg[0], cfg[1], cfg[2], cfg[3], cfg[4],
                                           cfg[5], cfg[6], rope_theta, cfg + 7);
}
void ref_zi_free(void *tf) { zi_transformer_free((zi_transformer_t *)tf); }

int ref_zi_forward(void *tf, const float *latent, int lh, int lw, float t,
                   const float *cap, int cap_seq, int in_ch, float *out) {
    float *v = zi_transformer_forward((zi_transformer_t *)tf, latent, lh, lw, t, cap, cap_seq);
    if (!v) return -1;
    memcpy(out, v, (size_t)in_ch * lh * lw * sizeof(float));
    free(v);
    return 0;
}

int ref_sample_euler_zimage(void *tf, float *z, int c, int h, int w, int ps,
                            const float *cap, int cap_seq, const float *schedule, int steps,
                            float *out) {
    float *r = iris_sample_euler_zimage(tf, z, 1, c, h, w, ps, cap, cap_seq, schedule, steps, NULL);
    if (!r) return -1;
    memcpy(out, r, (size_t)c * h * w * sizeof(float));
    free(r);
    return 0;
}

/* ------------------------------------------------------------------ VAE decode
 * The reference's CPU decoder on a model file (Flux layout: batch-norm latent
 * statistics, post-quant conv, z_channels latent channels before the 2x2
 * patchify; scaling != 0 selects the Z-Image latent scaling instead, as
 * iris_vae_load_safetensors_ex does).  Writes the uint8 RGB image
 * (height x width x 3) to out_rgb, which must hold 3 * (16 lh) * (16 lw)
 * bytes. */
typedef struct iris_vae iris_vae_t;
extern iris_vae_t *iris_vae_load_safetensors_ex(safetensors_file_t *sf, int z_channels,
                                                float scaling_factor, float shift_factor);
extern void iris_vae_free(iris_vae_t *vae);
extern iris_image *iris_vae_decode(iris_vae_t *vae, const float *latent, int batch,
                                   int latent_h, int latent_w);

int ref_vae_decode_ex(const char *vae_file, int z_channels, float scaling, float shift,
                      const float *latent, int lh, int lw, uint8_t *out_rgb, int *out_w, int *out_h) {
    safetensors_file_t *sf = safetensors_open(vae_file);
    if (!sf) return -1;
    iris_vae_t *vae = iris_vae_load_safetensors_ex(sf, z_channels, scaling, shift);
    if (!vae) { safetensors_close(sf); return -2; }
    iris_image *img = iris_vae_decode(vae, latent, 1, lh, lw);
    int rc = -3;
    if (img) {
        *out_w = img->width;
        *out_h = img->height;
        memcpy(out_rgb, img->data, (size_t)img->width * img->height * img->channels);
        rc = img->channels;
        iris_image_free(img);
    }
    iris_vae_free(vae);
    safetensors_close(sf);
    return rc;
}

/* Flux layout (batch-norm statistics, scaling 0) */
int ref_vae_decode(const char *vae_file, int z_channels, const float *latent, int lh, int lw,
                   uint8_t *out_rgb, int *out_w, int *out_h) {
    return ref_vae_decode_ex(vae_file, z_channels, 0.0f, 0.0f, latent, lh, lw, out_rgb, out_w, out_h);
}


/* ------------------------------------------------------------------ Qwen3 text encoder
 * The reference's CPU text encoder (qwen3_model_load + qwen3_forward,
 * iris_qwen3.c:1578, :1072) on a model directory (config.json + shards):
 * ids / mask [seq] -> out [seq, text_dim] (text_dim = 3 * hidden for Flux,
 * hidden for Z-Image extraction).  Returns text_dim or a negative status. */
#include "iris_qwen3.h"
#include <time.h>

static double g_qwen3_forward_s;
/* wall time of the last ref_qwen3_forward's qwen3_forward call (model load excluded) */
double ref_qwen3_last_forward_s(void) { return g_qwen3_forward_s; }

int ref_qwen3_forward(const char *model_dir, int zimage, const int *ids, const int *mask, int seq, float *out,
                      int out_cap) {
    qwen3_model_t *m = qwen3_model_load(model_dir);
    if (!m) return -1;
    qwen3_encoder_t enc = {NULL, m};
    qwen3_set_extraction_mode(&enc, zimage ? 1 : 0);
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    float *r = qwen3_forward(m, ids, mask, seq);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    g_qwen3_forward_s = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    if (!r) { qwen3_model_free(m); return -2; }
    /* out_cap = seq * text_dim floats (the caller knows the hidden size) */
    int text_dim = out_cap / seq;
    memcpy(out, r, (size_t)seq * text_dim * sizeof(float));
    free(r);
    qwen3_model_free(m);
    return text_dim;
}
