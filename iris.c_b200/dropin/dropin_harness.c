/*
 * Entry points for driving the reference's own transformer code on the CUDA
 * backend (see Makefile): every function calls one public function of the
 * reference, compiled with -DUSE_METAL, whose GPU branches call the
 * iris_metal.h surface that libiris_cuda.so exports.
 *
 *   drive_init           iris_metal_init                      (iris_metal.h:23)
 *   drive_flux_load      iris_transformer_load_safetensors    (iris_transformer_flux.c:5300)
 *                        / _mmap                              (:5550)
 *   drive_flux_forward   iris_transformer_forward             (:3939; bf16 GPU branch :4000)
 *   drive_sample_euler   iris_sample_euler                    (iris_sample.c:313)
 *   drive_zi_load        zi_transformer_load_safetensors      (iris_transformer_zimage.c:2164)
 *   drive_zi_forward     zi_transformer_forward               (:1696; GPU branch :1704)
 *   drive_*_free         the model's free function, then iris_metal_reset (iris.c:642)
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "iris_metal.h"

typedef struct iris_transformer iris_transformer_t;
typedef struct zi_transformer zi_transformer_t;

extern iris_transformer_t *iris_transformer_load_safetensors(const char *model_dir);
extern iris_transformer_t *iris_transformer_load_safetensors_mmap(const char *model_dir);
extern void iris_transformer_free(iris_transformer_t *tf);
extern float *iris_transformer_forward(iris_transformer_t *tf, const float *img_latent, int img_h, int img_w,
                                       const float *txt_emb, int txt_seq, float timestep);
extern float *iris_sample_euler(void *transformer, void *text_encoder, float *z, int batch, int channels, int h,
                                int w, const float *text_emb, int text_seq, const float *schedule, int num_steps,
                                void (*progress_callback)(int step, int total));
extern zi_transformer_t *zi_transformer_load_safetensors(const char *model_dir, int dim, int n_heads, int n_layers,
                                                         int n_refiner, int cap_feat_dim, int in_channels,
                                                         int patch_size, float rope_theta, const int *axes_dims);
extern void zi_transformer_free(zi_transformer_t *tf);
extern float *zi_transformer_forward(zi_transformer_t *tf, const float *latent, int latent_h, int latent_w,
                                     float timestep, const float *cap_feats, int cap_seq_len);

int drive_init(void) { return iris_metal_init(); }

void *drive_flux_load(const char *model_dir, int mmap_mode) {
    return mmap_mode ? iris_transformer_load_safetensors_mmap(model_dir) : iris_transformer_load_safetensors(model_dir);
}

/* Freeing a model also resets the backend's caches, as the reference's host
 * code does between models (iris_metal_reset, iris.c:642): the weight cache
 * is keyed by host address, and the next model's weights can land at the
 * addresses of this one's. */
void drive_flux_free(void *tf) {
    iris_transformer_free((iris_transformer_t *)tf);
    iris_metal_reset();
}

/* out: [channels, h, w] */
int drive_flux_forward(void *tf, const float *latent, int h, int w, const float *txt, int txt_seq, float t,
                       int channels, float *out) {
    float *v = iris_transformer_forward((iris_transformer_t *)tf, latent, h, w, txt, txt_seq, t);
    if (!v) return -1;
    memcpy(out, v, (size_t)channels * h * w * sizeof(float));
    free(v);
    return 0;
}

/* z: [channels, h, w] in/out; schedule has steps + 1 values */
int drive_sample_euler(void *tf, float *z, int channels, int h, int w, const float *txt, int txt_seq,
                       const float *schedule, int steps) {
    float *r = iris_sample_euler(tf, NULL, z, 1, channels, h, w, txt, txt_seq, schedule, steps, NULL);
    if (!r) return -1;
    if (r != z) {
        memcpy(z, r, (size_t)channels * h * w * sizeof(float));
        free(r);
    }
    return 0;
}

/* cfg: dim, n_heads, n_layers, n_refiner, cap_feat_dim, in_channels, patch_size, axes_dims[3] */
void *drive_zi_load(const char *model_dir, const int *cfg, float rope_theta) {
    return zi_transformer_load_safetensors(model_dir, cfg[0], cfg[1], cfg[2], cfg[3], cfg[4], cfg[5], cfg[6],
                                           rope_theta, cfg + 7);
}

void drive_zi_free(void *tf) {
    zi_transformer_free((zi_transformer_t *)tf);
    iris_metal_reset();
}

int drive_zi_forward(void *tf, const float *latent, int lh, int lw, float t, const float *cap, int cap_seq,
                     int in_ch, float *out) {
    float *v = zi_transformer_forward((zi_transformer_t *)tf, latent, lh, lw, t, cap, cap_seq);
    if (!v) return -1;
    memcpy(out, v, (size_t)in_ch * lh * lw * sizeof(float));
    free(v);
    return 0;
}
