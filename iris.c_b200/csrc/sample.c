/*
 * Samplers for the CUDA backend: timestep schedules, seed-stable initial
 * noise and the Euler rectified-flow loops, with the latent kept resident in
 * HBM across steps (one device->host copy per image instead of one per step).
 *
 * Reference: iris_sample.c — schedules :61-244, iris_sample_euler :313,
 * iris_sample_euler_with_multi_refs :630, iris_sample_euler_cfg :717,
 * iris_init_noise :1146; RNG iris_kernels.c:50-107.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "iris_internal.h"

/* flux.c */
int iris_flux_plan_and_inputs(iris_cuda_flux_t *tf, const float *d_latent, int img_h, int img_w,
                              const iris_cuda_ref_t *d_refs, int num_refs, const float *d_txt,
                              int txt_seq, enum cudaMemcpyKind kind);
float *iris_flux_plan_latent(iris_cuda_flux_t *tf);
float *iris_flux_plan_out(iris_cuda_flux_t *tf);
float *iris_flux_plan_txt(iris_cuda_flux_t *tf);
int iris_flux_run(iris_cuda_flux_t *tf, const float *t_src, enum cudaMemcpyKind kind);
int iris_flux_channels(iris_cuda_flux_t *tf);
int iris_flux_text_dim(iris_cuda_flux_t *tf);
int iris_flux_tp(iris_cuda_flux_t *tf);
int iris_flux_csd_branch(iris_cuda_flux_t *tf, int on);

#define IRIS_CUDA_MAX_STEPS 1000

/* ------------------------------------------------------------------ schedules */
float *iris_cuda_linear_schedule(int n) {
    if (n <= 0) return NULL;
    float *s = (float *)malloc((size_t)(n + 1) * sizeof(float));
    if (!s) return NULL;
    for (int i = 0; i <= n; i++) s[i] = 1.0f - (float)i / (float)n;
    return s;
}

/* empirical mu and SNR time shift of the Flux.2 schedule (iris_sample.c:144-182) */
static float empirical_mu(int seq, int steps) {
    const float a1 = 8.73809524e-05f, b1 = 1.89833333f, a2 = 0.00016927f, b2 = 0.45666666f;
    if (seq > 4300) return a2 * seq + b2;
    float m200 = a2 * seq + b2, m10 = a1 * seq + b1;
    float a = (m200 - m10) / 190.0f, b = m200 - 200.0f * a;
    return a * steps + b;
}

float *iris_cuda_official_schedule(int n, int seq) {
    if (n <= 0) return NULL;
    float *s = (float *)malloc((size_t)(n + 1) * sizeof(float));
    if (!s) return NULL;
    float mu = empirical_mu(seq, n);
    for (int i = 0; i <= n; i++) {
        float t = 1.0f - (float)i / (float)n;
        if (t <= 0.0f) s[i] = 0.0f;
        else if (t >= 1.0f) s[i] = 1.0f;
        else s[i] = expf(mu) / (expf(mu) + powf(1.0f / t - 1.0f, 1.0f));
    }
    return s;
}

float *iris_cuda_zimage_schedule(int n, int seq) {
    (void)seq;
    if (n <= 0) return NULL;
    float *s = (float *)malloc((size_t)(n + 1) * sizeof(float));
    if (!s) return NULL;
    float shift = 3.0f;
    const char *env = getenv("IRIS_ZIMAGE_SHIFT");
    if (env) {
        float v = (float)atof(env);
        if (v > 0.0f) shift = v;
    }
    const float smin = shift * (1.0f / 1000.0f) / (1.0f + (shift - 1.0f) * (1.0f / 1000.0f));
    for (int i = 0; i < n; i++) {
        float u = n > 1 ? (float)i / (float)(n - 1) : 0.0f;
        float raw = 1.0f + (smin - 1.0f) * u;
        s[i] = shift * raw / (1.0f + (shift - 1.0f) * raw);
    }
    s[n] = 0.0f;
    return s;
}

/* ------------------------------------------------------------------ noise */
/* xoshiro256** seeded by SplitMix64 with Box-Muller normals: the same stream
 * as the reference RNG, so a seed gives bit-identical latents. */
typedef struct { uint64_t s[4]; } xrng_t;

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static void xrng_seed(xrng_t *r, uint64_t seed) {
    for (int i = 0; i < 4; i++) {
        seed += 0x9e3779b97f4a7c15ULL;
        uint64_t z = seed;
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
        r->s[i] = z ^ (z >> 31);
    }
}

static uint64_t xrng_next(xrng_t *r) {
    uint64_t *s = r->s;
    uint64_t out = rotl64(s[1] * 5, 7) * 9, t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return out;
}

static float xrng_uniform(xrng_t *r) { return (float)((xrng_next(r) >> 11) * (1.0 / 9007199254740992.0)); }

static float xrng_normal(xrng_t *r) {
    float u1 = xrng_uniform(r), u2 = xrng_uniform(r);
    while (u1 == 0.0f) u1 = xrng_uniform(r);
    return sqrtf(-2.0f * logf(u1)) * cosf(2.0f * 3.14159265358979323846f * u2);
}

/* The reference RNG state is process-global and only re-seeded for seed >= 0;
 * the same holds here. */
static xrng_t g_noise_rng = {{0x853c49e6748fea9bULL, 0xda3e39cb94b95bdbULL, 0x647c4677a2884327ULL,
                              0xc6e7918d2e2969f5ULL}};

float *iris_cuda_init_noise(int batch, int c, int h, int w, int64_t seed) {
    if (batch <= 0 || c <= 0 || h <= 0 || w <= 0) return NULL;
    size_t n = (size_t)batch * c * h * w;
    float *out = (float *)malloc(n * sizeof(float));
    if (!out) return NULL;
    if (seed >= 0) xrng_seed(&g_noise_rng, (uint64_t)seed);
    const int M = 112;  /* noise is drawn at the largest latent size, then subsampled */
    if (h >= M && w >= M) {
        for (size_t i = 0; i < n; i++) out[i] = xrng_normal(&g_noise_rng);
        return out;
    }
    size_t big_n = (size_t)batch * c * M * M;
    float *big = (float *)malloc(big_n * sizeof(float));
    if (!big) { free(out); return NULL; }
    for (size_t i = 0; i < big_n; i++) big[i] = xrng_normal(&g_noise_rng);
    for (int b = 0; b < batch; b++)
        for (int ch = 0; ch < c; ch++)
            for (int y = 0; y < h; y++)
                for (int x = 0; x < w; x++) {
                    int sy = y * M / h, sx = x * M / w;
                    out[(((size_t)b * c + ch) * h + y) * w + x] =
                        big[(((size_t)b * c + ch) * M + sy) * M + sx];
                }
    free(big);
    return out;
}

/* ------------------------------------------------------------------ samplers */
/* Device scratch of the samplers (schedule copy, uncond velocity, the two
 * CFG contexts), kept across calls and grown on demand so back-to-back
 * images queue without allocations or host synchronisation. */
static struct {
    float *sched, *vu, *txt_c, *txt_u, *vpair;
    size_t sched_n, vu_n, txt_n, vpair_n;
} g_sws;

static int ws_grow(float **p, size_t *cap, size_t n) {
    if (*cap >= n) return 0;
    iris_stream_drain(); /* the old buffer may still be in use */
    iris_dfree(*p);
    *p = (float *)iris_dmalloc(n * 4);
    *cap = *p ? n : 0;
    return *p ? 0 : IRIS_CUDA_ERR_OOM;
}

/* Core loop.  The latent lives in the plan's latent buffer (the forward reads
 * it in place); z <- z + dt v after every forward.  Queued on the library
 * stream; does not synchronise. */
static int euler_core(iris_cuda_flux_t *tf, int h, int w, const float *txt_c, const float *txt_u,
                      int txt_seq, float guidance, const float *schedule, int steps,
                      enum cudaMemcpyKind txt_kind, void (*progress)(int, int)) {
    cudaStream_t st = g_rt.stream;
    float *z = iris_flux_plan_latent(tf), *v = iris_flux_plan_out(tf);
    size_t n = (size_t)iris_flux_channels(tf) * h * w;
    size_t txt_n = (size_t)txt_seq * iris_flux_text_dim(tf);
    int rc;
    if ((rc = ws_grow(&g_sws.sched, &g_sws.sched_n, IRIS_CUDA_MAX_STEPS + 1))) return rc;
    if (txt_u) {
        if ((rc = ws_grow(&g_sws.vu, &g_sws.vu_n, n))) return rc;
        if (g_sws.txt_n < txt_n) {
            size_t c1 = g_sws.txt_n, c2 = g_sws.txt_n;
            if ((rc = ws_grow(&g_sws.txt_c, &c1, txt_n)) || (rc = ws_grow(&g_sws.txt_u, &c2, txt_n)))
                return rc;
            g_sws.txt_n = txt_n;
        }
        if ((rc = iris_cuda_check(cudaMemcpyAsync(g_sws.txt_c, txt_c, txt_n * 4, txt_kind, st), "txt")) ||
            (rc = iris_cuda_check(cudaMemcpyAsync(g_sws.txt_u, txt_u, txt_n * 4, txt_kind, st), "txt")))
            return rc;
    }
    /* the host schedule is staged through pageable memory: the copy completes
       before cudaMemcpyAsync returns, so the caller's array may be freed */
    if ((rc = iris_cuda_check(cudaMemcpyAsync(g_sws.sched, schedule, (size_t)(steps + 1) * 4,
                                              cudaMemcpyHostToDevice, st), "schedule")))
        return rc;
    for (int s = 0; s < steps; s++) {
        float dt = schedule[s + 1] - schedule[s];
        /* the IP-Adapter schedule's multiplier for this step (iris_sample.c:351, :751) */
        if ((rc = iris_cuda_flux_set_ip_step(tf, s, steps))) return rc;
        if (txt_u) {
            if ((rc = iris_cuda_check(cudaMemcpyAsync(iris_flux_plan_txt(tf), g_sws.txt_u, txt_n * 4,
                                                      cudaMemcpyDeviceToDevice, st), "txt_u")))
                return rc;
            /* style CFG: the unconditional branch runs without the CSD delta (iris_sample.c:754) */
            if ((rc = iris_flux_csd_branch(tf, 0))) return rc;
            if ((rc = iris_flux_run(tf, g_sws.sched + s, cudaMemcpyDeviceToDevice))) return rc;
            if ((rc = iris_flux_csd_branch(tf, 1))) return rc;
            if ((rc = iris_cuda_check(cudaMemcpyAsync(g_sws.vu, v, n * 4, cudaMemcpyDeviceToDevice, st),
                                      "v_u")))
                return rc;
            if ((rc = iris_cuda_check(cudaMemcpyAsync(iris_flux_plan_txt(tf), g_sws.txt_c, txt_n * 4,
                                                      cudaMemcpyDeviceToDevice, st), "txt_c")))
                return rc;
        }
        if ((rc = iris_flux_run(tf, g_sws.sched + s, cudaMemcpyDeviceToDevice))) return rc;
        iris_count_launch(1);
        if ((rc = iris_cuda_check(iris_launch_euler(z, v, txt_u ? g_sws.vu : NULL, guidance, dt, (long)n, st),
                                  "euler")))
            return rc;
        if (progress) progress(s + 1, steps);
    }
    return 0;
}

static float *sample_host(iris_cuda_flux_t *tf, const float *z, int batch, int c, int h, int w,
                          const iris_cuda_ref_t *refs, int num_refs, const float *txt_c,
                          int seq_c, const float *txt_u, int seq_u, float g, const float *schedule,
                          int steps, void (*progress)(int, int)) {
    if (!tf || !z || !txt_c || !schedule) { iris_fail(IRIS_CUDA_ERR_ARG, "null argument"); return NULL; }
    if (batch != 1) { iris_fail(IRIS_CUDA_ERR_ARG, "batch must be 1"); return NULL; }
    if (c != iris_flux_channels(tf)) { iris_fail(IRIS_CUDA_ERR_ARG, "channel mismatch"); return NULL; }
    if (steps <= 0 || steps > IRIS_CUDA_MAX_STEPS) { iris_fail(IRIS_CUDA_ERR_ARG, "num_steps"); return NULL; }
    if (txt_u && seq_u != seq_c) {
        iris_fail(IRIS_CUDA_ERR_ARG, "cond/uncond text lengths must match");
        return NULL;
    }
    int rc = iris_flux_plan_and_inputs(tf, z, h, w, refs, num_refs, txt_c, seq_c,
                                       cudaMemcpyHostToDevice);
    if (!rc) rc = euler_core(tf, h, w, txt_c, txt_u, seq_c, g, schedule, steps,
                             cudaMemcpyHostToDevice, progress);
    size_t n = (size_t)c * h * w;
    float *out = rc ? NULL : (float *)malloc(n * 4);
    if (!rc && !out) rc = iris_fail(IRIS_CUDA_ERR_OOM, "output");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, iris_flux_plan_latent(tf), n * 4,
                                                  cudaMemcpyDeviceToHost, g_rt.stream), "z copy");
    if (!rc) rc = iris_cuda_synchronize();
    if (rc) { free(out); return NULL; }
    return out;
}

float *iris_cuda_sample_euler(iris_cuda_flux_t *tf, const float *z, int batch, int channels, int h,
                              int w, const float *text_emb, int text_seq, const float *schedule,
                              int num_steps, void (*progress_callback)(int, int)) {
    return sample_host(tf, z, batch, channels, h, w, NULL, 0, text_emb, text_seq, NULL, 0, 1.0f,
                       schedule, num_steps, progress_callback);
}

float *iris_cuda_sample_euler_cfg(iris_cuda_flux_t *tf, const float *z, int batch, int channels,
                                  int h, int w, const float *text_emb_cond, int text_seq_cond,
                                  const float *text_emb_uncond, int text_seq_uncond,
                                  float guidance_scale, const float *schedule, int num_steps,
                                  void (*progress_callback)(int, int)) {
    if (!text_emb_uncond) { iris_fail(IRIS_CUDA_ERR_ARG, "null uncond"); return NULL; }
    return sample_host(tf, z, batch, channels, h, w, NULL, 0, text_emb_cond, text_seq_cond,
                       text_emb_uncond, text_seq_uncond, guidance_scale, schedule, num_steps,
                       progress_callback);
}

float *iris_cuda_sample_euler_with_multi_refs(iris_cuda_flux_t *tf, const float *z, int batch,
                                              int channels, int h, int w,
                                              const iris_cuda_ref_t *refs, int num_refs,
                                              const float *text_emb, int text_seq,
                                              const float *schedule, int num_steps,
                                              void (*progress_callback)(int, int)) {
    return sample_host(tf, z, batch, channels, h, w, refs, num_refs, text_emb, text_seq, NULL, 0,
                       1.0f, schedule, num_steps, progress_callback);
}

int iris_cuda_sample_euler_dev(iris_cuda_flux_t *tf, float *d_z, int h, int w, const float *d_txt,
                               int txt_seq, const float *d_txt_uncond, int txt_seq_uncond,
                               float guidance, const float *schedule, int num_steps) {
    if (!tf || !d_z || !d_txt || !schedule) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (num_steps <= 0 || num_steps > IRIS_CUDA_MAX_STEPS) return iris_fail(IRIS_CUDA_ERR_ARG, "num_steps");
    if (d_txt_uncond && txt_seq_uncond != txt_seq)
        return iris_fail(IRIS_CUDA_ERR_ARG, "cond/uncond text lengths must match");
    int rc = iris_flux_plan_and_inputs(tf, d_z, h, w, NULL, 0, d_txt, txt_seq,
                                       cudaMemcpyDeviceToDevice);
    if (rc) return rc;
    rc = euler_core(tf, h, w, d_txt, d_txt_uncond, txt_seq, guidance, schedule, num_steps,
                    cudaMemcpyDeviceToDevice, NULL);
    if (rc) return rc;
    return iris_cuda_check(cudaMemcpyAsync(d_z, iris_flux_plan_latent(tf),
                                           (size_t)iris_flux_channels(tf) * h * w * 4,
                                           cudaMemcpyDeviceToDevice, g_rt.stream), "z copy");
}

/* ------------------------------------------------------------ CFG over a GPU pair
 * The two branches of classifier-free guidance run on the two ranks of the
 * process's communicator (rank 0 unconditional, rank 1 conditional).  After
 * every forward the pair all-gathers its velocities [v_uncond | v_cond] and
 * both ranks apply the same guided Euler update, so both hold the identical
 * latent, bit-equal to the one-GPU CFG sampler (iris_sample_euler_cfg,
 * iris_sample.c:717: v = v_uncond + g (v_cond - v_uncond)). */
static int euler_pair_core(iris_cuda_flux_t *tf, int h, int w, float guidance, const float *schedule,
                           int steps, void (*progress)(int, int)) {
    cudaStream_t st = g_rt.stream;
    float *z = iris_flux_plan_latent(tf), *v = iris_flux_plan_out(tf);
    size_t n = (size_t)iris_flux_channels(tf) * h * w;
    int rc;
    if ((rc = ws_grow(&g_sws.sched, &g_sws.sched_n, IRIS_CUDA_MAX_STEPS + 1)) ||
        (rc = ws_grow(&g_sws.vpair, &g_sws.vpair_n, 2 * n)))
        return rc;
    if ((rc = iris_cuda_check(cudaMemcpyAsync(g_sws.sched, schedule, (size_t)(steps + 1) * 4,
                                              cudaMemcpyHostToDevice, st), "schedule")))
        return rc;
    /* rank 2p runs the unconditional branch: no CSD delta there */
    if ((rc = iris_flux_csd_branch(tf, iris_comm_rank() % 2))) return rc;
    for (int s = 0; s < steps; s++) {
        if ((rc = iris_cuda_flux_set_ip_step(tf, s, steps))) return rc;
        if ((rc = iris_flux_run(tf, g_sws.sched + s, cudaMemcpyDeviceToDevice))) return rc;
        if ((rc = iris_comm_allgather_f32(v, g_sws.vpair, n))) return rc;
        iris_count_launch(1);
        if ((rc = iris_cuda_check(iris_launch_euler(z, g_sws.vpair + n, g_sws.vpair, guidance,
                                                    schedule[s + 1] - schedule[s], (long)n, st), "euler")))
            return rc;
        if (progress) progress(s + 1, steps);
    }
    return iris_flux_csd_branch(tf, 1);
}

static int pair_check(iris_cuda_flux_t *tf, const void *c, const void *u, int seq_c, int seq_u,
                      const float *schedule, int steps) {
    if (!tf || !c || !u || !schedule) return iris_fail(IRIS_CUDA_ERR_ARG, "null argument");
    if (steps <= 0 || steps > IRIS_CUDA_MAX_STEPS) return iris_fail(IRIS_CUDA_ERR_ARG, "num_steps");
    if (seq_c != seq_u) return iris_fail(IRIS_CUDA_ERR_ARG, "cond/uncond text lengths must match");
    if (iris_comm_world() != 2) return iris_fail(IRIS_CUDA_ERR_ARG, "CFG pair needs a 2-rank communicator");
    if (iris_flux_tp(tf) != 1) return iris_fail(IRIS_CUDA_ERR_ARG, "CFG pair needs an unsharded model");
    return 0;
}

int iris_cuda_sample_euler_cfg_pair_dev(iris_cuda_flux_t *tf, float *d_z, int h, int w,
                                        const float *d_txt_cond, const float *d_txt_uncond,
                                        int txt_seq, float guidance, const float *schedule,
                                        int num_steps) {
    int rc = pair_check(tf, d_txt_cond, d_txt_uncond, txt_seq, txt_seq, schedule, num_steps);
    if (rc) return rc;
    if (!d_z) return iris_fail(IRIS_CUDA_ERR_ARG, "null latent");
    const float *txt = iris_comm_rank() == 0 ? d_txt_uncond : d_txt_cond;
    if ((rc = iris_flux_plan_and_inputs(tf, d_z, h, w, NULL, 0, txt, txt_seq, cudaMemcpyDeviceToDevice)) ||
        (rc = euler_pair_core(tf, h, w, guidance, schedule, num_steps, NULL)))
        return rc;
    return iris_cuda_check(cudaMemcpyAsync(d_z, iris_flux_plan_latent(tf),
                                           (size_t)iris_flux_channels(tf) * h * w * 4,
                                           cudaMemcpyDeviceToDevice, g_rt.stream), "z copy");
}

float *iris_cuda_sample_euler_cfg_pair(iris_cuda_flux_t *tf, const float *z, int batch, int channels,
                                       int h, int w, const float *text_emb_cond, int text_seq_cond,
                                       const float *text_emb_uncond, int text_seq_uncond,
                                       float guidance_scale, const float *schedule, int num_steps,
                                       void (*progress_callback)(int, int)) {
    if (pair_check(tf, text_emb_cond, text_emb_uncond, text_seq_cond, text_seq_uncond, schedule, num_steps))
        return NULL;
    if (!z || batch != 1 || channels != iris_flux_channels(tf)) {
        iris_fail(IRIS_CUDA_ERR_ARG, "latent must be [1, %d, h, w]", iris_flux_channels(tf));
        return NULL;
    }
    const float *txt = iris_comm_rank() == 0 ? text_emb_uncond : text_emb_cond;
    int rc = iris_flux_plan_and_inputs(tf, z, h, w, NULL, 0, txt, text_seq_cond, cudaMemcpyHostToDevice);
    if (!rc) rc = euler_pair_core(tf, h, w, guidance_scale, schedule, num_steps, progress_callback);
    size_t n = (size_t)channels * h * w;
    float *out = rc ? NULL : (float *)malloc(n * 4);
    if (!rc && !out) rc = iris_fail(IRIS_CUDA_ERR_OOM, "output");
    if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(out, iris_flux_plan_latent(tf), n * 4,
                                                  cudaMemcpyDeviceToHost, g_rt.stream), "z copy");
    if (!rc) rc = iris_cuda_synchronize();
    if (rc) { free(out); return NULL; }
    return out;
}
