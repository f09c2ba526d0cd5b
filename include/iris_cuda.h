/*
 * iris_cuda.h — C ABI of the B200 (sm_100a) backend for iris.c.
 *
 * libiris_cuda.so replaces the reference's compute backends (make generic /
 * make blas / make mps) for the DiT denoising step: the Flux.2 Klein
 * transformer forward, the Z-Image S3-DiT forward and the Euler samplers that
 * drive them.  Plain C: host or device pointers, sizes, status codes; no C++
 * or framework types cross this boundary.
 *
 * Three layers, each citing the reference interface it replaces:
 *   1. runtime            iris_metal_init / iris_metal_available / iris_gpu_sync
 *                         (iris_metal.h:23-33, :309)
 *   2. model + sampler    iris_transformer_* (iris_transformer_flux.c:3939, :4579,
 *                         :5300), zi_transformer_* (iris_transformer_zimage.c:1696,
 *                         :2164), iris_sample_* (iris_sample.c:171-1188), and the
 *                         autoencoder decoder iris_vae_decode (iris_vae.c:835)
 *   3. tensor/op surface  the iris_gpu_* device-resident API of iris_metal.h
 *                         (:155-600), same names and signatures, so the
 *                         reference's bf16 block code can link against it.
 *
 * Conventions (same as the reference): latents are NCHW f32 [C, h, w] with
 * h, w in patches (image pixels / 16 for Flux); text embeddings are f32
 * [txt_seq, text_dim]; functions returning float* hand back malloc'd host
 * memory the caller frees; NULL / non-zero status means failure.  Status
 * codes are the IRIS_CUDA_* values below; iris_cuda_last_error() describes
 * the last failure.  All calls are synchronous with respect to the host
 * unless the name ends in _dev / _async, and are single-threaded like the
 * reference's (iris_kernels.h:100-106).
 */
#ifndef IRIS_CUDA_H
#define IRIS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define IRIS_CUDA_OK 0
#define IRIS_CUDA_ERR_ARG -1         /* bad argument / unsupported shape            */
#define IRIS_CUDA_ERR_OOM -2         /* device or host allocation failed            */
#define IRIS_CUDA_ERR_CUDA -3        /* CUDA runtime/driver error                   */
#define IRIS_CUDA_ERR_IO -4          /* model file missing or malformed             */
#define IRIS_CUDA_ERR_TIMEOUT -5     /* a kernel's bounded wait expired (see below) */
#define IRIS_CUDA_ERR_NODEV -6       /* no usable sm_100 device                     */
#define IRIS_CUDA_ERR_INJECTED -7    /* failure injected through IRIS_CUDA_FAULT    */

/* ------------------------------------------------------------------ 1. runtime */
/* Select and initialise a device (idempotent).  Replaces iris_metal_init
 * (iris_metal.h:23). */
int iris_cuda_init(int device);
/* 1 when an sm_100 device is usable.  Replaces iris_metal_available (iris_metal.h:28). */
int iris_cuda_available(void);
/* Release library state (streams, caches).  Replaces iris_metal_cleanup (iris_metal.h:33). */
void iris_cuda_cleanup(void);
/* Human-readable description of the last failure on this thread. */
const char *iris_cuda_last_error(void);
/* Non-zero code recorded by a kernel whose bounded wait expired (0 = none);
 * clear != 0 resets it.  No reference counterpart (the reference has no
 * device-side waits). */
int iris_cuda_device_status(int clear);
/* Wait for all queued work.  Replaces iris_gpu_sync (iris_metal.h:309). */
int iris_cuda_synchronize(void);
/* The cudaStream_t (as void*) all library work is queued on. */
void *iris_cuda_stream(void);
/* Number of kernels this library has enqueued since load (graph replays
 * count every kernel node).  Used by benchmarks to report launch counts. */
uint64_t iris_cuda_kernel_launches(void);
/* Self-test of the device-side failure path (no counterpart in the
 * reference, whose GPU path has no bounded waits): launches the
 * tensor-parallel adaLN kernel as a one-rank group whose partial-sum flag is
 * never raised.  Its bounded wait expires after 2 s, the kernel records
 * 0x301 in the device status word and returns, and the call returns
 * IRIS_CUDA_ERR_TIMEOUT from iris_cuda_synchronize.  The status word stays
 * set until iris_cuda_device_status(1) clears it; the library remains usable. */
int iris_cuda_selftest_wait_timeout(void);

/* ------------------------------------------------------------------ 2a. Flux.2 Klein */
typedef struct iris_cuda_flux iris_cuda_flux_t;

typedef struct {
    int hidden;          /* heads * head_dim (3072 for Klein 4B)          */
    int heads;           /* 24                                            */
    int head_dim;        /* must be 128                                   */
    int mlp;             /* hidden * mlp_ratio (9216)                     */
    int n_double;        /* 5                                             */
    int n_single;        /* 20                                            */
    int text_dim;        /* joint_attention_dim (7680)                    */
    int channels;        /* in_channels (128)                             */
    float rope_theta;    /* 2000                                          */
} iris_cuda_flux_config_t;

/* Multi-reference conditioning input.  Same fields as iris_ref_t
 * (iris_sample.c:282-286). */
typedef struct {
    const float *latent; /* NCHW [C, h, w]                                */
    int h, w;
    int t_offset;        /* RoPE T coordinate (10, 20, ...)               */
} iris_cuda_ref_t;

/* Load a model directory (transformer/config.json + safetensors shards),
 * uploading every weight once to HBM as bf16.  Replaces
 * iris_transformer_load_safetensors (iris_transformer_flux.c:5300). */
iris_cuda_flux_t *iris_cuda_flux_load(const char *model_dir);
/* Random-init model of the given shape: every tensor N(0, std) from a
 * counter-based RNG keyed by (seed, tensor name), generated on the device
 * (no reference counterpart; benchmark and test fixture).  norm_unit != 0
 * draws the QK-norm scales as 1 + N(0, 0.1) instead. */
iris_cuda_flux_t *iris_cuda_flux_random(const iris_cuda_flux_config_t *cfg, uint64_t seed,
                                        float std, int norm_unit);
/* Tensor-parallel shard tp_rank of tp_size (no reference counterpart; the
 * reference runs on one device).  The shard holds heads
 * [r*heads/tp, (r+1)*heads/tp) and MLP columns [r*mlp/tp, (r+1)*mlp/tp) of
 * every block (heads % (2*tp) == 0 and mlp % (128*tp) == 0 required); the
 * embedders, modulation and final layer are replicated.  Its forwards and
 * samplers need a communicator of size tp_size in which this process has rank
 * tp_rank (iris_cuda_comm_init); they all-reduce the hidden state after every
 * attention/MLP output projection and return the full result on every rank.
 * tp_size 1 is the same as iris_cuda_flux_load / iris_cuda_flux_random. */
iris_cuda_flux_t *iris_cuda_flux_load_tp(const char *model_dir, int tp_rank, int tp_size);
iris_cuda_flux_t *iris_cuda_flux_random_tp(const iris_cuda_flux_config_t *cfg, uint64_t seed,
                                           float std, int norm_unit, int tp_rank, int tp_size);
/* Replaces iris_transformer_free (iris_transformer_flux.c:4973). */
void iris_cuda_flux_free(iris_cuda_flux_t *tf);
int iris_cuda_flux_get_config(const iris_cuda_flux_t *tf, iris_cuda_flux_config_t *out);
/* Copy one weight, in the reference's (safetensors) layout, as bf16 bits.
 * numel must match the tensor's element count. */
int iris_cuda_flux_read_weight(iris_cuda_flux_t *tf, const char *name, uint16_t *out,
                               size_t numel);
/* Bytes of HBM held by the model's weights. */
size_t iris_cuda_flux_weight_bytes(const iris_cuda_flux_t *tf);

/* LoRA.  Replaces iris_load_lora (iris.h:163; lora_load iris_lora.c:504 +
 * iris_transformer_set_lora iris_transformer_flux.c:5131): reads an adapter
 * file in any of the reference's four formats (XLabs, Kohya, Diffusers, BFL,
 * detected from the tensor names like the reference) and applies it with
 * strength `scale`, replacing any adapter loaded before.  The adapter is
 * folded into the resident weights (W + scale * B A, once), so forwards and
 * samplers run at the speed of the base model; the base weights it touched are
 * kept on the device for the next load / unload.  Returns 0, or an error with
 * the previous state unchanged when the file has no adapter matching the model
 * (adapters whose shapes do not match are skipped, with a message on stderr). */
int iris_cuda_flux_load_lora(iris_cuda_flux_t *tf, const char *path, float scale);
/* Replaces iris_unload_lora (iris.h:168): back to the base weights. */
int iris_cuda_flux_unload_lora(iris_cuda_flux_t *tf);
/* Adapters applied by the last iris_cuda_flux_load_lora (0 without a LoRA). */
int iris_cuda_flux_lora_adapters(const iris_cuda_flux_t *tf);
/* Device time of the last load's fold kernels and the bytes they moved. */
int iris_cuda_flux_lora_stats(const iris_cuda_flux_t *tf, double *fold_ms, double *fold_bytes);
/* IP-Adapter.  Replaces iris_load_ip_adapter (iris.h; iris.c:520): loads the
 * bundle (adapter_meta.json + adapter_weights.safetensors, bf16 / f16 / f32 /
 * int8; cond_mode siglip, csd or hybrid), reads the conditioning features (raw
 * f32 rows of siglip_dim — csd: one csd_dim vector; hybrid: the SigLIP rows and
 * the zero-padded CSD vector as the last row), perceives them once and keeps
 * every block's k / v on the device; each forward then adds
 * ip_scale[block] * scale_mult * schedule * SDPA(pre-RoPE image Q, k, v) to the
 * image rows after every double and single block.  Replaces any adapter attached
 * before; returns 0 or an error (bundle / model mismatch: hidden size and block
 * counts must match; tensor-parallel shards are not supported). */
int iris_cuda_flux_load_ip_adapter(iris_cuda_flux_t *tf, const char *bundle_dir, const char *features_path,
                                   float scale_mult);
/* The same with the features in host memory ([n_rows, row width] f32). */
int iris_cuda_flux_load_ip_adapter_mem(iris_cuda_flux_t *tf, const char *bundle_dir, const float *features,
                                       int n_rows, float scale_mult);
/* Replaces iris_unload_ip_adapter. */
int iris_cuda_flux_unload_ip_adapter(iris_cuda_flux_t *tf);
/* Replaces iris_set_ip_schedule: "none", "late:F" (inject from step fraction F
 * on) or "early:F" (before F); a bad spec returns an error and leaves "none". */
int iris_cuda_flux_set_ip_schedule(iris_cuda_flux_t *tf, const char *spec);
/* Replaces iris_transformer_set_ip_step (the samplers call it every step). */
int iris_cuda_flux_set_ip_step(iris_cuda_flux_t *tf, int step, int num_steps);
/* The perceived embeddings [T, H] (f32) of the attached adapter; returns T*H. */
int iris_cuda_flux_ip_embeds(const iris_cuda_flux_t *tf, float *out, int cap);

/* SREF style controls.  iris_set_sref_csd (iris.h:178; iris.c:487): run the
 * CSDModulation MLP (csd_mod.safetensors: fc1 -> SiLU -> fc2) on the
 * reference's L2-normalised CSD vector [csd_dim], times scale, and add the
 * result to the timestep embedding of every forward (the CFG samplers leave it
 * out of the unconditional branch).  A NULL path / vector or scale 0 turns it
 * off.  Returns 0 or an error (dimension mismatch). */
int iris_cuda_flux_set_sref_csd(iris_cuda_flux_t *tf, const char *csdmod_path, const float *csd, int csd_dim,
                                float scale);
/* iris_transformer_set_csd_delta: a host delta [hidden] (copied), NULL = off. */
int iris_cuda_flux_set_csd_delta(iris_cuda_flux_t *tf, const float *delta);
/* iris_transformer_set_csd_skip: 1 leaves the delta out of the next forwards. */
int iris_cuda_flux_set_csd_skip(iris_cuda_flux_t *tf, int skip);
/* iris_transformer_set_sref_bands: the single blocks rotate the K of
 * reference-image rows with their H / W RoPE pairs scaled by
 * shf + (slf - shf) * (d / 15)^2 (high frequencies attenuated, low amplified);
 * shf outside [0, 1] or slf < 1 means 1 (off). */
int iris_cuda_flux_set_sref_bands(iris_cuda_flux_t *tf, float shf, float slf);

/* Host only (no device needed): the adapters of a LoRA file that match a model
 * of this shape (n_double / n_single blocks, hidden and MLP widths), like the
 * reference's "LoRA: loaded N adapters" report (iris_lora.c:276).  Returns
 * their number (a fused Q|K|V counts once) or an error; per_kind (5 ints, may
 * be NULL) receives the format (1 XLabs, 2 Kohya, 3 Diffusers, 4 BFL) and the
 * counts of Q/K/V, output-projection, single linear1 and linear2 adapters. */
int iris_cuda_lora_probe(const char *path, int n_double, int n_single, int hidden, int mlp, int *per_kind);

/* One denoising step: velocity v(z, t, ctx), host buffers in and out.
 * Replaces iris_transformer_forward (iris_transformer_flux.c:3939); returns
 * malloc'd NCHW [C, h, w] or NULL. */
float *iris_cuda_transformer_forward(iris_cuda_flux_t *tf, const float *img_latent, int img_h,
                                     int img_w, const float *txt_emb, int txt_seq,
                                     float timestep);
/* Replaces iris_transformer_forward_with_multi_refs (iris_transformer_flux.c:4579). */
float *iris_cuda_transformer_forward_with_multi_refs(iris_cuda_flux_t *tf,
                                                     const float *img_latent, int img_h,
                                                     int img_w, const iris_cuda_ref_t *refs,
                                                     int num_refs, const float *txt_emb,
                                                     int txt_seq, float timestep);
/* Device-resident forward: every pointer (latent, ref latents, txt_emb, out)
 * is device memory; work is queued on iris_cuda_stream() and this call does
 * not synchronise.  out = [C, img_h, img_w]. */
int iris_cuda_flux_forward_dev(iris_cuda_flux_t *tf, const float *d_latent, int img_h,
                               int img_w, const iris_cuda_ref_t *d_refs, int num_refs,
                               const float *d_txt_emb, int txt_seq, float timestep,
                               float *d_out);

/* Run ONE block on a caller-supplied hidden state (per-block parity hook).
 * hidden: host f32 [txt_seq + img_h*img_w, hidden] in [TXT, IMG] row order,
 * updated in place; modulations are computed from `timestep`.  kind 0 runs
 * double block idx (replaces double_block_forward, iris_transformer_flux.c:2366,
 * with hidden split into its txt/img streams), kind 1 single block idx
 * (single_block_forward, :3761). */
int iris_cuda_flux_run_block(iris_cuda_flux_t *tf, int kind, int idx, float *hidden, int txt_seq,
                             int img_h, int img_w, float timestep);

/* One kernel of a profiled forward (iris_cuda_flux_profile). */
typedef struct {
    char name[32];
    double flops;        /* algorithmic FLOPs of the launch (0 if not FLOP-bound) */
    double bytes;        /* algorithmic HBM bytes (operands once + outputs once)  */
    float ms;            /* CUDA-event time of the launch                          */
} iris_cuda_kernel_time_t;

/* Time every kernel of one forward over the most recent input shape (no
 * graph; an event after each launch).  Returns the number of entries or a
 * negative status.  No reference counterpart (the reference's BLAS profile
 * counters, iris_transformer_flux.c:40-76, play the same role on the CPU). */
int iris_cuda_flux_profile(iris_cuda_flux_t *tf, float timestep, iris_cuda_kernel_time_t *out,
                           int max_entries);

/* ------------------------------------------------------------------ 2b. samplers */
/* Replaces iris_official_schedule (iris_sample.c:171). malloc'd [steps+1]. */
float *iris_cuda_official_schedule(int num_steps, int image_seq_len);
/* Replaces iris_linear_schedule (iris_sample.c:61). */
float *iris_cuda_linear_schedule(int num_steps);
/* Replaces iris_zimage_schedule (iris_sample.c:216) (IRIS_ZIMAGE_SHIFT honoured). */
float *iris_cuda_zimage_schedule(int num_steps, int image_seq_len);
/* Replaces iris_init_noise (iris_sample.c:1146): same xoshiro256** stream,
 * bit-identical values. malloc'd [batch, C, h, w]. */
float *iris_cuda_init_noise(int batch, int channels, int h, int w, int64_t seed);

/* Euler rectified-flow loop, host buffers.  Replaces iris_sample_euler
 * (iris_sample.c:313): returns malloc'd final latent.  batch must be 1. */
float *iris_cuda_sample_euler(iris_cuda_flux_t *tf, const float *z, int batch, int channels,
                              int h, int w, const float *text_emb, int text_seq,
                              const float *schedule, int num_steps,
                              void (*progress_callback)(int step, int total));
/* Replaces iris_sample_euler_cfg (iris_sample.c:717). */
float *iris_cuda_sample_euler_cfg(iris_cuda_flux_t *tf, const float *z, int batch,
                                  int channels, int h, int w, const float *text_emb_cond,
                                  int text_seq_cond, const float *text_emb_uncond,
                                  int text_seq_uncond, float guidance_scale,
                                  const float *schedule, int num_steps,
                                  void (*progress_callback)(int step, int total));
/* Replaces iris_sample_euler_with_multi_refs (iris_sample.c:630). */
float *iris_cuda_sample_euler_with_multi_refs(iris_cuda_flux_t *tf, const float *z, int batch,
                                              int channels, int h, int w,
                                              const iris_cuda_ref_t *refs, int num_refs,
                                              const float *text_emb, int text_seq,
                                              const float *schedule, int num_steps,
                                              void (*progress_callback)(int step, int total));
/* Device-resident sampler: d_z [C,h,w] is updated in place, d_txt (and
 * d_txt_uncond when guidance is used; NULL otherwise) are device buffers,
 * schedule is a host array.  Queued on iris_cuda_stream(); the call returns
 * after the denoising loop has been queued and its scratch released. */
int iris_cuda_sample_euler_dev(iris_cuda_flux_t *tf, float *d_z, int h, int w,
                               const float *d_txt, int txt_seq, const float *d_txt_uncond,
                               int txt_seq_uncond, float guidance, const float *schedule,
                               int num_steps);

/* ------------------------------------------------------------------ 2b2. multi-GPU
 * One NCCL communicator per process (no reference counterpart: the reference
 * is single-device).  NCCL is loaded at first use (dlopen "libnccl.so.2").
 * Every host wait that depends on peers is bounded (env IRIS_COMM_TIMEOUT_MS,
 * default 60000): a peer that never joins or dies yields
 * IRIS_CUDA_ERR_TIMEOUT and the communicator is aborted. */
#define IRIS_CUDA_COMM_ID_BYTES 128
/* Fill id_out (>= IRIS_CUDA_COMM_ID_BYTES) with a new unique id; one rank
 * creates it and hands it to the others. */
int iris_cuda_comm_unique_id(void *id_out, size_t id_bytes);
/* Join the communicator `id` as rank `rank` of `world` (collective). */
int iris_cuda_comm_init(const void *id, int world, int rank);
void iris_cuda_comm_destroy(void);
int iris_cuda_comm_world(void); /* 1 without a communicator */
int iris_cuda_comm_rank(void);

/* Classifier-free guidance with the two branches on a 2-rank communicator:
 * rank 0 runs the unconditional forward, rank 1 the conditional one; after
 * every step the pair all-gathers the velocities and both apply the guided
 * Euler update, so both return the same latent as iris_cuda_sample_euler_cfg
 * on one GPU.  Both ranks pass both contexts.  Arguments as
 * iris_cuda_sample_euler_cfg / iris_cuda_sample_euler_dev. */
float *iris_cuda_sample_euler_cfg_pair(iris_cuda_flux_t *tf, const float *z, int batch,
                                       int channels, int h, int w, const float *text_emb_cond,
                                       int text_seq_cond, const float *text_emb_uncond,
                                       int text_seq_uncond, float guidance_scale,
                                       const float *schedule, int num_steps,
                                       void (*progress_callback)(int step, int total));
int iris_cuda_sample_euler_cfg_pair_dev(iris_cuda_flux_t *tf, float *d_z, int h, int w,
                                        const float *d_txt_cond, const float *d_txt_uncond,
                                        int txt_seq, float guidance, const float *schedule,
                                        int num_steps);

/* ------------------------------------------------------------------ 2c. Z-Image S3-DiT */
typedef struct iris_cuda_zimage iris_cuda_zimage_t;

typedef struct {
    int dim;             /* 3840 */
    int heads;           /* dim / 128 */
    int n_layers;        /* 30 main layers */
    int n_refiner;       /* 2 noise + 2 context refiners */
    int cap_feat_dim;    /* 2560 */
    int in_channels;     /* 16 */
    int patch_size;      /* 2 */
    int ffn_dim;         /* 10240 */
    int adaln_dim;       /* min(dim, 256) */
    int t_mid;           /* timestep MLP width, 1024 */
    float rope_theta;    /* 256 */
    int axes_dims[3];    /* 32, 48, 48 */
} iris_cuda_zimage_config_t;

/* Replaces zi_transformer_load_safetensors (iris_transformer_zimage.c:2164)
 * with the config keys of the reference's model autodetection (iris.c:300-330). */
iris_cuda_zimage_t *iris_cuda_zimage_load(const char *model_dir);
/* Random-init Z-Image model (seeded device RNG); no reference counterpart. */
iris_cuda_zimage_t *iris_cuda_zimage_random(const iris_cuda_zimage_config_t *cfg, uint64_t seed,
                                            float std, int norm_unit);
/* Replaces zi_transformer_free (iris_transformer_zimage.c:2429). */
void iris_cuda_zimage_free(iris_cuda_zimage_t *z);
int iris_cuda_zimage_get_config(const iris_cuda_zimage_t *z, iris_cuda_zimage_config_t *out);
size_t iris_cuda_zimage_weight_bytes(const iris_cuda_zimage_t *z);
/* Replaces zi_transformer_forward (iris_transformer_zimage.c:1696): latent
 * [in_channels, latent_h, latent_w] (pre-patch), caption features
 * [cap_seq, cap_feat_dim]; returns malloc'd model output of the latent's shape. */
float *iris_cuda_zi_transformer_forward(iris_cuda_zimage_t *z, const float *latent, int latent_h,
                                        int latent_w, float timestep, const float *cap_feats,
                                        int cap_seq);
/* Replaces iris_sample_euler_zimage (iris_sample.c:412): t = 1 - sigma,
 * z += (sigma_next - sigma) * (-v).  Returns the malloc'd final latent. */
float *iris_cuda_sample_euler_zimage(iris_cuda_zimage_t *z, const float *zin, int batch,
                                     int channels, int h, int w, int patch_size,
                                     const float *cap_feats, int cap_seq, const float *schedule,
                                     int num_steps, void (*progress_callback)(int step, int total));
/* Device-resident Z-Image sampler (d_z updated in place, d_cap device). */
int iris_cuda_sample_euler_zimage_dev(iris_cuda_zimage_t *z, float *d_z, int h, int w,
                                      const float *d_cap, int cap_seq, const float *schedule,
                                      int num_steps);

/* ------------------------------------------------------------------ 2e. text encoder (Qwen3)
 * The step before the denoising loop: token ids -> text embeddings.  The
 * tokenizer (qwen3_tokenize_chat / qwen3_pad_tokens, iris_qwen3.h) stays on
 * the host; this layer replaces the model half of iris_qwen3.c. */
typedef struct iris_cuda_qwen3 iris_cuda_qwen3_t;

typedef struct {
    int hidden;          /* hidden_size (2560 for Qwen3-4B)         */
    int intermediate;    /* intermediate_size (9728)                */
    int heads;           /* num_attention_heads (32)                */
    int kv_heads;        /* num_key_value_heads (8)                 */
    int head_dim;        /* must be 128                             */
    int vocab;           /* vocab_size (151936)                     */
    int layers;          /* num_hidden_layers (36)                  */
    float rope_theta;    /* 1e6                                     */
} iris_cuda_qwen3_config_t;

/* Replaces qwen3_model_load (iris_qwen3.c:1578): model_dir is the
 * text_encoder directory (config.json, model.safetensors.index.json and
 * shards); weights resident in HBM as bf16 (the layers up to the last one
 * either extraction mode reads). */
iris_cuda_qwen3_t *iris_cuda_qwen3_load(const char *model_dir);
/* Random-init encoder (device RNG; projections N(0, 1/fan_in), norm scales
 * 1 + N(0, 0.1), embeddings N(0, 1)); no reference counterpart. */
iris_cuda_qwen3_t *iris_cuda_qwen3_random(const iris_cuda_qwen3_config_t *cfg, uint64_t seed);
/* Replaces qwen3_model_free (iris_qwen3.c:1754). */
void iris_cuda_qwen3_free(iris_cuda_qwen3_t *m);
int iris_cuda_qwen3_get_config(const iris_cuda_qwen3_t *m, iris_cuda_qwen3_config_t *out);
size_t iris_cuda_qwen3_weight_bytes(const iris_cuda_qwen3_t *m);
/* Replaces qwen3_set_extraction_mode (iris_qwen3.c:1849): 0 Flux (hidden
 * states after layers 8, 17, 26 concatenated, text_dim 3 * hidden), 1 Z-Image
 * (after layer num_layers - 2, text_dim hidden). */
int iris_cuda_qwen3_set_extraction_mode(iris_cuda_qwen3_t *m, int mode);
int iris_cuda_qwen3_text_dim(const iris_cuda_qwen3_t *m);
/* Replaces qwen3_forward (iris_qwen3.c:1072): input_ids / attention_mask
 * [seq_len] host int arrays (mask 1 = real token; NULL = all real), seq_len
 * <= 512; causal attention with masked keys at -1e9 as the reference.
 * Returns malloc'd f32 [seq_len, text_dim] or NULL. */
float *iris_cuda_qwen3_forward(iris_cuda_qwen3_t *m, const int *input_ids, const int *attention_mask, int seq_len);
/* Same with the embeddings written to device memory d_out [seq_len, text_dim]
 * (queued on the library stream; feeds iris_cuda_sample_euler_dev directly). */
int iris_cuda_qwen3_forward_dev(iris_cuda_qwen3_t *m, const int *input_ids, const int *attention_mask, int seq_len,
                                float *d_out);
/* kernels in one captured forward (0 before the first) */
uint64_t iris_cuda_qwen3_graph_kernels(const iris_cuda_qwen3_t *m);
/* Time every kernel of one forward at the last sequence length (no graph;
 * an event after each launch).  Returns the number of entries or a negative
 * status. */
int iris_cuda_qwen3_profile(iris_cuda_qwen3_t *m, iris_cuda_kernel_time_t *out, int max_entries);

/* ------------------------------------------------------------------ 2d. autoencoder decoder
 * The step after the denoising loop: latent -> RGB image on the GPU.  The
 * decoder of AutoencoderKLFlux2 (32 latent channels, batch-norm latent
 * statistics, post-quant conv) and of the Z-Image autoencoder (16 channels,
 * scaling / shift), base 128 channels, multipliers 1/2/4/4, three resnets per
 * level, one single-head attention in the mid block (iris_vae.c:1-30). */
typedef struct iris_cuda_vae iris_cuda_vae_t;

/* Same layout as the reference's iris_image (iris.h:73-78): width x height
 * pixels, channel-interleaved uint8, row-major. */
typedef struct {
    int width;
    int height;
    int channels;
    uint8_t *data;
} iris_cuda_image_t;

/* Replaces iris_vae_load_safetensors_ex (iris_vae.c:1227) on the decoder
 * weights of vae_dir (diffusion_pytorch_model.safetensors).  z_channels <= 0
 * reads latent_channels, scaling_factor and shift_factor from
 * vae_dir/config.json as iris_parse_vae_config does (iris_vae_config.h);
 * scaling == 0 selects the Flux batch-norm branch (eps 1e-4), else Z-Image's
 * x / scaling + shift (eps 1e-6). */
iris_cuda_vae_t *iris_cuda_vae_load(const char *vae_dir, int z_channels, float scaling, float shift);
/* Random-init decoder (seeded host RNG: projections N(0, 1/fan_in), norm
 * scales 1 + N(0, 0.1), biases N(0, 0.02)) for benchmarks; no reference
 * counterpart.  scaling == 0: Flux layout (batch-norm statistics, post-quant
 * conv), else Z-Image's. */
iris_cuda_vae_t *iris_cuda_vae_random(int z_channels, float scaling, float shift, uint64_t seed);
/* Replaces iris_vae_free (iris_vae.c:1024). */
void iris_cuda_vae_free(iris_cuda_vae_t *vae);
size_t iris_cuda_vae_weight_bytes(const iris_cuda_vae_t *vae);
/* Replaces iris_vae_decode (iris_vae.c:835): latent [4 z, latent_h, latent_w]
 * f32 (the transformer's patchified layout) -> image of 16 latent_w x
 * 16 latent_h RGB pixels, rounded as the reference does.  batch must be 1
 * (the reference's GPU decoder has the same limit, iris_vae.c:568).  Free
 * with iris_cuda_image_free. */
iris_cuda_image_t *iris_cuda_vae_decode(iris_cuda_vae_t *vae, const float *latent, int batch,
                                        int latent_h, int latent_w);
void iris_cuda_image_free(iris_cuda_image_t *img);
/* The f32 RGB planes [3, 16 latent_h, 16 latent_w] in [-1, 1] before the
 * uint8 conversion (host buffer). */
int iris_cuda_vae_decode_f32(iris_cuda_vae_t *vae, const float *latent, int latent_h, int latent_w,
                             float *out);
/* Device-resident decode (enqueued on the library stream): d_latent device
 * f32; d_rgb8 (uint8 [16 h, 16 w, 3]) and / or d_rgb_f32 ([3, 16 h, 16 w])
 * device outputs, either may be NULL. */
int iris_cuda_vae_decode_dev(iris_cuda_vae_t *vae, const float *d_latent, int latent_h, int latent_w,
                             uint8_t *d_rgb8, float *d_rgb_f32);
/* kernels in one captured decode (0 before the first decode) */
uint64_t iris_cuda_vae_graph_kernels(const iris_cuda_vae_t *vae);
/* Time every kernel of one decode at the most recent latent size (no graph;
 * an event after each launch), as iris_cuda_flux_profile does for the
 * transformer.  Returns the number of entries or a negative status. */
int iris_cuda_vae_profile(iris_cuda_vae_t *vae, iris_cuda_kernel_time_t *out, int max_entries);

/* ------------------------------------------------------------------ 3. iris_gpu_* surface
 * Device-resident tensors and ops with the names and signatures of
 * iris_metal.h.  Tensors are f32 or bf16 device buffers; "host" weight
 * pointers (const uint16_t *W_bf16) are uploaded once and cached by
 * address, exactly like the Metal backend's weight cache (iris_metal.m:1001). */
typedef struct iris_gpu_tensor *iris_gpu_tensor_t;

iris_gpu_tensor_t iris_gpu_tensor_create(const float *data, size_t num_elements);   /* :172 */
iris_gpu_tensor_t iris_gpu_tensor_alloc(size_t num_elements);                       /* :177 */
iris_gpu_tensor_t iris_gpu_tensor_alloc_persistent(size_t num_elements);            /* :184 */
void iris_gpu_tensor_set_persistent(iris_gpu_tensor_t tensor, int persistent);      /* :189 */
void iris_gpu_tensor_read(iris_gpu_tensor_t tensor, float *out);                    /* :195 */
void iris_gpu_tensor_write(iris_gpu_tensor_t tensor, const float *data);            /* :201 */
void iris_gpu_tensor_free(iris_gpu_tensor_t tensor);                                /* :213 */
size_t iris_gpu_tensor_size(iris_gpu_tensor_t tensor);                              /* :218 */
int iris_gpu_tensor_is_f16(iris_gpu_tensor_t tensor);                               /* :223 */
iris_gpu_tensor_t iris_gpu_tensor_alloc_f16(size_t num_elements);                   /* :276 */
iris_gpu_tensor_t iris_gpu_tensor_create_bf16(const float *data, size_t num_elements); /* :283 */
iris_gpu_tensor_t iris_gpu_tensor_f32_to_bf16(iris_gpu_tensor_t f32_tensor);        /* :571 */
iris_gpu_tensor_t iris_gpu_tensor_bf16_to_f32(iris_gpu_tensor_t bf16_tensor);       /* :574 */
int iris_gpu_convert_f32_to_bf16_into(iris_gpu_tensor_t bf16_out, iris_gpu_tensor_t f32_in); /* :577 */
int iris_gpu_convert_bf16_to_f32_into(iris_gpu_tensor_t f32_out, iris_gpu_tensor_t bf16_in); /* :580 */
void iris_gpu_sync(void);                                                           /* :309 */
void iris_gpu_batch_begin(void);                                                    /* :315 */
void iris_gpu_batch_end(void);                                                      /* :320 */

/* y = x W^T with a bf16 weight; x and result bf16.  :583 / :589 */
iris_gpu_tensor_t iris_gpu_linear_bf16_native(iris_gpu_tensor_t x, const uint16_t *W_bf16,
                                              int seq_len, int in_dim, int out_dim);
int iris_gpu_linear_bf16_native_into(iris_gpu_tensor_t out, iris_gpu_tensor_t x,
                                     const uint16_t *W_bf16, int seq_len, int in_dim,
                                     int out_dim);
/* (1 + scale) * LayerNorm(x) + shift, bf16.  :433 */
void iris_gpu_adaln_norm_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t x,
                              iris_gpu_tensor_t shift_bf16, iris_gpu_tensor_t scale_bf16,
                              int seq, int hidden, float eps);
/* Same result as iris_gpu_adaln_norm_bf16, for callers that cannot allocate
 * device memory (a host application whose pool allocator owns all device
 * memory, or latency-critical loops that cannot take cudaMalloc/cudaFree's
 * implicit synchronisation).  No counterpart in the reference.  Takes raw
 * bf16 device pointers the caller owns (x, out [seq, hidden]; shift, scale
 * [hidden]; out 8-byte aligned, the others 2-byte aligned, else
 * IRIS_CUDA_ERR_ARG) and a cudaStream_t (void *, 0 = default stream); queues
 * work without synchronising and calls no allocating routine.  Its scratch is one fixed array inside the library
 * (about 16.8 MB per GPU, held until exit): seq * hidden <= 4194304 and
 * hidden <= 8192, larger calls return IRIS_CUDA_ERR_ARG.  All calls share that
 * array, so calls whose GPU work overlaps race; the first call on a device
 * looks up the array's address and should come before any stream capture. */
int iris_gpu_adaln_norm_bf16_noalloc(void *out, const void *x, const void *shift,
                                     const void *scale, int seq, int hidden, float eps,
                                     void *stream);
/* per-head RMSNorm of Q and K in place.  :438 */
void iris_gpu_qk_rms_norm_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k,
                               iris_gpu_tensor_t q_weight_bf16, iris_gpu_tensor_t k_weight_bf16,
                               int seq, int heads, int head_dim, float eps);
/* text rows [0, img_offset) with txt tables, image rows with img tables.  :466 */
void iris_gpu_rope_unified_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *txt_cos,
                                const float *txt_sin, const float *img_cos,
                                const float *img_sin, const float *img_cos_k,
                                const float *img_sin_k, int seq, int img_offset, int heads,
                                int head_dim, int axis_dim);
/* one table for all rows.  :473 */
void iris_gpu_rope_2d_bf16(iris_gpu_tensor_t x, const float *cos_freq, const float *sin_freq,
                           int seq, int heads, int head_dim, int axis_dim);
/* softmax(Q K^T scale) V, bf16.  :423 (no sequence-length limit here) */
int iris_gpu_attention_fused_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q,
                                  iris_gpu_tensor_t K, iris_gpu_tensor_t V, int seq_q,
                                  int seq_k, int num_heads, int head_dim, float scale);
void iris_gpu_silu_mul_bf16(iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int n);   /* :457 */
void iris_gpu_gated_add_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t gate_bf16,
                             iris_gpu_tensor_t proj, int seq, int hidden);          /* :460 */
void iris_gpu_concat_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t a,
                              iris_gpu_tensor_t b, int seq_a, int seq_b, int hidden); /* :501 */
void iris_gpu_slice_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t in, int seq_out,
                             int hidden, int start);                               /* :506 */
void iris_gpu_split_qkv_mlp_bf16(iris_gpu_tensor_t fused, iris_gpu_tensor_t q,
                                 iris_gpu_tensor_t k, iris_gpu_tensor_t v,
                                 iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int seq,
                                 int hidden, int mlp_hidden);                      /* :511 */
void iris_gpu_concat_attn_mlp_bf16(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp,
                                   iris_gpu_tensor_t out, int seq, int hidden,
                                   int mlp_hidden);                                /* :517 */
/* capability probes of the Metal backend, answered for CUDA:  :28, :703, :743 */
int iris_metal_available(void);
int iris_metal_shaders_available(void);
int iris_bf16_pipeline_available(void);

/* The rest of the C surface of iris_metal.h that the reference's
 * iris_transformer_flux.c and iris_transformer_zimage.c call when built with
 * -DUSE_METAL (iris.c_b200/dropin builds them that way and links them here).
 * f32 linears and attention run on the bf16 tensor cores with f32
 * accumulation: f32 operands are rounded to bf16 on the way in. */
void iris_gpu_add_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b, int n); /* :451 */
void iris_gpu_copy_bf16(iris_gpu_tensor_t dst, iris_gpu_tensor_t src, size_t n);     /* :454 */
/* per-head RMSNorm of a bf16 tensor in place, bf16 weight [128].  :443 */
int iris_gpu_head_rms_norm_bf16(iris_gpu_tensor_t x, iris_gpu_tensor_t weight_bf16, int seq, int heads,
                                int head_dim, float eps);
/* x (f32 or bf16) W^T -> new bf16 tensor.  :269 */
iris_gpu_tensor_t iris_gpu_linear_bf16_bf16out(iris_gpu_tensor_t x, const uint16_t *W_bf16, int seq_len,
                                               int in_dim, int out_dim);
/* the other names of iris_gpu_attention_fused_bf16:  :291, :415 */
int iris_gpu_attention_mps_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim,
                                float scale);
int iris_gpu_attention_bf16_native(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                   iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim,
                                   float scale);
/* f32 host view of a tensor: the first call after GPU work copies it out;
 * host writes to it are copied back before the next op that uses the tensor.
 * Valid until the tensor is freed.  :208 */
float *iris_gpu_tensor_data(iris_gpu_tensor_t tensor);
/* f32 tensor ops; W / b / shift / scale / gate / norm weights / RoPE tables
 * are host pointers.  Weights are cached on the device by address (like the
 * Metal weight cache), RoPE tables by (address, size) until
 * iris_metal_rope_cache_begin. */
iris_gpu_tensor_t iris_gpu_linear(iris_gpu_tensor_t x, const float *W, const float *b, int seq_len,
                                  int in_dim, int out_dim);                                /* :239 */
iris_gpu_tensor_t iris_gpu_linear_bf16(iris_gpu_tensor_t x, const uint16_t *W_bf16, int seq_len,
                                       int in_dim, int out_dim);                           /* :250 */
int iris_gpu_linear_bf16_into(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const uint16_t *W_bf16,
                              int seq_len, int in_dim, int out_dim);                       /* :260 */
void iris_gpu_adaln_norm(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const float *shift,
                         const float *scale, int seq, int hidden, float eps);              /* :353 */
void iris_gpu_rms_norm_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const float *weight, int seq,
                           int hidden, float eps);                                         /* :358 */
void iris_gpu_qk_rms_norm(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *q_weight,
                          const float *k_weight, int seq, int heads, int head_dim, float eps); /* :362 */
void iris_gpu_rope_single_f32(iris_gpu_tensor_t x, const float *cos_freq, const float *sin_freq, int seq,
                              int heads, int head_dim);                                    /* :368 */
void iris_gpu_rope_single_pair_f32(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *cos_freq,
                                   const float *sin_freq, int seq, int heads, int head_dim); /* :374 */
void iris_gpu_rope_unified(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *txt_cos,
                           const float *txt_sin, const float *img_cos, const float *img_sin, int seq,
                           int img_offset, int heads, int head_dim, int axis_dim);         /* :379 */
void iris_gpu_silu_mul(iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int n);           /* :385 */
void iris_gpu_gated_add(iris_gpu_tensor_t out, const float *gate, iris_gpu_tensor_t proj, int seq,
                        int hidden);                                                       /* :388 */
void iris_gpu_split_qkv_mlp(iris_gpu_tensor_t fused, iris_gpu_tensor_t q, iris_gpu_tensor_t k,
                            iris_gpu_tensor_t v, iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int seq,
                            int hidden, int mlp_hidden);                                   /* :392 */
void iris_gpu_concat_attn_mlp(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp, iris_gpu_tensor_t out,
                              int seq, int hidden, int mlp_hidden);                        /* :398 */
int iris_gpu_attention_fused(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                             iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim,
                             float scale);                                                 /* :402 */
int iris_gpu_attention_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                            iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim,
                            float scale);                                                  /* :301 */
void iris_gpu_add_f32(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b, int n); /* :537 */
void iris_gpu_copy_f32(iris_gpu_tensor_t dst, iris_gpu_tensor_t src, size_t n);       /* :556 */
void iris_gpu_copy_region_f32(iris_gpu_tensor_t dst, size_t dst_offset, iris_gpu_tensor_t src,
                              size_t src_offset, size_t n);                                /* :566 */
/* Host-pointer attention: Q, K, V, out f32 [seq, heads * 128] (fused) or
 * [heads, seq, 128] (scores_scratch unused).  :649, :613 */
int iris_metal_attention_fused(float *out, const float *Q, const float *K, const float *V, int seq_q,
                               int seq_k, int num_heads, int head_dim, float scale);
void iris_metal_attention(float *out, const float *Q, const float *K, const float *V,
                          float *scores_scratch, int heads, int seq_q, int seq_k, int head_dim,
                          float scale);
/* The reference-token key bias of the SREF strength control (Metal-only in
 * the reference).  Stored; while it is non-zero the attention ops return
 * failure, and the reference's callers fall back to their CPU path, which
 * does not apply it either.  :409 */
void iris_metal_set_attention_bias(int ref_start, float bias);
/* batching: work is queued on one stream in order, an end waits for it.  :315-344, :125-149 */
void iris_gpu_chain_begin(void);
void iris_gpu_chain_end(void);
int iris_gpu_in_chain(void);
void iris_metal_begin_batch(void);
void iris_metal_end_batch(void);
int iris_metal_in_batch(void);
void iris_metal_sync(void);
void iris_metal_wait_idle(void);
/* runtime and caches (:23-54, :154): init returns 1 on success; reset drops
 * the weight caches, RoPE tables and pooled tensor blocks; the "weight" cache
 * is the one of f32 host weights, "bf16" the one of bf16 host weights; there
 * is no f16 cache (a no-op); rope_cache_begin forgets the RoPE tables. */
int iris_metal_init(void);
void iris_metal_cleanup(void);
void iris_metal_reset(void);
void iris_metal_reset_transient(void);
void iris_metal_rope_cache_begin(void);
void iris_metal_clear_weight_cache_only(void);
void iris_metal_clear_bf16_cache_only(void);
void iris_metal_clear_f16_cache_only(void);
void iris_metal_clear_activation_pool_only(void);
size_t iris_metal_memory_used(void);
/* upload host bf16 weights into the cache ahead of the first linear.  :710-725 */
void iris_metal_warmup_bf16(const uint16_t *bf16_weights, size_t num_elements);
void iris_metal_warmup_bf16_buffer(const uint16_t *bf16_weights, size_t num_elements);
void iris_metal_warmup_bf16_buffers_parallel(const uint16_t **ptrs, const size_t *counts, int n);
/* Ops of this surface that reported a failure (NULL / 0 / an error string)
 * since the library was loaded.  No counterpart in the reference: a caller
 * that falls back to its CPU path when an op fails (as the reference does)
 * can check that the GPU path really ran. */
unsigned long iris_gpu_op_failures(void);

#ifdef __cplusplus
}
#endif
#endif /* IRIS_CUDA_H */
