/*
 * Private layout of the Flux transformer handle, shared by flux.c (loader,
 * plans, forward) and lora.c (adapter folding into the resident weights).
 */
#ifndef IRIS_FLUX_INTERNAL_H
#define IRIS_FLUX_INTERNAL_H

#include "iris_internal.h"

#define MAXREFS 8

typedef struct {
    uint16_t *w_qkv[2], *w_out[2], *w_in[2], *w_down[2]; /* [0] txt, [1] img */
    float *qn[2], *kn[2];
    CUtensorMap tm_qkv[2], tm_out[2], tm_in[2], tm_down[2];
} flux_dbl_t;

typedef struct {
    uint16_t *w_fused, *w_out;
    float *qn, *kn;
    CUtensorMap tm_fused, tm_out;
} flux_sgl_t;

typedef struct {
    int valid;
    int s_txt, img_h, img_w, n_img, n_img_total, S;
    int num_refs, ref_h[MAXREFS], ref_w[MAXREFS], ref_t[MAXREFS];
    float *hidden, *lat_in, *out, *txt_f32;
    uint16_t *rope_pos;      /* [S][4] RoPE position ids (T, H, W, L) per row */
    IrisRopeSpec *rope_spec; /* per rotation pair: frequency, axis, SREF K-side band scale */
    int rope_k_row0;         /* first row whose K takes the band scale in the single blocks (0 = off) */
    uint16_t *xmod, *q, *k, *v, *attn, *mlp, *cat, *tok_img, *tok_txt;
    /* tensor parallelism (symmetric memory, see comm.c): rows owned in chunks,
       partial updates received in recv [tp][chunk][H] f32, xmod shared */
    int chunk;
    float *recv;
    unsigned *flags;
    unsigned part_i, x_i;   /* (while enqueueing) partial / xmod syncs queued in this call */
    int part_pending;       /* a scattered update awaits the next adaLN */
    int ln_pending;         /* the last residual GEMM's reduction already applied the next adaLN */
    int a_box;              /* rows of the activation tensor maps' boxes (0 = 128): S rounded up to 8 when S <= 128 */
    uint16_t *ip_q, *ip_o;  /* IP-Adapter: pre-RoPE image Q and its attention output [S, H] */
    float *ws;              /* split-K workspace of short sequences (NULL otherwise) */
    size_t ws_bytes;
    CUtensorMap tm_xmod, tm_attn, tm_mlp, tm_cat, tm_tok_img, tm_tok_txt;
    cudaGraph_t graph;
    cudaGraphExec_t gexec;
    int graph_ok;
    uint64_t graph_kernels;
} flux_plan_t;

struct iris_cuda_flux {
    iris_cuda_flux_config_t cfg;
    int H, F, C, T, NH;
    /* tensor parallelism: this rank's shard of heads / MLP columns */
    int tp, tp_rank, NHl, Hl, Fl;
    uint16_t *w_x, *w_ctx, *w_t1, *w_t2, *w_mod, *w_proj;
    CUtensorMap tm_x, tm_ctx, tm_proj;
    flux_dbl_t *dbl;
    flux_sgl_t *sgl;
    size_t weight_bytes;
    float *t_dev, *sincos, *temb_h, *temb, *mods;
    flux_plan_t plan;
    /* weight source for iris_cuda_flux_read_weight */
    int random;
    uint64_t seed;
    float std;
    int norm_unit;
    char model_dir[1024];
    /* folded LoRA (NULL without one) */
    struct iris_flux_lora *lora;
    /* attached IP-Adapter (NULL without one) */
    struct iris_flux_ip *ip;
    /* SREF (sref.c): CSD temb delta [H] (NULL = off) and the device flag that
       gates it per forward (0 on the CFG sampler's unconditional branch);
       K-side RoPE band scaling of reference rows (1, 1 = off) */
    float *csd_delta, *csd_on;
    float sref_shf, sref_slf;
};

void iris_flux_sref_release(iris_cuda_flux_t *tf);
/* gate the CSD delta for the next forwards (stream-ordered): on = 0 or 1 */
int iris_flux_csd_branch(iris_cuda_flux_t *tf, int on);
/* K-side band scale of rotation pair d (0..15) of the H and W axes */
float iris_flux_sref_band(const iris_cuda_flux_t *tf, int d);

/* IP-Adapter state (ipadapter.c), read by the forward's hooks (flux.c) */
struct iris_flux_ip {
    int nb, nd, T;         /* adapter blocks (double then single), double blocks, image tokens */
    uint16_t *kv;          /* bf16 [2][nb][T][H]: every block's k, then every block's v */
    float *d_scale;        /* [nb] ip_scale * scale_mult * schedule multiplier (device) */
    float *h_scale;        /* [nb] ip_scale * scale_mult */
    float *h_cur;          /* [nb] staging of d_scale */
    float *embeds;         /* f32 [T, H] perceived embeddings */
    float mult;            /* current schedule multiplier */
    int sched_kind;        /* 0 none, 1 late, 2 early */
    float sched_param;
};
void iris_flux_ip_release(iris_cuda_flux_t *tf);
/* drop the plan (and its graph) so the next call rebuilds it with the current hooks */
void iris_flux_invalidate_plan(iris_cuda_flux_t *tf);

/* LoRA state (lora.c): the originals of the weights an adapter was folded
 * into, so a new adapter or an unload starts from the base model. */
void iris_flux_lora_release(iris_cuda_flux_t *tf);

#endif
