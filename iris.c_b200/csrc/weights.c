/*
 * Weight sources shared by the model loaders: a tensor of the reference's
 * safetensors layout is written to device memory either from a model file
 * (converted to bf16 on the host, uploaded through a pinned staging buffer)
 * or from the seeded counter-based device RNG (random-init models), plus the
 * TMA descriptor helper used for every weight and activation operand.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "iris_internal.h"


/* Norm-scale tensors of both model families (drawn as 1 + N(0, 0.1) when
 * norm_unit is set): Flux QK-RMSNorm scales, Z-Image QK/pre/post RMSNorm
 * scales and the caption-embedder RMSNorm. */
static int is_norm_name(const char *name) {
    static const char *keys[] = {"norm_q.", "norm_k.", "norm_added_q.", "norm_added_k.",
                                 "attention_norm1.", "attention_norm2.", "ffn_norm1.",
                                 "ffn_norm2.", "cap_embedder.0."};
    for (size_t i = 0; i < sizeof(keys) / sizeof(keys[0]); i++)
        if (strstr(name, keys[i])) return 1;
    return 0;
}

/* Write the reference-layout tensor `name` ([numel] bf16) to device memory d_dst. */
int iris_wsrc_get(iris_wsrc_t *ws, const char *name, size_t numel, uint16_t *d_dst) {
    if (ws->random) {
        int unit = ws->norm_unit && is_norm_name(name);
        cudaError_t e = iris_launch_randn_bf16(d_dst, (long)numel, ws->seed, iris_crc32(name),
                                               unit ? 1.0f : 0.0f, unit ? 0.1f : ws->std,
                                               g_rt.stream);
        iris_count_launch(1);
        return iris_cuda_check(e, name);
    }
    const st_tensor_t *t = st_find(&ws->st, name);
    if (!t) return iris_fail(IRIS_CUDA_ERR_IO, "tensor %s not found", name);
    if (ws->host_stage_n < numel) {
        if (ws->host_stage) cudaFreeHost(ws->host_stage);
        ws->host_stage = NULL;
        ws->host_stage_n = 0;
        if (cudaMallocHost((void **)&ws->host_stage, numel * 2) != cudaSuccess)
            return iris_fail(IRIS_CUDA_ERR_OOM, "pinned staging for %s", name);
        ws->host_stage_n = numel;
    }
    /* the staging buffer is reused: finish the previous upload first */
    cudaStreamSynchronize(g_rt.stream);
    if (st_read_bf16(&ws->st, t, ws->host_stage, numel) != 0)
        return iris_fail(IRIS_CUDA_ERR_IO, "tensor %s: bad shape or dtype", name);
    return iris_cuda_check(cudaMemcpyAsync(d_dst, ws->host_stage, numel * 2,
                                           cudaMemcpyHostToDevice, g_rt.stream), name);
}

/* f32 copy of a (small) tensor, through a bf16 device temp */
int iris_wsrc_get_f32(iris_wsrc_t *ws, const char *name, size_t numel, float *d_dst, uint16_t *tmp) {
    int rc = iris_wsrc_get(ws, name, numel, tmp);
    if (rc) return rc;
    iris_count_launch(1);
    return iris_cuda_check(iris_launch_bf16_to_f32(tmp, d_dst, (long)numel, g_rt.stream), name);
}

int iris_mk_tmap(CUtensorMap *m, const void *p, int rows, int cols, int ld, int box) {
    int r = iris_make_tmap_bf16(m, p, (uint64_t)rows, (uint64_t)cols, (uint64_t)ld, (uint32_t)box);
    return r ? iris_fail(IRIS_CUDA_ERR_CUDA, "tensor map encode failed (%d)", r) : 0;
}

