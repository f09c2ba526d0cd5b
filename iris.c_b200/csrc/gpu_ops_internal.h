/*
 * Internals shared by the two halves of the op-level iris_gpu_* surface
 * (gpu_ops.c: tensors, caches, bf16 ops; gpu_ops_f32.c: f32 ops and the
 * host-pointer attention entry points).
 */
#ifndef IRIS_GPU_OPS_INTERNAL_H
#define IRIS_GPU_OPS_INTERNAL_H

#include "iris_internal.h"

struct iris_gpu_tensor {
    void *d;         /* device block from the op pool                         */
    size_t n;        /* elements                                              */
    size_t bytes;    /* block size (pool key)                                 */
    int bf16;        /* 1: bf16 elements ("f16" in the Metal naming)          */
    int persistent;
    float *host;     /* f32 host mirror handed out by iris_gpu_tensor_data    */
    int host_live;   /* the mirror may hold host writes the device has not seen */
};

/* a tensor from the op pool (no initialisation) */
iris_gpu_tensor_t op_tensor_new(size_t n, int bf16);
/* device pointer of t; a live host mirror is copied back first */
void *op_dev(iris_gpu_tensor_t t);
/* device copy of a host f32 vector of n values, zero-padded to npad >= n;
 * valid for work queued on the library stream after this call */
const float *op_vec(const float *h, size_t n, size_t npad);
/* device copy of a host f32 table, cached by (address, size) until
 * iris_metal_rope_cache_begin / reset (the Metal backend's RoPE cache,
 * iris_metal.m:1018-1067) */
const float *op_table(const float *h, size_t n);
/* bf16 scratch of n elements from the op pool, returned with op_scratch_put
 * once the work that reads it is queued (stream order makes reuse safe) */
void *op_scratch_get(size_t bytes);
void op_scratch_put(void *p, size_t bytes);
/* y[seq, out_dim] = x[seq, in_dim] (bf16, device) * W^T (+ bias);
 * W is a host weight (bf16 bits, or f32 when w_f32) cached on the device by
 * address; out is bf16 or f32 (out_f32) with row stride out_dim.
 * Returns 1 on success, 0 with the reason in iris_cuda_last_error(). */
int op_linear(const void *x_bf16, int seq, int in_dim, const void *W, int w_f32, const float *bias_host,
              int out_dim, void *out, int out_f32);
/* the SREF key bias set by iris_metal_set_attention_bias (0: off) */
float op_attention_bias(void);

/* failure reporting of the ops: records the reason (iris_cuda_last_error)
 * and counts the failure (iris_gpu_op_failures) */
int op_fail(int code, const char *fmt, ...);
int op_check(cudaError_t e, const char *what);
#define OP_FAIL(...) op_fail(IRIS_CUDA_ERR_ARG, __VA_ARGS__)

#endif
