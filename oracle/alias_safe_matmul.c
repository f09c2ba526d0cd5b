/*
 * ORACLE BUILD SHIM — test infrastructure only.
 *
 * The reference's CPU Z-Image attention computes its output projection in
 * place: zi_attention (iris_transformer_zimage.c:716) accumulates the head
 * outputs in tf->work_tmp and then calls iris_matmul_t(out, attn_out, ...)
 * with out == tf->work_tmp as passed by zi_block_forward (:796).  A GEMM whose
 * output aliases its input is undefined; `make generic` and `make blas` give
 * different, both corrupted, results.
 *
 * The "_as" oracle libraries compile the reference's iris_kernels.c with its
 * iris_matmul_t renamed to iris_matmul_t_inplace_unsafe and link this
 * wrapper, which copies A first when it aliases C.  Every other line of the
 * reference is unchanged, and for non-aliased calls the result is identical.
 */
#include <stdlib.h>
#include <string.h>

void iris_matmul_t_inplace_unsafe(float *C, const float *A, const float *B, int M, int K, int N);

void iris_matmul_t(float *C, const float *A, const float *B, int M, int K, int N) {
    const char *c0 = (const char *)C, *c1 = c0 + (size_t)M * N * sizeof(float);
    const char *a0 = (const char *)A, *a1 = a0 + (size_t)M * K * sizeof(float);
    if (a0 < c1 && c0 < a1) {
        float *tmp = malloc((size_t)M * K * sizeof(float));
        if (tmp) {
            memcpy(tmp, A, (size_t)M * K * sizeof(float));
            iris_matmul_t_inplace_unsafe(C, tmp, B, M, K, N);
            free(tmp);
            return;
        }
    }
    iris_matmul_t_inplace_unsafe(C, A, B, M, K, N);
}
