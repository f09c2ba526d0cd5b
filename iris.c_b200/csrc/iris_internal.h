/*
 * Shared internals of the iris CUDA backend host code (C11).
 */
#ifndef IRIS_INTERNAL_H
#define IRIS_INTERNAL_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#include "iris_cuda.h"
#include "iris_kernels.h"

typedef struct {
    int initialized;
    int device;
    int num_sms;
    int cc_major, cc_minor;
    cudaStream_t stream;
    int *d_status;          /* device status word (bounded-wait failures) */
    uint64_t launches;      /* kernels enqueued (graph replays add their node count) */
} iris_rt_t;

extern iris_rt_t g_rt;

/* error reporting: sets the thread's last-error string and returns code */
int iris_fail(int code, const char *fmt, ...);
/* map a cudaError_t to a status, recording the message; 0 if success */
int iris_cuda_check(cudaError_t e, const char *what);

/* host-side fault injection (IRIS_CUDA_FAULT=alloc@N|launch@N|h2d@N):
 * returns 1 when the N-th call of that kind should fail. */
int iris_fault(const char *kind);

/* device allocation through the library (counts, fault injection) */
void *iris_dmalloc(size_t bytes);
void iris_dfree(void *p);

/* note `n` kernel launches (for iris_cuda_kernel_launches) */
static inline void iris_count_launch(uint64_t n) { g_rt.launches += n; }
/* the same, callable from the CUDA C++ translation units */
void iris_note_launches(uint64_t n);

/* ensure the runtime is up; returns status */
int iris_rt_ensure(void);
/* host -> device copy on the library stream, complete when it returns (use
 * instead of cudaMemcpy, whose DMA is not ordered with the library stream) */
int iris_h2d(void *dst, const void *src, size_t bytes);

/* ---------------- NCCL communicator (comm.c) ---------------- */
int iris_comm_world(void);  /* 1 without a communicator */
int iris_comm_rank(void);
int iris_comm_active(void);
/* in-place sum all-reduce of n f32 (bf16 = 0) or bf16 elements on the library stream */
int iris_comm_allreduce_sum(void *buf, size_t n, int bf16);
/* all-gather of n f32 per rank into recv [world * n] on the library stream */
int iris_comm_allgather_f32(const float *send, float *recv, size_t n);
/* bounded stream synchronisation while collectives may be queued */
int iris_comm_sync_stream(void);
/* wait for the library stream (bounded when a communicator exists) */
int iris_stream_drain(void);
/* symmetric device memory: an arena per rank mapped into every peer (CUDA IPC);
 * init is collective and (re)starts the bump allocation, alloc must follow the
 * same order on every rank; sym_peer maps a local object to peer's copy */
#define IRIS_COMM_MAX_PEERS 8
int iris_comm_sym_init(size_t bytes);
void *iris_comm_sym_alloc(size_t bytes);
void *iris_comm_sym_peer(const void *local_ptr, int peer);
int iris_comm_allgather_bytes(const void *send, void *recv, size_t bytes);

/* ---------------- safetensors (own reader) ---------------- */
typedef enum { ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2, ST_OTHER = 3, ST_I8 = 4 } st_dtype_t;

typedef struct {
    char name[256];
    st_dtype_t dtype;
    int ndim;
    int64_t shape[8];
    size_t offset, nbytes;
    int file;
} st_tensor_t;

typedef struct {
    int nfiles;
    void *maps[16];
    int fds[16];          /* kept open for pread (the weight uploads read with it) */
    size_t sizes[16];
    size_t data_start[16];
    int ntensors;
    st_tensor_t *tensors;
} st_model_t;

int st_open_dir(st_model_t *m, const char *transformer_dir);
int st_open_file(st_model_t *m, const char *path);
void st_close(st_model_t *m);
const st_tensor_t *st_find(const st_model_t *m, const char *name);
/* convert a tensor to bf16 bits into out (numel elements); returns 0 on success */
int st_read_bf16(const st_model_t *m, const st_tensor_t *t, uint16_t *out, size_t numel);
int st_read_f32(const st_model_t *m, const st_tensor_t *t, float *out, size_t numel);
/* the tensor's bytes in the mapped file (NULL when out of range) */
const void *st_raw(const st_model_t *m, const st_tensor_t *t);

/* ---------------- weight sources (weights.c) ---------------- */
typedef struct {
    int random;           /* 1: seeded device RNG, 0: safetensors file       */
    st_model_t st;
    uint64_t seed;
    float std;
    int norm_unit;        /* norm-scale tensors drawn as 1 + N(0, 0.1)       */
    /* file uploads (weights.c): a ring of pinned chunks filled by a pool of
       copy threads while earlier chunks are in flight to the device */
    uint8_t *ring[4];
    cudaEvent_t ring_ev[4];
    int ring_i;
    struct iris_cpool *pool;
    void *d_raw;          /* device landing for f32 / f16 tensors (converted there) */
    size_t d_raw_n;
    double bytes;         /* file bytes uploaded */
} iris_wsrc_t;

/* finish a weight source's uploads and release its device landing */
void iris_wsrc_free(iris_wsrc_t *ws);
/* the process-wide upload ring and reader threads (iris_cuda_cleanup) */
void iris_wsrc_release_staging(void);
/* device bytes -> pageable host memory through the pinned ring and the copy
 * threads, after the work queued on the library stream; synchronous */
int iris_d2h_staged(void *dst, const void *d_src, size_t bytes, const char *name);

/* Write the reference-layout tensor `name` ([numel] bf16) to device memory. */
int iris_wsrc_get(iris_wsrc_t *ws, const char *name, size_t numel, uint16_t *d_dst);
/* f32 copy of a small tensor through a bf16 device temp. */
int iris_wsrc_get_f32(iris_wsrc_t *ws, const char *name, size_t numel, float *d_dst, uint16_t *tmp);
/* bf16 tensor map over a row-major [rows, cols] matrix (row stride ld), box {64, box} */
int iris_mk_tmap(CUtensorMap *m, const void *p, int rows, int cols, int ld, int box);

/* simple "key": number extraction from a small JSON text */
int json_get_number(const char *json, const char *key, double *out);

/* 32-bit CRC (IEEE) of a string; keys the per-tensor RNG streams */
uint32_t iris_crc32(const char *s);

/* host bf16 helpers */
static inline uint16_t f32_to_bf16_bits(float f) {
    union { float f; uint32_t u; } v = {f};
    uint32_t u = v.u;
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf16_bits_to_f32(uint16_t b) {
    union { uint32_t u; float f; } v = {(uint32_t)b << 16};
    return v.f;
}

#endif
