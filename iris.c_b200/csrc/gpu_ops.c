/*
 * The iris_gpu_* device-tensor surface of iris_metal.h (:155-600) and the
 * C runtime entry points around it (iris_metal_init / reset / cache control /
 * warmup, :23-154, :703-743), implemented on CUDA with the same names,
 * signatures and failure conventions: NULL / 0 on failure, void ops report
 * through iris_cuda_last_error().  With them the reference's own GPU block
 * code — the bf16 Flux path (iris_transformer_flux.c:2024-2292, :3243-3751)
 * and the Z-Image GPU path (iris_transformer_zimage.c:934-1556) — runs on
 * this backend unchanged.  The fused model path (flux.c, zimage.c) does not
 * use these entry points.
 *
 * This file: tensor objects, the op pool, the host mirror of
 * iris_gpu_tensor_data, the weight / table / vector upload caches and the
 * bf16 ops.  gpu_ops_f32.c holds the f32 ops.
 *
 * Design points (all work is queued in order on the library stream):
 *  - tensors come from an op pool of device blocks keyed by size: freeing
 *    returns the block without a device synchronisation, and the next
 *    allocation of that size reuses it (stream order makes this safe); the
 *    reference allocates and frees every intermediate of every block;
 *  - host weight pointers are uploaded once and kept as bf16 K-major GEMM
 *    operands keyed by (address, elements), like the Metal backend's bf16
 *    weight cache (iris_metal.m:1001); f32 host weights are rounded to bf16;
 *  - host RoPE tables are cached by (address, size) until
 *    iris_metal_rope_cache_begin, as in iris_metal.m:1018-1067;
 *  - small host vectors (modulation shift / scale / gate, norm weights) go
 *    through a ring of pinned staging slots;
 *  - iris_gpu_tensor_data returns an f32 host mirror (there is no unified
 *    memory between host and GPU here): the first call after GPU work copies
 *    the tensor out, host writes to the mirror are copied back before the
 *    next op that uses the tensor.
 */
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gpu_ops_internal.h"

/* ------------------------------------------------------------------ failures */
static unsigned long g_op_failures = 0;

int op_fail(int code, const char *fmt, ...) {
    char msg[400];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    g_op_failures++;
    return iris_fail(code, "%s", msg);
}

int op_check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 0;
    g_op_failures++;
    return iris_cuda_check(e, what);
}

unsigned long iris_gpu_op_failures(void) { return g_op_failures; }

/* ------------------------------------------------------------------ op pool */
typedef struct {
    void *p;
    size_t bytes;
} pblk_t;

static pblk_t *g_pool = NULL;
static int g_pool_n = 0, g_pool_cap = 0;
static size_t g_pool_bytes = 0;       /* bytes held by free blocks */
static size_t g_live_bytes = 0;       /* bytes handed out          */
#define POOL_LIMIT ((size_t)16 << 30)  /* free blocks kept at most  */

static size_t round_bytes(size_t b) { return (b + 255) & ~(size_t)255; }

static void pool_release_all(void) {
    if (g_pool_n) cudaStreamSynchronize(g_rt.stream);
    for (int i = 0; i < g_pool_n; i++) iris_dfree(g_pool[i].p);
    g_pool_n = 0;
    g_pool_bytes = 0;
}

void *op_scratch_get(size_t bytes) {
    bytes = round_bytes(bytes ? bytes : 16);
    for (int i = g_pool_n - 1; i >= 0; i--) {
        if (g_pool[i].bytes == bytes) {
            void *p = g_pool[i].p;
            g_pool[i] = g_pool[--g_pool_n];
            g_pool_bytes -= bytes;
            g_live_bytes += bytes;
            return p;
        }
    }
    void *p = iris_dmalloc(bytes);
    if (!p && g_pool_n) {  /* out of memory: give the free blocks back and retry */
        pool_release_all();
        p = iris_dmalloc(bytes);
    }
    if (p)
        g_live_bytes += bytes;
    else
        g_op_failures++;
    return p;
}

void op_scratch_put(void *p, size_t bytes) {
    if (!p) return;
    bytes = round_bytes(bytes ? bytes : 16);
    g_live_bytes -= bytes;
    if (g_pool_bytes + bytes > POOL_LIMIT || (g_pool_n == g_pool_cap && g_pool_cap >= 4096)) {
        cudaStreamSynchronize(g_rt.stream);
        iris_dfree(p);
        return;
    }
    if (g_pool_n == g_pool_cap) {
        int nc = g_pool_cap ? 2 * g_pool_cap : 64;
        pblk_t *q = (pblk_t *)realloc(g_pool, sizeof(pblk_t) * (size_t)nc);
        if (!q) {
            cudaStreamSynchronize(g_rt.stream);
            iris_dfree(p);
            return;
        }
        g_pool = q;
        g_pool_cap = nc;
    }
    g_pool[g_pool_n].p = p;
    g_pool[g_pool_n].bytes = bytes;
    g_pool_n++;
    g_pool_bytes += bytes;
}

/* ------------------------------------------------------------------ tensors */
iris_gpu_tensor_t op_tensor_new(size_t n, int bf16) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    iris_gpu_tensor_t t = (iris_gpu_tensor_t)calloc(1, sizeof(*t));
    if (!t) {
        op_fail(IRIS_CUDA_ERR_OOM, "tensor: out of host memory");
        return NULL;
    }
    t->bytes = round_bytes((n ? n : 1) * (bf16 ? 2 : 4));
    t->d = op_scratch_get(t->bytes);
    if (!t->d) {
        free(t);
        return NULL;
    }
    t->n = n;
    t->bf16 = bf16;
    return t;
}

/* f32 device staging, grown on demand (conversions of host data) */
static float *g_stage = NULL;
static size_t g_stage_n = 0;

static float *stage_f32(size_t n) {
    if (n > g_stage_n) {
        cudaStreamSynchronize(g_rt.stream);
        iris_dfree(g_stage);
        g_stage = (float *)iris_dmalloc(n * 4);
        g_stage_n = g_stage ? n : 0;
    }
    return g_stage;
}

/* host f32 -> tensor (bf16 tensors are rounded on the device) */
static int upload_f32(iris_gpu_tensor_t t, const float *data, size_t n) {
    if (!t->bf16)
        return op_check(cudaMemcpyAsync(t->d, data, n * 4, cudaMemcpyHostToDevice, g_rt.stream),
                               "tensor upload");
    float *s = stage_f32(n);
    if (!s) return IRIS_CUDA_ERR_OOM;
    int rc = op_check(cudaMemcpyAsync(s, data, n * 4, cudaMemcpyHostToDevice, g_rt.stream), "tensor upload");
    if (!rc) {
        iris_count_launch(1);
        rc = op_check(iris_launch_f32_to_bf16(s, t->d, (long)n, g_rt.stream), "to_bf16");
    }
    /* the staging buffer may be regrown by the next call: finish before returning */
    return rc ? rc : op_check(cudaStreamSynchronize(g_rt.stream), "tensor upload");
}

/* tensor -> host f32 (synchronous) */
static int download_f32(iris_gpu_tensor_t t, float *out) {
    if (!t->bf16) {
        int rc = op_check(cudaMemcpyAsync(out, t->d, t->n * 4, cudaMemcpyDeviceToHost, g_rt.stream),
                                 "tensor read");
        return rc ? rc : op_check(cudaStreamSynchronize(g_rt.stream), "tensor read");
    }
    float *s = stage_f32(t->n);
    if (!s) return IRIS_CUDA_ERR_OOM;
    iris_count_launch(1);
    int rc = op_check(iris_launch_bf16_to_f32(t->d, s, (long)t->n, g_rt.stream), "to_f32");
    if (!rc)
        rc = op_check(cudaMemcpyAsync(out, s, t->n * 4, cudaMemcpyDeviceToHost, g_rt.stream), "tensor read");
    return rc ? rc : op_check(cudaStreamSynchronize(g_rt.stream), "tensor read");
}

void *op_dev(iris_gpu_tensor_t t) {
    if (!t) return NULL;
    if (t->host_live) {
        t->host_live = 0;
        if (upload_f32(t, t->host, t->n)) return NULL;
    }
    return t->d;
}

iris_gpu_tensor_t iris_gpu_tensor_alloc(size_t n) { return op_tensor_new(n, 0); }
iris_gpu_tensor_t iris_gpu_tensor_alloc_f16(size_t n) { return op_tensor_new(n, 1); }

iris_gpu_tensor_t iris_gpu_tensor_alloc_persistent(size_t n) {
    iris_gpu_tensor_t t = op_tensor_new(n, 0);
    if (t) t->persistent = 1;
    return t;
}

void iris_gpu_tensor_set_persistent(iris_gpu_tensor_t t, int p) {
    if (t) t->persistent = p;
}

static iris_gpu_tensor_t create_from(const float *data, size_t n, int bf16) {
    iris_gpu_tensor_t t = op_tensor_new(n, bf16);
    if (!t) return NULL;
    if (data && upload_f32(t, data, n)) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

iris_gpu_tensor_t iris_gpu_tensor_create(const float *data, size_t n) { return create_from(data, n, 0); }

iris_gpu_tensor_t iris_gpu_tensor_create_bf16(const float *data, size_t n) {
    iris_gpu_tensor_t t = create_from(data, n, 1);
    if (t) t->persistent = 1;
    return t;
}

void iris_gpu_tensor_read(iris_gpu_tensor_t t, float *out) {
    if (!t || !out) {
        OP_FAIL("tensor_read: null argument");
        return;
    }
    if (t->host_live) {
        memcpy(out, t->host, t->n * 4);
        return;
    }
    download_f32(t, out);
}

void iris_gpu_tensor_write(iris_gpu_tensor_t t, const float *data) {
    if (!t || !data) {
        OP_FAIL("tensor_write: null argument");
        return;
    }
    t->host_live = 0; /* the device copy is the current one again */
    upload_f32(t, data, t->n);
}

float *iris_gpu_tensor_data(iris_gpu_tensor_t t) {
    if (!t) {
        OP_FAIL("tensor_data: null tensor");
        return NULL;
    }
    if (!t->host) {
        t->host = (float *)malloc((t->n ? t->n : 1) * 4);
        if (!t->host) {
            op_fail(IRIS_CUDA_ERR_OOM, "tensor_data: out of host memory");
            return NULL;
        }
    }
    if (!t->host_live) {
        if (download_f32(t, t->host)) return NULL;
        t->host_live = 1;
    }
    return t->host;
}

void iris_gpu_tensor_free(iris_gpu_tensor_t t) {
    if (!t) return;
    op_scratch_put(t->d, t->bytes);
    free(t->host);
    free(t);
}

size_t iris_gpu_tensor_size(iris_gpu_tensor_t t) { return t ? t->n : 0; }
int iris_gpu_tensor_is_f16(iris_gpu_tensor_t t) { return t ? t->bf16 : 0; }

iris_gpu_tensor_t iris_gpu_tensor_f32_to_bf16(iris_gpu_tensor_t f) {
    if (!f || f->bf16) {
        OP_FAIL("tensor_f32_to_bf16: needs an f32 tensor");
        return NULL;
    }
    const float *src = (const float *)op_dev(f);
    iris_gpu_tensor_t t = op_tensor_new(f->n, 1);
    if (!t || !src) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    iris_count_launch(1);
    if (op_check(iris_launch_f32_to_bf16(src, t->d, (long)f->n, g_rt.stream), "to_bf16")) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

iris_gpu_tensor_t iris_gpu_tensor_bf16_to_f32(iris_gpu_tensor_t b) {
    if (!b || !b->bf16) {
        OP_FAIL("tensor_bf16_to_f32: needs a bf16 tensor");
        return NULL;
    }
    const void *src = op_dev(b);
    iris_gpu_tensor_t t = op_tensor_new(b->n, 0);
    if (!t || !src) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    iris_count_launch(1);
    if (op_check(iris_launch_bf16_to_f32(src, (float *)t->d, (long)b->n, g_rt.stream), "to_f32")) {
        iris_gpu_tensor_free(t);
        return NULL;
    }
    return t;
}

int iris_gpu_convert_f32_to_bf16_into(iris_gpu_tensor_t out, iris_gpu_tensor_t in) {
    if (!out || !in || !out->bf16 || in->bf16 || out->n < in->n)
        return OP_FAIL("convert_f32_to_bf16_into: needs f32 in, bf16 out of at least its size"), 0;
    const float *s = (const float *)op_dev(in);
    void *d = op_dev(out);
    if (!s || !d) return 0;
    iris_count_launch(1);
    return op_check(iris_launch_f32_to_bf16(s, d, (long)in->n, g_rt.stream), "to_bf16") == 0;
}

int iris_gpu_convert_bf16_to_f32_into(iris_gpu_tensor_t out, iris_gpu_tensor_t in) {
    if (!out || !in || out->bf16 || !in->bf16 || out->n < in->n)
        return OP_FAIL("convert_bf16_to_f32_into: needs bf16 in, f32 out of at least its size"), 0;
    const void *s = op_dev(in);
    float *d = (float *)op_dev(out);
    if (!s || !d) return 0;
    iris_count_launch(1);
    return op_check(iris_launch_bf16_to_f32(s, d, (long)in->n, g_rt.stream), "to_f32") == 0;
}

/* ------------------------------------------------------------------ batching and runtime names */
static int g_in_batch = 0, g_in_chain = 0;

void iris_gpu_sync(void) {
    if (g_rt.initialized) op_check(cudaStreamSynchronize(g_rt.stream), "sync");
}
/* Work is queued on one stream in order; a batch needs no extra encoding and
 * its end waits for the queued work, as the Metal batch's commit does. */
void iris_gpu_batch_begin(void) { g_in_batch = 1; }
void iris_gpu_batch_end(void) {
    g_in_batch = 0;
    iris_gpu_sync();
}
void iris_gpu_chain_begin(void) { g_in_chain = 1; }
void iris_gpu_chain_end(void) {
    g_in_chain = 0;
    iris_gpu_sync();
}
int iris_gpu_in_chain(void) { return g_in_chain; }
void iris_metal_begin_batch(void) { g_in_batch = 1; }
void iris_metal_end_batch(void) { iris_gpu_batch_end(); }
int iris_metal_in_batch(void) { return g_in_batch; }
void iris_metal_sync(void) { iris_gpu_sync(); }
void iris_metal_wait_idle(void) { iris_gpu_sync(); }

/* iris_metal_init returns 1 on success (iris_metal.h:23) */
int iris_metal_init(void) { return iris_rt_ensure() == IRIS_CUDA_OK; }

/* ------------------------------------------------------------------ small host vectors */
#define VR_SLOTS 256
#define VR_SLOT_FLOATS 16384
static float *g_vr_host = NULL, *g_vr_dev = NULL;
static cudaEvent_t g_vr_ev[VR_SLOTS];
static int g_vr_used[VR_SLOTS];
static int g_vr_next = 0;

static void vr_release(void) {
    if (!g_vr_host) return;
    cudaStreamSynchronize(g_rt.stream);
    for (int i = 0; i < VR_SLOTS; i++)
        if (g_vr_ev[i]) cudaEventDestroy(g_vr_ev[i]);
    memset(g_vr_ev, 0, sizeof(g_vr_ev));
    memset(g_vr_used, 0, sizeof(g_vr_used));
    cudaFreeHost(g_vr_host);
    iris_dfree(g_vr_dev);
    g_vr_host = g_vr_dev = NULL;
}

const float *op_vec(const float *h, size_t n, size_t npad) {
    if (!h) {
        OP_FAIL("null host vector");
        return NULL;
    }
    if (npad < n) npad = n;
    if (npad > VR_SLOT_FLOATS) { /* rare: a dedicated block returned to the pool right away */
        float *d = (float *)op_scratch_get(npad * 4);
        if (!d) return NULL;
        if (npad > n) cudaMemsetAsync(d + n, 0, (npad - n) * 4, g_rt.stream);
        if (op_check(cudaMemcpyAsync(d, h, n * 4, cudaMemcpyHostToDevice, g_rt.stream), "vector upload")) {
            op_scratch_put(d, npad * 4);
            return NULL;
        }
        op_scratch_put(d, npad * 4); /* later users of the block are queued after this op */
        return d;
    }
    if (!g_vr_host) {
        if (op_check(cudaMallocHost((void **)&g_vr_host, (size_t)VR_SLOTS * VR_SLOT_FLOATS * 4),
                            "pinned vector ring"))
            return NULL;
        g_vr_dev = (float *)iris_dmalloc((size_t)VR_SLOTS * VR_SLOT_FLOATS * 4);
        if (!g_vr_dev) {
            cudaFreeHost(g_vr_host);
            g_vr_host = NULL;
            return NULL;
        }
        for (int i = 0; i < VR_SLOTS; i++)
            if (op_check(cudaEventCreateWithFlags(&g_vr_ev[i], cudaEventDisableTiming), "event")) {
                vr_release();
                return NULL;
            }
    }
    const int s = g_vr_next;
    g_vr_next = (g_vr_next + 1) % VR_SLOTS;
    if (g_vr_used[s]) cudaEventSynchronize(g_vr_ev[s]); /* its previous DMA has read the slot */
    float *hs = g_vr_host + (size_t)s * VR_SLOT_FLOATS;
    float *ds = g_vr_dev + (size_t)s * VR_SLOT_FLOATS;
    memcpy(hs, h, n * 4);
    if (npad > n) memset(hs + n, 0, (npad - n) * 4);
    if (op_check(cudaMemcpyAsync(ds, hs, npad * 4, cudaMemcpyHostToDevice, g_rt.stream), "vector upload"))
        return NULL;
    cudaEventRecord(g_vr_ev[s], g_rt.stream);
    g_vr_used[s] = 1;
    return ds;
}

/* ------------------------------------------------------------------ RoPE tables */
#define TABLES 16
typedef struct {
    const float *host;
    size_t n;
    float *dev;
} table_t;
static table_t g_tab[TABLES];
static int g_tab_n = 0, g_tab_next = 0;

static void tables_clear(void) {
    for (int i = 0; i < g_tab_n; i++) op_scratch_put(g_tab[i].dev, g_tab[i].n * 4);
    memset(g_tab, 0, sizeof(g_tab));
    g_tab_n = g_tab_next = 0;
}

const float *op_table(const float *h, size_t n) {
    if (!h || !n) {
        OP_FAIL("null host table");
        return NULL;
    }
    for (int i = 0; i < g_tab_n; i++)
        if (g_tab[i].host == h && g_tab[i].n == n) return g_tab[i].dev;
    float *d = (float *)op_scratch_get(n * 4);
    if (!d) return NULL;
    if (op_check(cudaMemcpyAsync(d, h, n * 4, cudaMemcpyHostToDevice, g_rt.stream), "table upload")) {
        op_scratch_put(d, n * 4);
        return NULL;
    }
    int slot;
    if (g_tab_n < TABLES) {
        slot = g_tab_n++;
    } else { /* full: replace the oldest entry (its block returns to the pool in stream order) */
        slot = g_tab_next;
        g_tab_next = (g_tab_next + 1) % TABLES;
        op_scratch_put(g_tab[slot].dev, g_tab[slot].n * 4);
    }
    g_tab[slot].host = h;
    g_tab[slot].n = n;
    g_tab[slot].dev = d;
    return d;
}

void iris_metal_rope_cache_begin(void) { tables_clear(); }

/* ------------------------------------------------------------------ weight cache */
typedef struct {
    const void *host;  /* key: host address ...            */
    size_t n;          /* ... and element count            */
    int f32src;        /* uploaded from f32 (rounded to bf16) */
    uint16_t *dev;     /* bf16 [rows_pad, cols] (rows * cols before the first shaped use) */
    int rows, cols, rows_pad;
    CUtensorMap tm;
} wentry_t;

static wentry_t *g_wc = NULL;
static int g_wc_n = 0, g_wc_cap = 0;

static void wcache_clear(int f32src) {
    int k = 0;
    for (int i = 0; i < g_wc_n; i++) {
        if (g_wc[i].f32src == f32src) {
            iris_dfree(g_wc[i].dev);
        } else {
            g_wc[k++] = g_wc[i];
        }
    }
    g_wc_n = k;
}

/* An entry matches on (address, elements, source type) and, once it has been
 * used as a GEMM operand, on its shape; a warmed-up entry (no shape yet) is
 * adopted by the first shaped use.  Different shapes at one address (a host
 * buffer reused for another weight) get separate entries. */
static wentry_t *wcache_find(const void *w, size_t n, int f32src, int rows, int cols) {
    for (int i = g_wc_n - 1; i >= 0; i--) {
        const wentry_t *e = &g_wc[i];
        if (e->host == w && e->n == n && e->f32src == f32src &&
            (rows < 0 || e->rows == 0 || (e->rows == rows && e->cols == cols)))
            return &g_wc[i];
    }
    return NULL;
}

/* upload a host weight of n elements as bf16 (f32 sources rounded on the device) */
static wentry_t *wcache_add(const void *w, size_t n, int f32src, size_t n_alloc) {
    if (g_wc_n == g_wc_cap) {
        int nc = g_wc_cap ? 2 * g_wc_cap : 256;
        wentry_t *p = (wentry_t *)realloc(g_wc, sizeof(wentry_t) * (size_t)nc);
        if (!p) {
            op_fail(IRIS_CUDA_ERR_OOM, "weight cache: out of host memory");
            return NULL;
        }
        g_wc = p;
        g_wc_cap = nc;
    }
    wentry_t *e = &g_wc[g_wc_n];
    memset(e, 0, sizeof(*e));
    e->dev = (uint16_t *)iris_dmalloc(n_alloc * 2);
    if (!e->dev) return NULL;
    if (n_alloc > n) cudaMemsetAsync(e->dev + n, 0, (n_alloc - n) * 2, g_rt.stream);
    int rc;
    if (!f32src) {
        rc = iris_h2d(e->dev, w, n * 2);
    } else {
        float *s = stage_f32(n);
        rc = s ? op_check(cudaMemcpyAsync(s, w, n * 4, cudaMemcpyHostToDevice, g_rt.stream), "weight upload")
               : IRIS_CUDA_ERR_OOM;
        if (!rc) {
            iris_count_launch(1);
            rc = op_check(iris_launch_f32_to_bf16(s, e->dev, (long)n, g_rt.stream), "weight to bf16");
        }
        if (!rc) rc = op_check(cudaStreamSynchronize(g_rt.stream), "weight upload");
    }
    if (rc) {
        iris_dfree(e->dev);
        return NULL;
    }
    e->host = w;
    e->n = n;
    e->f32src = f32src;
    g_wc_n++;
    return e;
}

/* the entry of host weight W [rows, cols] with its GEMM operand ready: rows
 * padded with zeros to a multiple of 128 and a tensor map built */
static wentry_t *weight_for(const void *W, int f32src, int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    const int rows_pad = (rows + 127) / 128 * 128;
    wentry_t *e = wcache_find(W, n, f32src, rows, cols);
    if (!e) e = wcache_add(W, n, f32src, (size_t)rows_pad * cols);
    if (!e) return NULL;
    if (e->rows == rows && e->cols == cols) return e;
    if ((size_t)rows_pad * cols != n) {
        /* warmed up without a shape and rows not a multiple of 128: re-lay with padding */
        uint16_t *d = (uint16_t *)iris_dmalloc((size_t)rows_pad * cols * 2);
        if (!d) return NULL;
        cudaMemsetAsync(d, 0, (size_t)rows_pad * cols * 2, g_rt.stream);
        cudaMemcpyAsync(d, e->dev, n * 2, cudaMemcpyDeviceToDevice, g_rt.stream);
        cudaStreamSynchronize(g_rt.stream);
        iris_dfree(e->dev);
        e->dev = d;
    }
    if (iris_make_tmap_bf16(&e->tm, e->dev, (uint64_t)rows_pad, (uint64_t)cols, (uint64_t)cols, 128)) {
        op_fail(IRIS_CUDA_ERR_ARG, "weight [%d, %d]: tensor map", rows, cols);
        return NULL;
    }
    e->rows = rows;
    e->cols = cols;
    e->rows_pad = rows_pad;
    return e;
}

void iris_metal_warmup_bf16(const uint16_t *w, size_t n) {
    if (!w || !n || iris_rt_ensure() != IRIS_CUDA_OK) return;
    if (!wcache_find(w, n, 0, -1, -1)) wcache_add(w, n, 0, n);
}
void iris_metal_warmup_bf16_buffer(const uint16_t *w, size_t n) { iris_metal_warmup_bf16(w, n); }
void iris_metal_warmup_bf16_buffers_parallel(const uint16_t **ptrs, const size_t *counts, int n) {
    for (int i = 0; ptrs && counts && i < n; i++) iris_metal_warmup_bf16(ptrs[i], counts[i]);
}

/* cache control (iris_metal.h:41-54): the f32 weight cache is the Metal
 * "weight cache", the bf16 one its "bf16 cache"; there is no f16 cache */
void iris_metal_clear_weight_cache_only(void) {
    if (!g_rt.initialized) return;
    iris_gpu_sync();
    wcache_clear(1);
}
void iris_metal_clear_bf16_cache_only(void) {
    if (!g_rt.initialized) return;
    iris_gpu_sync();
    wcache_clear(0);
}
void iris_metal_clear_f16_cache_only(void) {
    if (g_rt.initialized) iris_gpu_sync();
}
void iris_metal_clear_activation_pool_only(void) {
    if (!g_rt.initialized) return;
    iris_gpu_sync();
    pool_release_all();
}
void iris_metal_reset_transient(void) {
    if (!g_rt.initialized) return;
    iris_gpu_sync();
    tables_clear();
    pool_release_all();
}
void iris_metal_reset(void) {
    if (!g_rt.initialized) return;
    iris_gpu_sync();
    wcache_clear(0);
    wcache_clear(1);
    tables_clear();
    pool_release_all();
}
void iris_metal_cleanup(void) {
    if (!g_rt.initialized) return;
    iris_metal_reset();
    vr_release();
    iris_dfree(g_stage);
    g_stage = NULL;
    g_stage_n = 0;
}
size_t iris_metal_memory_used(void) {
    size_t b = g_pool_bytes + g_live_bytes + g_stage_n * 4;
    for (int i = 0; i < g_wc_n; i++) b += (size_t)(g_wc[i].rows_pad ? (size_t)g_wc[i].rows_pad * g_wc[i].cols : g_wc[i].n) * 2;
    return b;
}

/* ------------------------------------------------------------------ GEMM */
int op_linear(const void *x_bf16, int seq, int in_dim, const void *W, int w_f32, const float *bias_host,
              int out_dim, void *out, int out_f32) {
    if (!x_bf16 || !W || !out) return OP_FAIL("linear: null argument"), 0;
    if (seq <= 0 || in_dim <= 0 || out_dim <= 0 || in_dim % 64)
        return OP_FAIL("linear: unsupported shape %d x %d -> %d (in_dim must be a multiple of 64)", seq, in_dim,
                       out_dim),
               0;
    wentry_t *w = weight_for(W, w_f32, out_dim, in_dim);
    if (!w) return 0;
    const int npad = w->rows_pad;
    const float *bias = NULL;
    if (bias_host && !(bias = op_vec(bias_host, (size_t)out_dim, (size_t)npad))) return 0;
    const size_t esz = out_f32 ? 4 : 2;
    void *dst = out;
    if (npad != out_dim && !(dst = op_scratch_get((size_t)seq * npad * esz))) return 0;
    IrisGemmParams p;
    memset(&p, 0, sizeof(p));
    if (iris_make_tmap_bf16(&p.tmap_a, x_bf16, (uint64_t)seq, (uint64_t)in_dim, (uint64_t)in_dim, 128)) {
        if (dst != out) op_scratch_put(dst, (size_t)seq * npad * esz);
        return OP_FAIL("linear: input tensor map"), 0;
    }
    p.tmap_b[0] = w->tm;
    p.ngroups = 1;
    p.rows[0] = seq;
    p.N = npad;
    p.K = in_dim;
    p.bn = (npad % 256 == 0) ? 256 : 128;
    p.mode = out_f32 ? IRIS_EPI_F32 : IRIS_EPI_BF16;
    p.out = dst;
    p.ldo = npad;
    p.bias = bias;
    p.status = g_rt.d_status;
    int launches = 1;
    int rc = op_check(iris_launch_gemm_ex(&p, g_rt.num_sms, g_rt.stream, &launches), "linear");
    iris_count_launch((uint64_t)launches);
    if (!rc && dst != out)
        rc = op_check(cudaMemcpy2DAsync(out, (size_t)out_dim * esz, dst, (size_t)npad * esz,
                                               (size_t)out_dim * esz, (size_t)seq, cudaMemcpyDeviceToDevice,
                                               g_rt.stream),
                             "linear output");
    if (dst != out) op_scratch_put(dst, (size_t)seq * npad * esz);
    return rc == 0;
}

int iris_gpu_linear_bf16_native_into(iris_gpu_tensor_t out, iris_gpu_tensor_t x, const uint16_t *W,
                                     int seq, int in_dim, int out_dim) {
    if (!out || !x || !W || !x->bf16 || !out->bf16)
        return OP_FAIL("linear_bf16_native: needs bf16 tensors and a weight"), 0;
    if (x->n < (size_t)seq * in_dim || out->n < (size_t)seq * out_dim)
        return OP_FAIL("linear_bf16_native: tensors smaller than %d x %d -> %d", seq, in_dim, out_dim), 0;
    const void *xd = op_dev(x);
    void *od = op_dev(out);
    return xd && od && op_linear(xd, seq, in_dim, W, 0, NULL, out_dim, od, 0);
}

iris_gpu_tensor_t iris_gpu_linear_bf16_native(iris_gpu_tensor_t x, const uint16_t *W, int seq,
                                              int in_dim, int out_dim) {
    iris_gpu_tensor_t out = op_tensor_new((size_t)seq * out_dim, 1);
    if (!out) return NULL;
    if (!iris_gpu_linear_bf16_native_into(out, x, W, seq, in_dim, out_dim)) {
        iris_gpu_tensor_free(out);
        return NULL;
    }
    return out;
}

/* bf16 view of a tensor's first n elements: the tensor itself, or a pool
 * block with its f32 contents rounded (*tmp set, returned with op_scratch_put) */
static const void *as_bf16(iris_gpu_tensor_t t, size_t n, void **tmp) {
    *tmp = NULL;
    const void *d = op_dev(t);
    if (!d || t->bf16) return d;
    void *b = op_scratch_get(n * 2);
    if (!b) return NULL;
    iris_count_launch(1);
    if (op_check(iris_launch_f32_to_bf16((const float *)d, b, (long)n, g_rt.stream), "to_bf16")) {
        op_scratch_put(b, n * 2);
        return NULL;
    }
    *tmp = b;
    return b;
}

/* x (f32 or bf16) * W^T -> bf16 tensor (iris_metal.h:269) */
iris_gpu_tensor_t iris_gpu_linear_bf16_bf16out(iris_gpu_tensor_t x, const uint16_t *W, int seq, int in_dim,
                                               int out_dim) {
    if (!x || !W || x->n < (size_t)seq * in_dim) {
        OP_FAIL("linear_bf16_bf16out: bad arguments");
        return NULL;
    }
    void *tmp;
    const void *xb = as_bf16(x, (size_t)seq * in_dim, &tmp);
    iris_gpu_tensor_t out = xb ? op_tensor_new((size_t)seq * out_dim, 1) : NULL;
    int ok = out && op_linear(xb, seq, in_dim, W, 0, NULL, out_dim, out->d, 0);
    if (tmp) op_scratch_put(tmp, (size_t)seq * in_dim * 2);
    if (!ok) {
        iris_gpu_tensor_free(out);
        return NULL;
    }
    return out;
}

/* ------------------------------------------------------------------ bf16 norms / rope */
/* bf16 or f32 tensor of n values -> f32 device vector (a pool block, *tmp) */
static const float *vec_f32(iris_gpu_tensor_t t, size_t n, void **tmp) {
    *tmp = NULL;
    if (!t || t->n < n) return NULL;
    const void *d = op_dev(t);
    if (!d || !t->bf16) return (const float *)d;
    float *f = (float *)op_scratch_get(n * 4);
    if (!f) return NULL;
    iris_count_launch(1);
    if (op_check(iris_launch_bf16_to_f32(d, f, (long)n, g_rt.stream), "to_f32")) {
        op_scratch_put(f, n * 4);
        return NULL;
    }
    *tmp = f;
    return f;
}

void iris_gpu_adaln_norm_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t x, iris_gpu_tensor_t shift,
                              iris_gpu_tensor_t scale, int seq, int hidden, float eps) {
    if (!out || !x || !shift || !scale || !out->bf16) {
        OP_FAIL("adaln_norm_bf16: needs a bf16 output and all inputs");
        return;
    }
    const size_t n = (size_t)seq * hidden;
    if (x->n < n || out->n < n || hidden % 4) {
        OP_FAIL("adaln_norm_bf16: bad shape %d x %d", seq, hidden);
        return;
    }
    void *t0, *t1, *t2;
    const float *xf = vec_f32(x, n, &t0);
    const float *sh = vec_f32(shift, (size_t)hidden, &t1);
    const float *sc = vec_f32(scale, (size_t)hidden, &t2);
    void *od = op_dev(out);
    if (xf && sh && sc && od) {
        iris_count_launch(1);
        op_check(iris_launch_adaln(xf, hidden, od, hidden, seq, hidden, sh, sc, NULL, NULL, seq, eps,
                                          g_rt.stream),
                        "adaln");
    }
    op_scratch_put(t0, n * 4);
    op_scratch_put(t1, (size_t)hidden * 4);
    op_scratch_put(t2, (size_t)hidden * 4);
}

void iris_gpu_qk_rms_norm_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k, iris_gpu_tensor_t qw,
                               iris_gpu_tensor_t kw, int seq, int heads, int head_dim, float eps) {
    if (!q || !k || !q->bf16 || !k->bf16 || head_dim != 128) {
        OP_FAIL("qk_rms_norm_bf16: needs bf16 q/k with head_dim 128");
        return;
    }
    void *t0, *t1;
    const float *wq = vec_f32(qw, 128, &t0), *wk = vec_f32(kw, 128, &t1);
    void *qd = op_dev(q), *kd = op_dev(k);
    if (wq && wk && qd && kd) {
        iris_count_launch(2);
        op_check(iris_launch_head_rmsnorm_rope(qd, heads * 128, seq, heads, wq, eps, NULL, NULL,
                                                      g_rt.stream),
                        "qk_norm");
        op_check(iris_launch_head_rmsnorm_rope(kd, heads * 128, seq, heads, wk, eps, NULL, NULL,
                                                      g_rt.stream),
                        "qk_norm");
    } else if (!wq || !wk) {
        OP_FAIL("qk_rms_norm_bf16: missing norm weights");
    }
    op_scratch_put(t0, 512);
    op_scratch_put(t1, 512);
}

int iris_gpu_head_rms_norm_bf16(iris_gpu_tensor_t x, iris_gpu_tensor_t w, int seq, int heads, int head_dim,
                                float eps) {
    if (!x || !x->bf16 || head_dim != 128) return OP_FAIL("head_rms_norm_bf16: needs bf16 x, head_dim 128"), 0;
    void *t0;
    const float *wf = vec_f32(w, 128, &t0);
    void *xd = op_dev(x);
    int ok = wf && xd;
    if (ok) {
        iris_count_launch(1);
        ok = op_check(iris_launch_head_rmsnorm_rope(xd, heads * 128, seq, heads, wf, eps, NULL, NULL,
                                                           g_rt.stream),
                             "head_rms_norm") == 0;
    }
    op_scratch_put(t0, 512);
    return ok;
}

/* rows [r0, r0 + rows) of a [*, heads * hd] tensor rotated by a host table
 * [rows, hd] (cached by address) */
static int rope_rows(iris_gpu_tensor_t x, int r0, int rows, int heads, int hd, const float *cs, const float *sn) {
    if (rows <= 0) return 1;
    if (!cs || !sn) return OP_FAIL("rope: missing table"), 0;
    const float *dc = op_table(cs, (size_t)rows * hd), *ds = op_table(sn, (size_t)rows * hd);
    char *xd = (char *)op_dev(x);
    if (!dc || !ds || !xd) return 0;
    const size_t esz = x->bf16 ? 2 : 4;
    iris_count_launch(1);
    return op_check(iris_launch_rope_pairs(xd + (size_t)r0 * heads * hd * esz, x->bf16, rows, heads, hd, dc,
                                                  ds, hd, g_rt.stream),
                           "rope") == 0;
}

static int rope_check(iris_gpu_tensor_t x, int seq, int heads, int hd) {
    if (!x || seq < 0 || heads <= 0 || hd <= 0 || (hd & 1) || x->n < (size_t)seq * heads * hd)
        return OP_FAIL("rope: bad tensor or shape (seq %d, heads %d, head_dim %d)", seq, heads, hd), 0;
    return 1;
}

void iris_gpu_rope_unified_bf16(iris_gpu_tensor_t q, iris_gpu_tensor_t k, const float *txt_cos,
                                const float *txt_sin, const float *img_cos, const float *img_sin,
                                const float *img_cos_k, const float *img_sin_k, int seq,
                                int img_offset, int heads, int head_dim, int axis_dim) {
    (void)axis_dim; /* the tables carry all axes side by side */
    if (!rope_check(q, seq, heads, head_dim) || !rope_check(k, seq, heads, head_dim)) return;
    if (img_offset < 0 || img_offset > seq) {
        OP_FAIL("rope_unified: img_offset %d outside [0, %d]", img_offset, seq);
        return;
    }
    const int n_img = seq - img_offset;
    rope_rows(q, 0, img_offset, heads, head_dim, txt_cos, txt_sin);
    rope_rows(q, img_offset, n_img, heads, head_dim, img_cos, img_sin);
    rope_rows(k, 0, img_offset, heads, head_dim, txt_cos, txt_sin);
    rope_rows(k, img_offset, n_img, heads, head_dim, img_cos_k ? img_cos_k : img_cos,
              img_sin_k ? img_sin_k : img_sin);
}

void iris_gpu_rope_2d_bf16(iris_gpu_tensor_t x, const float *cos_freq, const float *sin_freq,
                           int seq, int heads, int head_dim, int axis_dim) {
    (void)axis_dim;
    if (!rope_check(x, seq, heads, head_dim)) return;
    rope_rows(x, 0, seq, heads, head_dim, cos_freq, sin_freq);
}

/* ------------------------------------------------------------------ attention */
static float g_bias = 0.0f;
static int g_bias_start = 0;

void iris_metal_set_attention_bias(int ref_start, float bias) {
    g_bias_start = ref_start;
    g_bias = bias;
}
float op_attention_bias(void) { return g_bias; }

int iris_gpu_attention_fused_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                  iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads,
                                  int head_dim, float scale) {
    if (!out || !Q || !K || !V || head_dim != 128 || !(out->bf16 && Q->bf16 && K->bf16 && V->bf16))
        return OP_FAIL("attention_fused_bf16: needs bf16 tensors with head_dim 128"), 0;
    if (g_bias != 0.0f)
        return OP_FAIL("attention: the reference-token key bias (SREF strength, from key %d) is not supported "
                       "by this backend",
                       g_bias_start),
               0;
    const int ld = num_heads * 128;
    if (Q->n < (size_t)seq_q * ld || K->n < (size_t)seq_k * ld || V->n < (size_t)seq_k * ld ||
        out->n < (size_t)seq_q * ld)
        return OP_FAIL("attention_fused_bf16: tensors smaller than the shape"), 0;
    const void *q = op_dev(Q), *k = op_dev(K), *v = op_dev(V);
    void *o = op_dev(out);
    if (!q || !k || !v || !o) return 0;
    iris_count_launch(1);
    return op_check(iris_launch_attention(q, ld, k, v, ld, o, ld, seq_q, seq_k, num_heads, scale, NULL,
                                                 g_rt.stream),
                           "attention") == 0;
}

/* the other names of the bf16 attention in iris_metal.h (:291, :415) */
int iris_gpu_attention_bf16_native(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                   iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim,
                                   float scale) {
    return iris_gpu_attention_fused_bf16(out, Q, K, V, seq_q, seq_k, num_heads, head_dim, scale);
}
int iris_gpu_attention_mps_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t Q, iris_gpu_tensor_t K,
                                iris_gpu_tensor_t V, int seq_q, int seq_k, int num_heads, int head_dim, float scale) {
    return iris_gpu_attention_fused_bf16(out, Q, K, V, seq_q, seq_k, num_heads, head_dim, scale);
}

/* ------------------------------------------------------------------ bf16 elementwise */
void iris_gpu_silu_mul_bf16(iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int n) {
    if (!gate || !up || !gate->bf16 || !up->bf16 || gate->n < (size_t)n || up->n < (size_t)n) {
        OP_FAIL("silu_mul_bf16: needs bf16 tensors of %d elements", n);
        return;
    }
    void *g = op_dev(gate), *u = op_dev(up);
    if (!g || !u) return;
    iris_count_launch(1);
    op_check(iris_launch_silu_mul_bf16(g, u, n, g_rt.stream), "silu_mul");
}

void iris_gpu_gated_add_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t gate, iris_gpu_tensor_t proj,
                             int seq, int hidden) {
    const size_t n = (size_t)seq * hidden;
    if (!out || !gate || !proj || !out->bf16 || !gate->bf16 || !proj->bf16 || out->n < n || proj->n < n ||
        gate->n < (size_t)hidden) {
        OP_FAIL("gated_add_bf16: needs bf16 tensors of [%d, %d]", seq, hidden);
        return;
    }
    void *o = op_dev(out), *g = op_dev(gate), *p = op_dev(proj);
    if (!o || !g || !p) return;
    iris_count_launch(1);
    op_check(iris_launch_gated_add_bf16(o, g, p, seq, hidden, g_rt.stream), "gated_add");
}

void iris_gpu_add_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b, int n) {
    if (!out || !a || !b || !out->bf16 || !a->bf16 || !b->bf16 || out->n < (size_t)n || a->n < (size_t)n ||
        b->n < (size_t)n) {
        OP_FAIL("add_bf16: needs bf16 tensors of %d elements", n);
        return;
    }
    void *o = op_dev(out), *x = op_dev(a), *y = op_dev(b);
    if (!o || !x || !y) return;
    iris_count_launch(1);
    op_check(iris_launch_add_bf16(o, x, y, n, g_rt.stream), "add_bf16");
}

/* ------------------------------------------------------------------ layout copies */
static int copy2d(iris_gpu_tensor_t dst, size_t dst_off, int ldd, iris_gpu_tensor_t src, size_t src_off, int lds,
                  int rows, int cols) {
    if (rows <= 0 || cols <= 0) return 1;
    const size_t esz = src->bf16 ? 2 : 4;
    if (dst->bf16 != src->bf16) return OP_FAIL("copy: element types differ"), 0;
    if (dst_off + (size_t)(rows - 1) * ldd + cols > dst->n || src_off + (size_t)(rows - 1) * lds + cols > src->n)
        return OP_FAIL("copy: region outside the tensors"), 0;
    char *d = (char *)op_dev(dst);
    const char *s = (const char *)op_dev(src);
    if (!d || !s) return 0;
    return op_check(cudaMemcpy2DAsync(d + dst_off * esz, (size_t)ldd * esz, s + src_off * esz,
                                             (size_t)lds * esz, (size_t)cols * esz, (size_t)rows,
                                             cudaMemcpyDeviceToDevice, g_rt.stream),
                           "copy") == 0;
}

static int split_fused(iris_gpu_tensor_t fused, iris_gpu_tensor_t q, iris_gpu_tensor_t k, iris_gpu_tensor_t v,
                       iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int seq, int hidden, int mlp) {
    if (!fused) return OP_FAIL("split_qkv_mlp: null fused tensor"), 0;
    const int ld = 3 * hidden + 2 * mlp;
    iris_gpu_tensor_t dst[5] = {q, k, v, gate, up};
    const int width[5] = {hidden, hidden, hidden, mlp, mlp};
    int col = 0;
    for (int i = 0; i < 5; i++) {
        if (width[i] > 0) {
            if (!dst[i]) return OP_FAIL("split_qkv_mlp: null output %d", i), 0;
            if (!copy2d(dst[i], 0, width[i], fused, (size_t)col, ld, seq, width[i])) return 0;
        }
        col += width[i];
    }
    return 1;
}

static int concat_cols(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp, iris_gpu_tensor_t out, int seq, int hidden,
                       int mlp_hidden) {
    if (!attn || !mlp || !out) return OP_FAIL("concat_attn_mlp: null tensor"), 0;
    const int ld = hidden + mlp_hidden;
    return copy2d(out, 0, ld, attn, 0, hidden, seq, hidden) &&
           copy2d(out, (size_t)hidden, ld, mlp, 0, mlp_hidden, seq, mlp_hidden);
}

void iris_gpu_concat_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t a, iris_gpu_tensor_t b,
                              int seq_a, int seq_b, int hidden) {
    if (!out || !a || !b) {
        OP_FAIL("concat_seq_bf16: null tensor");
        return;
    }
    if (copy2d(out, 0, hidden, a, 0, hidden, seq_a, hidden))
        copy2d(out, (size_t)seq_a * hidden, hidden, b, 0, hidden, seq_b, hidden);
}

void iris_gpu_slice_seq_bf16(iris_gpu_tensor_t out, iris_gpu_tensor_t in, int seq_out, int hidden,
                             int start) {
    if (!out || !in || start < 0) {
        OP_FAIL("slice_seq_bf16: bad arguments");
        return;
    }
    copy2d(out, 0, hidden, in, (size_t)start * hidden, hidden, seq_out, hidden);
}

void iris_gpu_split_qkv_mlp_bf16(iris_gpu_tensor_t fused, iris_gpu_tensor_t q, iris_gpu_tensor_t k,
                                 iris_gpu_tensor_t v, iris_gpu_tensor_t gate, iris_gpu_tensor_t up,
                                 int seq, int hidden, int mlp) {
    split_fused(fused, q, k, v, gate, up, seq, hidden, mlp);
}

void iris_gpu_split_qkv_mlp(iris_gpu_tensor_t fused, iris_gpu_tensor_t q, iris_gpu_tensor_t k, iris_gpu_tensor_t v,
                            iris_gpu_tensor_t gate, iris_gpu_tensor_t up, int seq, int hidden, int mlp) {
    split_fused(fused, q, k, v, gate, up, seq, hidden, mlp);
}

void iris_gpu_concat_attn_mlp_bf16(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp,
                                   iris_gpu_tensor_t out, int seq, int hidden, int mlp_hidden) {
    concat_cols(attn, mlp, out, seq, hidden, mlp_hidden);
}

void iris_gpu_concat_attn_mlp(iris_gpu_tensor_t attn, iris_gpu_tensor_t mlp, iris_gpu_tensor_t out, int seq,
                              int hidden, int mlp_hidden) {
    concat_cols(attn, mlp, out, seq, hidden, mlp_hidden);
}

void iris_gpu_copy_bf16(iris_gpu_tensor_t dst, iris_gpu_tensor_t src, size_t n) {
    if (!dst || !src || !dst->bf16 || !src->bf16) {
        OP_FAIL("copy_bf16: needs bf16 tensors");
        return;
    }
    copy2d(dst, 0, (int)n, src, 0, (int)n, 1, (int)n);
}

void iris_gpu_copy_f32(iris_gpu_tensor_t dst, iris_gpu_tensor_t src, size_t n) {
    if (!dst || !src || dst->bf16 || src->bf16) {
        OP_FAIL("copy_f32: needs f32 tensors");
        return;
    }
    copy2d(dst, 0, (int)n, src, 0, (int)n, 1, (int)n);
}

void iris_gpu_copy_region_f32(iris_gpu_tensor_t dst, size_t dst_offset, iris_gpu_tensor_t src, size_t src_offset,
                              size_t n) {
    if (!dst || !src || dst->bf16 || src->bf16) {
        OP_FAIL("copy_region_f32: needs f32 tensors");
        return;
    }
    copy2d(dst, dst_offset, (int)n, src, src_offset, (int)n, 1, (int)n);
}
