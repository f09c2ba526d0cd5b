/*
 * Weight sources shared by the model loaders: a tensor of the reference's
 * safetensors layout is written to device memory either from a model file
 * (its bytes uploaded unchanged through a ring of pinned chunks, converted to
 * bf16 on the device when stored as f32 / f16) or from the seeded
 * counter-based device RNG (random-init models), plus the TMA descriptor
 * helper used for every weight and activation operand.
 */
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

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

/* ------------------------------------------------------------ file uploads
 *
 * The reference reads every tensor into host memory, converting to f32 where it
 * computes in f32 (iris_transformer_load_safetensors, iris_transformer_flux.c:5300;
 * shards opened in parallel, :533-556).  Here the tensor's bytes go from the
 * file to the device unchanged: reader threads pread them into pinned chunks
 * of a 4-deep ring while the DMA of earlier chunks is in flight, and f32 / f16
 * tensors are converted to bf16 on the device.  Nothing waits for the device
 * except the reuse of a ring slot. */
#define WS_RING 4
#define WS_CHUNK ((size_t)32 << 20)
#define WS_MAX_THREADS 16

struct iris_cpool {
    pthread_t th[WS_MAX_THREADS];
    int n;
    pthread_mutex_t mu;
    pthread_cond_t cv_job, cv_done;
    int fd;               /* the job: len bytes at file offset foff (or of msrc) -> dst */
    off_t foff;
    const uint8_t *msrc;
    uint8_t *dst;
    size_t len;
    unsigned gen;
    int pending, quit, err;
};

typedef struct {
    struct iris_cpool *pool;
    int idx;
} cpool_arg_t;

/* slice i of n + 1 (the caller reads the last one): [a, b) of the job */
static void cpool_slice(const struct iris_cpool *p, int i, size_t *a, size_t *b) {
    size_t per = (p->len / (size_t)(p->n + 1) + 4095) & ~(size_t)4095;
    *a = per * (size_t)i;
    *b = *a + per;
    if (*a > p->len) *a = p->len;
    if (*b > p->len || i == p->n) *b = p->len;
}

/* pread the whole range (the page cache copies straight into the pinned slot:
 * no page-table work for a mapping, unlike a copy out of the mmap) */
static int read_range(int fd, uint8_t *dst, off_t off, size_t n) {
    while (n) {
        ssize_t r = pread(fd, dst, n, off);
        if (r <= 0) return -1;
        dst += r;
        off += r;
        n -= (size_t)r;
    }
    return 0;
}

static void *cpool_worker(void *arg) {
    cpool_arg_t *a = (cpool_arg_t *)arg;
    struct iris_cpool *p = a->pool;
    const int idx = a->idx;
    free(a);
    unsigned seen = 0;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        while (p->gen == seen && !p->quit) pthread_cond_wait(&p->cv_job, &p->mu);
        if (p->quit) { pthread_mutex_unlock(&p->mu); return NULL; }
        seen = p->gen;
        size_t a, b;
        cpool_slice(p, idx, &a, &b);
        const int fd = p->fd;
        const off_t off = p->foff;
        const uint8_t *msrc = p->msrc;
        uint8_t *dst = p->dst;
        pthread_mutex_unlock(&p->mu);
        int bad = 0;
        if (b > a && msrc) memcpy(dst + a, msrc + a, b - a);
        else if (b > a) bad = read_range(fd, dst + a, off + (off_t)a, b - a);
        pthread_mutex_lock(&p->mu);
        if (bad) p->err = 1;
        if (--p->pending == 0) pthread_cond_signal(&p->cv_done);
        pthread_mutex_unlock(&p->mu);
    }
}

static struct iris_cpool *cpool_new(void) {
    struct iris_cpool *p = (struct iris_cpool *)calloc(1, sizeof(*p));
    if (!p) return NULL;
    pthread_mutex_init(&p->mu, NULL);
    pthread_cond_init(&p->cv_job, NULL);
    pthread_cond_init(&p->cv_done, NULL);
    long cpus = sysconf(_SC_NPROCESSORS_ONLN);
    int want = cpus > 1 ? (int)cpus : 1;
    if (want > WS_MAX_THREADS) want = WS_MAX_THREADS;
    for (int i = 0; i < want - 1; i++) {  /* the caller is the last copier */
        cpool_arg_t *a = (cpool_arg_t *)malloc(sizeof(*a));
        if (!a) break;
        a->pool = p;
        a->idx = p->n;
        if (pthread_create(&p->th[p->n], NULL, cpool_worker, a) != 0) { free(a); break; }
        p->n++;
    }
    return p;
}

/* len bytes of file fd at offset off (msrc == NULL) or of host memory msrc ->
 * dst, split over the pool; 0 or -1 */
static int cpool_run(struct iris_cpool *p, uint8_t *dst, const uint8_t *msrc, int fd, off_t off, size_t len) {
    if (!p || p->n == 0 || len < ((size_t)1 << 20)) {
        if (!msrc) return read_range(fd, dst, off, len);
        memcpy(dst, msrc, len);
        return 0;
    }
    pthread_mutex_lock(&p->mu);
    p->fd = fd;
    p->foff = off;
    p->msrc = msrc;
    p->dst = dst;
    p->len = len;
    p->err = 0;
    p->pending = p->n;
    p->gen++;
    pthread_cond_broadcast(&p->cv_job);
    size_t a, b;
    cpool_slice(p, p->n, &a, &b);
    pthread_mutex_unlock(&p->mu);
    int bad = 0;
    if (b > a && msrc) memcpy(dst + a, msrc + a, b - a);
    else if (b > a) bad = read_range(fd, dst + a, off + (off_t)a, b - a);
    pthread_mutex_lock(&p->mu);
    while (p->pending) pthread_cond_wait(&p->cv_done, &p->mu);
    bad |= p->err;
    pthread_mutex_unlock(&p->mu);
    return bad ? -1 : 0;
}

static void cpool_free(struct iris_cpool *p) {
    if (!p) return;
    pthread_mutex_lock(&p->mu);
    p->quit = 1;
    pthread_cond_broadcast(&p->cv_job);
    pthread_mutex_unlock(&p->mu);
    for (int i = 0; i < p->n; i++) pthread_join(p->th[i], NULL);
    pthread_mutex_destroy(&p->mu);
    pthread_cond_destroy(&p->cv_job);
    pthread_cond_destroy(&p->cv_done);
    free(p);
}

/* The ring and the reader threads live for the process (pinning 128 MB costs
 * tens of milliseconds: a second model load should not pay it again). */
static uint8_t *g_ring[WS_RING];
static cudaEvent_t g_ring_ev[WS_RING];
static struct iris_cpool *g_pool;

void iris_wsrc_free(iris_wsrc_t *ws) {
    if (!ws) return;
    if (ws->ring[0]) cudaStreamSynchronize(g_rt.stream);  /* the ring's last copies are done */
    for (int i = 0; i < WS_RING; i++) {
        ws->ring[i] = NULL;
        ws->ring_ev[i] = NULL;
    }
    ws->pool = NULL;
    iris_dfree(ws->d_raw);
    ws->d_raw = NULL;
    ws->d_raw_n = 0;
}

void iris_wsrc_release_staging(void) {
    for (int i = 0; i < WS_RING; i++) {
        if (g_ring_ev[i]) cudaEventSynchronize(g_ring_ev[i]);
        if (g_ring[i]) cudaFreeHost(g_ring[i]);
        if (g_ring_ev[i]) cudaEventDestroy(g_ring_ev[i]);
        g_ring[i] = NULL;
        g_ring_ev[i] = NULL;
    }
    cpool_free(g_pool);
    g_pool = NULL;
}

static int ring_ensure(void) {
    if (g_ring[0]) return 0;
    for (int i = 0; i < WS_RING; i++) {
        if (cudaMallocHost((void **)&g_ring[i], WS_CHUNK) != cudaSuccess ||
            cudaEventCreateWithFlags(&g_ring_ev[i], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            iris_wsrc_release_staging();
            return iris_fail(IRIS_CUDA_ERR_OOM, "pinned staging ring");
        }
    }
    g_pool = cpool_new();
    return 0;
}

static int ws_ring_init(iris_wsrc_t *ws) {
    if (ws->ring[0]) return 0;
    int rc = ring_ensure();
    if (rc) return rc;
    for (int i = 0; i < WS_RING; i++) {
        ws->ring[i] = g_ring[i];
        ws->ring_ev[i] = g_ring_ev[i];
    }
    ws->pool = g_pool;
    ws->ring_i = 0;
    return 0;
}

/* bytes of device memory d_src -> pageable host memory dst, after the work
 * already queued on the library stream.  Chunks are DMA'd into the pinned ring
 * up to WS_RING ahead while the pool copies earlier chunks out of their slots
 * (and takes the first-touch page faults of a fresh malloc'd dst in parallel);
 * a pageable cudaMemcpy instead stages through the driver's own buffers on one
 * thread.  Returns when dst holds the bytes. */
#define D2H_CHUNK ((size_t)8 << 20)
int iris_d2h_staged(void *dst, const void *d_src, size_t bytes, const char *name) {
    int rc = ring_ensure();
    const size_t nch = (bytes + D2H_CHUNK - 1) / D2H_CHUNK;
    size_t issued = 0;
    for (size_t c = 0; !rc && c < nch; c++) {
        for (; !rc && issued < nch && issued < c + WS_RING; issued++) {
            const int slot = (int)(issued % WS_RING);
            const size_t off = issued * D2H_CHUNK, n = bytes - off < D2H_CHUNK ? bytes - off : D2H_CHUNK;
            rc = iris_cuda_check(cudaEventSynchronize(g_ring_ev[slot]), name);
            if (!rc) rc = iris_cuda_check(cudaMemcpyAsync(g_ring[slot], (const uint8_t *)d_src + off, n,
                                                          cudaMemcpyDeviceToHost, g_rt.stream), name);
            if (!rc) rc = iris_cuda_check(cudaEventRecord(g_ring_ev[slot], g_rt.stream), name);
        }
        if (rc) break;
        const int slot = (int)(c % WS_RING);
        const size_t off = c * D2H_CHUNK, n = bytes - off < D2H_CHUNK ? bytes - off : D2H_CHUNK;
        rc = iris_cuda_check(cudaEventSynchronize(g_ring_ev[slot]), name);
        if (!rc) cpool_run(g_pool, (uint8_t *)dst + off, g_ring[slot], -1, 0, n);
    }
    if (rc) iris_cuda_synchronize();  /* no DMA into a slot outlives the call */
    return rc;
}

/* bytes of a file (fd, offset) -> device, through the ring */
static int ws_upload(iris_wsrc_t *ws, void *d_dst, int fd, off_t src, size_t bytes, const char *name) {
    int rc = ws_ring_init(ws);
    for (size_t off = 0; !rc && off < bytes; off += WS_CHUNK) {
        const size_t n = bytes - off < WS_CHUNK ? bytes - off : WS_CHUNK;
        const int slot = ws->ring_i;
        ws->ring_i = (slot + 1) % WS_RING;
        rc = iris_cuda_check(cudaEventSynchronize(ws->ring_ev[slot]), name);  /* the slot's last DMA is done */
        if (rc) break;
        if (cpool_run(ws->pool, ws->ring[slot], NULL, fd, src + (off_t)off, n)) {
            rc = iris_fail(IRIS_CUDA_ERR_IO, "tensor %s: read failed", name);
            break;
        }
        rc = iris_cuda_check(cudaMemcpyAsync((uint8_t *)d_dst + off, ws->ring[slot], n, cudaMemcpyHostToDevice,
                                             g_rt.stream), name);
        if (!rc) rc = iris_cuda_check(cudaEventRecord(ws->ring_ev[slot], g_rt.stream), name);
    }
    ws->bytes += (double)bytes;
    return rc;
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
    size_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= (size_t)t->shape[i];
    const size_t esz = t->dtype == ST_F32 ? 4 : 2;
    if (n != numel || (t->dtype != ST_F32 && t->dtype != ST_F16 && t->dtype != ST_BF16) || t->nbytes != numel * esz)
        return iris_fail(IRIS_CUDA_ERR_IO, "tensor %s: bad shape or dtype", name);
    const int fd = ws->st.fds[t->file];
    const off_t src = (off_t)(ws->st.data_start[t->file] + t->offset);
    if (t->dtype == ST_BF16) return ws_upload(ws, d_dst, fd, src, t->nbytes, name);
    /* f32 / f16: raw bytes to the device landing, converted there */
    if (ws->d_raw_n < t->nbytes) {
        cudaStreamSynchronize(g_rt.stream);  /* the landing may still be read by a conversion */
        iris_dfree(ws->d_raw);
        ws->d_raw = iris_dmalloc(t->nbytes);
        ws->d_raw_n = ws->d_raw ? t->nbytes : 0;
        if (!ws->d_raw) return iris_fail(IRIS_CUDA_ERR_OOM, "upload landing for %s", name);
    }
    int rc = ws_upload(ws, ws->d_raw, fd, src, t->nbytes, name);
    if (rc) return rc;
    iris_count_launch(1);
    cudaError_t e = t->dtype == ST_F32
                        ? iris_launch_f32_to_bf16((const float *)ws->d_raw, d_dst, (long)numel, g_rt.stream)
                        : iris_launch_f16_to_bf16(ws->d_raw, d_dst, (long)numel, g_rt.stream);
    return iris_cuda_check(e, name);
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

