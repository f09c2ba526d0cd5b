/*
 * Multi-GPU communication for the CUDA backend: one NCCL communicator per
 * process group (a CFG pair or a tensor-parallel group), created from a
 * unique id that the caller distributes (any out-of-band channel: a
 * torch.distributed store, MPI, a file).  NCCL is loaded with dlopen at first
 * use, so the library has no link-time dependency and shares the NCCL that a
 * host framework has already loaded (same soname).  The reference is
 * single-process and has no counterpart.
 *
 * Collectives run on the library stream.  Communicators are created with a
 * non-blocking config and every wait on them is bounded: a peer that dies or
 * never joins turns into IRIS_CUDA_ERR_TIMEOUT after IRIS_COMM_TIMEOUT_MS
 * (the communicator is then aborted), never into a hang.
 */
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "iris_internal.h"

/* bound on every host wait that depends on peers (env IRIS_COMM_TIMEOUT_MS) */
static int comm_timeout_ms(void) {
    static int ms = 0;
    if (!ms) {
        const char *e = getenv("IRIS_COMM_TIMEOUT_MS");
        ms = (e && atoi(e) > 0) ? atoi(e) : 60000;
    }
    return ms;
}

typedef ncclResult_t (*fn_get_unique_id)(ncclUniqueId *);
typedef ncclResult_t (*fn_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
typedef ncclResult_t (*fn_all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                      cudaStream_t);
typedef ncclResult_t (*fn_all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
typedef ncclResult_t (*fn_comm)(ncclComm_t);
typedef ncclResult_t (*fn_async_error)(ncclComm_t, ncclResult_t *);
typedef const char *(*fn_error_string)(ncclResult_t);

static struct {
    void *so;
    fn_get_unique_id get_unique_id;
    fn_init_rank_config init_rank_config;
    fn_all_reduce all_reduce;
    fn_all_gather all_gather;
    fn_comm destroy, abort_;
    fn_async_error async_error;
    fn_error_string error_string;
} g_nccl;

static struct {
    ncclComm_t comm;
    int world, rank;
} g_comm;

static int nccl_load(void) {
    if (g_nccl.so) return 0;
    const char *names[] = {"libnccl.so.2", "libnccl.so", "/usr/lib/x86_64-linux-gnu/libnccl.so.2"};
    for (size_t i = 0; i < sizeof(names) / sizeof(names[0]) && !g_nccl.so; i++)
        g_nccl.so = dlopen(names[i], RTLD_NOW | RTLD_GLOBAL);
    if (!g_nccl.so) return iris_fail(IRIS_CUDA_ERR_NODEV, "NCCL not found: %s", dlerror());
#define SYM(field, name) \
    if (!(g_nccl.field = (typeof(g_nccl.field))dlsym(g_nccl.so, name))) \
        return iris_fail(IRIS_CUDA_ERR_NODEV, "NCCL symbol %s missing", name)
    SYM(get_unique_id, "ncclGetUniqueId");
    SYM(init_rank_config, "ncclCommInitRankConfig");
    SYM(all_reduce, "ncclAllReduce");
    SYM(all_gather, "ncclAllGather");
    SYM(destroy, "ncclCommDestroy");
    SYM(abort_, "ncclCommAbort");
    SYM(async_error, "ncclCommGetAsyncError");
    SYM(error_string, "ncclGetErrorString");
#undef SYM
    return 0;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

/* Wait (bounded) until a non-blocking NCCL operation on the communicator has
 * left ncclInProgress; aborts the communicator on error or timeout. */
static int comm_wait(const char *what) {
    double t0 = now_ms();
    ncclResult_t st = ncclInProgress;
    while (1) {
        if (g_nccl.async_error(g_comm.comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st != ncclInProgress) break;
        if (now_ms() - t0 > comm_timeout_ms()) {
            g_nccl.abort_(g_comm.comm);
            g_comm.comm = NULL;
            return iris_fail(IRIS_CUDA_ERR_TIMEOUT, "%s: NCCL did not complete within %d ms", what,
                             comm_timeout_ms());
        }
        struct timespec ts = {0, 200000};
        nanosleep(&ts, NULL);
    }
    if (st != ncclSuccess) {
        const char *msg = g_nccl.error_string(st);
        g_nccl.abort_(g_comm.comm);
        g_comm.comm = NULL;
        return iris_fail(IRIS_CUDA_ERR_CUDA, "%s: NCCL error: %s", what, msg);
    }
    return 0;
}

int iris_cuda_comm_unique_id(void *id_out, size_t id_bytes) {
    if (!id_out || id_bytes < sizeof(ncclUniqueId))
        return iris_fail(IRIS_CUDA_ERR_ARG, "unique id buffer must hold %zu bytes", sizeof(ncclUniqueId));
    int rc = nccl_load();
    if (rc) return rc;
    ncclUniqueId id;
    if (g_nccl.get_unique_id(&id) != ncclSuccess) return iris_fail(IRIS_CUDA_ERR_CUDA, "ncclGetUniqueId failed");
    memcpy(id_out, &id, sizeof(id));
    return 0;
}

int iris_cuda_comm_init(const void *id, int world, int rank) {
    if (!id || world < 1 || rank < 0 || rank >= world) return iris_fail(IRIS_CUDA_ERR_ARG, "bad comm arguments");
    int rc = iris_rt_ensure();
    if (rc) return rc;
    if ((rc = nccl_load())) return rc;
    if (iris_fault("comm")) return iris_fail(IRIS_CUDA_ERR_INJECTED, "injected communicator failure");
    if (g_comm.comm) iris_cuda_comm_destroy();
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = g_nccl.init_rank_config(&g_comm.comm, world, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
        return iris_fail(IRIS_CUDA_ERR_CUDA, "ncclCommInitRankConfig: %s", g_nccl.error_string(r));
    g_comm.world = world;
    g_comm.rank = rank;
    return comm_wait("communicator init");
}

static void sym_release(void);

void iris_cuda_comm_destroy(void) {
    if (g_comm.comm && g_nccl.so) iris_comm_sync_stream();
    sym_release();
    if (g_comm.comm && g_nccl.so) {
        /* a collective that never completes (a peer gone) ends in an abort */
        if (iris_comm_sync_stream() == 0 && g_comm.comm) g_nccl.destroy(g_comm.comm);
    }
    memset(&g_comm, 0, sizeof(g_comm));
}

int iris_cuda_comm_world(void) { return iris_comm_world(); }
int iris_cuda_comm_rank(void) { return iris_comm_rank(); }
int iris_comm_world(void) { return g_comm.comm ? g_comm.world : 1; }
int iris_comm_rank(void) { return g_comm.comm ? g_comm.rank : 0; }
int iris_comm_active(void) { return g_comm.comm != NULL; }

/* Wait for the library stream with a bound: collectives wait on peers, so a
 * peer that died would otherwise block the host forever.  On timeout or an
 * NCCL error the communicator is aborted (its kernels then return) and the
 * stream is drained. */
int iris_comm_sync_stream(void) {
    double t0 = now_ms();
    while (1) {
        cudaError_t e = cudaStreamQuery(g_rt.stream);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) return iris_cuda_check(e, "stream query");
        if (g_comm.comm) {
            ncclResult_t st;
            if (g_nccl.async_error(g_comm.comm, &st) != ncclSuccess ||
                (st != ncclSuccess && st != ncclInProgress)) {
                g_nccl.abort_(g_comm.comm);
                g_comm.comm = NULL;
                cudaStreamSynchronize(g_rt.stream);
                return iris_fail(IRIS_CUDA_ERR_CUDA, "NCCL error while waiting for the stream");
            }
        }
        if (now_ms() - t0 > comm_timeout_ms()) {
            if (g_comm.comm) {
                g_nccl.abort_(g_comm.comm);
                g_comm.comm = NULL;
                cudaStreamSynchronize(g_rt.stream);
            }
            return iris_fail(IRIS_CUDA_ERR_TIMEOUT, "stream did not drain within %d ms (communicator aborted)",
                             comm_timeout_ms());
        }
        struct timespec ts = {0, 50000};
        nanosleep(&ts, NULL);
    }
}

/* in-place sum all-reduce of n bf16 (bf16 != 0) or f32 elements on the library stream */
int iris_comm_allreduce_sum(void *buf, size_t n, int bf16) {
    if (!g_comm.comm) return iris_fail(IRIS_CUDA_ERR_ARG, "no communicator");
    ncclResult_t r = g_nccl.all_reduce(buf, buf, n, bf16 ? ncclBfloat16 : ncclFloat32, ncclSum, g_comm.comm,
                                       g_rt.stream);
    if (r != ncclSuccess && r != ncclInProgress) return iris_fail(IRIS_CUDA_ERR_CUDA, "allreduce: %s", g_nccl.error_string(r));
    return r == ncclInProgress ? comm_wait("allreduce enqueue") : 0;
}

/* all-gather n f32 elements per rank into recv [world * n] */
int iris_comm_allgather_f32(const float *send, float *recv, size_t n) {
    if (!g_comm.comm) return iris_fail(IRIS_CUDA_ERR_ARG, "no communicator");
    ncclResult_t r = g_nccl.all_gather(send, recv, n, ncclFloat32, g_comm.comm, g_rt.stream);
    if (r != ncclSuccess && r != ncclInProgress) return iris_fail(IRIS_CUDA_ERR_CUDA, "allgather: %s", g_nccl.error_string(r));
    return r == ncclInProgress ? comm_wait("allgather enqueue") : 0;
}

/* ------------------------------------------------------------------ symmetric memory
 * One device arena per rank, mapped into every peer process (CUDA IPC over
 * NVLink), bump-allocated in the same order on every rank so that an object
 * has the same offset everywhere: a kernel reaches the peer's copy of an
 * object by adding the offset to the peer's arena base.  The handles are
 * exchanged with one NCCL all-gather, so no host channel is needed beyond
 * the communicator's. */
static struct {
    char *local;
    size_t bytes, used;
    char *peer[IRIS_COMM_MAX_PEERS];
} g_sym;

static void sym_release(void) {
    for (int p = 0; p < IRIS_COMM_MAX_PEERS; p++) {
        if (g_sym.peer[p] && g_sym.peer[p] != g_sym.local) cudaIpcCloseMemHandle(g_sym.peer[p]);
        g_sym.peer[p] = NULL;
    }
    if (g_sym.local) cudaFree(g_sym.local);
    memset(&g_sym, 0, sizeof(g_sym));
}

int iris_comm_sym_init(size_t bytes) {
    if (!g_comm.comm) return iris_fail(IRIS_CUDA_ERR_ARG, "no communicator");
    if (g_comm.world > IRIS_COMM_MAX_PEERS) return iris_fail(IRIS_CUDA_ERR_ARG, "at most %d ranks", IRIS_COMM_MAX_PEERS);
    bytes = (bytes + 4095) & ~(size_t)4095;
    if (g_sym.local && g_sym.bytes >= bytes) { g_sym.used = 0; return 0; }
    int rc = iris_comm_sync_stream();
    if (rc) return rc;
    sym_release();
    if ((rc = iris_cuda_check(cudaMalloc((void **)&g_sym.local, bytes), "symmetric arena"))) return rc;
    g_sym.bytes = bytes;
    if ((rc = iris_cuda_check(cudaMemsetAsync(g_sym.local, 0, bytes, g_rt.stream), "symmetric arena"))) return rc;
    cudaIpcMemHandle_t h;
    if ((rc = iris_cuda_check(cudaIpcGetMemHandle(&h, g_sym.local), "ipc handle"))) return rc;
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t *d = NULL;
    uint8_t all[IRIS_COMM_MAX_PEERS * sizeof(cudaIpcMemHandle_t)];
    if ((rc = iris_cuda_check(cudaMalloc((void **)&d, hb * g_comm.world), "handle exchange"))) return rc;
    rc = iris_h2d(d + hb * g_comm.rank, &h, hb);
    if (!rc) {
        ncclResult_t r = g_nccl.all_gather(d + hb * g_comm.rank, d, hb, ncclUint8, g_comm.comm, g_rt.stream);
        if (r != ncclSuccess && r != ncclInProgress) rc = iris_fail(IRIS_CUDA_ERR_CUDA, "handle all-gather: %s", g_nccl.error_string(r));
        else if (r == ncclInProgress) rc = comm_wait("handle all-gather");
    }
    if (!rc) rc = iris_comm_sync_stream();
    if (!rc) rc = iris_cuda_check(cudaMemcpy(all, d, hb * g_comm.world, cudaMemcpyDeviceToHost), "handle exchange");
    cudaFree(d);
    for (int p = 0; !rc && p < g_comm.world; p++) {
        if (p == g_comm.rank) { g_sym.peer[p] = g_sym.local; continue; }
        cudaIpcMemHandle_t ph;
        memcpy(&ph, all + hb * p, hb);
        rc = iris_cuda_check(cudaIpcOpenMemHandle((void **)&g_sym.peer[p], ph, cudaIpcMemLazyEnablePeerAccess),
                             "open peer arena");
    }
    if (rc) sym_release();
    return rc;
}

void *iris_comm_sym_alloc(size_t bytes) {
    size_t off = (g_sym.used + 255) & ~(size_t)255;
    if (!g_sym.local || off + bytes > g_sym.bytes) {
        iris_fail(IRIS_CUDA_ERR_OOM, "symmetric arena exhausted (%zu + %zu > %zu)", off, bytes, g_sym.bytes);
        return NULL;
    }
    g_sym.used = off + bytes;
    return g_sym.local + off;
}

void *iris_comm_sym_peer(const void *local_ptr, int peer) {
    if (!g_sym.local || peer < 0 || peer >= IRIS_COMM_MAX_PEERS || !g_sym.peer[peer]) return NULL;
    return g_sym.peer[peer] + ((const char *)local_ptr - g_sym.local);
}

int iris_comm_allgather_bytes(const void *send, void *recv, size_t bytes) {
    if (!g_comm.comm) return iris_fail(IRIS_CUDA_ERR_ARG, "no communicator");
    ncclResult_t r = g_nccl.all_gather(send, recv, bytes, ncclUint8, g_comm.comm, g_rt.stream);
    if (r != ncclSuccess && r != ncclInProgress) return iris_fail(IRIS_CUDA_ERR_CUDA, "allgather: %s", g_nccl.error_string(r));
    return r == ncclInProgress ? comm_wait("allgather enqueue") : 0;
}

