/*
 * Runtime layer of the iris CUDA backend: device selection, the library
 * stream, the device status word, error strings and host-side fault
 * injection.  Replaces the runtime parts of the Metal backend
 * (iris_metal_init / iris_metal_available / iris_metal_cleanup,
 * iris_metal.h:23-33; iris_gpu_sync :309).
 */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "iris_internal.h"

iris_rt_t g_rt;

static _Thread_local char t_err[512];

int iris_fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return code;
}

int iris_cuda_check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 0;
    return iris_fail(IRIS_CUDA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

const char *iris_cuda_last_error(void) { return t_err; }

/* IRIS_CUDA_FAULT="kind@N[,kind@N...]" makes the N-th (1-based) operation of
 * that kind fail on the host, before anything is queued on the GPU. */
int iris_fault(const char *kind) {
    static int parsed = 0;
    static struct { char kind[16]; long at; long count; } rules[8];
    static int nrules = 0;
    if (!parsed) {
        parsed = 1;
        const char *env = getenv("IRIS_CUDA_FAULT");
        if (env && *env) {
            char buf[256];
            snprintf(buf, sizeof(buf), "%s", env);
            char *save = NULL;
            for (char *tok = strtok_r(buf, ",", &save); tok && nrules < 8;
                 tok = strtok_r(NULL, ",", &save)) {
                char *at = strchr(tok, '@');
                if (!at) continue;
                *at = 0;
                snprintf(rules[nrules].kind, sizeof(rules[nrules].kind), "%s", tok);
                rules[nrules].at = atol(at + 1);
                rules[nrules].count = 0;
                nrules++;
            }
        }
    }
    for (int i = 0; i < nrules; i++) {
        if (strcmp(rules[i].kind, kind) == 0) {
            rules[i].count++;
            if (rules[i].count == rules[i].at) return 1;
        }
    }
    return 0;
}

int iris_rt_ensure(void) {
    if (g_rt.initialized) return IRIS_CUDA_OK;
    return iris_cuda_init(-1);
}

int iris_cuda_init(int device) {
    if (g_rt.initialized) return IRIS_CUDA_OK;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return iris_fail(IRIS_CUDA_ERR_NODEV, "no CUDA device: %s", cudaGetErrorString(e));
    if (device < 0) {
        e = cudaGetDevice(&device);
        if (e != cudaSuccess) device = 0;
    }
    if ((e = cudaSetDevice(device)) != cudaSuccess) return iris_cuda_check(e, "cudaSetDevice");
    struct cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess)
        return iris_cuda_check(e, "cudaGetDeviceProperties");
    if (prop.major != 10)
        return iris_fail(IRIS_CUDA_ERR_NODEV,
                         "device %d is sm_%d%d; this library is built for sm_100a only", device,
                         prop.major, prop.minor);
    g_rt.device = device;
    g_rt.num_sms = prop.multiProcessorCount;
    g_rt.cc_major = prop.major;
    g_rt.cc_minor = prop.minor;
    if ((e = cudaStreamCreateWithFlags(&g_rt.stream, cudaStreamNonBlocking)) != cudaSuccess)
        return iris_cuda_check(e, "cudaStreamCreate");
    if ((e = cudaMalloc((void **)&g_rt.d_status, sizeof(int))) != cudaSuccess)
        return iris_cuda_check(e, "cudaMalloc(status)");
    cudaMemsetAsync(g_rt.d_status, 0, sizeof(int), g_rt.stream);
    cudaStreamSynchronize(g_rt.stream);
    if ((e = iris_gemm_init()) != cudaSuccess) return iris_cuda_check(e, "gemm init");
    if ((e = iris_attention_tc_init()) != cudaSuccess) return iris_cuda_check(e, "attention init");
    iris_attention_set_status(g_rt.d_status);
    g_rt.initialized = 1;
    return IRIS_CUDA_OK;
}

int iris_cuda_available(void) { return iris_rt_ensure() == IRIS_CUDA_OK; }

void iris_cuda_cleanup(void) {
    if (!g_rt.initialized) return;
    cudaStreamSynchronize(g_rt.stream);
    iris_wsrc_release_staging();
    cudaFree(g_rt.d_status);
    cudaStreamDestroy(g_rt.stream);
    memset(&g_rt, 0, sizeof(g_rt));
}

int iris_cuda_device_status(int clear) {
    if (!g_rt.initialized) return 0;
    int v = 0;
    cudaMemcpy(&v, g_rt.d_status, sizeof(int), cudaMemcpyDeviceToHost);
    if (clear && v) {
        cudaMemsetAsync(g_rt.d_status, 0, sizeof(int), g_rt.stream);
        cudaStreamSynchronize(g_rt.stream);
    }
    return v;
}

int iris_stream_drain(void) {
    return iris_comm_active() ? iris_comm_sync_stream()
                              : iris_cuda_check(cudaStreamSynchronize(g_rt.stream), "cudaStreamSynchronize");
}

/* Host -> device copy ordered on the library stream and complete on return.
 * (A plain cudaMemcpy from pageable memory may return before its DMA lands,
 * and it is not ordered with the library's non-blocking stream, so a kernel
 * queued right after it could read the old contents.) */
int iris_h2d(void *dst, const void *src, size_t bytes) {
    int rc = iris_cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g_rt.stream), "host to device");
    return rc ? rc : iris_stream_drain();
}

int iris_cuda_synchronize(void) {
    if (!g_rt.initialized) return IRIS_CUDA_OK;
    int rc = iris_stream_drain();
    if (rc) return rc;
    int st = iris_cuda_device_status(0);
    if (st) return iris_fail(IRIS_CUDA_ERR_TIMEOUT, "device wait expired (code 0x%x)", st);
    return IRIS_CUDA_OK;
}

void *iris_cuda_stream(void) {
    if (iris_rt_ensure() != IRIS_CUDA_OK) return NULL;
    return (void *)g_rt.stream;
}

uint64_t iris_cuda_kernel_launches(void) { return g_rt.launches; }
/* launch counting for the C++ translation units, which do not include this header's inline */
void iris_note_launches(uint64_t n) { iris_count_launch(n); }

void *iris_dmalloc(size_t bytes) {
    if (iris_fault("alloc")) {
        iris_fail(IRIS_CUDA_ERR_INJECTED, "injected allocation failure (%zu bytes)", bytes);
        return NULL;
    }
    void *p = NULL;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        iris_fail(IRIS_CUDA_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        return NULL;
    }
    return p;
}

void iris_dfree(void *p) {
    if (p) cudaFree(p);
}

uint32_t iris_crc32(const char *s) {
    uint32_t c = 0xFFFFFFFFu;
    for (; *s; s++) {
        c ^= (uint8_t)*s;
        for (int k = 0; k < 8; k++) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
    }
    return ~c;
}

/* Self-test of the device-side failure path (no reference counterpart): one
 * launch of the tensor-parallel adaLN kernel as a one-rank group whose
 * partial-sum flag nothing ever raises.  Its bounded wait (IRIS_WAIT_NS,
 * 2 s of %globaltimer) expires, the kernel records IRIS_DEV_ERR_TP_WAIT in
 * the device status word and returns without touching its rows, and the
 * call returns what iris_cuda_synchronize reports (IRIS_CUDA_ERR_TIMEOUT).
 * The status word is left set for the caller to read and clear
 * (iris_cuda_device_status); the context stays usable. */
int iris_cuda_selftest_wait_timeout(void) {
    int rc = iris_rt_ensure();
    if (rc) return rc;
    const int H = 512;
    float *x = (float *)iris_dmalloc((size_t)2 * H * sizeof(float));
    unsigned *flags = (unsigned *)iris_dmalloc(64 * sizeof(unsigned));
    if (!x || !flags) {
        iris_dfree(x);
        iris_dfree(flags);
        return IRIS_CUDA_ERR_OOM;
    }
    cudaMemsetAsync(x, 0, (size_t)2 * H * sizeof(float), g_rt.stream);
    cudaMemsetAsync(flags, 0, 64 * sizeof(unsigned), g_rt.stream);
    IrisAdalnTpArgs a;
    memset(&a, 0, sizeof(a));
    a.x = x;
    a.recv = x + H;
    a.rows = a.chunk = 1;
    a.H = H;
    a.has_part = 1;
    a.part_index = 1; /* wait for one partial more than the base: never arrives */
    a.eps = 1e-6f;
    a.tp.size = 1;
    a.tp.chunk = 1;
    a.tp.flags[0] = flags;
    a.status = g_rt.d_status;
    iris_count_launch(1);
    rc = iris_cuda_check(iris_launch_adaln_tp(&a, g_rt.stream), "self-test launch");
    if (!rc) rc = iris_cuda_synchronize();
    cudaStreamSynchronize(g_rt.stream);
    iris_dfree(x);
    iris_dfree(flags);
    return rc;
}

/* Capability probes answered for the CUDA backend (iris_metal.h:28, :703, :743). */
int iris_metal_available(void) { return iris_cuda_available(); }
int iris_metal_shaders_available(void) { return iris_cuda_available(); }
int iris_bf16_pipeline_available(void) { return iris_cuda_available(); }
