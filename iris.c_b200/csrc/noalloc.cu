// adaLN (LayerNorm + shift/scale modulation) for callers that cannot allocate
// device memory.
//
// iris_gpu_adaln_norm_bf16 stages its bf16 inputs as f32 in device scratch
// that the library allocates (and grows) with cudaMalloc.  Some callers
// cannot let a library do that: a host application that owns every byte of
// device memory through its own pool allocator, or a latency-critical loop
// that cannot afford the implicit device synchronisation of
// cudaMalloc/cudaFree.
// iris_gpu_adaln_norm_bf16_noalloc computes the same result using only the
// caller's buffers plus one fixed-size array that is part of this library's
// image in device memory: it never calls cudaMalloc, cudaFree or any other
// allocating routine.
//
// The scratch array is a file-scope __device__ variable, so every GPU that
// loads this library holds it (kScratchFloats f32, about 16.8 MB) until the
// process exits.  In host code its name is only a host-side stand-in: the
// device address is obtained once per device with cudaGetSymbolAddress, with
// that device current, on the first call made on that device.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "iris_kernels.h"

extern "C" int iris_fail(int code, const char* fmt, ...);
extern "C" void iris_note_launches(uint64_t n);

#define IRIS_CUDA_OK 0
#define IRIS_CUDA_ERR_ARG -1
#define IRIS_CUDA_ERR_CUDA -3

namespace {

// Largest x staged per call: 4 Mi f32 elements (seq * hidden), e.g. 1365 rows
// at hidden 3072 or 1024 rows at hidden 4096; hidden itself is at most 8192.
constexpr size_t kMaxX = size_t(4) << 20;
constexpr int kMaxHidden = 8192;
constexpr size_t kScratchFloats = kMaxX + 2 * size_t(kMaxHidden);

static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
// Device address of g_noalloc_scratch, per device ordinal.  Atomic so that first
// calls on one device from two threads both store the same value without a data
// race.  The address belongs to the device's primary context: a process that
// calls cudaDeviceReset, or runs this entry point under a non-primary context, is
// not supported (the cached address would be stale there).
std::atomic<float*> g_scratch_addr[kMaxDevices];

}  // namespace

// out[r, :] = (1 + scale) * LayerNorm(x[r, :]) + shift, eps inside the sqrt,
// for r < seq; x, shift, scale and out are bf16 device buffers the caller
// owns ([seq, hidden], [hidden], [hidden], [seq, hidden]); work is queued on
// `stream` (a cudaStream_t, 0 = legacy default stream) and not synchronised.
//
// Alignment: `out` must be 8-byte aligned (rows are stored 4 bf16 at a time);
// x, shift and scale 2-byte aligned.  A sub-view of a caller's pool whose
// address breaks this is rejected before anything is queued.
//
// Returns IRIS_CUDA_OK, IRIS_CUDA_ERR_ARG (bad pointer, alignment or shape,
// including seq * hidden > 4 Mi or hidden > 8192) or IRIS_CUDA_ERR_CUDA, with
// the reason in iris_cuda_last_error().
//
// All calls share one scratch array, which keeps the previous call's
// contents; every element a call reads is written by that same call first,
// so nothing needs clearing.  Calls whose GPU work overlaps (on different
// streams, or from several threads) race on the scratch: issue them on one
// stream or order them with events.  The first call on a device looks up the
// scratch address (cudaGetSymbolAddress); make that first call before any
// stream capture begins.
extern "C" int iris_gpu_adaln_norm_bf16_noalloc(void* out, const void* x, const void* shift,
                                                const void* scale, int seq, int hidden, float eps,
                                                void* stream) {
  if (!out || !x || !shift || !scale)
    return iris_fail(IRIS_CUDA_ERR_ARG, "adaln_noalloc: null pointer");
  if ((reinterpret_cast<uintptr_t>(out) & 7) ||
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(shift) |
        reinterpret_cast<uintptr_t>(scale)) & 1))
    return iris_fail(IRIS_CUDA_ERR_ARG,
                     "adaln_noalloc: misaligned pointer (out needs 8-byte, x/shift/scale 2-byte "
                     "alignment)");
  if (seq <= 0 || hidden <= 0 || (hidden & 3))
    return iris_fail(IRIS_CUDA_ERR_ARG, "adaln_noalloc: bad shape seq=%d hidden=%d", seq, hidden);
  if (hidden > kMaxHidden || (size_t)seq * (size_t)hidden > kMaxX)
    return iris_fail(IRIS_CUDA_ERR_ARG,
                     "adaln_noalloc: seq*hidden=%zu (hidden %d) exceeds the fixed scratch "
                     "(seq*hidden <= %zu, hidden <= %d)",
                     (size_t)seq * (size_t)hidden, hidden, kMaxX, kMaxHidden);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return iris_fail(IRIS_CUDA_ERR_CUDA, "adaln_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return iris_fail(IRIS_CUDA_ERR_CUDA, "adaln_noalloc: device %d >= %d supported devices", dev,
                     kMaxDevices);
  float* xf = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!xf) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return iris_fail(IRIS_CUDA_ERR_CUDA, "adaln_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    xf = static_cast<float*>(p);
    g_scratch_addr[dev].store(xf, std::memory_order_release);
  }
  float* sh = xf + kMaxX;
  float* sc = sh + kMaxHidden;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  long n = (long)seq * hidden;
  if ((e = iris_launch_bf16_to_f32(x, xf, n, st)) != cudaSuccess ||
      (e = iris_launch_bf16_to_f32(shift, sh, hidden, st)) != cudaSuccess ||
      (e = iris_launch_bf16_to_f32(scale, sc, hidden, st)) != cudaSuccess ||
      (e = iris_launch_adaln(xf, hidden, out, hidden, seq, hidden, sh, sc, nullptr, nullptr, seq, eps,
                             st)) != cudaSuccess)
    return iris_fail(IRIS_CUDA_ERR_CUDA, "adaln_noalloc: launch: %s", cudaGetErrorString(e));
  iris_note_launches(4);
  return IRIS_CUDA_OK;
}
