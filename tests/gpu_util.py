"""Helpers for GPU tests that drive the iris_gpu_* tensor surface through ctypes."""
import ctypes as C

import numpy as np

import iris_cuda

_fp = C.POINTER(C.c_float)


def bf16_round(x):
    from oracle.model_gen import round_bf16
    return round_bf16(np.asarray(x, np.float32))


class Dev:
    """A device tensor owned by the test (bf16 or f32)."""

    def __init__(self, arr=None, n=None, bf16=True):
        L = iris_cuda.lib()
        if arr is not None:
            a = np.ascontiguousarray(arr, np.float32).reshape(-1)
            self.n = a.size
            if bf16:
                self.h = L.iris_gpu_tensor_create_bf16(a.ctypes.data_as(_fp), a.size)
            else:
                self.h = L.iris_gpu_tensor_create(a.ctypes.data_as(_fp), a.size)
        else:
            self.n = n
            self.h = L.iris_gpu_tensor_alloc_f16(n) if bf16 else L.iris_gpu_tensor_alloc(n)
        assert self.h, iris_cuda.last_error()

    def read(self, shape=None):
        out = np.zeros(self.n, np.float32)
        iris_cuda.lib().iris_gpu_tensor_read(self.h, out.ctypes.data_as(_fp))
        return out.reshape(shape) if shape is not None else out

    def free(self):
        if self.h:
            iris_cuda.lib().iris_gpu_tensor_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
