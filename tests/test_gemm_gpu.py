"""tcgen05 GEMM parity through the C ABI (iris_gpu_linear_bf16_native, the
replacement of the reference's iris_linear_nobias_bf16 / MPS bf16 linear).

Reference product: numpy f32 x @ W^T on the same bf16-valued operands.
Tolerance: relative L2 <= 4e-3 (the output is rounded to bf16, 2^-9 per
element, so the expected rel-L2 is ~1-2e-3).
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Dev, bf16_round, rel_l2
from oracle.model_gen import f32_to_bf16_bits

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 64, 128), (7, 128, 128), (128, 64, 256), (128, 128, 256), (129, 192, 384),
    (300, 256, 512), (512, 3072, 3072), (1024, 3072, 9216), (1536, 12288, 3072),
    (80, 7680, 3072), (16, 128, 3072), (1024, 3072, 128),
    # >= 512 rows with N % 256 == 0 run on the CTA-pair kernel (M tiles of
    # 256 rows); ragged row counts leave the odd CTA of the last pair partly
    # or wholly past the end
    (600, 512, 768), (777, 192, 512), (2000, 1024, 2304), (640, 3072, 256),
]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_linear_bf16_native(iris, m, k, n):
    rng = np.random.default_rng(m * 7 + k * 3 + n)
    x = bf16_round(rng.standard_normal((m, k)).astype(np.float32))
    w = bf16_round((rng.standard_normal((n, k)) * 0.05).astype(np.float32))
    wb = f32_to_bf16_bits(w)
    xd = Dev(x)
    out = iris.lib().iris_gpu_linear_bf16_native(xd.h, wb.ctypes.data_as(C.POINTER(C.c_uint16)), m, k, n)
    assert out, iris.last_error()
    y = np.zeros(m * n, np.float32)
    iris.lib().iris_gpu_tensor_read(out, y.ctypes.data_as(C.POINTER(C.c_float)))
    iris.lib().iris_gpu_tensor_free(out)
    ref = x @ w.T  # f32 BLAS on bf16-valued operands
    err = rel_l2(y.reshape(m, n), ref)
    # the weight cache is keyed by host address: forget this test's buffer
    iris.lib().iris_metal_clear_bf16_cache_only()
    assert err < 4e-3, (m, k, n, err)
    assert iris.lib().iris_cuda_device_status(0) == 0


@pytest.mark.parametrize("m,k,n", [(37, 64, 64), (300, 2560, 3840), (5, 128, 200)])
def test_linear_f32_with_bias(iris, m, k, n):
    """iris_gpu_linear (iris_metal.h:239): f32 tensors, f32 host weight and
    bias; N not a multiple of 128 takes the padded-weight path (Z-Image's
    final projection has N = 64).  Operands are rounded to bf16 on the way in,
    so the reference product is taken on the rounded values."""
    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    xd = Dev(x, bf16=False)
    fp = C.POINTER(C.c_float)
    out = iris.lib().iris_gpu_linear(xd.h, w.ctypes.data_as(fp), b.ctypes.data_as(fp), m, k, n)
    assert out, iris.last_error()
    y = np.zeros(m * n, np.float32)
    iris.lib().iris_gpu_tensor_read(out, y.ctypes.data_as(fp))
    iris.lib().iris_gpu_tensor_free(out)
    iris.lib().iris_metal_clear_weight_cache_only()
    ref = bf16_round(x) @ bf16_round(w).T + b
    assert rel_l2(y.reshape(m, n), ref) < 2e-3


def test_linear_rejects_unsupported_shape(iris):
    x = Dev(np.zeros((4, 100), np.float32))
    w = np.zeros(100 * 128, np.uint16)
    out = iris.lib().iris_gpu_linear_bf16_native(x.h, w.ctypes.data_as(C.POINTER(C.c_uint16)), 4, 100, 128)
    assert not out
    assert "unsupported" in iris.last_error()
