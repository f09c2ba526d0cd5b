"""The allocation-free adaLN entry point, checked against the allocating one.

iris_gpu_adaln_norm_bf16_noalloc exists for callers that must not let the
library allocate device memory: an application whose pool allocator owns all
device memory, or a loop that cannot take cudaMalloc/cudaFree's implicit
device synchronisation.  It keeps its scratch in one fixed array inside the
library instead.

The buffers below are the test's own (torch); the entry point receives raw
device pointers.  Its output must match iris_gpu_adaln_norm_bf16 on the same
inputs within the op tolerance used by the other tests (relative L2 <= 1e-2)
on two calls in a row, the second larger than the first, and also the CPU
oracle of apply_adaln; device free memory must not move across calls; calls
beyond the fixed scratch, or with misaligned pointers, must be rejected with
a clear error before anything is queued.  This file is named to be collected
last.
"""
import numpy as np
import pytest

from gpu_util import Dev, bf16_round, rel_l2
from oracle import flux_oracle as fo

pytestmark = pytest.mark.gpu


def _inputs(seq, hidden, seed):
    rng = np.random.default_rng(seed)
    x = bf16_round(rng.standard_normal((seq, hidden)) * 3 + 0.5)
    sh = bf16_round(rng.standard_normal(hidden) * 0.1)
    sc = bf16_round(rng.standard_normal(hidden) * 0.1)
    return x, sh, sc


def _allocating(iris, x, sh, sc):
    seq, hidden = x.shape
    X, SH, SC, O = Dev(x), Dev(sh), Dev(sc), Dev(n=seq * hidden)
    iris.lib().iris_gpu_adaln_norm_bf16(O.h, X.h, SH.h, SC.h, seq, hidden, 1e-6)
    return O.read((seq, hidden))


def _device_inputs(x, sh, sc):
    import torch
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    sht = torch.from_numpy(sh).to(dev).to(torch.bfloat16)
    sct = torch.from_numpy(sc).to(dev).to(torch.bfloat16)
    out = torch.full(x.shape, float("nan"), device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize()
    return xt, sht, sct, out


def _call(iris, xt, sht, sct, out):
    import torch
    seq, hidden = xt.shape
    stream = torch.cuda.current_stream(xt.device).cuda_stream
    return iris.lib().iris_gpu_adaln_norm_bf16_noalloc(out.data_ptr(), xt.data_ptr(), sht.data_ptr(),
                                                       sct.data_ptr(), seq, hidden, 1e-6, stream)


def _no_alloc(iris, x, sh, sc):
    import torch
    xt, sht, sct, out = _device_inputs(x, sh, sc)
    rc = _call(iris, xt, sht, sct, out)
    assert rc == 0, iris.last_error()
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def test_no_alloc_adaln_matches_allocating_entry_point(iris):
    for seq, hidden, seed in ((97, 512, 1), (1024, 3072, 2)):
        x, sh, sc = _inputs(seq, hidden, seed)
        got = _no_alloc(iris, x, sh, sc)
        want = _allocating(iris, x, sh, sc)
        assert np.isfinite(got).all()
        assert rel_l2(got, want) < 1e-2, (seq, hidden, rel_l2(got, want))
        assert rel_l2(got, fo.adaln(x, sh, sc)) < 1e-2


def test_no_alloc_adaln_moves_no_device_memory(iris):
    import torch
    x, sh, sc = _inputs(512, 3072, 3)
    xt, sht, sct, out = _device_inputs(x, sh, sc)
    assert _call(iris, xt, sht, sct, out) == 0, iris.last_error()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    n0 = iris.lib().iris_cuda_kernel_launches()
    for _ in range(3):
        assert _call(iris, xt, sht, sct, out) == 0, iris.last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0
    assert iris.lib().iris_cuda_kernel_launches() - n0 == 3 * 4
    assert rel_l2(out.float().cpu().numpy(), fo.adaln(x, sh, sc)) < 1e-2


def test_no_alloc_adaln_rejects_oversize_and_misaligned(iris):
    import torch
    dev = torch.device("cuda", 0)
    buf = torch.zeros(64, device=dev, dtype=torch.bfloat16)
    p = buf.data_ptr()
    rc = iris.lib().iris_gpu_adaln_norm_bf16_noalloc(p, p, p, p, 4097, 1024, 1e-6, 0)
    assert rc == iris.ERR_ARG
    assert "exceeds the fixed scratch" in iris.last_error()
    rc = iris.lib().iris_gpu_adaln_norm_bf16_noalloc(p, p, p, p, 1, 16384, 1e-6, 0)
    assert rc == iris.ERR_ARG
    # an offset view of a caller's pool whose output is not 8-byte aligned
    rc = iris.lib().iris_gpu_adaln_norm_bf16_noalloc(p + 2, p, p, p, 1, 16, 1e-6, 0)
    assert rc == iris.ERR_ARG
    assert "misaligned" in iris.last_error()
    rc = iris.lib().iris_gpu_adaln_norm_bf16_noalloc(p, p + 1, p, p, 1, 16, 1e-6, 0)
    assert rc == iris.ERR_ARG
    torch.cuda.synchronize()
