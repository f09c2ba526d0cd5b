"""Failure reporting that needs no GPU.

* Every op of the iris_gpu_* surface that rejects its arguments records why
  (iris_cuda_last_error) and counts the failure (iris_gpu_op_failures); the
  void ops of iris_metal.h have no return value to carry it.
* The host-side fault injector IRIS_CUDA_FAULT=kind@N fails exactly the N-th
  operation of that kind, before anything is queued (runtime.c, iris_fault):
  checked in a child process, since the variable is read once per process.
"""
import os
import subprocess
import sys

import iris_cuda
from conftest import ROOT


def test_ops_report_rejected_arguments():
    lib = iris_cuda.load()
    n0 = lib.iris_gpu_op_failures()
    lib.iris_gpu_adaln_norm_bf16(None, None, None, None, 4, 64, 1e-6)
    assert "adaln_norm_bf16" in iris_cuda.last_error()
    assert lib.iris_gpu_attention_fused_bf16(None, None, None, None, 4, 4, 1, 128, 0.1) == 0
    assert "attention_fused_bf16" in iris_cuda.last_error()
    lib.iris_gpu_gated_add(None, None, None, 1, 4)
    assert "gated_add" in iris_cuda.last_error()
    assert not lib.iris_gpu_tensor_data(None)
    assert lib.iris_gpu_op_failures() - n0 == 4


CHILD = r"""
import ctypes as C, sys
sys.path.insert(0, {lib_dir!r})
import iris_cuda
lib = iris_cuda.load()
lib.iris_dmalloc.restype = C.c_void_p
lib.iris_dmalloc.argtypes = [C.c_size_t]
lib.iris_dfree.argtypes = [C.c_void_p]
out = []
for i in range(4):
    p = lib.iris_dmalloc(64)
    out.append("injected" if (not p and "injected" in iris_cuda.last_error()) else "not-injected")
    if p:
        lib.iris_dfree(p)
print(",".join(out))
"""


def test_fault_injector_fails_exactly_the_nth_call():
    env = dict(os.environ, IRIS_CUDA_FAULT="alloc@3")
    code = CHILD.format(lib_dir=os.path.join(ROOT, "iris.c_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "not-injected,not-injected,injected,not-injected", r.stdout
