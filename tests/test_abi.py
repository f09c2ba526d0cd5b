"""C-ABI checks that need no GPU.

* libiris_cuda.so loads and exports every function include/iris_cuda.h declares;
* the ctypes binding covers the same set;
* the host-side parts of the sampler API (schedules, seeded noise) are the
  reference's values (tests/golden/sampler.npz);
* without a GPU the library fails loudly (no silent CPU fallback).
"""
import ctypes
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, gpu_available
import iris_cuda

HEADER = os.path.join(ROOT, "include", "iris_cuda.h")


def declared_functions(path=HEADER):
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b((?:iris|zi)\w*)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if not n.endswith("_t")))


def test_library_builds_and_loads():
    assert os.path.exists(iris_cuda.LIB_PATH), "run make -C iris.c_b200 cuda"
    iris_cuda.load()


def test_exports_every_declared_symbol():
    lib = iris_cuda.load()
    decl = declared_functions()
    assert len(decl) > 40
    missing = [n for n in decl if not hasattr(lib, n)]
    assert not missing, missing
    unbound = [n for n in decl if n not in iris_cuda.SIGNATURES]
    assert not unbound, unbound


def test_schedules_match_reference():
    g = dict(np.load(os.path.join(GOLDEN, "sampler.npz")))
    for key in g:
        if key.startswith("official_"):
            _, steps, seq = key.split("_")
            np.testing.assert_allclose(iris_cuda.official_schedule(int(steps), int(seq)), g[key], atol=1e-6)
    np.testing.assert_allclose(iris_cuda.zimage_schedule(8, 4096), g["zimage_8"], atol=1e-6)
    np.testing.assert_allclose(iris_cuda.zimage_schedule(9, 4096), g["zimage_9"], atol=1e-6)


def test_init_noise_matches_reference():
    g = dict(np.load(os.path.join(GOLDEN, "sampler.npz")))
    a = iris_cuda.init_noise(4, 16, 16, 42)
    np.testing.assert_allclose(a, g["noise_4x16x16_s42"], atol=1e-6)
    np.testing.assert_allclose(iris_cuda.init_noise(4, 8, 12, 7), g["noise_4x8x12_s7"], atol=1e-6)
    big = iris_cuda.init_noise(128, 32, 32, 1234)
    np.testing.assert_allclose(big.reshape(-1)[:512], g["noise_128x32x32_s1234_head"], atol=1e-6)
    s = g["noise_128x32x32_s1234_sum"]
    b64 = big.astype(np.float64)
    assert abs(b64.sum() - s[0]) < 1e-2 and abs((b64 ** 2).sum() - s[1]) < 1e-1


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_fails_loudly_without_gpu(tmp_path):
    lib = iris_cuda.load()
    assert lib.iris_cuda_available() == 0
    assert lib.iris_cuda_init(0) == iris_cuda.ERR_NODEV
    assert "device" in iris_cuda.last_error().lower()
    assert not lib.iris_cuda_flux_load(str(tmp_path).encode())
    with pytest.raises(iris_cuda.IrisCudaError):
        iris_cuda.Flux.load(str(tmp_path))


DROPIN = os.path.join(ROOT, "iris.c_b200", "dropin", "_build", "libiris_refdrive.so")


def test_dropin_build_resolves_against_this_library():
    """The reference's transformer / sampler sources, built unmodified with
    -DUSE_METAL (iris.c_b200/dropin), link and load against libiris_cuda.so:
    every iris_metal.h function they import is exported here."""
    if not os.path.exists(DROPIN):
        pytest.skip("drop-in build missing (needs the reference tree at build time)")
    iris_cuda.load()
    ctypes.CDLL(DROPIN, mode=os.RTLD_NOW)  # fails on any unresolved symbol
    if not shutil.which("nm"):
        return
    und = subprocess.run(["nm", "-D", "--undefined-only", DROPIN], capture_output=True, text=True).stdout
    imported = {line.split()[-1] for line in und.splitlines() if re.search(r"\biris_(gpu|metal|bf16)_", line)}
    exported = {line.split()[-1] for line in subprocess.run(["nm", "-D", "--defined-only", iris_cuda.LIB_PATH],
                                                            capture_output=True, text=True).stdout.splitlines()}
    assert len(imported) > 50, sorted(imported)
    assert imported <= exported, sorted(imported - exported)
    for name in ("iris_gpu_linear_bf16_native", "iris_gpu_attention_fused_bf16", "iris_gpu_rope_unified_bf16",
                 "iris_gpu_rms_norm_f32", "iris_gpu_rope_single_pair_f32", "iris_gpu_tensor_data",
                 "iris_metal_warmup_bf16", "iris_metal_set_attention_bias", "iris_metal_rope_cache_begin"):
        assert name in imported, name
