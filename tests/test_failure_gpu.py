"""Failure detection on one GPU, without faulting it.

* Device side: iris_cuda_selftest_wait_timeout runs the tensor-parallel adaLN
  kernel as a one-rank group whose partial-sum flag nothing raises; its
  bounded wait (2 s of %globaltimer) must expire, the status word must carry
  the wait's code, iris_cuda_synchronize must return IRIS_CUDA_ERR_TIMEOUT,
  and after clearing the status the same process must still compute a
  correct forward.  No trap, no assert, no endless loop.
* Host side: IRIS_CUDA_FAULT fails a model load's 3rd device allocation, a
  forward's upload and the next forward's launch (tests/fault_child.py, a
  fresh process); each returns its error, the failed load leaks no device
  memory, and the next forward matches the reference golden.
The reference has no counterpart: its GPU path has no bounded waits and
falls back to its CPU path on any failure (iris_transformer_flux.c:4007-4014).
"""
import json
import os
import subprocess
import sys
import time

import numpy as np
import pytest

import cases
from conftest import GOLDEN
from gpu_util import rel_l2
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_device_wait_expires_and_library_recovers(iris, tmp_path):
    lib = iris.lib()
    assert lib.iris_cuda_synchronize() == 0
    t0 = time.time()
    rc = lib.iris_cuda_selftest_wait_timeout()
    dt = time.time() - t0
    assert rc == iris.ERR_TIMEOUT, (rc, iris.last_error())
    assert "expired" in iris.last_error()
    assert 1.5 < dt < 30, dt
    assert lib.iris_cuda_device_status(0) == 0x301
    assert lib.iris_cuda_device_status(1) == 0x301
    assert lib.iris_cuda_device_status(0) == 0
    assert lib.iris_cuda_synchronize() == 0
    spec = cases.FLUX_CASES["flux_tiny"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_tiny.npz")))
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, w = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, w, spec["txt"], dims["text_dim"])
    m = iris.Flux.load(str(tmp_path))
    assert rel_l2(m.forward(lat, ctx, 0.7), g["v_t0.7"]) < 1e-2
    m.close()


def test_injected_host_faults_are_returned_and_recovered():
    env = dict(os.environ, IRIS_CUDA_FAULT="alloc@3,h2d@1,launch@1")
    r = subprocess.run([sys.executable, os.path.join(HERE, "fault_child.py")], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert "injected allocation failure" in res["load1"], res
    assert abs(res["leak_mb"]) < 4, res
    assert res["load2"] == "ok"
    assert "injected H2D failure" in str(res["fwd1"]), res
    assert "injected launch failure" in str(res["fwd2"]), res
    assert isinstance(res["fwd3"], float) and res["fwd3"] < 1e-2, res
