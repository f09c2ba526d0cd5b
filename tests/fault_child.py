"""Child process of tests/test_failure_gpu.py (run with IRIS_CUDA_FAULT set).

IRIS_CUDA_FAULT=alloc@3,h2d@1,launch@1: the model load fails on its 3rd
device allocation, the first forward on its host-to-device upload and the
second on its launch; each must return its error without leaking device
memory or leaving a half-built plan, and the third forward must be correct.
Prints one JSON line with what it saw.
"""
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "iris.c_b200"), os.path.join(HERE, "golden")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import cases  # noqa: E402
import iris_cuda  # noqa: E402
from oracle import model_gen as mg  # noqa: E402


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def main():
    res = {}
    lib = iris_cuda.lib()
    assert lib.iris_cuda_init(0) == 0, iris_cuda.last_error()
    spec = cases.FLUX_CASES["flux_tiny"]
    g = dict(np.load(os.path.join(HERE, "golden", "flux_tiny.npz")))
    dims = mg.flux_dims(spec["cfg"])
    h, w = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, w, spec["txt"], dims["text_dim"])
    with tempfile.TemporaryDirectory() as d:
        mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(0)[0]
        try:
            iris_cuda.Flux.load(d)
            res["load1"] = "ok"
        except iris_cuda.IrisCudaError as e:
            res["load1"] = str(e)
        torch.cuda.synchronize()
        res["leak_mb"] = (free0 - torch.cuda.mem_get_info(0)[0]) / 2**20
        m = iris_cuda.Flux.load(d)
        res["load2"] = "ok"
        for k in ("fwd1", "fwd2", "fwd3"):
            try:
                v = m.forward(lat, ctx, 0.7)
                res[k] = rel_l2(v, g["v_t0.7"])
            except iris_cuda.IrisCudaError as e:
                res[k] = str(e)
        m.close()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
