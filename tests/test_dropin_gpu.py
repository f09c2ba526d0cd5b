"""The reference's own transformer code driving this backend, unchanged.

iris.c_b200/dropin/Makefile compiles the unmodified iris_transformer_flux.c,
iris_transformer_zimage.c and iris_sample.c of the reference with -DUSE_METAL
(the switch of its GPU backend) and links them against libiris_cuda.so, which
exports the C surface of iris_metal.h.  These tests load that build and run:

* iris_transformer_forward, whose bf16 GPU branch
  (iris_transformer_flux.c:4000 -> iris_transformer_forward_bf16 :3452, the
  bf16 double / single blocks :2076, :3243) queues every linear, norm, RoPE,
  attention and residual op on this backend, in both of the reference's weight
  modes (resident bf16 and mmap);
* iris_sample_euler (iris_sample.c:313) over that forward;
* zi_transformer_forward, whose GPU branch (iris_transformer_zimage.c:1704 ->
  zi_transformer_forward_gpu :1222) runs the f32 op surface.

Each result is compared with the golden output of the reference's own f32 CPU
path on the same weights (tests/golden), within north_star's bf16 tolerance
(relative L2 <= 1e-2).  The reference falls back to its CPU path when a GPU op
fails, which would also match the goldens; so every test also checks that no op
of this backend reported a failure (iris_gpu_op_failures) and that kernels were
launched.
"""
import ctypes as C
import os

import numpy as np
import pytest

import cases
from conftest import GOLDEN, ROOT
from gpu_util import rel_l2
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

TOL = 1e-2
DRIVE = os.path.join(ROOT, "iris.c_b200", "dropin", "_build", "libiris_refdrive.so")
_fp = C.POINTER(C.c_float)


def _f(a):
    return a.ctypes.data_as(_fp)


@pytest.fixture(scope="module")
def drive(iris):
    if not os.path.exists(DRIVE):
        pytest.skip("drop-in build missing: run `make -C iris.c_b200/dropin` where the reference tree exists")
    L = C.CDLL(DRIVE, mode=os.RTLD_NOW)
    L.drive_flux_load.restype = C.c_void_p
    L.drive_flux_load.argtypes = [C.c_char_p, C.c_int]
    L.drive_flux_free.argtypes = [C.c_void_p]
    L.drive_flux_forward.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int, C.c_float, C.c_int, _fp]
    L.drive_sample_euler.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, _fp, C.c_int, _fp, C.c_int]
    L.drive_zi_load.restype = C.c_void_p
    L.drive_zi_load.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.c_float]
    L.drive_zi_free.argtypes = [C.c_void_p]
    L.drive_zi_forward.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, C.c_float, _fp, C.c_int, C.c_int, _fp]
    iris.lib().iris_gpu_op_failures.restype = C.c_ulong
    assert L.drive_init() == 1, iris.last_error()
    return L


class _Watch:
    """Op failures and kernel launches of this backend across a block of calls."""

    def __init__(self, iris):
        self.L = iris.lib()
        self.iris = iris

    def __enter__(self):
        self.f0 = self.L.iris_gpu_op_failures()
        self.k0 = self.L.iris_cuda_kernel_launches()
        return self

    def __exit__(self, *exc):
        self.failures = self.L.iris_gpu_op_failures() - self.f0
        self.launches = self.L.iris_cuda_kernel_launches() - self.k0
        return False

    def check(self, min_launches):
        assert self.failures == 0, self.iris.last_error()
        assert self.launches >= min_launches, self.launches


@pytest.mark.parametrize("mmap_mode", [0, 1])
@pytest.mark.parametrize("name", ["flux_tiny", "flux_small"])
def test_reference_flux_forward_on_cuda(iris, drive, tmp_path, name, mmap_mode):
    spec = cases.FLUX_CASES[name]
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, w = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, w, spec["txt"], dims["text_dim"])
    tf = drive.drive_flux_load(str(tmp_path).encode(), mmap_mode)
    assert tf
    try:
        for t in (1.0, 0.7):
            out = np.zeros_like(lat)
            with _Watch(iris) as wt:
                assert drive.drive_flux_forward(tf, _f(lat), h, w, _f(ctx), ctx.shape[0], t, dims["channels"],
                                                _f(out)) == 0
            # per block: 2 adaLN + 6 QKV + 4 QK-norm + 4 RoPE + 2 attention + ... well over 10 launches
            wt.check(10 * (dims["n_double"] + dims["n_single"]))
            assert rel_l2(out, g[f"v_t{t}"]) < TOL, (name, mmap_mode, t, rel_l2(out, g[f"v_t{t}"]))
    finally:
        drive.drive_flux_free(tf)


def test_reference_sampler_on_cuda(iris, drive, tmp_path):
    spec = cases.FLUX_CASES["flux_small"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_small.npz")))
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, w = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, w, spec["txt"], dims["text_dim"])
    tf = drive.drive_flux_load(str(tmp_path).encode(), 0)
    assert tf
    try:
        z = np.ascontiguousarray(g["z0"], np.float32).copy()
        sched = np.ascontiguousarray(g["sched4"], np.float32)
        with _Watch(iris) as wt:
            assert drive.drive_sample_euler(tf, _f(z), dims["channels"], h, w, _f(ctx), ctx.shape[0], _f(sched),
                                            len(sched) - 1) == 0
        wt.check(4 * 10 * (dims["n_double"] + dims["n_single"]))
        assert rel_l2(z, g["z4"]) < TOL, rel_l2(z, g["z4"])
    finally:
        drive.drive_flux_free(tf)


@pytest.mark.parametrize("name", list(cases.ZIMAGE_CASES))
def test_reference_zimage_forward_on_cuda(iris, drive, tmp_path, name):
    spec = cases.ZIMAGE_CASES[name]
    cfg = spec["cfg"]
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    mg.make_zimage_model(str(tmp_path), cfg, spec["seed"], spec["std"], spec["norm_mode"])
    lat, cap = cases.zimage_inputs(spec)
    arr = (C.c_int * 10)(cfg["dim"], cfg["dim"] // 128, cfg["n_layers"], cfg["n_refiner"], cfg["cap_feat_dim"],
                         cfg["in_channels"], cfg["patch_size"], *cfg["axes_dims"])
    tf = drive.drive_zi_load(str(tmp_path).encode(), arr, float(cfg["rope_theta"]))
    assert tf
    try:
        for t in (0.3, 0.9):
            out = np.zeros_like(lat)
            with _Watch(iris) as wt:
                assert drive.drive_zi_forward(tf, _f(lat), lat.shape[1], lat.shape[2], t, _f(cap), cap.shape[0],
                                              lat.shape[0], _f(out)) == 0
            wt.check(10 * (cfg["n_layers"] + 2 * cfg["n_refiner"]))
            assert rel_l2(out, g[f"v_t{t}"]) < TOL, (name, t, rel_l2(out, g[f"v_t{t}"]))
    finally:
        drive.drive_zi_free(tf)
