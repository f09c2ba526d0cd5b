"""Z-Image (S3-DiT) parity: CUDA backend through the C ABI vs the reference.

Goldens come from the reference's own CPU code with its in-place attention
output GEMM made alias-safe (oracle/alias_safe_matmul.c; the unmodified CPU
path gives backend-dependent results, see tests/test_oracle_golden.py).
Tolerance: relative L2 <= 1e-2 per model output and per sampled latent
(north_star's bf16 bound).  Cases cover image and caption padding (masked
keys) and refiner blocks on both row ranges.
"""
import os

import numpy as np
import pytest

import cases
from conftest import GOLDEN
from gpu_util import rel_l2
from oracle import model_gen as mg
from oracle import zimage_oracle as zo

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module", params=list(cases.ZIMAGE_CASES))
def zmodel(request, tmp_path_factory, iris):
    name = request.param
    spec = cases.ZIMAGE_CASES[name]
    d = str(tmp_path_factory.mktemp(name))
    w = mg.make_zimage_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.ZImage.load(d)
    yield name, spec, m, w
    m.close()


def test_zimage_config_from_model_dir(zmodel):
    name, spec, m, w = zmodel
    c = spec["cfg"]
    assert (m.cfg.dim, m.cfg.n_layers, m.cfg.n_refiner, m.cfg.ffn_dim, m.cfg.t_mid) == \
        (c["dim"], c["n_layers"], c["n_refiner"], c["ffn_dim"], c["t_mid"])
    assert list(m.cfg.axes_dims) == c["axes_dims"]


def test_zimage_forward_matches_reference(zmodel):
    name, spec, m, w = zmodel
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    lat, cap = cases.zimage_inputs(spec)
    for t in (0.3, 0.9):
        v = m.forward(lat, cap, t)
        assert rel_l2(v, g[f"v_t{t}"]) < TOL, (name, t, rel_l2(v, g[f"v_t{t}"]))
        assert rel_l2(v, zo.forward(w, spec["cfg"], lat, cap, t)) < TOL
    np.testing.assert_array_equal(m.forward(lat, cap, 0.3), m.forward(lat, cap, 0.3))


def test_zimage_sampler_matches_reference(zmodel):
    name, spec, m, w = zmodel
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    _, cap = cases.zimage_inputs(spec)
    z = m.sample_euler(g["z0"], cap, g["sched3"])
    assert rel_l2(z, g["z3"]) < TOL
    assert rel_l2(z - g["z0"], g["z3"] - g["z0"]) < 2e-2


def test_zimage_random_init_runs(iris):
    cfg = dict(dim=256, n_heads=2, n_layers=2, n_refiner=1, cap_feat_dim=64, in_channels=16, patch_size=2,
               rope_theta=256.0, axes_dims=[32, 48, 48], ffn_dim=768, adaln_dim=256, t_mid=256)
    m = iris.ZImage.random(iris.ZImageConfig.from_dict(cfg), seed=4, std=0.05, norm_unit=True)
    rng = np.random.default_rng(1)
    v = m.forward(rng.standard_normal((16, 12, 8)).astype(np.float32),
                  rng.standard_normal((33, 64)).astype(np.float32), 0.5)
    assert v.shape == (16, 12, 8) and np.isfinite(v).all() and np.abs(v).max() > 0
    m.close()


def test_zimage_long_sequence_matches_oracle(iris, tmp_path):
    """576 image + 64 caption rows: the CTA-pair GEMM under every Z-Image
    linear with N % 256 == 0."""
    cfg = dict(dim=256, n_heads=2, n_layers=1, n_refiner=1, cap_feat_dim=64, in_channels=16, patch_size=2,
               rope_theta=256.0, axes_dims=[32, 48, 48], ffn_dim=768, adaln_dim=256, t_mid=256)
    w = mg.make_zimage_model(str(tmp_path), cfg, 8, 0.04, "unit")
    m = iris.ZImage.load(str(tmp_path))
    rng = np.random.default_rng(5)
    lat = rng.standard_normal((16, 48, 48)).astype(np.float32)
    cap = rng.standard_normal((60, 64)).astype(np.float32)
    v = m.forward(lat, cap, 0.4)
    assert rel_l2(v, zo.forward(w, cfg, lat, cap, 0.4)) < TOL
    m.close()

