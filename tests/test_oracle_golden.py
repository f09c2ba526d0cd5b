"""Pin the CPU oracle (oracle/*.py) to the reference's own outputs.

tests/golden/*.npz were produced by the reference C code compiled from its
own sources (tests/golden/make_golden.py).  These tests check that the
numpy restatement reproduces them; the CUDA tests then compare against the
same fixtures and against this oracle.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import flux_oracle as fo
from oracle import model_gen as mg
from oracle import sample_oracle as so
import cases

FLUX_NAMES = list(cases.FLUX_CASES)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.fixture(scope="module", params=FLUX_NAMES)
def flux_case(request):
    name = request.param
    spec = cases.FLUX_CASES[name]
    g = load(name)
    meta = json.loads(bytes(g["meta"]).decode())
    assert meta["cfg"] == spec["cfg"]
    w = mg.flux_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    return name, spec, g, w, dims, lat, ctx


def test_forward_matches_reference(flux_case):
    name, spec, g, w, dims, lat, ctx = flux_case
    for t in (1.0, 0.7):
        v = fo.forward(w, spec["cfg"], lat, ctx, t)
        assert fo.rel_l2(v, g[f"v_t{t}"]) < 1e-4, (name, t)


def test_temb_and_modulations(flux_case):
    name, spec, g, w, dims, lat, ctx = flux_case
    te = fo.time_embed(w, 0.7)
    assert fo.rel_l2(te, g["t_emb"]) < 1e-4  # f32 sin/cos of angles up to 1000 rad
    mods = fo.modulations(w, g["t_emb"])
    for k in ("dbl_img", "dbl_txt", "single", "final"):
        assert fo.rel_l2(mods[k], g[f"mod_{k}"]) < 1e-5, k


def test_blocks_match_reference(flux_case):
    name, spec, g, w, dims, lat, ctx = flux_case
    h, wd = spec["img"]
    img_h, txt_h = cases.block_inputs(spec, dims["hidden"])
    rope_i = fo.rope_img(h, wd, dims["theta"])
    rope_t = fo.rope_txt(spec["txt"], dims["theta"])
    oi, ot = fo.double_block(w, 0, img_h, txt_h, g["mod_dbl_img"], g["mod_dbl_txt"], rope_i, rope_t, dims)
    # the block delta (output - input) is the meaningful part; check both
    assert fo.rel_l2(oi, g["dbl_out_img"]) < 1e-5
    assert fo.rel_l2(ot, g["dbl_out_txt"]) < 1e-5
    assert fo.rel_l2(oi - img_h, g["dbl_out_img"] - img_h) < 1e-4
    hid = np.concatenate([txt_h, img_h])
    rope_all = (np.concatenate([rope_t[0], rope_i[0]]), np.concatenate([rope_t[1], rope_i[1]]))
    so_ = fo.single_block(w, 0, hid, g["mod_single"], rope_all, dims)
    assert fo.rel_l2(so_, g["sgl_out"]) < 1e-5
    assert fo.rel_l2(so_ - hid, g["sgl_out"] - hid) < 1e-4


def test_euler_sampler_matches_reference(flux_case):
    name, spec, g, w, dims, lat, ctx = flux_case
    h, wd = spec["img"]
    sched = so.official_schedule(4, h * wd)
    np.testing.assert_allclose(sched, g["sched4"], rtol=1e-6, atol=1e-7)
    z = so.sample_euler(lambda z, t: fo.forward(w, spec["cfg"], z, ctx, t), g["z0"], g["sched4"])
    assert fo.rel_l2(z, g["z4"]) < 1e-4


def test_multi_ref_and_cfg_match_reference():
    spec = cases.FLUX_CASES["flux_tiny"]
    g = load("flux_tiny")
    w = mg.flux_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    refs, ctx_u = cases.ref_inputs(dims["channels"], ctx.shape)
    v = fo.forward(w, spec["cfg"], lat, ctx, 0.6, refs=refs)
    assert fo.rel_l2(v, g["v_refs"]) < 1e-4
    zc = so.sample_euler_cfg(lambda z, t, c: fo.forward(w, spec["cfg"], z, c, t), g["z0"], ctx, ctx_u,
                             4.0, g["sched3"])
    assert fo.rel_l2(zc, g["z_cfg"]) < 1e-4


def test_schedules_and_noise_match_reference():
    g = load("sampler")
    for key in g:
        if key.startswith("official_"):
            _, steps, seq = key.split("_")
            np.testing.assert_allclose(so.official_schedule(int(steps), int(seq)), g[key], atol=1e-6)
    np.testing.assert_allclose(so.zimage_schedule(8), g["zimage_8"], atol=1e-6)
    np.testing.assert_allclose(so.zimage_schedule(9), g["zimage_9"], atol=1e-6)
    np.testing.assert_allclose(so.init_noise(4, 8, 12, 7), g["noise_4x8x12_s7"], atol=1e-6)
    # first 512 values of a [128, 32, 32] latent = channel 0, rows 0..15, each
    # nearest-subsampled from the 112x112 draw
    draw = so.randn(1234, 112 * 56)
    ys, xs = np.meshgrid(np.arange(16) * 112 // 32, np.arange(32) * 112 // 32, indexing="ij")
    np.testing.assert_allclose(draw[(ys * 112 + xs).ravel()], g["noise_128x32x32_s1234_head"], atol=1e-6)


def test_oracle_detects_planted_mistake():
    """A wrong RoPE axis in the oracle must break parity with the reference."""
    spec = cases.FLUX_CASES["flux_tiny"]
    g = load("flux_tiny")
    w = mg.flux_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    orig = fo.rope_img
    try:
        # swap the H and W positions of every image token (transposed geometry)
        fo.rope_img = lambda ph, pw, theta, t_offset=0: fo.rope_table(
            np.full(ph * pw, t_offset), np.tile(np.arange(pw), ph), np.repeat(np.arange(ph), pw),
            np.zeros(ph * pw), theta)
        v = fo.forward(w, spec["cfg"], lat, ctx, 0.7)
    finally:
        fo.rope_img = orig
    assert fo.rel_l2(v, g["v_t0.7"]) > 1e-3


# ---------------------------------------------------------------- Z-Image
from oracle import zimage_oracle as zo  # noqa: E402


@pytest.fixture(scope="module", params=list(cases.ZIMAGE_CASES))
def zimage_case(request):
    name = request.param
    spec = cases.ZIMAGE_CASES[name]
    g = load(name)
    meta = json.loads(bytes(g["meta"]).decode())
    assert meta["cfg"] == spec["cfg"]
    w = mg.zimage_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    lat, cap = cases.zimage_inputs(spec)
    return name, spec, g, w, lat, cap


def test_zimage_forward_matches_reference(zimage_case):
    name, spec, g, w, lat, cap = zimage_case
    for t in (0.3, 0.9):
        v = zo.forward(w, spec["cfg"], lat, cap, t)
        assert fo.rel_l2(v, g[f"v_t{t}"]) < 1e-4, (name, t, fo.rel_l2(v, g[f"v_t{t}"]))


def test_zimage_sampler_matches_reference(zimage_case):
    name, spec, g, w, lat, cap = zimage_case
    np.testing.assert_allclose(so.zimage_schedule(3), g["sched3"], atol=1e-6)
    z = zo.sample_euler(w, spec["cfg"], g["z0"], cap, g["sched3"])
    assert fo.rel_l2(z, g["z3"]) < 1e-4


def test_reference_cpu_zimage_inplace_gemm_defect(zimage_case):
    """The reference's own CPU Z-Image output depends on its BLAS backend: the
    attention output projection writes over its own input (zimage.c:716/:796).
    The two unmodified builds disagree with each other and with the alias-safe
    build, which is the one the oracle (and the CUDA path) follow."""
    name, spec, g, w, lat, cap = zimage_case
    a, b, fixed = g["v_t0.3_unfixed_generic"], g["v_t0.3_unfixed_blas"], g["v_t0.3"]
    assert fo.rel_l2(a, b) > 1e-2
    assert fo.rel_l2(a, fixed) > 1e-2 and fo.rel_l2(b, fixed) > 1e-2
