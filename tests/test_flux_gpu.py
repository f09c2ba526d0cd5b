"""Flux.2 Klein parity: CUDA backend (through the C ABI) vs the reference.

Each golden case was produced by the reference's own C code on the same
seeded bf16 weights (tests/golden/make_golden.py).  Here the CUDA backend
loads the same safetensors (written by oracle/model_gen.py) with its own
loader and is compared per block, per step velocity and per sampled latent.

Tolerance (north_star): relative L2 <= 1e-2 for every block output and every
velocity; the block DELTA (output - input) is also held to 2e-2, since with
small gates a block is close to the identity and the plain output ratio
would hide errors in the block's own contribution.
"""
import os

import numpy as np
import pytest

import cases
from conftest import GOLDEN
from gpu_util import rel_l2
from oracle import flux_oracle as fo
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

TOL = 1e-2
TOL_DELTA = 2e-2


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.fixture(scope="module", params=list(cases.FLUX_CASES))
def model(request, tmp_path_factory, iris):
    name = request.param
    spec = cases.FLUX_CASES[name]
    d = str(tmp_path_factory.mktemp(name))
    w = mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.Flux.load(d)
    yield name, spec, m, w
    m.close()


def test_loader_reads_reference_layout(model):
    name, spec, m, w = model
    dims = mg.flux_dims(spec["cfg"])
    assert m.cfg.hidden == dims["hidden"] and m.cfg.n_double == dims["n_double"]
    bits = m.read_weight("single_transformer_blocks.0.attn.to_qkv_mlp_proj.weight",
                         w["single_transformer_blocks.0.attn.to_qkv_mlp_proj.weight"].shape)
    np.testing.assert_array_equal(mg.bf16_bits_to_f32(bits),
                                  w["single_transformer_blocks.0.attn.to_qkv_mlp_proj.weight"])


def test_blocks_match_reference(model):
    name, spec, m, w = model
    g = golden(name)
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    img_h, txt_h = cases.block_inputs(spec, dims["hidden"])
    hid = np.concatenate([txt_h, img_h])
    out = m.run_block(0, 0, hid, spec["txt"], h, wd, 0.7)
    ot, oi = out[:spec["txt"]], out[spec["txt"]:]
    assert rel_l2(oi, g["dbl_out_img"]) < TOL
    assert rel_l2(ot, g["dbl_out_txt"]) < TOL
    assert rel_l2(oi - img_h, g["dbl_out_img"] - img_h) < TOL_DELTA
    assert rel_l2(ot - txt_h, g["dbl_out_txt"] - txt_h) < TOL_DELTA
    so = m.run_block(1, 0, hid, spec["txt"], h, wd, 0.7)
    assert rel_l2(so, g["sgl_out"]) < TOL
    assert rel_l2(so - hid, g["sgl_out"] - hid) < TOL_DELTA


def test_velocity_matches_reference(model):
    name, spec, m, w = model
    g = golden(name)
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    for t in (1.0, 0.7):
        v = m.forward(lat, ctx, t)
        assert v.shape == g[f"v_t{t}"].shape
        assert rel_l2(v, g[f"v_t{t}"]) < TOL, (name, t, rel_l2(v, g[f"v_t{t}"]))
        # the oracle agrees with the reference to ~1e-6, so this is the same bar
        assert rel_l2(v, fo.forward(w, spec["cfg"], lat, ctx, t)) < TOL
    # repeated calls on one plan (CUDA graph replay) are deterministic
    v1 = m.forward(lat, ctx, 0.7)
    v2 = m.forward(lat, ctx, 0.7)
    np.testing.assert_array_equal(v1, v2)


def test_euler_sampler_matches_reference(model):
    name, spec, m, w = model
    g = golden(name)
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    z = m.sample_euler(g["z0"], ctx, g["sched4"])
    assert rel_l2(z, g["z4"]) < TOL
    assert rel_l2(z - g["z0"], g["z4"] - g["z0"]) < TOL_DELTA


def test_multi_ref_and_cfg_match_reference(iris, tmp_path):
    spec = cases.FLUX_CASES["flux_tiny"]
    g = golden("flux_tiny")
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.Flux.load(str(tmp_path))
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    refs, ctx_u = cases.ref_inputs(dims["channels"], ctx.shape)
    v = m.forward(lat, ctx, 0.6, refs=refs)
    assert rel_l2(v, g["v_refs"]) < TOL
    zc = m.sample_euler(g["z0"], ctx, g["sched3"], txt_uncond=ctx_u, guidance=4.0)
    assert rel_l2(zc, g["z_cfg"]) < TOL
    # switching back to the plain plan still matches
    assert rel_l2(m.forward(lat, ctx, 0.7), g["v_t0.7"]) < TOL
    m.close()


def test_random_init_model_matches_oracle(iris):
    """Device-side random init + read_weight round trip: the oracle run on the
    weights read back must agree with the CUDA forward."""
    cfg = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=1,
               joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)
    m = iris.Flux.random(iris.FluxConfig.from_hf(cfg), seed=5, std=0.05, norm_unit=True)
    w = {n: mg.bf16_bits_to_f32(m.read_weight(n, shp)) for n, shp, _ in mg.flux_tensor_specs(cfg)}
    norms = w["transformer_blocks.0.attn.norm_q.weight"]
    assert abs(norms.mean() - 1.0) < 0.05
    rng = np.random.default_rng(0)
    lat = rng.standard_normal((128, 3, 5)).astype(np.float32)
    ctx = rng.standard_normal((11, 64)).astype(np.float32)
    v = m.forward(lat, ctx, 0.5)
    assert rel_l2(v, fo.forward(w, cfg, lat, ctx, 0.5)) < TOL
    m.close()


def test_long_sequence_matches_oracle(iris):
    """677 rows (77 text + 600 image): every linear with N % 256 == 0 runs on
    the CTA-pair GEMM with its fused epilogue (QKV norm/RoPE, SwiGLU, gated
    residual, single-block split), with ragged row groups."""
    cfg = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=1,
               joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)
    m = iris.Flux.random(iris.FluxConfig.from_hf(cfg), seed=12, std=0.04, norm_unit=True)
    w = {n: mg.bf16_bits_to_f32(m.read_weight(n, shp)) for n, shp, _ in mg.flux_tensor_specs(cfg)}
    rng = np.random.default_rng(3)
    lat = rng.standard_normal((128, 20, 30)).astype(np.float32)
    ctx = rng.standard_normal((77, 64)).astype(np.float32)
    v = m.forward(lat, ctx, 0.6)
    assert rel_l2(v, fo.forward(w, cfg, lat, ctx, 0.6)) < TOL
    m.close()

