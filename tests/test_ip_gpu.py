"""IP-Adapter on the GPU (iris_cuda_flux_load_ip_adapter*) vs the reference's
own fixture, the numpy oracle (oracle/ip_oracle.py, pinned to the reference on
CPU by tests/test_ip_oracle.py) and the reference's forward and sampler with
the adapter attached (oracle/_ref).

* Perceived embeddings (f32 on the GPU, as in the reference): the fixture's
  goldens for the siglip (f16), csd, hybrid and int8 bundles.
* Forwards / samples: relative L2 <= 1e-2 (north_star's bf16 tolerance) against
  the oracle and the reference; the seeded adapters move the velocity by > 5 %.
* Every model here has 2 heads: the reference's BLAS attention caches its
  thread count from the first model's head count (iris_transformer_flux.c:1773)
  and computes wrong heads for a later model with fewer heads in one process.
"""
import json
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from gpu_util import rel_l2
from oracle import flux_oracle as fo
from oracle import ip_oracle as io
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

TOL = 1e-2
FIX_CFG = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=4,
               joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)
CFG = dict(FIX_CFG, num_single_layers=2)
FIX = {"bundle": ("", "in_siglip"), "bundle_csd": ("_csd", "in_csd"),
       "bundle_hybrid": ("_hybrid", "in_hybrid"), "bundle_int8": ("_int8", "in_siglip")}


def write_fixture(tmp_path):
    g = dict(np.load(os.path.join(GOLDEN, "ip_fixture.npz")))
    for b in FIX:
        os.makedirs(tmp_path / b, exist_ok=True)
        (tmp_path / b / "adapter_meta.json").write_bytes(g[f"{b}:meta"].tobytes())
        (tmp_path / b / "adapter_weights.safetensors").write_bytes(g[f"{b}:weights"].tobytes())
    return g


@pytest.fixture(scope="module")
def fix_model(tmp_path_factory, iris):
    d = str(tmp_path_factory.mktemp("ipfix"))
    mg.make_flux_model(d, FIX_CFG, 5, 0.05, "unit")
    g = write_fixture(tmp_path_factory.mktemp("ipb"))
    return iris.Flux.load(d), g


@pytest.mark.parametrize("bundle", list(FIX))
def test_perceived_embeddings_match_fixture(fix_model, tmp_path, bundle):
    m, _ = fix_model
    g = write_fixture(tmp_path)
    suf, inp = FIX[bundle]
    path = str(tmp_path / bundle)
    feats = g[inp].reshape(-1, g[inp].shape[-1])
    m.load_ip_adapter(path, feats, 1.0)
    a = io.load_bundle(path)
    emb = m.ip_embeds(a["num_image_tokens"])
    gold = g["gold_ip_embeds" + suf].reshape(emb.shape)
    corr = float(np.dot(emb.ravel(), gold.ravel()) / (np.linalg.norm(emb) * np.linalg.norm(gold)))
    assert corr > 0.9999 and np.abs(emb - gold).max() < 1e-3, (corr, np.abs(emb - gold).max())
    assert rel_l2(emb, io.perceive(a, feats)) < 1e-4
    m.unload_ip_adapter()


def _inputs():
    dims = mg.flux_dims(CFG)
    return cases.rng_inputs(107, dims["channels"], 4, 4, 8, dims["text_dim"])


@pytest.fixture(scope="module")
def model(tmp_path_factory, iris):
    d = str(tmp_path_factory.mktemp("ipm"))
    w = mg.make_flux_model(d, CFG, 7, 0.05, "unit")
    m = iris.Flux.load(d)
    yield d, w, m
    m.close()


VARIANTS = [("siglip", "bfloat16", {}), ("csd", "float16", {}), ("hybrid", "bfloat16", {}),
            ("siglip", "int8", {}), ("siglip", "float32", {"style_only": True, "in_norm": False})]


@pytest.mark.parametrize("mode,quant,kw", VARIANTS, ids=lambda v: v if isinstance(v, str) else "")
def test_forward_with_ip_matches_oracle_and_reference(model, tmp_path, mode, quant, kw):
    from oracle.ref_lib import RefFlux
    d, w, m = model
    b = str(tmp_path / "ip")
    mg.make_ip_bundle(b, CFG, mode, tokens=16 if mode == "hybrid" else 8, seed=3, quant=quant, **kw)
    feats = mg.ip_features(mode)
    lat, ctx = _inputs()
    base = m.forward(lat, ctx, 0.7)
    m.load_ip_adapter(b, feats, 0.9)
    v = m.forward(lat, ctx, 0.7)
    v_or = fo.forward(w, CFG, lat, ctx, 0.7, ip=io.ip_context(io.load_bundle(b), feats, 0.9))
    assert rel_l2(v, v_or) < TOL
    assert rel_l2(v_or, base) > 0.05
    ref = pu.ref_lib_or_skip()
    rf = RefFlux(ref, d)
    assert rf.set_ip(b, feats, 0.9) == 0
    assert rel_l2(v, rf.forward(lat, ctx, 0.7)) < TOL
    rf.close()
    # detaching restores the base model bit for bit
    m.unload_ip_adapter()
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.7), base)


def test_replace_and_features_file(model, tmp_path, iris):
    d, w, m = model
    lat, ctx = _inputs()
    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    mg.make_ip_bundle(a, CFG, "siglip", seed=4)
    mg.make_ip_bundle(b, CFG, "csd", seed=5)
    fa, fb = mg.ip_features("siglip", seed=2), mg.ip_features("csd", seed=3)
    m.load_ip_adapter(b, fb, 1.0)
    only_b = m.forward(lat, ctx, 0.5)
    m.load_ip_adapter(a, fa, 1.0)
    m.load_ip_adapter(b, fb, 1.0)   # replaces a
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.5), only_b)
    path = str(tmp_path / "feats.bin")
    fa.tofile(path)                 # the reference's features file: raw f32 rows
    m.load_ip_adapter(a, path, 1.0)
    v_file = m.forward(lat, ctx, 0.5)
    m.load_ip_adapter(a, fa, 1.0)
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.5), v_file)
    # errors leave the attached adapter in place
    other = str(tmp_path / "other")
    mg.make_ip_bundle(other, dict(CFG, num_single_layers=3), "siglip", seed=6)
    for bad in ((other, fa), (str(tmp_path / "missing"), fa)):
        with pytest.raises(iris.IrisCudaError):
            m.load_ip_adapter(bad[0], bad[1], 1.0)
    with pytest.raises(iris.IrisCudaError):
        m.load_ip_adapter(a, str(tmp_path / "nofile.bin"), 1.0)
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.5), v_file)
    with pytest.raises(iris.IrisCudaError):
        m.set_ip_schedule("sometimes:0.5")
    m.unload_ip_adapter()
    with pytest.raises(iris.IrisCudaError):
        m.set_ip_schedule("late:0.5")  # nothing attached


@pytest.mark.parametrize("spec", ["late:0.5", "early:0.4"])
def test_sampler_with_schedule_matches_reference(model, tmp_path, spec):
    """4-step Euler with an injection schedule: the GPU sampler sets the
    per-step multiplier like iris_sample_euler (iris_sample.c:351)."""
    from oracle.ref_lib import RefFlux
    d, w, m = model
    b = str(tmp_path / "ip")
    mg.make_ip_bundle(b, CFG, "siglip", seed=8)
    feats = mg.ip_features("siglip", seed=4)
    _, ctx = _inputs()
    z0 = np.random.default_rng(11).standard_normal((128, 4, 4)).astype(np.float32)
    sched = np.array([1.0, 0.75, 0.5, 0.25, 0.0], np.float32)
    m.load_ip_adapter(b, feats, 1.0)
    m.set_ip_schedule(spec)
    z = m.sample_euler(z0, ctx, sched)
    m.unload_ip_adapter()
    a = io.ip_context(io.load_bundle(b), feats, 1.0)
    assert io.set_schedule(a["adapter"], spec) == 0
    zo = z0.copy()
    for s in range(4):
        io.set_step(a["adapter"], s, 4)
        zo = zo + (sched[s + 1] - sched[s]) * fo.forward(w, CFG, zo, ctx, float(sched[s]), ip=a)
    assert rel_l2(z, zo) < TOL
    ref = pu.ref_lib_or_skip()
    rf = RefFlux(ref, d)
    assert rf.set_ip(b, feats, 1.0) == 0 and rf.set_ip_schedule(spec) == 0
    assert rel_l2(z, rf.sample_euler(z0, ctx, sched)) < TOL
    rf.close()


def test_lora_ip_and_references_together(model, tmp_path):
    """A LoRA folded into the weights, an IP-Adapter on the image rows (target
    and reference tokens, as the reference's img_seq includes them) and two
    reference latents in one forward, against the reference with its hooks and
    the oracle (folded weights + ip_context + refs)."""
    from oracle import lora_oracle as lo
    from oracle.ref_lib import RefFlux
    d, w, m = model
    dims = mg.flux_dims(CFG)
    lp = str(tmp_path / "l.safetensors")
    mg.make_flux_lora(lp, CFG, "bfl", rank=8, seed=9, std=0.15)
    b = str(tmp_path / "ip")
    mg.make_ip_bundle(b, CFG, "siglip", seed=12)
    feats = mg.ip_features("siglip", seed=6)
    lat, ctx = _inputs()
    refs = [np.random.default_rng(30 + i).standard_normal((128, 2, 3)).astype(np.float32) for i in range(2)]
    m.load_lora(lp, 0.7)
    m.load_ip_adapter(b, feats, 1.1)
    v = m.forward(lat, ctx, 0.6, refs=refs)
    m.unload_ip_adapter()
    m.unload_lora()
    L = lo.load_lora(lp, dims["n_double"], dims["n_single"], dims["hidden"])
    v_or = fo.forward(lo.merge(w, L, 0.7), CFG, lat, ctx, 0.6, refs=refs,
                      ip=io.ip_context(io.load_bundle(b), feats, 1.1))
    assert rel_l2(v, v_or) < TOL
    ref = pu.ref_lib_or_skip()
    rf = RefFlux(ref, d)
    assert rf.set_lora(lp, 0.7) and rf.set_ip(b, feats, 1.1) == 0
    assert rel_l2(v, rf.forward_refs(lat, refs, ctx, 0.6)) < TOL
    rf.close()
