"""The IP-Adapter oracle (oracle/ip_oracle.py) pinned on CPU:

* to the reference's own golden fixture (debug/fixtures/ip_adapter, an export of
  the training-side model checked by debug/test_ip_adapter.c; stored as
  tests/golden/ip_fixture.npz): perceive, get_kv and inject at block 0 for the
  siglip (f16), csd, hybrid and int8 bundles;
* to the reference's C stages (iris_ip_adapter.c through oracle/_ref) on seeded
  bundles, the schedule parser and step gate;
* to the reference forward with an adapter attached (per-block injection from
  the pre-RoPE image Q into the post-block hidden state).
"""
import json
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from oracle import flux_oracle as fo
from oracle import ip_oracle as io
from oracle import model_gen as mg

MODES = {"bundle": ("", "in_siglip"), "bundle_csd": ("_csd", "in_csd"),
         "bundle_hybrid": ("_hybrid", "in_hybrid"), "bundle_int8": ("_int8", "in_siglip")}


def fixture(tmp_path):
    g = dict(np.load(os.path.join(GOLDEN, "ip_fixture.npz")))
    for b in MODES:
        os.makedirs(tmp_path / b, exist_ok=True)
        (tmp_path / b / "adapter_meta.json").write_bytes(g[f"{b}:meta"].tobytes())
        (tmp_path / b / "adapter_weights.safetensors").write_bytes(g[f"{b}:weights"].tobytes())
    return g, json.loads(g["shapes_json"].tobytes())


def close(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    corr = a @ b / (np.linalg.norm(a) * np.linalg.norm(b))
    return corr, np.abs(a - b).max()


@pytest.mark.parametrize("bundle", list(MODES))
def test_fixture_stages(tmp_path, bundle):
    """debug/test_ip_adapter.c: perceive (tolerance 1e-3 there), get_kv from the
    golden embeddings, inject into zeros at block 0 from in_img_q."""
    g, shp = fixture(tmp_path)
    suf, inp = MODES[bundle]
    a = io.load_bundle(str(tmp_path / bundle))
    T, H = a["num_image_tokens"], a["hidden_dim"]
    emb = io.perceive(a, g[inp].reshape(-1, g[inp].shape[-1]))
    c, m = close(emb, g["gold_ip_embeds" + suf])
    assert c > 0.9999 and m < 1e-3, (c, m)
    gold_emb = g["gold_ip_embeds" + suf].reshape(T, H)
    k, v = io.get_kv(a, 0, gold_emb)
    for got, gold in ((k, g["gold_k_ip_b0" + suf]), (v, g["gold_v_ip_b0" + suf])):
        c, m = close(got, gold)
        assert c > 0.9999 and m < 1e-3, (c, m)
    gk, gv = g["gold_k_ip_b0" + suf].reshape(T, H), g["gold_v_ip_b0" + suf].reshape(T, H)
    h = io.inject(a, 0, g["in_img_q"], gk, gv, np.zeros((shp["img_seq"], H), np.float32))
    c, m = close(h, g["gold_inject_b0" + suf])
    assert c > 0.9999 and m < 1e-3, (c, m)


@pytest.mark.parametrize("bundle", list(MODES))
def test_oracle_matches_reference_stages_on_fixture(tmp_path, bundle):
    ref = pu.ref_lib_or_skip()
    g, shp = fixture(tmp_path)
    suf, inp = MODES[bundle]
    path = str(tmp_path / bundle)
    a = io.load_bundle(path)
    T, H = a["num_image_tokens"], a["hidden_dim"]
    feats = g[inp].reshape(-1, g[inp].shape[-1])
    e_ref = ref.ip_perceive(path, feats, T, H)
    assert fo.rel_l2(io.perceive(a, feats), e_ref) < 1e-4  # f32 LayerNorm of the reference vs f64 here
    for blk in (0, a["num_blocks"] - 1):
        k_ref, v_ref = ref.ip_get_kv(path, blk, e_ref)
        k, v = io.get_kv(a, blk, e_ref)
        assert fo.rel_l2(k, k_ref) < 1e-5 and fo.rel_l2(v, v_ref) < 1e-5
        h0 = np.random.default_rng(blk).standard_normal((shp["img_seq"], H)).astype(np.float32)
        h_ref = ref.ip_inject(path, blk, g["in_img_q"], k_ref, v_ref, h0)
        assert fo.rel_l2(io.inject(a, blk, g["in_img_q"], k_ref, v_ref, h0), h_ref) < 1e-5


def test_schedule_matches_reference(tmp_path):
    ref = pu.ref_lib_or_skip()
    g, shp = fixture(tmp_path)
    path = str(tmp_path / "bundle")
    a = io.load_bundle(path)
    T, H = a["num_image_tokens"], a["hidden_dim"]
    k, v = (g["gold_k_ip_b0"].reshape(T, H), g["gold_v_ip_b0"].reshape(T, H))
    h0 = np.zeros((shp["img_seq"], H), np.float32)
    for spec in ("late:0.5", "early:0.5", "none", "late:0"):
        for step in range(4):
            assert io.set_schedule(a, spec) == 0
            io.set_step(a, step, 4)
            h = io.inject(a, 0, g["in_img_q"], k, v, h0)
            np.testing.assert_allclose(h, ref.ip_inject(path, 0, g["in_img_q"], k, v, h0, spec, step, 4),
                                       rtol=1e-5, atol=1e-6)
    for bad in ("late:1.5", "sometimes:0.3", "late:x"):
        assert io.set_schedule(a, bad) == -1 and a["sched"] == (0, 0.0)
        with pytest.raises(RuntimeError):
            ref.ip_inject(path, 0, g["in_img_q"], k, v, h0, bad, 0, 4)


CFG = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=2,
           joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)


@pytest.mark.parametrize("mode,quant", [("siglip", "bfloat16"), ("csd", "float16"), ("hybrid", "bfloat16"),
                                        ("siglip", "int8")])
def test_oracle_forward_with_ip_matches_reference(tmp_path, mode, quant):
    """Reference forward with the adapter attached (its runtime hooks) vs the
    oracle forward with ip_context: within 1e-4, while the adapter moves the
    velocity by more than 5 %."""
    ref = pu.ref_lib_or_skip()
    from oracle.ref_lib import RefFlux
    d = str(tmp_path / "m")
    w = mg.make_flux_model(d, CFG, 7, 0.05, "unit")
    b = str(tmp_path / "ip")
    mg.make_ip_bundle(b, CFG, mode, tokens=8 if mode != "hybrid" else 16, seed=3, quant=quant)
    feats = mg.ip_features(mode)
    dims = mg.flux_dims(CFG)
    lat, ctx = cases.rng_inputs(107, dims["channels"], 4, 4, 8, dims["text_dim"])
    rf = RefFlux(ref, d)
    base = rf.forward(lat, ctx, 0.7)
    assert rf.set_ip(b, feats, 0.9) == 0
    v_ref = rf.forward(lat, ctx, 0.7)
    rf.clear_ip()
    np.testing.assert_array_equal(rf.forward(lat, ctx, 0.7), base)
    rf.close()
    ip = io.ip_context(io.load_bundle(b), feats, 0.9)
    v = fo.forward(w, CFG, lat, ctx, 0.7, ip=ip)
    assert fo.rel_l2(v, v_ref) < 1e-4
    assert fo.rel_l2(v_ref, base) > 0.05
