"""SREF style controls, oracle (oracle/flux_oracle.py: temb_delta, bands,
csd_mod_forward) pinned on CPU to the reference (oracle/_ref):

* the CSD modulation delta on the timestep embedding (iris_set_sref_csd,
  iris.c:487) in a forward and in the CFG sampler, whose unconditional branch
  leaves it out (iris_sample.c:754-758);
* the K-side RoPE band scaling of reference rows in the single blocks
  (iris_transformer_set_sref_bands :5153, band_scale_ref_krope :1272) in a
  multi-reference forward, and "off" for out-of-range values.
"""
import numpy as np
import pytest

import cases
import psnr_util as pu
from oracle import flux_oracle as fo
from oracle import model_gen as mg

CFG = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=2,
           joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    ref = pu.ref_lib_or_skip()
    from oracle.ref_lib import RefFlux
    d = str(tmp_path_factory.mktemp("sref"))
    w = mg.make_flux_model(d, CFG, 7, 0.05, "unit")
    csd_path = d + "/csd_mod.safetensors"
    cm = mg.make_csd_mod(csd_path, 32, 96, 256, seed=4)
    csd = np.random.default_rng(2).standard_normal(32).astype(np.float32)
    csd /= np.linalg.norm(csd)
    rf = RefFlux(ref, d)
    yield dict(w=w, rf=rf, csd_path=csd_path, cm=cm, csd=csd)
    rf.close()


def test_csd_delta_forward(setup):
    s = setup
    lat, ctx = cases.rng_inputs(107, 128, 4, 4, 8, 64)
    base = s["rf"].forward(lat, ctx, 0.7)
    assert s["rf"].set_sref_csd(s["csd_path"], s["csd"], 1.5) == 0
    v_ref = s["rf"].forward(lat, ctx, 0.7)
    delta = 1.5 * fo.csd_mod_forward(s["cm"], s["csd"])
    v = fo.forward(s["w"], CFG, lat, ctx, 0.7, temb_delta=delta)
    assert fo.rel_l2(v, v_ref) < 1e-4 and fo.rel_l2(v_ref, base) > 0.05
    assert s["rf"].set_sref_csd(None, s["csd"], 1.0) == 0  # off
    np.testing.assert_array_equal(s["rf"].forward(lat, ctx, 0.7), base)


def test_csd_delta_cfg_sampler_skips_unconditional(setup):
    s = setup
    lat, ctx = cases.rng_inputs(108, 128, 4, 4, 8, 64)
    ctx_u = np.random.default_rng(9).standard_normal(ctx.shape).astype(np.float32)
    sched = np.array([1.0, 0.6, 0.3, 0.0], np.float32)
    assert s["rf"].set_sref_csd(s["csd_path"], s["csd"], 1.0) == 0
    z_ref = s["rf"].sample_euler_cfg(lat, ctx, ctx_u, 3.0, sched)
    s["rf"].set_sref_csd(None, s["csd"], 1.0)
    delta = fo.csd_mod_forward(s["cm"], s["csd"])
    z = lat.copy()
    for i in range(3):
        vu = fo.forward(s["w"], CFG, z, ctx_u, float(sched[i]))
        vc = fo.forward(s["w"], CFG, z, ctx, float(sched[i]), temb_delta=delta)
        z = z + (sched[i + 1] - sched[i]) * (vu + 3.0 * (vc - vu))
    assert fo.rel_l2(z, z_ref) < 1e-4


@pytest.mark.parametrize("bands", [(0.3, 2.5), (1.0, 3.0), (0.5, 1.0)])
def test_band_scaled_reference_keys(setup, bands):
    s = setup
    lat, ctx = cases.rng_inputs(110, 128, 4, 4, 8, 64)
    refs = [np.random.default_rng(20 + i).standard_normal((128, 2, 3)).astype(np.float32) for i in range(2)]
    base = s["rf"].forward_refs(lat, refs, ctx, 0.6)
    s["rf"].set_sref_bands(*bands)
    v_ref = s["rf"].forward_refs(lat, refs, ctx, 0.6)
    s["rf"].set_sref_bands(1.0, 1.0)
    v = fo.forward(s["w"], CFG, lat, ctx, 0.6, refs=refs, bands=bands)
    assert fo.rel_l2(v, v_ref) < 1e-4 and fo.rel_l2(v_ref, base) > 1e-3
    # out of range = off; bands do nothing without reference rows
    s["rf"].set_sref_bands(1.5, 0.5)
    np.testing.assert_array_equal(s["rf"].forward_refs(lat, refs, ctx, 0.6), base)
    s["rf"].set_sref_bands(1.0, 1.0)
