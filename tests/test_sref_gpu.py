"""SREF style controls on the GPU vs the oracle and the reference (oracle/_ref):
the CSD temb delta (forward, CFG sampler without it on the unconditional
branch, off again) and the K-side band scaling of reference rows in a
multi-reference forward.  Tolerance: relative L2 <= 1e-2 (north_star)."""
import numpy as np
import pytest

import cases
import psnr_util as pu
from gpu_util import rel_l2
from oracle import flux_oracle as fo
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

TOL = 1e-2
CFG = dict(num_attention_heads=2, attention_head_dim=128, num_layers=1, num_single_layers=2,
           joint_attention_dim=64, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)


@pytest.fixture(scope="module")
def setup(tmp_path_factory, iris):
    from oracle.ref_lib import RefFlux
    d = str(tmp_path_factory.mktemp("sref"))
    w = mg.make_flux_model(d, CFG, 7, 0.05, "unit")
    csd_path = d + "/csd_mod.safetensors"
    cm = mg.make_csd_mod(csd_path, 32, 96, 256, seed=4)
    csd = np.random.default_rng(2).standard_normal(32).astype(np.float32)
    csd /= np.linalg.norm(csd)
    m = iris.Flux.load(d)
    ref = pu.ref_lib_or_skip()
    rf = RefFlux(ref, d)
    yield dict(w=w, m=m, rf=rf, csd_path=csd_path, cm=cm, csd=csd)
    rf.close()
    m.close()


def test_csd_delta_forward_and_cfg(setup, iris):
    s = setup
    m = s["m"]
    lat, ctx = cases.rng_inputs(107, 128, 4, 4, 8, 64)
    base = m.forward(lat, ctx, 0.7)
    m.set_sref_csd(s["csd_path"], s["csd"], 1.5)
    v = m.forward(lat, ctx, 0.7)
    delta = 1.5 * fo.csd_mod_forward(s["cm"], s["csd"])
    assert rel_l2(v, fo.forward(s["w"], CFG, lat, ctx, 0.7, temb_delta=delta)) < TOL
    assert s["rf"].set_sref_csd(s["csd_path"], s["csd"], 1.5) == 0
    assert rel_l2(v, s["rf"].forward(lat, ctx, 0.7)) < TOL
    assert rel_l2(v, base) > 0.05
    # CFG: the unconditional branch without the delta
    ctx_u = np.random.default_rng(9).standard_normal(ctx.shape).astype(np.float32)
    sched = np.array([1.0, 0.6, 0.3, 0.0], np.float32)
    m.set_sref_csd(s["csd_path"], s["csd"], 1.0)
    s["rf"].set_sref_csd(s["csd_path"], s["csd"], 1.0)
    z = m.sample_euler(lat, ctx, sched, txt_uncond=ctx_u, guidance=3.0)
    assert rel_l2(z, s["rf"].sample_euler_cfg(lat, ctx, ctx_u, 3.0, sched)) < TOL
    # the flag is back on after the sampler: a plain forward has the delta again
    m.set_sref_csd(s["csd_path"], s["csd"], 1.5)
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.7), v)
    # off: the base model bit for bit; a mismatched MLP is rejected
    m.set_sref_csd(None, None, 0.0)
    s["rf"].set_sref_csd(None, s["csd"], 1.0)
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.7), base)
    with pytest.raises(iris.IrisCudaError):
        m.set_sref_csd(s["csd_path"], s["csd"][:16], 1.0)


@pytest.mark.parametrize("bands", [(0.3, 2.5), (1.0, 3.0)])
def test_band_scaled_reference_keys(setup, bands):
    s = setup
    m = s["m"]
    lat, ctx = cases.rng_inputs(110, 128, 4, 4, 8, 64)
    refs = [np.random.default_rng(20 + i).standard_normal((128, 2, 3)).astype(np.float32) for i in range(2)]
    base = m.forward(lat, ctx, 0.6, refs=refs)
    m.set_sref_bands(*bands)
    v = m.forward(lat, ctx, 0.6, refs=refs)
    assert rel_l2(v, fo.forward(s["w"], CFG, lat, ctx, 0.6, refs=refs, bands=bands)) < TOL
    s["rf"].set_sref_bands(*bands)
    assert rel_l2(v, s["rf"].forward_refs(lat, refs, ctx, 0.6)) < TOL
    s["rf"].set_sref_bands(1.0, 1.0)
    # the band change reaches the output beyond the bf16 noise of the two runs
    assert rel_l2(v, base) > 1e-3
    m.set_sref_bands(1.5, 0.5)  # out of range: off
    np.testing.assert_array_equal(m.forward(lat, ctx, 0.6, refs=refs), base)
