"""Decoded-image PSNR gate for the CUDA backend (north_star: >= 40 dB).

The final latent of our sampler and the reference's are decoded by the same
reference CPU VAE (iris_vae_decode) on a seeded random Flux VAE:
* golden cases: 4-step Euler (flux_small), 3-step CFG 4.0 (flux_tiny);
* a 16x16-latent (256x256 image) 4-step run whose reference latent is
  computed here by the reference's own sampler (iris_sample_euler) from the
  same model files."""
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from oracle import model_gen as mg
from oracle import ref_lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def vae(tmp_path_factory):
    ref = pu.ref_lib_or_skip()
    return ref, pu.vae_file(tmp_path_factory)


def test_euler_golden_psnr(iris, vae, tmp_path):
    ref, path = vae
    spec = cases.FLUX_CASES["flux_small"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_small.npz")))
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.Flux.load(str(tmp_path))
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    z = m.sample_euler(g["z0"], ctx, g["sched4"])
    m.close()
    p = ref_lib.psnr(pu.decode(ref, path, z), pu.decode(ref, path, g["z4"]))
    assert p >= pu.PSNR_MIN, p


def test_cfg_golden_psnr(iris, vae, tmp_path):
    ref, path = vae
    spec = cases.FLUX_CASES["flux_tiny"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_tiny.npz")))
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.Flux.load(str(tmp_path))
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    _, ctx_u = cases.ref_inputs(dims["channels"], ctx.shape)
    z = m.sample_euler(g["z0"], ctx, g["sched3"], txt_uncond=ctx_u, guidance=4.0)
    m.close()
    p = ref_lib.psnr(pu.decode(ref, path, z), pu.decode(ref, path, g["z_cfg"]))
    assert p >= pu.PSNR_MIN, p


def test_256px_image_psnr_against_reference_sampler(iris, vae, tmp_path):
    ref, path = vae
    spec = cases.FLUX_CASES["flux_small"]
    mg.make_flux_model(str(tmp_path), spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    ctx = np.random.default_rng(41).standard_normal((64, dims["text_dim"])).astype(np.float32)
    z0 = iris.init_noise(dims["channels"], 16, 16, 1234)
    sched = iris.official_schedule(4, 256)
    rf = ref_lib.RefFlux(ref, str(tmp_path))
    z_ref = rf.sample_euler(z0, ctx, sched)
    rf.close()
    m = iris.Flux.load(str(tmp_path))
    z = m.sample_euler(z0, ctx, sched)
    m.close()
    a, b = pu.decode(ref, path, z), pu.decode(ref, path, z_ref)
    assert a.shape == (256, 256, 3)
    p = ref_lib.psnr(a, b)
    assert p >= pu.PSNR_MIN, p
