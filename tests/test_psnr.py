"""PSNR gate pinned on CPU: the numpy oracle's sampled latent, decoded by the
reference's CPU VAE, against the reference's own sampled latent (golden) —
checks the decode pipeline and that the gate separates close from unrelated
latents."""
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from oracle import flux_oracle as fo
from oracle import model_gen as mg
from oracle import ref_lib
from oracle import sample_oracle as so


@pytest.fixture(scope="module")
def vae(tmp_path_factory):
    ref = pu.ref_lib_or_skip()
    return ref, pu.vae_file(tmp_path_factory)


def test_oracle_latent_decodes_within_gate(vae):
    ref, path = vae
    spec = cases.FLUX_CASES["flux_small"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_small.npz")))
    w = mg.flux_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    z = so.sample_euler(lambda zz, t: fo.forward(w, spec["cfg"], zz, ctx, t), g["z0"], g["sched4"])
    a, b = pu.decode(ref, path, z), pu.decode(ref, path, g["z4"])
    assert a.shape == (16 * h, 16 * wd, 3)
    assert ref_lib.psnr(a, b) >= pu.PSNR_MIN
    # an unrelated latent is far below the gate: the decoder is not flat
    assert ref_lib.psnr(pu.decode(ref, path, g["z0"]), b) < 25.0
