"""The autoencoder-decoder oracle (oracle/vae_oracle.py) pinned on CPU against
the reference's own decoder (iris_vae_decode, iris_vae.c:835) compiled from
its sources (oracle/_ref): same random weights, same latents, the uint8
images must agree up to 1 level where f32 summation order moves a value
across a rounding boundary.  Flux (batch-norm statistics + post-quant conv)
and Z-Image (scaling / shift, no quant conv) layouts, square and ragged
latents."""
import numpy as np
import pytest

import psnr_util as pu
from oracle import model_gen as mg
from oracle import vae_oracle as vo

CASES = [  # (zimage, z, latent h, latent w)
    (False, 32, 2, 3),
    (False, 32, 4, 4),
    (True, 16, 3, 2),
]


@pytest.fixture(scope="module")
def ref():
    return pu.ref_lib_or_skip()


@pytest.mark.parametrize("zimage,z,h,w", CASES)
def test_oracle_matches_reference_decoder(ref, tmp_path, zimage, z, h, w):
    path = mg.make_vae_model(str(tmp_path), pu.VAE_SEED, z=z, zimage=zimage)
    wts = mg.vae_weights(pu.VAE_SEED, z, zimage)
    lat = np.random.default_rng(100 + h * 10 + w).standard_normal((4 * z, h, w)).astype(np.float32)
    sc, sh = (mg.ZIMAGE_VAE_SCALING, mg.ZIMAGE_VAE_SHIFT) if zimage else (0.0, 0.0)
    a = ref.vae_decode(path, lat, z, sc, sh)
    f = vo.decode_f32(wts, lat, z, sc, sh)
    b = vo.to_rgb8(f)
    assert a.shape == b.shape == (16 * h, 16 * w, 3)
    d = np.abs(a.astype(np.int32) - b.astype(np.int32))
    assert d.max() <= 1, d.max()
    assert (d == 0).mean() > 0.999
    # the decoder is not saturated: most pixels are inside (0, 255)
    assert 0.05 < f.std() and ((a > 0) & (a < 255)).mean() > 0.8


def test_oracle_unpatchify_order():
    """channel c * 4 + pi * 2 + pj of latent pixel (y, x) -> (2y + pi, 2x + pj)
    of channel c (iris_unpatchify, iris_kernels.c:1110-1135)."""
    z, h, w = 2, 2, 3
    x = np.arange(4 * z * h * w, dtype=np.float32).reshape(4 * z, h, w)
    u = vo.unpatchify(x, z)
    for c in range(z):
        for y in range(h):
            for xx in range(w):
                for pi in range(2):
                    for pj in range(2):
                        assert u[c, 2 * y + pi, 2 * xx + pj] == x[c * 4 + pi * 2 + pj, y, xx]
