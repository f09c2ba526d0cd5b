"""Shared pieces of the decoded-image PSNR gate (tests/test_psnr*.py).

Both latents of a comparison go through the same decoder: the reference's
own CPU VAE (iris_vae_decode, iris_vae.c:835) from the oracle build, on a
seeded random Flux VAE written by oracle/model_gen.make_vae_model.  The gate
(north_star): PSNR >= 40 dB between the image decoded from our final latent
and the one decoded from the reference's."""
import os

import pytest

from oracle import model_gen as mg

PSNR_MIN = 40.0
VAE_SEED = 17


def ref_lib_or_skip():
    from oracle import ref_lib
    try:
        return ref_lib.RefLib("blas")
    except FileNotFoundError as e:  # the prebuilt reference is test infrastructure
        pytest.skip(f"reference build missing: {e}")


def vae_file(tmp_path_factory) -> str:
    d = str(tmp_path_factory.mktemp("vae"))
    return mg.make_vae_model(d, VAE_SEED)


def decode(ref, path, latent):
    return ref.vae_decode(path, latent)
