"""Autoencoder decoder on the GPU through the C ABI (iris_cuda_vae_*), against
the numpy oracle (oracle/vae_oracle.py, itself pinned to the reference decoder
by tests/test_vae_oracle.py) and against the reference's own CPU decoder
(iris_vae_decode, iris_vae.c:835, from oracle/_ref).

Gates: the f32 RGB planes before quantisation within rel-L2 1e-2 of the
oracle (bf16 convolution inputs, f32 accumulation and residual stream); the
uint8 image at PSNR >= 40 dB against the reference's image."""
import numpy as np
import pytest

import psnr_util as pu
from gpu_util import rel_l2
from oracle import model_gen as mg
from oracle import ref_lib
from oracle import vae_oracle as vo

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module")
def flux_vae(iris, tmp_path_factory):
    d = str(tmp_path_factory.mktemp("vae_flux"))
    mg.make_vae_model(d, pu.VAE_SEED)
    v = iris.Vae.load(d + "/vae")
    yield v, mg.vae_weights(pu.VAE_SEED), d + "/vae/diffusion_pytorch_model.safetensors"
    v.close()


@pytest.fixture(scope="module")
def zimage_vae(iris, tmp_path_factory):
    d = str(tmp_path_factory.mktemp("vae_zi"))
    mg.make_vae_model(d, pu.VAE_SEED, z=16, zimage=True)
    v = iris.Vae.load(d + "/vae")
    yield v, mg.vae_weights(pu.VAE_SEED, 16, True), d + "/vae/diffusion_pytorch_model.safetensors"
    v.close()


def latent(z, h, w, seed=3):
    return np.random.default_rng(seed).standard_normal((4 * z, h, w)).astype(np.float32)


# square, ragged (image rows shorter than a 128-pixel tile), odd sizes
@pytest.mark.parametrize("h,w", [(2, 3), (4, 4), (5, 7), (8, 12)])
def test_flux_decode_matches_oracle(flux_vae, h, w):
    v, wts, _ = flux_vae
    lat = latent(32, h, w)
    got = v.decode_f32(lat)
    ref = vo.decode_f32(wts, lat)
    assert got.shape == ref.shape == (3, 16 * h, 16 * w)
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < TOL, rel_l2(got, ref)
    img = v.decode(lat)
    assert img.shape == (16 * h, 16 * w, 3) and img.dtype == np.uint8
    assert ref_lib.psnr(img, vo.to_rgb8(ref)) >= pu.PSNR_MIN


def test_zimage_decode_matches_oracle(zimage_vae):
    v, wts, _ = zimage_vae
    lat = latent(16, 4, 6, seed=9)
    sc, sh = mg.ZIMAGE_VAE_SCALING, mg.ZIMAGE_VAE_SHIFT
    got = v.decode_f32(lat)
    ref = vo.decode_f32(wts, lat, 16, sc, sh)
    assert rel_l2(got, ref) < TOL, rel_l2(got, ref)


@pytest.mark.parametrize("h,w", [(4, 4), (16, 16)])
def test_decode_psnr_vs_reference_decoder(flux_vae, h, w):
    """The image the reference's CPU decoder makes from the same latent
    (256 x 256 pixels at 16 x 16: a 1024-pixel mid-block attention)."""
    v, _, path = flux_vae
    ref = pu.ref_lib_or_skip()
    lat = latent(32, h, w, seed=h)
    a = v.decode(lat)
    b = ref.vae_decode(path, lat)
    assert ref_lib.psnr(a, b) >= pu.PSNR_MIN, ref_lib.psnr(a, b)


def test_decode_is_deterministic_and_graph_replays(flux_vae):
    v, _, _ = flux_vae
    lat = latent(32, 6, 5, seed=11)
    a = v.decode_f32(lat)
    n = v.graph_kernels()
    b = v.decode_f32(lat)
    assert np.array_equal(a, b)
    assert n > 50 and v.graph_kernels() == n
    # a different size re-plans, then the first size decodes the same again
    v.decode_f32(latent(32, 3, 3))
    assert np.array_equal(v.decode_f32(lat), a)


def test_device_entry_point_matches_host(iris, flux_vae):
    import ctypes as C
    import torch
    v, _, _ = flux_vae
    lat = latent(32, 4, 5, seed=5)
    host8 = v.decode(lat)
    d_lat = torch.from_numpy(lat).cuda()
    d_rgb8 = torch.zeros(16 * 4 * 16 * 5 * 3, dtype=torch.uint8, device="cuda")
    d_rgb = torch.zeros(3 * 64 * 80, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rc = iris.lib().iris_cuda_vae_decode_dev(v.h, C.c_void_p(d_lat.data_ptr()), 4, 5,
                                            C.c_void_p(d_rgb8.data_ptr()), C.c_void_p(d_rgb.data_ptr()))
    assert rc == 0, iris.last_error()
    assert iris.lib().iris_cuda_synchronize() == 0
    assert np.array_equal(d_rgb8.cpu().numpy().reshape(64, 80, 3), host8)
    assert np.array_equal(d_rgb.cpu().numpy().reshape(3, 64, 80), v.decode_f32(lat))


def test_bad_arguments_fail_loudly(iris, flux_vae):
    v, _, _ = flux_vae
    lat = latent(32, 2, 2)
    assert not iris.lib().iris_cuda_vae_decode(v.h, iris._f(lat), 2, 2, 2)  # batch 2
    assert "batch" in iris.last_error()
    big = np.zeros((128, 200, 200), np.float32)
    assert iris.lib().iris_cuda_vae_decode_f32(v.h, iris._f(big), 200, 200, iris._f(np.zeros(1, np.float32))) != 0
    with pytest.raises(iris.IrisCudaError):
        iris.Vae.load("/nonexistent/vae")


def test_random_init_decoder_is_finite_and_profiles(iris):
    v = iris.Vae.random(32, seed=5)
    lat = latent(32, 4, 4, seed=2)
    img = v.decode(lat)
    f = v.decode_f32(lat)
    assert np.isfinite(f).all() and 0.05 < f.std() < 10
    assert img.shape == (64, 64, 3)
    prof = v.profile()
    names = {e["name"] for e in prof}
    assert {"gn_stats", "gn_finalize", "gn_apply", "attn_gemm", "attn_softmax", "upsample"} <= names
    assert any(n.startswith("conv3x3_c512") for n in names)
    assert len(prof) == v.graph_kernels()
    v.close()
