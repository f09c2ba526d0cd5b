"""LoRA on the GPU (iris_cuda_flux_load_lora: every adapter folded once into
the resident bf16 weights) vs the reference's runtime hooks
(out += s * B (A x) after each adapted linear, iris_transformer_flux.c:2429-2532,
:3818, :3909; the reference compiled from its sources, oracle/_ref) and vs the
oracle (oracle/lora_oracle.py, folded f32 weights).

Tolerance (north_star): relative L2 <= 1e-2 for every velocity and sampled
latent.  The adapters are drawn strong enough (std 0.15, rank 8) to move the
velocity by 7-80 %, so agreement is not the base model agreeing with itself.
The fold kernel alone is checked against the reference's own MLX golden
fixture and against a torch f32 fold (within one bf16 rounding step).
"""
import ctypes as C
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from gpu_util import rel_l2
from oracle import flux_oracle as fo
from oracle import lora_oracle as lo
from oracle import model_gen as mg

pytestmark = pytest.mark.gpu

TOL = 1e-2
VARIANTS = [("xlabs", {}), ("kohya", {"dtype": "f32"}), ("diffusers", {}),
            ("diffusers", {"single_out": "proj_out"}), ("bfl", {}), ("bfl", {"prefix": "base_model.model"})]


def vid(v):
    return v[0] + "".join(f"-{x}" for x in v[1].values())


@pytest.fixture(scope="module")
def small(tmp_path_factory, iris):
    spec = cases.FLUX_CASES["flux_small"]
    d = str(tmp_path_factory.mktemp("lora_small"))
    w = mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris.Flux.load(d)
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    yield dict(spec=spec, dir=d, w=w, m=m, dims=dims, lat=lat, ctx=ctx)
    m.close()


def lora_file(tmp_path, cfg, fmt, seed=9, **kw):
    path = str(tmp_path / f"{fmt}.safetensors")
    mg.make_flux_lora(path, cfg, fmt, rank=8, seed=seed, std=0.15, **kw)
    return path


@pytest.mark.parametrize("variant", VARIANTS, ids=vid)
def test_forward_with_lora_matches_reference(small, tmp_path, variant):
    from oracle.ref_lib import RefFlux
    ref = pu.ref_lib_or_skip()
    fmt, kw = variant
    s, m, dims = small["spec"], small["m"], small["dims"]
    path = lora_file(tmp_path, s["cfg"], fmt, **kw)
    L = lo.load_lora(path, dims["n_double"], dims["n_single"], dims["hidden"])
    base = m.forward(small["lat"], small["ctx"], 0.7)
    assert m.load_lora(path, 0.8) == lo.count(L)
    v = m.forward(small["lat"], small["ctx"], 0.7)
    rf = RefFlux(ref, small["dir"])
    assert rf.set_lora(path, 0.8)
    v_ref = rf.forward(small["lat"], small["ctx"], 0.7)
    rf.close()
    v_or = fo.forward(lo.merge(small["w"], L, 0.8), s["cfg"], small["lat"], small["ctx"], 0.7)
    assert rel_l2(v, v_ref) < TOL
    assert rel_l2(v, v_or) < TOL
    assert rel_l2(v_ref, base) > 0.05
    # unload restores the base weights bit for bit
    m.unload_lora()
    assert m.lora_adapters == 0
    np.testing.assert_array_equal(m.forward(small["lat"], small["ctx"], 0.7), base)


def test_reload_rescale_and_zero_scale_do_not_drift(small, tmp_path):
    s, m = small["spec"], small["m"]
    p = lora_file(tmp_path, s["cfg"], "bfl")
    q = lora_file(tmp_path, s["cfg"], "diffusers", seed=5)
    base = m.forward(small["lat"], small["ctx"], 1.0)
    m.load_lora(p, 1.0)
    once = m.forward(small["lat"], small["ctx"], 1.0)
    for path, sc in ((p, 0.3), (q, 1.0), (p, -0.5), (p, 1.0)):  # replacing always starts from the base
        m.load_lora(path, sc)
    np.testing.assert_array_equal(m.forward(small["lat"], small["ctx"], 1.0), once)
    m.load_lora(p, 0.0)  # strength 0: the base model exactly
    np.testing.assert_array_equal(m.forward(small["lat"], small["ctx"], 1.0), base)
    m.unload_lora()
    m.unload_lora()  # idempotent


def test_unusable_files_leave_the_current_adapter(small, tmp_path, iris):
    s, m, dims = small["spec"], small["m"], small["dims"]
    p = lora_file(tmp_path, s["cfg"], "kohya")
    m.load_lora(p, 0.8)
    v = m.forward(small["lat"], small["ctx"], 0.7)
    bad = {}
    unknown = str(tmp_path / "unknown.safetensors")
    mg.write_safetensors(unknown, {"some.other.weight": np.zeros((2, 2), np.float32)})
    bad["unknown layout"] = unknown
    # every adapter of a model with another width: all skipped -> nothing to apply
    other = dict(s["cfg"], num_attention_heads=2)
    bad["other model"] = lora_file(tmp_path, other, "bfl")
    bad["missing file"] = str(tmp_path / "nope.safetensors")
    for why, path in bad.items():
        with pytest.raises(iris.IrisCudaError):
            m.load_lora(path, 1.0)
        assert m.lora_adapters == lo.count(lo.load_lora(p, dims["n_double"], dims["n_single"], dims["hidden"])), why
        np.testing.assert_array_equal(m.forward(small["lat"], small["ctx"], 0.7), v)
    m.unload_lora()


def test_sampler_with_lora_matches_reference(iris, tmp_path):
    """Euler sampling (the graph-replayed step) with a LoRA vs the reference's
    sampler with its hooks.  Same head count as the other reference runs of this
    process: the reference's BLAS attention caches its thread count from the
    first model's head count (get_attn_num_threads, iris_transformer_flux.c:1773)
    and computes wrong heads for a later model with fewer heads."""
    from oracle.ref_lib import RefFlux
    ref = pu.ref_lib_or_skip()
    spec = cases.FLUX_CASES["flux_small"]
    g = dict(np.load(os.path.join(GOLDEN, "flux_small.npz")))
    d = str(tmp_path / "m")
    mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    w = mg.flux_weights(spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    p = lora_file(tmp_path, spec["cfg"], "bfl")
    m = iris.Flux.load(d)
    m.load_lora(p, 0.9)
    z = m.sample_euler(g["z0"], ctx, g["sched4"])
    m.close()
    rf = RefFlux(ref, d)
    assert rf.set_lora(p, 0.9)
    z_ref = rf.sample_euler(g["z0"], ctx, g["sched4"])
    rf.close()
    wm = lo.merge(w, lo.load_lora(p, dims["n_double"], dims["n_single"], dims["hidden"]), 0.9)
    z_or = g["z0"].copy()
    s = g["sched4"]
    for i in range(len(s) - 1):
        z_or = z_or + (s[i + 1] - s[i]) * fo.forward(wm, spec["cfg"], z_or, ctx, float(s[i]))
    errs = (rel_l2(z, z_ref), rel_l2(z, z_or), rel_l2(z_ref, z_or))
    assert max(errs) < TOL, errs
    assert rel_l2(z_ref, g["z4"]) > 0.02  # the LoRA changed the sample


# ---------------------------------------------------------------- fold kernel


def _merge(iris, w, w0, ld, B, A, rowmap, nrows, cols, rank, scale):
    import torch
    fn = iris.lib().iris_launch_lora_merge
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                   C.c_int, C.c_float, C.c_void_p]
    rc = fn(w.data_ptr(), w0.data_ptr(), ld, B.data_ptr(), A.data_ptr(), rowmap.data_ptr(), nrows, cols, rank,
            scale, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


def test_fold_kernel_reproduces_reference_fixture(iris):
    """debug/fixtures/lora: W' = 0 + B A, then x W'^T equals the MLX golden
    delta (to within the bf16 rounding of the folded weight)."""
    import torch
    g = dict(np.load(os.path.join(GOLDEN, "lora_fixture.npz")))
    dev = torch.device("cuda:0")
    for key, gold, rows in (("transformer.transformer_blocks.0.attn.to_q", "golden", 8),
                            ("transformer.single_transformer_blocks.0.attn.to_qkv_mlp_proj", "golden_single1", 12),
                            ("transformer.single_transformer_blocks.0.attn.to_out", "golden_single2", 8)):
        A = torch.from_numpy(g[f"t:{key}.lora_A.weight"]).to(dev).contiguous()
        B = torch.from_numpy(g[f"t:{key}.lora_B.weight"]).to(dev).contiguous()
        w0 = torch.zeros(rows, 8, dtype=torch.bfloat16, device=dev)
        w = torch.zeros_like(w0)
        rowmap = torch.arange(rows, dtype=torch.int32, device=dev)
        assert _merge(iris, w, w0, 8, B, A, rowmap, rows, 8, 4, 1.0) == 0
        out = torch.from_numpy(g["x"]).to(dev) @ w.float().T
        assert rel_l2(out.cpu().numpy(), g[gold]) < TOL


def test_fold_kernel_matches_torch(iris):
    """Scattered rows (a permuted subset), rank 40 (two rank chunks, ragged),
    ragged row and column tiles, negative scale, w and w0 distinct: each folded
    element is within one bf16 step of the f64 fold, 99.9 % are its exact bf16
    rounding, and rows outside the map are untouched."""
    import torch
    dev = torch.device("cuda:0")
    gen = torch.Generator(device="cpu").manual_seed(3)
    R, Cc, r, n = 700, 3072 + 136, 40, 517
    w0 = (0.05 * torch.randn(R, Cc, generator=gen)).bfloat16().to(dev)
    w = torch.full_like(w0, 7.0)
    B = (0.1 * torch.randn(n, r, generator=gen)).to(dev)
    A = (0.1 * torch.randn(r, Cc, generator=gen)).to(dev)
    rows = torch.randperm(R, generator=gen)[:n].to(torch.int32).to(dev)
    assert _merge(iris, w, w0, Cc, B, A, rows, n, Cc, r, -0.7) == 0
    exp = w0.float()[rows.long()] + (-0.7) * (B.double() @ A.double()).float()
    got = w.float()[rows.long()]
    err = (got - exp).abs()
    # one bf16 step (2^-7 relative; a sum on the other side of a rounding
    # boundary) plus f32 summation noise where w0 and the update cancel
    assert bool((err <= exp.abs() * 2.0 ** -7 + 1e-6).all()), float((err - exp.abs() * 2.0 ** -7).max())
    assert float((got == exp.bfloat16().float()).float().mean()) > 0.999
    mask = torch.ones(R, dtype=torch.bool, device=dev)
    mask[rows.long()] = False
    assert bool((w[mask] == 7.0).all())
    # argument checks: columns not a multiple of 8, rank 0
    assert _merge(iris, w, w0, Cc, B, A, rows, n, Cc - 4, r, 1.0) != 0
    assert _merge(iris, w, w0, Cc, B, A, rows, n, Cc, 0, 1.0) != 0
