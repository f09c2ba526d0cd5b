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


class LoraFold(C.Structure):
    """IrisLoraFold (csrc/iris_kernels.h)."""
    _fields_ = [("w", C.c_void_p), ("w0", C.c_void_p), ("ld", C.c_int), ("cols", C.c_int), ("nrows", C.c_int),
                ("B", C.c_void_p), ("b_dtype", C.c_int), ("rank", C.c_int), ("bsrc", C.c_void_p),
                ("drow", C.c_void_p), ("A", C.c_void_p), ("a_dtype", C.c_int), ("in_dim", C.c_int),
                ("acol_seg", C.c_int), ("acol_off0", C.c_int), ("acol_off1", C.c_int), ("scale", C.c_float)]


DT = {"bf16": 0, "f16": 1, "f32": 2}


def _fold(iris, w, w0, B, A, bsrc, drow, scale, seg=None, off0=0, off1=0):
    """iris_launch_lora_fold on torch tensors; returns the CUDA error code."""
    import torch
    lib = iris.lib()
    lib.iris_launch_lora_fold.restype = C.c_int
    lib.iris_launch_lora_fold.argtypes = [C.POINTER(LoraFold), C.c_void_p, C.c_size_t, C.c_void_p, C.c_int,
                                          C.c_void_p, C.POINTER(C.c_int)]
    lib.iris_lora_fold_scratch_bytes.restype = C.c_size_t
    lib.iris_lora_fold_scratch_bytes.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
    dt = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}
    cols = w.shape[1]
    f = LoraFold(w.data_ptr(), w0.data_ptr(), cols, cols, bsrc.numel(), B.data_ptr(), DT[dt[B.dtype]], B.shape[1],
                 bsrc.data_ptr(), drow.data_ptr(), A.data_ptr(), DT[dt[A.dtype]], A.shape[1],
                 cols if seg is None else seg, off0, off1, scale)
    split = int(B.dtype != torch.bfloat16 or A.dtype != torch.bfloat16)
    nb = lib.iris_lora_fold_scratch_bytes(bsrc.numel(), cols, B.shape[1], split)
    scratch = torch.empty(max(nb, 1), dtype=torch.uint8, device=w.device)
    status = torch.zeros(1, dtype=torch.int32, device=w.device)
    n = C.c_int(0)
    rc = lib.iris_launch_lora_fold(C.byref(f), scratch.data_ptr(), nb, status.data_ptr(), 148,
                                   torch.cuda.current_stream().cuda_stream, C.byref(n))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return rc


def test_fold_kernel_reproduces_reference_fixture(iris):
    """debug/fixtures/lora: W' = 0 + B A, then x W'^T equals the MLX golden
    delta (to within the bf16 rounding of the folded weight); f32 operands (the
    fixture's type) take the hi/lo split path."""
    import torch
    g = dict(np.load(os.path.join(GOLDEN, "lora_fixture.npz")))
    dev = torch.device("cuda:0")
    for key, gold, rows in (("transformer.transformer_blocks.0.attn.to_q", "golden", 8),
                            ("transformer.single_transformer_blocks.0.attn.to_qkv_mlp_proj", "golden_single1", 12),
                            ("transformer.single_transformer_blocks.0.attn.to_out", "golden_single2", 8)):
        a = np.zeros((4, 128), np.float32)  # fold widths are multiples of 128: the 8 real columns, zeros after
        a[:, :8] = g[f"t:{key}.lora_A.weight"]
        A = torch.from_numpy(a).to(dev)
        B = torch.from_numpy(g[f"t:{key}.lora_B.weight"]).to(dev).contiguous()
        w0 = torch.zeros(rows, 128, dtype=torch.bfloat16, device=dev)
        w = torch.zeros_like(w0)
        idx = torch.arange(rows, dtype=torch.int32, device=dev)
        assert _fold(iris, w, w0, B, A, idx, idx, 1.0) == 0
        out = torch.from_numpy(g["x"]).to(dev) @ w[:, :8].float().T
        assert rel_l2(out.cpu().numpy(), g[gold]) < TOL


@pytest.mark.parametrize("dtype,cols", [("bf16", 3072), ("f32", 3200), ("f16", 3072)])
def test_fold_kernel_matches_torch(iris, dtype, cols):
    """Gathered B rows onto scattered target rows (517 of 700), a two-segment
    column map, rank 40, negative scale, w and w0 distinct; 3072 columns run
    on the CTA-pair GEMM, 3200 on the single-CTA one.  Each folded element is
    within one bf16 step of the f64 fold, 99.9 % are its exact bf16 rounding,
    and rows outside the map are untouched (f32 operands: 99 %)."""
    import torch
    dev = torch.device("cuda:0")
    tdt = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16}[dtype]
    gen = torch.Generator(device="cpu").manual_seed(3)
    R, r, n, nb, ind = 700, 40, 517, 900, cols + 300
    seg, off0, off1 = cols // 2, 100, cols // 2 + 250
    w0 = (0.05 * torch.randn(R, cols, generator=gen)).bfloat16().to(dev)
    w = torch.full_like(w0, 7.0)
    B = (0.1 * torch.randn(nb, r, generator=gen)).to(tdt).to(dev)
    A = (0.1 * torch.randn(r, ind, generator=gen)).to(tdt).to(dev)
    drow = torch.randperm(R, generator=gen)[:n].to(torch.int32).to(dev)
    bsrc = torch.randperm(nb, generator=gen)[:n].to(torch.int32).to(dev)
    assert _fold(iris, w, w0, B, A, bsrc, drow, -0.7, seg, off0, off1) == 0
    acol = torch.cat([torch.arange(seg) + off0, torch.arange(cols - seg) + off1]).to(dev)
    delta = (B.double()[bsrc.long()] @ A.double()[:, acol]) * -0.7
    exp = w0.double()[drow.long()] + delta
    got = w.double()[drow.long()]
    err = (got - exp).abs()
    # one bf16 step (2^-7 relative; a sum on the other side of a rounding boundary)
    # plus f32 accumulation noise where w0 and the update cancel
    assert bool((err <= exp.abs() * 2.0 ** -7 + 1e-6).all()), float((err - exp.abs() * 2.0 ** -7).max())
    # bf16 and f16 operands are exact; f32 ones keep 16 of 24 bits (hi + lo)
    exact = float((got == exp.float().bfloat16().double()).double().mean())
    assert exact > (0.99 if dtype == "f32" else 0.999), exact
    mask = torch.ones(R, dtype=torch.bool, device=dev)
    mask[drow.long()] = False
    assert bool((w[mask] == 7.0).all())


def test_fold_kernel_rejects_bad_shapes(iris):
    import torch
    dev = torch.device("cuda:0")
    w0 = torch.zeros(64, 256, dtype=torch.bfloat16, device=dev)
    w = torch.zeros_like(w0)
    B = torch.zeros(64, 8, dtype=torch.bfloat16, device=dev)
    A = torch.zeros(8, 256, dtype=torch.bfloat16, device=dev)
    idx = torch.arange(64, dtype=torch.int32, device=dev)
    assert _fold(iris, w[:, :200], w0[:, :200], B, A, idx, idx, 1.0) != 0  # columns not a multiple of 128
    assert _fold(iris, w, w0, B[:, :0], A[:0], idx, idx, 1.0) != 0          # rank 0
    flat = torch.zeros(64 * 256 + 8, dtype=torch.bfloat16, device=dev)
    assert _fold(iris, flat[1:1 + 64 * 256].view(64, 256), w0, B, A, idx, idx, 1.0) != 0  # misaligned w
