"""The LoRA oracle (oracle/lora_oracle.py) pinned on CPU:

* to the reference's own golden fixture (debug/fixtures/lora, an MLX
  LoRALinear export checked by debug/test_lora.c; stored as
  tests/golden/lora_fixture.npz): to_q delta, single linear1 / linear2 routing;
* to the reference loader (lora_load, compiled from its sources, oracle/_ref):
  the same adapter table, bit for bit, for all four key layouts (XLabs, Kohya,
  Diffusers, BFL with both prefixes, Diffusers proj_out fallback), and the same
  skips (mismatched shapes, unknown format, no matching keys);
* to the reference forward with a LoRA (runtime hooks): the oracle forward on
  the folded weights agrees to f32 rounding.
"""
import os

import numpy as np
import pytest

import cases
import psnr_util as pu
from conftest import GOLDEN
from oracle import flux_oracle as fo
from oracle import lora_oracle as lo
from oracle import model_gen as mg


def fixture_file(tmp_path):
    g = dict(np.load(os.path.join(GOLDEN, "lora_fixture.npz")))
    path = str(tmp_path / "fixture.safetensors")
    mg.write_safetensors(path, {k[2:]: v.astype(np.float32) for k, v in g.items() if k.startswith("t:")})
    return path, g


def corr_maxabs(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return a @ b / (np.linalg.norm(a) * np.linalg.norm(b)), np.abs(a - b).max()


def test_fixture_to_q_delta(tmp_path):
    """debug/test_lora.c test_parity_fixture: lora_load(.., 1, 0, 8) -> to_q."""
    path, g = fixture_file(tmp_path)
    L = lo.load_lora(path, 1, 0, 8)
    assert lo.count(L) == 1 and 0 in L["double_img_q"]
    out = lo.lora_apply(L["double_img_q"][0], 1.0, g["x"], np.zeros((5, 8), np.float32))
    c, m = corr_maxabs(out, g["golden"])
    assert c > 0.999 and m < 1e-3, (c, m)
    assert m < 1e-5  # f32 export of the same product: far tighter than the reference's 1e-3


def test_fixture_single_block_routing(tmp_path):
    """test_single_block_parity: to_qkv_mlp_proj -> linear1 (12 out), to_out -> linear2."""
    path, g = fixture_file(tmp_path)
    L = lo.load_lora(path, 0, 1, 8)
    assert set(L["single_linear1"]) == {0} and set(L["single_linear2"]) == {0}
    o1 = lo.lora_apply(L["single_linear1"][0], 1.0, g["x"], np.zeros((5, 12), np.float32))
    o2 = lo.lora_apply(L["single_linear2"][0], 1.0, g["x"], np.zeros((5, 8), np.float32))
    for out, gold in ((o1, g["golden_single1"]), (o2, g["golden_single2"])):
        c, m = corr_maxabs(out, gold)
        assert c > 0.999 and m < 1e-5, (c, m)


def test_scale_zero_and_rank1_by_hand():
    """test_scale_zero / test_rank1_correctness of debug/test_lora.c."""
    a = (np.array([[1, 0, 0, 0], [0, 1, 0, 0]], np.float32), np.eye(2, dtype=np.float32))
    x = np.arange(1, 13, dtype=np.float32).reshape(3, 4)
    out = np.array([[10, 20], [30, 40], [50, 60]], np.float32)
    np.testing.assert_array_equal(lo.lora_apply(a, 0.0, x, out), out)
    r1 = (np.array([[1.0, 2.0]], np.float32), np.array([[3.0], [4.0]], np.float32))
    np.testing.assert_allclose(lo.lora_apply(r1, 0.5, np.array([[1.0, 0.0]], np.float32),
                                             np.array([[10.0, 20.0]], np.float32)), [[11.5, 22.0]])


CFG = cases.FLUX_CASES["flux_tiny"]["cfg"]
DIMS = mg.flux_dims(CFG)
VARIANTS = [("xlabs", {}), ("kohya", {}), ("diffusers", {}), ("diffusers", {"single_out": "proj_out"}),
            ("bfl", {}), ("bfl", {"prefix": "base_model.model"})]


def vid(v):
    return v[0] + "".join(f"-{x}" for x in v[1].values())


@pytest.mark.parametrize("variant", VARIANTS, ids=vid)
def test_adapter_table_matches_reference_loader(tmp_path, variant):
    ref = pu.ref_lib_or_skip()
    fmt, kw = variant
    path = str(tmp_path / "l.safetensors")
    mg.make_flux_lora(path, CFG, fmt, rank=8, seed=4, dtype="f32" if fmt == "kohya" else "bf16", **kw)
    L = lo.load_lora(path, DIMS["n_double"], DIMS["n_single"], DIMS["hidden"])
    n = 0
    for k, kind in enumerate(lo.KINDS):
        nblk = DIMS["n_double"] if k < 8 else DIMS["n_single"]
        for i in range(nblk):
            r = ref.lora_get(path, DIMS["n_double"], DIMS["n_single"], DIMS["hidden"], k, i)
            o = L[kind].get(i)
            assert (r is None) == (o is None), (kind, i)
            if r is not None:
                np.testing.assert_array_equal(r[0], o[0])
                np.testing.assert_array_equal(r[1], o[1])
                n += 1
    # table entries: 8 per double block (a fused Q|K|V fills three), 2 per single block
    assert n == 8 * DIMS["n_double"] + (0 if fmt == "xlabs" else 2 * DIMS["n_single"])
    assert lo.count(L) == (4 if fmt != "diffusers" else 8) * DIMS["n_double"] + (
        0 if fmt == "xlabs" else 2 * DIMS["n_single"])


def test_loader_skips_match_reference(tmp_path):
    """Shape mismatches are skipped, an unknown layout or a file with no usable
    key loads nothing — in the reference and in the oracle alike."""
    ref = pu.ref_lib_or_skip()
    H = DIMS["hidden"]
    rng = np.random.default_rng(0)
    t = {  # Diffusers: to_q with the wrong input width, to_k fine
        "transformer.transformer_blocks.0.attn.to_q.lora_A.weight": rng.standard_normal((4, H + 8)).astype(np.float32),
        "transformer.transformer_blocks.0.attn.to_q.lora_B.weight": rng.standard_normal((H, 4)).astype(np.float32),
        "transformer.transformer_blocks.0.attn.to_k.lora_A.weight": rng.standard_normal((4, H)).astype(np.float32),
        "transformer.transformer_blocks.0.attn.to_k.lora_B.weight": rng.standard_normal((H, 4)).astype(np.float32),
    }
    p = str(tmp_path / "mixed.safetensors")
    mg.write_safetensors(p, t)
    L = lo.load_lora(p, 1, 2, H)
    assert lo.count(L) == 1 and set(L["double_img_k"]) == {0} and not L["double_img_q"]
    assert ref.lora_get(p, 1, 2, H, 0, 0) is None and ref.lora_get(p, 1, 2, H, 1, 0) is not None
    # fused QKV whose up matrix is not 3H rows: skipped (load_adapter_split_qkv)
    p2 = str(tmp_path / "badqkv.safetensors")
    mg.write_safetensors(p2, {"diffusion_model.double_blocks.0.img_attn.qkv.lora_A.weight": t[
        "transformer.transformer_blocks.0.attn.to_k.lora_A.weight"],
        "diffusion_model.double_blocks.0.img_attn.qkv.lora_B.weight": rng.standard_normal((2 * H, 4)).astype(
            np.float32)})
    assert lo.load_lora(p2, 1, 2, H) is None
    with pytest.raises(RuntimeError):
        ref.lora_get(p2, 1, 2, H, 0, 0)
    # unknown layout
    p3 = str(tmp_path / "unknown.safetensors")
    mg.write_safetensors(p3, {"some.other.weight": np.zeros((2, 2), np.float32)})
    assert lo.load_lora(p3, 1, 2, H) is None
    with pytest.raises(RuntimeError):
        ref.lora_get(p3, 1, 2, H, 0, 0)


@pytest.mark.parametrize("fmt", mg.LORA_FORMATS)
def test_oracle_forward_with_lora_matches_reference(tmp_path, fmt):
    """Reference: runtime hooks out += s B (A x); oracle: folded weights."""
    ref = pu.ref_lib_or_skip()
    from oracle.ref_lib import RefFlux
    spec = cases.FLUX_CASES["flux_tiny"]
    d = str(tmp_path / "m")
    w = mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    path = str(tmp_path / "l.safetensors")
    mg.make_flux_lora(path, spec["cfg"], fmt, rank=8, seed=9, std=0.15)
    h, wd = spec["img"]
    lat, ctx = cases.rng_inputs(spec["seed"] + 100, DIMS["channels"], h, wd, spec["txt"], DIMS["text_dim"])
    rf = RefFlux(ref, d)
    base = rf.forward(lat, ctx, 0.7)
    assert rf.set_lora(path, 0.8)
    v_ref = rf.forward(lat, ctx, 0.7)
    rf.clear_lora()
    np.testing.assert_array_equal(rf.forward(lat, ctx, 0.7), base)
    rf.close()
    L = lo.load_lora(path, DIMS["n_double"], DIMS["n_single"], DIMS["hidden"])
    v_or = fo.forward(lo.merge(w, L, 0.8), spec["cfg"], lat, ctx, 0.7)
    assert fo.rel_l2(v_or, v_ref) < 1e-4
    # the adapter changes the output substantially (the comparison is not vacuous)
    assert fo.rel_l2(base, v_ref) > 0.05


# ---------------------------------------------------------------- the C library's loader (host only)


@pytest.mark.parametrize("variant", VARIANTS, ids=vid)
def test_library_loader_routes_like_reference(tmp_path, variant):
    """iris_cuda_lora_probe runs the product's own key routing and shape checks
    (csrc/lora.c) without a GPU: same format, same adapters as the oracle."""
    import iris_cuda
    fmt, kw = variant
    path = str(tmp_path / "l.safetensors")
    mg.make_flux_lora(path, CFG, fmt, rank=8, seed=4, **kw)
    L = lo.load_lora(path, DIMS["n_double"], DIMS["n_single"], DIMS["hidden"])
    p = iris_cuda.lora_probe(path, DIMS["n_double"], DIMS["n_single"], DIMS["hidden"], DIMS["mlp"])
    assert p["format"] == fmt and p["adapters"] == lo.count(L)
    nd, ns = DIMS["n_double"], DIMS["n_single"]
    assert p["qkv"] == (6 if fmt == "diffusers" else 2) * nd and p["proj"] == 2 * nd
    assert p["linear1"] == p["linear2"] == (0 if fmt == "xlabs" else ns)
    # a model with fewer blocks reads only its own blocks' keys
    assert iris_cuda.lora_probe(path, nd, 1, DIMS["hidden"], DIMS["mlp"])["adapters"] == lo.count(
        lo.load_lora(path, nd, 1, DIMS["hidden"]))


def test_library_loader_skips(tmp_path):
    import iris_cuda
    H, F = DIMS["hidden"], DIMS["mlp"]
    rng = np.random.default_rng(1)
    n = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    p = str(tmp_path / "a.safetensors")
    mg.write_safetensors(p, {
        "transformer.transformer_blocks.0.attn.to_q.lora_A.weight": n(4, H + 8),   # wrong input width
        "transformer.transformer_blocks.0.attn.to_q.lora_B.weight": n(H, 4),
        "transformer.transformer_blocks.0.attn.to_k.lora_A.weight": n(4, H),
        "transformer.transformer_blocks.0.attn.to_k.lora_B.weight": n(H, 4),
        "transformer.transformer_blocks.0.attn.to_v.lora_A.weight": n(4, H),
        "transformer.transformer_blocks.0.attn.to_v.lora_B.weight": n(H, 3),       # B not [out, rank]
        # single linear1 of another model's width: the reference loads it unchecked
        # (iris_lora.c:327) and would index past its buffers; the library skips it
        "transformer.single_transformer_blocks.0.attn.to_qkv_mlp_proj.lora_A.weight": n(4, H),
        "transformer.single_transformer_blocks.0.attn.to_qkv_mlp_proj.lora_B.weight": n(3 * H + F + 128, 4),
        "transformer.single_transformer_blocks.1.attn.to_out.lora_A.weight": n(4, H + F),
        "transformer.single_transformer_blocks.1.attn.to_out.lora_B.weight": n(H, 4),
    })
    q = iris_cuda.lora_probe(p, 1, 2, H, F)
    assert q == {"format": "diffusers", "adapters": 2, "qkv": 1, "proj": 0, "linear1": 0, "linear2": 1}
    unknown = str(tmp_path / "u.safetensors")
    mg.write_safetensors(unknown, {"x.weight": n(2, 2)})
    with pytest.raises(iris_cuda.IrisCudaError):
        iris_cuda.lora_probe(unknown, 1, 2, H, F)
    with pytest.raises(iris_cuda.IrisCudaError):
        iris_cuda.lora_probe(str(tmp_path / "missing.safetensors"), 1, 2, H, F)
    # truncated file: header claims more data than present
    bad = str(tmp_path / "trunc.safetensors")
    mg.write_safetensors(bad, {"lora_unet_double_blocks_0_img_attn_proj.lora_down.weight": n(4, H),
                               "lora_unet_double_blocks_0_img_attn_proj.lora_up.weight": n(H, 4)})
    raw = open(bad, "rb").read()
    open(bad, "wb").write(raw[:-64])
    with pytest.raises(iris_cuda.IrisCudaError):
        iris_cuda.lora_probe(bad, 1, 2, H, F)
