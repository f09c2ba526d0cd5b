"""Op-level parity of the iris_gpu_* surface against the oracle's functions
(oracle/flux_oracle.py, each citing the reference code it restates).

Inputs are bf16-valued; outputs are bf16, so tolerances are bf16-level:
relative L2 <= 1e-2 (north_star's per-op/per-block bound), most ops land
near 2e-3.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import Dev, bf16_round, rel_l2
from oracle import flux_oracle as fo

pytestmark = pytest.mark.gpu
_fp = C.POINTER(C.c_float)


@pytest.mark.parametrize("sq,sk,heads", [(16, 80, 2), (80, 80, 2), (128, 128, 3), (128, 129, 2), (129, 128, 2),
                                         (200, 333, 3), (1536, 1536, 4), (1, 64, 1), (130, 1, 1)])
@pytest.mark.parametrize("scale_std", [1.0, 4.0])
def test_attention(iris, sq, sk, heads, scale_std):
    rng = np.random.default_rng(sq + sk + heads)
    q = bf16_round(rng.standard_normal((sq, heads * 128)) * scale_std)
    k = bf16_round(rng.standard_normal((sk, heads * 128)))
    v = bf16_round(rng.standard_normal((sk, heads * 128)))
    Q, K, V, O = Dev(q), Dev(k), Dev(v), Dev(n=sq * heads * 128)
    ok = iris.lib().iris_gpu_attention_fused_bf16(O.h, Q.h, K.h, V.h, sq, sk, heads, 128,
                                                  1.0 / np.sqrt(128.0))
    assert ok, iris.last_error()
    ref = fo.attention(q, k, v, heads)
    assert rel_l2(O.read((sq, heads * 128)), ref) < 1e-2


# Shapes with many heads take the CTA-pair kernel (cta_group::2, four query
# tiles per pair): the Klein-4B single-block shape, ragged query and key
# counts, a key count under one tile (the IP-Adapter's 64 tokens) and a long
# sequence.  `ramp` grows the keys' norm along the sequence so that later key
# tiles raise the rows' maximum and the rescaling of O in TMEM is exercised.
@pytest.mark.parametrize("sq,sk,heads,scale_std,ramp", [(1536, 1536, 24, 1.0, 0.0), (1100, 1100, 40, 4.0, 0.0),
                                                        (1024, 64, 48, 1.0, 0.0), (300, 2000, 40, 2.0, 3.0),
                                                        (4608, 4608, 6, 1.0, 3.0)])
def test_attention_pair_kernel(iris, sq, sk, heads, scale_std, ramp):
    rng = np.random.default_rng(sq * 7 + sk + heads)
    q = bf16_round(rng.standard_normal((sq, heads * 128)) * scale_std)
    k = bf16_round(rng.standard_normal((sk, heads * 128)) * (1.0 + ramp * np.arange(sk) / sk)[:, None])
    v = bf16_round(rng.standard_normal((sk, heads * 128)))
    Q, K, V, O = Dev(q), Dev(k), Dev(v), Dev(n=sq * heads * 128)
    ok = iris.lib().iris_gpu_attention_fused_bf16(O.h, Q.h, K.h, V.h, sq, sk, heads, 128,
                                                  1.0 / np.sqrt(128.0))
    assert ok, iris.last_error()
    assert iris.lib().iris_cuda_synchronize() == 0, iris.last_error()  # no device wait ran out
    got = O.read((sq, heads * 128))
    assert np.isfinite(got).all()
    ref = fo.attention(q, k, v, heads)
    assert rel_l2(got, ref) < 1e-2


@pytest.mark.parametrize("seq,hidden", [(24, 256), (1536, 3072), (97, 512), (13, 4096), (9, 3072)])
def test_adaln(iris, seq, hidden):
    rng = np.random.default_rng(seq)
    x = bf16_round(rng.standard_normal((seq, hidden)) * 3 + 0.5)
    sh = bf16_round(rng.standard_normal(hidden) * 0.1)
    sc = bf16_round(rng.standard_normal(hidden) * 0.1)
    X, SH, SC, O = Dev(x), Dev(sh), Dev(sc), Dev(n=seq * hidden)
    iris.lib().iris_gpu_adaln_norm_bf16(O.h, X.h, SH.h, SC.h, seq, hidden, 1e-6)
    assert rel_l2(O.read((seq, hidden)), fo.adaln(x, sh, sc)) < 1e-2


def test_qk_norm_and_rope(iris):
    seq, heads, img_off = 40, 3, 8
    rng = np.random.default_rng(3)
    q = bf16_round(rng.standard_normal((seq, heads * 128)))
    k = bf16_round(rng.standard_normal((seq, heads * 128)) * 2)
    wq = bf16_round(1 + 0.1 * rng.standard_normal(128))
    wk = bf16_round(1 + 0.1 * rng.standard_normal(128))
    Q, K, WQ, WK = Dev(q), Dev(k), Dev(wq), Dev(wk)
    iris.lib().iris_gpu_qk_rms_norm_bf16(Q.h, K.h, WQ.h, WK.h, seq, heads, 128, 1e-6)
    qn = fo.head_rms_norm(q, wq, heads)
    kn = fo.head_rms_norm(k, wk, heads)
    assert rel_l2(Q.read((seq, heads * 128)), qn) < 1e-2
    assert rel_l2(K.read((seq, heads * 128)), kn) < 1e-2
    # unified RoPE: text rows [0, img_off) use the L axis, image rows H/W
    tc, ts = fo.rope_txt(img_off, 2000.0)
    ic, isn = fo.rope_img(4, 8, 2000.0)
    tc, ts, ic, isn = (np.ascontiguousarray(a, np.float32) for a in (tc, ts, ic, isn))
    iris.lib().iris_gpu_rope_unified_bf16(Q.h, K.h, tc.ctypes.data_as(_fp), ts.ctypes.data_as(_fp),
                                          ic.ctypes.data_as(_fp), isn.ctypes.data_as(_fp), None, None,
                                          seq, img_off, heads, 128, 32)
    cs = np.concatenate([tc, ic]), np.concatenate([ts, isn])
    assert rel_l2(Q.read((seq, heads * 128)), fo.apply_rope(bf16_round(qn), *cs, heads)) < 1e-2
    assert rel_l2(K.read((seq, heads * 128)), fo.apply_rope(bf16_round(kn), *cs, heads)) < 1e-2


def test_silu_mul_gated_add_and_layout_ops(iris):
    rng = np.random.default_rng(9)
    seq, hid, mlp = 10, 256, 384
    g = bf16_round(rng.standard_normal((seq, mlp)))
    u = bf16_round(rng.standard_normal((seq, mlp)))
    G, U = Dev(g), Dev(u)
    iris.lib().iris_gpu_silu_mul_bf16(G.h, U.h, seq * mlp)
    assert rel_l2(G.read((seq, mlp)), fo.silu(g) * u) < 1e-2
    out = bf16_round(rng.standard_normal((seq, hid)))
    gate = bf16_round(rng.standard_normal(hid))
    proj = bf16_round(rng.standard_normal((seq, hid)))
    OUT, GATE, PROJ = Dev(out), Dev(gate), Dev(proj)
    iris.lib().iris_gpu_gated_add_bf16(OUT.h, GATE.h, PROJ.h, seq, hid)
    assert rel_l2(OUT.read((seq, hid)), out + gate * proj) < 1e-2
    # split [Q,K,V,gate,up] and concat [attn, mlp] are exact copies
    fused = bf16_round(rng.standard_normal((seq, 3 * hid + 2 * mlp)))
    F_ = Dev(fused)
    parts = [Dev(n=seq * hid) for _ in range(3)] + [Dev(n=seq * mlp) for _ in range(2)]
    iris.lib().iris_gpu_split_qkv_mlp_bf16(F_.h, *[p.h for p in parts], seq, hid, mlp)
    offs = [0, hid, 2 * hid, 3 * hid, 3 * hid + mlp, 3 * hid + 2 * mlp]
    for i, p in enumerate(parts):
        np.testing.assert_array_equal(p.read((seq, offs[i + 1] - offs[i])), fused[:, offs[i]:offs[i + 1]])
    cat = Dev(n=seq * (hid + mlp))
    iris.lib().iris_gpu_concat_attn_mlp_bf16(parts[0].h, parts[3].h, cat.h, seq, hid, mlp)
    np.testing.assert_array_equal(cat.read((seq, hid + mlp)),
                                  np.concatenate([fused[:, :hid], fused[:, 3 * hid:3 * hid + mlp]], 1))
    a = bf16_round(rng.standard_normal((3, hid)))
    b = bf16_round(rng.standard_normal((5, hid)))
    A, B, AB = Dev(a), Dev(b), Dev(n=8 * hid)
    iris.lib().iris_gpu_concat_seq_bf16(AB.h, A.h, B.h, 3, 5, hid)
    np.testing.assert_array_equal(AB.read((8, hid)), np.concatenate([a, b]))
    S = Dev(n=4 * hid)
    iris.lib().iris_gpu_slice_seq_bf16(S.h, AB.h, 4, hid, 2)
    np.testing.assert_array_equal(S.read((4, hid)), np.concatenate([a, b])[2:6])


def _masked_ref(q, k, v, heads, group, keep, causal, scale):
    """fp32 causal / key-masked grouped-query attention: masked scores are
    -1e9 (the reference encoder's value), so a row with no kept key averages
    every value row."""
    import torch
    S, Sk = q.shape[0], k.shape[0]
    qh = q.float().view(S, heads, 128).transpose(0, 1)
    kh = k.float().view(Sk, heads // group, 128).transpose(0, 1).repeat_interleave(group, 0)
    vh = v.float().view(Sk, heads // group, 128).transpose(0, 1).repeat_interleave(group, 0)
    s = qh @ kh.transpose(1, 2) * scale
    dead = ~keep.bool()[None, None, :].expand(1, S, Sk)
    if causal:
        i = torch.arange(S, device=q.device)
        dead = dead | (i[None, None, :] > i[None, :, None])
    s = s.masked_fill(dead, -1e9)
    return (torch.softmax(s, -1) @ vh).transpose(0, 1).reshape(S, heads * 128)


@pytest.mark.parametrize("S,heads,group", [(512, 32, 4), (2560, 16, 2), (96, 8, 4), (128, 4, 1)])
@pytest.mark.parametrize("mask", ["right", "left", "holes", "none_kept", "all_kept"])
@pytest.mark.parametrize("causal", [1, 0])
def test_masked_attention_key_tile_bound(iris, S, heads, group, mask, causal):
    """iris_launch_attention_gqa with a key mask and / or the causal mask: CTAs
    stop after the last key tile any of their rows can use (the last kept key,
    and under the causal mask their last row), except where a row keeps no key
    and averages all of them.  512 rows x 32 heads runs one query tile per
    CTA, 2560 x 16 the CTA pairs, 96 and 128 rows the short-sequence kernel
    (f32 on the FMA pipe); fp32 reference, relative L2 <= 1e-2."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(S + heads + causal)
    kvh = heads // group
    q = torch.randn(S, heads * 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(S, kvh * 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(S, kvh * 128, device="cuda", generator=g).bfloat16()
    keep = torch.zeros(S, dtype=torch.uint8, device="cuda")
    if mask == "right":
        keep[:77] = 1
    elif mask == "left":
        keep[300:] = 1
    elif mask == "holes":
        keep[5:40] = 1
        keep[200:260] = 1
    elif mask == "all_kept":
        keep[:] = 1
    o = torch.empty_like(q)
    scale = 1.0 / np.sqrt(128.0)
    st = torch.cuda.current_stream().cuda_stream
    rc = iris.lib().iris_launch_attention_gqa(
        C.c_void_p(q.data_ptr()), heads * 128, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), kvh * 128,
        C.c_void_p(o.data_ptr()), heads * 128, S, S, heads, group, causal, C.c_float(scale),
        C.c_void_p(keep.data_ptr()), C.c_void_p(st))
    assert rc == 0
    torch.cuda.synchronize()
    assert iris.lib().iris_cuda_device_status(0) == 0
    ref = _masked_ref(q, k, v, heads, group, keep, causal, scale)
    err = float((o.float() - ref).norm() / ref.norm())
    assert err < 1e-2, err


# ---------------------------------------------------------------- f32 surface
def test_f32_norms_rope_and_gated_add(iris):
    """The f32 ops the reference's Z-Image GPU block and the f32 fallbacks of
    its Flux blocks call (iris_metal.h:353-398), with host-pointer weights and
    tables, against the oracle.  f32 in and out: tolerance 1e-5 except where
    noted."""
    L = iris.lib()
    seq, heads, H = 40, 3, 384
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((seq, H)) * 2 + 0.3).astype(np.float32)
    sh, sc, g, w = (rng.standard_normal(H).astype(np.float32) * 0.1 for _ in range(4))
    X, O = Dev(x, bf16=False), Dev(n=seq * H, bf16=False)
    L.iris_gpu_adaln_norm(O.h, X.h, sh.ctypes.data_as(_fp), sc.ctypes.data_as(_fp), seq, H, 1e-6)
    assert rel_l2(O.read((seq, H)), fo.adaln(x, sh, sc)) < 1e-5
    L.iris_gpu_rms_norm_f32(O.h, X.h, w.ctypes.data_as(_fp), seq, H, 1e-5)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-5) * w
    assert rel_l2(O.read((seq, H)), ref) < 1e-5
    # out += gate * proj, gate a host vector
    L.iris_gpu_gated_add(O.h, g.ctypes.data_as(_fp), X.h, seq, H)
    assert rel_l2(O.read((seq, H)), ref + g * x) < 1e-5
    # per-head RMSNorm of q and k, then the unified (text | image) RoPE in f32
    q = rng.standard_normal((seq, heads * 128)).astype(np.float32)
    k = rng.standard_normal((seq, heads * 128)).astype(np.float32)
    wq = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    wk = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    Q, K = Dev(q, bf16=False), Dev(k, bf16=False)
    L.iris_gpu_qk_rms_norm(Q.h, K.h, wq.ctypes.data_as(_fp), wk.ctypes.data_as(_fp), seq, heads, 128, 1e-6)
    qn, kn = fo.head_rms_norm(q, wq, heads), fo.head_rms_norm(k, wk, heads)
    assert rel_l2(Q.read((seq, heads * 128)), qn) < 1e-5
    img_off = 8
    tc, ts = (np.ascontiguousarray(a, np.float32) for a in fo.rope_txt(img_off, 2000.0))
    ic, isn = (np.ascontiguousarray(a, np.float32) for a in fo.rope_img(4, 8, 2000.0))
    L.iris_metal_rope_cache_begin()
    L.iris_gpu_rope_unified(Q.h, K.h, tc.ctypes.data_as(_fp), ts.ctypes.data_as(_fp), ic.ctypes.data_as(_fp),
                            isn.ctypes.data_as(_fp), seq, img_off, heads, 128, 32)
    cs = np.concatenate([tc, ic]), np.concatenate([ts, isn])
    assert rel_l2(Q.read((seq, heads * 128)), fo.apply_rope(qn, *cs, heads)) < 1e-5
    assert rel_l2(K.read((seq, heads * 128)), fo.apply_rope(kn, *cs, heads)) < 1e-5
    # one table for all rows, applied to q and k (Z-Image)
    c2, s2 = (np.ascontiguousarray(a) for a in cs)
    L.iris_metal_rope_cache_begin()
    L.iris_gpu_rope_single_pair_f32(Q.h, K.h, c2.ctypes.data_as(_fp), s2.ctypes.data_as(_fp), seq, heads, 128)
    q2 = fo.apply_rope(fo.apply_rope(qn, *cs, heads), *cs, heads)
    assert rel_l2(Q.read((seq, heads * 128)), q2) < 1e-5
    L.iris_metal_rope_cache_begin()


def test_f32_attention_and_host_attention(iris):
    """f32-interface attention (bf16 compute, so bf16 tolerance) on device
    tensors and on host pointers in both layouts (iris_metal.h:402, :613, :649)."""
    L = iris.lib()
    sq, sk, heads = 70, 150, 2
    rng = np.random.default_rng(5)
    q = rng.standard_normal((sq, heads * 128)).astype(np.float32)
    k = rng.standard_normal((sk, heads * 128)).astype(np.float32)
    v = rng.standard_normal((sk, heads * 128)).astype(np.float32)
    ref = fo.attention(q, k, v, heads)
    Q, K, V = Dev(q, bf16=False), Dev(k, bf16=False), Dev(v, bf16=False)
    O = Dev(n=sq * heads * 128, bf16=False)
    scale = 1.0 / np.sqrt(128.0)
    assert L.iris_gpu_attention_fused(O.h, Q.h, K.h, V.h, sq, sk, heads, 128, scale), iris.last_error()
    assert rel_l2(O.read((sq, heads * 128)), ref) < 1e-2
    out = np.zeros_like(q)
    assert L.iris_metal_attention_fused(out.ctypes.data_as(_fp), q.ctypes.data_as(_fp), k.ctypes.data_as(_fp),
                                        v.ctypes.data_as(_fp), sq, sk, heads, 128, scale)
    assert rel_l2(out, ref) < 1e-2
    # [heads, seq, 128] layout
    qt, kt, vt = (np.ascontiguousarray(a.reshape(-1, heads, 128).transpose(1, 0, 2)) for a in (q, k, v))
    ot = np.zeros_like(qt)
    L.iris_metal_attention(ot.ctypes.data_as(_fp), qt.ctypes.data_as(_fp), kt.ctypes.data_as(_fp),
                           vt.ctypes.data_as(_fp), None, heads, sq, sk, 128, scale)
    assert rel_l2(ot.transpose(1, 0, 2).reshape(sq, heads * 128), ref) < 1e-2
    # the SREF key bias is refused (the caller then takes its CPU path)
    L.iris_metal_set_attention_bias(sk - 10, 0.5)
    assert L.iris_gpu_attention_fused(O.h, Q.h, K.h, V.h, sq, sk, heads, 128, scale) == 0
    assert "key bias" in iris.last_error()
    L.iris_metal_set_attention_bias(0, 0.0)


def test_tensor_data_host_view_round_trip(iris):
    """iris_gpu_tensor_data (iris_metal.h:208): the host view shows the GPU
    result; host writes reach the next op that uses the tensor."""
    L = iris.lib()
    n = 1000
    a = np.arange(n, dtype=np.float32)
    A, B, O = Dev(a, bf16=False), Dev(np.ones(n, np.float32), bf16=False), Dev(n=n, bf16=False)
    L.iris_gpu_add_f32(O.h, A.h, B.h, n)
    p = L.iris_gpu_tensor_data(O.h)
    view = np.ctypeslib.as_array(p, shape=(n,))
    np.testing.assert_array_equal(view, a + 1)
    view[:10] = -5.0                      # host write through the view
    L.iris_gpu_add_f32(O.h, O.h, B.h, n)  # the next op sees it
    got = O.read()
    np.testing.assert_array_equal(got[:10], -4.0)
    np.testing.assert_array_equal(got[10:], a[10:] + 2)
    # bf16 tensors get an f32 view
    Hb = Dev(a)
    vb = np.ctypeslib.as_array(L.iris_gpu_tensor_data(Hb.h), shape=(n,))
    np.testing.assert_array_equal(vb, bf16_round(a))
