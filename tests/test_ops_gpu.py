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


@pytest.mark.parametrize("sq,sk,heads", [(16, 80, 2), (80, 80, 2), (200, 333, 3), (1536, 1536, 4),
                                         (1, 64, 1), (130, 1, 1)])
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


@pytest.mark.parametrize("S,heads,group", [(512, 32, 4), (2560, 16, 2)])
@pytest.mark.parametrize("mask", ["right", "left", "holes", "none_kept", "all_kept"])
@pytest.mark.parametrize("causal", [1, 0])
def test_masked_attention_key_tile_bound(iris, S, heads, group, mask, causal):
    """iris_launch_attention_gqa with a key mask and / or the causal mask: CTAs
    stop after the last key tile any of their rows can use (the last kept key,
    and under the causal mask their last row), except where a row keeps no key
    and averages all of them.  512 rows x 32 heads runs one query tile per
    CTA, 2560 x 16 the CTA pairs; fp32 reference, relative L2 <= 1e-2."""
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
