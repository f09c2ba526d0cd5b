"""CPU restatement of the reference Z-Image (S3-DiT) forward — TEST INFRASTRUCTURE ONLY.

numpy float32, one function per reference function (iris_transformer_zimage.c
file:line cited).  Pinned to the reference build by tests/test_oracle_golden.py
(tests/golden/zimage_*.npz).  Imported only by tests, smoke and bench legs.

Sequence layout: [IMG (padded to 32) | CAP (padded to 32)] (:1905-1907).
"""
from __future__ import annotations

import numpy as np

from .flux_oracle import attention, linear, silu, timestep_embedding

F32 = np.float32
SEQ_MULTI = 32       # ZI_SEQ_MULTI_OF (:41)
NORM_EPS = 1e-5      # ZI_NORM_EPS (:42)


def zi_dims(cfg: dict, w: dict) -> dict:
    """Derived sizes (zi_transformer_load_safetensors :2164-2290): ffn and t-MLP
    widths come from the weight shapes, adaln_dim = min(dim, 256)."""
    dim = cfg["dim"]
    ffn_key = next((k for k in w if k.endswith("feed_forward.w1.weight")), None)
    return dict(dim=dim, heads=dim // 128, ffn=w[ffn_key].shape[0] if ffn_key else cfg.get("ffn_dim"),
                adaln=min(dim, 256), ps=cfg["patch_size"], cin=cfg["in_channels"],
                theta=float(cfg["rope_theta"]), axes=list(cfg["axes_dims"]),
                n_layers=cfg["n_layers"], n_refiner=cfg["n_refiner"])


def rms_norm(x, w, eps=NORM_EPS):
    """x * rsqrt(mean(x^2) + eps) * w (zi_rms_norm :657-669)."""
    x = x.astype(F32)
    r = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True, dtype=F32) + F32(eps))
    return (x * r * w.astype(F32)).astype(F32)


def t_embed(w, t):
    """Linear(256->mid)+b, SiLU, Linear(mid->adaln)+b on sincos(1000 t) (zi_timestep_embed :563-585)."""
    s = timestep_embedding(F32(t) * F32(1000.0))[None]
    h = silu(linear(s, w["t_embedder.mlp.0.weight"]) + w["t_embedder.mlp.0.bias"])
    return (linear(h, w["t_embedder.mlp.2.weight"]) + w["t_embedder.mlp.2.bias"])[0]


def rope_tables(pos, theta, axes):
    """Per-token cos/sin [S, 64] for the 3 axes (T 32, H 48, W 48 dims) with
    freq_i = 1/theta^(2i/d) (zi_precompute_rope :595-612); positions outside
    [0, 1024) leave that axis unrotated (zi_apply_rope :620-650)."""
    s = pos.shape[0]
    cs, sn = [], []
    for ax, d in enumerate(axes):
        half = d // 2
        i = np.arange(half, dtype=F32)
        freq = (1.0 / np.power(F32(theta), (2 * i).astype(F32) / F32(d))).astype(F32)
        p = pos[:, ax]
        ang = (p.astype(F32)[:, None] * freq[None, :]).astype(F32)
        c, sv = np.cos(ang).astype(F32), np.sin(ang).astype(F32)
        bad = (p < 0) | (p >= 1024)
        c[bad] = 1.0
        sv[bad] = 0.0
        cs.append(c)
        sn.append(sv)
    return np.concatenate(cs, 1), np.concatenate(sn, 1)


def apply_rope_pairs(x, cos, sin, heads):
    """Consecutive-pair rotation with one (cos, sin) per pair [S, 64]."""
    s = x.shape[0]
    xh = x.reshape(s, heads, 64, 2).astype(F32)
    c, sn = cos[:, None, :], sin[:, None, :]
    x0, x1 = xh[..., 0], xh[..., 1]
    return np.stack([x0 * c - x1 * sn, x1 * c + x0 * sn], -1).reshape(s, heads * 128).astype(F32)


def masked_attention(q, k, v, heads, mask):
    """softmax(QK^T/sqrt(d)) V with padding keys set to -1e9 (zi_attention :689-762)."""
    if mask is None or mask.all():
        return attention(q, k, v, heads)
    s = q.shape[0]
    qh = q.reshape(s, heads, 128).transpose(1, 0, 2)
    kh = k.reshape(-1, heads, 128).transpose(1, 0, 2)
    vh = v.reshape(-1, heads, 128).transpose(1, 0, 2)
    sc = (qh @ kh.transpose(0, 2, 1)) * F32(1.0 / np.sqrt(128.0))
    sc[:, :, ~mask] = F32(-1e9)
    sc = sc - sc.max(-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(-1, keepdims=True)
    return (p @ vh).transpose(1, 0, 2).reshape(s, heads * 128).astype(F32)


def block(w, prefix, x, rope, mask, t_emb, d, modulated):
    """One S3-DiT block (zi_block_forward :790-858; attention :689, FFN :764)."""
    D, heads = d["dim"], d["heads"]
    p = prefix + "."
    if modulated:
        mod = linear(t_emb[None], w[p + "adaLN_modulation.0.weight"])[0] + w[p + "adaLN_modulation.0.bias"]
        scale_msa, gate_msa = 1.0 + mod[:D], np.tanh(mod[D:2 * D])
        scale_mlp, gate_mlp = 1.0 + mod[2 * D:3 * D], np.tanh(mod[3 * D:])
    else:
        scale_msa = scale_mlp = np.ones(D, F32)
        gate_msa = gate_mlp = np.ones(D, F32)
    h = rms_norm(x, w[p + "attention_norm1.weight"]) * scale_msa
    q = linear(h, w[p + "attention.to_q.weight"])
    k = linear(h, w[p + "attention.to_k.weight"])
    v = linear(h, w[p + "attention.to_v.weight"])
    q = apply_rope_pairs(rms_norm(q.reshape(-1, 128), w[p + "attention.norm_q.weight"]).reshape(q.shape),
                         *rope, heads)
    k = apply_rope_pairs(rms_norm(k.reshape(-1, 128), w[p + "attention.norm_k.weight"]).reshape(k.shape),
                         *rope, heads)
    a = linear(masked_attention(q, k, v, heads, mask), w[p + "attention.to_out.0.weight"])
    x = x + gate_msa * rms_norm(a, w[p + "attention_norm2.weight"])
    h = rms_norm(x, w[p + "ffn_norm1.weight"]) * scale_mlp
    f = linear(silu(linear(h, w[p + "feed_forward.w1.weight"])) * linear(h, w[p + "feed_forward.w3.weight"]),
               w[p + "feed_forward.w2.weight"])
    x = x + gate_mlp * rms_norm(f, w[p + "ffn_norm2.weight"])
    return x.astype(F32)


def patchify(lat, ps):
    """[C, H, W] -> [n_patches, ps*ps*C] in (ph, pw, c) order (zi_patchify :1634-1660)."""
    c, H, W = lat.shape
    x = lat.reshape(c, H // ps, ps, W // ps, ps).transpose(1, 3, 2, 4, 0)
    return x.reshape((H // ps) * (W // ps), ps * ps * c).astype(F32)


def unpatchify(tok, c, H, W, ps):
    """Inverse of patchify (zi_unpatchify :1663-1690)."""
    x = tok.reshape(H // ps, W // ps, ps, ps, c).transpose(4, 0, 2, 1, 3)
    return x.reshape(c, H, W).astype(F32)


def forward(w, cfg, latent, cap, t, return_hidden=False):
    """Model output for one step (zi_transformer_forward :1696-1980)."""
    d = zi_dims(cfg, w)
    D, ps, cin = d["dim"], d["ps"], d["cin"]
    _, H, W = latent.shape
    ht, wt = H // ps, W // ps
    n_img, n_cap = ht * wt, cap.shape[0]
    img_pad = (SEQ_MULTI - n_img % SEQ_MULTI) % SEQ_MULTI
    cap_pad = (SEQ_MULTI - n_cap % SEQ_MULTI) % SEQ_MULTI
    ni, nc = n_img + img_pad, n_cap + cap_pad
    t_emb = t_embed(w, t)

    pt = patchify(latent, ps)
    pt = np.concatenate([pt, np.repeat(pt[-1:], img_pad, 0)])
    img = linear(pt, w[f"all_x_embedder.{ps}-1.weight"]) + w[f"all_x_embedder.{ps}-1.bias"]
    img[n_img:] = w["x_pad_token"].reshape(-1)
    cf = np.concatenate([cap, np.repeat(cap[-1:], cap_pad, 0)]).astype(F32)
    capx = linear(rms_norm(cf, w["cap_embedder.0.weight"]), w["cap_embedder.1.weight"]) + w["cap_embedder.1.bias"]
    capx[n_cap:] = w["cap_pad_token"].reshape(-1)

    img_pos = np.zeros((ni, 3), np.int64)
    yy, xx = np.meshgrid(np.arange(ht), np.arange(wt), indexing="ij")
    img_pos[:n_img, 0] = nc + 1
    img_pos[:n_img, 1] = yy.ravel()
    img_pos[:n_img, 2] = xx.ravel()
    cap_pos = np.zeros((nc, 3), np.int64)
    cap_pos[:, 0] = 1 + np.arange(nc)
    img_mask = np.arange(ni) < n_img
    cap_mask = np.arange(nc) < n_cap
    rope_i = rope_tables(img_pos, d["theta"], d["axes"])
    rope_c = rope_tables(cap_pos, d["theta"], d["axes"])

    for i in range(d["n_refiner"]):
        img = block(w, f"noise_refiner.{i}", img, rope_i, img_mask, t_emb, d, True)
    for i in range(d["n_refiner"]):
        capx = block(w, f"context_refiner.{i}", capx, rope_c, cap_mask, None, d, False)
    x = np.concatenate([img, capx])
    rope_u = (np.concatenate([rope_i[0], rope_c[0]]), np.concatenate([rope_i[1], rope_c[1]]))
    mask_u = np.concatenate([img_mask, cap_mask])
    for i in range(d["n_layers"]):
        x = block(w, f"layers.{i}", x, rope_u, mask_u, t_emb, d, True)

    # final layer: LayerNorm (eps 1e-6, no affine) * (1 + W SiLU(t_emb) + b), linear + bias (:1581-1630)
    fp = f"all_final_layer.{ps}-1."
    scale = 1.0 + linear(silu(t_emb)[None], w[fp + "adaLN_modulation.1.weight"])[0] + w[fp + "adaLN_modulation.1.bias"]
    xi = x[:n_img]
    mean = xi.mean(-1, keepdims=True, dtype=F32)
    var = ((xi - mean) ** 2).mean(-1, keepdims=True, dtype=F32)
    xn = (xi - mean) / np.sqrt(var + F32(1e-6)) * scale
    out = linear(xn, w[fp + "linear.weight"]) + w[fp + "linear.bias"]
    v = unpatchify(out, cin, H, W, ps)
    return (v, x) if return_hidden else v


def sample_euler(w, cfg, z, cap, schedule):
    """z <- z + (s_{n+1} - s_n) * (-model(z, 1 - s_n)) (iris_sample_euler_zimage, iris_sample.c:412-480)."""
    z = z.astype(F32).copy()
    for n in range(len(schedule) - 1):
        out = forward(w, cfg, z, cap, float(F32(1.0) - F32(schedule[n])))
        z = (z + F32(schedule[n + 1] - schedule[n]) * (-out)).astype(F32)
    return z
