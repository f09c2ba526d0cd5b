"""CPU restatement of the reference Flux.2 Klein DiT forward — TEST INFRASTRUCTURE ONLY.

This is the oracle the CUDA backend is checked against.  It restates, in
numpy float32, the reference's CPU path (``make blas`` / ``make generic``)
function by function; each function names the reference file:line it
follows.  It is pinned against the reference itself: tests/golden/ holds
outputs of the reference compiled from its own sources (oracle/Makefile,
oracle/ref_harness.c) and tests/test_oracle_golden.py checks this module
against them.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module.  The product path never does.

Layout conventions (same as the reference):
* latents are NCHW f32 [C, h, w]; tokens are NLC rows, row = y*w + x
  (iris_transformer_flux.c:3986-3993);
* hidden states are [S, H] row-major, heads interleaved [S, heads*128];
* the joint sequence order is [TXT, IMG] (:1899-1905, :4110-4114).
"""
from __future__ import annotations

import numpy as np

from .model_gen import flux_dims

F32 = np.float32


def silu(x):
    """x * sigmoid(x) (iris_kernels.c:610-638)."""
    x = x.astype(F32)
    return (x / (1.0 + np.exp(-x))).astype(F32)


def linear(x, w):
    """y = x @ W^T, no bias (iris_linear_nobias, iris_kernels.c:220-265)."""
    return (x.astype(F32) @ w.astype(F32).T).astype(F32)


def timestep_embedding(t, dim=256, max_period=10000.0):
    """[cos(t*f), sin(t*f)], f = exp(-ln(max_period)*i/half)
    (get_timestep_embedding, iris_transformer_flux.c:1349-1363)."""
    half = dim // 2
    i = np.arange(half, dtype=F32)
    freq = np.exp(-np.log(F32(max_period)) * i / F32(half)).astype(F32)
    ang = (F32(t) * freq).astype(F32)
    return np.concatenate([np.cos(ang), np.sin(ang)]).astype(F32)


def time_embed(w, t):
    """fc2(SiLU(fc1(sincos(1000 t)))) (time_embed_forward :1366-1382; called at :3962-3967)."""
    s = timestep_embedding(F32(t) * F32(1000.0))
    h = silu(linear(s[None], w["time_guidance_embed.timestep_embedder.linear_1.weight"]))
    return linear(h, w["time_guidance_embed.timestep_embedder.linear_2.weight"])[0]


def modulations(w, t_emb):
    """All per-step modulation vectors from SiLU(t_emb):
    double img/txt 6H (:4055-4069), single 3H (:3787-3797), final 2H (:4270-4281)."""
    s = silu(t_emb)[None]
    return dict(dbl_img=linear(s, w["double_stream_modulation_img.linear.weight"])[0],
                dbl_txt=linear(s, w["double_stream_modulation_txt.linear.weight"])[0],
                single=linear(s, w["single_stream_modulation.linear.weight"])[0],
                final=linear(s, w["norm_out.linear.weight"])[0])


def adaln(x, shift, scale, eps=1e-6):
    """LayerNorm without affine, then (1+scale)*xhat + shift (apply_adaln :1391-1460)."""
    x = x.astype(F32)
    mean = x.mean(axis=-1, keepdims=True, dtype=F32)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True, dtype=F32)
    xn = (x - mean) / np.sqrt(var + F32(eps))
    return ((F32(1.0) + scale) * xn + shift).astype(F32)


def head_rms_norm(x, weight, heads, eps=1e-6):
    """Per-head RMSNorm x*rsqrt(mean(x^2)+eps)*w over 128-dim heads (apply_qk_norm :1464-1518)."""
    s, hd = x.shape[0], x.shape[1] // heads
    xh = x.reshape(s, heads, hd).astype(F32)
    r = 1.0 / np.sqrt((xh * xh).mean(axis=-1, keepdims=True, dtype=F32) + F32(eps))
    return (xh * r * weight.astype(F32)).reshape(s, heads * hd).astype(F32)


def rope_base_freqs(theta, axis_dim=32):
    """1/theta^(2d/axis_dim), d < axis_dim/2 (compute_rope_2d :903-906)."""
    d = np.arange(axis_dim // 2, dtype=F32)
    return (1.0 / np.power(F32(theta), (2 * d).astype(F32) / F32(axis_dim))).astype(F32)


def rope_table(pos_t, pos_h, pos_w, pos_l, theta, axis_dim=32):
    """Per-token cos/sin [S, 4*axis_dim] for the 4 RoPE axes (T, H, W, L), each pair
    entry duplicated (compute_rope_2d :897, compute_rope_2d_with_t_offset :961,
    compute_rope_text :1055).  Position 0 on an axis gives the identity rotation."""
    f = rope_base_freqs(theta, axis_dim)
    cos_parts, sin_parts = [], []
    for p in (pos_t, pos_h, pos_w, pos_l):
        ang = (np.asarray(p, dtype=F32)[:, None] * f[None, :]).astype(F32)
        c, s = np.cos(ang), np.sin(ang)
        cos_parts.append(np.repeat(c, 2, axis=1))
        sin_parts.append(np.repeat(s, 2, axis=1))
    return np.concatenate(cos_parts, 1).astype(F32), np.concatenate(sin_parts, 1).astype(F32)


def rope_img(ph, pw, theta, t_offset=0):
    """Image tokens: T = t_offset, H = row, W = col, L = 0 (:897, :961)."""
    yy, xx = np.meshgrid(np.arange(ph), np.arange(pw), indexing="ij")
    n = ph * pw
    return rope_table(np.full(n, t_offset), yy.ravel(), xx.ravel(), np.zeros(n), theta)


def rope_txt(n, theta):
    """Text tokens: L = index, other axes 0 (compute_rope_text :1055-1084)."""
    z = np.zeros(n)
    return rope_table(z, z, z, np.arange(n), theta)


def apply_rope(x, cos, sin, heads):
    """Consecutive-pair rotation (x0 c - x1 s, x1 c + x0 s) (apply_rope_2d :1026-1048)."""
    s, hd = x.shape[0], x.shape[1] // heads
    xh = x.reshape(s, heads, hd // 2, 2).astype(F32)
    c = cos.reshape(s, 1, hd // 2, 2)[..., 0]
    sn = sin.reshape(s, 1, hd // 2, 2)[..., 0]
    x0, x1 = xh[..., 0], xh[..., 1]
    out = np.stack([x0 * c - x1 * sn, x1 * c + x0 * sn], axis=-1)
    return out.reshape(s, heads * hd).astype(F32)


def attention(q, k, v, heads):
    """softmax(Q K^T / sqrt(d)) V per head, [S, heads*d] layout
    (mha_forward :1789-1881, joint_attention :1886-2022)."""
    sq, hd = q.shape[0], q.shape[1] // heads
    sk = k.shape[0]
    qh = q.reshape(sq, heads, hd).transpose(1, 0, 2).astype(F32)
    kh = k.reshape(sk, heads, hd).transpose(1, 0, 2).astype(F32)
    vh = v.reshape(sk, heads, hd).transpose(1, 0, 2).astype(F32)
    sc = (qh @ kh.transpose(0, 2, 1)) * F32(1.0 / np.sqrt(hd))
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    o = (p.astype(F32) @ vh).transpose(1, 0, 2).reshape(sq, heads * hd)
    return o.astype(F32)


def swiglu(x, w_in, w_out, mlp):
    """down(SiLU(gate) * up) with linear_in = [gate; up] rows (:633-640, swiglu_ffn_bf16 :2299)."""
    gu = linear(x, w_in)
    return linear(silu(gu[:, :mlp]) * gu[:, mlp:], w_out)


def _ip_add(ip, blk, q_pre, rows):
    """IP-Adapter contribution after block blk (ip_inject_block :2355): rows +=
    s * SDPA(pre-RoPE image Q, k_ip, v_ip) (oracle/ip_oracle.py)."""
    from oracle import ip_oracle
    k, v = ip["kv"][blk]
    return ip_oracle.inject(ip["adapter"], blk, q_pre, k, v, rows)


def double_block(w, i, img, txt, mod_img, mod_txt, rope_i, rope_t, d, ip=None):
    """One MM-DiT double block (double_block_forward :2366-2614). Returns new (img, txt).
    ``ip``: an ip_oracle.ip_context; its contribution goes to the image rows
    after the block, from the post-QK-norm, pre-RoPE image Q (:2440-2446, :2607-2612)."""
    H, heads, F = d["hidden"], d["heads"], d["mlp"]
    p = f"transformer_blocks.{i}."
    mi = [mod_img[j * H:(j + 1) * H] for j in range(6)]
    mt = [mod_txt[j * H:(j + 1) * H] for j in range(6)]

    xi = adaln(img, mi[0], mi[1])
    qi = linear(xi, w[p + "attn.to_q.weight"])
    ki = linear(xi, w[p + "attn.to_k.weight"])
    vi = linear(xi, w[p + "attn.to_v.weight"])
    qi = head_rms_norm(qi, w[p + "attn.norm_q.weight"], heads)
    qi_pre = qi
    qi = apply_rope(qi, *rope_i, heads)
    ki = apply_rope(head_rms_norm(ki, w[p + "attn.norm_k.weight"], heads), *rope_i, heads)

    xt = adaln(txt, mt[0], mt[1])
    qt = linear(xt, w[p + "attn.add_q_proj.weight"])
    kt = linear(xt, w[p + "attn.add_k_proj.weight"])
    vt = linear(xt, w[p + "attn.add_v_proj.weight"])
    qt = apply_rope(head_rms_norm(qt, w[p + "attn.norm_added_q.weight"], heads), *rope_t, heads)
    kt = apply_rope(head_rms_norm(kt, w[p + "attn.norm_added_k.weight"], heads), *rope_t, heads)

    k = np.concatenate([kt, ki])
    v = np.concatenate([vt, vi])
    ai = attention(qi, k, v, heads)
    at = attention(qt, k, v, heads)

    img = img + mi[2] * linear(ai, w[p + "attn.to_out.0.weight"])
    txt = txt + mt[2] * linear(at, w[p + "attn.to_add_out.weight"])
    img = img + mi[5] * swiglu(adaln(img, mi[3], mi[4]), w[p + "ff.linear_in.weight"],
                               w[p + "ff.linear_out.weight"], F)
    txt = txt + mt[5] * swiglu(adaln(txt, mt[3], mt[4]), w[p + "ff_context.linear_in.weight"],
                               w[p + "ff_context.linear_out.weight"], F)
    img = img.astype(F32)
    if ip is not None:
        img = _ip_add(ip, i, qi_pre, img)
    return img, txt.astype(F32)


def single_block(w, i, hidden, mod_single, rope_all, d, ip=None, n_txt=0, rope_k=None):
    """One parallel DiT block over [TXT, IMG] (single_block_forward :3761-3928).
    ``ip``: contribution to the rows after the n_txt text rows, adapter block
    n_double + i (:3848-3855, :3921-3926)."""
    H, heads, F = d["hidden"], d["heads"], d["mlp"]
    p = f"single_transformer_blocks.{i}."
    shift, scale, gate = (mod_single[j * H:(j + 1) * H] for j in range(3))
    x = adaln(hidden, shift, scale)
    fused = linear(x, w[p + "attn.to_qkv_mlp_proj.weight"])
    q, k, v = fused[:, :H], fused[:, H:2 * H], fused[:, 2 * H:3 * H]
    g, u = fused[:, 3 * H:3 * H + F], fused[:, 3 * H + F:]
    q = head_rms_norm(q, w[p + "attn.norm_q.weight"], heads)
    q_pre = q
    q = apply_rope(q, *rope_all, heads)
    # SREF band control: K of reference rows rotated with the band-scaled table (:3872)
    k = apply_rope(head_rms_norm(k, w[p + "attn.norm_k.weight"], heads), *(rope_k or rope_all), heads)
    a = attention(q, k, v, heads)
    cat = np.concatenate([a, silu(g) * u], axis=1)
    out = (hidden + gate * linear(cat, w[p + "attn.to_out.weight"])).astype(F32)
    if ip is not None:
        out[n_txt:] = _ip_add(ip, d["n_double"] + i, q_pre[n_txt:], out[n_txt:])
    return out


def sref_band_table(cos, sin, ref_start, shf, slf, axis_dim=32):
    """band_scale_ref_krope (:1272): rows >= ref_start get their H and W pairs
    scaled by s(d) = shf + (slf - shf) (d / (half - 1))^2."""
    half = axis_dim // 2
    dn = np.arange(half, dtype=F32) / F32(half - 1)
    sd = (F32(shf) + (F32(slf) - F32(shf)) * dn * dn).astype(F32)
    f = np.repeat(sd, 2)
    c, s = cos.copy(), sin.copy()
    for a in (1, 2):
        c[ref_start:, a * axis_dim:(a + 1) * axis_dim] *= f
        s[ref_start:, a * axis_dim:(a + 1) * axis_dim] *= f
    return c, s


def csd_mod_forward(m, csd):
    """csd_mod_forward (iris_csdmod.c): fc2(SiLU(fc1(csd)))."""
    h = m["fc1.weight"].astype(np.float64) @ csd.astype(np.float64) + m["fc1.bias"]
    h = h / (1.0 + np.exp(-h))
    return (m["fc2.weight"].astype(np.float64) @ h + m["fc2.bias"]).astype(F32)


def forward(w, cfg, latent, txt_emb, t, refs=(), return_blocks=False, ip=None, temb_delta=None, bands=None):
    """Velocity v(z, t, ctx) for one denoising step.

    iris_transformer_forward (:3939-4326); with ``refs`` (list of NCHW
    reference latents, T offsets 10*(i+1)) it follows
    iris_transformer_forward_with_multi_refs (:4579-4840): reference tokens
    are appended to the image stream with their own RoPE T coordinate and only
    the target rows reach the final layer.
    """
    d = flux_dims(cfg)
    H, C = d["hidden"], d["channels"]
    c, h, wd = latent.shape
    n_img = h * wd
    toks = [latent.reshape(C, n_img).T]
    ropes = [rope_img(h, wd, d["theta"])]
    for r_i, r in enumerate(refs):
        toks.append(r.reshape(C, -1).T)
        ropes.append(rope_img(r.shape[1], r.shape[2], d["theta"], t_offset=10 * (r_i + 1)))
    img_tok = np.concatenate(toks).astype(F32)
    rope_i = (np.concatenate([r[0] for r in ropes]), np.concatenate([r[1] for r in ropes]))
    n_txt = txt_emb.shape[0]
    rope_t = rope_txt(n_txt, d["theta"])

    t_emb = time_embed(w, t)
    if temb_delta is not None:  # SREF CSD modulation (:3972)
        t_emb = (t_emb + temb_delta).astype(F32)
    mods = modulations(w, t_emb)
    img = linear(img_tok, w["x_embedder.weight"])
    txt = linear(txt_emb.astype(F32), w["context_embedder.weight"])
    blocks = []
    for i in range(d["n_double"]):
        img, txt = double_block(w, i, img, txt, mods["dbl_img"], mods["dbl_txt"], rope_i, rope_t, d, ip)
        if return_blocks:
            blocks.append(np.concatenate([txt, img]))
    hidden = np.concatenate([txt, img])
    rope_all = (np.concatenate([rope_t[0], rope_i[0]]), np.concatenate([rope_t[1], rope_i[1]]))
    rope_k = None
    if bands is not None and refs and (bands[0] != 1.0 or bands[1] != 1.0):
        rope_k = sref_band_table(*rope_all, n_txt + n_img, *bands)
    for i in range(d["n_single"]):
        hidden = single_block(w, i, hidden, mods["single"], rope_all, d, ip, n_txt, rope_k)
        if return_blocks:
            blocks.append(hidden)
    img = hidden[n_txt:n_txt + n_img]
    scale, shift = mods["final"][:H], mods["final"][H:]
    out = linear(adaln(img, shift, scale), w["proj_out.weight"])
    v = out.T.reshape(C, h, wd).astype(F32)
    return (v, blocks) if return_blocks else v


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
