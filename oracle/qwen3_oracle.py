"""CPU restatement of the reference Qwen3 text encoder — TEST INFRASTRUCTURE ONLY.

The oracle the CUDA text encoder is checked against: numpy float32, one
function per reference function (iris_qwen3.c), pinned against the reference
itself compiled from its own sources (tests/test_qwen3_oracle.py,
ref_qwen3_forward in oracle/ref_harness.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module.  The product path never does.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
EPS = 1e-6                 # QWEN3_RMS_NORM_EPS (iris_qwen3.h)
FLUX_LAYERS = (8, 17, 26)  # QWEN3_OUTPUT_LAYER_1..3 (iris_qwen3.h)


def rms_norm(x, w, eps=EPS):
    """x / sqrt(mean(x^2) + eps) * w per row (qwen3_rms_norm, iris_qwen3.c:191)."""
    x = x.astype(F32)
    r = (1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + eps)).astype(F32)
    return (x * r * w).astype(F32)


def rope_tables(seq, head_dim, theta):
    """cos/sin [seq, head_dim / 2]: freq_i = 1 / theta^(2i / head_dim), angle =
    pos * freq_i in f32 (compute_rope_freqs, iris_qwen3.c:258-275)."""
    i = np.arange(head_dim // 2, dtype=F32)
    freq = (F32(1.0) / np.power(F32(theta), (F32(2.0) * i) / F32(head_dim))).astype(F32)
    ang = (np.arange(seq, dtype=F32)[:, None] * freq[None, :]).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def apply_rope_half(x, cos, sin, heads, head_dim):
    """Split-half rotation of each head: (x_i, x_{i+d/2}) -> (x_i c - x_{i+d/2} s,
    x_i s + x_{i+d/2} c) (apply_rope, iris_qwen3.c:277-329)."""
    s = x.shape[0]
    h = x.reshape(s, heads, head_dim)
    half = head_dim // 2
    x0, x1 = h[..., :half], h[..., half:]
    c, sn = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x0 * c - x1 * sn, x0 * sn + x1 * c], -1).reshape(s, -1).astype(F32)


def attention(q, k, v, mask, heads, kv_heads, head_dim):
    """Causal GQA attention with a key padding mask: masked scores -1e9, then
    softmax, query head h reads kv head h / (heads / kv_heads)
    (qwen3_attention_forward, iris_qwen3.c:331-466)."""
    s = q.shape[0]
    scale = F32(1.0 / np.sqrt(head_dim))
    out = np.zeros((s, heads * head_dim), F32)
    causal = np.triu(np.ones((s, s), bool), 1)
    pad = np.asarray(mask)[None, :] == 0
    for h in range(heads):
        g = h // (heads // kv_heads)
        qh = q[:, h * head_dim:(h + 1) * head_dim]
        kh = k[:, g * head_dim:(g + 1) * head_dim]
        vh = v[:, g * head_dim:(g + 1) * head_dim]
        sc = (qh @ kh.T) * scale
        sc[causal | pad] = F32(-1e9)
        sc = np.exp(sc - sc.max(1, keepdims=True))
        sc = sc / sc.sum(1, keepdims=True)
        out[:, h * head_dim:(h + 1) * head_dim] = sc.astype(F32) @ vh
    return out


def layer(w, i, x, cos, sin, mask, cfg):
    """Pre-norm decoder layer: RMSNorm -> attention (per-head q/k RMSNorm,
    RoPE) -> residual -> RMSNorm -> SwiGLU MLP -> residual
    (qwen3_layer_forward, iris_qwen3.c:496-535)."""
    p = f"model.layers.{i}."
    nh, nkv, d = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    s = x.shape[0]
    h = rms_norm(x, w[p + "input_layernorm.weight"])
    q = h @ w[p + "self_attn.q_proj.weight"].T
    k = h @ w[p + "self_attn.k_proj.weight"].T
    v = h @ w[p + "self_attn.v_proj.weight"].T
    q = rms_norm(q.reshape(s * nh, d), w[p + "self_attn.q_norm.weight"]).reshape(s, nh * d)
    k = rms_norm(k.reshape(s * nkv, d), w[p + "self_attn.k_norm.weight"]).reshape(s, nkv * d)
    q = apply_rope_half(q, cos, sin, nh, d)
    k = apply_rope_half(k, cos, sin, nkv, d)
    a = attention(q, k, v.astype(F32), mask, nh, nkv, d)
    x = (x + a @ w[p + "self_attn.o_proj.weight"].T).astype(F32)
    h = rms_norm(x, w[p + "post_attention_layernorm.weight"])
    g = h @ w[p + "mlp.gate_proj.weight"].T
    u = h @ w[p + "mlp.up_proj.weight"].T
    m = (g / (1.0 + np.exp(-g)) * u).astype(F32)
    return (x + m @ w[p + "mlp.down_proj.weight"].T).astype(F32)


def forward(w, cfg, ids, mask, zimage=False):
    """Token ids [S] + mask [S] -> text embeddings: Flux concatenates the hidden
    states after layers 8, 17, 26 -> [S, 3H]; Z-Image takes the state after
    layer num_layers - 2 -> [S, H] (qwen3_forward, iris_qwen3.c:1072-1196).
    Unknown token ids embed as zeros."""
    H = cfg["hidden_size"]
    ids = np.asarray(ids)
    emb = w["model.embed_tokens.weight"]
    x = np.zeros((len(ids), H), F32)
    ok = (ids >= 0) & (ids < emb.shape[0])
    x[ok] = emb[ids[ok]]
    cos, sin = rope_tables(len(ids), cfg["head_dim"], cfg["rope_theta"])
    last = cfg["num_hidden_layers"] - 2 if zimage else FLUX_LAYERS[-1]
    outs = []
    for i in range(last + 1):
        x = layer(w, i, x, cos, sin, mask, cfg)
        if (zimage and i == last) or (not zimage and i in FLUX_LAYERS):
            outs.append(x.copy())
    return np.concatenate(outs, 1) if len(outs) > 1 else outs[0]
