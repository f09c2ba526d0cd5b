"""ORACLE — test infrastructure only; never imported by the product path.

numpy restatement of the reference's IP-Adapter for the Flux transformer
(iris_ip_adapter.c, iris_ip_adapter.h):

* ``load_bundle``  iris_ip_adapter_load (:113): adapter_meta.json dims and
  modes, weights dequantised to f32 (int8 rows times their ``.scale``, :80);
* ``perceive``     iris_ip_adapter_perceive (:331): the SigLIP
  PerceiverResampler (:265; optional per-dimension input standardisation,
  multi-head cross-attention with ``perceiver_heads`` heads, out_proj,
  LayerNorm), the CSD FiLM module (:235) and the hybrid of both;
* ``get_kv``       iris_ip_adapter_get_kv (:366): ip_embeds @ stacked[block],
  hybrid group gate on V;
* ``inject``       iris_ip_adapter_inject (:386): hidden += s * SDPA(q, k, v)
  over 128-wide heads, s = ip_scale[block] * schedule multiplier;
* ``set_schedule`` / ``step_mult`` (:401, :424);
* ``ip_context``   what the transformer hooks consume: per block k, v and the
  scale; ``flux_oracle.forward(..., ip=...)`` adds the contribution after
  each block to its image rows using the post-QK-norm, pre-RoPE image Q
  (iris_transformer_flux.c:2355-2365, :2440-2446, :2607-2612, :3848-3855,
  :3921-3926).

Pinned in tests/test_ip_oracle.py against the reference's own golden fixtures
(debug/fixtures/ip_adapter: siglip, csd, hybrid, int8 bundles; stored as
tests/golden/ip_fixture.npz) and against the reference's forward with an
adapter attached.
"""
from __future__ import annotations

import json
import os
import re
import struct

import numpy as np

F32 = np.float32
LN_EPS = 1e-5


def _read_st_raw(path):
    """{name: (dtype, shape, raw bytes)} of a safetensors file."""
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    out = {}
    for name, e in hdr.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        out[name] = (e["dtype"], tuple(e["shape"]), raw[8 + n + a:8 + n + b])
    return out


def _to_f32(dtype, shape, buf):
    if dtype == "F32":
        x = np.frombuffer(buf, "<f4")
    elif dtype == "F16":
        x = np.frombuffer(buf, "<f2").astype(F32)
    elif dtype == "BF16":
        x = (np.frombuffer(buf, "<u2").astype(np.uint32) << 16).view(F32)
    elif dtype == "I8":
        x = np.frombuffer(buf, np.int8).astype(F32)
    else:
        raise ValueError(dtype)
    return x.astype(F32).reshape(shape)


def _meta_int(meta, key, default):
    """cfg_int semantics: the first number after "key": (iris_config_parse.h)."""
    m = re.search(r'"%s"\s*:\s*(-?[0-9.eE+-]+|true|false)' % re.escape(key), meta)
    if not m:
        return default
    v = m.group(1)
    if v in ("true", "false"):
        return 1 if v == "true" else 0
    return int(float(v))


def _meta_str(meta, key, default):
    m = re.search(r'"%s"\s*:\s*"([^"]*)"' % re.escape(key), meta)
    return m.group(1)[:15] if m else default


def load_bundle(bundle_dir: str) -> dict | None:
    with open(os.path.join(bundle_dir, "adapter_meta.json")) as f:
        meta = f.read()[:4095]
    a = dict(num_blocks=_meta_int(meta, "num_blocks", 0),
             num_double_blocks=_meta_int(meta, "num_double_blocks", 0),
             num_single_blocks=_meta_int(meta, "num_single_blocks", 0),
             hidden_dim=_meta_int(meta, "hidden_dim", 0),
             num_image_tokens=_meta_int(meta, "num_image_tokens", 0),
             siglip_dim=_meta_int(meta, "siglip_dim", 0),
             perceiver_heads=_meta_int(meta, "perceiver_heads", 0),
             style_only=_meta_int(meta, "style_only", 0),
             cond_mode=_meta_str(meta, "cond_mode", "siglip"),
             csd_dim=_meta_int(meta, "csd_dim", 768),
             quant=_meta_str(meta, "quant", ""))
    H = a["hidden_dim"]
    if H <= 0 or a["num_blocks"] <= 0:
        return None
    if a["perceiver_heads"] <= 0 or H % a["perceiver_heads"]:
        a["perceiver_heads"] = H // 128
    t = _read_st_raw(os.path.join(bundle_dir, "adapter_weights.safetensors"))

    def get(name):
        if name not in t:
            return None
        dt, shp, buf = t[name]
        x = _to_f32(dt, shp, buf)
        if dt == "I8":
            if name + ".scale" not in t:
                return None
            sc = _to_f32(*t[name + ".scale"]).reshape(-1)
            cols = shp[-1] if shp else x.size
            rows = x.size // cols
            if sc.size != rows:
                return None
            x = (x.reshape(rows, cols) * sc[:, None]).reshape(shp)
        return x.astype(F32)

    mode = a["cond_mode"]
    names = ["query_tokens", "norm_weight", "norm_bias"]
    names += ["film_weight", "film_bias"] if mode == "csd" else \
        ["query_proj", "key_proj", "value_proj", "out_proj", "in_gamma", "in_beta"]
    for n_ in names:
        a[n_] = get("perceiver." + n_)
    if mode == "hybrid":
        for n_ in ("query_tokens", "film_weight", "film_bias", "norm_weight", "norm_bias"):
            a["csd_" + n_] = get("csd." + n_)
        a["group_gate"] = get("group_gate")
    else:
        a["group_gate"] = None
    for n_ in ("ip_k_stacked", "ip_v_stacked", "ip_scale"):
        a[n_] = get(n_)
    need = ["query_tokens", "norm_weight", "norm_bias", "ip_k_stacked", "ip_v_stacked", "ip_scale"]
    need += ["film_weight", "film_bias"] if mode == "csd" else ["query_proj", "key_proj", "value_proj", "out_proj"]
    if mode == "hybrid":
        need += ["csd_query_tokens", "csd_film_weight", "csd_film_bias", "csd_norm_weight", "csd_norm_bias"]
    if any(a.get(n_) is None for n_ in need):
        return None
    a["ip_scale"] = a["ip_scale"].reshape(-1).copy()
    a["sched"] = (0, 0.0)
    a["sched_mult"] = 1.0
    return a


def _layernorm_rows(x, w, b):
    x = x.astype(np.float64)
    mu = x.mean(axis=1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
    return ((x - mu) / np.sqrt(var + LN_EPS) * w + b).astype(F32)


def _mha(q, k, v, heads):
    """softmax(q k^T / sqrt(hd)) v per head over flat [seq, heads*hd] tensors."""
    sq, hid = q.shape
    hd = hid // heads
    qh = q.astype(np.float64).reshape(sq, heads, hd).transpose(1, 0, 2)
    kh = k.astype(np.float64).reshape(-1, heads, hd).transpose(1, 0, 2)
    vh = v.astype(np.float64).reshape(-1, heads, hd).transpose(1, 0, 2)
    s = qh @ kh.transpose(0, 2, 1) / np.sqrt(hd)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return (p @ vh).transpose(1, 0, 2).reshape(sq, hid).astype(F32)


def _csd_film(H, T, csd, qtok, fw, fb, nw, nb):
    """perceive_csd_film (:235)."""
    film = fw.astype(np.float64) @ csd.astype(np.float64) + fb
    scale, shift = film[:H], film[H:]
    tok = qtok[:T].astype(np.float64) * (1.0 + scale) + shift
    return _layernorm_rows(tok, nw, nb)


def _siglip_mha(a, siglip, T):
    """perceive_siglip_mha (:265)."""
    x = siglip.astype(np.float64)
    if a.get("in_gamma") is not None and a.get("in_beta") is not None:
        mu = x.mean(axis=0, keepdims=True)
        var = ((x - mu) ** 2).mean(axis=0, keepdims=True)
        x = (x - mu) / np.sqrt(var + LN_EPS) * a["in_gamma"] + a["in_beta"]
    q = a["query_tokens"][:T].astype(np.float64) @ a["query_proj"].T
    k = x @ a["key_proj"].T
    v = x @ a["value_proj"].T
    att = _mha(q, k, v, a["perceiver_heads"]).astype(np.float64)
    return _layernorm_rows(att @ a["out_proj"].T, a["norm_weight"], a["norm_bias"])


def perceive(a, feats):
    """iris_ip_adapter_perceive (:331) -> ip_embeds [T, H]."""
    H, T = a["hidden_dim"], a["num_image_tokens"]
    feats = np.asarray(feats, F32)
    if a["cond_mode"] == "csd":
        return _csd_film(H, T, feats.reshape(-1)[:a["csd_dim"]], a["query_tokens"], a["film_weight"],
                         a["film_bias"], a["norm_weight"], a["norm_bias"])
    if a["cond_mode"] == "hybrid":
        half = T // 2
        sig = feats[:-1]
        csd = feats[-1][:a["csd_dim"]]
        return np.concatenate([_siglip_mha(a, sig, half),
                               _csd_film(H, half, csd, a["csd_query_tokens"], a["csd_film_weight"],
                                         a["csd_film_bias"], a["csd_norm_weight"], a["csd_norm_bias"])])
    return _siglip_mha(a, feats, T)


def get_kv(a, block, embeds):
    """iris_ip_adapter_get_kv (:366): embeds @ stacked[block] (no transpose), gated V."""
    H, T = a["hidden_dim"], a["num_image_tokens"]
    W = a["ip_k_stacked"].reshape(-1, H, H)[block].astype(np.float64)
    Wv = a["ip_v_stacked"].reshape(-1, H, H)[block].astype(np.float64)
    k = (embeds.astype(np.float64) @ W).astype(F32)
    v = (embeds.astype(np.float64) @ Wv).astype(F32)
    if a.get("group_gate") is not None:
        g = a["group_gate"].reshape(-1, 2)[block]
        v[:T // 2] *= g[0]
        v[T // 2:] *= g[1]
    return k, v


def block_scale(a, block):
    return float(a["ip_scale"][block]) * a["sched_mult"]


def inject(a, block, q, k, v, hidden):
    """iris_ip_adapter_inject (:386): hidden + s * SDPA over 128-wide heads."""
    s = block_scale(a, block)
    if s == 0.0:
        return hidden
    return (hidden.astype(np.float64) + s * _mha(q, k, v, a["hidden_dim"] // 128)).astype(F32)


def set_schedule(a, spec):
    """iris_ip_adapter_set_schedule (:401); returns 0 or -1 (state reset to none)."""
    a["sched"], a["sched_mult"] = (0, 0.0), 1.0
    if not spec or spec == "none":
        return 0
    m = re.match(r"(late|early):(.*)$", spec)
    try:
        f = float(m.group(2)) if m else None
    except ValueError:
        f = None
    if m is None or f is None:
        return -1
    if not np.isfinite(f) or f < 0.0 or f > 1.0:
        return -1
    a["sched"] = (1 if m.group(1) == "late" else 2, f)
    return 0


def set_step(a, step, num_steps):
    """iris_ip_adapter_set_step (:424)."""
    kind, f = a["sched"]
    if kind == 0 or num_steps <= 0:
        a["sched_mult"] = 1.0
        return
    frac = step / (num_steps - 1) if num_steps > 1 else 1.0
    a["sched_mult"] = 1.0 if ((frac >= f) if kind == 1 else (frac < f)) else 0.0


def ip_context(a, feats, scale_mult=1.0):
    """What iris_load_ip_adapter (iris.c:520) attaches: ip_scale *= scale_mult,
    ip_embeds = perceive(feats); the hooks then compute k/v per block."""
    a = dict(a)
    a["ip_scale"] = (a["ip_scale"] * F32(scale_mult)).astype(F32)
    emb = perceive(a, feats)
    kv = [get_kv(a, b, emb) for b in range(a["num_blocks"])]
    return {"adapter": a, "embeds": emb, "kv": kv}
