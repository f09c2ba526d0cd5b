"""Seeded random-init model directories — TEST INFRASTRUCTURE ONLY.

Writes HF-style model directories (``transformer/config.json`` plus a bf16
``diffusion_pytorch_model.safetensors``) whose tensor names and shapes are the
ones the reference loaders read:

* Flux.2 Klein: ``iris_transformer_load_safetensors``
  (iris_transformer_flux.c:5300-5497; config keys parsed at :395-455).
* Z-Image S3-DiT: ``zi_transformer_load_safetensors``
  (iris_transformer_zimage.c:2164-2427).

Every tensor is drawn from its own generator seeded by (seed, crc32(name)),
so any subset of tensors can be regenerated bit-identically without
generating the rest.  Values are N(0, std) rounded to bf16 (round to nearest
even), so the f32 reference oracle and the bf16 CUDA path see identical
weights.
"""
from __future__ import annotations

import json
import os
import struct
import zlib

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bit patterns.

    Computed in uint32: exact for every finite value and for infinities (the
    largest finite pattern plus the rounding bias is below 2^32); only
    negative NaN payloads above 0xFFFF7FFF would wrap, and no generator here
    produces NaN."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = u + np.uint32(0x7FFF)
    r += (u >> np.uint32(16)) & np.uint32(1)
    r >>= np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ---------------------------------------------------------------------------
# Flux.2 Klein
# ---------------------------------------------------------------------------

KLEIN_4B = dict(num_attention_heads=24, attention_head_dim=128, num_layers=5,
                num_single_layers=20, joint_attention_dim=7680, in_channels=128,
                mlp_ratio=3.0, rope_theta=2000.0)
KLEIN_9B = dict(num_attention_heads=32, attention_head_dim=128, num_layers=8,
                num_single_layers=24, joint_attention_dim=12288, in_channels=128,
                mlp_ratio=3.0, rope_theta=2000.0)


def flux_dims(cfg: dict) -> dict:
    h = cfg["num_attention_heads"] * cfg["attention_head_dim"]
    return dict(hidden=h, heads=cfg["num_attention_heads"], head_dim=cfg["attention_head_dim"],
                mlp=int(h * cfg.get("mlp_ratio", 3.0)), n_double=cfg["num_layers"],
                n_single=cfg["num_single_layers"], text_dim=cfg["joint_attention_dim"],
                channels=cfg["in_channels"], theta=float(cfg.get("rope_theta", 2000.0)))


def flux_tensor_specs(cfg: dict) -> list[tuple[str, tuple, str]]:
    """(name, shape, kind) for every tensor the Flux loader reads.

    kind is "linear" for projection matrices and "norm" for the per-head
    QK-RMSNorm scale vectors (iris_transformer_flux.c:5374-5497)."""
    d = flux_dims(cfg)
    H, F, D, C, T = d["hidden"], d["mlp"], d["head_dim"], d["channels"], d["text_dim"]
    s = [("x_embedder.weight", (H, C), "linear"),
         ("context_embedder.weight", (H, T), "linear"),
         ("time_guidance_embed.timestep_embedder.linear_1.weight", (H, 256), "linear"),
         ("time_guidance_embed.timestep_embedder.linear_2.weight", (H, H), "linear"),
         ("double_stream_modulation_img.linear.weight", (6 * H, H), "linear"),
         ("double_stream_modulation_txt.linear.weight", (6 * H, H), "linear"),
         ("single_stream_modulation.linear.weight", (3 * H, H), "linear")]
    for i in range(d["n_double"]):
        p = f"transformer_blocks.{i}."
        s += [(p + "attn.norm_q.weight", (D,), "norm"), (p + "attn.norm_k.weight", (D,), "norm"),
              (p + "attn.to_q.weight", (H, H), "linear"), (p + "attn.to_k.weight", (H, H), "linear"),
              (p + "attn.to_v.weight", (H, H), "linear"),
              (p + "attn.to_out.0.weight", (H, H), "linear"),
              (p + "ff.linear_in.weight", (2 * F, H), "linear"),
              (p + "ff.linear_out.weight", (H, F), "linear"),
              (p + "attn.norm_added_q.weight", (D,), "norm"),
              (p + "attn.norm_added_k.weight", (D,), "norm"),
              (p + "attn.add_q_proj.weight", (H, H), "linear"),
              (p + "attn.add_k_proj.weight", (H, H), "linear"),
              (p + "attn.add_v_proj.weight", (H, H), "linear"),
              (p + "attn.to_add_out.weight", (H, H), "linear"),
              (p + "ff_context.linear_in.weight", (2 * F, H), "linear"),
              (p + "ff_context.linear_out.weight", (H, F), "linear")]
    for i in range(d["n_single"]):
        p = f"single_transformer_blocks.{i}."
        s += [(p + "attn.norm_q.weight", (D,), "norm"), (p + "attn.norm_k.weight", (D,), "norm"),
              (p + "attn.to_qkv_mlp_proj.weight", (3 * H + 2 * F, H), "linear"),
              (p + "attn.to_out.weight", (H, H + F), "linear")]
    s += [("norm_out.linear.weight", (2 * H, H), "linear"),
          ("proj_out.weight", (C, H), "linear")]
    return s


def gen_tensor(seed: int, name: str, shape: tuple, kind: str, std: float = 0.02,
               norm_mode: str = "random") -> np.ndarray:
    """bf16 bit pattern (uint16) of one seeded tensor.

    norm_mode "random": N(0, std) like every other tensor.
    norm_mode "unit":   1 + N(0, 0.1) so QK-RMSNorm keeps O(1) logits and the
                        softmax is actually exercised."""
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    if kind == "norm" and norm_mode == "unit":
        x = 1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)
    else:
        x = std * rng.standard_normal(shape, dtype=np.float32)
    return f32_to_bf16_bits(x)


def write_safetensors_generated(path: str, specs, make, threads: int | None = None) -> None:
    """Stream a bf16 safetensors file whose tensors are produced by make(name, shape, kind)
    (uint16 bit patterns), generating up to 2*threads tensors ahead on a thread pool
    (numpy's generators and ufuncs release the GIL) and writing them in order.  Used for
    the full-width models (Klein-4B: 7.7 GB), which must not be held in memory whole."""
    from concurrent.futures import ThreadPoolExecutor

    header, off = {}, 0
    for name, shp, _ in specs:
        n = 2 * int(np.prod(shp))
        header[name] = {"dtype": "BF16", "shape": list(shp), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    threads = threads or min(32, os.cpu_count() or 1)
    with open(path, "wb") as f, ThreadPoolExecutor(threads) as ex:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        pending = []
        it = iter(specs)
        for spec in it:
            pending.append(ex.submit(make, *spec))
            if len(pending) >= 2 * threads:
                break
        for spec in it:
            f.write(pending.pop(0).result().tobytes())
            pending.append(ex.submit(make, *spec))
        for fut in pending:
            f.write(fut.result().tobytes())


def write_safetensors(path: str, tensors: dict[str, np.ndarray]) -> None:
    """Write uint16 (bf16) / float16 / int8 / float32 arrays in the safetensors container format."""
    header = {}
    off = 0
    for name, arr in tensors.items():
        dt = {np.dtype(np.uint16): "BF16", np.dtype(np.float16): "F16", np.dtype(np.int8): "I8"}.get(arr.dtype, "F32")
        n = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + n]}
        off += n
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for arr in tensors.values():
            f.write(np.ascontiguousarray(arr).tobytes())


def make_flux_model(model_dir: str, cfg: dict, seed: int, std: float = 0.02,
                    norm_mode: str = "random", keep: bool = True) -> dict[str, np.ndarray] | None:
    """Create a random Flux model directory; returns {name: f32 values}, or None
    with keep=False (full-width models: the file is streamed, nothing is held)."""
    os.makedirs(os.path.join(model_dir, "transformer"), exist_ok=True)
    full = dict(_class_name="Flux2Transformer2DModel", **cfg)
    with open(os.path.join(model_dir, "transformer", "config.json"), "w") as f:
        json.dump(full, f, indent=1)
    with open(os.path.join(model_dir, "model_index.json"), "w") as f:
        json.dump({"_class_name": "Flux2KleinPipeline"}, f)
    path = os.path.join(model_dir, "transformer", "diffusion_pytorch_model.safetensors")
    if not keep:
        write_safetensors_generated(path, flux_tensor_specs(cfg),
                                    lambda n, shp, kind: gen_tensor(seed, n, shp, kind, std, norm_mode))
        return None
    bits = {n: gen_tensor(seed, n, shp, kind, std, norm_mode)
            for n, shp, kind in flux_tensor_specs(cfg)}
    write_safetensors(path, bits)
    return {n: bf16_bits_to_f32(b) for n, b in bits.items()}


def flux_weights(cfg: dict, seed: int, std: float = 0.02, norm_mode: str = "random"):
    """Regenerate the f32 (bf16-valued) weights of make_flux_model without disk I/O."""
    return {n: bf16_bits_to_f32(gen_tensor(seed, n, shp, kind, std, norm_mode))
            for n, shp, kind in flux_tensor_specs(cfg)}


def flux_weights_bits(cfg: dict, seed: int, std: float = 0.02, norm_mode: str = "random"):
    return {n: gen_tensor(seed, n, shp, kind, std, norm_mode)
            for n, shp, kind in flux_tensor_specs(cfg)}


# ---------------------------------------------------------------------------
# Flux LoRA adapters (the four key layouts lora_load reads, iris_lora.c:240-486)
# ---------------------------------------------------------------------------

LORA_FORMATS = ("xlabs", "kohya", "diffusers", "bfl")


def flux_lora_specs(cfg: dict, fmt: str, rank: int, singles: bool = True,
                    prefix: str = "diffusion_model", single_out: str = "to_out",
                    blocks: tuple | None = None) -> list[tuple[str, tuple]]:
    """(name, shape) of every adapter tensor of a full-coverage LoRA.

    fmt: "xlabs" (double blocks only, fused Q|K|V), "kohya", "bfl" (fused
    Q|K|V, single linear1/linear2), "diffusers" (separate Q/K/V, single
    to_qkv_mlp_proj and `single_out` = "to_out" or the fallback "proj_out").
    blocks: double-block indices to cover (all by default)."""
    d = flux_dims(cfg)
    H, F, r = d["hidden"], d["mlp"], rank
    dbl = range(d["n_double"]) if blocks is None else blocks
    out = []
    for i in dbl:
        for st, n in (("img", 1), ("txt", 2)):
            if fmt == "xlabs":
                p = f"double_blocks.{i}.processor."
                out += [(p + f"qkv_lora{n}.down.weight", (r, H)), (p + f"qkv_lora{n}.up.weight", (3 * H, r)),
                        (p + f"proj_lora{n}.down.weight", (r, H)), (p + f"proj_lora{n}.up.weight", (H, r))]
            elif fmt == "kohya":
                for what, o in (("qkv", 3 * H), ("proj", H)):
                    p = f"lora_unet_double_blocks_{i}_{st}_attn_{what}."
                    out += [(p + "lora_down.weight", (r, H)), (p + "lora_up.weight", (o, r))]
            elif fmt == "bfl":
                for what, o in (("qkv", 3 * H), ("proj", H)):
                    p = f"{prefix}.double_blocks.{i}.{st}_attn.{what}."
                    out += [(p + "lora_A.weight", (r, H)), (p + "lora_B.weight", (o, r))]
            else:
                names = (("to_q", "to_k", "to_v", "to_out.0") if st == "img"
                         else ("add_q_proj", "add_k_proj", "add_v_proj", "to_add_out"))
                for nm in names:
                    p = f"transformer.transformer_blocks.{i}.attn.{nm}."
                    out += [(p + "lora_A.weight", (r, H)), (p + "lora_B.weight", (H, r))]
    if singles and fmt != "xlabs":
        for i in range(d["n_single"]):
            for k, (din, dout) in ((1, (H, 3 * H + 2 * F)), (2, (H + F, H))):
                if fmt == "kohya":
                    p = f"lora_unet_single_blocks_{i}_linear{k}."
                    dn, up = p + "lora_down.weight", p + "lora_up.weight"
                elif fmt == "bfl":
                    p = f"{prefix}.single_blocks.{i}.linear{k}."
                    dn, up = p + "lora_A.weight", p + "lora_B.weight"
                else:
                    p = (f"transformer.single_transformer_blocks.{i}.attn.to_qkv_mlp_proj." if k == 1 else
                         f"transformer.single_transformer_blocks.{i}." +
                         ("attn.to_out." if single_out == "to_out" else "proj_out."))
                    dn, up = p + "lora_A.weight", p + "lora_B.weight"
                out += [(dn, (r, din)), (up, (dout, r))]
    return out


def make_flux_lora(path: str, cfg: dict, fmt: str, rank: int = 8, seed: int = 0, std: float = 0.06,
                   dtype: str = "bf16", **kw) -> dict[str, np.ndarray]:
    """Write a seeded LoRA file; returns {name: f32 values as stored}."""
    tensors, vals = {}, {}
    for name, shp in flux_lora_specs(cfg, fmt, rank, **kw):
        rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
        x = std * rng.standard_normal(shp, dtype=np.float32)
        if dtype == "bf16":
            tensors[name] = f32_to_bf16_bits(x)
            vals[name] = bf16_bits_to_f32(tensors[name])
        else:
            tensors[name] = x
            vals[name] = x
    write_safetensors(path, tensors)
    return vals


# ---------------------------------------------------------------------------
# Flux IP-Adapter bundles (the layout iris_ip_adapter_load reads,
# iris_ip_adapter.c:113-216: adapter_meta.json + adapter_weights.safetensors)
# ---------------------------------------------------------------------------


def make_ip_bundle(bundle_dir: str, cfg: dict, mode: str = "siglip", tokens: int = 8, siglip_dim: int = 64,
                   csd_dim: int = 32, perceiver_heads: int = 4, seed: int = 0, quant: str = "bfloat16",
                   in_norm: bool = True, gate: bool = True, style_only: bool = False,
                   kv_std: float = 0.25) -> dict:
    """Write a seeded IP-Adapter bundle for a Flux model of config cfg (one IP
    block per double and single block).  mode: siglip | csd | hybrid; quant:
    bfloat16 | float16 | float32 | int8 (large matrices as int8 + per-row
    f32 .scale).  Returns the meta dict."""
    d = flux_dims(cfg)
    H, nb = d["hidden"], d["n_double"] + d["n_single"]
    rng = np.random.default_rng(seed)
    f32 = {}

    def r(name, shape, std, mean=0.0):
        f32[name] = (mean + std * rng.standard_normal(shape)).astype(np.float32)

    T = tokens
    r("perceiver.query_tokens", (T, H), 1.0)
    r("perceiver.norm_weight", (H,), 0.1, 1.0)
    r("perceiver.norm_bias", (H,), 0.1)
    if mode == "csd":
        r("perceiver.film_weight", (2 * H, csd_dim), 0.2)
        r("perceiver.film_bias", (2 * H,), 0.1)
    else:
        for n_, shp in (("query_proj", (H, H)), ("key_proj", (H, siglip_dim)), ("value_proj", (H, siglip_dim)),
                        ("out_proj", (H, H))):
            r("perceiver." + n_, shp, 1.0 / np.sqrt(shp[1]))
        if in_norm:
            r("perceiver.in_gamma", (siglip_dim,), 0.1, 1.0)
            r("perceiver.in_beta", (siglip_dim,), 0.1)
    if mode == "hybrid":
        r("csd.query_tokens", (T // 2, H), 1.0)
        r("csd.film_weight", (2 * H, csd_dim), 0.2)
        r("csd.film_bias", (2 * H,), 0.1)
        r("csd.norm_weight", (H,), 0.1, 1.0)
        r("csd.norm_bias", (H,), 0.1)
        if gate:
            f32["group_gate"] = rng.uniform(0.3, 1.2, (nb, 2)).astype(np.float32)
    r("ip_k_stacked", (nb, H, H), kv_std / np.sqrt(H))
    r("ip_v_stacked", (nb, H, H), kv_std / np.sqrt(H))
    sc = rng.uniform(0.4, 1.0, nb).astype(np.float32)
    if style_only:
        sc[:d["n_double"]] = 0.0
    f32["ip_scale"] = sc
    big = {"perceiver.query_proj", "perceiver.key_proj", "perceiver.value_proj", "perceiver.out_proj",
           "ip_k_stacked", "ip_v_stacked"}
    out = {}
    for name, x in f32.items():
        if quant == "int8" and name in big:
            rows = x.reshape(-1, x.shape[-1])
            s_ = np.maximum(np.abs(rows).max(axis=1), 1e-12) / 127.0
            out[name] = np.clip(np.rint(rows / s_[:, None]), -127, 127).astype(np.int8).reshape(x.shape)
            out[name + ".scale"] = s_.astype(np.float32)
        elif name in ("ip_scale", "group_gate") or quant == "float32":
            out[name] = x
        elif quant == "float16":
            out[name] = x.astype(np.float16)
        else:
            out[name] = f32_to_bf16_bits(x)
    meta = dict(version=1, adapter_type="ip_adapter_klein", num_blocks=nb, num_double_blocks=d["n_double"],
                num_single_blocks=d["n_single"], hidden_dim=H, num_image_tokens=T,
                siglip_dim=0 if mode == "csd" else siglip_dim, cond_mode=mode,
                csd_dim=0 if mode == "siglip" else csd_dim, perceiver_heads=perceiver_heads,
                style_only=style_only, quant=quant)
    os.makedirs(bundle_dir, exist_ok=True)
    with open(os.path.join(bundle_dir, "adapter_meta.json"), "w") as f:
        json.dump(meta, f, indent=1)
    write_safetensors(os.path.join(bundle_dir, "adapter_weights.safetensors"), out)
    return meta


def make_csd_mod(path: str, csd_dim: int, mlp: int, hidden: int, seed: int = 0) -> dict:
    """A CSDModulation MLP file (csd_mod.safetensors: fc1 [mlp, csd], fc2 [hidden, mlp],
    biases; read by csd_mod_load, iris_csdmod.c); returns the f32 tensors."""
    rng = np.random.default_rng(seed)
    t = {"fc1.weight": (rng.standard_normal((mlp, csd_dim)) / np.sqrt(csd_dim)).astype(np.float32),
         "fc1.bias": (0.1 * rng.standard_normal(mlp)).astype(np.float32),
         "fc2.weight": (rng.standard_normal((hidden, mlp)) / np.sqrt(mlp)).astype(np.float32),
         "fc2.bias": (0.1 * rng.standard_normal(hidden)).astype(np.float32)}
    write_safetensors(path, t)
    return t


def ip_features(mode: str, siglip_seq: int = 16, siglip_dim: int = 64, csd_dim: int = 32, seed: int = 1):
    """Conditioning features as iris_load_ip_adapter reads them (iris.c:546-567):
    siglip [n, siglip_dim]; csd [1, csd_dim]; hybrid [n + 1, siglip_dim], last row
    the CSD vector zero-padded."""
    rng = np.random.default_rng(seed)
    if mode == "csd":
        return rng.standard_normal((1, csd_dim)).astype(np.float32)
    sig = (rng.standard_normal((siglip_seq, siglip_dim)) * rng.uniform(0.5, 3.0, siglip_dim)).astype(np.float32)
    if mode == "siglip":
        return sig
    last = np.zeros((1, siglip_dim), np.float32)
    last[0, :csd_dim] = rng.standard_normal(csd_dim)
    return np.concatenate([sig, last])


# ---------------------------------------------------------------------------
# Z-Image S3-DiT
# ---------------------------------------------------------------------------

ZIMAGE_6B = dict(dim=3840, n_heads=30, n_layers=30, n_refiner=2, cap_feat_dim=2560,
                 in_channels=16, patch_size=2, rope_theta=256.0, axes_dims=[32, 48, 48],
                 ffn_dim=10240, adaln_dim=256, t_mid=1024)


def zimage_tensor_specs(cfg: dict) -> list[tuple[str, tuple, str]]:
    """(name, shape, kind) for the tensors zi_transformer_load_safetensors reads
    (iris_transformer_zimage.c:2024-2383).  Biases are kind "bias"."""
    D, F, A = cfg["dim"], cfg["ffn_dim"], cfg["adaln_dim"]
    hd = D // cfg["n_heads"]
    ps, ic, cap = cfg["patch_size"], cfg["in_channels"], cfg["cap_feat_dim"]
    pf = ps * ps * ic
    s = [("t_embedder.mlp.0.weight", (cfg["t_mid"], 256), "linear"),
         ("t_embedder.mlp.0.bias", (cfg["t_mid"],), "bias"),
         ("t_embedder.mlp.2.weight", (A, cfg["t_mid"]), "linear"),
         ("t_embedder.mlp.2.bias", (A,), "bias"),
         ("cap_embedder.0.weight", (cap,), "norm"),
         ("cap_embedder.1.weight", (D, cap), "linear"),
         ("cap_embedder.1.bias", (D,), "bias"),
         (f"all_x_embedder.{ps}-1.weight", (D, pf), "linear"),
         (f"all_x_embedder.{ps}-1.bias", (D,), "bias"),
         ("x_pad_token", (1, D), "linear"),
         ("cap_pad_token", (1, D), "linear"),
         (f"all_final_layer.{ps}-1.adaLN_modulation.1.weight", (D, A), "linear"),
         (f"all_final_layer.{ps}-1.adaLN_modulation.1.bias", (D,), "bias"),
         (f"all_final_layer.{ps}-1.linear.weight", (pf, D), "linear"),
         (f"all_final_layer.{ps}-1.linear.bias", (pf,), "bias")]

    def block(p, modulated):
        b = [(p + "attention.to_q.weight", (D, D), "linear"),
             (p + "attention.to_k.weight", (D, D), "linear"),
             (p + "attention.to_v.weight", (D, D), "linear"),
             (p + "attention.to_out.0.weight", (D, D), "linear"),
             (p + "attention.norm_q.weight", (hd,), "norm"),
             (p + "attention.norm_k.weight", (hd,), "norm"),
             (p + "attention_norm1.weight", (D,), "norm"),
             (p + "attention_norm2.weight", (D,), "norm"),
             (p + "ffn_norm1.weight", (D,), "norm"),
             (p + "ffn_norm2.weight", (D,), "norm"),
             (p + "feed_forward.w1.weight", (F, D), "linear"),
             (p + "feed_forward.w2.weight", (D, F), "linear"),
             (p + "feed_forward.w3.weight", (F, D), "linear")]
        if modulated:
            b += [(p + "adaLN_modulation.0.weight", (4 * D, A), "linear"),
                  (p + "adaLN_modulation.0.bias", (4 * D,), "bias")]
        return b

    for i in range(cfg["n_refiner"]):
        s += block(f"noise_refiner.{i}.", True)
    for i in range(cfg["n_refiner"]):
        s += block(f"context_refiner.{i}.", False)
    for i in range(cfg["n_layers"]):
        s += block(f"layers.{i}.", True)
    return s


def make_zimage_model(model_dir: str, cfg: dict, seed: int, std: float = 0.02,
                      norm_mode: str = "random", keep: bool = True) -> dict[str, np.ndarray] | None:
    """Random Z-Image model directory (config keys as read by the reference's
    model autodetection, iris.c:300-330); returns {name: f32 values}."""
    os.makedirs(os.path.join(model_dir, "transformer"), exist_ok=True)
    conf = {k: cfg[k] for k in ("dim", "n_layers", "cap_feat_dim", "in_channels", "patch_size",
                                "rope_theta", "axes_dims")}
    conf.update(_class_name="ZImageTransformer2DModel", n_refiner_layers=cfg["n_refiner"],
                n_heads=cfg["dim"] // 128)
    with open(os.path.join(model_dir, "transformer", "config.json"), "w") as f:
        json.dump(conf, f, indent=1)
    with open(os.path.join(model_dir, "model_index.json"), "w") as f:
        json.dump({"_class_name": "ZImagePipeline"}, f)
    path = os.path.join(model_dir, "transformer", "diffusion_pytorch_model.safetensors")
    if not keep:
        write_safetensors_generated(path, zimage_tensor_specs(cfg),
                                    lambda n, shp, kind: gen_tensor(seed, n, shp, kind, std, norm_mode))
        return None
    bits = {n: gen_tensor(seed, n, shp, kind, std, norm_mode) for n, shp, kind in zimage_tensor_specs(cfg)}
    write_safetensors(path, bits)
    return {n: bf16_bits_to_f32(b) for n, b in bits.items()}


def zimage_weights(cfg: dict, seed: int, std: float = 0.02, norm_mode: str = "random"):
    return {n: bf16_bits_to_f32(gen_tensor(seed, n, shp, kind, std, norm_mode))
            for n, shp, kind in zimage_tensor_specs(cfg)}


def zimage_ffn_dim(dim: int) -> int:
    """ffn width used by the reference when no weight says otherwise: 8*dim/3 rounded up to 256."""
    return (8 * dim // 3 + 255) // 256 * 256


# ------------------------------------------------------------------ Flux VAE
def vae_tensor_specs(z: int = 32, zimage: bool = False) -> list[tuple[str, tuple, str]]:
    """Tensors of the Flux autoencoder as the reference's loader reads them
    (iris_vae_load_safetensors_ex, iris_vae.c:1227-1385: base 128 channels,
    multipliers 1/2/4/4, two resnets per encoder level and three per decoder
    level, one attention in each mid block, batch-norm latent statistics).
    zimage: the Z-Image autoencoder, which has neither the batch-norm latent
    statistics nor the quant / post-quant 1x1 convolutions (the loader treats
    both as optional, :1333-1363)."""
    mult = [1, 2, 4, 4]
    s = []

    def resblock(prefix, cin, cout):
        s.extend([(f"{prefix}.norm1.weight", (cin,), "gn_w"), (f"{prefix}.norm1.bias", (cin,), "bias"),
                  (f"{prefix}.conv1.weight", (cout, cin, 3, 3), "conv"), (f"{prefix}.conv1.bias", (cout,), "bias"),
                  (f"{prefix}.norm2.weight", (cout,), "gn_w"), (f"{prefix}.norm2.bias", (cout,), "bias"),
                  (f"{prefix}.conv2.weight", (cout, cout, 3, 3), "conv"), (f"{prefix}.conv2.bias", (cout,), "bias")])
        if cin != cout:
            s.extend([(f"{prefix}.conv_shortcut.weight", (cout, cin, 1, 1), "conv"),
                      (f"{prefix}.conv_shortcut.bias", (cout,), "bias")])

    def attn(prefix, c):
        s.extend([(f"{prefix}.group_norm.weight", (c,), "gn_w"), (f"{prefix}.group_norm.bias", (c,), "bias")])
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            s.extend([(f"{prefix}.{n}.weight", (c, c), "conv"), (f"{prefix}.{n}.bias", (c,), "bias")])

    s.extend([("encoder.conv_in.weight", (128, 3, 3, 3), "conv"), ("encoder.conv_in.bias", (128,), "bias")])
    for level in range(4):
        ch = 128 * mult[level]
        prev = 128 if level == 0 else 128 * mult[level - 1]
        for r in range(2):
            resblock(f"encoder.down_blocks.{level}.resnets.{r}", prev if (r == 0 and level > 0) else ch, ch)
    for i in range(3):
        ch = 128 * mult[i]
        s.extend([(f"encoder.down_blocks.{i}.downsamplers.0.conv.weight", (ch, ch, 3, 3), "conv"),
                  (f"encoder.down_blocks.{i}.downsamplers.0.conv.bias", (ch,), "bias")])
    resblock("encoder.mid_block.resnets.0", 512, 512)
    attn("encoder.mid_block.attentions.0", 512)
    resblock("encoder.mid_block.resnets.1", 512, 512)
    s.extend([("encoder.conv_norm_out.weight", (512,), "gn_w"), ("encoder.conv_norm_out.bias", (512,), "bias"),
              ("encoder.conv_out.weight", (2 * z, 512, 3, 3), "conv"), ("encoder.conv_out.bias", (2 * z,), "bias")])
    if not zimage:
        s.extend([("quant_conv.weight", (2 * z, 2 * z, 1, 1), "conv"), ("quant_conv.bias", (2 * z,), "bias")])
    s.extend([("decoder.conv_in.weight", (512, z, 3, 3), "conv"), ("decoder.conv_in.bias", (512,), "bias")])
    resblock("decoder.mid_block.resnets.0", 512, 512)
    attn("decoder.mid_block.attentions.0", 512)
    resblock("decoder.mid_block.resnets.1", 512, 512)
    for level in range(3, -1, -1):
        ch = 128 * mult[level]
        prev = 512 if level == 3 else 128 * mult[level + 1]
        for r in range(3):
            resblock(f"decoder.up_blocks.{3 - level}.resnets.{r}", prev if r == 0 else ch, ch)
    for i in range(3):
        ch = 128 * mult[3 - i]
        s.extend([(f"decoder.up_blocks.{i}.upsamplers.0.conv.weight", (ch, ch, 3, 3), "conv"),
                  (f"decoder.up_blocks.{i}.upsamplers.0.conv.bias", (ch,), "bias")])
    s.extend([("decoder.conv_norm_out.weight", (128,), "gn_w"), ("decoder.conv_norm_out.bias", (128,), "bias"),
              ("decoder.conv_out.weight", (3, 128, 3, 3), "conv"), ("decoder.conv_out.bias", (3,), "bias")])
    if not zimage:
        s.extend([("bn.running_mean", (4 * z,), "bn_mean"), ("bn.running_var", (4 * z,), "bn_var"),
                  ("post_quant_conv.weight", (z, z, 1, 1), "conv"), ("post_quant_conv.bias", (z,), "bias")])
    return s


# Z-Image autoencoder latent scaling (its vae/config.json; read by the
# reference through iris_parse_vae_config, iris_vae_config.h)
ZIMAGE_VAE_SCALING = 0.3611
ZIMAGE_VAE_SHIFT = 0.1159


def _vae_tensor(seed: int, name: str, shp: tuple, kind: str) -> np.ndarray:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    g = rng.standard_normal(shp, dtype=np.float32)
    if kind == "conv":
        x = g / np.float32(np.sqrt(np.prod(shp[1:])))
    elif kind == "gn_w":
        x = 1.0 + 0.1 * g
    elif kind == "bn_mean":
        x = 0.5 * g
    elif kind == "bn_var":
        x = 1.0 + np.abs(0.2 * g)
    else:
        x = 0.02 * g
    return f32_to_bf16_bits(x.astype(np.float32))


def vae_weights(seed: int, z: int = 32, zimage: bool = False) -> dict[str, np.ndarray]:
    """f32 (bf16-valued) tensors of make_vae_model without disk I/O."""
    return {n: bf16_bits_to_f32(_vae_tensor(seed, n, shp, kind)) for n, shp, kind in vae_tensor_specs(z, zimage)}


def make_vae_model(model_dir: str, seed: int, z: int = 32, zimage: bool = False) -> str:
    """Random autoencoder (bf16 safetensors) under model_dir/vae/; returns the
    weights file.  Convolutions ~ N(0, 1/fan_in) so activations keep O(1)
    scale through the decoder; GroupNorm scales 1 + N(0, 0.1); batch-norm
    latent statistics mean N(0, 0.5), variance 1 + |N(0, 0.2)|.  zimage: the
    Z-Image variant (no batch-norm statistics or quant convolutions; latent
    scaling and shift in config.json)."""
    os.makedirs(os.path.join(model_dir, "vae"), exist_ok=True)
    cfg = {"_class_name": "AutoencoderKLFlux2", "latent_channels": z}
    if zimage:
        cfg = {"_class_name": "AutoencoderKL", "latent_channels": z,
               "scaling_factor": ZIMAGE_VAE_SCALING, "shift_factor": ZIMAGE_VAE_SHIFT}
    with open(os.path.join(model_dir, "vae", "config.json"), "w") as f:
        json.dump(cfg, f)
    bits = {name: _vae_tensor(seed, name, shp, kind) for name, shp, kind in vae_tensor_specs(z, zimage)}
    path = os.path.join(model_dir, "vae", "diffusion_pytorch_model.safetensors")
    write_safetensors(path, bits)
    return path



# ------------------------------------------------------------------ Qwen3 text encoder
# Qwen3-4B as Flux.2 Klein uses it (iris_qwen3.c:1436-1447 defaults)
QWEN3_4B = dict(hidden_size=2560, intermediate_size=9728, num_attention_heads=32, num_key_value_heads=8,
                head_dim=128, vocab_size=151936, num_hidden_layers=36, rope_theta=1000000.0)


def qwen3_tensor_specs(cfg: dict, layers: int | None = None) -> list[tuple[str, tuple, str]]:
    """Tensors of the Qwen3 text encoder as the reference's loader reads them
    (load_layer_weights / qwen3_model_load, iris_qwen3.c:1254-1300, :1604-1619).
    layers: how many decoder layers to emit (default: all)."""
    H, F = cfg["hidden_size"], cfg["intermediate_size"]
    q, kv = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]
    s = [("model.embed_tokens.weight", (cfg["vocab_size"], H), "embed")]
    for i in range(cfg["num_hidden_layers"] if layers is None else layers):
        p = f"model.layers.{i}."
        s += [(p + "input_layernorm.weight", (H,), "norm"), (p + "post_attention_layernorm.weight", (H,), "norm"),
              (p + "self_attn.q_proj.weight", (q, H), "linear"), (p + "self_attn.k_proj.weight", (kv, H), "linear"),
              (p + "self_attn.v_proj.weight", (kv, H), "linear"), (p + "self_attn.o_proj.weight", (H, q), "linear"),
              (p + "self_attn.q_norm.weight", (cfg["head_dim"],), "norm"),
              (p + "self_attn.k_norm.weight", (cfg["head_dim"],), "norm"),
              (p + "mlp.gate_proj.weight", (F, H), "linear"), (p + "mlp.up_proj.weight", (F, H), "linear"),
              (p + "mlp.down_proj.weight", (H, F), "linear")]
    s += [("model.norm.weight", (H,), "norm")]
    return s


def _qwen3_tensor(seed: int, name: str, shp: tuple, kind: str) -> np.ndarray:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    g = rng.standard_normal(shp, dtype=np.float32)
    if kind == "linear":
        x = g / np.float32(np.sqrt(shp[1]))
    elif kind == "norm":
        x = 1.0 + 0.1 * g
    else:  # embeddings
        x = g
    return f32_to_bf16_bits(x.astype(np.float32))


def qwen3_weights(cfg: dict, seed: int) -> dict[str, np.ndarray]:
    """f32 (bf16-valued) tensors of make_qwen3_model without disk I/O."""
    return {n: bf16_bits_to_f32(_qwen3_tensor(seed, n, shp, kind)) for n, shp, kind in qwen3_tensor_specs(cfg)}


def make_qwen3_model(model_dir: str, cfg: dict, seed: int) -> str:
    """Random Qwen3 text encoder (bf16) under model_dir/text_encoder/ in the
    layout the reference opens (config.json, model.safetensors.index.json and
    model-00001-of-00001.safetensors, iris_qwen3.c:1450-1520); projections
    N(0, 1/fan_in), norm scales 1 + N(0, 0.1), embeddings N(0, 1).  Returns
    the text_encoder directory."""
    d = os.path.join(model_dir, "text_encoder")
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(dict(cfg, architectures=["Qwen3ForCausalLM"]), f, indent=1)
    bits = {name: _qwen3_tensor(seed, name, shp, kind) for name, shp, kind in qwen3_tensor_specs(cfg)}
    shard = "model-00001-of-00001.safetensors"
    write_safetensors(os.path.join(d, shard), bits)
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": {n: shard for n in bits}}, f)
    return d
