"""ORACLE — test infrastructure only; never imported by the product path.

numpy restatement of the reference's LoRA support for the Flux transformer:

* format detection and key routing of ``lora_load`` (iris_lora.c:504; formats
  :87-114; loaders XLabs :240, Kohya :281, Diffusers :342, BFL :423), returning
  the reference's adapter table (``lora_state_t``, iris_lora.h:28-49): per
  double block img/txt q, k, v, proj, per single block linear1 / linear2, each
  ``(A [rank, in], B [out, rank])`` in f32, a fused Q|K|V up matrix split into
  three adapters sharing one A (load_adapter_split_qkv :184);
* ``lora_apply`` (iris_lora.c:43): ``out += scale * (x A^T) B^T``;
* ``merge``: the same update folded into the reference-layout weights,
  ``W + scale * B A`` (f64 product), which is what the blocks compute when the
  hooks (iris_transformer_flux.c:2429-2532, :3818, :3909) add the adapter to
  the output of every adapted linear.  ``flux_oracle.forward`` run on the merged
  weights is the oracle of a forward with a LoRA.

Pinned in tests/test_lora_oracle.py against the reference's own golden
fixture (debug/fixtures/lora, stored as tests/golden/lora_fixture.npz), the
reference loader's adapter tables and the reference forward with a LoRA.
"""
from __future__ import annotations

import json
import struct

import numpy as np

F32 = np.float32

KINDS = ("double_img_q", "double_img_k", "double_img_v", "double_img_proj",
         "double_txt_q", "double_txt_k", "double_txt_v", "double_txt_proj",
         "single_linear1", "single_linear2")

# reference-layout weight each adapter kind adds to (diffusers tensor names
# read by the reference loader, iris_transformer_flux.c:5300-5497)
TARGETS = {
    "double_img_q": "transformer_blocks.{i}.attn.to_q.weight",
    "double_img_k": "transformer_blocks.{i}.attn.to_k.weight",
    "double_img_v": "transformer_blocks.{i}.attn.to_v.weight",
    "double_img_proj": "transformer_blocks.{i}.attn.to_out.0.weight",
    "double_txt_q": "transformer_blocks.{i}.attn.add_q_proj.weight",
    "double_txt_k": "transformer_blocks.{i}.attn.add_k_proj.weight",
    "double_txt_v": "transformer_blocks.{i}.attn.add_v_proj.weight",
    "double_txt_proj": "transformer_blocks.{i}.attn.to_add_out.weight",
    "single_linear1": "single_transformer_blocks.{i}.attn.to_qkv_mlp_proj.weight",
    "single_linear2": "single_transformer_blocks.{i}.attn.to_out.weight",
}


def read_safetensors(path: str) -> dict[str, np.ndarray]:
    """{name: f32 array} in header order (F32 / F16 / BF16)."""
    with open(path, "rb") as f:
        raw = f.read()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, e in hdr.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        buf = raw[base + a:base + b]
        shape = tuple(e["shape"])
        if e["dtype"] == "F32":
            x = np.frombuffer(buf, "<f4").astype(F32)
        elif e["dtype"] == "F16":
            x = np.frombuffer(buf, "<f2").astype(F32)
        elif e["dtype"] == "BF16":
            x = (np.frombuffer(buf, "<u2").astype(np.uint32) << 16).view(F32)
        else:
            continue
        out[name] = x.reshape(shape)
    return out


def detect_format(names) -> str | None:
    """First name that identifies a format decides it (detect_format :95-113)."""
    for n in names:
        if "processor." in n:
            return "xlabs"
        if "lora_unet_" in n:
            return "kohya"
        if ("transformer.transformer_blocks" in n or "transformer.single_transformer_blocks" in n
                or "transformer.x_embedder" in n):
            return "diffusers"
        if "diffusion_model.double_blocks." in n or "base_model.model.double_blocks." in n:
            return "bfl"
    return None


def _pair(t, dk, uk, exp_in=-1, exp_out=-1):
    """load_adapter (:142): both present, 2-D, expected sizes (-1 = unchecked)."""
    if dk not in t or uk not in t:
        return None
    a, b = t[dk], t[uk]
    if a.ndim < 2 or b.ndim < 2:
        return None
    if exp_in >= 0 and a.shape[1] != exp_in:
        return None
    if exp_out >= 0 and b.shape[0] != exp_out:
        return None
    return a.astype(F32), b.astype(F32)


def _split_qkv(t, dk, uk, hidden):
    """load_adapter_split_qkv (:184): B [3H, r] -> three [H, r], A shared."""
    p = _pair(t, dk, uk)
    if p is None or p[1].shape[0] != 3 * hidden:
        return None
    a, b = p
    return [(a, b[j * hidden:(j + 1) * hidden]) for j in range(3)]


def load_lora(path: str, n_double: int, n_single: int, hidden: int):
    """lora_load: {kind: {block: (A, B)}} or None (unknown format / nothing loaded)."""
    t = read_safetensors(path)
    fmt = detect_format(t.keys())
    if fmt is None:
        return None
    L = {k: {} for k in KINDS}
    L["pairs"] = 0  # (down, up) pairs loaded, the reference's `loaded` count

    def put_qkv(stream, i, trio):
        if trio is not None:
            for j, nm in enumerate("qkv"):
                L[f"double_{stream}_{nm}"][i] = trio[j]
            L["pairs"] += 1

    def put(kind, i, p):
        if p is not None:
            L[kind][i] = p
            L["pairs"] += 1

    if fmt in ("xlabs", "kohya", "bfl"):
        pre = "diffusion_model"
        if fmt == "bfl" and any("base_model.model.double_blocks." in n for n in t):
            pre = "base_model.model"
        for i in range(n_double):
            for stream, n in (("img", 1), ("txt", 2)):
                if fmt == "xlabs":
                    q = (f"double_blocks.{i}.processor.qkv_lora{n}.down.weight",
                         f"double_blocks.{i}.processor.qkv_lora{n}.up.weight")
                    pj = (f"double_blocks.{i}.processor.proj_lora{n}.down.weight",
                          f"double_blocks.{i}.processor.proj_lora{n}.up.weight")
                elif fmt == "kohya":
                    q = (f"lora_unet_double_blocks_{i}_{stream}_attn_qkv.lora_down.weight",
                         f"lora_unet_double_blocks_{i}_{stream}_attn_qkv.lora_up.weight")
                    pj = (f"lora_unet_double_blocks_{i}_{stream}_attn_proj.lora_down.weight",
                          f"lora_unet_double_blocks_{i}_{stream}_attn_proj.lora_up.weight")
                else:
                    q = (f"{pre}.double_blocks.{i}.{stream}_attn.qkv.lora_A.weight",
                         f"{pre}.double_blocks.{i}.{stream}_attn.qkv.lora_B.weight")
                    pj = (f"{pre}.double_blocks.{i}.{stream}_attn.proj.lora_A.weight",
                          f"{pre}.double_blocks.{i}.{stream}_attn.proj.lora_B.weight")
                put_qkv(stream, i, _split_qkv(t, *q, hidden))
                put(f"double_{stream}_proj", i, _pair(t, *pj, hidden, hidden))
        if fmt != "xlabs":
            for i in range(n_single):
                for k in (1, 2):
                    if fmt == "kohya":
                        dk = f"lora_unet_single_blocks_{i}_linear{k}.lora_down.weight"
                        uk = f"lora_unet_single_blocks_{i}_linear{k}.lora_up.weight"
                    else:
                        dk = f"{pre}.single_blocks.{i}.linear{k}.lora_A.weight"
                        uk = f"{pre}.single_blocks.{i}.linear{k}.lora_B.weight"
                    put(f"single_linear{k}", i, _pair(t, dk, uk))
    else:
        names = {"img": ("to_q", "to_k", "to_v", "to_out.0"),
                 "txt": ("add_q_proj", "add_k_proj", "add_v_proj", "to_add_out")}
        for i in range(n_double):
            for stream in ("img", "txt"):
                for nm, kind in zip(names[stream], ("q", "k", "v", "proj")):
                    p = f"transformer.transformer_blocks.{i}.attn.{nm}"
                    put(f"double_{stream}_{kind}", i,
                        _pair(t, p + ".lora_A.weight", p + ".lora_B.weight", hidden, hidden))
        for i in range(n_single):
            p = f"transformer.single_transformer_blocks.{i}."
            put("single_linear1", i, _pair(t, p + "attn.to_qkv_mlp_proj.lora_A.weight",
                                           p + "attn.to_qkv_mlp_proj.lora_B.weight"))
            l2 = _pair(t, p + "attn.to_out.lora_A.weight", p + "attn.to_out.lora_B.weight")
            if l2 is None:
                l2 = _pair(t, p + "proj_out.lora_A.weight", p + "proj_out.lora_B.weight")
            put("single_linear2", i, l2)
    if not any(L[k] for k in KINDS):
        return None
    return L


def count(L) -> int:
    """Adapters as the loaders count them (a fused Q|K|V counts once)."""
    return 0 if L is None else L["pairs"]


def lora_apply(adapter, scale: float, x: np.ndarray, out: np.ndarray) -> np.ndarray:
    """out + scale * (x A^T) B^T (iris_lora.c:43)."""
    a, b = adapter
    return (out.astype(np.float64) + scale * ((x.astype(np.float64) @ a.T.astype(np.float64))
                                               @ b.T.astype(np.float64))).astype(F32)


def merge(weights: dict[str, np.ndarray], L, scale: float) -> dict[str, np.ndarray]:
    """Reference-layout weights with every adapter folded in (W + scale * B A)."""
    w = dict(weights)
    if L is None:
        return w
    for kind in KINDS:
        for i, (a, b) in L[kind].items():
            name = TARGETS[kind].format(i=i)
            w[name] = (w[name].astype(np.float64)
                       + scale * (b.astype(np.float64) @ a.astype(np.float64))).astype(F32)
    return w
