"""Generate the golden fixtures in this directory from the REFERENCE itself.

Run where the reference tree exists (it is read-only and absent on GPU boxes):

    make -C oracle && python tests/golden/make_golden.py        # everything
    python tests/golden/make_golden.py lora                      # lora_fixture.npz only
    python tests/golden/make_golden.py ip                        # ip_fixture.npz only

Each fixture is produced by the reference's own C code, compiled from its
unmodified sources by oracle/Makefile and driven through
oracle/ref_harness.c (``make generic`` math).  Model weights are not stored:
they are regenerated bit-identically from (config, seed, std, norm_mode) by
oracle/model_gen.py, which is also what wrote the safetensors the reference
loaded.  Inputs and outputs are stored as float32 arrays.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from oracle import model_gen as mg  # noqa: E402
from oracle.ref_lib import (RefFlux, RefLib, RefZImage, ref_init_noise,  # noqa: E402
                            ref_official_schedule, ref_zimage_schedule)

OUT = os.path.dirname(os.path.abspath(__file__))

from cases import (FLUX_CASES, ZIMAGE_CASES, block_inputs, ref_inputs, rng_inputs,  # noqa: E402
                   zimage_inputs)


def flux_case(ref: RefLib, name: str, spec: dict) -> dict:
    out = {}
    with tempfile.TemporaryDirectory() as d:
        mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
        rf = RefFlux(ref, d)
        dims = mg.flux_dims(spec["cfg"])
        h, w = spec["img"]
        lat, ctx = rng_inputs(spec["seed"] + 100, dims["channels"], h, w, spec["txt"], dims["text_dim"])
        for t in (1.0, 0.7):
            out[f"v_t{t}"] = rf.forward(lat, ctx, t)
        # per-block: double block 0 and single block 0 on seeded hidden states
        t_emb = rf.temb(0.7)
        mods = rf.mods(t_emb)
        out["t_emb"] = t_emb
        for k, v in mods.items():
            out[f"mod_{k}"] = v
        img_h, txt_h = block_inputs(spec, dims["hidden"])
        oi, ot = rf.double_block(0, img_h, txt_h, mods["dbl_img"], mods["dbl_txt"], h, w)
        out["dbl_out_img"], out["dbl_out_txt"] = oi, ot
        hid = np.concatenate([txt_h, img_h])
        out["sgl_out"] = rf.single_block(0, hid, t_emb, h, w, spec["txt"])
        # 4-step Euler from seeded noise on the official schedule
        z0 = ref_init_noise(ref, dims["channels"], h, w, 42)
        sched = ref_official_schedule(ref, 4, h * w)
        out["z0"], out["sched4"] = z0, sched
        out["z4"] = rf.sample_euler(z0, ctx, sched)
        if name == "flux_tiny":
            # multi-reference forward: two reference latents, T offsets 10 and 20
            refs, ctx_u = ref_inputs(dims["channels"], ctx.shape)
            out["v_refs"] = rf.forward_refs(lat, refs, ctx, 0.6)
            # CFG: 3 steps, guidance 4.0, uncond context of the same length
            sched3 = ref_official_schedule(ref, 3, h * w)
            out["sched3"] = sched3
            out["z_cfg"] = rf.sample_euler_cfg(z0, ctx, ctx_u, 4.0, sched3)
        rf.close()
    meta = dict(cfg=spec["cfg"], seed=spec["seed"], std=spec["std"], norm_mode=spec["norm_mode"],
                img=list(spec["img"]), txt=spec["txt"], variant="generic")
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return out


def zimage_case(name: str, spec: dict) -> dict:
    """Z-Image outputs from the alias-safe reference build (oracle/alias_safe_matmul.c:
    the reference's code with its in-place attention output GEMM made alias-safe),
    plus the unmodified builds' velocities, which disagree with each other."""
    out = {}
    lat, cap = zimage_inputs(spec)
    with tempfile.TemporaryDirectory() as d:
        mg.make_zimage_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
        for variant, tag in (("generic_as", ""), ("generic", "_unfixed_generic"), ("blas", "_unfixed_blas")):
            ref = RefLib(variant)
            rz = RefZImage(ref, d, spec["cfg"])
            for t in ((0.3, 0.9) if not tag else (0.3,)):
                out[f"v_t{t}{tag}"] = rz.forward(lat, cap, t)
            if not tag:
                n_img = (spec["latent"][1] // 2) * (spec["latent"][2] // 2)
                sched = ref_zimage_schedule(ref, 3, n_img)
                z0 = ref_init_noise(ref, *spec["latent"], 42)
                out["sched3"], out["z0"] = sched, z0
                out["z3"] = rz.sample_euler(z0, cap, sched)
            rz.close()
    meta = dict(cfg=spec["cfg"], seed=spec["seed"], std=spec["std"], norm_mode=spec["norm_mode"],
                latent=list(spec["latent"]), cap=spec["cap"], variant="generic_as")
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    return out


def sampler_case(ref: RefLib) -> dict:
    out = {}
    for steps, seq in ((4, 1024), (4, 256), (50, 4096), (28, 4608), (4, 12544)):
        out[f"official_{steps}_{seq}"] = ref_official_schedule(ref, steps, seq)
    out["zimage_8"] = ref_zimage_schedule(ref, 8, 4096)
    out["zimage_9"] = ref_zimage_schedule(ref, 9, 4096)
    out["noise_4x16x16_s42"] = ref_init_noise(ref, 4, 16, 16, 42)
    out["noise_4x8x12_s7"] = ref_init_noise(ref, 4, 8, 12, 7)
    big = ref_init_noise(ref, 128, 32, 32, 1234)
    out["noise_128x32x32_s1234_head"] = big.reshape(-1)[:512].copy()
    out["noise_128x32x32_s1234_sum"] = np.array([big.astype(np.float64).sum(),
                                                 (big.astype(np.float64) ** 2).sum()])
    return out


REF_TREE = os.environ.get("IRIS_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))


def lora_fixture() -> dict:
    """The reference's own LoRA golden fixture (debug/fixtures/lora: an MLX
    LoRALinear export, rank 4, dim 8, seq 5, checked by debug/test_lora.c),
    stored as arrays: every tensor of lora.safetensors under its name, the
    input x [5, 8] and the goldens (to_q delta [5, 8], single linear1 delta
    [5, 12], single linear2 delta [5, 8])."""
    from oracle.lora_oracle import read_safetensors
    d = os.path.join(REF_TREE, "debug", "fixtures", "lora")
    out = {f"t:{k}": v for k, v in read_safetensors(os.path.join(d, "lora.safetensors")).items()}
    out["x"] = np.fromfile(os.path.join(d, "x.bin"), "<f4").reshape(5, 8)
    out["golden"] = np.fromfile(os.path.join(d, "golden.bin"), "<f4").reshape(5, 8)
    out["golden_single1"] = np.fromfile(os.path.join(d, "golden_single1.bin"), "<f4").reshape(5, 12)
    out["golden_single2"] = np.fromfile(os.path.join(d, "golden_single2.bin"), "<f4").reshape(5, 8)
    return out


IP_BUNDLES = ("bundle", "bundle_csd", "bundle_hybrid", "bundle_int8")
IP_BINS = ("in_siglip", "in_csd", "in_hybrid", "in_img_q",
           "gold_ip_embeds", "gold_k_ip_b0", "gold_v_ip_b0", "gold_inject_b0",
           "gold_ip_embeds_csd", "gold_k_ip_b0_csd", "gold_v_ip_b0_csd", "gold_inject_b0_csd",
           "gold_ip_embeds_hybrid", "gold_k_ip_b0_hybrid", "gold_v_ip_b0_hybrid", "gold_inject_b0_hybrid",
           "gold_ip_embeds_int8", "gold_k_ip_b0_int8", "gold_v_ip_b0_int8", "gold_inject_b0_int8")


def ip_fixture() -> dict:
    """The reference's own IP-Adapter golden fixture (debug/fixtures/ip_adapter,
    checked by debug/test_ip_adapter.c): the siglip, csd, hybrid and int8
    bundles byte for byte (adapter_meta.json text and adapter_weights.safetensors
    as uint8 arrays, to be written back to a directory by the tests), the inputs
    and the goldens (f32, shapes from shapes.json)."""
    d = os.path.join(REF_TREE, "debug", "fixtures", "ip_adapter")
    out = {}
    for b in IP_BUNDLES:
        for fn, key in (("adapter_meta.json", "meta"), ("adapter_weights.safetensors", "weights")):
            with open(os.path.join(d, b, fn), "rb") as f:
                out[f"{b}:{key}"] = np.frombuffer(f.read(), np.uint8).copy()
    with open(os.path.join(d, "shapes.json")) as f:
        shapes = json.load(f)
    out["shapes_json"] = np.frombuffer(json.dumps(shapes).encode(), np.uint8).copy()
    for n in IP_BINS:
        x = np.fromfile(os.path.join(d, n + ".bin"), "<f4")
        out[n] = x.reshape(shapes[n]) if n in shapes else x
    return out


def main():
    if sys.argv[1:] == ["ip"]:
        np.savez_compressed(os.path.join(OUT, "ip_fixture.npz"), **ip_fixture())
        print("wrote ip_fixture")
        return
    if sys.argv[1:] == ["lora"]:
        np.savez_compressed(os.path.join(OUT, "lora_fixture.npz"), **lora_fixture())
        print("wrote lora_fixture")
        return
    ref = RefLib("generic")
    for name, spec in FLUX_CASES.items():
        data = flux_case(ref, name, spec)
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **data)
        print("wrote", name, {k: v.shape for k, v in data.items() if k != "meta"})
    for name, spec in ZIMAGE_CASES.items():
        data = zimage_case(name, spec)
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **data)
        print("wrote", name, {k: v.shape for k, v in data.items() if k != "meta"})
    np.savez_compressed(os.path.join(OUT, "sampler.npz"), **sampler_case(ref))
    print("wrote sampler")
    np.savez_compressed(os.path.join(OUT, "lora_fixture.npz"), **lora_fixture())
    print("wrote lora_fixture")
    np.savez_compressed(os.path.join(OUT, "ip_fixture.npz"), **ip_fixture())
    print("wrote ip_fixture")


if __name__ == "__main__":
    main()
