"""Reference computations in a child process — TEST INFRASTRUCTURE ONLY.

The full-width parity tests (tests/test_baseline_configs_gpu.py) run the
reference's own CPU build (oracle/_ref/libiris_ref_blas*.so) on models of
up to 7.7 GB.  Each model is evaluated in a fresh process started with the
`spawn` method, for three reasons:
* the f32 copy the reference loader makes (15.4 GB for Klein-4B) is released
  when the child exits;
* the reference's BLAS attention caches its thread count from the first model
  it sees (get_attn_num_threads, iris_transformer_flux.c:1773), so one model
  per process keeps every head count correct;
* a spawned child shares no CUDA state with the test process.
"""
from __future__ import annotations

import multiprocessing as mp
import os
from concurrent.futures import ProcessPoolExecutor


def _flux_jobs(model_dir: str, jobs: list) -> list:
    from oracle.ref_lib import RefFlux, RefLib
    ref = RefLib("blas")
    ref.set_threads(os.cpu_count() or 1)
    rf = RefFlux(ref, model_dir)
    out = []
    for job in jobs:
        kind = job[0]
        if kind == "forward":
            _, lat, ctx, t = job
            out.append(rf.forward(lat, ctx, t))
        elif kind == "blocks":
            # double block `idx` on (img, txt) and single block `idx` on [TXT, IMG]
            _, idx, img_h, txt_h, ph, pw, t = job
            import numpy as np
            t_emb = rf.temb(t)
            mods = rf.mods(t_emb)
            oi, ot = rf.double_block(idx, img_h, txt_h, mods["dbl_img"], mods["dbl_txt"], ph, pw)
            hid = np.concatenate([txt_h, img_h])
            so = rf.single_block(idx, hid, t_emb, ph, pw, txt_h.shape[0])
            out.append((oi, ot, so))
        else:
            raise ValueError(kind)
    rf.close()
    return out


def _zimage_forward(model_dir: str, cfg: dict, lat, cap, t: float):
    from oracle.ref_lib import RefLib, RefZImage
    ref = RefLib("blas_as")  # alias-safe attention output GEMM (oracle/alias_safe_matmul.c)
    ref.set_threads(os.cpu_count() or 1)
    rz = RefZImage(ref, model_dir, cfg)
    v = rz.forward(lat, cap, t)
    rz.close()
    return v


def _run(fn, *args):
    with ProcessPoolExecutor(1, mp_context=mp.get_context("spawn")) as ex:
        return ex.submit(fn, *args).result()


def flux(model_dir: str, jobs: list) -> list:
    """Run ("forward", latent, ctx, t) and ("blocks", idx, img_h, txt_h, ph, pw, t) jobs
    on the reference Flux transformer loaded from model_dir."""
    return _run(_flux_jobs, model_dir, jobs)


def zimage_forward(model_dir: str, cfg: dict, lat, cap, t: float):
    return _run(_zimage_forward, model_dir, cfg, lat, cap, t)
