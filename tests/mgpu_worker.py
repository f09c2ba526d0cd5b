"""One rank of the multi-GPU tests (tests/test_multigpu_gpu.py), launched by
torch.distributed.run with one process per GPU.  The gloo process group only
carries the NCCL unique id and the result barrier; every collective of the
backend goes through its own NCCL communicator.

usage: python -m torch.distributed.run ... mgpu_worker.py MODE OUT_DIR
  cfg_pair  CFG branches split over rank pairs vs the one-GPU CFG sampler and
            the reference golden
  tp        tensor-parallel shards (tp = world) vs the unsharded model and,
            at tp 2, the reference golden
  tp_k9b    Klein-9B-width blocks and forward, sharded, vs the unsharded model
            and the reference's CPU build
  nojoin    rank 0 creates a communicator that rank 1 never joins: the join
            must end in a timeout status, not a hang
"""
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "iris.c_b200"), os.path.join(HERE, "golden"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402

import cases  # noqa: E402
import iris_cuda  # noqa: E402
from gpu_util import rel_l2  # noqa: E402
from oracle import flux_oracle as fo  # noqa: E402
from oracle import model_gen as mg  # noqa: E402

# 16 heads: even head pairs per shard up to tp = 8
TP_CFG = dict(num_attention_heads=16, attention_head_dim=128, num_layers=1, num_single_layers=2,
              joint_attention_dim=128, in_channels=128, mlp_ratio=3.0, rope_theta=2000.0)


def golden(name):
    return dict(np.load(os.path.join(HERE, "golden", f"{name}.npz")))


def run_cfg_pair(rank, world, out_dir, exchange):
    group, r = iris_cuda.comm_init_group(exchange, rank, world, 2)
    spec = cases.FLUX_CASES["flux_tiny"]
    g = golden("flux_tiny")
    d = os.path.join(out_dir, f"model_r{rank}")
    mg.make_flux_model(d, spec["cfg"], spec["seed"], spec["std"], spec["norm_mode"])
    m = iris_cuda.Flux.load(d)
    dims = mg.flux_dims(spec["cfg"])
    h, wd = spec["img"]
    _, ctx = cases.rng_inputs(spec["seed"] + 100, dims["channels"], h, wd, spec["txt"], dims["text_dim"])
    _, ctx_u = cases.ref_inputs(dims["channels"], ctx.shape)
    zp = m.sample_euler(g["z0"], ctx, g["sched3"], txt_uncond=ctx_u, guidance=4.0, cfg_pair=True)
    z1 = m.sample_euler(g["z0"], ctx, g["sched3"], txt_uncond=ctx_u, guidance=4.0)
    m.close()
    return dict(group=list(group), pair_rank=r, rel_golden=rel_l2(zp, g["z_cfg"]),
                max_abs_vs_one_gpu=float(np.abs(zp - z1).max()))


def run_tp(rank, world, out_dir, exchange):
    group, r = iris_cuda.comm_init_group(exchange, rank, world, world)
    res = dict(tp=world)
    cases_to_run = [("tp_cfg", TP_CFG, 21, 0.04, "unit", (6, 10), 40)]
    if world == 2:
        s = cases.FLUX_CASES["flux_small"]
        cases_to_run.append(("flux_small", s["cfg"], s["seed"], s["std"], s["norm_mode"], s["img"], s["txt"]))
    for name, cfg, seed, std, norm, (h, wd), txt in cases_to_run:
        d = os.path.join(out_dir, f"{name}_r{rank}")
        w = mg.make_flux_model(d, cfg, seed, std, norm)
        dims = mg.flux_dims(cfg)
        lat, ctx = cases.rng_inputs(seed + 100, dims["channels"], h, wd, txt, dims["text_dim"])
        full = iris_cuda.Flux.load(d)
        v_full = {t: full.forward(lat, ctx, t) for t in (1.0, 0.7)}
        img_h = np.random.default_rng(seed + 200).standard_normal((h * wd, dims["hidden"])).astype(np.float32)
        txt_h = np.random.default_rng(seed + 201).standard_normal((txt, dims["hidden"])).astype(np.float32)
        hid = np.concatenate([txt_h, img_h])
        b_full = [full.run_block(k, 0, hid, txt, h, wd, 0.7) for k in (0, 1)]
        # a LoRA folded into the shards' rows / columns (fused or separate Q|K|V,
        # interleaved gate/up rows, split output-projection inputs)
        lp = os.path.join(out_dir, f"{name}_lora_r{rank}.safetensors")
        mg.make_flux_lora(lp, cfg, "bfl" if name == "tp_cfg" else "diffusers", rank=8, seed=9, std=0.15)
        full.load_lora(lp, 0.8)
        v_full_lora = full.forward(lat, ctx, 0.7)
        full.close()
        shard = iris_cuda.Flux.load(d, tp_rank=r, tp_size=world)
        entry = {}
        for t in (1.0, 0.7):
            v = shard.forward(lat, ctx, t)
            ref = fo.forward(w, cfg, lat, ctx, t)
            entry[f"v_t{t}_vs_full"] = rel_l2(v, v_full[t])
            entry[f"v_t{t}_vs_oracle"] = rel_l2(v, ref)
            entry[f"v_t{t}_full_vs_oracle"] = rel_l2(v_full[t], ref)
        for k in (0, 1):
            entry[f"block{k}_vs_full"] = rel_l2(shard.run_block(k, 0, hid, txt, h, wd, 0.7), b_full[k])
        if name == "flux_small":
            g = golden(name)
            entry["v_t1.0_vs_golden"] = rel_l2(shard.forward(lat, ctx, 1.0), g["v_t1.0"])
            z = shard.sample_euler(g["z0"], ctx, g["sched4"])
            entry["z4_vs_golden"] = rel_l2(z, g["z4"])
        shard.load_lora(lp, 0.8)
        entry["lora_v_t0.7_vs_full"] = rel_l2(shard.forward(lat, ctx, 0.7), v_full_lora)
        entry["weight_bytes"] = shard.weight_bytes()
        shard.close()
        res[name] = entry
    return res


K9B_WIDTH = dict(mg.KLEIN_9B, num_layers=1, num_single_layers=1)


def run_tp_k9b(rank, world, out_dir, exchange):
    """Klein-9B width (hidden 4096, 32 heads, context 12288), one double and
    one single block, sharded over the ranks: both blocks and a forward
    against the unsharded model and (rank 0) the reference's own CPU build."""
    group, r = iris_cuda.comm_init_group(exchange, rank, world, world)
    d = os.path.join(out_dir, f"k9b_r{rank}")
    mg.make_flux_model(d, K9B_WIDTH, seed=909, std=0.02, norm_mode="unit", keep=False)
    rng = np.random.default_rng(4)
    ph, pw, nt = 24, 40, 96
    img_h = rng.standard_normal((ph * pw, 4096)).astype(np.float32)
    txt_h = rng.standard_normal((nt, 4096)).astype(np.float32)
    hid = np.concatenate([txt_h, img_h])
    r5 = np.random.default_rng(5)
    lat = r5.standard_normal((128, 14, 18)).astype(np.float32)
    ctx = r5.standard_normal((77, 12288)).astype(np.float32)
    full = iris_cuda.Flux.load(d)
    b_full = [full.run_block(k, 0, hid, nt, ph, pw, 0.9) for k in (0, 1)]
    v_full = full.forward(lat, ctx, 0.7)
    full.close()
    shard = iris_cuda.Flux.load(d, tp_rank=r, tp_size=world)
    b = [shard.run_block(k, 0, hid, nt, ph, pw, 0.9) for k in (0, 1)]
    v = shard.forward(lat, ctx, 0.7)
    shard.close()
    res = dict(tp=world, block0_vs_full=rel_l2(b[0], b_full[0]), block1_vs_full=rel_l2(b[1], b_full[1]),
               v_vs_full=rel_l2(v, v_full))
    if rank == 0:
        import ref_worker
        (ri, rt, rs), v_ref = ref_worker.flux(d, [("blocks", 0, img_h, txt_h, ph, pw, 0.9),
                                                   ("forward", lat, ctx, 0.7)])
        res.update(dbl_vs_reference=rel_l2(b[0], np.concatenate([rt, ri])),
                   dbl_delta_vs_reference=rel_l2(b[0] - hid, np.concatenate([rt, ri]) - hid),
                   sgl_vs_reference=rel_l2(b[1], rs), sgl_delta_vs_reference=rel_l2(b[1] - hid, rs - hid),
                   v_vs_reference=rel_l2(v, v_ref))
    return res


def run_nojoin(rank, world, out_dir, exchange):
    if rank == 0:
        uid = iris_cuda.comm_unique_id()
        exchange(None)
        t0 = time.time()
        try:
            iris_cuda.comm_init(uid, 2, 0)
            err = ""
        except iris_cuda.IrisCudaError as e:
            err = str(e)
        return dict(error=err, seconds=time.time() - t0, world_after=iris_cuda.lib().iris_cuda_comm_world())
    exchange(None)  # rank 1 never joins the NCCL communicator
    return dict(error="", seconds=0.0)


def main():
    mode, out_dir = sys.argv[1], sys.argv[2]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
    assert iris_cuda.lib().iris_cuda_init(local) == 0, iris_cuda.last_error()

    def exchange(obj):
        lst = [None] * world
        dist.all_gather_object(lst, obj)
        return lst

    fn = dict(cfg_pair=run_cfg_pair, tp=run_tp, tp_k9b=run_tp_k9b, nojoin=run_nojoin)[mode]
    res = fn(rank, world, out_dir, exchange)
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    dist.barrier()
    iris_cuda.comm_destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
