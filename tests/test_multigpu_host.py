"""Host-side logic of the multi-GPU paths, on CPU with gloo ranks.

The NCCL id exchange and group formation of iris_cuda.comm_init_group run
over a real world_size-4 gloo process group; the two library calls that need
a GPU (unique id, communicator join) are replaced by fakes that record what
each rank was given.  A rank that raises before the exchange makes the others
fail with an error within the process-group timeout instead of waiting.
"""
import datetime
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import iris_cuda


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _exchange(world):
    def ex(obj):
        lst = [None] * world
        dist.all_gather_object(lst, obj)
        return lst
    return ex


def _group_worker(rank, world, port, group_size, q):
    _init(rank, world, port)
    joined = {}
    iris_cuda.comm_unique_id = lambda: f"id-of-{rank}".encode().ljust(128, b"\0")
    iris_cuda.comm_init = lambda uid, w, r: joined.update(uid=uid.rstrip(b"\0").decode(), world=w, rank=r)
    group, r = iris_cuda.comm_init_group(_exchange(world), rank, world, group_size)
    q.put((rank, list(group), r, joined))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("group_size", [2, 4])
def test_groups_share_the_id_of_their_first_rank(group_size):
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_group_worker, args=(r, world, port, group_size, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, group, r, joined in out:
        first = rank - rank % group_size
        assert group == list(range(first, first + group_size))
        assert r == rank % group_size
        assert joined == dict(uid=f"id-of-{first}", world=group_size, rank=r)


def _dying_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        raise SystemExit(3)  # leaves before the exchange
    try:
        iris_cuda.comm_unique_id = lambda: b"x" * 128
        iris_cuda.comm_init = lambda *a: None
        iris_cuda.comm_init_group(_exchange(world), rank, world, 2)
        q.put((rank, "no error"))
    except Exception as e:  # gloo reports the lost peer
        q.put((rank, type(e).__name__))


def test_rank_that_leaves_fails_the_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, what = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and what != "no error"


def test_comm_groups_partition():
    assert iris_cuda.comm_groups(8, 2) == [(0, 1), (2, 3), (4, 5), (6, 7)]
    assert iris_cuda.comm_groups(4, 4) == [(0, 1, 2, 3)]
    with pytest.raises(ValueError):
        iris_cuda.comm_groups(6, 4)


def test_no_communicator_by_default():
    lib = iris_cuda.load()
    assert lib.iris_cuda_comm_world() == 1 and lib.iris_cuda_comm_rank() == 0
