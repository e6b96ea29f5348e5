"""The tensor split over NCCL on two GPUs (skipped with fewer): each rank
builds its cut with `tensor_split.build_block`, runs the block through the C
ABI and all-reduces the float32 partials; rank 0 compares the result with
the oracle's tensor-split block."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from knurlogic_b200 import synth, tensor_split
from oracle import moe_ref as R
from tests.conftest import oracle_params, to_np

pytestmark = pytest.mark.gpu
N = 2
CFG = synth.MoEConfig("tp2", 16, 4, 512, 256, 128, 24)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=N, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = synth.make_weights(CFG, seed=8, scales="random")
        x = synth.make_input(CFG, seed=8)
        blk = tensor_split.build_block({k: v.to(f"cuda:{rank}") for k, v in w.items()}, CFG.top_k,
                                       rank=rank, n=N, group=dist.group.WORLD)
        y = to_np(blk(x.to(f"cuda:{rank}")))
        if rank == 0:
            ref = R.tp_sparse_moe_block(to_np(x), oracle_params(w), CFG.top_k, vq=True, n=N)
            scale = float(np.abs(ref).max())
            q.put(float(np.abs(y - ref).max()) / scale)
    except Exception as e:  # report, never hang the other rank's test
        q.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < N, reason="needs 2 GPUs")
def test_two_gpu_tensor_split_matches_the_oracle():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(N)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    rel = q.get(timeout=5)
    assert isinstance(rel, float), rel
    assert rel <= 1e-2
