"""The tensor split's host side on two gloo ranks (CPU): each rank takes
its cut with `tensor_split.shard_state_dict`, computes its partial block
output (the oracle stands in for the GPU), and `moe.tp_reduce` sums the
partials in float32 and rounds once. The result must equal the oracle's
tensor-split block bit for bit, and each rank's cut must be the one the
oracle makes from the whole weights."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

from knurlogic_b200 import synth, tensor_split
from knurlogic_b200.moe import tp_reduce
from oracle import moe_ref as R
from tests.conftest import oracle_params, to_np

N = 2
CFG = synth.MoEConfig("tp", 8, 2, 256, 128, 64, 6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=N)
    try:
        w = synth.make_weights(CFG, seed=5, scales="random")
        x = to_np(synth.make_input(CFG, seed=5))
        mine = tensor_split.shard_state_dict(w, rank, N)
        p_mine = oracle_params(mine)
        p_ref = R.shard_block_params(oracle_params(w), rank, N)
        for key in ("gate", "up", "down"):
            assert np.array_equal(p_mine[key].codes, p_ref[key].codes), key
            assert np.array_equal(p_mine[key].scales, p_ref[key].scales), key
        for key in ("shared_gate", "shared_up", "shared_down", "router", "shared_expert_gate"):
            assert np.array_equal(p_mine[key], p_ref[key]), key
        part = torch.from_numpy(R.sparse_moe_block(x, p_mine, CFG.top_k, vq=True).astype(np.float32))
        y = tp_reduce(part, dist.group.WORLD)
        if rank == 0:
            ref = R.tp_sparse_moe_block(x, oracle_params(w), CFG.top_k, vq=True, n=N)
            q.put(bool(np.array_equal(to_np(y), ref)))
    except Exception as e:  # report, never hang the other rank's test
        q.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_and_reduce_like_the_reference():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(N)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def test_tp_reduce_rejects_bf16_partials():
    import pytest
    with pytest.raises(TypeError):
        tp_reduce(torch.zeros(2, 2, dtype=torch.bfloat16), None)
