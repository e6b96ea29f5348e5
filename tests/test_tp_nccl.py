"""The tensor split and the expert split on 2, 4 and 8 GPUs (each skipped
with fewer). For the tensor split each rank builds its cut with
`tensor_split.build_block` and runs the block through the C ABI; the ranks'
partials are reduced either by the peer-memory kernel (the combine and the
float32 reduction in one kernel, `vqmoe_sparse_moe_block_tp`, over torch
symmetric-memory buffers) or over NCCL, and rank 0 compares both with the
oracle's tensor-split block and with each other. For the expert split
(`expert_split.build_block`, `vqmoe_sparse_moe_block_ep`) each rank holds
whole experts and rank 0 requires the unsplit block's output bit for bit.
All over eager calls, repeated calls (the kernels' barrier epochs advance)
and CUDA-graph replays."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from knurlogic_b200 import CapturedBlock, SparseMoeBlock, expert_split, synth, tensor_split
from oracle import moe_ref as R
from tests.conftest import assert_bf16_close, oracle_params, to_np

pytestmark = pytest.mark.gpu
# I 512 and a shared I 256 leave whole scale groups on each of up to 8 ranks
CFG = synth.MoEConfig("tpn", 16, 4, 512, 512, 256, 24)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, N, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=N, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        w = synth.make_weights(CFG, seed=8, scales="random")
        wd = {k: v.to(dev) for k, v in w.items()}
        out = {}
        for mode in ("p2p", "nccl"):
            blk = tensor_split.build_block(wd, CFG.top_k, rank=rank, n=N, group=dist.group.WORLD, tp_reduce=mode)
            ys = []
            for seed in (8, 9, 10):                     # repeated calls
                ys.append(to_np(blk(synth.make_input(CFG, seed=seed).to(dev))))
            blk.check_status()
            cap = CapturedBlock(blk, CFG.tokens)
            for seed in (11, 12):                       # graph replays
                ys.append(to_np(cap(synth.make_input(CFG, seed=seed).to(dev)).clone()))
            cap.check_status()
            out[mode] = ys
            del cap, blk
            torch.cuda.synchronize(dev)
        # the expert split: whole experts by id, the combine over peer memory
        blk = expert_split.build_block(wd, CFG.top_k, rank, N, dist.group.WORLD)
        ys = [to_np(blk(synth.make_input(CFG, seed=seed).to(dev))) for seed in (8, 9, 10)]
        blk.check_status()
        cap = CapturedBlock(blk, CFG.tokens)
        for seed in (11, 12):
            ys.append(to_np(cap(synth.make_input(CFG, seed=seed).to(dev)).clone()))
        cap.check_status()
        out["ep"] = ys
        del cap, blk
        full = SparseMoeBlock.from_weights(wd, CFG.top_k)     # the unsplit block, this GPU alone
        out["full"] = [to_np(full(synth.make_input(CFG, seed=seed).to(dev))) for seed in (8, 9, 10, 11, 12)]
        torch.cuda.synchronize(dev)
        # every rank's kernels and collectives end here, before rank 0's checks
        # (a failed check must not leave a peer inside a collective)
        dist.barrier()
        torch.cuda.synchronize(dev)
        if rank == 0:
            p = oracle_params(w)
            res = []
            for i, seed in enumerate((8, 9, 10, 11, 12)):
                ref = R.tp_sparse_moe_block(to_np(synth.make_input(CFG, seed=seed)), p, CFG.top_k, vq=True, n=N)
                assert_bf16_close(out["p2p"][i], ref, f"tp{N} p2p call {i}")
                assert_bf16_close(out["nccl"][i], ref, f"tp{N} nccl call {i}")
                # the expert split's combine is the block's own: bit for bit
                assert np.array_equal(out["ep"][i], out["full"][i]), f"ep{N} call {i}"
                a = out["p2p"][i].astype(np.float32)
                b = out["nccl"][i].astype(np.float32)
                ulp = np.abs(a - b) / np.maximum(np.abs(a), 1e-30)
                res.append((int((a != b).sum()), float(ulp.max())))
            q.put(res)
    except Exception as e:  # report, never hang the other rank's test
        q.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N", [2, 4, 8])
def test_tensor_split_across_gpus_matches_the_oracle(N):
    if torch.cuda.device_count() < N:
        pytest.skip(f"needs {N} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, N, port, q)) for r in range(N)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = q.get(timeout=5)
    assert not isinstance(res, str), res
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    # the two reductions sum the same bf16 partials in float32, the kernel in
    # rank order and NCCL in its own: two terms give equal bits; more may
    # round differently where the partials' magnitudes are far apart
    if N == 2:
        assert [d for d, _ in res] == [0] * 5, res
    else:
        n_out = CFG.tokens * CFG.hidden
        assert all(d <= n_out // 1000 and u <= 2.0 ** -7 for d, u in res), res
