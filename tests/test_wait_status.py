"""Bounded device waits surface as VQMOE_TIMEOUT (on a B200).

A phase 2 (down) tile of the routed experts waits for every phase 1
(gate/up) tile of its expert. Here one expert has 64 phase 1 tiles and its
down tiles are taken at the same moment by other CTAs, so with a limit of a
single poll their waits must run out: the kernel stores the kind of wait in
the workspace's status word and returns (nothing hangs; the tile's output is
then wrong), and `vqmoe_workspace_status` reports VQMOE_TIMEOUT. The next
call with the default limit clears the word, finishes normally and matches
the oracle: the context stays usable. No GPU fault is involved -- the wait
just gives up.
"""
import numpy as np
import pytest

from knurlogic_b200 import SparseMoeBlock, _lib, synth
from oracle import moe_ref as R
from tests.conftest import oracle_params, to_np

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TIMEOUT = 7


@pytest.mark.parametrize("tokens", [4, 64], ids=["decode", "prefill"])
def test_a_wait_that_runs_out_reports_timeout(tokens):
    # 1 expert, top-1: 4 tokens take the mma.sync decode kernel, 64 tokens
    # (64 pairs per expert) the tcgen05 prefill kernel; I = 8192 gives 64
    # phase 1 tiles of 128 rows, H = 2048 eight down tiles of 256 rows
    cfg = synth.MoEConfig("wait", 1, 1, 2048, 8192, 0, tokens)
    w = synth.make_weights(cfg, seed=3, scales="random")
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    x = synth.make_input(cfg, seed=3).to(DEV)
    blk.wait_polls = 1
    blk(x)
    with pytest.raises(_lib.VQMoEError) as e:
        blk.check_status()
    assert e.value.status == TIMEOUT
    assert b"phase 1" in _lib.lib().vqmoe_last_error()
    blk.wait_polls = 0
    y = to_np(blk(x))
    blk.check_status()
    ref = R.sparse_moe_block(to_np(x.cpu()), oracle_params(w), cfg.top_k, vq=True)
    err = np.abs(y - ref).max()
    assert err <= 1e-2 * np.abs(ref).max(), err


def test_status_is_ok_after_a_normal_call():
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, seed=2, scales="random")
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    blk(synth.make_input(cfg, seed=2).to(DEV))
    blk.check_status()
