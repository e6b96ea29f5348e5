"""The expert split (experts placed by id across ranks; §8(f) rank 4's
second half): the cuts and refusals on CPU, and on one GPU the split entry
with a single rank, which must equal the unsplit block bit for bit (its
combine sums the k slots in slot order, as the block's own does). The 2-,
4- and 8-rank runs are in test_tp_nccl.py."""
import ctypes

import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, _lib, expert_split, synth

DEV = "cuda:0"


def test_cuts_and_refusals():
    cfg = synth.MoEConfig("e", 16, 4, 256, 128, 64, 4)
    w = synth.make_weights(cfg, seed=1)
    sh = expert_split.shard_state_dict(w, 1, 4)
    assert sh["mlp.switch_mlp.up_proj.codes"].shape[0] == 4
    assert torch.equal(sh["mlp.switch_mlp.up_proj.codes"], w["mlp.switch_mlp.up_proj.codes"][4:8])
    assert torch.equal(sh["mlp.switch_mlp.down_proj.vq_scales"], w["mlp.switch_mlp.down_proj.vq_scales"][4:8])
    assert sh["mlp.gate.weight"] is w["mlp.gate.weight"]                          # the router stays whole
    assert sh["mlp.switch_mlp.gate_proj.codebook"] is w["mlp.switch_mlp.gate_proj.codebook"]
    assert sh["mlp.shared_expert.down_proj.weight"] is w["mlp.shared_expert.down_proj.weight"]
    shapes = {k: tuple(v.shape) for k, v in w.items()}
    assert expert_split.refusals(shapes, 4) == []
    assert any("do not divide" in r for r in expert_split.refusals(shapes, 3))
    assert any("hidden" in r for r in expert_split.refusals(shapes, 8) + expert_split.refusals(
        dict(shapes, **{"mlp.gate.weight": (16, 200)}), 2))


def test_entry_refuses_on_the_host():
    so = _lib.lib()
    lin = _lib.Linear(format=_lib.FMT_VQ_U8, num_experts=2, out_features=32, in_features=64, codes=256,
                      codebook=512, scales=768, codebook_size=256, dim=4, group_size=64)
    b = _lib.Block(hidden=64, num_experts=4, top_k=2, gate=lin, up=lin, down=_lib.Linear(
        format=_lib.FMT_VQ_U8, num_experts=2, out_features=64, in_features=32, codes=256, codebook=512,
        scales=768, codebook_size=256, dim=4, group_size=32))
    tp = _lib.Tp(rank=0, world=3, buffer_bytes=1 << 20)
    st = so.vqmoe_sparse_moe_block_ep(ctypes.byref(b), ctypes.byref(tp), None, 4, None, None, 0, None)
    assert _lib.STATUS[st] == "BAD_SHAPE" and b"experts over 3 ranks" in so.vqmoe_last_error()
    tp.world = 2
    tp.buffer_bytes = 16
    st = so.vqmoe_sparse_moe_block_ep(ctypes.byref(b), ctypes.byref(tp), None, 4, None, None, 0, None)
    assert _lib.STATUS[st] == "WORKSPACE_TOO_SMALL"


@pytest.mark.gpu
@pytest.mark.parametrize("name,tokens", [("c2", 64), ("c4", 16)])
def test_one_rank_equals_the_block(name, tokens):
    cfg = synth.CONFIGS[name]
    w = synth.make_weights(cfg, seed=41, scales="random")
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    x = synth.make_input(cfg, seed=41, tokens=tokens).to(DEV)
    need = _lib.lib().vqmoe_ep_buffer_bytes(cfg.hidden, tokens, cfg.top_k)
    buf = torch.zeros(need, dtype=torch.uint8, device=DEV)
    tp = _lib.Tp(rank=0, world=1, buffer_bytes=need)
    tp.buffers[0] = buf.data_ptr()
    b = blk._desc()
    ws = blk.workspace(tokens, torch.device(DEV))
    ref = blk(x)
    for _ in range(3):                                   # repeated calls: the barrier epochs advance
        out = torch.empty_like(x)
        _lib.call("vqmoe_sparse_moe_block_ep", ctypes.byref(b), ctypes.byref(tp), x.data_ptr(), tokens,
                  out.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        blk.check_status()
        assert torch.equal(out, ref)
