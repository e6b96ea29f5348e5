"""The peer-memory reduction kernel of the tensor split on ONE GPU (world
size 1): `vqmoe_sparse_moe_block_tp` with the rank's own buffer as the only
one. The kernel's three phases, its two barriers and its epochs run as they
do across GPUs; the result must equal the unsplit block bit for bit (a
single partial, rounded as the combine rounds it), over repeated calls and
CUDA-graph replays, and a buffer that is too small is refused."""
import ctypes

import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, _lib, synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_world_of_one_equals_the_block():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=61, scales="random")
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    T = cfg.tokens
    need = _lib.lib().vqmoe_tp_buffer_bytes(cfg.hidden, T)
    buf = torch.zeros(need, dtype=torch.uint8, device=DEV)
    tp = _lib.Tp(rank=0, world=1, buffer_bytes=need)
    tp.buffers[0] = buf.data_ptr()
    b = blk._desc()
    ws = blk.workspace(T, torch.device(DEV))
    stream = torch.cuda.current_stream().cuda_stream

    def fused(x, out):
        _lib.call("vqmoe_sparse_moe_block_tp", ctypes.byref(b), ctypes.byref(tp), x.data_ptr(), T,
                  out.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        return out

    for seed in range(3):
        x = synth.make_input(cfg, seed=seed).to(DEV)
        y = fused(x, torch.empty_like(x))
        blk.check_status()
        assert torch.equal(y, blk(x)), f"call {seed}"
    # the epoch lives in device memory: graph replays see it advance
    x = synth.make_input(cfg, seed=7).to(DEV)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        stream = s.cuda_stream
        fused(x, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stream = torch.cuda.current_stream().cuda_stream
        fused(x, out)
    ref = blk(x)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    # calls that ran (capturing runs nothing): 3 eager, 1 warm-up, 3 replays
    assert int(buf[:4].view(torch.int32).item()) == 3 + 1 + 3
    tp.buffer_bytes = need - 16
    st = _lib.lib().vqmoe_sparse_moe_block_tp(ctypes.byref(b), ctypes.byref(tp), x.data_ptr(), T, out.data_ptr(),
                                             ws.data_ptr(), ws.numel(), stream)
    assert _lib.STATUS[st] == "WORKSPACE_TOO_SMALL"


def test_timed_entry_records_the_stages():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=62, scales="random")
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    T = cfg.tokens
    need = _lib.lib().vqmoe_tp_buffer_bytes(cfg.hidden, T)
    buf = torch.zeros(need, dtype=torch.uint8, device=DEV)
    tp = _lib.Tp(rank=0, world=1, buffer_bytes=need)
    tp.buffers[0] = buf.data_ptr()
    b = blk._desc()
    ws = blk.workspace(T, torch.device(DEV))
    x = synth.make_input(cfg, seed=62).to(DEV)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for e in evs:
        e.record()
    arr = (ctypes.c_void_p * 5)(*[e.cuda_event for e in evs])
    _lib.call("vqmoe_sparse_moe_block_tp_timed", ctypes.byref(b), ctypes.byref(tp), x.data_ptr(), T, out.data_ptr(),
              ws.data_ptr(), ws.numel(), stream, arr, 5)
    torch.cuda.synchronize()
    assert torch.equal(out, blk(x))
    assert all(evs[i].elapsed_time(evs[i + 1]) >= 0 for i in range(4))
    st = _lib.lib().vqmoe_sparse_moe_block_tp_timed(ctypes.byref(b), ctypes.byref(tp), x.data_ptr(), T,
                                                   out.data_ptr(), ws.data_ptr(), ws.numel(), stream, arr, 4)
    assert _lib.STATUS[st] == "BAD_POINTER"
