"""vqmoe_switch_glu_noalloc (the fixed-scratch form of vqmoe_switch_glu),
called through the C ABI: two calls in a row equal vqmoe_switch_glu with a
caller workspace bit for bit (the same kernels on the same inputs, each
output element summed in a fixed order), and a call whose workspace would
exceed the scratch is refused. Named to be collected last, and self-contained so that it also
runs alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from knurlogic_b200 import SwitchGLU, VQSwitchLinear, _lib, synth
from knurlogic_b200.switch_layers import c_stream

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCRATCH_BYTES = 4 << 20
WORKSPACE_TOO_SMALL = 4


def _vq_linear(w, name):
    q = f"mlp.switch_mlp.{name}."
    return VQSwitchLinear(w[q + "codes"].to(DEV), w[q + "codebook"].to(DEV),
                          w[q + "vq_scales"].to(DEV), group_size=64)


def _noalloc(glu, x, inds):
    T, k = inds.shape
    y = torch.empty((T, k, glu.down_proj.output_dims), dtype=torch.bfloat16, device=DEV)
    g, u, d = (m.descriptor() for m in (glu.gate_proj, glu.up_proj, glu.down_proj))
    st = _lib.lib().vqmoe_switch_glu_noalloc(
        ctypes.byref(g), ctypes.byref(u), ctypes.byref(d), x.data_ptr(), inds.data_ptr(), T, k,
        y.data_ptr(), c_stream(x.device))
    return st, y


def test_noalloc_switch_glu_matches_the_workspace_entry_on_two_calls():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=31, scales="random")
    glu = SwitchGLU(_vq_linear(w, "gate_proj"), _vq_linear(w, "up_proj"), _vq_linear(w, "down_proj"))
    g, d = glu.gate_proj.descriptor(), glu.down_proj.descriptor()
    need = _lib.lib().vqmoe_switch_glu_workspace_size(ctypes.byref(g), ctypes.byref(d), 64, cfg.top_k)
    assert 0 < need <= SCRATCH_BYTES
    gen = torch.Generator().manual_seed(31)
    for call in range(2):
        x = synth.make_input(cfg, seed=40 + call, tokens=64).to(DEV)
        inds = torch.stack([torch.randperm(cfg.experts, generator=gen)[:cfg.top_k]
                            for _ in range(64)]).to(torch.int32).to(DEV)
        ref = glu(x, inds)                      # vqmoe_switch_glu, caller workspace
        st, y = _noalloc(glu, x, inds)
        assert st == 0, _lib.lib().vqmoe_last_error()
        torch.cuda.synchronize()
        a = y.float().cpu().numpy()
        b = ref.float().cpu().numpy()
        assert np.isfinite(a).all()
        assert np.array_equal(a, b), f"call {call}: {int((a != b).sum())} of {a.size} elements differ"


def test_noalloc_switch_glu_refuses_more_than_its_scratch():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=32, scales="random")
    glu = SwitchGLU(_vq_linear(w, "gate_proj"), _vq_linear(w, "up_proj"), _vq_linear(w, "down_proj"))
    T = 1024                                   # ~17 MB of workspace at c2's shapes
    x = torch.zeros(T, cfg.hidden, dtype=torch.bfloat16, device=DEV)
    inds = torch.zeros(T, cfg.top_k, dtype=torch.int32, device=DEV)
    st, _ = _noalloc(glu, x, inds)
    assert st == WORKSPACE_TOO_SMALL
    assert b"scratch" in _lib.lib().vqmoe_last_error()
