"""The VQ code formats beyond uint8 / dim 4 (the reference-layout path,
VQMOE_FMT_VQ_REF): uint16 codes for codebooks of up to 65536 entries, dim 2
and dim 8 codebooks, other scale-group sizes.

Reference: `deepseek_v4.py:111-121` -- codes are one code per entry (uint8
when K <= 256, uint16 above) or uint32-packed fields; the reference's own VQ
fixture (`tests/support/artifacts/gemma-4-26b-a4b-it-VQ-6.2bpw/config.json`)
is K 2048, dim 2, group 64 on experts of hidden 2816 and intermediate 704,
128 experts, top-8. Packed fields stay refused (their bit order is not
pinned). GPU tests compare with the oracle; the CPU tests check the module's
arguments.
"""
import ctypes

import numpy as np
import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, SwitchGLU, VQSwitchLinear, _lib, synth, tensor_split
from oracle import moe_ref as R
from tests.conftest import assert_bf16_close, oracle_params, to_np

DEV = "cuda:0"
# the reference fixture's expert geometry (Gemma-4 26B-A4B VQ-6.2bpw)
FIXTURE = synth.MoEConfig("fixture", 128, 8, 2816, 704, 0, 16, router="uniform", dim=2,
                          codebook_size=2048, group=64)


def _vq(w, name, dev=DEV):
    q = f"mlp.switch_mlp.{name}."
    cb, vs = w[q + "codebook"], w[q + "vq_scales"]
    IN = w[q + "codes"].shape[-1] * cb.shape[-1]
    return VQSwitchLinear(w[q + "codes"].to(dev), cb.to(dev), vs.to(dev), group_size=IN // vs.shape[-1])


# ------------------------------------------------------------------ CPU

def test_module_takes_the_one_code_per_entry_formats():
    for K, dim, dt, fast in ((256, 4, torch.uint8, True), (2048, 2, torch.uint16, False),
                             (256, 8, torch.uint8, False), (65536, 4, torch.uint16, False)):
        m = VQSwitchLinear(torch.zeros(2, 16, 64 // dim, dtype=dt), torch.zeros(K, dim),
                           torch.ones(2, 16, 1), group_size=64)
        assert m.fast == fast and m.input_dims == 64 and m._k_expect == K
    with pytest.raises(ValueError, match="uint16"):       # K > 256 needs uint16 codes
        VQSwitchLinear(torch.zeros(2, 16, 32, dtype=torch.uint8), torch.zeros(2048, 2),
                       torch.ones(2, 16, 1), group_size=64)
    with pytest.raises(ValueError, match="dim 3"):
        VQSwitchLinear(torch.zeros(2, 16, 32, dtype=torch.uint8), torch.zeros(256, 3),
                       torch.ones(2, 16, 3), group_size=32)
    with pytest.raises(NotImplementedError, match="packed"):
        VQSwitchLinear(torch.zeros(2, 16, 11, dtype=torch.int32), torch.zeros(2048, 2),
                       torch.ones(2, 16, 1), group_size=64, pack_bits=11, in_features=64)


def test_reference_layout_descriptors_are_checked():
    so = _lib.lib()
    # placeholder device addresses (aligned, never dereferenced: every call
    # below is refused on the host before anything is launched)
    ptrs = dict(codes=256, codebook=512, scales=768)
    lin = _lib.Linear(format=_lib.FMT_VQ_REF, num_experts=4, out_features=32, in_features=128,
                      codebook_size=2048, dim=2, group_size=64, **ptrs)
    b = _lib.Block(hidden=128, num_experts=4, top_k=2, shared_inter=0, gate=lin, up=lin, down=_lib.Linear(
        format=_lib.FMT_VQ_REF, num_experts=4, out_features=128, in_features=32, codebook_size=2048, dim=2,
        group_size=32, **ptrs))
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 4, None, 0, None, 0, None)
    assert _lib.STATUS[st] == "BAD_SHAPE" and b"in_features 32" in so.vqmoe_last_error()
    b.gate.dim = b.up.dim = 3
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 4, None, 0, None, 0, None)
    assert _lib.STATUS[st] == "BAD_FORMAT" and b"dim 3" in so.vqmoe_last_error()
    b.gate.dim = b.up.dim = 2
    b.down.format = _lib.FMT_VQ_U8
    b.down.in_features, b.gate.out_features, b.up.out_features = 64, 64, 64
    b.down.dim, b.down.codebook_size, b.down.group_size = 4, 256, 64
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), None, 4, None, 0, None, 0, None)
    assert _lib.STATUS[st] == "BAD_FORMAT" and b"reference-layout" in so.vqmoe_last_error()


def test_split_refusals_read_the_codebook_dim():
    shapes = {"mlp.switch_mlp.down_proj.codes": (128, 2816, 352),          # I 704 at dim 2
              "mlp.switch_mlp.down_proj.codebook": (2048, 2),
              "mlp.switch_mlp.down_proj.vq_scales": (128, 2816, 11)}
    assert any("inputs" in r for r in tensor_split.refusals(shapes, 2))    # 352 inputs: not whole 64s
    shapes["mlp.switch_mlp.down_proj.codes"] = (128, 2816, 768)           # I 1536 at dim 2
    shapes["mlp.switch_mlp.down_proj.vq_scales"] = (128, 2816, 24)
    assert tensor_split.refusals(shapes, 2) == []


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
@pytest.mark.parametrize("K,dim,group", [(2048, 2, 64), (256, 8, 64), (1024, 4, 64), (256, 4, 32),
                                         (65536, 2, 128)])
def test_reference_layout_dequant_is_bit_exact(K, dim, group):
    cfg = synth.MoEConfig("w", 3, 2, 256, 96, 0, 1, dim=dim, codebook_size=K, group=group)
    w = synth.make_weights(cfg, seed=K + dim, scales="random")
    m = _vq(w, "up_proj")
    assert not m.fast
    got = to_np(m.dequantize(1, 2))
    q = "mlp.switch_mlp.up_proj."
    ref = R.dequant(to_np(w[q + "codes"])[1:3], to_np(w[q + "codebook"]), to_np(w[q + "vq_scales"])[1:3], group)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,seed", [(16, 0), (5, 1), (300, 2)])
def test_block_at_the_reference_fixture_geometry(tokens, seed):
    """K 2048, dim 2, group 64, uint16 codes, H 2816, I 704, 128 experts
    top-8: 16 decode tokens (about one pair per expert), 5, and 300
    (about 19 pairs per expert)."""
    cfg = FIXTURE.with_tokens(tokens)
    w = synth.make_weights(cfg, seed=seed, scales="random")
    assert w["mlp.switch_mlp.up_proj.codes"].dtype == torch.uint16
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)
    assert not blk.switch_mlp.up_proj.fast
    x = synth.make_input(cfg, seed=seed)
    y = to_np(blk(x.to(DEV)))
    blk.check_status()
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y, ref, f"fixture geometry T={tokens}")


@pytest.mark.gpu
@pytest.mark.parametrize("K,dim,group", [(256, 8, 64), (4096, 4, 64), (256, 4, 128)])
def test_switch_glu_other_formats(K, dim, group):
    cfg = synth.MoEConfig("w", 16, 4, 512, 256, 0, 24, dim=dim, codebook_size=K, group=group)
    w = synth.make_weights(cfg, seed=dim * 7 + K, scales="random")
    glu = SwitchGLU(_vq(w, "gate_proj"), _vq(w, "up_proj"), _vq(w, "down_proj"))
    x = synth.make_input(cfg, seed=3)
    p = oracle_params(w)
    inds, _, _ = R.router(to_np(x), p["router"], cfg.top_k)
    y = glu(x.to(DEV), torch.from_numpy(inds).to(DEV))
    ref = R.switch_glu(to_np(x), inds, p["gate"], p["up"], p["down"], vq=True)
    assert_bf16_close(to_np(y), ref, f"switch_glu K={K} dim={dim} group={group}")


@pytest.mark.gpu
def test_tensor_split_of_the_fixture_geometry_emulated():
    """The fixture layer cut 2 ways would leave 352 inputs per rank (refused);
    at I 1536 (c4's width) a rank keeps 768, and the float32 sum of the
    ranks' partials matches the oracle's split block."""
    cfg = synth.MoEConfig("w", 32, 8, 1024, 1536, 0, 8, router="uniform", dim=2, codebook_size=2048)
    w = synth.make_weights(cfg, seed=19, scales="random")
    x = synth.make_input(cfg, seed=19).to(DEV)
    acc = torch.zeros(cfg.tokens, cfg.hidden, dtype=torch.float32, device=DEV)
    for r in range(2):
        blk = tensor_split.build_block({k: v.to(DEV) for k, v in w.items()}, cfg.top_k, rank=r, n=2)
        part = torch.empty(cfg.tokens, cfg.hidden, dtype=torch.float32, device=DEV)
        blk.forward_into(x, part)
        acc += part
    ref = R.tp_sparse_moe_block(to_np(x.cpu()), oracle_params(w), cfg.top_k, vq=True, n=2)
    assert_bf16_close(to_np(acc.to(torch.bfloat16)), ref, "fixture-format tp2")
