"""Affine-quantized experts (VQMOE_FMT_AFFINE): mlx-lm's
`QuantizedSwitchLinear` (`switch_layers.py:24-86`, `mx.gather_qmm` in mode
"affine") -- packed uint32 weights of 2-8 bits per value, a bf16 scale and
bias per group of 32, 64 or 128 inputs.

The packing is mlx's (each row a little-endian bit stream); the rounding of
the dequantised weight, W = bf16(fmaf(scale, q, bias)), is this build's
definition (MLX's kernels cannot run here: unpinned), restated by
`oracle.moe_ref.dequant_affine`. CPU tests check the packing and the module's
arguments; GPU tests compare the kernels with the oracle.
"""
import numpy as np
import pytest
import torch

from knurlogic_b200 import QuantizedSwitchLinear, SparseMoeBlock, SwitchGLU, synth, tensor_split
from oracle import moe_ref as R
from tests.conftest import assert_bf16_close, oracle_params, to_np

DEV = "cuda:0"


def _cfg(bits, group, E=16, k=4, H=512, I=256, Is=0, T=24):
    return synth.MoEConfig("affine", E, k, H, I, Is, T, router="uniform", group=group, quant="affine", bits=bits)


def _lin(w, name, group, dev=DEV):
    q = f"mlp.switch_mlp.{name}."
    wt, sc = w[q + "weight"], w[q + "scales"]
    bits = wt.shape[-1] * 32 // (sc.shape[-1] * group)
    return QuantizedSwitchLinear(wt.to(dev), sc.to(dev), w[q + "biases"].to(dev), group_size=group, bits=bits)


# ------------------------------------------------------------------ CPU

@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_packing_round_trips_through_the_oracle(bits):
    q = torch.randint(0, 1 << bits, (2, 3, 128), generator=torch.Generator().manual_seed(bits))
    words = synth.pack_affine(q, bits)
    assert words.shape == (2, 3, 128 * bits // 32)
    assert np.array_equal(R.unpack_affine(words.numpy(), bits), q.numpy())


def test_module_arguments():
    w, s, b = torch.zeros(2, 16, 32, dtype=torch.int32), torch.ones(2, 16, 2), torch.zeros(2, 16, 2)
    m = QuantizedSwitchLinear(w, s, b, group_size=64, bits=8)
    assert (m.num_experts, m.output_dims, m.input_dims, m.bits, m.mode) == (2, 16, 128, 8, "affine")
    with pytest.raises(ValueError, match="describe"):          # 32 words of 4-bit values are 256 inputs
        QuantizedSwitchLinear(w, s, b, group_size=64, bits=4)
    with pytest.raises(NotImplementedError, match="mxfp4"):
        QuantizedSwitchLinear(w, s, b, group_size=64, bits=8, mode="mxfp4")
    with pytest.raises(ValueError, match="bits 7"):
        QuantizedSwitchLinear(w, s, b, group_size=64, bits=7)


def test_split_refusals_of_packed_weights():
    # c4's down at 4 bits, cut 8 ways: 24 packed words (192 inputs) per rank
    shapes = {"mlp.switch_mlp.down_proj.weight": (256, 4096, 192),
              "mlp.switch_mlp.down_proj.scales": (256, 4096, 24),
              "mlp.switch_mlp.down_proj.biases": (256, 4096, 24)}
    assert tensor_split.refusals(shapes, 8) == []


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
@pytest.mark.parametrize("bits,group", [(2, 128), (3, 64), (4, 64), (5, 32), (6, 64), (8, 32)])
def test_affine_dequant_is_bit_exact(bits, group):
    cfg = _cfg(bits, group, E=3, H=256, I=96)
    w = synth.make_weights(cfg, seed=bits * 10 + group)
    m = _lin(w, "up_proj", group)
    got = to_np(m.dequantize(1, 2))
    q = "mlp.switch_mlp.up_proj."
    ref = R.dequant_affine(to_np(w[q + "weight"])[1:3], to_np(w[q + "scales"])[1:3],
                           to_np(w[q + "biases"])[1:3], group, bits)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("bits,group", [(4, 64), (3, 32), (8, 128)])
def test_switch_glu_matches_oracle(bits, group):
    cfg = _cfg(bits, group)
    w = synth.make_weights(cfg, seed=bits + group)
    glu = SwitchGLU(_lin(w, "gate_proj", group), _lin(w, "up_proj", group), _lin(w, "down_proj", group))
    x = synth.make_input(cfg, seed=5)
    p = oracle_params(w, group_size=group)
    inds, _, _ = R.router(to_np(x), p["router"], cfg.top_k)
    y = glu(x.to(DEV), torch.from_numpy(inds).to(DEV))
    ref = R.switch_glu(to_np(x), inds, p["gate"], p["up"], p["down"], vq=False)
    assert_bf16_close(to_np(y), ref, f"affine switch_glu bits={bits} group={group}")


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,bits", [(16, 4), (300, 4), (64, 2)])
def test_block_matches_oracle(tokens, bits):
    """A c2-shaped block (128 experts top-8, H 2048, I 768, shared expert)
    with affine experts, as the reference's QuantizedSwitchLinear layers."""
    cfg = _cfg(bits, 64, E=128, k=8, H=2048, I=768, Is=768, T=tokens)
    w = synth.make_weights(cfg, seed=tokens + bits)
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k, group_size=64)
    assert isinstance(blk.switch_mlp.gate_proj, QuantizedSwitchLinear) and blk.switch_mlp.gate_proj.bits == bits
    x = synth.make_input(cfg, seed=tokens)
    y = to_np(blk(x.to(DEV)))
    blk.check_status()
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=False)
    assert_bf16_close(y, ref, f"affine block T={tokens} bits={bits}")


@pytest.mark.gpu
def test_tensor_split_emulated():
    cfg = _cfg(4, 64, E=32, k=8, H=1024, I=1024, T=8)
    w = synth.make_weights(cfg, seed=23)
    x = synth.make_input(cfg, seed=23).to(DEV)
    acc = torch.zeros(cfg.tokens, cfg.hidden, dtype=torch.float32, device=DEV)
    for r in range(2):
        blk = tensor_split.build_block({k: v.to(DEV) for k, v in w.items()}, cfg.top_k, rank=r, n=2)
        part = torch.empty(cfg.tokens, cfg.hidden, dtype=torch.float32, device=DEV)
        blk.forward_into(x, part)
        acc += part
    ref = R.tp_sparse_moe_block(to_np(x.cpu()), oracle_params(w), cfg.top_k, vq=False, n=2)
    assert_bf16_close(to_np(acc.to(torch.bfloat16)), ref, "affine tp2")
