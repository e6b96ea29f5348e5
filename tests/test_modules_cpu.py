"""Host-side behaviour of the drop-in modules (CPU): constructor checks that
mirror the reference's bind errors, the names they read, and that they
refuse to compute anywhere but on CUDA."""
import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, SwitchGLU, SwitchLinear, VQSwitchLinear
from knurlogic_b200 import synth, tensor_split


def _vq(E=2, OUT=32, IN=128, K=256, dim=4, group=64):
    codes = torch.randint(0, K, (E, OUT, IN // dim), dtype=torch.uint8)
    cb = torch.randn(K, dim).to(torch.float16)
    vs = torch.ones(E, OUT, IN // group, dtype=torch.float16)
    return codes, cb, vs


def test_vq_switch_linear_exposes_the_reference_attributes():
    codes, cb, vs = _vq()
    m = VQSwitchLinear(codes, cb, vs, group_size=64)
    assert (m.num_experts, m.output_dims, m.input_dims) == (2, 32, 128)
    assert m.group_size == 64 and m.pack_bits == 0 and m._k_expect == 256
    assert m.codes is not None and m.codebook.dtype == torch.float16


def test_vq_switch_linear_rejects_what_bind_rejects():
    """Shape checks of deepseek_v4._vq_module (deepseek_v4.py:101-125)."""
    codes, cb, vs = _vq()
    with pytest.raises(ValueError, match="shape mismatch"):
        VQSwitchLinear(codes, cb, vs[:1], group_size=64)
    with pytest.raises(ValueError, match="scale groups"):
        VQSwitchLinear(codes, cb, vs, group_size=32)
    with pytest.raises(ValueError, match="codes rows"):
        VQSwitchLinear(codes, cb, vs, group_size=64, in_features=130)
    with pytest.raises(NotImplementedError, match="packed"):
        VQSwitchLinear(codes, cb, vs, group_size=64, pack_bits=8)


def test_modules_refuse_cpu_tensors():
    codes, cb, vs = _vq()
    m = VQSwitchLinear(codes, cb, vs, group_size=64)
    x = torch.zeros(3, 1, 1, 128, dtype=torch.bfloat16)
    idx = torch.zeros(3, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(x, idx)
    glu = SwitchGLU(SwitchLinear(torch.zeros(2, 16, 128)), SwitchLinear(torch.zeros(2, 16, 128)),
                    SwitchLinear(torch.zeros(2, 128, 16)))
    with pytest.raises(RuntimeError, match="CUDA"):
        glu(torch.zeros(3, 128, dtype=torch.bfloat16), idx)


def test_gemma4_modules_check_their_arguments():
    """Gemma-4's Router and Experts (gemma4_text.py:156-214): shapes and the
    GeGLU activation are checked at construction; CPU tensors are refused."""
    from knurlogic_b200 import GeGLU
    from knurlogic_b200.gemma4 import Experts, Router
    E, H = 8, 128
    proj = torch.zeros(E, H)
    with pytest.raises(ValueError, match="per_expert_scale"):
        Router(proj, torch.ones(H), torch.ones(E + 1), 2)
    with pytest.raises(ValueError, match="top_k_experts"):
        Router(proj, torch.ones(H), torch.ones(E), E + 1)
    r = Router(proj, torch.ones(H), torch.ones(E), 2)
    assert r.per_expert_scale.dtype == torch.float32 and r.proj.weight.dtype == torch.bfloat16
    with pytest.raises(RuntimeError, match="CUDA"):
        r(torch.zeros(3, H, dtype=torch.bfloat16))
    lins = [SwitchLinear(torch.zeros(E, 16, H)), SwitchLinear(torch.zeros(E, 16, H)),
            SwitchLinear(torch.zeros(E, H, 16))]
    with pytest.raises(ValueError, match="GeGLU"):
        Experts(SwitchGLU(*lins))
    ex = Experts(SwitchGLU(*lins, activation=GeGLU()))
    with pytest.raises(RuntimeError, match="CUDA"):
        ex(torch.zeros(3, H, dtype=torch.bfloat16), torch.zeros(3, 2, dtype=torch.int32), torch.ones(3, 2))


def test_gemma4_router_norm_weight_and_no_cpu_path():
    """The router's RMS-norm weight is scale * hidden**-0.5 rounded to bf16
    once, at construction; the norm itself (`vqmoe_rms_norm`) has no CPU
    path."""
    import numpy as np
    from knurlogic_b200.gemma4 import Router
    from oracle import moe_ref as R
    g = np.random.default_rng(0)
    H = 256
    scale = torch.from_numpy(g.uniform(0.5, 1.5, H).astype(np.float32))
    r = Router(torch.zeros(4, H), scale, torch.ones(4), 2)
    w = R.bf16(R.bf16(scale.numpy()) * np.float32(H ** -0.5))
    assert np.array_equal(r.norm_weight.float().numpy(), w)
    with pytest.raises(RuntimeError, match="CUDA"):
        r.normalize(torch.zeros(2, H, dtype=torch.bfloat16))


def test_block_reads_the_reference_state_dict_names():
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, seed=0)
    blk = SparseMoeBlock.from_weights(w, cfg.top_k)
    assert isinstance(blk.switch_mlp.gate_proj, VQSwitchLinear)
    assert blk.num_experts == 8 and blk.top_k == 2 and blk.shared_expert is None
    cfg2 = synth.CONFIGS["c2"].with_tokens(4)
    w2 = synth.make_weights(cfg2, seed=0)
    blk2 = SparseMoeBlock.from_weights(w2, cfg2.top_k)
    assert blk2.shared_expert.gate_proj.weight.shape == (768, 2048)
    assert blk2.shared_expert_gate.weight.shape == (1, 2048)
    with pytest.raises(RuntimeError, match="CUDA"):
        blk2(torch.zeros(4, 2048, dtype=torch.bfloat16))


def test_hf_fused_gate_up_is_split_in_half(golden):
    from tests.conftest import golden_state_dict
    w = golden_state_dict(golden)
    gu = torch.cat([w.pop("mlp.switch_mlp.gate_proj.weight"),
                    w.pop("mlp.switch_mlp.up_proj.weight")], dim=1)
    w["mlp.experts.gate_up_proj"] = gu
    w["mlp.experts.down_proj"] = w.pop("mlp.switch_mlp.down_proj.weight")
    blk = SparseMoeBlock.from_weights(w, 2)
    assert torch.equal(blk.switch_mlp.gate_proj.weight, gu[:, :16])
    assert torch.equal(blk.switch_mlp.up_proj.weight, gu[:, 16:])


def test_tensor_split_refusals_follow_the_reference_rule():
    """C2's I = 768 has 12 scale groups: 8 ranks refuse (tensor_rules
    refusals); C4's I = 1536 splits 2, 4 and 8 ways."""
    c2 = synth.make_weights(synth.CONFIGS["c2"].with_tokens(1), seed=0)
    shapes = {k: tuple(v.shape) for k, v in c2.items()}
    assert tensor_split.refusals(shapes, 2) == []
    assert tensor_split.refusals(shapes, 4) == []
    why = tensor_split.refusals(shapes, 8)
    assert any("down_proj.vq_scales: 12 on axis 2 do not divide by 8" in s for s in why)
    E, H, I = 256, 4096, 1536
    c4 = {"mlp.switch_mlp.down_proj.codes": (E, H, I // 4),
          "mlp.switch_mlp.down_proj.vq_scales": (E, H, I // 64),
          "mlp.switch_mlp.down_proj.codebook": (256, 4),
          "mlp.switch_mlp.gate_proj.codes": (E, I, H // 4),
          "mlp.switch_mlp.gate_proj.vq_scales": (E, I, H // 64)}
    for n in (2, 4, 8):
        assert tensor_split.refusals(c4, n) == []


def test_tensor_split_cuts_codes_and_never_codebooks():
    w = synth.make_weights(synth.CONFIGS["c2"].with_tokens(1), seed=0)
    parts = [tensor_split.shard_state_dict(w, r, 2) for r in range(2)]
    q = "mlp.switch_mlp."
    for r, p in enumerate(parts):
        assert torch.equal(p[q + "gate_proj.codebook"], w[q + "gate_proj.codebook"])
        assert p[q + "gate_proj.codes"].shape == (128, 384, 512)
        assert p[q + "down_proj.codes"].shape == (128, 2048, 96)
        assert p[q + "down_proj.vq_scales"].shape == (128, 2048, 6)
        assert torch.equal(p["mlp.gate.weight"], w["mlp.gate.weight"])
        assert torch.equal(p["mlp.shared_expert_gate.weight"], w["mlp.shared_expert_gate.weight"])
    assert torch.equal(torch.cat([parts[0][q + "down_proj.codes"], parts[1][q + "down_proj.codes"]], -1),
                       w[q + "down_proj.codes"])
    assert torch.equal(torch.cat([parts[0][q + "up_proj.codes"], parts[1][q + "up_proj.codes"]], 1),
                       w[q + "up_proj.codes"])
