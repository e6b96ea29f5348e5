"""The decoder stack around the MoE block (§8(f) rank 1): the residual +
RMSNorm kernel, the trunk and the MTP head against the numpy oracle, KV-cache
decoding against whole-prompt forwards, and greedy MTP decoding against plain
greedy decoding (the reference's own property, tests/engine/
test_deepseek_v4_mtp.py `test_vq_head_greedy_drafting_is_the_plain_steps_
token_for_token`: drafting changes no emitted token).

Reference: qwen3_5.py:120-130 (RMSNorm), 368-432 (Attention), 549-674
(DecoderLayer, Qwen3_5TextModel); heads/qwen35.py:204-227 (the MTP head);
engine/mtp/block_loop.py (the verify loop)."""
import ctypes
from dataclasses import replace

import numpy as np
import pytest
import torch

from knurlogic_b200 import _lib, decoder, synth
from oracle import decoder_ref as D
from oracle import moe_ref as R
from tests.conftest import oracle_params, to_np

DEV = "cuda:0"
TINY = decoder.CONFIGS["tiny"]


def _np(w):
    return {k: (to_np(v) if v.dtype != torch.float32 else v.cpu().numpy()) for k, v in w.items()}


def _rel_rms(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.sqrt(((got - ref) ** 2).mean()) / max(np.sqrt((ref ** 2).mean()), 1e-30))


# ------------------------------------------------------------------ CPU

def test_configs_and_weight_names():
    c5 = decoder.CONFIGS["c5"]
    assert (c5.layers, c5.hidden, c5.heads, c5.kv_heads, c5.head_dim, c5.vocab) == (48, 4096, 32, 4, 128, 151936)
    assert (c5.moe.experts, c5.moe.top_k, c5.moe.inter) == (256, 8, 1536) and c5.moe.shared_inter > 0
    assert c5.rotary_dims == 32 and TINY.rotary_dims == 16
    w = decoder.make_weights(TINY, seed=1)
    assert w["model.layers.1.self_attn.q_proj.weight"].shape == (TINY.heads * 2 * TINY.head_dim, TINY.hidden)
    assert w["model.layers.0.input_layernorm.weight"].dtype == torch.float32
    assert w["model.layers.0.mlp.switch_mlp.up_proj.codes"].dtype == torch.uint8
    assert w["mtp.fc.weight"].shape == (TINY.hidden, 2 * TINY.hidden)
    assert "mtp.layers.0.mlp.gate.weight" in w


def test_no_cpu_path():
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        decoder.add_rms_norm(x, None, torch.ones(8), 1e-6)


def test_oracle_rope_and_norm_properties():
    x = R.bf16(np.random.default_rng(0).standard_normal((3, 2, 64)).astype(np.float32))
    assert np.array_equal(D.rope(x, 0, 16, 10000.0)[0], x[0])            # position 0 rotates by 0
    y = D.rope(x, 5, 16, 10000.0)
    assert np.array_equal(y[..., 16:], x[..., 16:])                       # only the rotary dims move
    n = D.rms_norm(x, np.ones(64, np.float32), 1e-6)
    assert np.allclose((n.astype(np.float64) ** 2).mean(-1), 1.0, atol=2e-2)


def test_add_rms_norm_refuses_bad_arguments():
    so = _lib.lib()
    st = so.vqmoe_add_rms_norm(None, None, None, 4, 8, ctypes.c_float(1e-6), None, None, None)
    assert _lib.STATUS[st] == "BAD_POINTER"
    st = so.vqmoe_add_rms_norm(None, None, None, 0, 8, ctypes.c_float(1e-6), None, None, None)
    assert _lib.STATUS[st] == "BAD_SHAPE"


# ------------------------------------------------------------------ GPU

@pytest.mark.gpu
@pytest.mark.parametrize("rows,H", [(7, 64), (33, 256), (5, 2048), (3, 4096)])
def test_add_rms_norm_is_bit_exact(rows, H):
    g = torch.Generator().manual_seed(rows * H)
    x = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    r = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    w = 1.0 + 0.1 * torch.randn(H, generator=g)
    s = torch.empty(rows, H, dtype=torch.bfloat16, device=DEV)
    n = decoder.add_rms_norm(x.to(DEV), r.to(DEV), w.to(DEV), 1e-6, sum_out=s)
    hs = R.bf16(to_np(x) + to_np(r))
    assert np.array_equal(to_np(s), hs)
    assert np.array_equal(to_np(n).view(np.uint32), D.rms_norm(hs, w.numpy(), 1e-6).view(np.uint32))
    n0 = decoder.add_rms_norm(x.to(DEV), None, w.to(DEV), 1e-6)
    assert np.array_equal(to_np(n0), D.rms_norm(to_np(x), w.numpy(), 1e-6))


def _oracle_model(w):
    wn = _np(w)
    moe = [oracle_params(w, f"model.layers.{i}.mlp.") for i in range(TINY.layers)]
    return wn, moe


@pytest.mark.gpu
def test_trunk_and_head_match_the_oracle():
    w = decoder.make_weights(TINY, seed=3, device=DEV)
    model = decoder.TextModel(w, TINY, torch.device(DEV))
    wc = {k: v.cpu() for k, v in w.items()}
    wn, moe = _oracle_model(wc)
    B, P = 2, 12
    tok = torch.randint(0, TINY.vocab, (B, P), generator=torch.Generator().manual_seed(3))
    caches = model.new_caches(B, 32, torch.device(DEV))
    normed, pre = model(tok.to(DEV), caches, 0)
    logits = to_np(model.logits(normed))
    hc = model.mtp.new_cache(B, 32, torch.device(DEV))
    nxt = torch.roll(tok, -1, dims=1)
    hn, _ = model.mtp(pre, nxt.to(DEV), hc, 0)
    hlog = to_np(model.logits(hn))
    mp = oracle_params(wc, "mtp.layers.0.mlp.")
    for b in range(B):
        kvs = [{"k": None, "v": None} for _ in range(TINY.layers)]
        ref, h = D.text_model(tok[b].numpy(), wn, TINY, moe, kvs, 0)
        assert _rel_rms(logits[b], ref) < 2e-2, _rel_rms(logits[b], ref)
        assert (logits[b].argmax(-1) == ref.argmax(-1)).mean() >= 0.9
        href, _ = D.mtp_head(h, nxt[b].numpy(), wn, TINY, mp, {"k": None, "v": None}, 0)
        assert _rel_rms(hlog[b], href) < 3e-2, _rel_rms(hlog[b], href)


@pytest.mark.gpu
def test_cached_decoding_equals_the_whole_prompt():
    """Positions fed one at a time through the KV cache give the logits of
    one forward over the whole sequence (the same kernels per token)."""
    w = decoder.make_weights(TINY, seed=4, device=DEV)
    model = decoder.TextModel(w, TINY, torch.device(DEV))
    B, P = 3, 10
    tok = torch.randint(0, TINY.vocab, (B, P + 4), generator=torch.Generator().manual_seed(4)).to(DEV)
    full, _ = model(tok, model.new_caches(B, 32, torch.device(DEV)), 0)
    caches = model.new_caches(B, 32, torch.device(DEV))
    model(tok[:, :P], caches, 0)
    steps = [model(tok[:, P + i:P + i + 1], caches, P + i)[0] for i in range(4)]
    inc = torch.cat(steps, dim=1)
    ref = full[:, P:]
    assert _rel_rms(to_np(model.logits(inc)), to_np(model.logits(ref))) < 1e-2
    assert torch.equal(model.logits(inc).argmax(-1), model.logits(ref).argmax(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 3])
def test_mtp_drafting_emits_the_plain_greedy_tokens(k):
    w = decoder.make_weights(TINY, seed=5, device=DEV)
    model = decoder.TextModel(w, TINY, torch.device(DEV))
    prompts = torch.randint(0, TINY.vocab, (4, 16), generator=torch.Generator().manual_seed(5)).to(DEV)
    plain = decoder.generate_greedy(model, prompts, 24)
    drafted, stats = decoder.generate_mtp(model, prompts, 24, k=k)
    assert torch.equal(plain, drafted)
    assert stats["steps"] > 0 and stats["drafted"] == stats["steps"] * 4 * k


@pytest.mark.gpu
def test_mtp_on_a_one_layer_trunk_with_two_drafts():
    """The same property at another depth and draft count; the reported
    acceptance counts drafts the verify agreed with."""
    cfg = replace(TINY, layers=1)
    w = decoder.make_weights(cfg, seed=6, device=DEV)
    model = decoder.TextModel(w, cfg, torch.device(DEV))
    prompts = torch.randint(0, cfg.vocab, (2, 8), generator=torch.Generator().manual_seed(6)).to(DEV)
    plain = decoder.generate_greedy(model, prompts, 16)
    drafted, stats = decoder.generate_mtp(model, prompts, 16, k=2)
    assert torch.equal(plain, drafted)
    assert 0 <= stats["accepted"] <= stats["drafted"]


@pytest.mark.gpu
def test_released_sources_leave_the_block_unchanged():
    cfg = synth.MoEConfig("r", 8, 2, 256, 256, 128, 12)
    w = synth.make_weights(cfg, seed=9, device=DEV, scales="random")
    from knurlogic_b200 import SparseMoeBlock
    blk = SparseMoeBlock.from_weights(w, cfg.top_k)
    x = synth.make_input(cfg, seed=9).to(DEV)
    before = blk(x)
    decoder._release(blk)
    up = blk.switch_mlp.up_proj
    assert up.codes.is_meta and (up.num_experts, up.output_dims, up.input_dims) == (8, 256, 256)
    assert torch.equal(blk(x), before)


@pytest.mark.gpu
def test_graph_replayed_decoding_emits_the_same_tokens():
    """Each decode step as one CUDA-graph replay (the position a device
    tensor, the whole cache read under a mask) gives the eager loop's tokens,
    for plain greedy decoding and for MTP drafting."""
    w = decoder.make_weights(TINY, seed=7, device=DEV)
    model = decoder.TextModel(w, TINY, torch.device(DEV))
    prompts = torch.randint(0, TINY.vocab, (3, 12), generator=torch.Generator().manual_seed(7)).to(DEV)
    plain = decoder.generate_greedy(model, prompts, 20)
    assert torch.equal(decoder.generate_greedy(model, prompts, 20, graphs=True), plain)
    drafted, stats = decoder.generate_mtp(model, prompts, 20, k=3, graphs=True)
    assert torch.equal(drafted, plain) and stats["steps"] > 0
