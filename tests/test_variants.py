"""Router and activation variants of the same expert path: the Qwen4-exp
router (`qwen4_exp.py:800-815`: softmax over the top-k logits with
`norm_topk_prob`, or the top-k of the full softmax without it), Gemma-4's
GeGLU activation (`gemma4_text.py:131-135, 186-189`) and Gemma-4's router
(per-expert scale) and experts module (`gemma4_text.py:156-214`).

CPU: the oracle's pieces against independent restatements, and the ABI's
argument checks (they return before any CUDA call). GPU: the kernels
against the oracle, under the bars of test_gpu_parity."""
import ctypes

import numpy as np
import pytest
import torch

from knurlogic_b200 import GeGLU, SparseMoeBlock, _lib, synth
from oracle import moe_ref as R
from tests.conftest import oracle_params, to_np

DEV = "cuda:0"


# ------------------------------------------------------------------- CPU

def test_oracle_gelu_is_torch_tanh_gelu():
    g = np.random.default_rng(0).normal(0, 3, 20000).astype(np.float32)
    g = R.bf16(g).astype(np.float32)
    ours = R._gelu_tanh_f32(g)
    ref = torch.nn.functional.gelu(torch.from_numpy(g), approximate="tanh").numpy()
    # 1 + tanh(.) cancels for negative inputs, so each library's tanh
    # rounding shows there as an absolute error of a few ulp of |x| (the
    # reference's own gelu_approx is one more such tanh): bound it so
    assert np.all(np.abs(ours - ref) <= 8 * 2.0 ** -23 * np.maximum(np.abs(g), 1.0))


def test_oracle_router_modes():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=2, scales="ones")
    x = to_np(synth.make_input(cfg, seed=2))
    gw = to_np(w["mlp.gate.weight"])
    i0, s0, _ = R.router(x, gw, cfg.top_k, R.ROUTER_SOFTMAX_TOPK_RENORM)
    i1, s1, _ = R.router(x, gw, cfg.top_k, R.ROUTER_TOPK_SOFTMAX)
    i2, s2, _ = R.router(x, gw, cfg.top_k, R.ROUTER_SOFTMAX_TOPK)
    assert np.array_equal(i0, i1) and np.array_equal(i0, i2)
    # top-k-then-softmax is the renormalised top-k of the full softmax
    assert np.all(np.abs(s1 - s0) <= np.abs(s0) * 2.0 ** -7)
    # without renormalisation the k weights sum below one, each below its
    # renormalised value
    assert np.all(s2.sum(-1) < 1.0) and np.all(s2 <= s0 * (1 + 2.0 ** -7))


def _fake_linear(out, inp, E=8, act=0):
    p = 1 << 12                                  # never dereferenced
    return _lib.Linear(format=_lib.FMT_VQ_U8, num_experts=E, out_features=out, in_features=inp,
                       codes=p, codebook=p, scales=p, codebook_size=256, dim=4, group_size=64,
                       activation=act)


def test_oracle_expert_scale():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=3, scales="ones")
    x = to_np(synth.make_input(cfg, seed=3))
    gw = to_np(w["mlp.gate.weight"])
    es = np.random.default_rng(3).uniform(0.5, 1.5, cfg.experts).astype(np.float32)
    i1, s1, _ = R.router(x, gw, cfg.top_k, R.ROUTER_TOPK_SOFTMAX)
    i2, s2, _ = R.router(x, gw, cfg.top_k, R.ROUTER_TOPK_SOFTMAX, es)
    assert np.array_equal(i1, i2)
    assert np.array_equal(s2, R.bf16(s1 * es[i1]))


def test_oracle_rms_norm_matches_torch():
    x = R.bf16(np.random.default_rng(4).normal(0, 2, (16, 512)).astype(np.float32))
    w = R.bf16(np.random.default_rng(5).uniform(0.5, 1.5, 512).astype(np.float32))
    ours = R.rms_norm(x, w, 1e-6)
    xt = torch.from_numpy(x)
    inv = torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6)
    ref = ((xt * inv).to(torch.bfloat16).float() * torch.from_numpy(w)).to(torch.bfloat16).float().numpy()
    # float32 rsqrt and a float32 mean against the exact mean and 1/sqrt:
    # the rare bf16 tie may land apart
    assert (ours != ref).mean() < 1e-3
    assert np.all(np.abs(ours - ref) <= np.abs(ref) * 2.0 ** -7)


@pytest.mark.gpu
@pytest.mark.parametrize("H", [256, 2816, 4096])
def test_router_rms_norm_is_bit_exact(H):
    """`vqmoe_rms_norm` (Gemma-4's router input) against the oracle's
    restatement, bit for bit: the exact mean of the squares rounded once,
    IEEE square root and division, two bf16 roundings."""
    from knurlogic_b200.gemma4 import Router
    g = np.random.default_rng(H)
    x = torch.from_numpy(R.bf16(g.normal(0, 2, (37, H)).astype(np.float32))).to(torch.bfloat16)
    scale = torch.from_numpy(g.uniform(0.5, 1.5, H).astype(np.float32))
    r = Router(torch.zeros(4, H).to(DEV), scale.to(DEV), torch.ones(4).to(DEV), 2)
    got = to_np(r.normalize(x.to(DEV)))
    ref = R.rms_norm(x.float().numpy(), r.norm_weight.float().cpu().numpy(), r.eps)
    assert np.array_equal(got, ref), f"{int((got != ref).sum())} of {ref.size} differ"


def test_moe_experts_arguments_are_checked():
    so = _lib.lib()
    H, I, E = 256, 128, 8
    g, u, d = _fake_linear(I, H, E, act=_lib.ACT_GEGLU), _fake_linear(I, H, E), _fake_linear(H, I, E)
    assert so.vqmoe_moe_experts_workspace_size(ctypes.byref(g), ctypes.byref(d), 4, 2) > \
        so.vqmoe_switch_glu_workspace_size(ctypes.byref(g), ctypes.byref(d), 4, 2)
    p = 1 << 12
    st = so.vqmoe_moe_experts(ctypes.byref(g), ctypes.byref(u), ctypes.byref(d), p, p, None, 4, 2, p, p,
                              1 << 30, None)
    assert _lib.STATUS[st] == "BAD_POINTER"
    st = so.vqmoe_moe_experts(ctypes.byref(g), ctypes.byref(u), ctypes.byref(u), p, p, p, 4, 2, p, p,
                              1 << 30, None)
    assert _lib.STATUS[st] == "BAD_SHAPE"


def test_variant_arguments_are_checked():
    so = _lib.lib()
    H, I, E = 256, 128, 8
    b = _lib.Block(hidden=H, num_experts=E, top_k=2, shared_inter=0, router_w=1 << 12,
                   gate=_fake_linear(I, H, E), up=_fake_linear(I, H, E), down=_fake_linear(H, I, E),
                   router_mode=5)
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), 1 << 12, 4, 1 << 12, 0, 1 << 12, 1 << 30, None)
    assert _lib.STATUS[st] == "BAD_FORMAT"
    assert b"router_mode" in so.vqmoe_last_error()
    b.router_mode = _lib.ROUTER_TOPK_SOFTMAX
    b.gate = _fake_linear(I, H, E, act=3)
    st = so.vqmoe_sparse_moe_block(ctypes.byref(b), 1 << 12, 4, 1 << 12, 0, 1 << 12, 1 << 30, None)
    assert _lib.STATUS[st] == "BAD_FORMAT"
    assert b"activation" in so.vqmoe_last_error()


# ------------------------------------------------------------------- GPU

def _router_ex(x, w, k, mode, expert_scale=None):
    T, H = x.shape
    E = w.shape[0]
    inds = torch.empty(T, k, dtype=torch.int32, device=DEV)
    scores = torch.empty(T, k, dtype=torch.float32, device=DEV)
    n = _lib.lib().vqmoe_router_workspace_size(T, E)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    es = None if expert_scale is None else expert_scale.to(DEV, torch.float32).contiguous()
    _lib.call("vqmoe_router_ex", x.data_ptr(), w.data_ptr(), None, T, H, E, k, mode,
              None if es is None else es.data_ptr(), inds.data_ptr(), scores.data_ptr(), None,
              ws.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return inds.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [_lib.ROUTER_TOPK_SOFTMAX, _lib.ROUTER_SOFTMAX_TOPK])
@pytest.mark.parametrize("name,tokens", [("c2", 64), ("c3", 1024)])
def test_router_variants_match_oracle(mode, name, tokens):
    """Indices bit-exact; weights within one bf16 step (CUDA's expf against
    numpy's exp in float32). c3's token count takes the multi-CTA top-k."""
    cfg = synth.CONFIGS[name]
    w = synth.make_weights(cfg, seed=6, scales="ones")
    x = synth.make_input(cfg, seed=6, tokens=tokens)
    inds, scores = _router_ex(x.to(DEV), w["mlp.gate.weight"].to(DEV), cfg.top_k, mode)
    oi, osc, _ = R.router(to_np(x), to_np(w["mlp.gate.weight"]), cfg.top_k, mode)
    assert np.array_equal(inds, oi), f"{int((inds != oi).sum())} indices differ"
    assert np.all(np.abs(scores - osc) <= np.abs(osc) * 2.0 ** -7 + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [_lib.ROUTER_TOPK_SOFTMAX, _lib.ROUTER_SOFTMAX_TOPK])
def test_block_router_variants_match_oracle(mode):
    from tests.conftest import assert_bf16_close
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=8, scales="random")
    x = synth.make_input(cfg, seed=8)
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k, router_mode=mode)
    y = to_np(blk(x.to(DEV)))
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True, router_mode=mode)
    assert_bf16_close(y, ref, f"router mode {mode}")


@pytest.mark.gpu
@pytest.mark.parametrize("name,tokens", [("c1", 16), ("c2", 64), ("pf", 1024)])
def test_geglu_block_matches_oracle(name, tokens):
    """GeGLU experts on the decode path (c1, c2) and on the tcgen05 prefill
    path ("pf": about 256 pairs per expert)."""
    from tests.conftest import assert_bf16_close
    cfg = (synth.MoEConfig("pf", 16, 4, 512, 256, 192, tokens, router="uniform")
           if name == "pf" else synth.CONFIGS[name])
    w = synth.make_weights(cfg, seed=12, scales="random")
    x = synth.make_input(cfg, seed=12, tokens=tokens)
    blk = SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k, activation=GeGLU())
    y = to_np(blk(x.to(DEV)))
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True, act=R.ACT_GEGLU)
    assert_bf16_close(y, ref, f"geglu {name}")


@pytest.mark.gpu
@pytest.mark.parametrize("name,tokens", [("c2", 64), ("c3", 2048)])
def test_router_expert_scale_matches_oracle(name, tokens):
    """Gemma-4's per-expert scale on the softmax over the top-k logits;
    c3's 2048 tokens take the blocked logits kernel and the multi-CTA top-k."""
    cfg = synth.CONFIGS[name]
    w = synth.make_weights(cfg, seed=9, scales="ones")
    x = synth.make_input(cfg, seed=9, tokens=tokens)
    es = torch.from_numpy(np.random.default_rng(9).uniform(0.5, 1.5, cfg.experts).astype(np.float32))
    inds, scores = _router_ex(x.to(DEV), w["mlp.gate.weight"].to(DEV), cfg.top_k, _lib.ROUTER_TOPK_SOFTMAX, es)
    oi, osc, _ = R.router(to_np(x), to_np(w["mlp.gate.weight"]), cfg.top_k, R.ROUTER_TOPK_SOFTMAX, es.numpy())
    assert np.array_equal(inds, oi), f"{int((inds != oi).sum())} indices differ"
    # one bf16 step from the softmax (CUDA's expf against numpy's exp), and
    # up to half a step more where the scaled weight is rounded again
    assert np.all(np.abs(scores - osc) <= np.abs(osc) * 2.0 ** -6 + 1e-30)


def _gemma_experts(w, cfg):
    from knurlogic_b200 import SwitchGLU, VQSwitchLinear
    from knurlogic_b200.gemma4 import Experts
    lin = {n: VQSwitchLinear(w[f"mlp.switch_mlp.{n}_proj.codes"].to(DEV), w[f"mlp.switch_mlp.{n}_proj.codebook"].to(DEV),
                             w[f"mlp.switch_mlp.{n}_proj.vq_scales"].to(DEV), group_size=cfg.group)
           for n in ("gate", "up", "down")}
    return Experts(SwitchGLU(lin["gate"], lin["up"], lin["down"], activation=GeGLU()))


@pytest.mark.gpu
@pytest.mark.parametrize("name,tokens", [("c2", 64), ("pf", 1024)])
def test_gemma4_router_and_experts_match_oracle(name, tokens):
    """The Gemma-4 modules end to end: the router on its own normalised
    input (the oracle takes the module's RMS-normed rows, an unpinned step
    restated separately), then the GeGLU experts and the weighted sum on the
    decode path (c2) and the tcgen05 prefill path ("pf")."""
    from tests.conftest import assert_bf16_close
    from knurlogic_b200.gemma4 import Router
    cfg = (synth.MoEConfig("pf", 16, 4, 512, 256, 0, tokens, router="uniform")
           if name == "pf" else synth.CONFIGS[name])
    w = synth.make_weights(cfg, seed=14, scales="random")
    x = synth.make_input(cfg, seed=14, tokens=tokens)
    g = np.random.default_rng(14)
    scale = torch.from_numpy(g.uniform(0.5, 1.5, cfg.hidden).astype(np.float32))
    pes = torch.from_numpy(g.uniform(0.5, 1.5, cfg.experts).astype(np.float32))
    router = Router(w["mlp.gate.weight"].to(DEV), scale.to(DEV), pes.to(DEV), cfg.top_k)
    inds, weights = router(x.to(DEV))
    xn = to_np(router.normalize(x.to(DEV)))
    oi, osc, _ = R.router(xn, to_np(w["mlp.gate.weight"]), cfg.top_k, R.ROUTER_TOPK_SOFTMAX, pes.numpy())
    assert np.array_equal(inds.cpu().numpy(), oi)
    assert np.all(np.abs(weights.float().cpu().numpy() - osc) <= np.abs(osc) * 2.0 ** -6 + 1e-30)
    experts = _gemma_experts(w, cfg)
    y = to_np(experts(x.to(DEV), inds, weights))
    p = oracle_params(w)
    ref = R.moe_experts(to_np(x), oi, osc, p["gate"], p["up"], p["down"], vq=True, act=R.ACT_GEGLU)
    assert_bf16_close(y, ref, f"gemma4 experts {name}")
