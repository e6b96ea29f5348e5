"""Parity of the CUDA path (through the C ABI) with the oracle, on a B200.

Bars:
* the reference golden (dense bf16 experts): bit for bit;
* router indices: bit for bit (the logits are correctly rounded);
* dequantised VQ weights: bit for bit;
* router weights and sigmoid gate: within one bf16 step (CUDA's expf vs
  numpy's exp in float32);
* layer outputs (bf16): `tests.conftest.assert_bf16_close` -- max
  |gpu - oracle| <= 1e-2 * max |oracle| (the north star's 1e-2 relative)
  on every element, and within 2 bf16 steps of |oracle| + 2^-9 rms(oracle)
  on all but 0.5% of the elements.
"""
import ctypes

import numpy as np
import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, SwitchGLU, VQSwitchLinear, _lib, synth, tensor_split
from oracle import moe_ref as R
from tests.conftest import assert_bf16_close, golden_state_dict, oracle_params, to_np

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _cuda(w):
    return {k: v.to(DEV) for k, v in w.items()}


def _router(x, w, k, shared_gate=None):
    T, H = x.shape
    E = w.shape[0]
    inds = torch.empty(T, k, dtype=torch.int32, device=DEV)
    scores = torch.empty(T, k, dtype=torch.float32, device=DEV)
    sg = torch.empty(T, dtype=torch.float32, device=DEV)
    n = _lib.lib().vqmoe_router_workspace_size(T, E)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    _lib.call("vqmoe_router", x.data_ptr(), w.data_ptr(),
              shared_gate.data_ptr() if shared_gate is not None else None, T, H, E, k,
              inds.data_ptr(), scores.data_ptr(), sg.data_ptr(), ws.data_ptr(), n,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return inds.cpu().numpy(), scores.cpu().numpy(), sg.cpu().numpy()


def test_golden_block_is_bit_exact_on_gpu(golden):
    """The reference's bf16 MoE-block golden, through SparseMoeBlock and
    vqmoe_sparse_moe_block with dense bf16 experts."""
    blk = SparseMoeBlock.from_weights(_cuda(golden_state_dict(golden)), int(golden["top_k"]))
    x = torch.from_numpy(golden["x"]).to(torch.bfloat16).to(DEV)
    y = to_np(blk(x))
    g = golden["golden"]
    assert np.array_equal(y, g), f"{int((y != g).sum())} of {g.size} differ, max {np.abs(y - g).max()}"


@pytest.mark.parametrize("name,tokens", [("c1", 16), ("c2", 64), ("c3", 512), ("c4", 64)])
def test_router_indices_are_bit_exact(name, tokens):
    cfg = synth.CONFIGS[name]
    w = synth.make_weights(cfg, seed=5, scales="random")
    x = synth.make_input(cfg, seed=5, tokens=tokens)
    sgw = w.get("mlp.shared_expert_gate.weight")
    inds, scores, sg = _router(x.to(DEV), w["mlp.gate.weight"].to(DEV), cfg.top_k,
                               sgw.to(DEV) if sgw is not None else None)
    oi, osc, _ = R.router(to_np(x), to_np(w["mlp.gate.weight"]), cfg.top_k)
    assert np.array_equal(inds, oi), f"{int((inds != oi).sum())} indices differ"
    assert np.all(np.abs(scores - osc) <= np.abs(osc) * 2.0 ** -7 + 1e-30)
    if sgw is not None:
        gl = R.linear(to_np(x), to_np(sgw))[:, 0]
        osg = R.bf16(R._sigmoid_f32(gl))
        assert np.all(np.abs(sg - osg) <= np.abs(osg) * 2.0 ** -7)


def test_dequantised_weights_are_bit_exact():
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, seed=3, scales="random")
    q = "mlp.switch_mlp.down_proj."
    m = VQSwitchLinear(w[q + "codes"].to(DEV), w[q + "codebook"].to(DEV),
                       w[q + "vq_scales"].to(DEV), group_size=64)
    got = to_np(m.dequantize(2, 3))
    ref = R.dequant(to_np(w[q + "codes"])[2:5], to_np(w[q + "codebook"]),
                    to_np(w[q + "vq_scales"])[2:5], 64)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("E,OUT,IN", [(3, 32, 192), (2, 48, 320), (2, 64, 512)])
def test_device_layout_matches_the_oracle_and_inverts(E, OUT, IN):
    codes = torch.randint(0, 256, (E, OUT, IN // 4), dtype=torch.uint8)
    scales = (0.5 + torch.rand(E, OUT, IN // 64)).to(torch.float16)
    m = VQSwitchLinear(codes.to(DEV), torch.zeros(256, 4, dtype=torch.float16, device=DEV),
                       scales.to(DEV), group_size=64)
    dc, ds = m.prepared()
    rc, rs = R.prepare_vq(codes.numpy(), scales.numpy())
    assert np.array_equal(dc.cpu().numpy(), rc)
    assert np.array_equal(ds.cpu().numpy().view(np.uint16), rs.view(np.uint16))
    back = torch.empty_like(codes, device=DEV)
    _lib.call("vqmoe_unprepare_codes", dc.data_ptr(), E, OUT, IN, back.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    assert torch.equal(back.cpu(), codes)


def _vq_linear(w, name):
    q = f"mlp.switch_mlp.{name}."
    return VQSwitchLinear(w[q + "codes"].to(DEV), w[q + "codebook"].to(DEV),
                          w[q + "vq_scales"].to(DEV), group_size=64)


@pytest.mark.parametrize("tokens", [1, 13, 40])
def test_switch_linear_matches_oracle(tokens):
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, seed=tokens, scales="random")
    x = synth.make_input(cfg, seed=tokens, tokens=tokens)
    m = _vq_linear(w, "up_proj")
    rng = np.random.default_rng(tokens)
    idx = np.stack([rng.choice(cfg.experts, cfg.top_k, replace=False) for _ in range(tokens)])
    y = m(x.to(DEV)[:, None, None, :], torch.from_numpy(idx).to(DEV))
    assert y.shape == (tokens, cfg.top_k, 1, cfg.inter)
    p = oracle_params(w)
    ref = R.switch_linear(np.repeat(to_np(x), cfg.top_k, 0), idx.reshape(-1), p["up"], vq=True)
    assert_bf16_close(to_np(y).reshape(-1, cfg.inter), ref, "switch_linear")
    # the sorted form: x [N, 1, IN] with indices [N]
    order = np.argsort(idx.reshape(-1), kind="stable")
    xs = np.repeat(to_np(x), cfg.top_k, 0)[order]
    ys = m(torch.from_numpy(xs).to(torch.bfloat16).to(DEV)[:, None, :],
           torch.from_numpy(idx.reshape(-1)[order]).to(DEV), sorted_indices=True)
    assert ys.shape == (tokens * cfg.top_k, 1, cfg.inter)
    assert np.array_equal(to_np(ys)[:, 0], to_np(y).reshape(-1, cfg.inter)[order])


def test_switch_glu_matches_oracle():
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, seed=21, scales="random")
    x = synth.make_input(cfg, seed=21)
    glu = SwitchGLU(_vq_linear(w, "gate_proj"), _vq_linear(w, "up_proj"), _vq_linear(w, "down_proj"))
    p = oracle_params(w)
    inds, _, _ = R.router(to_np(x), p["router"], cfg.top_k)
    y = glu(x.to(DEV), torch.from_numpy(inds).to(DEV))
    ref = R.switch_glu(to_np(x), inds, p["gate"], p["up"], p["down"], vq=True)
    assert_bf16_close(to_np(y), ref, "switch_glu")


@pytest.mark.parametrize("name,tokens,seed", [("c1", 16, 0), ("c1", 1, 1), ("c1", 7, 2),
                                              ("c2", 64, 0), ("c2", 5, 3), ("c4", 16, 4)])
def test_block_matches_oracle(name, tokens, seed):
    cfg = synth.CONFIGS[name]
    w = synth.make_weights(cfg, seed=seed, scales="random")
    x = synth.make_input(cfg, seed=seed, tokens=tokens)
    blk = SparseMoeBlock.from_weights(_cuda(w), cfg.top_k)
    y = to_np(blk(x.to(DEV)))
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y, ref, f"{name} T={tokens}")


def test_block_beyond_one_launch_of_tokens():
    """T > 2048 runs as independent token chunks (here a dense first chunk
    on the tcgen05 prefill path and a 52-token second chunk on the decode
    path); tokens on either side of the cut, and the same tokens run alone
    (decode path), match the oracle."""
    cfg = synth.MoEConfig("small", 16, 4, 256, 128, 64, 2100)
    w = synth.make_weights(cfg, seed=9, scales="random")
    x = synth.make_input(cfg, seed=9)
    blk = SparseMoeBlock.from_weights(_cuda(w), cfg.top_k)
    y = to_np(blk(x.to(DEV)))
    y_tail = to_np(blk(x[2000:].to(DEV)))
    ref = R.sparse_moe_block(to_np(x[2000:]), oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y[2000:], ref, "chunked")
    assert_bf16_close(y_tail, ref, "alone")


@pytest.mark.parametrize("zipf,hidden,inter", [(0.0, 512, 256), (1.1, 512, 256), (1.1, 384, 320)])
def test_prefill_block_matches_oracle(zipf, hidden, inter):
    """Many pairs per expert (about 256 here): the routed experts take the
    tcgen05 grouped-GEMM path (128-pair tiles, partial last tiles, a Zipf
    load imbalance), and the shared expert (192 rows: a partial row tile) the
    tcgen05 dense GEMMs. hidden = 384: the last 256-row down tile is half
    out of range; inter = 320: down's inputs end inside a 256-input chunk."""
    cfg = synth.MoEConfig("pf", 16, 4, hidden, inter, 192, 1024, router="uniform", zipf=zipf)
    w = synth.make_weights(cfg, seed=17, scales="random")
    x = synth.make_input(cfg, seed=17)
    blk = SparseMoeBlock.from_weights(_cuda(w), cfg.top_k)
    y = to_np(blk(x.to(DEV)))
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y, ref, f"prefill zipf={zipf} H={hidden} I={inter}")


def test_small_codebook_and_idle_experts():
    """K = 200 < 256, and 64 experts for 3 tokens (most experts idle)."""
    cfg = synth.MoEConfig("k200", 64, 2, 256, 64, 0, 3, codebook_size=200)
    w = synth.make_weights(cfg, seed=4, scales="random")
    x = synth.make_input(cfg, seed=4)
    blk = SparseMoeBlock.from_weights(_cuda(w), cfg.top_k)
    ref = R.sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(to_np(blk(x.to(DEV))), ref, "K=200")


def test_out_of_range_codes_are_refused():
    codes = torch.full((1, 16, 16), 250, dtype=torch.uint8, device=DEV)
    m = VQSwitchLinear(codes, torch.zeros(200, 4, dtype=torch.float16, device=DEV),
                       torch.ones(1, 16, 1, dtype=torch.float16, device=DEV), group_size=64)
    with pytest.raises(ValueError, match="codebook size 200"):
        m.prepared()


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tensor_split_emulated_on_one_gpu(n):
    """Each rank's cut (T = 16) through the C ABI with float32 output,
    summed in float32 and rounded once: the reference's Reduce. C2 for 2
    and 4 ranks; its I 768 refuses 8, which runs at I 1536 (c4's width)."""
    cfg = synth.CONFIGS["c2"] if n < 8 else synth.MoEConfig("tp8", 32, 8, 1024, 1536, 512, 16)
    w = synth.make_weights(cfg, seed=12, scales="random")
    x = synth.make_input(cfg, seed=12, tokens=16).to(DEV)
    acc = torch.zeros(16, cfg.hidden, dtype=torch.float32, device=DEV)
    for r in range(n):
        blk = tensor_split.build_block(_cuda(w), cfg.top_k, rank=r, n=n)
        part = torch.empty(16, cfg.hidden, dtype=torch.float32, device=DEV)
        blk.forward_into(x, part)
        # a float32 partial holds a bf16 value
        assert torch.equal(part, part.to(torch.bfloat16).float())
        acc += part
    y = to_np(acc.to(torch.bfloat16))
    ref = R.tp_sparse_moe_block(to_np(x), oracle_params(w), cfg.top_k, vq=True, n=n)
    assert_bf16_close(y, ref, f"tp{n}")


def test_block_replays_in_a_cuda_graph():
    cfg = synth.CONFIGS["c2"]
    w = synth.make_weights(cfg, seed=1, scales="random")
    blk = SparseMoeBlock.from_weights(_cuda(w), cfg.top_k)
    x = synth.make_input(cfg, seed=1).to(DEV)
    out = torch.empty_like(x)
    eager = blk(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blk.forward_into(x, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        blk.forward_into(x, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
