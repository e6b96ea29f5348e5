"""Parity at the benchmark configurations' own shapes (on a B200).

* c3: H 2048, 128 experts top-8, I 768 + shared 768, 4096 prefill tokens
  with Zipf 1.1 routing -- two 2048-token launches on the tcgen05 grouped
  GEMM. Tokens are independent, so a seeded 256-token subset of the GPU's
  output is compared with the oracle run on those tokens alone.
* c4: H 4096, 256 experts top-8, I 1536, 256 tokens (the tensor-split
  configuration's MoE layer, whole), a 32-token subset against the oracle.
* The decode (mma.sync) and prefill (tcgen05) expert paths on the same
  tokens: both within the oracle bar, and close to each other.
* The routing at 257-512 tokens, where one launch spreads the top-k over 64
  CTAs with global atomic ranks and the last CTA scatters the per-expert
  lists: router indices equal the oracle's and the per-expert counts and
  lists equal a CPU histogram of them, read from the block's workspace.

Reference: `SparseMoeBlock.__call__`, `qwen3_5.py:170-192`.
"""
import numpy as np
import pytest
import torch

from knurlogic_b200 import SparseMoeBlock, synth
from oracle import moe_ref as R
from tests.conftest import assert_bf16_close, oracle_params, to_np

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _block(cfg, seed, scales="random"):
    w = synth.make_weights(cfg, seed=seed, scales=scales)
    return w, SparseMoeBlock.from_weights({k: v.to(DEV) for k, v in w.items()}, cfg.top_k)


def _subset(T, n, seed):
    return np.sort(np.random.default_rng(seed).choice(T, n, replace=False))


def test_c3_prefill_at_full_shape():
    cfg = synth.CONFIGS["c3"]
    w, blk = _block(cfg, seed=41)
    x = synth.make_input(cfg, seed=41)
    y = to_np(blk(x.to(DEV)))
    blk.check_status()
    sel = _subset(cfg.tokens, 256, 41)
    ref = R.sparse_moe_block(to_np(x)[sel], oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y[sel], ref, "c3 T=4096 (256-token subset)")


def test_c4_at_full_shape():
    cfg = synth.CONFIGS["c4"]
    w, blk = _block(cfg, seed=43)
    x = synth.make_input(cfg, seed=43)
    y = to_np(blk(x.to(DEV)))
    blk.check_status()
    sel = _subset(cfg.tokens, 32, 43)
    ref = R.sparse_moe_block(to_np(x)[sel], oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y[sel], ref, "c4 T=256 (32-token subset)")


@pytest.mark.parametrize("scales", ["ones", "random"])
def test_decode_and_prefill_paths_agree(scales):
    """The same 1024 tokens of a c2 layer as one call (8192 pairs, 64 per
    expert: the tcgen05 path) and as 16 calls of 64 tokens (the mma.sync
    path). With unit scales both paths multiply the same fp16 weights and
    differ only in float32 summation order; with random scales the decode
    kernels apply each group's scale to the partial sum, s * (codebook . x),
    where the prefill kernel multiplies fp16(codebook * s) -- at most half an
    fp16 step per weight."""
    cfg = synth.CONFIGS["c2"].with_tokens(1024)
    w, blk = _block(cfg, seed=47, scales=scales)
    x = synth.make_input(cfg, seed=47).to(DEV)
    y_pf = to_np(blk(x))
    y_dc = np.concatenate([to_np(blk(x[i:i + 64])) for i in range(0, 1024, 64)])
    blk.check_status()
    assert_bf16_close(y_dc, y_pf, f"decode vs prefill ({scales} scales)")
    sel = _subset(1024, 96, 47)
    ref = R.sparse_moe_block(to_np(x.cpu())[sel], oracle_params(w), cfg.top_k, vq=True)
    assert_bf16_close(y_pf[sel], ref, "prefill path")
    assert_bf16_close(y_dc[sel], ref, "decode path")


def _routing_tables(blk, T):
    """(inds [T, k], cnt [E], off [E], list [T*k]) from the block's
    workspace after a call. The regions, each 256-byte aligned, in the order
    the library carves them: status words, logits [T, E+1] f32, inds [T*k]
    i32, scores, sgate [T], the fp16 copy of x [T, H], then the routing
    tables cnt [E+1], off [E+1], list [T*k]."""
    E, k, H = blk.num_experts, blk.top_k, blk.hidden
    off = 0
    regions = {}
    for name, nbytes in (("status", 256), ("logits", T * (E + 1) * 4), ("inds", T * k * 4),
                         ("scores", T * k * 4), ("sgate", T * 4), ("x16", T * H * 2),
                         ("cnt", (E + 1) * 4), ("off", (E + 1) * 4), ("list", T * k * 4)):
        off = (off + 255) // 256 * 256
        regions[name] = (off, nbytes)
        off += nbytes
    ws = blk._ws.cpu()

    def get(name):
        o, n = regions[name]
        return ws[o:o + n].view(torch.int32).numpy()
    return get("inds").reshape(T, k), get("cnt")[:E], get("off")[:E], get("list")


@pytest.mark.parametrize("name,tokens", [("c2", 512), ("c4", 512), ("c2", 300)])
def test_spread_routing_at_up_to_512_tokens(name, tokens):
    cfg = synth.CONFIGS[name].with_tokens(tokens)
    w, blk = _block(cfg, seed=53)
    x = synth.make_input(cfg, seed=53)
    y = to_np(blk(x.to(DEV)))
    torch.cuda.synchronize()
    blk.check_status()
    inds, cnt, off, lst = _routing_tables(blk, tokens)
    p = oracle_params(w)
    oi, _, _ = R.router(to_np(x), p["router"], cfg.top_k)
    assert np.array_equal(inds, oi), f"{int((inds != oi).sum())} router indices differ"
    hist = np.bincount(oi.reshape(-1), minlength=cfg.experts)
    assert np.array_equal(cnt, hist)
    flat = oi.reshape(-1)
    for e in np.nonzero(hist)[0]:
        got = np.sort(lst[off[e]:off[e] + cnt[e]])
        assert np.array_equal(got, np.nonzero(flat == e)[0]), f"expert {e}'s pair list"
    sel = _subset(tokens, 32, 53)
    ref = R.sparse_moe_block(to_np(x)[sel], p, cfg.top_k, vq=True)
    assert_bf16_close(y[sel], ref, f"{name} T={tokens} (32-token subset)")
