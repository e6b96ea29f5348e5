"""The oracle, pinned against the reference before anything is checked
against it (CPU only)."""
from fractions import Fraction

import numpy as np
import pytest
import torch

from oracle import moe_ref as R


def test_oracle_reproduces_the_reference_bf16_moe_golden(golden):
    """`qwen3_5_moe/bf16/0.mlp` of the reference's qwen_reference.npz: the
    bf16 MoE block the reference requires MLX to match bit for bit
    (tests/engine/test_qwen_reference.py:213-241)."""
    p = {k: golden[k] for k in ("router", "gate", "up", "down", "shared_gate",
                                "shared_up", "shared_down", "shared_expert_gate")}
    for k, v in p.items():
        assert np.array_equal(R.bf16(v), v), f"{k} is not bf16-valued"
    y = R.sparse_moe_block(golden["x"], p, int(golden["top_k"]), vq=False)
    assert y.shape == golden["golden"].shape == (21, 32)
    assert np.array_equal(y, golden["golden"]), \
        f"{int((y != golden['golden']).sum())} of {y.size} differ"


def test_bf16_rounding_of_float32_matches_torch():
    rng = np.random.default_rng(0)
    a = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 100000),
                        np.array([0.0, -0.0, 1.0, 65504.0, 3.0e38], np.float32)]).astype(np.float32)
    got = R.bf16(a)
    ref = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def _exact_bf16(x: float) -> float:
    """Round a float64 to bf16 with rationals (nearest, ties to even)."""
    if x == 0:
        return 0.0
    f = Fraction(x)
    sign = -1 if f < 0 else 1
    f = abs(f)
    e = 0
    while f >= 2:
        f /= 2
        e += 1
    while f < 1:
        f *= 2
        e -= 1
    m = f * 128                      # 8 significant bits: 1.xxxxxxx
    lo = int(m)
    rem = m - lo
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and lo % 2 == 1):
        lo += 1
    return sign * float(Fraction(lo, 128) * Fraction(2) ** e)


def test_bf16_rounding_of_float64_is_single_rounding():
    rng = np.random.default_rng(1)
    a = rng.standard_normal(3000) * 10.0 ** rng.integers(-20, 20, 3000)
    # values straddling bf16 midpoints: a float32 step would double-round
    mids = (1.0 + (2 * np.arange(1, 200) + 1) / 256.0)
    a = np.concatenate([a, mids + 1e-12, mids - 1e-12, mids]).astype(np.float64)
    got = R.bf16(a)
    ref = np.array([_exact_bf16(float(v)) for v in a], np.float32)
    assert np.array_equal(got, ref)


def test_device_layout_gives_each_lane_its_mma_codes():
    """In the device layout, lane 4g+t's 8 bytes of (half, mt, h) are the
    codes of row 16mt+8h+g it feeds into MMA sub-steps 8*half .. 8*half+7
    (chunk code 4q+t), and the 8 padded rows / tail inputs are zero."""
    rng = np.random.default_rng(2)
    E, OUT, IN = 2, 48, 320                # 2 row blocks (16 padded), 2 chunks
    codes = rng.integers(1, 256, (E, OUT, IN // 4), dtype=np.uint8)
    scales = (0.5 + rng.random((E, OUT, IN // 64))).astype(np.float16)
    dc, ds = R.prepare_vq(codes, scales)
    RB, C = 2, 2
    assert dc.size == E * RB * C * 2048 and ds.size == E * RB * C * 128
    for e, rb, c, half, mt, h, g, t in [(1, 0, 1, 0, 1, 0, 3, 2), (0, 1, 0, 1, 0, 1, 7, 0),
                                         (1, 1, 1, 1, 0, 1, 5, 3)]:
        tile = (e * RB + rb) * C + c
        got = dc[tile * 2048 + half * 1024 + (2 * mt + h) * 256 + (4 * g + t) * 8:][:8]
        row = rb * 32 + mt * 16 + h * 8 + g
        for b in range(8):
            u = c * 64 + 4 * (half * 8 + b) + t
            want = codes[e, row, u] if row < OUT and u < IN // 4 else 0
            assert got[b] == want
        for jj in range(2):
            grp = c * 4 + half * 2 + jj
            want = scales[e, row, grp] if row < OUT and grp < IN // 64 else 0
            assert ds[tile * 128 + half * 64 + (2 * mt + h) * 16 + 2 * g + jj] == want
    # padded rows 48..63 carry zero scales: their weights are exactly zero
    assert (dc.size - np.count_nonzero(dc)) >= E * 16 * C * 64


def test_dequant_is_the_rounded_product_of_codebook_and_scale():
    rng = np.random.default_rng(3)
    cb = (rng.standard_normal((256, 4)) * 0.02).astype(np.float16)
    codes = rng.integers(0, 256, (2, 16, 32), dtype=np.uint8)
    sc = (0.5 + rng.random((2, 16, 2))).astype(np.float16)
    w = R.dequant(codes, cb, sc, 64)
    e, o, i = 1, 7, 77
    expect = np.float16(np.float32(cb[codes[e, o, i // 4], i % 4]) * np.float32(sc[e, o, i // 64]))
    assert w[e, o, i] == np.float32(expect)
    lazy = R.LazyVQ(codes, cb, sc, 64)
    assert np.array_equal(lazy[1], w[1])


def test_router_picks_by_logit_with_ties_to_the_lower_expert():
    x = np.ones((1, 16), np.float32)
    wg = np.zeros((6, 16), np.float32)
    wg[[1, 4], 0] = 0.5               # a tie between experts 1 and 4
    wg[2, 0] = 0.25
    inds, scores, logits = R.router(x, wg, 3)
    assert inds.tolist() == [[1, 4, 2]]
    assert scores[0, 0] == scores[0, 1]
    assert np.isclose(scores.sum(), 1.0, atol=1e-2)


def test_tensor_split_of_one_rank_is_the_block():
    rng = np.random.default_rng(4)
    H, E, I = 64, 4, 32
    p = {"router": R.bf16(rng.standard_normal((E, H)) * 0.1),
         "gate": R.bf16(rng.standard_normal((E, I, H)) * 0.1),
         "up": R.bf16(rng.standard_normal((E, I, H)) * 0.1),
         "down": R.bf16(rng.standard_normal((E, H, I)) * 0.1)}
    x = R.bf16(rng.standard_normal((5, H)))
    a = R.sparse_moe_block(x, p, 2, vq=False)
    b = R.tp_sparse_moe_block(x, p, 2, vq=False, n=1)
    assert np.array_equal(a, b)
    c = R.tp_sparse_moe_block(x, p, 2, vq=False, n=2)
    assert np.abs(c - a).max() <= 2 * np.abs(a).max() * 2 ** -8
