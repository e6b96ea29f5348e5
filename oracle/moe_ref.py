"""CPU oracle for the VQ-MoE expert layer -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what Knurlogic's Qwen3.5-MoE sparse block
computes, so the CUDA path can be checked against it. Only `tests/`,
`__graft_entry__.smoke()` and the CPU-baseline legs of `bench.py` may import
it; the product path (`knurlogic_b200`) never does, and has no CPU fallback.

Parity status
-------------
* Router, SwiGLU, top-k combine and shared expert (dense bf16 experts):
  PINNED. `sparse_moe_block` on dense bf16 experts reproduces the reference
  golden `tests/support/goldens/qwen_reference.npz["qwen3_5_moe/bf16/0.mlp"]`
  bit for bit (committed here as `tests/golden/qwen3_5_moe_bf16_mlp.npz`, see
  `tests/golden/make_golden.py`). The reference test that holds MLX to the
  same golden is `tests/engine/test_qwen_reference.py:213-241`.
* VQ dequantisation: PARITY UNPINNED. The reference ships no VQ runtime and
  no VQ numerics test (the kernels live in each artifact's `model.py`,
  `src/knurlogic/engine/model/loading.py:106-177`). The layout is pinned by
  `src/knurlogic/engine/families/deepseek/heads/deepseek_v4.py:35-42,
  77-130`; the arithmetic below is this build's definition (see `dequant`).

Rounding recipe (reference order, `qwen3_5.py:35-40, 108-112, 170-192`):
* a matmul is computed exactly (float64 over operands that are bf16 / fp16
  values; every product is exact) and rounded once to bf16;
* softmax, top-k and renormalisation in float32, the weights then rounded
  to bf16;
* silu / sigmoid in float32 on a bf16 input, rounded once to bf16;
* elementwise products of bf16 values are rounded once to bf16;
* the top-k sum accumulates in float32 and rounds once.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16", "f16", "f16_sat", "dequant", "prepare_vq",
    "linear", "router", "switch_linear", "switch_glu", "sparse_moe_block",
    "tp_sparse_moe_block", "shard_block_params", "LazyVQ", "LazyAffine", "dequant_affine",
    "unpack_affine",
]


# ----------------------------------------------------------------- rounding

def bf16(a) -> np.ndarray:
    """Round to bfloat16 (nearest, ties to even), returned as float32.

    Rounds float64 input directly (no intermediate float32 rounding, which
    could double-round a value that lands on a bf16 midpoint)."""
    a = np.asarray(a)
    if a.dtype == np.float64:
        # round the float64 significand straight to bf16's 8 bits (RNE);
        # the result has 8 significant bits, so the float32 cast after it
        # is exact for every value in float32's normal range
        u = np.ascontiguousarray(a).view(np.uint64)
        low = u & np.uint64((1 << 45) - 1)
        half = np.uint64(1 << 44)
        odd = (u >> np.uint64(45)) & np.uint64(1)
        up = (low > half) | ((low == half) & (odd == 1))
        r = (u & ~np.uint64((1 << 45) - 1)) + np.where(
            up, np.uint64(1 << 45), np.uint64(0))
        out = r.view(np.float64).astype(np.float32)
        # below float32's normal range bf16 rounds at a coarser position:
        # take the float32 route there (and for inf / nan)
        small = ~(np.abs(a) >= 2.0 ** -126) | ~np.isfinite(a)
        if small.any():
            out = np.where(small, bf16(a.astype(np.float32)), out)
        return out.astype(np.float32).reshape(a.shape)
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    u = ((u.astype(np.uint64) + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000)
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


def f16(a) -> np.ndarray:
    """Round to IEEE half (nearest even), returned as float32."""
    return np.asarray(a).astype(np.float16).astype(np.float32)


F16_MAX = 65504.0


def f16_sat(a) -> np.ndarray:
    """bf16 activations as the VQ expert matmul consumes them: converted to
    fp16 (exact for |a| in [2^-14, 65504]; smaller values become fp16
    subnormals) and saturated to +-65504 instead of overflowing to inf."""
    a = np.clip(np.asarray(a, np.float32), -F16_MAX, F16_MAX)
    return f16(a)


# ------------------------------------------------------------- VQ weights

def dequant(codes: np.ndarray, codebook: np.ndarray, scales: np.ndarray,
            group_size: int) -> np.ndarray:
    """Dense weights of a VQ switch linear, [E, OUT, IN] float32 holding fp16
    values.

    Layout (reference `deepseek_v4.py:35-42, 111-130`): `codes [E, OUT,
    IN/dim]` one code per entry (uint8 when K <= 256), `codebook [K, dim]`
    fp16, `vq_scales [E, OUT, IN/group]` fp16, group = IN / vq_scales.shape[-1].

    Arithmetic (this build's definition; the reference pins none):
        W[e, o, i] = fp16( f32(codebook[codes[e, o, i // dim], i % dim])
                           * f32(vq_scales[e, o, i // group]) )
    i.e. the exact product rounded once to fp16 -- the dense fp16 expert the
    VQ runtime's prefill path decodes to (`src/knurlogic/tuning/measured.py:
    21-33`, "experts decoded to dense fp16")."""
    E, OUT, NC = codes.shape
    K, dim = codebook.shape
    IN = NC * dim
    cb = codebook.astype(np.float32)
    w = cb[codes.astype(np.int64)].reshape(E, OUT, IN)
    s = np.repeat(scales.astype(np.float32), group_size, axis=-1)
    assert s.shape == w.shape, (s.shape, w.shape)
    return f16(w * s)


class LazyVQ:
    """Dequantised expert weights computed one expert at a time (`w[e]`),
    so the oracle can hold a full-size layer without materialising it."""

    def __init__(self, codes, codebook, scales, group_size: int):
        self.codes, self.codebook, self.scales = codes, codebook, scales
        self.group_size = group_size
        E, OUT, NC = codes.shape
        self.shape = (E, OUT, NC * codebook.shape[1])

    def __getitem__(self, e: int) -> np.ndarray:
        return dequant(self.codes[e:e + 1], self.codebook,
                       self.scales[e:e + 1], self.group_size)[0]


def prepare_vq(codes: np.ndarray, scales: np.ndarray):
    """The device layout `vqmoe_prepare_vq` writes (restated from its
    definition, for the layout tests): rows padded to a multiple of 32,
    inputs to a multiple of 256 (padding codes and scales 0), tiles of 32
    rows x 256 inputs. In a 2048-byte code tile, row r = 16*mt + 8*h + g and
    chunk code u = 4*(8*half + b) + t sit at half*1024 + (2*mt + h)*256 +
    (4*g + t)*8 + b; in a 128-element scale tile, group 4*c + 2*half + jj of
    row r sits at half*64 + (2*mt + h)*16 + 2*g + jj.
    Returns (codes uint8 [tiles*2048], scales fp16 [tiles*128])."""
    E, OUT, NC = codes.shape
    IN = NC * 4
    RB, C = -(-OUT // 32), -(-IN // 256)
    cp = np.zeros((E, RB * 32, C * 64), np.uint8)
    cp[:, :OUT, :NC] = codes
    sp = np.zeros((E, RB * 32, C * 4), np.float16)
    sp[:, :OUT, :IN // 64] = scales
    # codes: [E, RB, mt, h, g, C, half, b, t] -> [E, RB, C, half, mt, h, g, t, b]
    c9 = cp.reshape(E, RB, 2, 2, 8, C, 2, 8, 4)
    dc = c9.transpose(0, 1, 5, 6, 2, 3, 4, 8, 7).reshape(-1)
    # scales: [E, RB, mt, h, g, C, half, jj] -> [E, RB, C, half, mt, h, g, jj]
    s8 = sp.reshape(E, RB, 2, 2, 8, C, 2, 2)
    ds = s8.transpose(0, 1, 5, 6, 2, 3, 4, 7).reshape(-1)
    return np.ascontiguousarray(dc), np.ascontiguousarray(ds)


# ---------------------------------------------------------------- matmuls

def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16(x @ w.T), exact accumulation (float64 over exact products)."""
    return bf16(x.astype(np.float64) @ w.astype(np.float64).T)


def _silu_f32(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1) + np.exp(-g))).astype(np.float32)


def _gelu_tanh_f32(g: np.ndarray) -> np.ndarray:
    """gelu's tanh form in float32 (mlx `nn.gelu_approx`, torch's
    gelu_pytorch_tanh): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    g = g.astype(np.float32)
    c = np.float32(0.7978845608028654)
    inner = c * (g + np.float32(0.044715) * g * g * g)
    return (np.float32(0.5) * g * (np.float32(1) + np.tanh(inner.astype(np.float32)))).astype(np.float32)


def _sigmoid_f32(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    with np.errstate(over="ignore"):
        return (np.float32(1) / (np.float32(1) + np.exp(-g))).astype(np.float32)


ROUTER_SOFTMAX_TOPK_RENORM, ROUTER_TOPK_SOFTMAX, ROUTER_SOFTMAX_TOPK = 0, 1, 2


def router(x: np.ndarray, gate_w: np.ndarray, k: int, mode: int = ROUTER_SOFTMAX_TOPK_RENORM,
           expert_scale: np.ndarray | None = None):
    """`SparseMoeBlock.__call__` router, `qwen3_5.py:174-179`.

    logits = bf16(x @ Wg^T); probs = softmax_f32(logits); the k largest;
    scores = bf16(p_sel / sum(p_sel)) with the renormalisation in float32.
    The Qwen4-exp variants (`qwen4_exp.py:800-815`): mode 1
    (`norm_topk_prob`) scores = bf16(softmax_f32 over the k selected
    logits) -- e_sel / sum(e_sel), e = exp(l - max), the max being the top-1
    logit; mode 2 scores = bf16(p_sel), not renormalised. Gemma-4's
    per-expert scale (`gemma4_text.py:179-180`, with mode 1):
    scores = bf16(scores * expert_scale[inds]).

    Selection order: descending logit, ties to the lower expert index.
    softmax is monotone in the logit, so this is a top-k of `probs` (the
    reference's argpartition leaves the order inside the top-k, and the
    choice among exactly tied probabilities, unspecified). Returns
    (inds [T,k] int32, scores [T,k] float32 bf16 values, logits [T,E])."""
    logits = linear(x, gate_w)                      # [T, E] bf16 values
    T, E = logits.shape
    # stable sort on -logit keeps lower indices first among equal logits
    order = np.argsort(-logits, axis=-1, kind="stable")[:, :k]
    l32 = logits.astype(np.float32)
    m = l32.max(axis=-1, keepdims=True)
    e = np.exp(l32 - m).astype(np.float32)
    z = np.zeros((T, 1), np.float32)
    for j in range(E):                              # sequential fp32 sum
        z[:, 0] += e[:, j]
    p = (e / z).astype(np.float32)
    psel = np.take_along_axis(p, order, axis=-1)
    if mode == ROUTER_SOFTMAX_TOPK:
        scores = bf16(psel)
    else:
        vsel = np.take_along_axis(e, order, axis=-1) if mode == ROUTER_TOPK_SOFTMAX else psel
        den = np.zeros((T, 1), np.float32)
        for j in range(k):
            den[:, 0] += vsel[:, j]
        scores = bf16((vsel / den).astype(np.float32))
    if expert_scale is not None:
        scores = bf16(scores.astype(np.float32) * np.asarray(expert_scale, np.float32)[order])
    return order.astype(np.int32), scores, logits


def switch_linear(x_rows: np.ndarray, experts: np.ndarray, w: np.ndarray,
                  vq: bool) -> np.ndarray:
    """One expert matmul per row: y[r] = bf16(x_rows[r] @ w[experts[r]].T)
    (`switch_layers.py:116-125`, the gather_mm / VQ gather_qmm equivalent).
    VQ experts take the activations in fp16 (`f16_sat`); dense bf16 experts
    take them as they are."""
    xin = f16_sat(x_rows) if vq else x_rows
    out = np.empty((x_rows.shape[0], w.shape[1]), np.float32)
    for e in np.unique(experts):
        sel = np.nonzero(experts == e)[0]
        out[sel] = linear(xin[sel], w[e])
    return out


def swiglu(up: np.ndarray, gate: np.ndarray) -> np.ndarray:
    """`_SwiGLU` (`qwen3_5.py:108-112`): bf16(bf16(silu_f32(gate)) * up)."""
    return bf16(bf16(_silu_f32(gate)).astype(np.float64) * up)


def geglu(up: np.ndarray, gate: np.ndarray) -> np.ndarray:
    """`geglu` (`gemma4_text.py:131-135`): bf16(bf16(gelu_tanh_f32(gate)) * up)."""
    return bf16(bf16(_gelu_tanh_f32(gate)).astype(np.float64) * up)


ACT_SWIGLU, ACT_GEGLU = 0, 1


def switch_glu(x: np.ndarray, inds: np.ndarray, gate_w, up_w, down_w,
               vq: bool, act: int = ACT_SWIGLU) -> np.ndarray:
    """`SwitchGLU.__call__` (`switch_layers.py:172-193`): [T, k, H] bf16.
    The sort by expert it does for >= 64 pairs does not change any value."""
    T, k = inds.shape
    rows = np.repeat(x, k, axis=0)                  # pair p = t*k + s
    ex = inds.reshape(-1)
    u = switch_linear(rows, ex, up_w, vq)
    g = switch_linear(rows, ex, gate_w, vq)
    a = geglu(u, g) if act == ACT_GEGLU else swiglu(u, g)
    y = switch_linear(a, ex, down_w, vq)
    return y.reshape(T, k, -1)


def combine(y: np.ndarray, scores: np.ndarray) -> np.ndarray:
    """`(y * scores[..., None]).sum(axis=-2)` (`qwen3_5.py:181-182`): each
    product rounded to bf16, the k-sum in float32 rounded once."""
    prod = bf16(y.astype(np.float64) * scores[..., None])
    acc = np.zeros(prod.shape[:1] + prod.shape[2:], np.float32)
    for j in range(prod.shape[1]):
        acc += prod[:, j]
    return bf16(acc)


def moe_experts(x: np.ndarray, inds: np.ndarray, scores: np.ndarray, gate_w, up_w, down_w,
                vq: bool, act: int = ACT_GEGLU) -> np.ndarray:
    """Gemma-4's `Experts.__call__` (`gemma4_text.py:196-214`):
    `(w * switch_glu(x, inds)).sum(-2)` with `combine`'s roundings."""
    return combine(switch_glu(x, inds, gate_w, up_w, down_w, vq, act), scores)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """`mx.fast.rms_norm(x, w, eps)` as restated for the Gemma-4 router
    input (`gemma4_text.py:171`): the mean of the squares summed exactly
    (float64 over bf16 squares, each exact) and rounded once to float32,
    r = 1 / sqrt(ms + eps) in float32, the normalised value rounded to bf16,
    then times the bf16 weight, rounded again. The reference's MLX kernel is
    not available here: this order of roundings is this build's reading of
    it (unpinned)."""
    xf = np.asarray(x, np.float32)
    xd = xf.astype(np.float64)
    ms = ((xd * xd).sum(axis=-1, keepdims=True) / xf.shape[-1]).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return bf16(bf16(xf * inv).astype(np.float32) * np.asarray(w, np.float32))


def shared_expert(x, sg_w, sup_w, sgate_w, sdown_w):
    """`qwen3_5.py:184-186`: bf16(bf16(sigmoid(x @ w_sg^T)) * down(
    bf16(silu(gate(x))) * up(x)))."""
    g = linear(x, sgate_w)
    u = linear(x, sup_w)
    a = bf16(bf16(_silu_f32(g)).astype(np.float64) * u)
    sh = linear(a, sdown_w)
    gl = linear(x, sg_w)                            # [T, 1]
    return bf16(bf16(_sigmoid_f32(gl)).astype(np.float64) * sh)


def sparse_moe_block(x: np.ndarray, p: dict, k: int, vq: bool,
                     return_parts: bool = False, router_mode: int = ROUTER_SOFTMAX_TOPK_RENORM,
                     act: int = ACT_SWIGLU):
    """`SparseMoeBlock.__call__` (`qwen3_5.py:170-192`) on [T, H] bf16 input.

    `p` holds float32 arrays of bf16 (router, shared expert) and, for the
    experts, either dense bf16 `gate`, `up`, `down` [E, OUT, IN] or, with
    vq=True, already dequantised fp16 weights under the same names."""
    inds, scores, logits = router(x, p["router"], k, router_mode)
    y = switch_glu(x, inds, p["gate"], p["up"], p["down"], vq, act)
    routed = combine(y, scores)
    out = routed
    if "shared_gate" in p:
        sh = shared_expert(x, p["shared_expert_gate"], p["shared_up"],
                           p["shared_gate"], p["shared_down"])
        out = bf16(routed.astype(np.float64) + sh)
    if return_parts:
        return out, dict(inds=inds, scores=scores, logits=logits, y=y,
                         routed=routed)
    return out


# ----------------------------------------------------------- tensor split

def shard_block_params(p: dict, rank: int, n: int) -> dict:
    """The reference's cut of one MoE block (`src/knurlogic/engine/split/
    tensor_rules.py:57-101`): gate/up and the shared gate/up split on the
    output axis, down and the shared down on the input axis; the router and
    `shared_expert_gate` replicated (dequantised weights are cut the same
    way the codes and vq_scales are, and the codebook is never cut)."""
    def a2s(w):
        if isinstance(w, LazyAffine):
            o = w.shape[1] // n
            cut = slice(rank * o, (rank + 1) * o)
            return LazyAffine(w.weight[:, cut], w.scales[:, cut], w.biases[:, cut], w.group_size, w.bits)
        if isinstance(w, LazyVQ):
            o = w.shape[1] // n
            return LazyVQ(w.codes[:, rank * o:(rank + 1) * o], w.codebook,
                          w.scales[:, rank * o:(rank + 1) * o], w.group_size)
        o = w.shape[-2] // n
        return w[..., rank * o:(rank + 1) * o, :]

    def s2a(w):
        if isinstance(w, LazyAffine):
            c, g = w.weight.shape[-1] // n, w.scales.shape[-1] // n
            return LazyAffine(w.weight[..., rank * c:(rank + 1) * c], w.scales[..., rank * g:(rank + 1) * g],
                              w.biases[..., rank * g:(rank + 1) * g], w.group_size, w.bits)
        if isinstance(w, LazyVQ):
            c = w.codes.shape[-1] // n
            g = w.scales.shape[-1] // n
            return LazyVQ(w.codes[..., rank * c:(rank + 1) * c], w.codebook,
                          w.scales[..., rank * g:(rank + 1) * g], w.group_size)
        i = w.shape[-1] // n
        return w[..., rank * i:(rank + 1) * i]
    q = dict(p)
    q["gate"], q["up"], q["down"] = a2s(p["gate"]), a2s(p["up"]), s2a(p["down"])
    if "shared_gate" in p:
        q["shared_gate"] = a2s(p["shared_gate"])
        q["shared_up"] = a2s(p["shared_up"])
        q["shared_down"] = s2a(p["shared_down"])
    return q


def tp_sparse_moe_block(x, p, k, vq, n):
    """The tensor-split block (`src/knurlogic/engine/split/tensor.py:
    159-187`): every rank runs the whole block on its cut, its output
    rounded to bf16; the partials are summed in float32 and rounded once."""
    acc = np.zeros((x.shape[0], p["router"].shape[1]), np.float64)
    for r in range(n):
        acc += sparse_moe_block(x, shard_block_params(p, r, n), k, vq)
    return bf16(acc.astype(np.float32))


# ----------------------------------------------------------- affine experts

def unpack_affine(weight: np.ndarray, bits: int) -> np.ndarray:
    """The `bits`-bit values of mlx's affine packing (`mx.quantize`, read by
    `mx.gather_qmm` in `switch_layers.py:71-86`): each row of uint32 words
    is a little-endian bit stream, element j at bits [j*bits, (j+1)*bits).
    Returns [..., IN] int64."""
    w = np.ascontiguousarray(np.asarray(weight).astype(np.uint32))
    raw = np.unpackbits(w.view(np.uint8), axis=-1, bitorder="little")      # [..., W*32]
    IN = raw.shape[-1] // bits
    b = raw[..., :IN * bits].reshape(*raw.shape[:-1], IN, bits).astype(np.int64)
    return (b << np.arange(bits, dtype=np.int64)).sum(axis=-1)


def dequant_affine(weight: np.ndarray, scales: np.ndarray, biases: np.ndarray, group_size: int,
                   bits: int) -> np.ndarray:
    """Dense weights of affine-quantized experts, [E, OUT, IN] float32 holding
    bf16 values: W = bf16(f32(scale * q + bias)), the product and sum exact
    (float64 over a bf16 scale, a small integer and a bf16 bias), rounded once
    to float32 -- what a fused multiply-add gives -- then to bf16. The scale
    and bias are the group's (`mx.quantize`'s affine layout). This rounding is
    the build's definition: MLX's kernels cannot run here (unpinned)."""
    q = unpack_affine(weight, bits).astype(np.float64)
    s = np.repeat(np.asarray(scales, np.float64), group_size, axis=-1)
    b = np.repeat(np.asarray(biases, np.float64), group_size, axis=-1)
    return bf16((q * s + b).astype(np.float32))


class LazyAffine:
    """Dequantised affine experts one expert at a time (`w[e]`)."""

    def __init__(self, weight, scales, biases, group_size: int, bits: int):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits
        E, OUT, W = weight.shape
        self.shape = (E, OUT, W * 32 // bits)

    def __getitem__(self, e: int) -> np.ndarray:
        return dequant_affine(self.weight[e:e + 1], self.scales[e:e + 1], self.biases[e:e + 1],
                              self.group_size, self.bits)[0]
