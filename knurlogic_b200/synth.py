"""Seeded synthetic layers and inputs for the benchmark configurations.

No dataset or checkpoint is involved: every tensor is drawn from a seeded
torch generator with the shapes and distributions the configurations name.

c1  8 experts, top-2, H 1024, I 512, 16 tokens, no shared expert; router
    N(0, 0.02); codebooks N(0, 0.02)
c2  128 experts, top-8, H 2048, I 768 + shared expert 768, 64 tokens
    (16 sequences x (1 + 3 MTP drafts)); router uniform U(-1/sqrt(H),
    1/sqrt(H)) (mlx-lm's SwitchLinear init range)
c3  c2's layer at 4096 prefill tokens, router logits biased so expert
    popularity follows Zipf s=1.1 over a seeded expert permutation: input
    feature 0 is held at 1.0 and router column 0 carries b_e = log p_e
c4  256 experts, top-8, H 4096, I 1536, 256 tokens (the tensor-split
    configuration's MoE layer), router N(0, 0.02)

Every VQ matrix: codes U[0, K) (uint8 for K <= 256, else uint16), its own
K x dim fp16 codebook N(0, 0.02) (K 256, dim 4 unless the configuration
names others: the reference's VQ fixture is K 2048, dim 2, group 64),
vq_scales [E, OUT, IN/group] fp16 -- 1.0 ("ones", the 2-bit headline; the
kernel still reads them) or 0.5 + U(0, 1) ("random", the numerics tests).
Activations N(0, 1) rounded to bf16. Shared expert and its gate bf16
N(0, 0.02).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class MoEConfig:
    name: str
    experts: int
    top_k: int
    hidden: int
    inter: int
    shared_inter: int
    tokens: int
    router: str = "normal"      # normal | uniform
    zipf: float = 0.0
    dim: int = 4
    codebook_size: int = 256
    group: int = 64
    quant: str = "vq"           # vq | affine (mlx's weight / scales / biases)
    bits: int = 4               # affine bits per weight

    def with_tokens(self, t: int) -> "MoEConfig":
        return replace(self, tokens=t)


CONFIGS = {
    "c1": MoEConfig("c1", 8, 2, 1024, 512, 0, 16),
    "c2": MoEConfig("c2", 128, 8, 2048, 768, 768, 64, router="uniform"),
    "c3": MoEConfig("c3", 128, 8, 2048, 768, 768, 4096, router="uniform", zipf=1.1),
    "c4": MoEConfig("c4", 256, 8, 4096, 1536, 0, 256),
}


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _normal(shape, std, g, device, dtype):
    return (torch.randn(shape, generator=g, device=device) * std).to(dtype)


def zipf_bias(cfg: MoEConfig, seed: int) -> torch.Tensor:
    """b_e = log p_e with p over a seeded permutation of experts, p_rank ~
    rank^-s (float32, CPU)."""
    g = _gen(seed + 7, "cpu")
    perm = torch.randperm(cfg.experts, generator=g)
    ranks = torch.empty(cfg.experts, dtype=torch.float64)
    ranks[perm] = torch.arange(1, cfg.experts + 1, dtype=torch.float64)
    p = ranks ** (-cfg.zipf)
    p = p / p.sum()
    return torch.log(p).to(torch.float32)


def pack_affine(q: torch.Tensor, bits: int) -> torch.Tensor:
    """`bits`-bit values [..., IN] -> mlx's affine packing: each row a
    little-endian bit stream in uint32 words (element j at bits
    [j*bits, (j+1)*bits)), returned as int32 words (the same bits)."""
    import numpy as np
    qn = q.to(torch.int64).cpu().numpy()
    stream = ((qn[..., :, None] >> np.arange(bits)) & 1).astype(np.uint8)
    stream = stream.reshape(*qn.shape[:-1], qn.shape[-1] * bits)
    words = np.packbits(stream, axis=-1, bitorder="little").view(np.int32)
    return torch.from_numpy(np.ascontiguousarray(words)).to(q.device)


def _affine_matrix(E, out, inp, cfg: MoEConfig, g: torch.Generator, device) -> dict:
    """q uniform over [0, 2^bits); per group a bf16 scale 0.04 (0.5 + U(0,1))
    / (2^bits - 1) and a bf16 bias that centres the range (weights about
    N(0, 0.02)-sized)."""
    levels = (1 << cfg.bits) - 1
    q = torch.randint(0, levels + 1, (E, out, inp), generator=g, device=device)
    ng = inp // cfg.group
    s = (0.5 + torch.rand((E, out, ng), generator=g, device=device)) * (0.04 / levels)
    b = -s * (levels / 2) + torch.randn((E, out, ng), generator=g, device=device) * 0.002
    return {"weight": pack_affine(q, cfg.bits), "scales": s.to(torch.bfloat16), "biases": b.to(torch.bfloat16)}


def make_weights(cfg: MoEConfig, seed: int = 0, device="cpu",
                 scales: str = "ones", prefix: str = "mlp.") -> dict:
    """State dict with the reference's names (reference layout for codes)."""
    g = _gen(seed, device)
    E, H, I = cfg.experts, cfg.hidden, cfg.inter
    w = {}
    if cfg.router == "uniform":
        a = 1.0 / math.sqrt(H)
        r = (torch.rand((E, H), generator=g, device=device) * 2 - 1) * a
    else:
        r = torch.randn((E, H), generator=g, device=device) * 0.02
    if cfg.zipf:
        r[:, 0] = zipf_bias(cfg, seed).to(device)
    w[prefix + "gate.weight"] = r.to(torch.bfloat16)
    for name, out, inp in (("gate_proj", I, H), ("up_proj", I, H), ("down_proj", H, I)):
        q = f"{prefix}switch_mlp.{name}."
        if cfg.quant == "affine":
            for leaf, t in _affine_matrix(E, out, inp, cfg, g, device).items():
                w[q + leaf] = t
            continue
        if cfg.codebook_size <= 256:
            w[q + "codes"] = torch.randint(0, cfg.codebook_size, (E, out, inp // cfg.dim),
                                           generator=g, device=device, dtype=torch.uint8)
        else:
            w[q + "codes"] = torch.randint(0, cfg.codebook_size, (E, out, inp // cfg.dim), generator=g,
                                           device=device, dtype=torch.int32).to(torch.uint16)
        w[q + "codebook"] = _normal((cfg.codebook_size, cfg.dim), 0.02, g, device,
                                    torch.float16)
        ng = inp // cfg.group
        if scales == "ones":
            s = torch.ones((E, out, ng), device=device)
        else:
            s = 0.5 + torch.rand((E, out, ng), generator=g, device=device)
        w[q + "vq_scales"] = s.to(torch.float16)
    if cfg.shared_inter:
        Is = cfg.shared_inter
        w[prefix + "shared_expert.gate_proj.weight"] = _normal((Is, H), 0.02, g, device, torch.bfloat16)
        w[prefix + "shared_expert.up_proj.weight"] = _normal((Is, H), 0.02, g, device, torch.bfloat16)
        w[prefix + "shared_expert.down_proj.weight"] = _normal((H, Is), 0.02, g, device, torch.bfloat16)
        w[prefix + "shared_expert_gate.weight"] = _normal((1, H), 0.02, g, device, torch.bfloat16)
    return w


def make_input(cfg: MoEConfig, seed: int = 0, device="cpu",
               tokens: int | None = None) -> torch.Tensor:
    T = cfg.tokens if tokens is None else tokens
    g = _gen(seed + 1000003, device)
    x = torch.randn((T, cfg.hidden), generator=g, device=device)
    if cfg.zipf:
        x[:, 0] = 1.0
    return x.to(torch.bfloat16)


def algorithmic_bytes(cfg: MoEConfig, distinct_experts: int, tokens: int | None = None,
                      with_scales: bool = True) -> int:
    """HBM bytes one block call must move at least: the codes (and scales)
    of every expert the routing touched, the codebooks, the shared expert,
    the router weight, the activations in and out."""
    T = cfg.tokens if tokens is None else tokens
    H, I = cfg.hidden, cfg.inter
    code_bytes = 1 if cfg.codebook_size <= 256 else 2
    per = 3 * H * I // cfg.dim * code_bytes
    if with_scales:
        per += 3 * 2 * H * I // cfg.group
    b = distinct_experts * per + 3 * cfg.codebook_size * cfg.dim * 2
    if cfg.shared_inter:
        b += 3 * 2 * cfg.shared_inter * H + 2 * H
    b += 2 * cfg.experts * H + 2 * 2 * T * H
    return int(b)


def algorithmic_flops(cfg: MoEConfig, tokens: int | None = None) -> int:
    T = cfg.tokens if tokens is None else tokens
    H, I = cfg.hidden, cfg.inter
    f = 2 * T * cfg.top_k * 3 * I * H + 2 * T * cfg.experts * H
    if cfg.shared_inter:
        f += 2 * T * 3 * cfg.shared_inter * H + 2 * T * H
    return int(f)
