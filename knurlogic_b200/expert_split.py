"""Expert parallelism: the MoE block's experts placed by id across the ranks
of a split, an alternative to the tensor split at large E (SURVEY's §8(f)
rank 4 second half; the reference has no EP, so nothing here restates its
code).

Rank r of n holds experts [r*E/n, (r+1)*E/n) whole: their codes and scales
cut on the expert axis; the codebooks, the router and the shared expert are
kept whole on every rank. Every rank routes every token and runs the pairs
of its own experts; one kernel then sums each token's k slots in slot order
over NVLink peer memory, reading each slot from its expert's owner, and adds
the gated shared expert -- the unsplit block's combine (qwen3_5.py:181-187)
bit for bit (`vqmoe_sparse_moe_block_ep`). Against the tensor split, every
expert tile keeps its full width (the tensor split's down projection at
N = 4 or 8 streams only 384 or 192 inputs a tile), the router is not cut,
and the exchange moves each token's k expert outputs of its column slice
instead of one partial.
"""
from __future__ import annotations

from .moe import SparseMoeBlock

_EXPERT_LEAVES = ("codes", "vq_scales")


def refusals(shapes: dict, n: int, prefix: str = "mlp.") -> list[str]:
    """Why an n-way expert split of a block (tensor shapes by name) cannot
    run; empty when it can."""
    out = []
    codes = shapes.get(prefix + "switch_mlp.gate_proj.codes")
    if codes is None:
        return [f"expert split: VQ experts only ({prefix}switch_mlp.*.codes missing)"]
    E = codes[0]
    if E % n:
        out.append(f"expert split: {E} experts do not divide over {n} ranks")
    H = shapes[prefix + "gate.weight"][1]
    if H % (8 * n):
        out.append(f"expert split: hidden {H} is not a multiple of 8 x {n}")
    cb = shapes.get(prefix + "switch_mlp.gate_proj.codebook")
    if cb is not None and (cb[0] > 256 or cb[1] != 4):
        out.append("expert split: the uint8 dim-4 VQ layout only")
    return out


def shard_state_dict(w: dict, rank: int, n: int, prefix: str = "mlp.") -> dict:
    """Rank `rank`'s share of a block's state dict: each expert linear's
    codes and scales cut to experts [rank*E/n, (rank+1)*E/n); everything
    else (router, codebooks, shared expert) kept whole."""
    E = w[prefix + "switch_mlp.gate_proj.codes"].shape[0]
    if E % n:
        raise ValueError(f"expert split: {E} experts over {n} ranks")
    e0, e1 = rank * E // n, (rank + 1) * E // n
    out = {}
    for k, v in w.items():
        if k.startswith(prefix + "switch_mlp.") and k.rsplit(".", 1)[-1] in _EXPERT_LEAVES:
            out[k] = v[e0:e1].contiguous()
        else:
            out[k] = v
    return out


def build_block(w: dict, top_k: int, rank: int, n: int, group, prefix: str = "mlp.") -> SparseMoeBlock:
    """This rank's block of an n-way expert split over process group
    `group` (one process per GPU); its forward returns the whole block's
    output on every rank."""
    shapes = {k: tuple(v.shape) for k, v in w.items()}
    why = refusals(shapes, n, prefix)
    if why:
        raise ValueError("; ".join(why))
    return SparseMoeBlock.from_weights(shard_state_dict(w, rank, n, prefix), top_k, prefix=prefix,
                                       sharding_group=group, expert_split=True)
