"""Tensor split of the MoE block across the GPUs of one node.

The reference's rules for this block (`src/knurlogic/engine/split/
tensor_rules.py:57-101, 123-139`):
  mlp.switch_mlp.{gate,up}_proj     all-to-sharded: cut the output axis
  mlp.switch_mlp.down_proj          sharded-to-all: cut the input axis
  mlp.shared_expert.{gate,up}_proj  all-to-sharded
  mlp.shared_expert.down_proj       sharded-to-all
  mlp.gate, mlp.shared_expert_gate  replicated
  any `codebook`                    replicated, never cut
and the block's output is summed across ranks in float32, then rounded once
(`Reduce`, `src/knurlogic/engine/split/tensor.py:159-187`).

A cut that does not divide is refused before anything loads, one line per
array, as `tensor_rules.refusals` does (`tensor_rules.py:256-311`); on top
of the reference's divisibility, the B200 kernels need every VQ shard's
input width to be a multiple of 64 and every output width a multiple of 16.
"""
from __future__ import annotations


import torch

A2S, S2A, WHOLE = "all-to-sharded", "sharded-to-all", "whole"

RULES = {
    "switch_mlp.gate_proj": A2S,
    "switch_mlp.up_proj": A2S,
    "switch_mlp.down_proj": S2A,
    "shared_expert.gate_proj": A2S,
    "shared_expert.up_proj": A2S,
    "shared_expert.down_proj": S2A,
}


def _rule(name: str, prefix: str):
    if not name.startswith(prefix):
        return None, None
    rest = name[len(prefix):]
    for mod, kind in RULES.items():
        if rest.startswith(mod + "."):
            return kind, rest[len(mod) + 1:]
    return None, None


def split_axis(kind: str, leaf: str, ndim: int):
    """The reference's predicate (`tensor_rules.predicate`): codebooks are
    never cut; all-to-sharded cuts axis ndim-2, sharded-to-all the last."""
    if leaf.endswith("codebook"):
        return None
    if kind == A2S:
        return max(ndim - 2, 0)
    if kind == S2A:
        return ndim - 1
    return None


def refusals(shapes: dict, n: int, prefix: str = "mlp.") -> list:
    """{name: shape} -> why the block cannot be cut n ways ([] if it can)."""
    out = []
    for name in sorted(shapes):
        kind, leaf = _rule(name, prefix)
        if kind is None:
            continue
        shape = tuple(shapes[name])
        ax = split_axis(kind, leaf, len(shape))
        if ax is None:
            continue
        if shape[ax] % n:
            unit = f"on axis {ax}"
            out.append(f"{name}: {shape[ax]} {unit} do not divide by {n}")
            continue
        part = shape[ax] // n
        # the codebook's dim turns a rank's codes into inputs (4 unless named)
        dim = tuple(shapes.get(name[:-len("codes")] + "codebook", (0, 4)))[-1] if leaf == "codes" else 4
        if leaf == "codes" and kind == S2A and (part * dim) % 64:
            out.append(f"{name}: a rank's {part * dim} inputs are not a multiple "
                       f"of 64 (whole scale groups and 256-input code chunks)")
        if leaf in ("codes", "vq_scales", "weight") and kind == A2S and part % 16:
            out.append(f"{name}: a rank's {part} output rows are not a multiple of 16")
        affine = leaf == "weight" and (name[:-len("weight")] + "biases") in shapes
        if leaf == "weight" and kind == S2A and part % 16 and not affine:
            out.append(f"{name}: a rank's {part} inputs are not a multiple of 16")
    return out


def shard_state_dict(w: dict, rank: int, n: int, prefix: str = "mlp.") -> dict:
    """This rank's cut of the block's tensors (codebooks and the routers
    whole). Raises ValueError with every refusal when it cannot cut."""
    why = refusals({k: tuple(v.shape) for k, v in w.items()}, n, prefix)
    if why:
        raise ValueError("cannot split the MoE block %d ways: %s" % (n, "; ".join(why)))
    out = {}
    for name, t in w.items():
        kind, leaf = _rule(name, prefix)
        ax = split_axis(kind, leaf, t.dim()) if kind else None
        if ax is None:
            out[name] = t
            continue
        size = t.shape[ax] // n
        out[name] = t.narrow(ax, rank * size, size).contiguous()
    return out


def build_block(w: dict, top_k: int, rank: int = 0, n: int = 1, group=None,
                prefix: str = "mlp.", tp_reduce: str = "p2p"):
    """A SparseMoeBlock holding rank `rank`'s cut; `group` is the process
    group its partials are reduced over (None when n == 1), by the
    peer-memory kernel (`tp_reduce="p2p"`) or NCCL ("nccl")."""
    from .moe import SparseMoeBlock
    ws = shard_state_dict(w, rank, n, prefix) if n > 1 else w
    return SparseMoeBlock.from_weights(ws, top_k, prefix=prefix,
                                       sharding_group=group if n > 1 else None, tp_reduce=tp_reduce)
