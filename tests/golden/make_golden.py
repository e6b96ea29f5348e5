"""Writes `qwen3_5_moe_bf16_mlp.npz`: the reference's bf16 MoE-block golden
with the exact weights and input it was computed on.

Run in a container where the reference is mounted, naming its checkout:

    python tests/golden/make_golden.py --reference <reference checkout>

Sources (reference paths):
* golden output: `tests/support/goldens/qwen_reference.npz`
  ["qwen3_5_moe/bf16/0.mlp"], shape (1, 21, 32) -- HF transformers 5.16.1's
  bf16 Qwen3.5-MoE sparse block on CPU, which
  `tests/engine/test_qwen_reference.py:213-241` requires knurlogic's MLX
  block to equal bit for bit;
* weights: `build_qwen_reference.component_weights` (seeded numpy by
  parameter name, rounded to bf16) over the stored shapes
  `meta["qwen3_5_moe/shapes"]`, layer 0's mlp;
* input: `build_qwen_reference.component_input(32)`.

The fixture stores the arrays themselves (a few KB), so the tests need
neither the reference nor its numpy seeding recipe.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "qwen3_5_moe_bf16_mlp.npz"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="the reference checkout (its tests/support/goldens is read)")
    args = ap.parse_args(argv)
    gdir = Path(args.reference) / "tests" / "support" / "goldens"
    sys.path.insert(0, str(gdir))
    import build_qwen_reference as G            # numpy-only at module level

    z = np.load(gdir / "qwen_reference.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    shapes = {k: tuple(v) for k, v in meta["qwen3_5_moe/shapes"].items()}
    w = G.component_weights(shapes)
    cfg = meta["qwen3_5_moe/config"]
    pre = "model.layers.0.mlp."
    gate_up = w[pre + "experts.gate_up_proj"]           # [E, 2I, H]
    mid = gate_up.shape[-2] // 2
    arrays = {
        "x": G.component_input(cfg["hidden_size"])[0],  # [21, 32]
        "router": w[pre + "gate.weight"],               # [E, H]
        # qwen3_5_moe.py:36-50: gate = gate_up[:, :I], up = gate_up[:, I:]
        "gate": gate_up[:, :mid, :],
        "up": gate_up[:, mid:, :],
        "down": w[pre + "experts.down_proj"],           # [E, H, I]
        "shared_gate": w[pre + "shared_expert.gate_proj.weight"],
        "shared_up": w[pre + "shared_expert.up_proj.weight"],
        "shared_down": w[pre + "shared_expert.down_proj.weight"],
        "shared_expert_gate": w[pre + "shared_expert_gate.weight"],
        "golden": z["qwen3_5_moe/bf16/0.mlp"][0],       # [21, 32]
        "top_k": np.int32(cfg["num_experts_per_tok"]),
    }
    arrays = {k: (np.ascontiguousarray(v) if np.ndim(v) else np.asarray(v))
              for k, v in arrays.items()}
    info = {"source": "tests/support/goldens/qwen_reference.npz",
            "key": "qwen3_5_moe/bf16/0.mlp", "build": meta["build"],
            "config": {k: cfg[k] for k in (
                "hidden_size", "num_experts", "num_experts_per_tok",
                "moe_intermediate_size", "shared_expert_intermediate_size")}}
    arrays["info"] = np.frombuffer(json.dumps(info).encode(), np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
