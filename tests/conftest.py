"""Shared test fixtures.

`-m "not gpu"` runs here without a GPU: the oracle against the reference's
golden, the host-side logic, and that libvqmoe.so loads and exports what
include/vqmoe.h declares. `-m gpu` runs the parity tests proper on a B200,
through the C ABI, against the oracle.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def to_np(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.detach().cpu().numpy()


def oracle_params(w: dict, prefix: str = "mlp.") -> dict:
    """Oracle parameters (numpy; VQ experts as lazily dequantised views)
    from a state dict with the reference's names."""
    from oracle import moe_ref as R
    p = {"router": to_np(w[prefix + "gate.weight"])}
    for n, key in (("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
        q = f"{prefix}switch_mlp.{n}."
        if q + "codes" in w:
            codes = to_np(w[q + "codes"])
            cb = to_np(w[q + "codebook"])
            vs = to_np(w[q + "vq_scales"])
            gs = codes.shape[-1] * cb.shape[-1] // vs.shape[-1]
            p[key] = R.LazyVQ(codes, cb, vs, gs)
        else:
            p[key] = to_np(w[q + "weight"])
    if prefix + "shared_expert.gate_proj.weight" in w:
        p["shared_gate"] = to_np(w[prefix + "shared_expert.gate_proj.weight"])
        p["shared_up"] = to_np(w[prefix + "shared_expert.up_proj.weight"])
        p["shared_down"] = to_np(w[prefix + "shared_expert.down_proj.weight"])
        p["shared_expert_gate"] = to_np(w[prefix + "shared_expert_gate.weight"])
    return p


@pytest.fixture(scope="session")
def golden():
    z = np.load(ROOT / "tests" / "golden" / "qwen3_5_moe_bf16_mlp.npz")
    return {k: z[k] for k in z.files}


def golden_state_dict(g: dict) -> dict:
    """The golden's weights under Knurlogic's post-sanitize names (bf16)."""
    import torch

    def bf(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16)
    return {
        "mlp.gate.weight": bf(g["router"]),
        "mlp.switch_mlp.gate_proj.weight": bf(g["gate"]),
        "mlp.switch_mlp.up_proj.weight": bf(g["up"]),
        "mlp.switch_mlp.down_proj.weight": bf(g["down"]),
        "mlp.shared_expert.gate_proj.weight": bf(g["shared_gate"]),
        "mlp.shared_expert.up_proj.weight": bf(g["shared_up"]),
        "mlp.shared_expert.down_proj.weight": bf(g["shared_down"]),
        "mlp.shared_expert_gate.weight": bf(g["shared_expert_gate"]),
    }
