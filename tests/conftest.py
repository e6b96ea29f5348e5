"""Shared test fixtures.

`-m "not gpu"` runs here without a GPU: the oracle against the reference's
golden, the host-side logic, and that libvqmoe.so loads and exports what
include/vqmoe.h declares. `-m gpu` runs the parity tests proper on a B200,
through the C ABI, against the oracle.
"""
import json
import os
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


def oracle_params(w: dict, prefix: str = "mlp.", group_size: int = 64) -> dict:
    """Oracle parameters (numpy; VQ and affine experts as lazily dequantised
    views) from a state dict with the reference's names; `group_size` is the
    affine experts' group (their packed width gives the bits)."""
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
        elif q + "biases" in w:
            wt, sc = to_np(w[q + "weight"]), to_np(w[q + "scales"])
            bits = wt.shape[-1] * 32 // (sc.shape[-1] * group_size)
            p[key] = R.LazyAffine(wt, sc, to_np(w[q + "biases"]), group_size, bits)
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


# ------------------------------------------------------------ tolerances
#
# Layer outputs (bf16) against the oracle, two bars:
# * max |gpu - oracle| <= REL * max |oracle| -- the north star's 1e-2
#   relative, on every element;
# * per element |gpu - oracle| <= ULPS bf16 steps of |oracle| + FLOOR *
#   rms(oracle), on all but FRAC of the elements. The GPU accumulates in
#   float32 (tensor cores), the oracle exactly, and the decode kernels apply
#   each 64-input group's scale to the partial sum (s * (codebook . x)) where
#   the oracle dequantises fp16(codebook * s): an expert output or SwiGLU
#   activation now and then rounds to the neighbouring bf16 value. Through
#   the top-k sum such a step is a step of the summands' magnitude, which
#   cancellation can make several steps of a small output element -- the
#   rms floor covers that.
REL = 1e-2
ULPS = 2
FLOOR = 2.0 ** -9
FRAC = 0.005


def bf16_ulp(a):
    """The bf16 step at |a| (2^(e-7) for |a| in [2^e, 2^(e+1)); the
    smallest normal's step below it)."""
    a = np.abs(np.asarray(a, np.float64))
    _, e = np.frexp(np.maximum(a, 2.0 ** -126))
    return np.ldexp(1.0, e - 8)


def bf16_error_stats(got, ref) -> dict:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    u = d / bf16_ulp(ref)
    rms = float(np.sqrt(np.mean(np.square(ref)))) or 1.0
    return {"n": int(ref.size), "equal": float((d == 0).mean()),
            "beyond_1ulp": float((u > 1).mean()), "beyond_2ulp": float((u > 2).mean()),
            "beyond_bar": float((d > ULPS * bf16_ulp(ref) + FLOOR * rms).mean()),
            "max_ulp": float(u.max()), "max_rel_rms": float(d.max() / rms),
            "max_rel": float(d.max() / (np.abs(ref).max() or 1.0))}


def assert_bf16_close(got, ref, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    st = bf16_error_stats(got, ref)
    log = os.environ.get("VQMOE_TOLERANCE_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps({"what": what, **st}) + "\n")
    assert st["max_rel"] <= REL, f"{what}: max diff {st['max_rel']:.3e} of max |ref| > {REL}"
    assert st["beyond_bar"] <= FRAC, (f"{what}: {st['beyond_bar']:.3%} of elements off by more than "
                                      f"{ULPS} bf16 steps + 2^-9 rms ({st})")
