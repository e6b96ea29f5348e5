"""Gemma-4's MoE router and experts over libvqmoe, with the reference's
module interface.

Reference: `Router`, `GeGLU` and `Experts` of
`src/knurlogic/engine/families/gemma4/architecture/gemma4_text.py:131-214`:

* `Router(x)`: `rms_norm(x, scale * hidden**-0.5, eps)`, the projection
  `proj` (Linear H -> E, no bias), the top-k by logit, a softmax over the k
  selected logits, times `per_expert_scale[index]`; returns
  `(top_k_indices, top_k_weights)`.
* `Experts(x, top_k_indices, top_k_weights)`: `SwitchGLU` with the GeGLU
  activation, each expert output times its weight, summed over the k slots.

The router's RMS norm runs in `vqmoe_rms_norm`, the projection, top-k,
softmax and per-expert scale in `vqmoe_router_ex` (exact bf16 logits; the
softmax in float32), the experts and the weighted sum in
`vqmoe_moe_experts`. The norm's order of roundings (an exact mean of the
squares rounded once to float32) is this build's reading of MLX's fused
kernel, which cannot run here: unpinned.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _lib
from .switch_layers import GeGLU, SwitchGLU, _contig, c_stream, ctypes_ref, require_cuda


class Router(nn.Module):
    """`gemma4_text.py:156-182`. `proj_weight [E, H]`, `scale [H]` and
    `per_expert_scale [E]` as the checkpoint holds them."""

    def __init__(self, proj_weight: torch.Tensor, scale: torch.Tensor, per_expert_scale: torch.Tensor,
                 top_k_experts: int, eps: float = 1e-6):
        super().__init__()
        E, H = proj_weight.shape
        if scale.shape != (H,) or per_expert_scale.shape != (E,):
            raise ValueError(f"scale {tuple(scale.shape)} / per_expert_scale {tuple(per_expert_scale.shape)} "
                             f"for a [{E}, {H}] projection")
        if not 0 < top_k_experts <= min(E, 32):
            raise ValueError(f"top_k_experts {top_k_experts} (1 .. min(E, 32))")
        self.proj = nn.Linear(H, E, bias=False, device="meta")
        self.proj.weight = nn.Parameter(proj_weight.to(torch.bfloat16).contiguous(), requires_grad=False)
        self.scale = nn.Parameter(scale.to(torch.bfloat16), requires_grad=False)
        self.per_expert_scale = nn.Parameter(per_expert_scale.to(torch.float32).contiguous(), requires_grad=False)
        self.top_k_experts = top_k_experts
        self.eps = eps
        self._root_size = H ** -0.5
        # the norm's weight, scale * hidden**-0.5 rounded to bf16 (load time)
        self.norm_weight = nn.Parameter((self.scale.float() * self._root_size).to(torch.bfloat16),
                                        requires_grad=False)

    def normalize(self, x: torch.Tensor) -> torch.Tensor:
        """The router input: `rms_norm(x, scale * hidden**-0.5, eps)` in bf16
        (`vqmoe_rms_norm`)."""
        require_cuda(x)
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        H = self.proj.weight.shape[1]
        xi = _contig(x.reshape(-1, H))
        out = torch.empty_like(xi)
        _lib.call("vqmoe_rms_norm", xi.data_ptr(), self.norm_weight.data_ptr(), xi.shape[0], H,
                  float(self.eps), out.data_ptr(), c_stream(x.device))
        return out.reshape(x.shape)

    def forward(self, x: torch.Tensor):
        require_cuda(x)
        E, H = self.proj.weight.shape
        k = self.top_k_experts
        lead = x.shape[:-1]
        xn = _contig(self.normalize(x).reshape(-1, H))
        T = xn.shape[0]
        inds = torch.empty((T, k), dtype=torch.int32, device=x.device)
        scores = torch.empty((T, k), dtype=torch.float32, device=x.device)
        n = _lib.lib().vqmoe_router_workspace_size(T, E)
        ws = torch.empty(n, dtype=torch.uint8, device=x.device)
        _lib.call("vqmoe_router_ex", xn.data_ptr(), self.proj.weight.data_ptr(), None, T, H, E, k,
                  _lib.ROUTER_TOPK_SOFTMAX, self.per_expert_scale.data_ptr(), inds.data_ptr(),
                  scores.data_ptr(), None, ws.data_ptr(), n, c_stream(x.device))
        return inds.reshape(*lead, k), scores.to(torch.bfloat16).reshape(*lead, k)


class Experts(nn.Module):
    """`gemma4_text.py:196-214`: `switch_glu` is a `SwitchGLU` whose
    activation is `GeGLU` (VQ or bf16 experts)."""

    def __init__(self, switch_glu: SwitchGLU):
        super().__init__()
        if not isinstance(switch_glu.activation, GeGLU):
            raise ValueError("Gemma-4 experts use the GeGLU activation")
        self.switch_glu = switch_glu

    def forward(self, x: torch.Tensor, top_k_indices: torch.Tensor, top_k_weights: torch.Tensor) -> torch.Tensor:
        require_cuda(x, top_k_indices, top_k_weights)
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        sg = self.switch_glu
        H = sg.gate_proj.input_dims
        k = top_k_indices.shape[-1]
        lead = x.shape[:-1]
        xi = _contig(x.reshape(-1, H))
        T = xi.shape[0]
        ii = _contig(top_k_indices.reshape(T, k).to(torch.int32))
        ww = _contig(top_k_weights.reshape(T, k).to(torch.float32))
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        g, u, d = sg.gate_descriptor(), sg.up_proj.descriptor(), sg.down_proj.descriptor()
        n = _lib.lib().vqmoe_moe_experts_workspace_size(ctypes_ref(g), ctypes_ref(d), T, k)
        ws = torch.empty(n, dtype=torch.uint8, device=x.device)
        _lib.call("vqmoe_moe_experts", ctypes_ref(g), ctypes_ref(u), ctypes_ref(d), xi.data_ptr(), ii.data_ptr(),
                  ww.data_ptr(), T, k, out.data_ptr(), ws.data_ptr(), n, c_stream(x.device))
        return out.reshape(*lead, H)
