"""The Qwen3.5-MoE sparse block over libvqmoe, with the reference's module
interface and state-dict names.

Reference: `SparseMoeBlock` (`src/knurlogic/engine/families/qwen/
architecture/qwen3_5.py:151-192`): router `gate` (Linear H -> E, no bias),
`switch_mlp` (SwitchGLU of VQSwitchLinear / SwitchLinear experts),
`shared_expert` (MLP with gate_proj / up_proj / down_proj) and
`shared_expert_gate` (Linear H -> 1). `top_k` experts per token, the top-k
always renormalised (`norm_topk_prob = True`, vendored edit 7).

The whole block is one `vqmoe_sparse_moe_block` call (router, fused
gate/up + SwiGLU, down with the routing weight, shared expert, combine).
Under a tensor split (`sharding_group`), each rank runs the block on its
cut and the ranks' partials are summed in float32 and rounded once to bf16
(`src/knurlogic/engine/split/tensor.py:159-187`): by default in one kernel
with the combine, over NVLink peer memory (`vqmoe_sparse_moe_block_tp`,
buffers from torch's symmetric memory); `tp_reduce="nccl"` all-reduces
float32 partials over NCCL instead.
"""
from __future__ import annotations

import ctypes

import torch
from torch import nn

from . import _lib
from .switch_layers import (QuantizedSwitchLinear, SwitchGLU, SwitchLinear, VQSwitchLinear, c_stream,
                            require_cuda)


def _bf16_linear(weight: torch.Tensor) -> nn.Linear:
    out, inp = weight.shape
    lin = nn.Linear(inp, out, bias=False, device="meta")
    lin.weight = nn.Parameter(weight.to(torch.bfloat16).contiguous(),
                              requires_grad=False)
    return lin


def tp_reduce(part: torch.Tensor, group) -> torch.Tensor:
    """The ranks' partial block outputs (bf16 values held in float32) summed
    in float32 over `group`, in place, and rounded once to bf16: the
    reference's `Reduce` (`src/knurlogic/engine/split/tensor.py:159-187`)."""
    import torch.distributed as dist
    if part.dtype != torch.float32:
        raise TypeError(f"partials must be float32, got {part.dtype}")
    dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
    return part.to(torch.bfloat16)


class SharedExpert(nn.Module):
    """mlx-lm's MLP weights (`qwen3_5.py:115-117`): gate/up [I_s, H], down
    [H, I_s], bf16."""

    def __init__(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor):
        super().__init__()
        self.gate_proj = _bf16_linear(gate)
        self.up_proj = _bf16_linear(up)
        self.down_proj = _bf16_linear(down)


class SparseMoeBlock(nn.Module):
    """Qwen3.5-MoE `SparseMoeBlock` on B200. `forward(x [..., H] bf16)`.

    `router_mode` picks how the k weights come from the router logits:
    `_lib.ROUTER_SOFTMAX_TOPK_RENORM` (Qwen3.5, `qwen3_5.py:174-179`, the
    default), `_lib.ROUTER_TOPK_SOFTMAX` (Qwen4-exp's block with
    `norm_topk_prob`, `qwen4_exp.py:806-810`) or `_lib.ROUTER_SOFTMAX_TOPK`
    (Qwen4-exp without it, `qwen4_exp.py:811-814`)."""

    def __init__(self, gate_weight: torch.Tensor, switch_mlp: SwitchGLU,
                 top_k: int, shared_expert: SharedExpert | None = None,
                 shared_expert_gate_weight: torch.Tensor | None = None,
                 sharding_group=None, router_mode: int = _lib.ROUTER_SOFTMAX_TOPK_RENORM,
                 tp_reduce: str = "p2p", expert_split: bool = False):
        super().__init__()
        if tp_reduce not in ("p2p", "nccl"):
            raise ValueError(f"tp_reduce {tp_reduce!r} ('p2p' or 'nccl')")
        if expert_split and sharding_group is None:
            raise ValueError("expert_split needs the sharding group")
        # expert_split: this rank holds E / n whole experts (ids rank*E/n ..)
        # instead of a cut of every expert; reduced over peer memory
        self.expert_split = bool(expert_split)
        self.tp_reduce = "p2p" if expert_split else tp_reduce
        self._tp = None
        E, H = gate_weight.shape
        self.num_experts, self.hidden = int(E), int(H)
        self.top_k = int(top_k)
        if router_mode not in (_lib.ROUTER_SOFTMAX_TOPK_RENORM, _lib.ROUTER_TOPK_SOFTMAX,
                               _lib.ROUTER_SOFTMAX_TOPK):
            raise ValueError(f"router_mode {router_mode} (0, 1 or 2)")
        self.router_mode = int(router_mode)
        self.norm_topk_prob = router_mode != _lib.ROUTER_SOFTMAX_TOPK
        self.gate = _bf16_linear(gate_weight)
        self.switch_mlp = switch_mlp
        if (shared_expert is None) != (shared_expert_gate_weight is None):
            raise ValueError("shared_expert and shared_expert_gate go together")
        self.shared_expert = shared_expert
        self.shared_expert_gate = (_bf16_linear(shared_expert_gate_weight)
                                   if shared_expert_gate_weight is not None else None)
        self.sharding_group = sharding_group
        # polls before a phase 2 tile gives up waiting for its expert's
        # phase 1 tiles (0: the library default, about four seconds)
        self.wait_polls = 0
        sm = switch_mlp
        held = E
        if expert_split:
            import torch.distributed as dist
            n = dist.get_world_size(sharding_group)
            if E % n:
                raise ValueError(f"expert split: {E} experts over {n} ranks")
            held = E // n
        for name, mod, shape in (("gate_proj", sm.gate_proj, None),
                                 ("up_proj", sm.up_proj, None),
                                 ("down_proj", sm.down_proj, None)):
            if mod.num_experts != held:
                raise ValueError(f"switch_mlp.{name}: {mod.num_experts} experts, "
                                 f"router {E}" + (f" over the split ({held} a rank)" if expert_split else ""))
        if sm.gate_proj.input_dims != H or sm.down_proj.output_dims != H:
            raise ValueError("switch_mlp does not map hidden size "
                             f"{H} -> {H}")
        self._ws = None

    # ------------------------------------------------------------------
    def _desc(self) -> _lib.Block:
        sm = self.switch_mlp
        b = _lib.Block()
        b.hidden, b.num_experts, b.top_k = self.hidden, self.num_experts, self.top_k
        b.router_w = self.gate.weight.data_ptr()
        b.gate, b.up, b.down = (sm.gate_descriptor(), sm.up_proj.descriptor(),
                                sm.down_proj.descriptor())
        b.router_mode = self.router_mode
        b.wait_polls = self.wait_polls
        if self.shared_expert is not None:
            se = self.shared_expert
            b.shared_inter = se.gate_proj.weight.shape[0]
            b.shared_gate_w = se.gate_proj.weight.data_ptr()
            b.shared_up_w = se.up_proj.weight.data_ptr()
            b.shared_down_w = se.down_proj.weight.data_ptr()
            b.shared_expert_gate_w = self.shared_expert_gate.weight.data_ptr()
        else:
            b.shared_inter = 0
        return b

    def workspace(self, tokens: int, device) -> torch.Tensor:
        """The block's scratch for `tokens` tokens, kept between calls (so
        a captured CUDA graph reuses the same addresses)."""
        b = self._desc()
        need = _lib.lib().vqmoe_block_workspace_size(ctypes.byref(b), min(tokens, 2048))
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
        return self._ws

    def check_status(self, device=None) -> None:
        """Raise `_lib.VQMoEError` (status TIMEOUT) when one of the last
        call's bounded device waits ran out -- its output is then wrong.
        Synchronises the current stream (`vqmoe_workspace_status`)."""
        if self._ws is None:
            return
        _lib.call("vqmoe_workspace_status", self._ws.data_ptr(), c_stream(device or self._ws.device))

    def tp_buffers(self, tokens: int, device):
        """This rank's view of the split's symmetric buffers (`vqmoe_tp`),
        made once per device and size: a torch symmetric-memory buffer of
        `vqmoe_tp_buffer_bytes` per rank, zeroed, exchanged with the other
        ranks (a collective: every rank calls it in the same order), and a
        barrier so that no rank's kernel meets another's unzeroed flags."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        if self.expert_split:
            need = _lib.lib().vqmoe_ep_buffer_bytes(self.hidden, min(tokens, 2048), self.top_k)
        else:
            need = _lib.lib().vqmoe_tp_buffer_bytes(self.hidden, min(tokens, 2048))
        if self._tp is not None and self._tp[0] >= need and self._tp[1].device == device:
            return self._tp[2]
        g = self.sharding_group
        buf = symm_mem.empty(need, dtype=torch.uint8, device=device)
        buf.zero_()
        torch.cuda.synchronize(device)
        hdl = symm_mem.rendezvous(buf, g)
        d = _lib.Tp()
        d.rank, d.world = dist.get_rank(g), dist.get_world_size(g)
        for q in range(d.world):
            d.buffers[q] = hdl.buffer_ptrs[q]
        d.buffer_bytes = need
        dist.barrier(group=g)
        self._tp = (need, buf, d, hdl)
        return d

    def forward_into(self, x2d: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """The block on contiguous [T, H] bf16 into `out` ([T, H] bf16 or
        float32 -- float32 holds the bf16 result widened, for a reduction).
        Under a split with `tp_reduce="p2p"` (bf16 `out`) the result is the
        whole split's, reduced over peer memory."""
        T = x2d.shape[0]
        b = self._desc()
        ws = self.workspace(T, x2d.device)
        if self.expert_split and out.dtype != torch.bfloat16:
            raise TypeError("the expert split writes a bf16 output")
        if self.sharding_group is not None and self.tp_reduce == "p2p" and out.dtype == torch.bfloat16:
            tp = self.tp_buffers(T, x2d.device)
            _lib.call("vqmoe_sparse_moe_block_ep" if self.expert_split else "vqmoe_sparse_moe_block_tp",
                      ctypes.byref(b), ctypes.byref(tp), x2d.data_ptr(), T, out.data_ptr(), ws.data_ptr(),
                      ws.numel(), c_stream(x2d.device))
            return out
        odt = _lib.OUT_F32 if out.dtype == torch.float32 else _lib.OUT_BF16
        _lib.call("vqmoe_sparse_moe_block", ctypes.byref(b), x2d.data_ptr(), T,
                  out.data_ptr(), odt, ws.data_ptr(), ws.numel(), c_stream(x2d.device))
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        require_cuda(x)
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        shape = x.shape
        x2d = x.reshape(-1, self.hidden)
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        if self.sharding_group is None or self.tp_reduce == "p2p":
            out = torch.empty_like(x2d)
            return self.forward_into(x2d, out).reshape(shape)
        part = torch.empty(x2d.shape, dtype=torch.float32, device=x.device)
        self.forward_into(x2d, part)
        return tp_reduce(part, self.sharding_group).reshape(shape)

    # ------------------------------------------------------------------
    @classmethod
    def from_weights(cls, w: dict, top_k: int, prefix: str = "mlp.",
                     group_size: int | None = None, sharding_group=None,
                     router_mode: int = _lib.ROUTER_SOFTMAX_TOPK_RENORM, activation=None,
                     bits: int | None = None, tp_reduce: str = "p2p", expert_split: bool = False):
        """Build from a state dict with the reference's names:
        `{prefix}gate.weight`; `{prefix}switch_mlp.{gate,up,down}_proj.`
        `{codes, codebook, vq_scales}` (VQ), `{weight, scales, biases}`
        (affine-quantized; `group_size` default 64, `bits` from the packed
        width) or `.weight` (bf16), or the HF
        fused `{prefix}experts.gate_up_proj [E, 2I, H]` /
        `{prefix}experts.down_proj [E, H, I]` (split as
        `qwen3_5_moe.py:36-50`); `{prefix}shared_expert.{gate,up,down}_proj.`
        `weight`, `{prefix}shared_expert_gate.weight`. `router_mode` and
        `activation` (a `SwiGLU` or `GeGLU`) select the router and the
        experts' activation variants."""
        p = prefix
        sw = f"{p}switch_mlp."
        if f"{p}experts.gate_up_proj" in w:
            gu = w[f"{p}experts.gate_up_proj"]
            mid = gu.shape[-2] // 2
            projs = {"gate_proj": SwitchLinear(gu[..., :mid, :]),
                     "up_proj": SwitchLinear(gu[..., mid:, :]),
                     "down_proj": SwitchLinear(w[f"{p}experts.down_proj"])}
        else:
            projs = {}
            for n in ("gate_proj", "up_proj", "down_proj"):
                q = f"{sw}{n}."
                if q + "codes" in w:
                    codes, cb, vs = w[q + "codes"], w[q + "codebook"], w[q + "vq_scales"]
                    IN = codes.shape[-1] * cb.shape[-1]
                    gs = group_size or IN // vs.shape[-1]
                    projs[n] = VQSwitchLinear(codes, cb, vs, group_size=gs)
                elif q + "scales" in w and q + "biases" in w:
                    # affine-quantized (mlx's weight / scales / biases); the
                    # bits follow from the packed width at the group size
                    wt, sc = w[q + "weight"], w[q + "scales"]
                    gs = group_size or 64
                    nbits = bits or (wt.shape[-1] * 32) // (sc.shape[-1] * gs)
                    projs[n] = QuantizedSwitchLinear(wt, sc, w[q + "biases"], group_size=gs, bits=nbits)
                elif q + "weight" in w:
                    projs[n] = SwitchLinear(w[q + "weight"])
                else:
                    raise KeyError(f"no weights for {q}")
        se = None
        seg = None
        if f"{p}shared_expert.gate_proj.weight" in w:
            se = SharedExpert(w[f"{p}shared_expert.gate_proj.weight"],
                              w[f"{p}shared_expert.up_proj.weight"],
                              w[f"{p}shared_expert.down_proj.weight"])
            seg = w[f"{p}shared_expert_gate.weight"]
        return cls(w[f"{p}gate.weight"], SwitchGLU(**projs, activation=activation), top_k, se, seg,
                   sharding_group=sharding_group, router_mode=router_mode, tp_reduce=tp_reduce,
                   expert_split=expert_split)


class CapturedBlock:
    """One block call at a fixed token count, captured in a CUDA graph --
    the decode-step form a server replays every step.

    `__call__(x, out=None)` copies `x` ([T, H] bf16, host (pinned) or
    device) into the graph's static input, replays the graph, and copies
    the result into `out` (host or device) when given; otherwise it returns
    the static output buffer (overwritten by the next call). Under a tensor
    split the reduction is part of the graph (the peer-memory kernel, or the
    float32 NCCL all-reduce)."""

    def __init__(self, block: SparseMoeBlock, tokens: int):
        dev = block.gate.weight.device
        self.block = block
        H = block.hidden
        self.x = torch.zeros(tokens, H, dtype=torch.bfloat16, device=dev)
        self.y = torch.empty(tokens, H, dtype=torch.bfloat16, device=dev)
        self.part = (torch.empty(tokens, H, dtype=torch.float32, device=dev)
                     if block.sharding_group is not None and block.tp_reduce == "nccl" else None)
        if block.sharding_group is not None and block.tp_reduce == "p2p":
            block.tp_buffers(tokens, dev)          # a collective: before the capture
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self._step()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()

    def _step(self):
        if self.part is None:
            self.block.forward_into(self.x, self.y)
        else:
            import torch.distributed as dist
            self.block.forward_into(self.x, self.part)
            dist.all_reduce(self.part, op=dist.ReduceOp.SUM, group=self.block.sharding_group)
            self.y.copy_(self.part)

    def check_status(self) -> None:
        """The last replay's device-side status (`SparseMoeBlock.check_status`)."""
        self.block.check_status(self.x.device)

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None):
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        if out is None:
            return self.y
        out.copy_(self.y, non_blocking=True)
        return out
