"""Switch (expert) linears and SwitchGLU over libvqmoe, with the reference's
module interface.

Reference interfaces mirrored here:
* `VQSwitchLinear(codes, codebook, vq_scales, *, group_size, pack_bits,
  in_features=None)` -- the VQ runtime's module, as Knurlogic builds and
  calls it (`src/knurlogic/engine/families/deepseek/heads/deepseek_v4.py:
  77-130`; attributes read by `engine/split/viability.py:37-40` and
  `engine/split/tensor.py:258-267`), called `mod(x, indices,
  sorted_indices=...)` (`switch_layers.py:71-86`).
* `SwitchLinear(weight)` -- mlx-lm's bf16 expert linear
  (`glm5_next/_mlx_vlm/models/switch_layers.py:89-125`).
* `SwitchGLU(gate_proj, up_proj, down_proj)` -- `switch_layers.py:151-193`.

Every call runs on the CUDA path; there is no CPU implementation.
"""
from __future__ import annotations

import numpy as np
import torch
from torch import nn

from . import _lib


def _stream(t: torch.Tensor):
    return c_stream(t.device)


def c_stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "knurlogic_b200 runs on CUDA tensors only (there is no CPU "
                f"path); got a tensor on {t.device}")


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


class _SwitchBase(nn.Module):
    """What both switch linears share: the call convention."""

    num_experts: int
    output_dims: int
    input_dims: int

    def descriptor(self) -> _lib.Linear:           # pragma: no cover
        raise NotImplementedError

    def _x_dtype(self):
        return torch.bfloat16

    def forward(self, x: torch.Tensor, indices: torch.Tensor,
                sorted_indices: bool = False) -> torch.Tensor:
        """y[..., k, 1, OUT] = x @ W[indices]^T.

        x is `[..., 1, 1, IN]` (one row per token, SwitchGLU's
        `expand_dims(x, (-2, -3))`), `[..., k, 1, IN]` (one row per
        (token, slot)), or, with indices `[N]`, `[N, 1, IN]` (the sorted
        form `_gather_sort` makes). `sorted_indices` is accepted for the
        reference's signature; the kernel groups pairs by expert itself."""
        require_cuda(x, indices)
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        if x.shape[-1] != self.input_dims:
            raise ValueError(f"x has {x.shape[-1]} features, the module "
                             f"{self.input_dims}")
        # gather_mm's rule: x's batch shape x.shape[:-2] broadcasts against
        # the indices' shape; one output row per index
        if x.dim() < 2 or x.shape[-2] != 1:
            raise ValueError(f"x must be [..., 1, IN], got {tuple(x.shape)}")
        xb, ib = tuple(x.shape[:-2]), tuple(indices.shape)
        try:
            B = tuple(torch.broadcast_shapes(xb, ib))
        except RuntimeError:
            raise ValueError(f"x {tuple(x.shape)} does not broadcast with "
                             f"indices {ib}") from None
        if B != ib:
            raise ValueError(f"indices {ib} must cover x's batch {xb}")
        P = int(np.prod(B)) if B else 1
        k = B[-1] if B else 1
        if len(xb) == len(B) and xb[:-1] == B[:-1] and xb[-1] == 1 and k > 1:
            per_pair, tokens = 0, P // k          # one x row per token
        else:
            if xb != B:
                x = x.expand(*B, 1, self.input_dims)
            per_pair, tokens, k = 1, P, 1         # one x row per index
        xi = _contig(x.reshape(-1, self.input_dims))
        ii = _contig(indices.reshape(-1).to(torch.int32))
        y = torch.empty((P, self.output_dims), dtype=torch.bfloat16, device=x.device)
        d = self.descriptor()
        n = _lib.lib().vqmoe_switch_linear_workspace_size(ctypes_ref(d), tokens, k, per_pair)
        ws = torch.empty(n, dtype=torch.uint8, device=x.device)
        _lib.call("vqmoe_switch_linear", ctypes_ref(d), xi.data_ptr(),
                  per_pair, ii.data_ptr(), tokens, k, y.data_ptr(), ws.data_ptr(), n,
                  _stream(x))
        return y.reshape(*B, 1, self.output_dims)


def ctypes_ref(s):
    import ctypes
    return ctypes.byref(s)


class SwitchLinear(_SwitchBase):
    """bf16 experts: weight [E, OUT, IN] (`switch_layers.py:89-125`)."""

    def __init__(self, weight: torch.Tensor):
        super().__init__()
        if weight.dim() != 3:
            raise ValueError(f"weight must be [E, OUT, IN], got {tuple(weight.shape)}")
        self.weight = nn.Parameter(weight.to(torch.bfloat16).contiguous(),
                                   requires_grad=False)

    @property
    def num_experts(self):
        return self.weight.shape[0]

    @property
    def output_dims(self):
        return self.weight.shape[1]

    @property
    def input_dims(self):
        return self.weight.shape[2]

    def descriptor(self) -> _lib.Linear:
        w = self.weight
        require_cuda(w)
        return _lib.Linear(format=_lib.FMT_DENSE_BF16, num_experts=w.shape[0],
                           out_features=w.shape[1], in_features=w.shape[2],
                           weight=w.data_ptr())


class VQSwitchLinear(_SwitchBase):
    """VQ experts: codes [E, OUT, IN/dim] with one code per entry (uint8
    when K <= 256, uint16 above: `deepseek_v4.py:111-121`), codebook
    [K, dim] fp16 with dim 2, 4 or 8 (shared by all experts, never split),
    vq_scales [E, OUT, IN/group] fp16.

    Weight of expert e, row o, input i (the dequantisation this build
    defines; the reference runtime is absent):
        W = fp16(codebook[codes[e, o, i // dim], i % dim] * vq_scales[e, o, i // group])
    and the activations enter the matmul as fp16.

    `codes` and `vq_scales` stay in the reference layout. uint8 codes of a
    dim-4 codebook with 64-input groups take the fast path: the kernels read
    a tiled copy (`vqmoe_prepare_vq`) made on the module's device at first
    use. Every other format (dim 2 or 8, K up to 65536, other group sizes)
    runs on the reference layout itself (`VQMOE_FMT_VQ_REF`). Packed codes
    (`pack_bits` > 0, uint32 words of ceil(log2 K)-bit fields) are rejected:
    their bit order is not pinned by the reference."""

    def __init__(self, codes: torch.Tensor, codebook: torch.Tensor,
                 vq_scales: torch.Tensor, *, group_size: int, pack_bits: int = 0,
                 in_features: int | None = None):
        super().__init__()
        if codes.dim() != 3 or vq_scales.dim() != 3 or codebook.dim() != 2:
            raise ValueError("VQ needs codes [E, OUT, W], codebook [K, dim] and "
                             "vq_scales [E, OUT, IN/group]")
        E, OUT, W = (int(n) for n in codes.shape)
        K, dim = (int(n) for n in codebook.shape)
        if pack_bits:
            raise NotImplementedError(
                f"packed {pack_bits}-bit VQ codes are not supported (the field "
                "order inside a uint32 word is not pinned); pass one code per "
                "entry (pack_bits=0)")
        IN = W * dim
        if in_features is not None and int(in_features) != IN:
            raise ValueError(f"codes rows are {W} wide; in={in_features} at dim "
                             f"{dim} needs {int(in_features) // dim} codes")
        ngrp = int(vq_scales.shape[-1])
        if tuple(vq_scales.shape[:2]) != (E, OUT):
            raise ValueError(f"vq_scales {tuple(vq_scales.shape)}: shape mismatch "
                             f"with codes {tuple(codes.shape)}")
        if ngrp <= 0 or IN % ngrp or IN // ngrp != int(group_size):
            raise ValueError(f"in={IN} does not divide into {ngrp} scale groups "
                             f"of {group_size}")
        want = torch.uint8 if K <= 256 else torch.uint16
        if K > 65536 or codes.dtype != want:
            raise ValueError(f"codes for K={K} must be {want} with one code per entry "
                             f"(K <= 65536), got {codes.dtype}")
        if dim not in (2, 4, 8):
            raise ValueError(f"VQ dim {dim} is not supported (2, 4 or 8)")
        if int(group_size) % dim:
            raise ValueError(f"group_size {group_size} is not a multiple of dim {dim}")
        self.group_size = int(group_size)
        # the tiled fast path, or the reference layout as it is
        self.fast = K <= 256 and dim == 4 and self.group_size == 64
        self.pack_bits = 0
        self._k_expect = K
        self.register_buffer("codes", codes.contiguous(), persistent=True)
        self.register_buffer("codebook", codebook.to(torch.float16).contiguous())
        self.register_buffer("vq_scales", vq_scales.to(torch.float16).contiguous())
        self._dev = None          # (device, data_ptr, prepared codes)

    @property
    def num_experts(self):
        return self.codes.shape[0]

    @property
    def output_dims(self):
        return self.codes.shape[1]

    @property
    def input_dims(self):
        return self.codes.shape[2] * self.codebook.shape[1]

    def prepared(self):
        """(codes, scales) as the kernels read them: on the fast path the
        tiled device layout (tiles of 32 rows x 256 inputs,
        `vqmoe_prepare_vq`), made once per device and weight version; else
        the module's own tensors. Checks every code against the codebook size
        (one host synchronisation, at first use: call it before capturing a
        CUDA graph)."""
        c, vs = self.codes, self.vq_scales
        if c.is_meta:                                    # released: the device layout is all there is
            return self._dev[1], self._dev[2]
        require_cuda(c, vs)
        key = (c.device, c.data_ptr(), c._version, vs.data_ptr(), vs._version)
        if self._dev is None or self._dev[0] != key:
            E, OUT, W = c.shape
            K, dim = (int(n) for n in self.codebook.shape)
            bad = torch.zeros(1, dtype=torch.int32, device=c.device)
            _lib.call("vqmoe_count_bad_codes" if c.dtype == torch.uint8 else "vqmoe_count_bad_codes_u16",
                      c.data_ptr(), c.numel(), K, bad.data_ptr(), _stream(c))
            n_bad = int(bad.item())
            if n_bad:
                raise ValueError(f"{n_bad} VQ codes are >= the codebook size {K}")
            if not self.fast:
                self._dev = (key, c, vs)
                return c, vs
            IN = W * dim
            nc, ns = _lib.vq_layout_bytes(E, OUT, IN)
            dc = torch.empty(nc, dtype=torch.uint8, device=c.device)
            ds = torch.empty(ns // 2, dtype=torch.float16, device=c.device)
            _lib.call("vqmoe_prepare_vq", c.data_ptr(), vs.data_ptr(), E, OUT, IN,
                      dc.data_ptr(), ds.data_ptr(), _stream(c))
            self._dev = (key, dc, ds)
        return self._dev[1], self._dev[2]

    def release_source(self) -> None:
        """Keep only what the kernels read. On the fast path the tiled
        device layout is a converted copy of `codes` and `vq_scales`; this
        drops the artifact-layout tensors (they become shape-only tensors on
        the meta device, so `num_experts` / `output_dims` / `input_dims`
        still answer) to halve the module's device memory -- for a whole
        model held on one GPU. The reference layout is the kernels' own
        (nothing to drop)."""
        if not self.fast or self.codes.is_meta:
            return
        self.prepared()
        self.codes = torch.empty(self.codes.shape, dtype=self.codes.dtype, device="meta")
        self.vq_scales = torch.empty(self.vq_scales.shape, dtype=self.vq_scales.dtype, device="meta")

    def descriptor(self) -> _lib.Linear:
        dc, ds = self.prepared()
        require_cuda(self.codebook)
        return _lib.Linear(format=_lib.FMT_VQ_U8 if self.fast else _lib.FMT_VQ_REF,
                           num_experts=self.num_experts,
                           out_features=self.output_dims,
                           in_features=self.input_dims, codes=dc.data_ptr(),
                           codebook=self.codebook.data_ptr(),
                           scales=ds.data_ptr(),
                           codebook_size=int(self.codebook.shape[0]),
                           dim=int(self.codebook.shape[1]),
                           group_size=self.group_size)

    def dequantize(self, first: int = 0, count: int | None = None) -> torch.Tensor:
        """Dense fp16 weights of experts [first, first + count) -- what the
        VQ runtime's prefill path decodes experts to (`tuning/measured.py:
        21-33`)."""
        count = self.num_experts - first if count is None else count
        out = torch.empty((count, self.output_dims, self.input_dims),
                          dtype=torch.float16, device=self.codebook.device)
        d = self.descriptor()
        _lib.call("vqmoe_dequant", ctypes_ref(d), first, count, out.data_ptr(),
                  _stream(out))
        return out


class QuantizedSwitchLinear(_SwitchBase):
    """Affine-quantized experts, mlx-lm's `QuantizedSwitchLinear`
    (`switch_layers.py:24-86`, called through `mx.gather_qmm` in mode
    "affine"): `weight [E, OUT, IN*bits/32]` uint32 -- each row a
    little-endian bit stream of `bits`-bit values q, element j at bits
    [j*bits, (j+1)*bits), as `mx.quantize` packs them -- and `scales`,
    `biases [E, OUT, IN/group_size]` bf16.

    Weight of expert e, row o, input i (this build's rounding; MLX's own
    kernels cannot run here): W = bf16(fmaf(scale, q, bias)) with the
    group's scale and bias; the bf16 activations enter a bf16 matmul as they
    are. `bits` 2, 3, 4, 5, 6 or 8; `group_size` 32, 64 or 128. The
    reference's optional per-expert output `bias` is not taken."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
                 group_size: int = 64, bits: int = 4, mode: str = "affine", bias: torch.Tensor | None = None):
        super().__init__()
        if mode != "affine":
            raise NotImplementedError(f"quantization mode {mode!r}: only 'affine' is supported")
        if bias is not None:
            raise NotImplementedError("a per-expert output bias on a quantized switch linear is not supported")
        if weight.dim() != 3 or scales.dim() != 3 or biases is None or biases.shape != scales.shape:
            raise ValueError("affine experts need weight [E, OUT, W], scales and biases [E, OUT, IN/group]")
        if int(bits) not in (2, 3, 4, 5, 6, 8) or int(group_size) not in (32, 64, 128):
            raise ValueError(f"bits {bits} (2, 3, 4, 5, 6, 8) / group_size {group_size} (32, 64, 128)")
        E, OUT, W = (int(n) for n in weight.shape)
        IN = int(scales.shape[-1]) * int(group_size)
        if tuple(scales.shape[:2]) != (E, OUT) or W * 32 != IN * int(bits):
            raise ValueError(f"weight {tuple(weight.shape)} holds {W * 32 // int(bits)} {bits}-bit values per "
                             f"row; scales {tuple(scales.shape)} at group {group_size} describe {IN}")
        if weight.dtype not in (torch.uint32, torch.int32):
            raise ValueError(f"weight must be packed uint32 words, got {weight.dtype}")
        self.group_size, self.bits, self.mode = int(group_size), int(bits), mode
        self.register_buffer("weight", weight.contiguous())
        self.register_buffer("scales", scales.to(torch.bfloat16).contiguous())
        self.register_buffer("biases", biases.to(torch.bfloat16).contiguous())

    @property
    def num_experts(self):
        return self.weight.shape[0]

    @property
    def output_dims(self):
        return self.weight.shape[1]

    @property
    def input_dims(self):
        return self.scales.shape[2] * self.group_size

    def descriptor(self) -> _lib.Linear:
        require_cuda(self.weight, self.scales, self.biases)
        return _lib.Linear(format=_lib.FMT_AFFINE, num_experts=self.num_experts,
                           out_features=self.output_dims, in_features=self.input_dims,
                           weight=self.weight.data_ptr(), scales=self.scales.data_ptr(),
                           biases=self.biases.data_ptr(), group_size=self.group_size, bits=self.bits)

    def dequantize(self, first: int = 0, count: int | None = None) -> torch.Tensor:
        """Dense bf16 weights of experts [first, first + count)."""
        count = self.num_experts - first if count is None else count
        out = torch.empty((count, self.output_dims, self.input_dims), dtype=torch.bfloat16,
                          device=self.weight.device)
        d = self.descriptor()
        _lib.call("vqmoe_dequant", ctypes_ref(d), first, count, out.data_ptr(), _stream(out))
        return out


class SwiGLU(nn.Module):
    """`_SwiGLU` (`qwen3_5.py:108-112`): bf16(bf16(silu(gate)) * x), silu in
    float32. A marker for `SwitchGLU(activation=...)`: the kernels apply it
    in the gate/up epilogue."""
    code = _lib.ACT_SWIGLU


class GeGLU(nn.Module):
    """`GeGLU` (`gemma4_text.py:186-189`, `geglu` 131-135): bf16(bf16(
    gelu_tanh(gate)) * x), gelu's tanh form in float32. A marker for
    `SwitchGLU(activation=...)`."""
    code = _lib.ACT_GEGLU


class SwitchGLU(nn.Module):
    """`SwitchGLU` (`switch_layers.py:151-193`): y = down(act(gate(x), up(x)))
    per (token, slot), act the Qwen3.5 `_SwiGLU` (default, `qwen3_5.py:
    108-112`) or Gemma-4's `GeGLU`. One fused gate/up launch and one down
    launch."""

    def __init__(self, gate_proj: _SwitchBase, up_proj: _SwitchBase,
                 down_proj: _SwitchBase, activation: nn.Module | None = None):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.activation = activation if activation is not None else SwiGLU()
        if not isinstance(self.activation, (SwiGLU, GeGLU)):
            raise ValueError(f"activation {type(self.activation).__name__}: "
                             "SwiGLU or GeGLU (the kernels apply it in the gate/up epilogue)")

    def gate_descriptor(self) -> _lib.Linear:
        """The gate linear's descriptor, naming the activation."""
        g = self.gate_proj.descriptor()
        g.activation = self.activation.code
        return g

    def forward(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        require_cuda(x, indices)
        if x.dtype != torch.bfloat16:
            raise TypeError(f"x must be bfloat16, got {x.dtype}")
        H = self.gate_proj.input_dims
        k = indices.shape[-1]
        lead = indices.shape[:-1]
        xi = _contig(x.reshape(-1, H))
        T = xi.shape[0]
        ii = _contig(indices.reshape(T, k).to(torch.int32))
        y = torch.empty((T, k, self.down_proj.output_dims), dtype=torch.bfloat16,
                        device=x.device)
        g, u, d = self.gate_descriptor(), self.up_proj.descriptor(), self.down_proj.descriptor()
        ws_bytes = _lib.lib().vqmoe_switch_glu_workspace_size(ctypes_ref(g), ctypes_ref(d), T, k)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        _lib.call("vqmoe_switch_glu", ctypes_ref(g), ctypes_ref(u), ctypes_ref(d),
                  xi.data_ptr(), ii.data_ptr(), T, k, y.data_ptr(), ws.data_ptr(),
                  ws_bytes, _stream(x))
        return y.reshape(*lead, k, -1)
