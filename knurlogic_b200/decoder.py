"""The VQ-MoE decoder stack with multi-token-prediction drafting, around the
B200-native MoE block.

Reference (`src/knurlogic/engine/families/qwen/architecture/qwen3_5.py`):
`DecoderLayer` (549-587), `Qwen3_5TextModel` (590-674), full-attention
`Attention` (368-432), `RMSNorm` (120-130); the MTP head
`engine/families/qwen/heads/qwen35.py:53-227` (`Qwen35Head._trunk`); greedy
speculative decoding `engine/mtp/block_loop.py` (K drafts, a (K+1)-wide
verify, the longest agreeing prefix plus the verifier's own next token).

What runs where on the GPU:
  * the MoE block of every layer: `SparseMoeBlock` (libvqmoe: router, VQ
    experts, shared expert, combine);
  * every RMSNorm and the residual adds around it: `vqmoe_add_rms_norm`
    (libvqmoe), including the attention's per-head q/k norms;
  * projections, embeddings and the LM head: cuBLAS through torch (plain
    bf16 GEMMs); attention: torch's scaled-dot-product attention (a library
    kernel) over a per-sequence KV cache; rotary embedding: torch elementwise.
The decoder follows the baseline's C5 description -- every layer full GQA
attention (32 query / 4 key-value heads of 128) -- where the reference's
Qwen3.5 trunk alternates gated-delta-net layers with full attention
(`layer_types`, qwen3_5.py:255-265): the linear-attention layers are out of
this build's scope and not built.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib, synth
from .moe import SparseMoeBlock
from .switch_layers import c_stream, require_cuda


@dataclass(frozen=True)
class DecoderConfig:
    """A decoder's shapes. `moe` carries the MoE block's (its `tokens` is
    unused here)."""
    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    moe: synth.MoEConfig
    rope_theta: float = 10000.0          # qwen3_5.py:238
    partial_rotary: float = 0.25         # qwen3_5.py:237: rotary over a quarter of each head
    eps: float = 1e-6                    # qwen3_5.py:202
    mtp: bool = True                     # a one-layer MTP head

    @property
    def rotary_dims(self) -> int:
        return int(self.head_dim * self.partial_rotary)


# C5 of the baseline: 48 layers, hidden 4096, GQA 32/4 x 128, 256 experts
# top-8 of intermediate 1536 plus a shared expert (its width unstated: 1536),
# vocab 151936, 2-bit VQ experts, a one-layer MTP head.
CONFIGS = {
    "c5": DecoderConfig("c5", 48, 4096, 32, 4, 128, 151936,
                        synth.MoEConfig("c5-moe", 256, 8, 4096, 1536, 1536, 1)),
    # small shapes for tests and the CPU oracle
    "tiny": DecoderConfig("tiny", 2, 256, 4, 2, 64, 512,
                          synth.MoEConfig("tiny-moe", 8, 2, 256, 256, 256, 1)),
}


# ---------------------------------------------------------------- weights

def make_weights(cfg: DecoderConfig, seed: int = 0, device="cpu", scales: str = "random") -> dict:
    """Random-init weights with the reference's names (`model.layers.{i}.`,
    `mtp.`), seeded; norm gains are stored as float32 (1 + w), the form the
    reference keeps them in (qwen3_5.py:120-130, `sanitize`)."""
    g = synth._gen(seed, device)
    H, d, nh, kv = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads

    def normal(shape, std=0.02):
        return synth._normal(shape, std, g, device, torch.bfloat16)

    def gain(n):
        return 1.0 + torch.randn((n,), generator=g, device=device) * 0.02

    w = {"model.embed_tokens.weight": normal((cfg.vocab, H), 1.0),
         "model.norm.weight": gain(H),
         "lm_head.weight": normal((cfg.vocab, H))}

    def layer(p, lseed):
        w[p + "input_layernorm.weight"] = gain(H)
        w[p + "post_attention_layernorm.weight"] = gain(H)
        w[p + "self_attn.q_proj.weight"] = normal((nh * 2 * d, H))     # queries and the output gate
        w[p + "self_attn.k_proj.weight"] = normal((kv * d, H))
        w[p + "self_attn.v_proj.weight"] = normal((kv * d, H))
        w[p + "self_attn.o_proj.weight"] = normal((H, nh * d))
        w[p + "self_attn.q_norm.weight"] = gain(d)
        w[p + "self_attn.k_norm.weight"] = gain(d)
        w.update(synth.make_weights(cfg.moe, seed=lseed, device=device, scales=scales, prefix=p + "mlp."))

    for i in range(cfg.layers):
        layer(f"model.layers.{i}.", seed * 1000 + i + 1)
    if cfg.mtp:
        w["mtp.pre_fc_norm_embedding.weight"] = gain(H)
        w["mtp.pre_fc_norm_hidden.weight"] = gain(H)
        w["mtp.fc.weight"] = normal((H, 2 * H))
        w["mtp.norm.weight"] = gain(H)
        layer("mtp.layers.0.", seed * 1000 + 999)
    return w


# ------------------------------------------------------------------ norms

def add_rms_norm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
                 sum_out: torch.Tensor | None = None) -> torch.Tensor:
    """`vqmoe_add_rms_norm` over the last axis: returns norm(x + residual)
    (bf16), writing bf16(x + residual) into `sum_out` when given."""
    require_cuda(x, weight)
    H = x.shape[-1]
    rows = x.numel() // H
    out = torch.empty_like(x)
    _lib.call("vqmoe_add_rms_norm", x.data_ptr(), residual.data_ptr() if residual is not None else None,
              weight.data_ptr(), rows, H, ctypes.c_float(eps), sum_out.data_ptr() if sum_out is not None else None,
              out.data_ptr(), c_stream(x.device))
    return out


def _gain(w: torch.Tensor) -> torch.Tensor:
    return w.to(torch.float32).contiguous()


def _sigmoid_bf16(x: torch.Tensor) -> torch.Tensor:
    """`_sigmoid` (qwen3_5.py:35-36): in float32, rounded once."""
    return torch.sigmoid(x.float()).to(torch.bfloat16)


# --------------------------------------------------------------- attention

class KVCache:
    """One layer's keys and values, [B, max_len, kv_heads, head_dim] bf16,
    with one write index shared by every row (the reference's batched
    caches: block_loop.py commits the same count for every row)."""

    def __init__(self, B: int, max_len: int, kv_heads: int, head_dim: int, device):
        self.k = torch.zeros((B, max_len, kv_heads, head_dim), dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)

    @property
    def max_len(self) -> int:
        return self.k.shape[1]


def _positions(pos0, L: int, device) -> torch.Tensor:
    """pos0 .. pos0 + L - 1 on the device; pos0 an int, or a 0-d int64
    device tensor (a CUDA graph's position, advanced between replays)."""
    return torch.arange(L, device=device) + pos0


def rope(x: torch.Tensor, pos0, dims: int, base: float) -> torch.Tensor:
    """mlx `nn.RoPE(dims, traditional=False, base)` at offset pos0 over the
    first `dims` features of each head (x [B, L, heads, d] bf16): the two
    halves of those features rotated by pos * base^(-2i/dims), in float32,
    rounded once; the rest passed through."""
    L = x.shape[1]
    half = dims // 2
    inv = base ** (-torch.arange(0, half, device=x.device, dtype=torch.float32) * 2.0 / dims)
    pos = _positions(pos0, L, x.device).to(torch.float32)
    ang = pos[:, None] * inv[None, :]
    cos, sin = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
    xf = x[..., :dims].float()
    x1, x2 = xf[..., :half], xf[..., half:]
    rot = torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(torch.bfloat16)
    return torch.cat([rot, x[..., dims:]], dim=-1)


class Attention:
    """The full-attention block of qwen3_5.py:368-432: q_proj gives the
    queries and an output gate per head; per-head RMSNorm of queries and
    keys; partial rotary embedding; GQA attention over the cache; the output
    times sigmoid(gate), then o_proj."""

    def __init__(self, w: dict, p: str, cfg: DecoderConfig):
        self.cfg = cfg
        self.wq = w[p + "q_proj.weight"]
        self.wk = w[p + "k_proj.weight"]
        self.wv = w[p + "v_proj.weight"]
        self.wo = w[p + "o_proj.weight"]
        self.q_norm = _gain(w[p + "q_norm.weight"])
        self.k_norm = _gain(w[p + "k_norm.weight"])

    def __call__(self, x: torch.Tensor, cache: KVCache, pos0) -> torch.Tensor:
        """pos0: the first new position -- an int, or a 0-d device tensor,
        with which the step reads the whole cache under a mask and so can
        be captured in a CUDA graph and replayed at any position."""
        c = self.cfg
        B, L, _ = x.shape
        nh, kv, d = c.heads, c.kv_heads, c.head_dim
        q = F.linear(x, self.wq).view(B, L, nh, 2 * d)
        queries = add_rms_norm(q[..., :d].contiguous(), None, self.q_norm, c.eps)
        gate = q[..., d:].reshape(B, L, nh * d)
        keys = add_rms_norm(F.linear(x, self.wk).view(B, L, kv, d), None, self.k_norm, c.eps)
        values = F.linear(x, self.wv).view(B, L, kv, d)
        queries = rope(queries, pos0, c.rotary_dims, c.rope_theta)
        keys = rope(keys, pos0, c.rotary_dims, c.rope_theta)
        rep = nh // kv
        if torch.is_tensor(pos0):
            idx = _positions(pos0, L, x.device)
            cache.k.index_copy_(1, idx, keys)
            cache.v.index_copy_(1, idx, values)
            Q = queries.view(B, L, kv, rep, d).permute(0, 2, 3, 1, 4).reshape(B, kv, rep * L, d)
            mask = torch.arange(cache.max_len, device=x.device)[None, :] <= idx.repeat(rep)[:, None]
            o = F.scaled_dot_product_attention(Q, cache.k.transpose(1, 2), cache.v.transpose(1, 2), attn_mask=mask,
                                               scale=d ** -0.5)
            o = o.view(B, kv, rep, L, d).permute(0, 3, 1, 2, 4).reshape(B, L, nh * d)
            return F.linear(o * _sigmoid_bf16(gate), self.wo)
        if pos0 + L > cache.max_len:
            raise ValueError(f"KV cache of {cache.max_len} positions: writing {pos0}..{pos0 + L}")
        cache.k[:, pos0:pos0 + L] = keys
        cache.v[:, pos0:pos0 + L] = values
        S = pos0 + L
        K = cache.k[:, :S].transpose(1, 2)                     # [B, kv, S, d]
        V = cache.v[:, :S].transpose(1, 2)
        if pos0 == 0:
            o = F.scaled_dot_product_attention(queries.transpose(1, 2), K, V, is_causal=True, scale=d ** -0.5,
                                               enable_gqa=True).transpose(1, 2)
        else:
            # decode / verify: the query heads of one key-value head become
            # rows of one attention over that head's keys (no copies of K, V);
            # row (r, l), position pos0 + l, sees keys 0 .. pos0 + l
            Q = queries.view(B, L, kv, rep, d).permute(0, 2, 3, 1, 4).reshape(B, kv, rep * L, d)
            if L == 1:
                o = F.scaled_dot_product_attention(Q, K, V, scale=d ** -0.5)
            else:
                qpos = (pos0 + torch.arange(L, device=x.device)).repeat(rep)
                mask = torch.arange(S, device=x.device)[None, :] <= qpos[:, None]
                o = F.scaled_dot_product_attention(Q, K, V, attn_mask=mask, scale=d ** -0.5)
            o = o.view(B, kv, rep, L, d).permute(0, 3, 1, 2, 4)
        o = o.reshape(B, L, nh * d)
        return F.linear(o * _sigmoid_bf16(gate), self.wo)


class DecoderLayer:
    """DecoderLayer.__call__ (qwen3_5.py:578-587): h = x + attn(norm(x));
    out = h + mlp(post_norm(h)). The residual adds are fused with the norm
    that follows them: a layer takes (x, the previous layer's MoE output)
    and returns (h, its own MoE output) -- the caller's next norm adds it."""

    def __init__(self, w: dict, p: str, cfg: DecoderConfig):
        self.cfg = cfg
        self.input_layernorm = _gain(w[p + "input_layernorm.weight"])
        self.post_attention_layernorm = _gain(w[p + "post_attention_layernorm.weight"])
        self.self_attn = Attention(w, p + "self_attn.", cfg)
        self.mlp = SparseMoeBlock.from_weights(w, cfg.moe.top_k, prefix=p + "mlp.")

    def __call__(self, x: torch.Tensor, res: torch.Tensor | None, cache: KVCache, pos0: int):
        eps = self.cfg.eps
        if res is None:
            xs = x
            n1 = add_rms_norm(x, None, self.input_layernorm, eps)
        else:
            xs = torch.empty_like(x)
            n1 = add_rms_norm(x, res, self.input_layernorm, eps, sum_out=xs)
        a = self.self_attn(n1, cache, pos0)
        h = torch.empty_like(x)
        n2 = add_rms_norm(xs, a, self.post_attention_layernorm, eps, sum_out=h)
        B, L, H = x.shape
        m = self.mlp(n2.reshape(B * L, H)).reshape(B, L, H)
        return h, m


# ------------------------------------------------------------------ model

class TextModel:
    """Qwen3_5TextModel + the LM head (qwen3_5.py:590-674 and TextModel):
    embeddings, the decoder layers, the final norm. `__call__` returns the
    normed hidden states (for the LM head) and the hidden states before the
    final norm (what the MTP head reads: h_source "pre_norm")."""

    def __init__(self, w: dict, cfg: DecoderConfig, device, consume: bool = False):
        """consume: drop each layer's raw expert tensors from `w` once its
        MoE block has converted them (halves the peak memory of a build)."""
        self.cfg = cfg
        self.embed_tokens = w["model.embed_tokens.weight"]
        self.layers = []
        for i in range(cfg.layers):
            self.layers.append(DecoderLayer(w, f"model.layers.{i}.", cfg))
            if consume:
                _drop(w, f"model.layers.{i}.mlp.switch_mlp.")
                _release(self.layers[-1].mlp)
        self.norm = _gain(w["model.norm.weight"])
        self.lm_head = w["lm_head.weight"]
        self.mtp = MTPHead(w, cfg, self) if cfg.mtp else None
        if consume and self.mtp is not None:
            _drop(w, "mtp.layers.0.mlp.switch_mlp.")
            _release(self.mtp.layer.mlp)
        share_workspace([l.mlp for l in self.all_layers()], device)

    def all_layers(self):
        return self.layers + ([self.mtp.layer] if self.mtp is not None else [])

    def new_caches(self, B: int, max_len: int, device) -> list:
        c = self.cfg
        return [KVCache(B, max_len, c.kv_heads, c.head_dim, device) for _ in self.layers]

    def __call__(self, tokens: torch.Tensor, caches: list, pos0: int):
        require_cuda(tokens)
        x = F.embedding(tokens, self.embed_tokens)
        res = None
        for layer, cache in zip(self.layers, caches):
            x, res = layer(x, res, cache, pos0)
        pre = torch.empty_like(x)
        normed = add_rms_norm(x, res, self.norm, self.cfg.eps, sum_out=pre)
        return normed, pre

    def logits(self, normed: torch.Tensor) -> torch.Tensor:
        return F.linear(normed, self.lm_head)


class MTPHead:
    """The one-layer MTP head (Qwen35Head._trunk, heads/qwen35.py:204-227):
    e = norm_e(embed(token t+1)), h = norm_h(trunk hidden at t, before the
    final norm), x = [e, h] . fc^T ("eh" order), one decoder layer of full
    attention + MoE, norm_out; the trunk's LM head gives its logits."""

    def __init__(self, w: dict, cfg: DecoderConfig, trunk: TextModel):
        self.cfg = cfg
        self.trunk = trunk
        self.norm_e = _gain(w["mtp.pre_fc_norm_embedding.weight"])
        self.norm_h = _gain(w["mtp.pre_fc_norm_hidden.weight"])
        self.fc = w["mtp.fc.weight"]
        self.norm_out = _gain(w["mtp.norm.weight"])
        self.layer = DecoderLayer(w, "mtp.layers.0.", cfg)

    def new_cache(self, B: int, max_len: int, device) -> KVCache:
        c = self.cfg
        return KVCache(B, max_len, c.kv_heads, c.head_dim, device)

    def __call__(self, h: torch.Tensor, nxt: torch.Tensor, cache: KVCache, pos0: int):
        """h [B, L, H] hidden states at positions pos0.., nxt [B, L] the
        tokens after them -> (normed output, output before norm_out)."""
        eps = self.cfg.eps
        e = add_rms_norm(F.embedding(nxt, self.trunk.embed_tokens), None, self.norm_e, eps)
        hh = add_rms_norm(h, None, self.norm_h, eps)
        x = F.linear(torch.cat([e, hh], dim=-1), self.fc)
        x, res = self.layer(x, None, cache, pos0)
        pre = torch.empty_like(x)
        normed = add_rms_norm(x, res, self.norm_out, eps, sum_out=pre)
        return normed, pre


def _release(block: SparseMoeBlock) -> None:
    """Drop the artifact-layout copies of a block's VQ experts (the kernels
    read their own layout)."""
    sw = block.switch_mlp
    for lin in (sw.gate_proj, sw.up_proj, sw.down_proj):
        if hasattr(lin, "release_source"):
            lin.release_source()


def _drop(w: dict, prefix: str) -> None:
    for k in [k for k in w if k.startswith(prefix)]:
        del w[k]


def share_workspace(blocks: list, device, tokens: int = 2048) -> None:
    """One scratch for every layer's MoE block: the layers run one after
    another on one stream, so a single workspace (sized for the largest
    block at `tokens`) serves them all."""
    need = 0
    for b in blocks:
        need = max(need, _lib.lib().vqmoe_block_workspace_size(ctypes.byref(b._desc()), tokens))
    ws = torch.empty(need, dtype=torch.uint8, device=device)
    for b in blocks:
        b._ws = ws


def build(cfg: DecoderConfig, seed: int = 0, device="cuda") -> TextModel:
    """A random-init decoder (weights generated on `device`)."""
    dev = torch.device(device)
    return TextModel(make_weights(cfg, seed=seed, device=dev), cfg, dev, consume=True)


# -------------------------------------------------------------- generation

def _argmax(model: TextModel, normed: torch.Tensor) -> torch.Tensor:
    """The greedy choice from float32 logits (bf16 operands, float32
    output): at a vocabulary of 152k the bf16-rounded logits tie often, and
    a tie would be broken by rounding noise that differs between a 1-wide
    and a (k+1)-wide forward."""
    H = normed.shape[-1]
    lg = torch.mm(normed.reshape(-1, H), model.lm_head.t(), out_dtype=torch.float32)
    return lg.argmax(dim=-1).view(normed.shape[:-1])


class _Captured:
    """`fn` (no arguments; it reads static input tensors the caller fills
    between calls) captured as one CUDA graph; calling replays it and
    returns its static outputs. One eager run before the capture warms the
    kernels: its cache writes land on positions the first replay writes
    again before anything reads them."""

    def __init__(self, fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn()

    def __call__(self):
        self.graph.replay()
        return self.out


class _Clock:
    """CUDA events at the end of the prefill and of the decoding; the
    device times land in `stats` (prefill_ms, decode_ms) at the end."""

    def __init__(self, stats: dict | None):
        self.stats = stats
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if stats is not None else None
        if self.ev:
            self.ev[0].record()

    def mark(self, i: int):
        if self.ev:
            self.ev[i].record()

    def done(self):
        if self.ev:
            self.ev[2].record()
            self.ev[2].synchronize()
            self.stats["prefill_ms"] = self.ev[0].elapsed_time(self.ev[1])
            self.stats["decode_ms"] = self.ev[1].elapsed_time(self.ev[2])


@torch.no_grad()
def generate_greedy(model: TextModel, prompts: torch.Tensor, steps: int, graphs: bool = False,
                    stats: dict | None = None) -> torch.Tensor:
    """Plain greedy decoding: the prompt in one forward, then one token per
    forward. prompts [B, P] int64 -> the next `steps` tokens [B, steps].
    graphs: each one-token step is one CUDA-graph replay (the position a
    device tensor). stats: filled with the device time of the prefill (and
    first token; with graphs, the capture too) and of the decoding
    (prefill_ms, decode_ms)."""
    B, P = prompts.shape
    clock = _Clock(stats)
    caches = model.new_caches(B, P + steps + 1, prompts.device)
    normed, _ = model(prompts, caches, 0)
    nxt = _argmax(model, normed[:, -1])
    out = [nxt]
    if graphs and steps > 1:
        tok = nxt[:, None].clone()
        pos = torch.full((), P, dtype=torch.int64, device=prompts.device)

        def step():
            return _argmax(model, model(tok, caches, pos)[0][:, -1])

        g = _Captured(step)
        clock.mark(1)                                                # (the capture is not decoding)
        for _ in range(1, steps):
            y = g()
            out.append(y.clone())
            tok.copy_(y[:, None])
            pos.add_(1)
    else:
        clock.mark(1)
        for s in range(1, steps):
            normed, _ = model(nxt[:, None], caches, P + s - 1)
            nxt = _argmax(model, normed[:, -1])
            out.append(nxt)
    clock.done()
    return torch.stack(out, dim=1)


@torch.no_grad()
def generate_mtp(model: TextModel, prompts: torch.Tensor, steps: int, k: int = 3, graphs: bool = False):
    """Greedy decoding with the MTP head drafting k tokens a step and one
    (k+1)-wide trunk forward verifying them (block_loop.py's loop, greedy
    verdicts): every row commits the same count, m = the fewest drafts any
    row had accepted; each row emits its pending token and its first m
    drafts, and its next pending token is the trunk's own choice at position
    m. The head's cache takes only committed positions, from the verify's
    hidden states (a (k+1)-row head forward that also gives the next first
    draft); drafts 2..k chain the head on its own output.
    graphs: the verify, the head's catch-up and its one-row draft each
    replay as one CUDA graph; one host read per step (m).
    Returns (tokens [B, steps], {"steps", "drafted", "accepted",
    "prefill_ms", "decode_ms"}); the tokens are plain greedy decoding's."""
    if model.mtp is None:
        raise ValueError("the model has no MTP head")
    B, P = prompts.shape
    dev = prompts.device
    stats = {"steps": 0, "drafted": 0, "accepted": 0}
    clock = _Clock(stats)
    max_len = P + steps + 2 * k + 2
    caches = model.new_caches(B, max_len, dev)
    hc = model.mtp.new_cache(B, max_len, dev)
    normed, pre = model(prompts, caches, 0)
    t1 = _argmax(model, normed[:, -1])                              # token P
    # head rows 0..P-1: (trunk hidden at j, token j + 1)
    hn, hp = model.mtp(pre, torch.cat([prompts[:, 1:], t1[:, None]], dim=1), hc, 0)
    g = hp[:, -1:]
    drafts = [_argmax(model, hn[:, -1])]
    del normed, pre, hn, hp
    L = P                                                            # committed trunk positions
    out = [t1]
    if graphs:
        H = model.cfg.hidden
        vtok = torch.zeros((B, k + 1), dtype=torch.int64, device=dev)
        vpos = torch.full((), L, dtype=torch.int64, device=dev)
        dtok = torch.zeros((B, 1), dtype=torch.int64, device=dev)
        dg = torch.zeros((B, 1, H), dtype=torch.bfloat16, device=dev)
        dpos = torch.full((), L, dtype=torch.int64, device=dev)

        def fv():
            n, p = model(vtok, caches, vpos)
            return _argmax(model, n), p

        verify = _Captured(fv)
        vy, vpre = verify.out

        def fc():
            n, p = model.mtp(vpre, vy, hc, vpos)
            return _argmax(model, n), p

        def fd():
            n, p = model.mtp(dg, dtok, hc, dpos)
            return _argmax(model, n)[:, 0], p

        catchup, draft = _Captured(fc), _Captured(fd)
    clock.mark(1)                                                    # (the captures are not decoding)
    while len(out) < steps:
        for i in range(1, k):                                        # head rows L .. L + k - 2
            if graphs:
                dg.copy_(g)
                dtok.copy_(drafts[-1][:, None])
                dpos.fill_(L - 1 + i)
                di, g = draft()
                drafts.append(di.clone())
            else:
                hn, g = model.mtp(g, drafts[-1][:, None], hc, L - 1 + i)
                drafts.append(_argmax(model, hn[:, -1]))
        d = torch.stack(drafts, dim=1)                               # [B, k]
        if graphs:                                                   # trunk rows L .. L + k
            vtok[:, 0] = t1
            vtok[:, 1:] = d
            vpos.fill_(L)
            y, pre = verify()
        else:
            normed, pre = model(torch.cat([t1[:, None], d], dim=1), caches, L)
            y = _argmax(model, normed)                               # [B, k + 1]
        agree = torch.cumprod((d == y[:, :k]).to(torch.int32), dim=1).sum(dim=1)
        m = int(agree.min().item())
        stats["steps"] += 1
        stats["drafted"] += B * k
        stats["accepted"] += B * m
        out.extend(drafts[:m])
        t1 = y[:, m].clone()
        out.append(t1)
        # head rows L .. L + k: (trunk hidden at L + i, token L + i + 1 = y_i for i <= m)
        if graphs:
            hy, hp = catchup()
            drafts = [hy[:, m].clone()]
        else:
            hn, hp = model.mtp(pre, y, hc, L)
            drafts = [_argmax(model, hn[:, m])]
        g = hp[:, m:m + 1].clone()
        L += m + 1
    clock.done()
    return torch.stack(out[:steps], dim=1), stats
