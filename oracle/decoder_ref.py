"""CPU oracle for the decoder stack around the MoE block -- TEST
INFRASTRUCTURE ONLY (imported by `tests/` alone; the product never).

A numpy restatement, for small shapes, of the Qwen3.5 decoder the way this
build's decoder runs it (`knurlogic_b200/decoder.py`), in the reference's
order of roundings:
* `rms_norm` (RMSNorm.__call__, qwen3_5.py:120-130): float32 normalisation
  times the float32 (1 + w) gain, rounded once to bf16; the mean of squares
  summed exactly and rounded to float32 (the build's reading of MLX's fused
  kernel, unpinned);
* `attention` (Attention.__call__, qwen3_5.py:383-432): q_proj split into
  queries and gate per head, per-head q/k norms, rotary embedding over the
  first quarter of each head (mlx nn.RoPE, traditional=False), softmax
  attention (float64 here; MLX's bf16 SDPA rounds in between: unpinned, so
  the tests hold the GPU within a tolerance), output * bf16(sigmoid(gate)),
  o_proj;
* `decoder_layer` (DecoderLayer.__call__, qwen3_5.py:578-587): h = x + attn,
  out = h + mlp, bf16 adds; the MoE block is `moe_ref.sparse_moe_block`;
* `text_model` (Qwen3_5TextModel.__call__, qwen3_5.py:621-674): embed,
  layers, final norm, LM head;
* `mtp_head` (Qwen35Head._trunk, heads/qwen35.py:204-227): norm_e(embed),
  norm_h(h before the final norm), [e, h] . fc^T, one layer, norm_out.
Parity status: the norms, rotary and attention have no reference golden
here (MLX cannot run in this container): UNPINNED beyond the MoE block's
own pins.
"""
from __future__ import annotations

import numpy as np

from oracle import moe_ref as R


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm over the last axis: bf16(f32(f32(x * rs) * w)), rs =
    1 / sqrt(mean(x^2) + eps) in float32 (qwen3_5.py:120-130)."""
    x32 = np.asarray(x, np.float32)
    ms = (np.asarray(x32, np.float64) ** 2).mean(axis=-1, keepdims=True).astype(np.float32)
    rs = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return R.bf16((x32 * rs).astype(np.float32) * np.asarray(w, np.float32))


def rope(x: np.ndarray, pos0: int, dims: int, base: float) -> np.ndarray:
    """mlx nn.RoPE(dims, traditional=False, base) over x [L, heads, d]."""
    L = x.shape[0]
    half = dims // 2
    inv = (np.float32(base) ** (-np.arange(0, half, dtype=np.float32) * np.float32(2.0) / np.float32(dims)))
    ang = (np.arange(pos0, pos0 + L, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2 = x[..., :half].astype(np.float32), x[..., half:dims].astype(np.float32)
    rot = R.bf16(np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], axis=-1))
    return np.concatenate([rot, x[..., dims:]], axis=-1)


def attention(x: np.ndarray, w: dict, p: str, cfg, kv: dict, pos0: int) -> np.ndarray:
    """One sequence's attention: x [L, H] (normed), kv the layer's cache
    {"k": [n, kv_heads, d], "v": ...} of earlier positions (extended here)."""
    L = x.shape[0]
    nh, nkv, d = cfg.heads, cfg.kv_heads, cfg.head_dim
    q = R.linear(x, w[p + "q_proj.weight"]).reshape(L, nh, 2 * d)
    queries, gate = q[..., :d], q[..., d:].reshape(L, nh * d)
    queries = rms_norm(queries, w[p + "q_norm.weight"], cfg.eps)
    keys = rms_norm(R.linear(x, w[p + "k_proj.weight"]).reshape(L, nkv, d), w[p + "k_norm.weight"], cfg.eps)
    values = R.linear(x, w[p + "v_proj.weight"]).reshape(L, nkv, d)
    queries = rope(queries, pos0, cfg.rotary_dims, cfg.rope_theta)
    keys = rope(keys, pos0, cfg.rotary_dims, cfg.rope_theta)
    kv["k"] = np.concatenate([kv["k"], keys], axis=0) if kv["k"] is not None else keys
    kv["v"] = np.concatenate([kv["v"], values], axis=0) if kv["v"] is not None else values
    K, V = kv["k"].astype(np.float64), kv["v"].astype(np.float64)
    S = K.shape[0]
    rep = nh // nkv
    out = np.empty((L, nh, d), np.float64)
    qpos = pos0 + np.arange(L)
    for h in range(nh):
        s = queries[:, h, :].astype(np.float64) @ K[:, h // rep, :].T * (d ** -0.5)
        s = np.where(np.arange(S)[None, :] <= qpos[:, None], s, -np.inf)
        s = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h, :] = (s / s.sum(axis=1, keepdims=True)) @ V[:, h // rep, :]
    o = R.bf16(out.reshape(L, nh * d))
    g = R.bf16(R._sigmoid_f32(R.bf16(gate)))
    return R.linear(R.bf16(o * g), w[p + "o_proj.weight"])


def decoder_layer(x, w, p, cfg, moe_params, kv, pos0):
    """DecoderLayer.__call__ (qwen3_5.py:578-587) for one sequence."""
    r = attention(rms_norm(x, w[p + "input_layernorm.weight"], cfg.eps), w, p + "self_attn.", cfg, kv, pos0)
    h = R.bf16(x + r)
    m = R.sparse_moe_block(rms_norm(h, w[p + "post_attention_layernorm.weight"], cfg.eps), moe_params,
                           cfg.moe.top_k, vq=True)
    return R.bf16(h + m)


def text_model(tokens: np.ndarray, w: dict, cfg, moe_params: list, kvs: list, pos0: int):
    """One sequence: tokens [L] -> (logits [L, V] bf16, hidden before the
    final norm [L, H])."""
    x = np.asarray(w["model.embed_tokens.weight"], np.float32)[tokens]
    for i in range(cfg.layers):
        x = decoder_layer(x, w, f"model.layers.{i}.", cfg, moe_params[i], kvs[i], pos0)
    normed = rms_norm(x, w["model.norm.weight"], cfg.eps)
    return R.linear(normed, w["lm_head.weight"]), x


def mtp_head(h: np.ndarray, nxt: np.ndarray, w: dict, cfg, moe_params: dict, kv: dict, pos0: int):
    """Qwen35Head._trunk (heads/qwen35.py:204-227), "eh" order, h_source
    "pre_norm": -> (logits, the head's output before norm_out)."""
    e = rms_norm(np.asarray(w["model.embed_tokens.weight"], np.float32)[nxt], w["mtp.pre_fc_norm_embedding.weight"],
                 cfg.eps)
    hh = rms_norm(h, w["mtp.pre_fc_norm_hidden.weight"], cfg.eps)
    x = R.linear(np.concatenate([e, hh], axis=-1), w["mtp.fc.weight"])
    x = decoder_layer(x, w, "mtp.layers.0.", cfg, moe_params, kv, pos0)
    return R.linear(rms_norm(x, w["mtp.norm.weight"], cfg.eps), w["lm_head.weight"]), x
