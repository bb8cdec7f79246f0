"""An independent float64 PyTorch implementation of the network (exact erf GELU, torch
softmax/LayerNorm), used only to cross-check the C oracle's restatement of the reference's
CPU backend. Built from the architecture's definition, not from the oracle's code."""

from __future__ import annotations

import math

import numpy as np
import torch


def forward64(arch, w, boards: np.ndarray):
    """Policy logits [n, 4672] and value logits [n, 3] in float64."""
    T = lambda name: torch.from_numpy(w[name].astype(np.float64))  # noqa: E731
    b = torch.from_numpy(boards.astype(np.int64))
    n, d, t, s0 = b.shape[0], arch.d_model, arch.tokens, arch.square_token_start
    bits = torch.stack([(b[:, 64] >> k) & 1 for k in range(4)], -1).double()
    state = T("state_embed") + bits @ T("castling_proj.weight").T + T("castling_proj.bias") \
        + T("en_passant_embed.weight")[b[:, 65].clamp(max=8)]
    squares = T("piece_embed.weight")[b[:, :64]] + T("square_embed.weight")[None]
    x = torch.zeros(n, t, d, dtype=torch.float64)
    x[:, 0] = state
    x[:, s0:s0 + 64] = squares
    ln = lambda v, p: torch.nn.functional.layer_norm(v, (d,), T(p + ".weight"), T(p + ".bias"), arch.layer_norm_eps)  # noqa: E731
    gelu = (lambda v: torch.nn.functional.gelu(v)) if arch.gelu == 0 else \
        (lambda v: torch.nn.functional.gelu(v, approximate="tanh"))
    H, hd = arch.n_heads, arch.head_dim
    for i in range(arch.n_layers):
        p = f"encoder.layers.{i}."
        h = ln(x, p + "norm1")
        qkv = h @ T(p + "self_attn.in_proj_weight").T + T(p + "self_attn.in_proj_bias")
        q, k, v = (qkv[..., j * d:(j + 1) * d].reshape(n, t, H, hd).transpose(1, 2) for j in range(3))
        a = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(hd), -1) @ v
        a = a.transpose(1, 2).reshape(n, t, d)
        x = x + a @ T(p + "self_attn.out_proj.weight").T + T(p + "self_attn.out_proj.bias")
        h = ln(x, p + "norm2")
        f = gelu(h @ T(p + "linear1.weight").T + T(p + "linear1.bias"))
        x = x + f @ T(p + "linear2.weight").T + T(p + "linear2.bias")
    h = ln(x, "final_norm")
    sq = ln(h[:, s0:s0 + 64], "policy_head.norm")
    policy = (sq @ T("policy_head.proj.weight").T + T("policy_head.proj.bias")).reshape(n, 64 * 73)
    vh = torch.nn.functional.gelu(ln(h[:, 0], "value_head.norm") @ T("value_head.ff.0.weight").T
                                  + T("value_head.ff.0.bias"))
    value = vh @ T("value_head.ff.2.weight").T + T("value_head.ff.2.bias")
    return policy.numpy(), value.numpy()


def priors_from_logits(policy: np.ndarray, legal: np.ndarray) -> np.ndarray:
    out = np.zeros(legal.shape, dtype=np.float64)
    for p in range(legal.shape[0]):
        acts = legal[p][legal[p] >= 0]
        z = policy[p, acts].astype(np.float64)
        e = np.exp(z - z.max())
        out[p, :len(acts)] = e / e.sum()
    return out


def softmax(z: np.ndarray) -> np.ndarray:
    e = np.exp(z - z.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)
