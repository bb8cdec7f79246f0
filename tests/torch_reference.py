"""Independent PyTorch implementations of the network, built from the architecture's definition
(exact erf GELU, torch softmax/LayerNorm), not from the oracle's code: a float64 forward used to
cross-check the C oracle's restatement of the reference's CPU backend, and a float32 forward
that rounds the four GEMM inputs of every layer as a given precision does (bf16, or e4m3 at one
of several scale granularities), used to study what each precision costs."""

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


def e4m3_round(x: torch.Tensor) -> torch.Tensor:
    """Round to the nearest e4m3 value (saturating at +-448), as float32."""
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).to(torch.float32)


def quantise(x: torch.Tensor, mode: str | None, amax: float) -> torch.Tensor:
    """One GEMM input as a quantised precision would see it (dequantised back to float32):
    None = float32; "bf16"; "tensor" = e4m3 with the static per-tensor scale amax * 1.25 / 448 of
    the reference's FP8 path (src/net/cuda/mod.rs:83-90, 454-466); "row" = e4m3 with a dynamic
    scale per row (row amax / 448); "mx32" = e4m3 with one power-of-two scale per 32 consecutive
    elements of the row (the OCP MX block scaling B200's block-scaled MMA reads); "nv16" = e4m3
    with an exact (float32) scale per 16 elements (block amax / 448); "x2" = two e4m3 terms with the
    static per-tensor scale s, hi = e4m3(x / s) and lo = e4m3(x / s - hi), taken as (hi + lo) * s
    (the fp8x2 precision)."""
    if mode is None:
        return x
    if mode == "bf16":
        return x.to(torch.bfloat16).to(torch.float32)
    if mode == "x2":
        s = amax * 1.25 / 448.0
        v = x / s
        hi = e4m3_round(v)
        return (hi + (v - hi).to(torch.float8_e4m3fn).to(torch.float32)) * s
    if mode == "tensor":
        s = amax * 1.25 / 448.0
        return e4m3_round(x / s) * s
    if mode == "row":
        s = (x.abs().amax(-1, keepdim=True) / 448.0).clamp_min(1e-30)
        return e4m3_round(x / s) * s
    block = {"mx32": 32, "nv16": 16}[mode]
    xb = x.reshape(*x.shape[:-1], x.shape[-1] // block, block)
    a = xb.abs().amax(-1, keepdim=True).clamp_min(1e-30)
    s = torch.exp2(torch.floor(torch.log2(a)) - 8) if mode == "mx32" else a / 448.0
    return (e4m3_round(xb / s) * s).reshape(x.shape)


def activation_amax(arch, w, boards: np.ndarray, device="cpu") -> list[list[float]]:
    """Per layer the largest |value| at the four GEMM inputs (norm1 out, attention out, norm2 out,
    GELU out) of the float32 forward on `boards`: a card's FP8 calibration
    (`encoder.fp8.activation_amax`, src/net/model.rs:87-95) for a network built in a test."""
    rows: list[list[float]] = []
    forward_quantised(arch, w, boards, {}, device=device, record=rows)
    return rows


def forward_quantised(arch, w, boards: np.ndarray, sites: dict, device="cpu", resid16: bool = True,
                      record: list | None = None):
    """Policy logits [n, 4672] and value logits [n, 3] in float32 with the four GEMM inputs of every
    layer quantised as `sites` says ({"n1": norm1 out, "at": attention out, "n2": norm2 out, "ge":
    GELU out} -> a `quantise` mode; missing sites stay float32) and, with `resid16`, the residual
    stream rounded to f16 after every update as the GPU keeps it. Weights are used as given (pass
    e4m3-quantised weights for the FP8 precisions). A simulation of the arithmetic of each
    precision, for the precision study in tests/test_precision.py and the GPU tests. With
    `record`, appends each layer's four site maxima (before quantisation) to it."""
    dev = torch.device(device)
    T = lambda name: torch.from_numpy(np.ascontiguousarray(w[name], dtype=np.float32)).to(dev)  # noqa: E731
    b = torch.from_numpy(boards.astype(np.int64)).to(dev)
    n, d, t, s0 = b.shape[0], arch.d_model, arch.tokens, arch.square_token_start
    amax = arch.fp8_amax
    f16 = (lambda v: v.to(torch.float16).to(torch.float32)) if resid16 else (lambda v: v)  # noqa: E731
    bits = torch.stack([(b[:, 64] >> k) & 1 for k in range(4)], -1).float()
    state = T("state_embed") + bits @ T("castling_proj.weight").T + T("castling_proj.bias") \
        + T("en_passant_embed.weight")[b[:, 65].clamp(max=8)]
    x = torch.zeros(n, t, d, device=dev)
    x[:, 0] = state
    x[:, s0:s0 + 64] = T("piece_embed.weight")[b[:, :64]] + T("square_embed.weight")[None]
    x = f16(x)
    ln = lambda v, p: torch.nn.functional.layer_norm(v, (d,), T(p + ".weight"), T(p + ".bias"), arch.layer_norm_eps)  # noqa: E731
    gelu = (lambda v: torch.nn.functional.gelu(v)) if arch.gelu == 0 else \
        (lambda v: torch.nn.functional.gelu(v, approximate="tanh"))
    H, hd = arch.n_heads, arch.head_dim
    for i in range(arch.n_layers):
        p = f"encoder.layers.{i}."
        am = amax[i] if amax is not None else [1.0] * 4
        seen = []
        site = lambda v, key, j: (seen.append(float(v.abs().max())), quantise(v, sites.get(key), am[j]))[1]  # noqa: E731
        h = site(ln(x, p + "norm1"), "n1", 0)
        qkv = h @ T(p + "self_attn.in_proj_weight").T + T(p + "self_attn.in_proj_bias")
        q, k, v = (qkv[..., j * d:(j + 1) * d].reshape(n, t, H, hd).transpose(1, 2) for j in range(3))
        a = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(hd), -1) @ v
        a = site(a.transpose(1, 2).reshape(n, t, d), "at", 1)
        x = f16(x + a @ T(p + "self_attn.out_proj.weight").T + T(p + "self_attn.out_proj.bias"))
        h = site(ln(x, p + "norm2"), "n2", 2)
        f = site(gelu(h @ T(p + "linear1.weight").T + T(p + "linear1.bias")), "ge", 3)
        x = f16(x + f @ T(p + "linear2.weight").T + T(p + "linear2.bias"))
        if record is not None:
            record.append(seen)
    h = ln(x, "final_norm")
    sq = ln(h[:, s0:s0 + 64], "policy_head.norm")
    policy = (sq @ T("policy_head.proj.weight").T + T("policy_head.proj.bias")).reshape(n, 64 * 73)
    vh = torch.nn.functional.gelu(ln(h[:, 0], "value_head.norm") @ T("value_head.ff.0.weight").T
                                  + T("value_head.ff.0.bias"))
    value = vh @ T("value_head.ff.2.weight").T + T("value_head.ff.2.bias")
    return policy.double().cpu().numpy(), value.double().cpu().numpy()


def agreement(priors: np.ndarray, ref_priors: np.ndarray, counts, tie: float = 2e-4) -> tuple[float, float]:
    """(tie-aware, raw) argmax agreement of `priors` with `ref_priors` over the legal slots: a
    position disagrees tie-aware only when the move ranked first has a reference prior more than
    `tie` below the reference's best."""
    raw = np.mean([np.argmax(priors[p, :c]) == np.argmax(ref_priors[p, :c]) for p, c in enumerate(counts)])
    tied = np.mean([ref_priors[p, np.argmax(priors[p, :c])] >= ref_priors[p, :c].max() - tie
                    for p, c in enumerate(counts)])
    return float(tied), float(raw)
