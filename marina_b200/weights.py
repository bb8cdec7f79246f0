"""Network parameters under the reference's PyTorch names (src/net/weights.rs:94-134), with
seeded random initialisation for the benchmark configurations, the per-matrix e4m3
quantisation of the reference's FP8 path, and safetensors I/O."""

from __future__ import annotations

import json
import struct
from ctypes import POINTER, c_float

import numpy as np

from .model import POLICY_PLANES, WDL_OUTPUTS, Architecture

PIECE_VOCAB = 13
EN_PASSANT_VOCAB = 9
CASTLING_BITS = 4
E4M3_MAX = 448.0

# The four Linear layers of an encoder layer that run on the tensor cores (and are the ones
# the FP8 path quantises, src/net/cuda/mod.rs:406-416).
LAYER_LINEARS = ("self_attn.in_proj_weight", "self_attn.out_proj.weight", "linear1.weight", "linear2.weight")


class WeightsError(ValueError):
    """A safetensors file that does not fit the architecture (src/net/weights.rs:15-29)."""


def tensor_specs(arch: Architecture) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) of every parameter, in a fixed order; kind is one of "weight",
    "bias", "norm_weight", "norm_bias"."""
    d, ff = arch.d_model, arch.d_ff
    specs: list[tuple[str, tuple[int, ...], str]] = [
        ("piece_embed.weight", (PIECE_VOCAB, d), "weight"),
        ("square_embed.weight", (64, d), "weight"),
        ("state_embed", (d,), "weight"),
        ("castling_proj.weight", (d, CASTLING_BITS), "weight"),
        ("castling_proj.bias", (d,), "bias"),
        ("en_passant_embed.weight", (EN_PASSANT_VOCAB, d), "weight"),
    ]
    for i in range(arch.n_layers):
        p = f"encoder.layers.{i}."
        specs += [
            (p + "norm1.weight", (d,), "norm_weight"), (p + "norm1.bias", (d,), "norm_bias"),
            (p + "self_attn.in_proj_weight", (3 * d, d), "weight"), (p + "self_attn.in_proj_bias", (3 * d,), "bias"),
            (p + "self_attn.out_proj.weight", (d, d), "weight"), (p + "self_attn.out_proj.bias", (d,), "bias"),
            (p + "norm2.weight", (d,), "norm_weight"), (p + "norm2.bias", (d,), "norm_bias"),
            (p + "linear1.weight", (ff, d), "weight"), (p + "linear1.bias", (ff,), "bias"),
            (p + "linear2.weight", (d, ff), "weight"), (p + "linear2.bias", (d,), "bias"),
        ]
    specs += [
        ("final_norm.weight", (d,), "norm_weight"), ("final_norm.bias", (d,), "norm_bias"),
        ("policy_head.norm.weight", (d,), "norm_weight"), ("policy_head.norm.bias", (d,), "norm_bias"),
        ("policy_head.proj.weight", (POLICY_PLANES, d), "weight"), ("policy_head.proj.bias", (POLICY_PLANES,), "bias"),
        ("value_head.norm.weight", (d,), "norm_weight"), ("value_head.norm.bias", (d,), "norm_bias"),
        ("value_head.ff.0.weight", (d, d), "weight"), ("value_head.ff.0.bias", (d,), "bias"),
        ("value_head.ff.2.weight", (WDL_OUTPUTS, d), "weight"), ("value_head.ff.2.bias", (WDL_OUTPUTS,), "bias"),
    ]
    return specs


class Weights:
    """fp32 tensors by name, C-contiguous."""

    def __init__(self, arch: Architecture, tensors: dict[str, np.ndarray]):
        self.arch = arch
        self.tensors: dict[str, np.ndarray] = {}
        for name, shape, _ in tensor_specs(arch):
            if name not in tensors:
                raise WeightsError(f"tensor {name} is missing")
            t = np.ascontiguousarray(tensors[name], dtype=np.float32)
            if t.shape != shape:
                raise WeightsError(f"tensor {name} has shape {list(t.shape)}, expected {list(shape)}")
            self.tensors[name] = t

    def __getitem__(self, name: str) -> np.ndarray:
        return self.tensors[name]

    def copy(self) -> "Weights":
        return Weights(self.arch, {k: v.copy() for k, v in self.tensors.items()})

    def ptr(self, name: str):
        return self.tensors[name].ctypes.data_as(POINTER(c_float))

    # ---- safetensors (the format `Weights::from_bytes` reads) -----------------------------
    def to_safetensors(self, dtype: str = "F32") -> bytes:
        """The tensors as a safetensors file in `dtype` ("F32", "F16" or "BF16", rounded to nearest
        even), the three element types `Weights::from_bytes` reads."""
        header, offset, blobs = {}, 0, []
        for name, _, _ in tensor_specs(self.arch):
            t = self.tensors[name]
            if dtype == "F32":
                data = t.astype("<f4").tobytes()
            elif dtype == "F16":
                data = t.astype("<f2").tobytes()
            elif dtype == "BF16":
                bits = t.astype("<f4").view("<u4").astype(np.uint64)
                data = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype("<u2").tobytes()
            else:
                raise WeightsError(f"cannot write dtype {dtype}")
            header[name] = {"dtype": dtype, "shape": list(t.shape), "data_offsets": [offset, offset + len(data)]}
            offset += len(data)
            blobs.append(data)
        head = json.dumps(header, separators=(",", ":")).encode()
        head += b" " * (-len(head) % 8)
        return struct.pack("<Q", len(head)) + head + b"".join(blobs)

    @classmethod
    def from_safetensors(cls, blob: bytes, arch: Architecture) -> "Weights":
        """src/net/weights.rs:94-135, 191-221: F32, F16 and BF16 are read."""
        if len(blob) < 8:
            raise WeightsError("model.safetensors is not valid: too short")
        (n,) = struct.unpack("<Q", blob[:8])
        if 8 + n > len(blob):
            raise WeightsError("model.safetensors is not valid: header exceeds the file")
        try:
            header = json.loads(blob[8:8 + n])
        except json.JSONDecodeError as e:
            raise WeightsError(f"model.safetensors is not valid: {e}") from e
        data = memoryview(blob)[8 + n:]
        tensors = {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            lo, hi = info["data_offsets"]
            raw = np.frombuffer(data[lo:hi], dtype=np.uint8)
            dtype = info["dtype"]
            if dtype == "F32":
                arr = raw.view("<f4").astype(np.float32)
            elif dtype == "F16":
                arr = raw.view("<f2").astype(np.float32)
            elif dtype == "BF16":
                arr = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
            else:
                raise WeightsError(f"tensor {name} has dtype {dtype}; only F32, F16 and BF16 are read")
            tensors[name] = arr.reshape(info["shape"])
        return cls(arch, tensors)


# Largest files read from a network directory (src/net/mod.rs:62-65).
MAX_MODEL_JSON_BYTES = 16 << 20
MAX_SAFETENSORS_BYTES = 4 << 30


def _read_bounded(path, limit: int) -> bytes:
    """A regular file read whole, refusing FIFOs / devices and anything larger than `limit`
    (src/net/mod.rs:67-91)."""
    import os
    import stat

    st = os.stat(path)
    if not stat.S_ISREG(st.st_mode):
        raise WeightsError(f"{path} is not a regular file")
    if st.st_size > limit:
        raise WeightsError(f"{path} is {st.st_size} bytes; at most {limit} are read")
    with open(path, "rb") as f:
        return f.read()


def parse_dir(path) -> tuple[Architecture, "Weights"]:
    """A network directory: `model.json` (the card) next to `model.safetensors` (the parameters
    in F32, F16 or BF16), parsed with the reference's validation (`net::parse`,
    src/net/mod.rs:118-160, model.rs:112-182, weights.rs:94-134)."""
    from pathlib import Path

    d = Path(path)
    card = _read_bounded(d / "model.json", MAX_MODEL_JSON_BYTES)
    try:
        text = card.decode("utf-8")
    except UnicodeDecodeError as e:
        raise WeightsError(f"{d / 'model.json'}: {e}") from e
    arch = Architecture.from_json(text)
    return arch, Weights.from_safetensors(_read_bounded(d / "model.safetensors", MAX_SAFETENSORS_BYTES), arch)


def write_dir(path, arch: Architecture, w: "Weights", dtype: str = "F32") -> None:
    """Write `model.json` and `model.safetensors` (in `dtype`) into directory `path`."""
    from pathlib import Path

    d = Path(path)
    d.mkdir(parents=True, exist_ok=True)
    (d / "model.json").write_text(arch.to_json())
    (d / "model.safetensors").write_bytes(w.to_safetensors(dtype))


def random_init(arch: Architecture, seed: int = 0, std: float = 0.02, bias_std: float = 0.0,
                norm_std: float = 0.0) -> Weights:
    """Weights and embeddings N(0, std), biases N(0, bias_std) (zero by default), LayerNorm
    gamma 1 / beta 0 (plus N(0, norm_std)); tensors drawn in `tensor_specs` order from one
    numpy PCG64 stream seeded with `seed`."""
    rng = np.random.Generator(np.random.PCG64(seed))
    tensors = {}
    for name, shape, kind in tensor_specs(arch):
        if kind == "weight":
            t = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        elif kind == "bias":
            t = rng.standard_normal(shape, dtype=np.float32) * np.float32(bias_std) if bias_std else np.zeros(shape, np.float32)
        elif kind == "norm_weight":
            t = np.ones(shape, np.float32)
            if norm_std:
                t += rng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
        else:
            t = rng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std) if norm_std else np.zeros(shape, np.float32)
        tensors[name] = t
    return Weights(arch, tensors)


# ---- e4m3 ------------------------------------------------------------------------------
def e4m3_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest e4m3 value (ties to even), saturating at +-448:
    3 mantissa bits, exponents down to 2^-6, subnormal step 2^-9."""
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x), np.float32(E4M3_MAX))
    _, ex = np.frexp(a)
    e = np.maximum(ex.astype(np.int32) - 1, -6)
    step = np.ldexp(np.float32(1.0), e - 3).astype(np.float32)
    q = (np.rint(a / step) * step).astype(np.float32)
    q = np.minimum(q, np.float32(E4M3_MAX))
    return np.copysign(q, x).astype(np.float32)


def fp8_quantize(w: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """Per-matrix e4m3 quantisation as the reference's FP8 path applies it at load
    (src/net/cuda/mod.rs:378-381, kernels.cu:396-401): scale = max(amax / 448, FLT_MIN),
    code = e4m3(w * (1 / scale)). Returns (code values as float32, scale); the dequantised
    weight is code * scale, exactly representable in float32."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.float32(np.max(np.abs(w))) if w.size else np.float32(0)
    scale = np.float32(max(amax / np.float32(E4M3_MAX), np.float32(np.finfo(np.float32).tiny)))
    inv = np.float32(1.0) / scale
    codes = e4m3_round((w * inv).astype(np.float32))
    return codes, scale


def fp8_weights(w: Weights) -> Weights:
    """The network the FP8 path computes with: every encoder Linear weight replaced by its
    dequantised e4m3 quantisation (code * scale); everything else unchanged."""
    out = w.copy()
    for i in range(w.arch.n_layers):
        for name in LAYER_LINEARS:
            key = f"encoder.layers.{i}.{name}"
            codes, scale = fp8_quantize(w[key])
            out.tensors[key] = (codes * scale).astype(np.float32)
    return out
