"""The architecture card (``model.json``), as the reference's ``Architecture``
(src/net/model.rs:85-182): parsing with the same validation, plus the two network shapes
the benchmark configurations use."""

from __future__ import annotations

import json
from dataclasses import dataclass, field

FORMAT = "marina-weights"
FORMAT_VERSION = 1
BOARD_TOKENS = 65
POLICY_PLANES = 73
WDL_OUTPUTS = 3
MAX_SQUARE_TOKEN_START = 64

GELU_ERF = 0
GELU_TANH = 1


class ModelError(ValueError):
    """A card the engine cannot use (`ModelError`, src/net/model.rs:25-57)."""


def parse_gelu(text: str) -> int | None:
    """src/net/model.rs:69-83."""
    s = text.strip().lower()
    if not s.startswith("gelu"):
        return None
    if "tanh" in s:
        return GELU_TANH
    if s == "gelu" or "erf" in s or "exact" in s:
        return GELU_ERF
    return None


@dataclass
class Architecture:
    d_model: int
    n_layers: int
    n_heads: int
    d_ff: int
    layer_norm_eps: float = 1e-5
    gelu: int = GELU_ERF
    # Per layer: max |.| of norm1 out, attention out, norm2 out, GELU out (or None).
    fp8_amax: list[list[float]] | None = None
    tokens: int = BOARD_TOKENS
    square_token_start: int = 1
    parameters: int = 0
    checkpoint: dict = field(default_factory=dict)

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def describe(self) -> str:
        """src/net/model.rs:186-203."""
        step = self.checkpoint.get("step") if isinstance(self.checkpoint, dict) else None
        step = f" step {step}" if isinstance(step, int) else ""
        params = f", {self.parameters / 1e6:.2f}M parameters" if self.parameters > 0 else ""
        return f"{self.d_model}x{self.n_layers} ({self.n_heads} heads, d_ff {self.d_ff}{params}{step})"

    def parameter_count(self) -> int:
        d, ff = self.d_model, self.d_ff
        per_layer = 4 * d + (3 * d * d + 3 * d) + (d * d + d) + (ff * d + ff) + (d * ff + d)
        return (13 * d + 64 * d + d + 4 * d + d + 9 * d + self.n_layers * per_layer + 2 * d + 2 * d
                + 73 * d + 73 + 2 * d + d * d + d + 3 * d + 3)

    @classmethod
    def from_json(cls, text: str) -> "Architecture":
        """Parse and validate a card (src/net/model.rs:112-182)."""
        try:
            card = json.loads(text)
        except json.JSONDecodeError as e:
            raise ModelError(f"model.json is not valid: {e}") from e
        try:
            fmt, version = card["format"], card["format_version"]
            model, tokens, encoder = card["model"], card["tokens"], card["encoder"]
            d, layers, heads, ff = (int(model[k]) for k in ("d_model", "n_layers", "n_heads", "d_ff"))
            mode = model["context_mode"]
            eps = float(encoder["layer_norm_eps"])
            activation = encoder["activation"]
            count, start = int(tokens["count"]), int(tokens["square_token_start"])
        except (KeyError, TypeError, ValueError) as e:
            raise ModelError(f"model.json is not valid: missing or malformed field {e}") from e
        if fmt != FORMAT or version != FORMAT_VERSION:
            raise ModelError(f"model.json format is {fmt!r} version {version}; this engine reads {FORMAT!r} "
                             f"version {FORMAT_VERSION}")
        if mode != "board":
            raise ModelError(f"context_mode {mode!r} is not supported by this engine (only \"board\")")
        if d == 0 or heads == 0 or layers == 0 or ff == 0 or not eps > 0:
            raise ModelError("model.json describes a degenerate network (a zero dimension or a non-positive "
                             "layer_norm_eps)")
        if d % heads != 0:
            raise ModelError(f"d_model {d} is not divisible by n_heads {heads}")
        if start < 1 or start > MAX_SQUARE_TOKEN_START or start + 64 != count:
            raise ModelError(f"tokens {count} with square_token_start {start}: board mode needs one or more state "
                             "tokens followed by exactly 64 square tokens")
        gelu = parse_gelu(activation)
        if gelu is None:
            raise ModelError(f"encoder activation {activation!r} is not supported")
        amax = None
        fp8 = encoder.get("fp8")
        if fp8 is not None:
            rows = fp8.get("activation_amax", [])
            ok = len(rows) == layers and all(len(r) == 4 and all(
                isinstance(v, (int, float)) and v > 0 and v != float("inf") for v in r) for r in rows)
            if not ok:
                raise ModelError(f"encoder.fp8.activation_amax must hold four positive maxima for each of the "
                                 f"{layers} layers")
            amax = [[float(v) for v in r] for r in rows]
        return cls(d, layers, heads, ff, eps, gelu, amax, count, start, int(model.get("parameters", 0)),
                   card.get("checkpoint", {}) or {})

    def to_json(self) -> str:
        encoder = {"layers": self.n_layers, "layer_norm_eps": self.layer_norm_eps,
                   "activation": "gelu (exact, erf)" if self.gelu == GELU_ERF else "gelu (tanh approximation)"}
        if self.fp8_amax is not None:
            encoder["fp8"] = {"activation_amax": self.fp8_amax}
        card = {
            "format": FORMAT, "format_version": FORMAT_VERSION,
            "model": {"d_model": self.d_model, "n_layers": self.n_layers, "n_heads": self.n_heads,
                      "d_ff": self.d_ff, "context_mode": "board", "parameters": self.parameter_count()},
            "checkpoint": self.checkpoint,
            "tokens": {"count": self.tokens, "state_token_index": 0, "square_token_start": self.square_token_start},
            "encoder": encoder,
        }
        return json.dumps(card, indent=1)


def nano() -> Architecture:
    """The `nano` shape: d_model 192, 6 pre-LN layers, 6 heads of 32, FFN 768."""
    return Architecture(192, 6, 6, 768)


def small() -> Architecture:
    """The `small` shape: d_model 512, 12 layers, 8 heads of 64, FFN 2048."""
    return Architecture(512, 12, 8, 2048)


NETS = {"nano": nano, "small": small}
