"""The load path a trained network comes through: the architecture card (model.json, parsed
and validated like src/net/model.rs:112-182, whose tests are src/net/model.rs:244-343) and the
safetensors weights (src/net/weights.rs:94-135, 191-221; the reference round-trips F16 at
src/net/weights.rs:288-312). CPU only."""

import json
import struct

import numpy as np
import pytest

from marina_b200 import model, weights
from marina_b200.model import GELU_ERF, GELU_TANH, Architecture, ModelError
from marina_b200.weights import Weights, WeightsError


def _card(**edits) -> dict:
    card = json.loads(model.nano().to_json())
    for path, value in edits.items():
        node = card
        keys = path.split("__")
        for k in keys[:-1]:
            node = node[k]
        if value is None:
            del node[keys[-1]]
        else:
            node[keys[-1]] = value
    return card


def _parse(card: dict) -> Architecture:
    return Architecture.from_json(json.dumps(card))


# ---- the card -------------------------------------------------------------------------------

def test_card_round_trip_keeps_every_field():
    for arch in (model.nano(), model.small(), Architecture(128, 2, 4, 256, 1e-6, GELU_TANH, [[1.0, 2.0, 3.0, 4.0]] * 2)):
        back = Architecture.from_json(arch.to_json())
        assert (back.d_model, back.n_layers, back.n_heads, back.d_ff) == (arch.d_model, arch.n_layers, arch.n_heads,
                                                                           arch.d_ff)
        assert back.layer_norm_eps == arch.layer_norm_eps and back.gelu == arch.gelu
        assert back.fp8_amax == arch.fp8_amax
        assert (back.tokens, back.square_token_start) == (65, 1)
        assert back.parameters == arch.parameter_count()


def test_parameter_count_matches_the_tensor_list():
    for arch in (model.nano(), model.small(), Architecture(64, 3, 2, 96)):
        total = sum(int(np.prod(shape)) for _, shape, _ in weights.tensor_specs(arch))
        assert arch.parameter_count() == total


@pytest.mark.parametrize("text,form", [
    ("gelu", GELU_ERF), ("GELU", GELU_ERF), (" gelu (exact, erf) ", GELU_ERF), ("gelu_exact", GELU_ERF),
    ("gelu (tanh approximation)", GELU_TANH), ("GELU_TANH", GELU_TANH),
    ("relu", None), ("gelu_new", None), ("silu", None), ("", None),
])
def test_activation_names(text, form):
    assert model.parse_gelu(text) == form


def test_tanh_card_and_calibration_rows_are_read():
    card = _card(encoder__activation="gelu (tanh approximation)",
                 encoder__fp8={"activation_amax": [[1, 2.5, 3, 4]] * 6})
    arch = _parse(card)
    assert arch.gelu == GELU_TANH and arch.fp8_amax == [[1.0, 2.5, 3.0, 4.0]] * 6


@pytest.mark.parametrize("edits,message", [
    ({"format": "other-weights"}, "format"),
    ({"format_version": 2}, "version 2"),
    ({"model__context_mode": "sequence"}, "context_mode"),
    ({"model__d_model": 0}, "degenerate"),
    ({"model__n_layers": 0}, "degenerate"),
    ({"encoder__layer_norm_eps": 0.0}, "degenerate"),
    ({"model__n_heads": 5}, "not divisible"),
    ({"tokens__count": 64}, "square_token_start"),
    ({"tokens__square_token_start": 0, "tokens__count": 64}, "square_token_start"),
    ({"tokens__square_token_start": 65, "tokens__count": 129}, "square_token_start"),
    ({"encoder__activation": "relu"}, "not supported"),
    ({"encoder__fp8": {"activation_amax": [[1, 2, 3, 4]] * 5}}, "four positive maxima"),
    ({"encoder__fp8": {"activation_amax": [[1, 2, 3]] * 6}}, "four positive maxima"),
    ({"encoder__fp8": {"activation_amax": [[1, 2, 0, 4]] * 6}}, "four positive maxima"),
    ({"encoder__fp8": {"activation_amax": [[1, 2, float("inf"), 4]] * 6}}, "four positive maxima"),
    ({"model__d_ff": None}, "missing or malformed"),
    ({"tokens": None}, "missing or malformed"),
])
def test_invalid_cards_are_refused_with_a_reason(edits, message):
    with pytest.raises(ModelError) as e:
        _parse(_card(**edits))
    assert message in str(e.value)


def test_more_state_tokens_are_accepted():
    arch = _parse(_card(tokens__square_token_start=3, tokens__count=67))
    assert (arch.tokens, arch.square_token_start) == (67, 3)


def test_malformed_json_is_refused():
    with pytest.raises(ModelError) as e:
        Architecture.from_json("{not json")
    assert "not valid" in str(e.value)


def test_describe():
    arch = _parse(_card(checkpoint={"step": 1200}))
    assert arch.describe() == f"192x6 (6 heads, d_ff 768, {arch.parameter_count() / 1e6:.2f}M parameters step 1200)"
    assert model.small().describe() == "512x12 (8 heads, d_ff 2048)"


# ---- safetensors ----------------------------------------------------------------------------

def _blob(tensors: dict, dtype: str) -> bytes:
    """A safetensors file with every tensor stored as `dtype` (F32, F16 or BF16 by truncation)."""
    header, blobs, offset = {"__metadata__": {"format": "pt"}}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, dtype=np.float32)
        if dtype == "F32":
            data = a.astype("<f4").tobytes()
        elif dtype == "F16":
            data = a.astype("<f2").tobytes()
        elif dtype == "BF16":
            data = (a.view(np.uint32) >> 16).astype("<u2").tobytes()
        else:
            data = a.astype("<i1").tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    head = json.dumps(header).encode()
    return struct.pack("<Q", len(head)) + head + b"".join(blobs)


@pytest.fixture(scope="module")
def tiny():
    arch = Architecture(64, 2, 2, 128)
    return arch, weights.random_init(arch, seed=3, bias_std=0.01, norm_std=0.1)


def test_f32_round_trip_is_exact(tiny):
    arch, w = tiny
    back = Weights.from_safetensors(w.to_safetensors(), arch)
    for name, t in w.tensors.items():
        assert np.array_equal(back[name], t), name


def test_f16_and_bf16_files_are_widened_exactly(tiny):
    arch, w = tiny
    f16 = {k: v.astype(np.float16).astype(np.float32) for k, v in w.tensors.items()}
    bf16 = {k: (v.view(np.uint32) & 0xFFFF0000).view(np.float32) for k, v in w.tensors.items()}
    for dtype, expect in (("F16", f16), ("BF16", bf16)):
        back = Weights.from_safetensors(_blob(expect, dtype), arch)
        for name, t in expect.items():
            assert back[name].dtype == np.float32 and np.array_equal(back[name], t), (dtype, name)


def test_weight_file_errors(tiny):
    arch, w = tiny
    missing = {k: v for k, v in w.tensors.items() if k != "final_norm.bias"}
    with pytest.raises(WeightsError, match="final_norm.bias is missing"):
        Weights.from_safetensors(_blob(missing, "F32"), arch)
    reshaped = dict(w.tensors)
    reshaped["policy_head.proj.weight"] = np.zeros((72, 64), np.float32)
    with pytest.raises(WeightsError, match=r"policy_head.proj.weight has shape \[72, 64\], expected \[73, 64\]"):
        Weights.from_safetensors(_blob(reshaped, "F32"), arch)
    with pytest.raises(WeightsError, match="only F32, F16 and BF16"):
        Weights.from_safetensors(_blob({"state_embed": w["state_embed"]}, "I8"), arch)
    with pytest.raises(WeightsError, match="too short"):
        Weights.from_safetensors(b"\x01\x02", arch)
    with pytest.raises(WeightsError, match="header exceeds"):
        Weights.from_safetensors(struct.pack("<Q", 1 << 20) + b"{}", arch)
    with pytest.raises(WeightsError, match="not valid"):
        Weights.from_safetensors(struct.pack("<Q", 4) + b"{no}", arch)


def test_other_architectures_do_not_load(tiny):
    arch, w = tiny
    with pytest.raises(WeightsError):
        Weights.from_safetensors(w.to_safetensors(), Architecture(64, 3, 2, 128))


def test_network_directory_round_trip(tmp_path):
    """write_dir / parse_dir: model.json + model.safetensors in F32 (exact), F16 and BF16 (rounded
    to nearest even, as torch rounds), read back with the card's fields intact."""
    import torch

    arch = model.nano()
    arch.fp8_amax = [[1.0, 2.0, 3.0, 4.0]] * arch.n_layers
    w = weights.random_init(arch, seed=9, bias_std=0.1)
    for dtype, tdt in (("F32", torch.float32), ("F16", torch.float16), ("BF16", torch.bfloat16)):
        d = tmp_path / dtype
        weights.write_dir(d, arch, w, dtype)
        a2, w2 = weights.parse_dir(d)
        assert a2.to_json() == arch.to_json()
        for name in w.tensors:
            want = torch.from_numpy(w[name]).to(tdt).to(torch.float32).numpy()
            assert np.array_equal(w2[name], want), (dtype, name)


def test_network_directory_errors(tmp_path):
    with pytest.raises(FileNotFoundError):
        weights.parse_dir(tmp_path / "missing")
    (tmp_path / "model.json").mkdir()
    with pytest.raises(weights.WeightsError, match="not a regular file"):
        weights.parse_dir(tmp_path)
