"""The load path on the GPU: a network directory (`model.json` + `model.safetensors`, the files
the reference's `net::parse` reads, src/net/mod.rs:118-160) written in F32, F16 and BF16, parsed
with the reference's validation (src/net/model.rs:112-182, src/net/weights.rs:94-134, 191-221),
loaded into the evaluator through `mrn_create` and checked against the oracle on the weights as
read. The `small` card (with its FP8 calibration) in the default precision, and `nano` in bf16."""

import numpy as np
import pytest

import oracle
from marina_b200 import chess, model, weights
from marina_b200.network import B200Network

pytestmark = pytest.mark.gpu

WDL_TOL, PRIOR_TOL, KL_TOL, ARGMAX_MIN, TIE = 2e-2, 3e-2, 1e-2, 0.99, 2e-4


def _card(name):
    from pathlib import Path

    return model.Architecture.from_json((Path(model.__file__).parent / "cards" / f"{name}.json").read_text())


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("net,precision", [("small", "fp8w"), ("nano", "bf16")])
def test_directory_loads_and_matches_the_oracle(tmp_path, dtype, net, precision):
    arch = _card(net)
    weights.write_dir(tmp_path, arch, weights.random_init(arch, seed=0, bias_std=0.02), dtype)
    arch2, w = weights.parse_dir(tmp_path)
    assert arch2.fp8_amax == arch.fp8_amax and arch2.d_model == arch.d_model
    boards, legal, counts, _ = chess.random_positions(31, 128, 0, 80)
    ev = B200Network(arch2, w, device=0, max_batch=128, precision=precision)
    assert str(arch.d_model) in ev.describe()
    priors, wdl = ev.evaluate_packed(boards, legal)
    ref_w = weights.fp8_weights(w) if precision != "bf16" else w
    ref_p, ref_v = oracle.OracleNetwork(arch2, ref_w, threads=16).evaluate(boards, legal)
    prior = max(float(np.abs(priors[p, :c] - ref_p[p, :c]).max()) for p, c in enumerate(counts))
    kl = max(float(np.sum(ref_p[p, :c] * (np.log(np.maximum(ref_p[p, :c], 1e-30))
                                          - np.log(np.maximum(priors[p, :c], 1e-30))))) for p, c in enumerate(counts))
    agree = np.mean([ref_p[p, np.argmax(priors[p, :c])] >= ref_p[p, :c].max() - TIE for p, c in enumerate(counts)])
    print(dtype, net, precision, prior, float(np.abs(wdl - ref_v).max()), kl, agree)
    assert prior <= PRIOR_TOL and float(np.abs(wdl - ref_v).max()) <= WDL_TOL and kl <= KL_TOL
    assert agree >= ARGMAX_MIN
    ev.close()
