"""Generate the committed fixtures of this test-suite from the CPU oracle (the C restatement
of the reference's CPU backend, src/net/cpu.rs):

* ``tests/golden/nano_b64.npz`` -- configuration 0: the `nano` net, weights N(0, 0.02) with
  seed 0 (LayerNorm gamma 1 / beta 0, zero biases), 64 positions from uniform-random legal
  playouts of 0-80 plies (seed 1); boards, legal actions, priors and WDL.
* ``marina_b200/cards/{nano,small}.json`` -- model cards of the same random-init nets with
  the FP8 calibration (`encoder.fp8.activation_amax`, src/net/model.rs:87-95): per layer the
  largest |value| of norm1 out, attention out, norm2 out and GELU out over 512 calibration
  positions (seed 2), measured on the e4m3-quantised weights the FP8 path computes with.

Run: ``python -m tests.golden.make_golden``.
"""

from __future__ import annotations

import os
from pathlib import Path

import numpy as np

import oracle
from marina_b200 import chess, model, weights

ROOT = Path(__file__).resolve().parents[2]
THREADS = os.cpu_count() or 1


def golden_nano() -> None:
    arch = model.nano()
    w = weights.random_init(arch, seed=0)
    boards, legal, counts, fens = chess.random_positions(1, 64, 0, 80, fens=True)
    net = oracle.OracleNetwork(arch, w, threads=THREADS)
    priors, wdl = net.evaluate(boards, legal)
    policy, value = net.logits(boards)
    np.savez_compressed(ROOT / "tests/golden/nano_b64.npz", boards=boards, legal=legal, counts=counts,
                        fens=np.array(fens), priors=priors, wdl=wdl, value_logits=value,
                        legal_logits=np.where(legal >= 0, np.take_along_axis(policy, np.maximum(legal, 0), 1), 0))


def card(name: str) -> None:
    arch = getattr(model, name)()
    w = weights.fp8_weights(weights.random_init(arch, seed=0))
    boards, _, _, _ = chess.random_positions(2, 512, 0, 80)
    arch.fp8_amax = [[float(f"{v:.6g}") for v in row] for row in oracle.calibrate(arch, w, boards, THREADS)]
    arch.checkpoint = {"init": "N(0, 0.02) seed 0, LayerNorm gamma 1 beta 0, zero biases",
                       "fp8_calibration": "512 random-playout positions, seed 2"}
    (ROOT / f"marina_b200/cards/{name}.json").write_text(arch.to_json() + "\n")


if __name__ == "__main__":
    golden_nano()
    card("nano")
    card("small")
    print("written")
