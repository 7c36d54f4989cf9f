"""Pins the MoE oracle (oracle/moe_ref.py) to the reference's golden MoE decoder
(src/clef/model/tests.rs:81-109 against src/clef/model/mini_expected.in,
committed as tests/golden/clef_mini_expected.json) and to its routing
tie-break test (src/clef/model/tests.rs:147-160). CPU only."""
import json
from pathlib import Path

import numpy as np

from oracle import moe_ref

GOLDEN = Path(__file__).resolve().parent / "golden" / "clef_mini_expected.json"


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def test_mini_decoder_matches_reference_golden():
    doc = json.loads(GOLDEN.read_text())
    cfg = doc["config"]
    x = moe_ref.val(cfg["tokens"] * cfg["hidden"], 99.0, 1.0).reshape(cfg["tokens"], cfg["hidden"])
    for l, want in enumerate(doc["layers"]):
        y, ids, w, _ = moe_ref.layer_forward(x, moe_ref.mini_layer_weights(cfg, l), cfg)
        assert ids.ravel().tolist() == want["ids"], (l, ids.ravel().tolist())
        assert np.abs(w.ravel() - np.asarray(want["weights"])).max() < 1e-5
        hw = np.asarray(want["hidden"], np.float64)
        assert np.abs(y.ravel() - hw).max() / np.abs(hw).max() < 2e-6
        assert cosine(y, hw) > 0.999999
        x = np.asarray(want["hidden"], np.float32).reshape(cfg["tokens"], cfg["hidden"])


def test_routing_breaks_ties_to_the_lower_id_and_renormalizes():
    ids, w, m = moe_ref.route(np.array([[1.0, 1.0, 1.0, 0.0]]), 2)
    assert ids.tolist() == [[0, 1]]
    assert abs(w[0, 0] - 0.5) < 1e-6 and abs(w[0, 1] - 0.5) < 1e-6
    assert abs(m[0]) < 1e-7
    ids, w, _ = moe_ref.route(np.array([[0.0, 3.0, 1.0, 2.0]]), 2)
    assert ids.tolist() == [[1, 3]]
    p1 = np.exp(3.0) / (np.exp(3.0) + np.exp(2.0))
    assert abs(w[0, 0] - p1) < 1e-6
