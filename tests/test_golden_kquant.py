"""The oracle's dequantisation against the committed known-answer vectors
(tests/golden/kquant_kat.json, made by tests/golden/make_golden.py from an
independent numpy restatement plus hand-worked blocks).  Bit-exact."""
import base64
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = json.load(open(os.path.join(HERE, "golden", "kquant_kat.json")))["cases"]


def _case(c):
    data = np.frombuffer(base64.b64decode(c["data"]), dtype=np.uint8).copy()
    exp = np.frombuffer(base64.b64decode(c["expected_f32"]), dtype="<f4").copy()
    return data, exp


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_dequant_golden(oracle, case):
    data, exp = _case(case)
    out = oracle.dequantize(data, case["type"], case["rows"], case["row_elems"])
    assert bits_equal(out, exp), f"{case['name']}: first mismatch at {np.argmax(out.view(np.uint32) != exp.view(np.uint32))}"


def test_hand_q4k_values():
    """Spot-check the hand-worked block against the values derived by hand."""
    c = [c for c in CASES if c["name"] == "hand_q4_k"][0]
    _, exp = _case(c)
    assert exp[0] == -8 and exp[33] == -15 and exp[255] == 49
