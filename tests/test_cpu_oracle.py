"""The CPU oracle (oracle/qwen_oracle.c, a plain-C restatement of the reference's decode
and prefill arithmetic) against the golden vectors that the reference engine itself
produced (tests/golden/make_golden.py: the reference's src/*.cpp built into
oracle/_ref/libqwen_ref.so). This pins the oracle that every GPU parity test uses.

Bars: step / prefill logits rel_l2 <= 1e-5 (same fp32 arithmetic, different summation
order and vectorisation), greedy tokens identical, top-64 logits of the last prompt
position identical in index and within 1e-4 in value."""
import os

import numpy as np
import pytest

from conftest import model_dir, rel_l2

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-5


def golden(name):
    return np.load(os.path.join(GOLDEN, f"{name.replace('-', '_')}.npz"))


@pytest.mark.parametrize("shape", ["tiny", "tiny-rep", "tiny-untied"])
def test_oracle_step_and_greedy_match_reference(pkg, oracle, shape):
    g = golden(shape)
    d = model_dir(pkg, shape)
    prompt = g["prompt"]
    m = oracle.OracleModel(d, len(prompt) + len(g["greedy"]) + 2)
    for i, t in enumerate(prompt):
        lg = m.step(int(t))
        assert rel_l2(lg, g["step_logits"][i]) < TOL, f"step {i}"
    assert m.generate_greedy(prompt, len(g["greedy"])).tolist() == g["greedy"].tolist()


def test_oracle_prefill_matches_reference(pkg, oracle):
    g = golden("tiny")
    d = model_dir(pkg, "tiny")
    m = oracle.OracleModel(d, 64)
    got = m.prefill(g["prompt"])
    assert got.shape == g["prefill_logits"].shape
    assert rel_l2(got, g["prefill_logits"]) < TOL
    # QwenForward::prefill and stepping agree (the reference's two paths)
    assert rel_l2(g["prefill_logits"], g["step_logits"]) < TOL


def _check_large(pkg, oracle, shape, fname):
    g = np.load(os.path.join(GOLDEN, fname))
    d = model_dir(pkg, shape)
    prompt = g["prompt"]
    m = oracle.OracleModel(d, len(prompt) + len(g["greedy"]) + 2)
    last = None
    for t in prompt:
        last = m.step(int(t))
    idx = np.argsort(-last, kind="stable")[:64]
    assert idx.tolist() == g["last_top_idx"].tolist()
    np.testing.assert_allclose(last[idx], g["last_top_val"], rtol=1e-4, atol=1e-5)
    assert abs(np.linalg.norm(last.astype(np.float64)) - float(g["last_norm"])) < 1e-4 * float(g["last_norm"])
    assert m.generate_greedy(prompt, len(g["greedy"])).tolist() == g["greedy"].tolist()


def test_oracle_matches_reference_small_0_8b_widths(pkg, oracle):
    _check_large(pkg, oracle, "small-0.8b-widths", "small_0_8b_widths.npz")


@pytest.mark.slow
def test_oracle_matches_reference_full_0_8b(pkg, oracle):
    """The 24-layer 0.8B-shaped model of the benchmark (writes a 1.6 GB checkpoint)."""
    _check_large(pkg, oracle, "qwen3.5-0.8b-shaped", "qwen35_0_8b.npz")


def test_reference_engine_reproduces_its_golden_vectors(pkg, oracle):
    """When the reference's own sources are present (this build host), re-run them: the
    golden vectors are reproducible from the reference, not hand-edited."""
    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built on this host")
    g = golden("tiny")
    d = model_dir(pkg, "tiny")
    ref = oracle.RefModel(d, 64)
    for i, t in enumerate(g["prompt"]):
        assert rel_l2(ref.step(int(t)), g["step_logits"][i]) < 1e-6
    assert ref.generate_greedy(g["prompt"], len(g["greedy"])).tolist() == g["greedy"].tolist()
