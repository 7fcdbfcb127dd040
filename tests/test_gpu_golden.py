"""Parity on the benchmark configurations themselves, against golden vectors that the
reference engine produced (tests/golden/make_golden.py: oracle/_ref is the reference's
own src/*.cpp, compiled from the reference tree).

- the full 24-layer 0.8B-shaped model. The north star's bar: the first 64
  greedy tokens identical to the reference's QwenModel::generate_greedy
  (src/qwen_model.cpp:241-255), and the logits after the prompt within rel_l2 2e-3
  (checked on the reference's top-64 entries, the part of the vector the fixture keeps).
- configs[3]'s model: the 24-layer 2B-shaped model (hidden 2048, FFN 6144) with a
  512-token prompt, and the 4-layer 2B-width model (fast check of the H = 2048 paths).
Both the decode path (step / generate_greedy) and the batched prefill (qwc_prefill, which
seeds the decode state) are checked.
"""
import os

import numpy as np
import pytest

from conftest import model_dir, rel_l2

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = [("small-0.8b-widths", "small_0_8b_widths.npz"),
         ("small-2b-widths", "small_2b_widths.npz"),
         ("qwen3.5-0.8b-shaped", "qwen35_0_8b.npz"),
         ("qwen3.5-2b-shaped", "qwen35_2b.npz")]


def load_golden(fname):
    path = os.path.join(GOLDEN, fname)
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {fname} not generated")
    return np.load(path)


def check_top(logits, g):
    """The reference's 64 largest logits: same entries, values within the logit bar."""
    idx, val = g["last_top_idx"], g["last_top_val"]
    assert rel_l2(logits[idx], val) < LOGIT_TOL
    assert int(np.argmax(logits)) == int(idx[0])
    ours = np.argsort(-logits, kind="stable")[:16]
    assert set(ours.tolist()) == set(idx[:16].tolist())
    norm = float(np.linalg.norm(logits.astype(np.float64)))
    assert abs(norm - float(g["last_norm"])) < LOGIT_TOL * float(g["last_norm"])


@pytest.mark.parametrize("shape,fname", CASES)
def test_decode_greedy_matches_reference_golden(pkg, shape, fname):
    g = load_golden(fname)
    prompt, want = g["prompt"], g["greedy"]
    d = model_dir(pkg, shape)
    m = pkg.abi.Model(d, max_context=len(prompt) + len(want) + 8)
    lg = None
    for t in prompt:
        lg, _ = m.step(int(t))
    check_top(lg, g)
    got = m.generate_greedy(prompt, len(want))
    assert got.tolist() == want.tolist()
    m.close()


@pytest.mark.parametrize("shape,fname", CASES)
def test_prefill_then_greedy_matches_reference_golden(pkg, shape, fname):
    g = load_golden(fname)
    prompt, want = g["prompt"], g["greedy"]
    d = model_dir(pkg, shape)
    m = pkg.abi.Model(d, max_context=len(prompt) + len(want) + 8)
    lg = m.prefill(prompt)
    check_top(lg, g)
    # continue greedily from the prefilled state: the same tokens as stepping the prompt
    toks = [int(np.argmax(lg))]
    for _ in range(len(want) - 1):
        _, am = m.step(toks[-1], logits=False)
        toks.append(int(am))
    assert toks == want.tolist()
    m.close()
