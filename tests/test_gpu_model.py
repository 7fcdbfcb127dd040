"""Whole-model parity on the GPU through the C ABI against the CPU oracle (the plain-C
restatement of the reference, itself pinned to the reference's own outputs).

Bar (north star): greedy tokens identical; logits rel_l2 <= 2e-3. The decode path keeps
fp32 activations and accumulation over bf16 weights like the reference, so the observed
error is ~1e-6."""
import os

import numpy as np
import pytest

from conftest import model_dir, rel_l2

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3


@pytest.mark.parametrize("shape", ["tiny", "tiny-rep", "tiny-untied", "small-0.8b-widths"])
def test_step_logits_and_greedy(pkg, oracle, shape):
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    prompt = pkg.synth.random_prompt(s.vocab_size, 8, seed=11)
    m = pkg.abi.Model(d, max_context=96)
    orc = oracle.OracleModel(d, 96)
    for i, t in enumerate(prompt):
        lg, am = m.step(int(t))
        ref = orc.step(int(t))
        assert rel_l2(lg, ref) < LOGIT_TOL, f"step {i}"
        assert am == int(np.argmax(lg))
    assert m.position() == len(prompt)
    n_new = 24
    got = m.generate_greedy(prompt, n_new)
    want = orc.generate_greedy(prompt, n_new)
    assert got.tolist() == want.tolist()
    assert m.position() == len(prompt) + n_new
    m.close()


@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_forward_logits_matches_oracle_prefill(pkg, oracle, kv_dtype):
    d = model_dir(pkg, "tiny")
    s = pkg.synth.SHAPES["tiny"]
    ids = pkg.synth.random_prompt(s.vocab_size, 12, seed=5)
    m = pkg.abi.Model(d, max_context=64, kv_dtype=kv_dtype)
    got = m.forward_logits(ids)
    want = oracle.OracleModel(d, 64).prefill(ids)
    assert got.shape == want.shape
    assert rel_l2(got, want) < LOGIT_TOL
    last = m.forward_logits(ids, last_only=True)
    assert rel_l2(last[0], want[-1]) < LOGIT_TOL
    assert m.position() == 0  # stateless
    m.close()


def test_prefill_seeds_decode_state(pkg, oracle):
    d = model_dir(pkg, "tiny-untied")
    s = pkg.synth.SHAPES["tiny-untied"]
    ids = pkg.synth.random_prompt(s.vocab_size, 10, seed=9)
    m = pkg.abi.Model(d, max_context=64)
    lg = m.prefill(ids)
    assert m.position() == len(ids)
    orc = oracle.OracleModel(d, 64)
    for t in ids:
        ref = orc.step(int(t))
    assert rel_l2(lg, ref) < LOGIT_TOL
    nxt, _ = m.step(int(np.argmax(lg)))
    ref = orc.step(int(np.argmax(ref)))
    assert rel_l2(nxt, ref) < LOGIT_TOL
    m.close()


def test_errors_are_reported(pkg):
    d = model_dir(pkg, "tiny")
    m = pkg.abi.Model(d, max_context=4)
    with pytest.raises(pkg.abi.QwcError) as e:
        m.step(10**6)
    assert e.value.code == -1
    for t in range(4):
        m.step(t)
    with pytest.raises(pkg.abi.QwcError) as e:
        m.step(1)
    assert e.value.code == -5
    with pytest.raises(pkg.abi.QwcError) as e:
        m.generate_greedy([1, 2, 3], 2)
    assert e.value.code == -5
    m.close()


def test_measurement_entry_points(pkg, oracle):
    """qwc_profile_step / qwc_trace_step run a real step on the production path: the
    position advances and the following step still matches the oracle."""
    d = model_dir(pkg, "small-0.8b-widths")
    s = pkg.synth.SHAPES["small-0.8b-widths"]
    prompt = pkg.synth.random_prompt(s.vocab_size, 6, seed=3)
    m = pkg.abi.Model(d, max_context=64)
    m.generate_greedy(prompt, 2)
    pos = m.position()
    prof = m.profile_step()
    assert len(prof) >= 1 and all(ms > 0 and b > 0 for _, ms, b in prof)
    kinds = {k for k, _, _ in prof}
    assert kinds == {"decode_step"} or "lm_head" in kinds
    assert m.position() == pos + 1
    if kinds == {"decode_step"}:
        tk, st = m.trace_step()
        assert st.shape[1] == len(tk) and st.shape[2] == 8
        assert tk[-1] == "lm_head"
        # stamps are ordered within every CTA and phase: start <= barrier <= end
        assert (st[:, :, 1] >= st[:, :, 0]).all() and (st[:, :, 3] >= st[:, :, 1]).all()
        assert m.position() == pos + 2
    m.close()


def test_context_planned_from_free_memory(pkg):
    """max_context <= 0: the capacity is planned from the device's free memory with the
    memory equation (capped at the config's native context); decoding is unchanged."""
    d = model_dir(pkg, "tiny")
    s = pkg.synth.SHAPES["tiny"]
    prompt = pkg.synth.random_prompt(s.vocab_size, 6, seed=2)
    m = pkg.abi.Model(d, max_context=0)
    cfg = pkg.abi.load_config(os.path.join(d, "config.json"))
    assert 1024 < m.max_context <= cfg.native_max_context
    ref = pkg.abi.Model(d, max_context=32)
    assert ref.max_context == 32
    for t in prompt:
        a, _ = m.step(int(t))
        b, _ = ref.step(int(t))
        assert np.array_equal(a, b)
    m.close()
    ref.close()


def test_bounded_wait_expiry_returns_device_error_and_recovers(pkg, oracle):
    """One CTA withholds its first grid-barrier arrival (qwc_check_step_timeout): the other
    CTAs' waits run out after 50 ms, the step stops with an error code, the call returns
    QWC_E_DEVICE; after qwc_reset the handle decodes exactly as before."""
    d = model_dir(pkg, "small-0.8b-widths")
    s = pkg.synth.SHAPES["small-0.8b-widths"]
    prompt = pkg.synth.random_prompt(s.vocab_size, 5, seed=8)
    m = pkg.abi.Model(d, max_context=32)
    m.step(int(prompt[0]))
    assert m.check_step_timeout(50) == -7
    m.reset()
    orc = oracle.OracleModel(d, 32)
    for t in prompt:
        lg, _ = m.step(int(t))
        ref = orc.step(int(t))
        assert rel_l2(lg, ref) < LOGIT_TOL
    assert m.generate_greedy(prompt, 6).tolist() == orc.generate_greedy(prompt, 6).tolist()
    m.close()
