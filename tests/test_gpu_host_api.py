"""The C++ drop-in API on the GPU: a caller compiled against host/include (the
reference's QwenModel / QwenForward interface, include/qwen_model.h:21-32 and
include/qwen_forward.h:18-25) gives the same tokens and logits as the C ABI, and the
reference's own greedy tokens."""
import json
import os

import numpy as np
import pytest

import host_api
from conftest import model_dir, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,kv_dtype", [("tiny", 0), ("tiny-untied", 1), ("small-0.8b-widths", 0)])
def test_qwen_model_cpp_matches_c_abi_and_oracle(pkg, oracle, shape, kv_dtype):
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    prompt = pkg.synth.random_prompt(s.vocab_size, 7, seed=21)
    n_new = 12
    p = host_api.run("gen", d, 64, n_new, kv_dtype, 0, *prompt.tolist())
    assert p.returncode == 0, p.stderr
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r["ok"] and r["position"] == len(prompt) and r["final_position"] == len(prompt) + n_new
    m = pkg.abi.Model(d, max_context=64, kv_dtype=kv_dtype)
    am = []
    for t in prompt:
        lg, a = m.step(int(t))
        am.append(a)
    assert r["step_argmax"] == am
    assert abs(r["last_norm"] - float(np.linalg.norm(lg.astype(np.float64)))) < 1e-5 * r["last_norm"]
    assert r["greedy"] == m.generate_greedy(prompt, n_new).tolist()
    m.close()
    if kv_dtype == 0:  # the reference's fp32 KV cache: its greedy tokens exactly
        assert r["greedy"] == oracle.OracleModel(d, 64).generate_greedy(prompt, n_new).tolist()


def test_qwen_forward_cpp_matches_c_abi(pkg, oracle, tmp_path):
    d = model_dir(pkg, "tiny")
    s = pkg.synth.SHAPES["tiny"]
    ids = pkg.synth.random_prompt(s.vocab_size, 20, seed=4)
    out = str(tmp_path / "fwd.bin")
    p = host_api.run("fwd", d, out, *ids.tolist())
    assert p.returncode == 0, p.stderr
    got = np.fromfile(out, np.float32).reshape(len(ids), s.vocab_size)
    m = pkg.abi.Model(d, max_context=4096)
    assert rel_l2(got, m.forward_logits(ids)) < 1e-6
    assert rel_l2(got, oracle.OracleModel(d, 64).prefill(ids)) < 2e-3
    m.close()
