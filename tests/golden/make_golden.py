"""Generate the golden fixtures of tests/golden/ from the reference engine itself.

The reference ships no tests, fixtures or golden vectors, so the golden vectors are
produced by running the reference's own code: oracle/_ref/libqwen_ref.so is the
reference's src/*.cpp compiled from the reference tree (oracle/Makefile) behind a C
driver (oracle/ref_harness.cpp). Inputs are the seeded synthetic checkpoints of
synth.py and seeded prompts, so the fixtures stay small: outputs only.

Run from the repository root:  python tests/golden/make_golden.py [--full] [--2b] [--only NAME ...]
--full adds the 24-layer 0.8B-shaped model (about a minute); --2b adds the 24-layer
2B-shaped model with a 512-id prompt (a few minutes on 8 cores); --only regenerates the
named cases alone (config, tiny, tiny-rep, tiny-untied, small-0.8b, small-2b, 0.8b, 2b).
"""
import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402
from oracle import bindings as B  # noqa: E402

synth = __graft_entry__.load_package().synth
CACHE = os.environ.get("QWC_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "qwc_models"))


def mdir(name, seed=0):
    return synth.write_model(synth.SHAPES[name], os.path.join(CACHE, f"{name}-s{seed}"), seed=seed)


def topk(v, k=64):
    idx = np.argsort(-v, kind="stable")[:k]
    return idx.astype(np.int32), v[idx].astype(np.float32)


def small_case(name, n_prompt, n_new, prefill):
    d = mdir(name)
    s = synth.SHAPES[name]
    prompt = synth.random_prompt(s.vocab_size, n_prompt, seed=11)
    ref = B.RefModel(d, n_prompt + n_new + 2)
    logits = np.stack([ref.step(int(t)) for t in prompt])
    out = {"prompt": prompt, "step_logits": logits.astype(np.float32),
           "greedy": ref.generate_greedy(prompt, n_new).astype(np.int32)}
    if prefill:
        out["prefill_logits"] = ref.prefill(prompt).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, f"{name.replace('-', '_')}.npz"), **out)
    print(name, "greedy", out["greedy"].tolist())


def large_case(name, n_prompt, n_new, fname):
    d = mdir(name)
    s = synth.SHAPES[name]
    prompt = synth.random_prompt(s.vocab_size, n_prompt, seed=11)
    ref = B.RefModel(d, n_prompt + n_new + 2)
    last = None
    for t in prompt:
        last = ref.step(int(t))
    ti, tv = topk(last)
    greedy = ref.generate_greedy(prompt, n_new).astype(np.int32)
    out = {"prompt": prompt, "greedy": greedy, "last_top_idx": ti, "last_top_val": tv,
           "last_norm": np.float64(np.linalg.norm(last.astype(np.float64))),
           "last_sum": np.float64(last.astype(np.float64).sum())}
    np.savez_compressed(os.path.join(HERE, fname), **out)
    print(name, "greedy", greedy[:16].tolist(), "...")


def config_budget_case():
    """load_model_config / compute_budget / solve_max_context of the reference."""
    L = B.ref_lib()
    cases = {}
    for name in ("qwen3.5-0.8b-shaped", "qwen3.5-2b-shaped", "tiny", "tiny-rep"):
        s = synth.SHAPES[name]
        path = os.path.join(tempfile.gettempdir(), f"qwc_cfg_{name}.json")
        with open(path, "w") as f:
            json.dump(synth.config_json(s), f, indent=1)
        ints = np.zeros(16, np.int32)
        dbl = np.zeros(4, np.float64)
        L.ref_load_config(path.encode(), ints, dbl)
        budgets = {}
        for ctx, kvb in ((1024, 4), (32768, 2), (131072, 2)):
            o = np.zeros(6, np.uint64)
            L.ref_compute_budget(path.encode(), 2, ctx, kvb, o)
            budgets[f"{ctx}_{kvb}"] = [int(x) for x in o]
        solve = {}
        for ram in (2 << 30, 8 << 30, 180 << 30, 1 << 20):
            solve[str(ram)] = int(L.ref_solve_max_context(path.encode(), ram, 1 << 29, 1 << 24,
                                                          1 << 20, 0, 1 << 26, 2))
        cases[name] = {"config": synth.config_json(s), "ints": ints.tolist(), "dbl": dbl.tolist(),
                       "budgets": budgets, "solve": solve}
    with open(os.path.join(HERE, "config_budget.json"), "w") as f:
        json.dump(cases, f, indent=1)
    print("config/budget cases", list(cases))


CASES = {
    "config": config_budget_case,
    "tiny": lambda: small_case("tiny", 8, 16, prefill=True),
    "tiny-rep": lambda: small_case("tiny-rep", 8, 16, prefill=False),
    "tiny-untied": lambda: small_case("tiny-untied", 8, 24, prefill=False),
    "small-0.8b": lambda: large_case("small-0.8b-widths", 32, 32, "small_0_8b_widths.npz"),
    "small-2b": lambda: large_case("small-2b-widths", 32, 32, "small_2b_widths.npz"),
    "0.8b": lambda: large_case("qwen3.5-0.8b-shaped", 32, 64, "qwen35_0_8b.npz"),
    # configs[3]'s model: a longer prompt so that the attention layers see a real context
    "2b": lambda: large_case("qwen3.5-2b-shaped", 512, 64, "qwen35_2b.npz"),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--2b", dest="two_b", action="store_true")
    ap.add_argument("--only", nargs="*", choices=sorted(CASES))
    a = ap.parse_args()
    B.build()
    if not B.ref_available():
        sys.exit("oracle/_ref/libqwen_ref.so is missing: the reference tree is needed to make fixtures")
    names = a.only or (["config", "tiny", "tiny-rep", "tiny-untied", "small-0.8b", "small-2b"] +
                       (["0.8b"] if a.full else []) + (["2b"] if a.two_b else []))
    for n in names:
        CASES[n]()


if __name__ == "__main__":
    main()
