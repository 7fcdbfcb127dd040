"""Host-side checks of libqwen_cuda that need no GPU: every entry point that
include/qwen_cuda.h declares is exported; the config loader, compute_budget and
solve_max_context reproduce the reference's results (tests/golden/config_budget.json,
made by running the reference's memory_budget.cpp / config_loader.cpp); argument and
device errors are reported as status codes, never as crashes."""
import ctypes as C
import json
import os
import re
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qwen_cuda.h")
GOLDEN = os.path.join(ROOT, "tests", "golden", "config_budget.json")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qwc_\w+)\s*\(", text)))


def test_header_declares_the_documented_entry_points(pkg):
    names = declared_functions()
    for must in ("qwc_create", "qwc_step", "qwc_generate_greedy", "qwc_prefill", "qwc_forward_logits",
                 "qwc_compute_budget", "qwc_solve_max_context", "qwc_gemm_bf16", "qwc_attention_decode_noalloc"):
        assert must in names
    assert set(pkg.abi.EXPORTS) <= set(names)


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.abi.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


@pytest.fixture(scope="module")
def cases():
    with open(GOLDEN) as f:
        return json.load(f)


def _cfg(pkg, case, name):
    path = os.path.join(tempfile.gettempdir(), f"qwc_cputest_{name}.json")
    with open(path, "w") as f:
        json.dump(case["config"], f)
    return pkg.abi.load_config(path)


@pytest.mark.parametrize("name", ["qwen3.5-0.8b-shaped", "qwen3.5-2b-shaped", "tiny", "tiny-rep"])
def test_config_loader_matches_reference(pkg, cases, name):
    c = _cfg(pkg, cases[name], name)
    ints = [c.hidden_size, c.n_layers_total, c.n_layers_gdn, c.n_layers_attn, c.gdn_k_heads, c.gdn_v_heads,
            c.gdn_k_head_dim, c.gdn_v_head_dim, c.gdn_conv_kernel, c.attn_q_heads, c.attn_kv_heads,
            c.attn_head_dim, c.ffn_intermediate, c.vocab_size, c.attn_interval, c.tie_word_embeddings]
    assert ints == cases[name]["ints"]
    eps, theta, prf, native = cases[name]["dbl"]
    assert abs(c.rms_norm_eps - eps) <= 1e-12
    assert c.rope_theta == theta
    assert abs(c.partial_rotary_factor - prf) < 1e-7
    assert c.native_max_context == int(native)


@pytest.mark.parametrize("name", ["qwen3.5-0.8b-shaped", "qwen3.5-2b-shaped", "tiny", "tiny-rep"])
def test_compute_budget_matches_reference(pkg, cases, name):
    c = _cfg(pkg, cases[name], name)
    keys = ("weight_bytes", "gdn_state_bytes", "gdn_conv_bytes", "kv_cache_bytes", "activation_bytes",
            "vision_scratch_bytes")
    for key, want in cases[name]["budgets"].items():
        ctx, kvb = (int(x) for x in key.split("_"))
        got = pkg.abi.compute_budget(c, 2, ctx, kvb)
        assert [got[k] for k in keys] == want, key


@pytest.mark.parametrize("name", ["qwen3.5-0.8b-shaped", "qwen3.5-2b-shaped", "tiny", "tiny-rep"])
def test_solve_max_context_matches_reference(pkg, cases, name):
    c = _cfg(pkg, cases[name], name)
    fn = pkg.abi.lib().qwc_solve_max_context
    for ram, want in cases[name]["solve"].items():
        got = fn(C.byref(c), int(ram), 1 << 29, 1 << 24, 1 << 20, 0, 1 << 26, 2)
        assert got == want, ram


def test_bad_config_and_arguments_are_status_codes(pkg):
    abi = pkg.abi
    lib = abi.lib()
    c = abi.qwc_config()
    assert lib.qwc_load_config(b"/nonexistent/config.json", C.byref(c)) != 0
    assert lib.qwc_last_error(None)  # a message is recorded
    out = C.c_void_p()
    assert lib.qwc_create_from_dir(b"/nonexistent", 64, 0, 0, C.byref(out)) != 0
    assert not out.value
    # invalid kernel-level arguments are rejected before any device work
    assert lib.qwc_gemv_bf16(None, None, None, 0, 0, None) != 0
    f = lib.qwc_gemm_bf16
    f.argtypes = [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_void_p]
    assert f(None, None, None, 128, 128, 100, 0, None) != 0  # K not a multiple of 64
