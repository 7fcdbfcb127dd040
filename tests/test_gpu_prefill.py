"""The batched forward pass (tensor-core GEMMs, GDN scan, causal attention) against the
CPU oracle's QwenForward::prefill and QwenModel::step restatements, at lengths that
cross chunk boundaries (QWC_PREFILL_CHUNK shrinks the chunk so that small models cover
the multi-chunk path: KV from earlier chunks, GDN state and conv ring carried over).

Bar (north star): logits rel_l2 <= 2e-3, greedy continuation identical."""
import os

import numpy as np
import pytest

from conftest import model_dir, rel_l2

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3


@pytest.fixture
def chunk(request):
    old = os.environ.get("QWC_PREFILL_CHUNK")
    os.environ["QWC_PREFILL_CHUNK"] = str(request.param)
    yield request.param
    if old is None:
        del os.environ["QWC_PREFILL_CHUNK"]
    else:
        os.environ["QWC_PREFILL_CHUNK"] = old


@pytest.mark.parametrize("chunk", [128, 4096], indirect=True)
@pytest.mark.parametrize("kv_dtype", [0, 1])
def test_forward_logits_long_all_rows(pkg, oracle, chunk, kv_dtype):
    d = model_dir(pkg, "tiny")
    s = pkg.synth.SHAPES["tiny"]
    T = 300
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=21)
    m = pkg.abi.Model(d, max_context=T + 8, kv_dtype=kv_dtype)
    got = m.forward_logits(ids)
    want = oracle.OracleModel(d, T + 8).prefill(ids)
    assert got.shape == want.shape == (T, s.vocab_size)
    per_row = np.array([rel_l2(got[i], want[i]) for i in range(T)])
    assert per_row.max() < LOGIT_TOL, (per_row.argmax(), per_row.max())
    assert (got.argmax(1) == want.argmax(1)).mean() > 0.99
    m.close()


@pytest.mark.parametrize("chunk", [96], indirect=True)
@pytest.mark.parametrize("shape", ["tiny-rep", "small-0.8b-widths"])
def test_prefill_then_decode_matches_stepping(pkg, oracle, chunk, shape):
    """qwc_prefill seeds KV / GDN state / conv ring; the decode that follows matches the
    oracle stepping the same prompt (the reference's generate_greedy path)."""
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    T, n_new = 250, 16
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=5)
    m = pkg.abi.Model(d, max_context=T + n_new + 4)
    lg = m.prefill(ids)
    assert m.position() == T
    orc = oracle.OracleModel(d, T + n_new + 4)
    ref = None
    for t in ids:
        ref = orc.step(int(t))
    assert rel_l2(lg, ref) < LOGIT_TOL
    tok, want_tok = int(np.argmax(lg)), int(np.argmax(ref))
    assert tok == want_tok
    for i in range(n_new):
        lg, am = m.step(tok)
        ref = orc.step(tok)
        assert rel_l2(lg, ref) < LOGIT_TOL, f"decode step {i}"
        assert am == int(np.argmax(ref))
        tok = am
    m.close()


def test_prefill_is_repeatable_and_resets_state(pkg):
    d = model_dir(pkg, "tiny")
    s = pkg.synth.SHAPES["tiny"]
    ids = pkg.synth.random_prompt(s.vocab_size, 40, seed=2)
    m = pkg.abi.Model(d, max_context=64)
    a = m.prefill(ids)
    m.step(3)
    b = m.prefill(ids)  # starts again from a reset state
    assert np.array_equal(a, b)
    assert m.position() == len(ids)
    m.close()


@pytest.fixture
def attn_impl():
    """Switch the batched pass's attention between the tcgen05 kernel (default) and the
    fp32 CUDA-core kernel; restores the environment afterwards."""
    old = os.environ.get("QWC_PREFILL_ATTN")

    def use(name):
        if name == "tc":
            os.environ.pop("QWC_PREFILL_ATTN", None)
        else:
            os.environ["QWC_PREFILL_ATTN"] = name

    yield use
    if old is None:
        os.environ.pop("QWC_PREFILL_ATTN", None)
    else:
        os.environ["QWC_PREFILL_ATTN"] = old


@pytest.mark.parametrize("chunk", [128, 4096], indirect=True)
@pytest.mark.parametrize("shape,T", [("tiny", 333), ("tiny-rep", 64), ("small-0.8b-widths", 203)])
def test_tensor_core_attention_matches_simt_and_oracle(pkg, oracle, chunk, attn_impl, shape, T):
    """The tcgen05 flash attention (bf16-pair operands, three products) against the fp32
    kernel and the oracle: GQA groups of 2 and 4 query heads, ragged lengths (a partial
    last key block, a partial last query block), one chunk and several."""
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=31)
    last = s.vocab_size > 4096  # wide vocabulary: the last position's logits only
    m = pkg.abi.Model(d, max_context=T + 8)
    attn_impl("tc")
    got = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
    attn_impl("simt")
    simt = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
    m.close()
    want = oracle.OracleModel(d, T + 8).prefill(ids, last_only=last).reshape(-1, s.vocab_size)
    assert got.shape == want.shape == simt.shape
    for i in range(got.shape[0]):
        assert rel_l2(got[i], want[i]) < LOGIT_TOL, i
        assert rel_l2(got[i], simt[i]) < LOGIT_TOL, i
    assert (got.argmax(1) == simt.argmax(1)).mean() > 0.99


@pytest.fixture
def fattn_splits():
    """Force the number of key ranges each query block of the tcgen05 attention is split
    into (QWC_FATTN_SPLITS, read per call); restores the environment afterwards."""
    old = os.environ.get("QWC_FATTN_SPLITS")

    def use(n):
        os.environ["QWC_FATTN_SPLITS"] = str(n)

    yield use
    if old is None:
        os.environ.pop("QWC_FATTN_SPLITS", None)
    else:
        os.environ["QWC_FATTN_SPLITS"] = old


@pytest.mark.parametrize("chunk", [128, 4096], indirect=True)
@pytest.mark.parametrize("shape,T", [("tiny", 333), ("tiny-rep", 64), ("small-0.8b-widths", 203)])
def test_tensor_core_attention_key_splits_match_unsplit_and_oracle(pkg, oracle, chunk, fattn_splits, shape, T):
    """Key-range splits of the tcgen05 attention (partials of O, m, l per range merged by
    the combine kernel): 2 and 3 ranges, and 16 -- more ranges than a short causal range
    has key blocks, so some splits are empty and some rows see only masked keys in a
    range -- against the unsplit kernel and the oracle."""
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=37)
    last = s.vocab_size > 4096
    m = pkg.abi.Model(d, max_context=T + 8)
    fattn_splits(1)
    base = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
    want = oracle.OracleModel(d, T + 8).prefill(ids, last_only=last).reshape(-1, s.vocab_size)
    for n in (2, 3, 16):
        fattn_splits(n)
        got = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
        for i in range(got.shape[0]):
            assert rel_l2(got[i], base[i]) < 1e-4, (n, i)
            assert rel_l2(got[i], want[i]) < LOGIT_TOL, (n, i)
        assert (got.argmax(1) == base.argmax(1)).mean() > 0.99
    m.close()


@pytest.fixture
def gdn_state_cols():
    """Force the column-slice width of the GDN state pass (QWC_GDN_STATE_COLS, read per
    call); restores the environment afterwards."""
    old = os.environ.get("QWC_GDN_STATE_COLS")

    def use(n):
        os.environ["QWC_GDN_STATE_COLS"] = str(n)

    yield use
    if old is None:
        os.environ.pop("QWC_GDN_STATE_COLS", None)
    else:
        os.environ["QWC_GDN_STATE_COLS"] = old


@pytest.mark.parametrize("chunk", [96, 4096], indirect=True)
@pytest.mark.parametrize("shape,T", [("tiny", 300), ("small-0.8b-widths", 203)])
def test_gdn_state_pass_slice_widths_match(pkg, oracle, chunk, gdn_state_cols, shape, T):
    """The GDN state pass with 8- and 4-column state slices (the tensor-parallel launch
    shapes: the key-dim and token sums split over more lanes) against 16-column slices and
    the oracle, across chunk boundaries; the decode state it leaves behind as well."""
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=43)
    last = s.vocab_size > 4096
    m = pkg.abi.Model(d, max_context=T + 8)
    gdn_state_cols(16)
    base = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
    base_next = m.prefill(ids)
    base_step, _ = m.step(int(np.argmax(base_next)))
    want = oracle.OracleModel(d, T + 8).prefill(ids, last_only=last).reshape(-1, s.vocab_size)
    for n in (8, 4):
        gdn_state_cols(n)
        got = m.forward_logits(ids, last_only=last).reshape(-1, s.vocab_size)
        for i in range(got.shape[0]):
            assert rel_l2(got[i], base[i]) < 1e-4, (n, i)
            assert rel_l2(got[i], want[i]) < LOGIT_TOL, (n, i)
        nxt = m.prefill(ids)
        assert int(np.argmax(nxt)) == int(np.argmax(base_next))
        step, _ = m.step(int(np.argmax(nxt)))
        assert rel_l2(step, base_step) < 1e-4, n
    m.close()


@pytest.mark.parametrize("chunk", [96, 4096], indirect=True)
@pytest.mark.parametrize("shape,T", [("tiny", 200), ("small-0.8b-widths", 150)])
def test_per_layer_hidden_states_match_oracle(pkg, oracle, chunk, shape, T):
    """The north star's bar on every layer: the residual stream after the embedding and
    after each layer of the batched pass (tcgen05 GEMMs, GDN, attention), across chunk
    boundaries, against the oracle's QwenForward::prefill, rel_l2 <= 2e-3 per layer."""
    d = model_dir(pkg, shape)
    s = pkg.synth.SHAPES[shape]
    ids = pkg.synth.random_prompt(s.vocab_size, T, seed=41)
    m = pkg.abi.Model(d, max_context=T + 8)
    got = m.forward_hidden(ids)
    m.close()
    _, want = oracle.OracleModel(d, T + 8).prefill(ids, last_only=True, hidden=True)
    assert got.shape == want.shape == (s.num_hidden_layers + 1, T, s.hidden_size)
    errs = [rel_l2(got[l], want[l]) for l in range(got.shape[0])]
    assert max(errs) < LOGIT_TOL, errs
