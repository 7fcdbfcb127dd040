"""The allocation-free attention-decode entry point (qwc_attention_decode_noalloc).

Some callers may not allocate device memory while they run: a plugin whose host
application hands out all device memory from its own pool, or a latency-critical serving
loop where cudaMalloc's implicit synchronisation is not acceptable. For them the library
keeps a fixed 4 MiB device array and this entry point uses it as its split-K workspace.
The test checks it against the regular entry point (qwc_attention_decode), on two calls
in a row with different shapes, so that the second call runs on the contents the first
left behind. This file is collected last; it passes alone or after the other tests.
"""
import numpy as np
import pytest

from conftest import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5  # same bar as the other kernel parity tests


def _inputs(pkg, n_ctx, kv_dtype, NQ=8, NKV=2, seed=0):
    HD = 256
    max_ctx = n_ctx + 3
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal((NQ, HD), dtype=np.float32) * 0.1).cuda()
    gate = torch.from_numpy(rng.standard_normal((NQ, HD), dtype=np.float32)).cuda()
    K = rng.standard_normal((NKV, max_ctx, HD), dtype=np.float32)
    V = rng.standard_normal((NKV, max_ctx, HD), dtype=np.float32)
    if kv_dtype == 1:
        K = pkg.synth.f32_to_bf16_bits(K).view(np.int16)
        V = pkg.synth.f32_to_bf16_bits(V).view(np.int16)
    return q, gate, torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(), max_ctx


@pytest.mark.parametrize("NQ,NKV,cases", [
    (8, 2, [(4099, 0), (777, 1)]),   # several splits, then the array's leftovers reused
    (8, 2, [(20, 0), (32, 1)]),      # one split: the result is written without a combine
    (8, 1, [(8192, 1), (5000, 0)]),  # GQA group 8 with > 128 splits: the unstaged combine
])
def test_noalloc_matches_regular_entry_two_calls(pkg, NQ, NKV, cases):
    for call, (n_ctx, kv_dtype) in enumerate(cases):
        q, gate, K, V, max_ctx = _inputs(pkg, n_ctx, kv_dtype, NQ, NKV, seed=call)
        want = torch.empty((NQ, 256), device="cuda")
        got = torch.full((NQ, 256), float("nan"), device="cuda")
        args = (q.data_ptr(), gate.data_ptr(), K.data_ptr(), V.data_ptr(), kv_dtype, NQ, NKV,
                max_ctx, n_ctx)
        pkg.abi.attention_decode(*args, want.data_ptr())
        pkg.abi.attention_decode_noalloc(*args, got.data_ptr())
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}"
        assert rel_l2(g, w) < TOL, f"call {call}"


def test_noalloc_rejects_workspace_beyond_limit(pkg):
    # 64 query heads x 296 splits needs ~19 MB of workspace: more than the 4 MiB array.
    # Real buffers of the full size are passed, so nothing could read out of bounds even
    # if the size check were missing.
    NQ, NKV, n_ctx = 64, 8, 32768
    q, gate, K, V, max_ctx = _inputs(pkg, n_ctx, 1, NQ, NKV)
    out = torch.empty((NQ, 256), device="cuda")
    with pytest.raises(pkg.abi.QwcError) as e:
        pkg.abi.attention_decode_noalloc(q.data_ptr(), gate.data_ptr(), K.data_ptr(),
                                         V.data_ptr(), 1, NQ, NKV, max_ctx, n_ctx,
                                         out.data_ptr())
    assert e.value.code == -1
    assert "exceeds" in str(e.value)


def test_noalloc_leaves_device_memory_unchanged(pkg):
    """A warmed-up call allocates nothing: the device's free memory is the same after it
    (the first call of the process may load the library's device module, which reserves
    the array; that happens in the warm-up call)."""
    NQ, NKV, n_ctx = 8, 2, 3000
    q, gate, K, V, max_ctx = _inputs(pkg, n_ctx, 0, NQ, NKV, seed=9)
    out = torch.empty((NQ, 256), device="cuda")
    args = (q.data_ptr(), gate.data_ptr(), K.data_ptr(), V.data_ptr(), 0, NQ, NKV, max_ctx, n_ctx,
            out.data_ptr())
    pkg.abi.attention_decode_noalloc(*args)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        pkg.abi.attention_decode_noalloc(*args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
