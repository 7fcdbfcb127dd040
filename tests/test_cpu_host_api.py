"""The C++ drop-in API compiled as a caller would compile it (host/include + the in-tree
libqwen_cuda.so): SafeTensors::view / get_f32 / get_row_f32 (the reference's interface,
include/safetensors_loader.h) against the raw bytes of the checkpoint file."""
import os

import numpy as np
import pytest

import host_api
from conftest import model_dir

LM = "model.language_model."


@pytest.mark.parametrize("name,row", [(LM + "embed_tokens.weight", 17),           # BF16 matrix
                                      (LM + "layers.0.linear_attn.A_log", 0),    # F32 vector
                                      (LM + "layers.3.self_attn.o_proj.weight", 255),
                                      (LM + "norm.weight", 0)])                   # BF16 vector
def test_safetensors_accessors_match_file_bytes(pkg, tmp_path, name, row):
    d = model_dir(pkg, "tiny")
    raw = pkg.synth.load_safetensors(os.path.join(d, "model.safetensors"))
    dtype, shape, arr = raw[name]
    want = pkg.synth.bf16_bits_to_f32(arr) if dtype == "BF16" else np.asarray(arr, np.float32)
    out = str(tmp_path / "st.bin")
    p = host_api.run("st", d, name, row, out)
    assert p.returncode == 0, p.stderr
    r = host_api.read_st(out)
    assert r["view_numel"] == int(np.prod(shape))
    assert r["view_kind"] == (1 if dtype == "BF16" else 0)
    assert r["cached"] and r["f32_numel"] == want.size
    assert np.array_equal(r["f32"], want.reshape(-1))  # exact widening, no rounding
    if len(shape) == 2:
        assert r["row_ok"] and np.array_equal(r["row"], want[row])
        assert r["oob_refused"]
    else:
        assert not r["row_ok"]  # rows exist for 2-D tensors only
    assert r["missing_refused"]
