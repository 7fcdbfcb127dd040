"""Failure paths of model construction (the reference's only error model is a false ok()
and a message, src/qwen_model.cpp:22-31; here a status code and qwc_last_error):
a truncated safetensors shard, a missing tensor, and a config whose vocab_size exceeds the
embedding rows (the reference would read past the embedding at src/qwen_model.cpp:236).
Construction touches the device, so these run with the GPU tests."""
import json
import os
import shutil
import struct

import numpy as np
import pytest

from conftest import model_dir

pytestmark = pytest.mark.gpu
E_MISSING, E_SHAPE, E_IO = -3, -4, -6
LM = "model.language_model."


def copy_model(pkg, tmp_path, shape="tiny"):
    src = model_dir(pkg, shape)
    dst = tmp_path / "model"
    dst.mkdir()
    for f in ("config.json", "model.safetensors"):
        shutil.copy(os.path.join(src, f), dst / f)
    return str(dst)


def rewrite_without(path, drop):
    """The shard again with tensor `drop` left out of the header and the data."""
    raw = open(path, "rb").read()
    (hl,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + hl])
    meta = hdr.pop("__metadata__", None)
    out_hdr, blobs, off = {}, [], 0
    for name, e in hdr.items():
        if name == drop:
            continue
        a, b = e["data_offsets"]
        blobs.append(raw[8 + hl + a:8 + hl + b])
        out_hdr[name] = {"dtype": e["dtype"], "shape": e["shape"], "data_offsets": [off, off + (b - a)]}
        off += b - a
    if meta is not None:
        out_hdr["__metadata__"] = meta
    hj = json.dumps(out_hdr).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj + b"".join(blobs))


def test_truncated_shard_is_an_io_error(pkg, tmp_path):
    d = copy_model(pkg, tmp_path)
    p = os.path.join(d, "model.safetensors")
    size = os.path.getsize(p)
    with open(p, "r+b") as f:
        f.truncate(size - 4096)  # the last tensors now end past the file
    with pytest.raises(pkg.abi.QwcError) as e:
        pkg.abi.Model(d, max_context=16)
    assert e.value.code == E_IO


def test_missing_tensor_is_reported_by_name(pkg, tmp_path):
    d = copy_model(pkg, tmp_path)
    name = LM + "layers.1.linear_attn.in_proj_z.weight"
    rewrite_without(os.path.join(d, "model.safetensors"), name)
    with pytest.raises(pkg.abi.QwcError) as e:
        pkg.abi.Model(d, max_context=16)
    assert e.value.code == E_MISSING
    assert name in str(e.value)


def test_vocab_larger_than_embedding_is_a_shape_error(pkg, tmp_path):
    d = copy_model(pkg, tmp_path)
    cp = os.path.join(d, "config.json")
    cfg = json.load(open(cp))
    cfg["text_config"]["vocab_size"] += 8
    json.dump(cfg, open(cp, "w"))
    with pytest.raises(pkg.abi.QwcError) as e:
        pkg.abi.Model(d, max_context=16)
    assert e.value.code == E_SHAPE


def test_vocab_smaller_than_embedding_uses_the_first_rows(pkg, oracle, tmp_path):
    """An embedding with more rows than vocab_size (padded vocabularies) is accepted: the
    first vocab_size rows are the vocabulary, as in the reference, which sizes its
    logits by vocab_size."""
    d = copy_model(pkg, tmp_path)
    cp = os.path.join(d, "config.json")
    cfg = json.load(open(cp))
    cfg["text_config"]["vocab_size"] -= 24
    json.dump(cfg, open(cp, "w"))
    m = pkg.abi.Model(d, max_context=16)
    assert m.vocab == cfg["text_config"]["vocab_size"]
    lg, am = m.step(5)
    assert lg.shape == (m.vocab,) and np.isfinite(lg).all() and 0 <= am < m.vocab
    m.close()
