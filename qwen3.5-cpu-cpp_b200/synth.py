"""Seeded synthetic Qwen3.5 checkpoints: ``config.json`` + bf16 ``model.safetensors``.

There is no network here for real checkpoints, so every model this project runs is
generated from a seed with the shapes of a real Qwen3.5 size.  The files use the
Hugging Face layout the reference engine reads:

* ``config.json`` with the architecture under ``text_config`` (the reference reads
  ``text_config`` first, ``src/config_loader.cpp:67-68``);
* tensor names ``model.language_model.layers.{L}.{linear_attn|self_attn|mlp}.*``,
  ``model.language_model.embed_tokens.weight`` and ``model.language_model.norm.weight``
  (``src/qwen_model.cpp:8,38-76``), with tied embeddings (no ``lm_head.weight``) unless
  the shape says otherwise.

Value conventions (fixed here so that every consumer sees the same model):

* projection matrices and the embedding ~ N(0, 0.02), stored bf16;
* the (1 + w)-form RMSNorm weights (input/post-attention layernorms, q_norm, k_norm,
  final norm) = 0, so the effective scale is 1 (``include/forward_pass.h:38-42``);
* the GDN gated-norm ``linear_attn.norm.weight`` is a plain multiplier
  (``include/forward_pass.h:44-47``) and is set to 1 -- zero would make every GDN
  mixer output exactly 0;
* ``dt_bias`` = 1, ``A_log`` ~ U(0, ln 16) stored f32, causal conv1d weights
  ``[C, 1, 4]`` ~ N(0, 0.1).

bf16 rounding is round-to-nearest-even from the fp32 draw.
"""
from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import dataclass, asdict, field

import numpy as np

LM = "model.language_model."


@dataclass(frozen=True)
class ModelShape:
    """Architecture of one Qwen3.5 text model (the keys of ``text_config``)."""

    name: str
    hidden_size: int
    num_hidden_layers: int
    intermediate_size: int
    vocab_size: int
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    head_dim: int = 256
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 16
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    full_attention_interval: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e7
    partial_rotary_factor: float = 0.25
    max_position_embeddings: int = 262144
    tie_word_embeddings: bool = True

    def is_attention_layer(self, layer: int) -> bool:
        # same rule as ModelConfig::is_attention_layer (include/model_config.h:60-62)
        return (layer + 1) % self.full_attention_interval == 0

    @property
    def conv_dim(self) -> int:
        return (2 * self.linear_num_key_heads * self.linear_key_head_dim
                + self.linear_num_value_heads * self.linear_value_head_dim)


# The sizes the benchmark configurations name, plus small shapes for fast tests.
QWEN35_0_8B = ModelShape("qwen3.5-0.8b-shaped", 1024, 24, 3584, 151936)
QWEN35_2B = ModelShape("qwen3.5-2b-shaped", 2048, 24, 6144, 151936)
# 4 layers (3 GDN + 1 attention), two kv heads (GQA group 2), small vocab.
TINY = ModelShape("tiny", 256, 4, 512, 1024, num_attention_heads=4, num_key_value_heads=2,
                  linear_num_key_heads=2, linear_num_value_heads=2)
# value heads = 2 x key heads: q/k heads are shared by two value heads
# (QwenModel::gdn_step handles this, src/qwen_model.cpp:159,194).
TINY_REP = ModelShape("tiny-rep", 256, 4, 512, 1024, num_attention_heads=4,
                      num_key_value_heads=2, linear_num_key_heads=2, linear_num_value_heads=4)
# real widths, few layers: exercises every kernel at production shapes quickly
SMALL_0_8B = ModelShape("small-0.8b-widths", 1024, 4, 3584, 151936)
# separate lm_head.weight (QwenModel prefers it over the tied embedding,
# src/qwen_model.cpp:67-69); random heads give non-degenerate greedy sequences
TINY_UNTIED = ModelShape("tiny-untied", 256, 4, 512, 1024, num_attention_heads=4,
                         num_key_value_heads=2, linear_num_key_heads=2,
                         linear_num_value_heads=2, tie_word_embeddings=False)
# 2B widths with few layers, for fast checks of the H=2048 / I=6144 code paths
SMALL_2B = ModelShape("small-2b-widths", 2048, 4, 6144, 151936)

SHAPES = {s.name: s for s in (QWEN35_0_8B, QWEN35_2B, TINY, TINY_REP, SMALL_0_8B,
                              TINY_UNTIED, SMALL_2B)}


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest-even) and return the raw uint16 bits."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b >> 16) & 1) + np.uint32(0x7FFF)
    return ((b + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def tensor_specs(s: ModelShape):
    """(name, shape, kind) for every tensor of the checkpoint, in a fixed order.

    kind: 'mat' N(0,0.02) bf16; 'norm1' (1+w) norm stored 0; 'one' plain weight 1;
    'dt' dt_bias 1; 'alog' U(0, ln16) f32; 'conv' N(0,0.1) bf16.
    """
    H, I = s.hidden_size, s.intermediate_size
    KD = s.linear_num_key_heads * s.linear_key_head_dim
    VD = s.linear_num_value_heads * s.linear_value_head_dim
    out = [(LM + "embed_tokens.weight", (s.vocab_size, H), "mat")]
    for L in range(s.num_hidden_layers):
        P = f"{LM}layers.{L}."
        out.append((P + "input_layernorm.weight", (H,), "norm1"))
        out.append((P + "post_attention_layernorm.weight", (H,), "norm1"))
        if s.is_attention_layer(L):
            A = P + "self_attn."
            NQ, NKV, HD = s.num_attention_heads, s.num_key_value_heads, s.head_dim
            out += [(A + "q_proj.weight", (NQ * HD * 2, H), "mat"),
                    (A + "k_proj.weight", (NKV * HD, H), "mat"),
                    (A + "v_proj.weight", (NKV * HD, H), "mat"),
                    (A + "o_proj.weight", (H, NQ * HD), "mat"),
                    (A + "q_norm.weight", (HD,), "norm1"),
                    (A + "k_norm.weight", (HD,), "norm1")]
        else:
            G = P + "linear_attn."
            VH = s.linear_num_value_heads
            out += [(G + "in_proj_qkv.weight", (2 * KD + VD, H), "mat"),
                    (G + "in_proj_z.weight", (VD, H), "mat"),
                    (G + "in_proj_b.weight", (VH, H), "mat"),
                    (G + "in_proj_a.weight", (VH, H), "mat"),
                    (G + "conv1d.weight", (2 * KD + VD, 1, s.linear_conv_kernel_dim), "conv"),
                    (G + "dt_bias", (VH,), "dt"),
                    (G + "A_log", (VH,), "alog"),
                    (G + "norm.weight", (s.linear_value_head_dim,), "one"),
                    (G + "out_proj.weight", (H, VD), "mat")]
        out += [(P + "mlp.gate_proj.weight", (I, H), "mat"),
                (P + "mlp.up_proj.weight", (I, H), "mat"),
                (P + "mlp.down_proj.weight", (H, I), "mat")]
    out.append((LM + "norm.weight", (H,), "norm1"))
    if not s.tie_word_embeddings:
        out.append(("lm_head.weight", (s.vocab_size, H), "mat"))
    return out


def _draw(rng: np.random.Generator, shape, kind):
    n = int(np.prod(shape))
    if kind == "mat":
        v = rng.standard_normal(n, dtype=np.float32)
        v *= np.float32(0.02)
        return "BF16", f32_to_bf16_bits(v)
    if kind == "conv":
        v = rng.standard_normal(n, dtype=np.float32)
        v *= np.float32(0.1)
        return "BF16", f32_to_bf16_bits(v)
    if kind == "norm1":
        return "BF16", np.zeros(n, np.uint16)
    if kind in ("one", "dt"):
        return "BF16", f32_to_bf16_bits(np.ones(n, np.float32))
    if kind == "alog":
        return "F32", rng.uniform(0.0, math.log(16.0), n).astype(np.float32)
    raise ValueError(kind)


def config_json(s: ModelShape) -> dict:
    tc = {k: v for k, v in asdict(s).items() if k not in ("name", "tie_word_embeddings")}
    del tc["rope_theta"], tc["partial_rotary_factor"]
    tc["rope_parameters"] = {"rope_type": "default", "rope_theta": s.rope_theta,
                             "partial_rotary_factor": s.partial_rotary_factor}
    tc["layer_types"] = ["full_attention" if s.is_attention_layer(L) else "linear_attention"
                         for L in range(s.num_hidden_layers)]
    tc["attn_output_gate"] = True
    tc["tie_word_embeddings"] = s.tie_word_embeddings
    tc["model_type"] = "qwen3_5_text"
    return {"architectures": ["Qwen3_5ForConditionalGeneration"], "model_type": "qwen3_5",
            "tie_word_embeddings": s.tie_word_embeddings, "text_config": tc,
            "_synthetic": {"name": s.name}}


def write_model(s: ModelShape, out_dir: str, seed: int = 0) -> str:
    """Write ``config.json`` + ``model.safetensors`` for shape ``s`` drawn from ``seed``.

    Reuses an existing directory whose ``.complete`` stamp matches (shape, seed).
    Returns ``out_dir``.
    """
    os.makedirs(out_dir, exist_ok=True)
    stamp = os.path.join(out_dir, ".complete")
    key = json.dumps({"shape": asdict(s), "seed": seed}, sort_keys=True)
    if os.path.exists(stamp) and open(stamp).read() == key:
        return out_dir
    rng = np.random.Generator(np.random.PCG64(seed))
    specs = tensor_specs(s)
    arrays, header, off = [], {}, 0
    for name, shape, kind in specs:
        dt, arr = _draw(rng, shape, kind)
        nb = arr.nbytes
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + nb]}
        arrays.append(arr)
        off += nb
    header["__metadata__"] = {"format": "pt", "seed": str(seed), "shape": s.name}
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    tmp = os.path.join(out_dir, "model.safetensors.tmp")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for a in arrays:
            f.write(a.tobytes())
    os.replace(tmp, os.path.join(out_dir, "model.safetensors"))
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(config_json(s), f, indent=1)
    with open(stamp, "w") as f:
        f.write(key)
    return out_dir


def load_safetensors(path: str) -> dict:
    """Minimal numpy reader: name -> (dtype str, shape, ndarray of raw elements)."""
    with open(path, "rb") as f:
        (hl,) = struct.unpack("<Q", f.read(8))
        hdr = json.loads(f.read(hl))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + hl
    out = {}
    for name, e in hdr.items():
        if name == "__metadata__":
            continue
        a, b = e["data_offsets"]
        raw = mm[base + a: base + b]
        dt = {"BF16": np.uint16, "F32": np.float32}[e["dtype"]]
        out[name] = (e["dtype"], tuple(e["shape"]), raw.view(dt).reshape(e["shape"]))
    return out


def random_prompt(vocab: int, n: int, seed: int = 1234) -> np.ndarray:
    """``n`` token ids ~ U[0, vocab) from ``seed`` (int32)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
