"""ctypes bindings for the CPU checkers -- TEST INFRASTRUCTURE.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference arm
load this module. It wraps

* ``liboracle.so``: the plain-C restatement of the reference's fp32 forward pass
  (qwen_oracle.c), fed the checkpoint's tensors from a numpy memmap;
* ``_ref/libqwen_ref.so``: the reference engine's own sources compiled here, driven
  through ref_harness.cpp (present only where the reference tree was available at
  build time; the file itself travels with the repository snapshot).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libqwen_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


class orc_config(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "hidden", "layers", "interval", "ffn", "vocab", "q_heads", "kv_heads", "head_dim",
        "rot_dim", "k_heads", "v_heads", "k_dim", "v_dim", "conv_k")] + [
        ("eps", C.c_float), ("theta", C.c_double)]


def build(ref_dir: str = "/root/reference") -> None:
    """make -C oracle (the reference library only when its sources exist)."""
    import subprocess
    targets = ["oracle"] + (["ref"] if os.path.isdir(os.path.join(ref_dir, "src")) else [])
    subprocess.run(["make", "-s", "-C", HERE, f"REF={ref_dir}"] + targets, check=True)


def read_text_config(model_dir: str) -> dict:
    with open(os.path.join(model_dir, "config.json")) as f:
        cfg = json.load(f)
    return cfg.get("text_config", cfg)


def _orc_config(tc: dict) -> orc_config:
    rp = tc.get("rope_parameters", {})
    hd = tc["head_dim"]
    prf = tc.get("partial_rotary_factor", rp.get("partial_rotary_factor", 0.25))
    return orc_config(
        hidden=tc["hidden_size"], layers=tc["num_hidden_layers"],
        interval=tc.get("full_attention_interval", 4), ffn=tc["intermediate_size"],
        vocab=tc["vocab_size"], q_heads=tc["num_attention_heads"],
        kv_heads=tc["num_key_value_heads"], head_dim=hd, rot_dim=int(hd * prf),
        k_heads=tc["linear_num_key_heads"], v_heads=tc["linear_num_value_heads"],
        k_dim=tc["linear_key_head_dim"], v_dim=tc["linear_value_head_dim"],
        conv_k=tc["linear_conv_kernel_dim"], eps=tc.get("rms_norm_eps", 1e-6),
        theta=tc.get("rope_theta", rp.get("rope_theta", 1e7)))


def _load_lib(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run oracle/Makefile)")
    return C.CDLL(path)


_orc = None


def orc_lib():
    global _orc
    if _orc is None:
        L = _load_lib(ORACLE_SO)
        L.orc_create.restype = C.c_void_p
        L.orc_create.argtypes = [C.POINTER(orc_config), C.c_int]
        L.orc_destroy.argtypes = [C.c_void_p]
        L.orc_set_tensor.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
        L.orc_finalize.argtypes = [C.c_void_p, C.c_char_p, C.c_int]
        L.orc_reset.argtypes = [C.c_void_p]
        L.orc_position.argtypes = [C.c_void_p]
        L.orc_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.orc_generate_greedy.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p]
        L.orc_prefill.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_void_p, C.c_void_p, C.c_int]
        L.orc_matmul_bf16.argtypes = [_u16p, _f32p, _f32p, C.c_int, C.c_int]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        L.orc_rmsnorm_gated.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_float]
        L.orc_l2norm.argtypes = [_f32p, C.c_int, C.c_float]
        L.orc_apply_rope.argtypes = [_f32p, C.c_int, C.c_int, C.c_double]
        L.orc_gdn_core.argtypes = [C.c_int] * 6 + [_f32p] * 6 + [_f32p, _f32p, _f32p]
        L.orc_attention.argtypes = [C.c_int] * 4 + [_f32p] * 4 + [_f32p]
        _orc = L
    return _orc


def _ptr(a: np.ndarray) -> int:
    return a.__array_interface__["data"][0]


class OracleModel:
    """The C restatement holding one model (QwenModel + QwenForward semantics)."""

    def __init__(self, model_dir: str, max_context: int = 4096):
        from_path = os.path.join(model_dir, "model.safetensors")
        self.tc = read_text_config(model_dir)
        self.cfg = _orc_config(self.tc)
        self.max_context = max_context
        L = orc_lib()
        self._h = L.orc_create(C.byref(self.cfg), max_context)
        self._keep = []
        with open(from_path, "rb") as f:
            (hl,) = struct.unpack("<Q", f.read(8))
            hdr = json.loads(f.read(hl))
        mm = np.memmap(from_path, dtype=np.uint8, mode="r")
        self._keep.append(mm)
        for name, e in hdr.items():
            if name == "__metadata__":
                continue
            a, b = e["data_offsets"]
            raw = mm[8 + hl + a: 8 + hl + b]
            dt = {"F32": 0, "BF16": 1}[e["dtype"]]
            n = (b - a) // (4 if dt == 0 else 2)
            L.orc_set_tensor(self._h, name.encode(), dt, _ptr(raw), n)
        buf = C.create_string_buffer(512)
        if L.orc_finalize(self._h, buf, 512) != 0:
            raise KeyError(f"missing weight {buf.value.decode()}")

    @property
    def vocab(self):
        return self.cfg.vocab

    def __del__(self):
        if getattr(self, "_h", None):
            orc_lib().orc_destroy(self._h)
            self._h = None

    def reset(self):
        orc_lib().orc_reset(self._h)

    def position(self):
        return orc_lib().orc_position(self._h)

    def step(self, token: int, hidden: bool = False):
        lg = np.empty(self.cfg.vocab, np.float32)
        hs = np.empty((self.cfg.layers + 1, self.cfg.hidden), np.float32) if hidden else None
        rc = orc_lib().orc_step(self._h, int(token), _ptr(lg), _ptr(hs) if hidden else None)
        if rc:
            raise ValueError("orc_step: bad token id or context full")
        return (lg, hs) if hidden else lg

    def generate_greedy(self, prompt, n_new: int):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        n = orc_lib().orc_generate_greedy(self._h, p, len(p), n_new, out)
        return out[:n]

    def prefill(self, ids, last_only: bool = False, hidden: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T = len(ids)
        lg = np.empty((1 if last_only else T, self.cfg.vocab), np.float32)
        hs = np.empty((self.cfg.layers + 1, T, self.cfg.hidden), np.float32) if hidden else None
        rc = orc_lib().orc_prefill(self._h, ids, T, _ptr(lg), _ptr(hs) if hidden else None,
                                   1 if last_only else 0)
        if rc:
            raise ValueError("orc_prefill: bad token id")
        return (lg, hs) if hidden else lg


_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        L = _load_lib(REF_SO)
        L.ref_open.restype = C.c_void_p
        L.ref_open.argtypes = [C.c_char_p, C.c_int]
        L.ref_close.argtypes = [C.c_void_p]
        for fn in ("ref_vocab", "ref_hidden", "ref_layers", "ref_position"):
            getattr(L, fn).argtypes = [C.c_void_p]
        L.ref_reset.argtypes = [C.c_void_p]
        L.ref_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.ref_generate_greedy.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p]
        L.ref_prefill.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p]
        L.ref_budget.argtypes = [C.c_void_p, np.ctypeslib.ndpointer(np.uint64)]
        L.ref_compute_budget.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int,
                                         np.ctypeslib.ndpointer(np.uint64)]
        L.ref_solve_max_context.restype = C.c_int64
        L.ref_solve_max_context.argtypes = [C.c_char_p] + [C.c_uint64] * 6 + [C.c_int]
        L.ref_load_config.argtypes = [C.c_char_p, _i32p, np.ctypeslib.ndpointer(np.float64)]
        L.ref_matmul_bf16.argtypes = [_u16p, _f32p, _f32p, C.c_int, C.c_int]
        L.ref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        L.ref_rmsnorm_gated.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_float]
        L.ref_l2norm.argtypes = [_f32p, C.c_int, C.c_float]
        L.ref_apply_rope.argtypes = [_f32p, C.c_int, C.c_int, C.c_double]
        L.ref_time_generate.restype = C.c_double
        L.ref_time_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, _i32p]
        _ref = L
    return _ref


class RefModel:
    """The reference engine itself (QwenModel / QwenForward) via oracle/_ref."""

    def __init__(self, model_dir: str, max_context: int = 4096):
        self._h = ref_lib().ref_open(model_dir.encode(), max_context)
        if not self._h:
            raise RuntimeError(f"reference engine could not load {model_dir}")
        self.vocab = ref_lib().ref_vocab(self._h)

    def __del__(self):
        if getattr(self, "_h", None):
            ref_lib().ref_close(self._h)
            self._h = None

    def reset(self):
        ref_lib().ref_reset(self._h)

    def position(self):
        return ref_lib().ref_position(self._h)

    def step(self, token: int):
        lg = np.empty(self.vocab, np.float32)
        ref_lib().ref_step(self._h, int(token), _ptr(lg))
        return lg

    def generate_greedy(self, prompt, n_new: int):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        n = ref_lib().ref_generate_greedy(self._h, p, len(p), n_new, out)
        return out[:n]

    def time_generate(self, prompt, n_new: int):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        secs = ref_lib().ref_time_generate(self._h, p, len(p), n_new, out)
        return secs, out[:n_new]

    def prefill(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lg = np.empty(len(ids) * self.vocab, np.float32)
        if not ref_lib().ref_prefill(self._h, ids, len(ids), lg):
            raise RuntimeError("reference prefill failed")
        return lg.reshape(len(ids), self.vocab)

    def budget(self):
        out = np.zeros(6, np.uint64)
        ref_lib().ref_budget(self._h, out)
        return out


# ---------------------------------------------------------------- int8 weight format
# No reference counterpart (the reference streams bf16 weights and names 8/4-bit weights as
# its next step, README.md:80-81): the format's definition restated in numpy, as the checker
# of qwc_quantize_q8 / qwc_gemv_q8. Groups of 128 columns per row.
Q8_GROUP = 128


def q8_quantize(w_bf16_bits: np.ndarray):
    """bf16 bits [rows][cols] -> (int8 codes, fp32 scales [rows][cols / 128]):
    scale = max |w| / 127 in fp32, q = round-half-even(w / scale) clamped to +-127."""
    w = (w_bf16_bits.astype(np.uint32) << 16).view(np.float32)
    rows, cols = w.shape
    g = w.reshape(rows, cols // Q8_GROUP, Q8_GROUP)
    scale = (np.abs(g).max(axis=2) / np.float32(127.0)).astype(np.float32)
    safe = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.rint((g / safe[:, :, None]).astype(np.float32))
    q = np.where(scale[:, :, None] > 0, np.clip(q, -127, 127), 0).astype(np.int8)
    return q.reshape(rows, cols), scale


def q8_gemv(q: np.ndarray, scale: np.ndarray, x: np.ndarray) -> np.ndarray:
    """y = dequant(q, scale) . x in float64 (the exact value the fp32 kernel approximates)."""
    rows, cols = q.shape
    w = q.astype(np.float64).reshape(rows, cols // Q8_GROUP, Q8_GROUP) * scale.astype(np.float64)[:, :, None]
    return w.reshape(rows, cols) @ x.astype(np.float64)
