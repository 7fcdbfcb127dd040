"""ctypes binding of libqwen_cuda's C ABI (include/qwen_cuda.h).

``Model`` mirrors the reference's ``QwenModel`` (``reset``, ``step``, ``position``,
``generate_greedy``, ``budget``) plus the ``QwenForward::prefill`` semantics
(``forward_logits``) and the state-seeding ``prefill``. The kernel-level functions
take device pointers (e.g. ``torch.Tensor.data_ptr()``) and a CUDA stream handle.

Loading fails loudly when the library is not built: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import LIB_PATH

QWC_OK = 0
ERRORS = {-1: "QWC_E_INVALID", -2: "QWC_E_CUDA", -3: "QWC_E_MISSING", -4: "QWC_E_SHAPE",
          -5: "QWC_E_CONTEXT", -6: "QWC_E_IO", -7: "QWC_E_DEVICE", -8: "QWC_E_OOM"}
DTYPE_F32, DTYPE_BF16 = 0, 1

# every symbol include/qwen_cuda.h declares
EXPORTS = ("qwc_load_config", "qwc_default_config", "qwc_compute_budget", "qwc_solve_max_context",
           "qwc_create", "qwc_create_from_dir", "qwc_destroy", "qwc_last_error", "qwc_get_budget",
           "qwc_get_config", "qwc_reset", "qwc_position", "qwc_step", "qwc_generate_greedy",
           "qwc_forward_logits", "qwc_forward_hidden", "qwc_prefill", "qwc_stream", "qwc_set_prompt",
           "qwc_enqueue_greedy", "qwc_read_tokens", "qwc_profile_step", "qwc_trace_step",
           "qwc_gemv_bf16", "qwc_gemm_bf16", "qwc_quantize_q8", "qwc_gemv_q8",
           "qwc_tp_shard_of", "qwc_tp_unique_id", "qwc_create_tp", "qwc_create_from_dir_tp",
           "qwc_tp_gather_state", "qwc_max_context", "qwc_check_step_timeout", "qwc_tp_set_timeout", "qwc_tp_allreduce_path",
           "qwc_gdn_decode_step", "qwc_gdn_prefill", "qwc_gdn_prefill_workspace",
           "qwc_attention_decode")
KERNEL_KINDS = {0: "mix_in", 1: "gdn", 2: "attn", 3: "mix_out", 4: "gate_up", 5: "down",
                6: "lm_head", 7: "decode_step"}


class qwc_config(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "hidden_size", "n_layers_total", "n_layers_gdn", "n_layers_attn", "gdn_k_heads",
        "gdn_v_heads", "gdn_k_head_dim", "gdn_v_head_dim", "gdn_conv_kernel", "attn_q_heads",
        "attn_kv_heads", "attn_head_dim", "ffn_intermediate", "vocab_size", "native_max_context",
        "attn_interval", "tie_word_embeddings")] + [
        ("rms_norm_eps", C.c_float), ("partial_rotary_factor", C.c_float),
        ("rope_theta", C.c_double), ("n_params", C.c_int64)]


class qwc_budget(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "weight_bytes", "gdn_state_bytes", "gdn_conv_bytes", "kv_cache_bytes",
        "activation_bytes", "vision_scratch_bytes")]

    def as_dict(self):
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


class qwc_tp_shard(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("kh0", "n_kh", "vh0", "n_vh", "q0", "n_q", "kv0", "n_kv",
                                       "i0", "n_i")]

    def as_dict(self):
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


class qwc_tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p)]


class QwcError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


_lib = None


def lib():
    """The loaded libqwen_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
    L = C.CDLL(LIB_PATH)
    vp, ip, fp = C.c_void_p, C.POINTER(C.c_int), C.c_void_p
    L.qwc_load_config.argtypes = [C.c_char_p, C.POINTER(qwc_config)]
    L.qwc_default_config.argtypes = [C.POINTER(qwc_config)]
    L.qwc_default_config.restype = None
    L.qwc_compute_budget.argtypes = [C.POINTER(qwc_config), C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.POINTER(qwc_budget)]
    L.qwc_solve_max_context.argtypes = [C.POINTER(qwc_config)] + [C.c_uint64] * 6 + [C.c_int]
    L.qwc_solve_max_context.restype = C.c_int64
    L.qwc_create.argtypes = [C.POINTER(qwc_config), C.POINTER(qwc_tensor), C.c_int, C.c_int,
                             C.c_int, C.c_int, C.POINTER(vp)]
    L.qwc_create_from_dir.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(vp)]
    L.qwc_create_from_dir_tp.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_char_p, C.POINTER(vp)]
    L.qwc_tp_unique_id.argtypes = [C.c_char_p, C.c_int]
    L.qwc_tp_shard_of.argtypes = [C.POINTER(qwc_config), C.c_int, C.c_int, C.POINTER(qwc_tp_shard)]
    L.qwc_destroy.argtypes = [vp]
    L.qwc_destroy.restype = None
    L.qwc_last_error.argtypes = [vp]
    L.qwc_last_error.restype = C.c_char_p
    L.qwc_get_budget.argtypes = [vp, C.POINTER(qwc_budget)]
    L.qwc_get_config.argtypes = [vp, C.POINTER(qwc_config)]
    L.qwc_reset.argtypes = [vp]
    L.qwc_position.argtypes = [vp]
    L.qwc_max_context.argtypes = [vp]
    L.qwc_step.argtypes = [vp, C.c_int, fp, ip]
    L.qwc_generate_greedy.argtypes = [vp, ip, C.c_int, C.c_int, ip]
    L.qwc_forward_logits.argtypes = [vp, ip, C.c_int, fp, C.c_int]
    L.qwc_forward_hidden.argtypes = [vp, ip, C.c_int, fp]
    L.qwc_prefill.argtypes = [vp, ip, C.c_int, fp, C.c_int]
    L.qwc_stream.argtypes = [vp]
    L.qwc_stream.restype = C.c_void_p
    L.qwc_set_prompt.argtypes = [vp, ip, C.c_int]
    L.qwc_enqueue_greedy.argtypes = [vp, C.c_int, C.c_int]
    L.qwc_read_tokens.argtypes = [vp, C.c_int, C.c_int, ip]
    L.qwc_profile_step.argtypes = [vp, C.c_int, ip, C.POINTER(C.c_float), C.POINTER(C.c_int64)]
    L.qwc_trace_step.argtypes = [vp, C.c_int, C.POINTER(C.c_int64)]
    L.qwc_gemv_bf16.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp]
    L.qwc_gdn_decode_step.argtypes = [vp] * 9 + [C.c_int, C.c_int, C.c_int, vp]
    L.qwc_attention_decode.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_int, vp, vp]
    _lib = L
    return L


def check(rc, handle=None):
    if rc != QWC_OK:
        msg = lib().qwc_last_error(handle)
        raise QwcError(rc, msg.decode() if msg else "")
    return rc


def _iptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int))


def load_config(path: str) -> qwc_config:
    c = qwc_config()
    check(lib().qwc_load_config(path.encode(), C.byref(c)))
    return c


def compute_budget(cfg: qwc_config, bpw=2, max_context=1024, kv_bytes=4, tiles=4, vit=1024):
    b = qwc_budget()
    check(lib().qwc_compute_budget(C.byref(cfg), bpw, max_context, kv_bytes, tiles, vit, C.byref(b)))
    return b.as_dict()


def tp_unique_id() -> bytes:
    """qwc_tp_unique_id: the NCCL id rank 0 sends to the other ranks."""
    buf = C.create_string_buffer(128)
    check(lib().qwc_tp_unique_id(buf, 128))
    return buf.raw


def tp_shard(cfg: qwc_config, rank: int, world: int) -> dict:
    """qwc_tp_shard_of: the heads / rows / columns that `rank` holds."""
    sh = qwc_tp_shard()
    check(lib().qwc_tp_shard_of(C.byref(cfg), rank, world, C.byref(sh)))
    return sh.as_dict()


class Model:
    """One device-resident model + decode state (QwenModel over the C ABI). With
    world > 1 the handle is rank `rank`'s tensor-parallel shard (prefill only); every
    rank must construct it concurrently with the same `unique_id`."""

    def __init__(self, model_dir: str, max_context: int = 4096, kv_dtype: int = DTYPE_F32,
                 device: int = 0, rank: int = 0, world: int = 1, unique_id: bytes | None = None):
        h = C.c_void_p()
        if world == 1:
            check(lib().qwc_create_from_dir(model_dir.encode(), max_context, kv_dtype, device,
                                            C.byref(h)))
        else:
            check(lib().qwc_create_from_dir_tp(model_dir.encode(), max_context, kv_dtype, device,
                                               rank, world, unique_id, C.byref(h)))
        self.rank, self.world = rank, world
        self._h = h
        cfg = qwc_config()
        check(lib().qwc_get_config(self._h, C.byref(cfg)), self._h)
        self.cfg = cfg
        self.vocab = cfg.vocab_size
        self.max_context = lib().qwc_max_context(self._h)  # the planned size for max_context <= 0

    def close(self):
        if getattr(self, "_h", None):
            lib().qwc_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):
            pass  # interpreter shutdown: module globals already cleared

    def reset(self):
        check(lib().qwc_reset(self._h), self._h)

    def position(self) -> int:
        return lib().qwc_position(self._h)

    def budget(self) -> dict:
        b = qwc_budget()
        check(lib().qwc_get_budget(self._h, C.byref(b)), self._h)
        return b.as_dict()

    def step(self, token: int, logits: bool = True):
        """QwenModel::step: returns (logits[vocab] or None, greedy id)."""
        lg = np.empty(self.vocab, np.float32) if logits else None
        am = C.c_int(-1)
        check(lib().qwc_step(self._h, int(token), lg.ctypes.data if logits else None,
                             C.byref(am)), self._h)
        return lg, am.value

    def generate_greedy(self, prompt, n_new: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        check(lib().qwc_generate_greedy(self._h, _iptr(p), len(p), n_new, _iptr(out)), self._h)
        return out[:n_new] if len(p) else out[:0]

    def forward_logits(self, ids, last_only: bool = False) -> np.ndarray:
        """QwenForward::prefill semantics (stateless): [T, vocab] logits."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T = len(ids)
        lg = np.empty((1 if last_only else T, self.vocab), np.float32)
        check(lib().qwc_forward_logits(self._h, _iptr(ids), T, lg.ctypes.data,
                                       1 if last_only else 0), self._h)
        return lg

    def forward_hidden(self, ids) -> np.ndarray:
        """The stateless pass's residual stream: [n_layers + 1, T, hidden] (slot 0 the
        embedding rows, slot l + 1 after layer l), the oracle's per-layer hidden states."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        T = len(ids)
        hs = np.empty((self.cfg.n_layers_total + 1, T, self.cfg.hidden_size), np.float32)
        check(lib().qwc_forward_hidden(self._h, _iptr(ids), T, hs.ctypes.data), self._h)
        return hs

    # ---- measurement hooks (no reference counterpart)
    def stream(self) -> int:
        return lib().qwc_stream(self._h)

    def set_prompt(self, prompt):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        check(lib().qwc_set_prompt(self._h, _iptr(p), len(p)), self._h)

    def enqueue_greedy(self, n_prompt: int, n_new: int):
        check(lib().qwc_enqueue_greedy(self._h, n_prompt, n_new), self._h)

    def read_tokens(self, start: int, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), np.int32)
        check(lib().qwc_read_tokens(self._h, start, n, _iptr(out)), self._h)
        return out[:n]

    def profile_step(self, cap: int = 512):
        """One eager decode step at the current position with per-launch CUDA-event
        timings: list of (kind, ms, algorithmic bytes)."""
        kind = np.zeros(cap, np.int32)
        ms = np.zeros(cap, np.float32)
        by = np.zeros(cap, np.int64)
        n = lib().qwc_profile_step(self._h, cap, _iptr(kind),
                                   ms.ctypes.data_as(C.POINTER(C.c_float)),
                                   by.ctypes.data_as(C.POINTER(C.c_int64)))
        if n < 0:
            check(n, self._h)
        n = min(n, cap)
        return [(KERNEL_KINDS[int(kind[i])], float(ms[i]), int(by[i])) for i in range(n)]

    def trace_step(self):
        """One eager step of the persistent decode kernel with device timestamps.
        Returns (kinds[P], stamps[G, P, 8]) or None when that kernel is not in use."""
        need = lib().qwc_trace_step(self._h, 0, None)
        if need < 0:
            if need == -1:
                return None
            check(need, self._h)
        buf = np.zeros(need, np.int64)
        rc = lib().qwc_trace_step(self._h, need, buf.ctypes.data_as(C.POINTER(C.c_int64)))
        if rc < 0:
            check(rc, self._h)
        G, P = int(buf[0]), int(buf[1])
        kinds = [KERNEL_KINDS[int(k)] for k in buf[2:2 + P]]
        return kinds, buf[2 + P:].reshape(G, P, 8)

    def check_step_timeout(self, wait_ms: int):
        """qwc_check_step_timeout: one step whose grid barrier cannot complete; returns the
        status code (QWC_E_DEVICE expected) instead of raising."""
        fn = lib().qwc_check_step_timeout
        fn.argtypes = [C.c_void_p, C.c_int]
        return int(fn(self._h, int(wait_ms)))

    def tp_set_timeout(self, ms: int):
        """qwc_tp_set_timeout: bound on every wait of this rank for its group."""
        fn = lib().qwc_tp_set_timeout
        fn.argtypes = [C.c_void_p, C.c_int]
        check(fn(self._h, int(ms)), self._h)

    def tp_allreduce_path(self) -> int:
        """qwc_tp_allreduce_path: 1 peer-memory all-reduce, 0 NCCL, 2 not decided yet."""
        fn = lib().qwc_tp_allreduce_path
        fn.argtypes = [C.c_void_p]
        r = int(fn(self._h))
        check(min(r, 0), self._h)
        return r

    def tp_gather_state(self, full: "Model | None"):
        """qwc_tp_gather_state: collective over the tensor-parallel group; rank 0 passes
        its single-GPU Model, which then continues decoding after the prefilled prompt."""
        fn = lib().qwc_tp_gather_state
        fn.argtypes = [C.c_void_p, C.c_void_p]
        check(fn(self._h, full._h if full is not None else None), self._h)

    def prefill(self, ids, logits: bool = True, last_only: bool = True):
        """Prefill that seeds the decode state; returns the last position's logits [vocab]
        (last_only) or every position's [T, vocab]."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        shape = (self.vocab,) if last_only else (len(ids), self.vocab)
        lg = np.empty(shape, np.float32) if logits else None
        check(lib().qwc_prefill(self._h, _iptr(ids), len(ids),
                                lg.ctypes.data if logits else None, 1 if last_only else 0), self._h)
        return lg


def gemv_bf16(W_ptr, x_ptr, y_ptr, out_dim, in_dim, stream=0):
    check(lib().qwc_gemv_bf16(W_ptr, x_ptr, y_ptr, out_dim, in_dim, stream))


def quantize_q8(W_ptr, Wq_ptr, scales_ptr, out_dim, in_dim, stream=0):
    """qwc_quantize_q8: int8 codes + per-(row, 128-group) fp32 scales from bf16 W."""
    fn = lib().qwc_quantize_q8
    fn.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int, C.c_void_p]
    check(fn(W_ptr, Wq_ptr, scales_ptr, out_dim, in_dim, stream))


def gemv_q8(Wq_ptr, scales_ptr, x_ptr, y_ptr, out_dim, in_dim, stream=0):
    """qwc_gemv_q8: y = dequant(Wq, scales) . x."""
    fn = lib().qwc_gemv_q8
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_int, C.c_void_p]
    check(fn(Wq_ptr, scales_ptr, x_ptr, y_ptr, out_dim, in_dim, stream))


def gemm_bf16(W_ptr, Xs_ptr, Y_ptr, M, N, K, accumulate=False, stream=0):
    """qwc_gemm_bf16: Y[N][M] (+)= X W^T on the tensor cores, X as hi/lo bf16 [N][2K]."""
    fn = lib().qwc_gemm_bf16
    fn.argtypes = [C.c_void_p] * 3 + [C.c_int] * 4 + [C.c_void_p]
    check(fn(W_ptr, Xs_ptr, Y_ptr, M, N, K, int(bool(accumulate)), stream))


def gdn_decode_step(mixed, a, b, conv_w, neg_exp_A, dt_bias, conv_ring, state, out, KH, VH,
                    pos, stream=0):
    check(lib().qwc_gdn_decode_step(mixed, a, b, conv_w, neg_exp_A, dt_bias, conv_ring, state,
                                    out, KH, VH, pos, stream))


def gdn_prefill(mixed, a, b, conv_w, neg_exp_A, dt_bias, conv_ring, state, out, KH, VH, T, pos0,
                workspace, workspace_bytes, stream=0):
    """qwc_gdn_prefill: T tokens of the GDN mixer core (chunked WY recurrence)."""
    fn = lib().qwc_gdn_prefill
    fn.argtypes = [C.c_void_p] * 9 + [C.c_int] * 4 + [C.c_void_p, C.c_size_t, C.c_void_p]
    check(fn(mixed, a, b, conv_w, neg_exp_A, dt_bias, conv_ring, state, out, KH, VH, T, pos0,
             workspace, workspace_bytes, stream))


def gdn_prefill_workspace(KH, VH, T) -> int:
    fn = lib().qwc_gdn_prefill_workspace
    fn.argtypes = [C.c_int] * 3
    fn.restype = C.c_size_t
    return int(fn(KH, VH, T))


def attention_decode_noalloc(q, gate, k_cache, v_cache, kv_dtype, NQ, NKV, max_ctx, n_ctx,
                             out, stream=0):
    """qwc_attention_decode_noalloc: same result as attention_decode, with its split-K
    workspace in the library's fixed device array instead of a cudaMalloc'd one."""
    L = lib()
    fn = L.qwc_attention_decode_noalloc
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int] * 5 + [C.c_void_p, C.c_void_p]
    check(fn(q, gate, k_cache, v_cache, kv_dtype, NQ, NKV, max_ctx, n_ctx, out, stream))


def attention_decode(q, gate, k_cache, v_cache, kv_dtype, NQ, NKV, max_ctx, n_ctx, out,
                     stream=0):
    check(lib().qwc_attention_decode(q, gate, k_cache, v_cache, kv_dtype, NQ, NKV, max_ctx,
                                     n_ctx, out, stream))
