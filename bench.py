#!/usr/bin/env python
"""Decode benchmark of the B200 Qwen3.5 hybrid forward pass.

Workload: the 0.8B-shaped seeded model, a 32-token random prompt and
128 greedy tokens, i.e. exactly QwenModel::generate_greedy (src/qwen_model.cpp:241-255):
160 single-token decode steps. One bench "step" is one such generation; the metric is
decode tokens per second (step() calls per second, prompt tokens included, as the
reference processes its prompt one token at a time).

  value      device time of K generations with the prompt already in HBM (CUDA events
             on the engine's stream; max over ranks); inputs (1.31 GB of weights per
             token) are far larger than the 126 MB L2, so no flush is needed.
  e2e        the same through the C ABI call qwc_generate_greedy with host buffers:
             prompt H2D, reset, 160 graph replays, token ids D2H, all in the timed region.
  roofline   the dominant kernel: the persistent decode-step kernel (one launch = one
             token), timed live per launch with CUDA events against MEASURED_PEAKS.json's
             HBM copy bandwidth; `traffic` is the DRAM bytes per launch from the ncu
             capture summarised in profiles/ (null when no summary is present).
  cpu_baseline  the reference engine itself (oracle/_ref: its own sources, built here)
             on this host's cores, one full generation.

--impl reference times the reference's CPU path on the same workload: generate_greedy for
decode, QwenForward::prefill of a bounded prefix of the prompt for prefill.
Multi-GPU: single-sequence decode does not shard; N ranks run N independent replicas
(weak scaling), value = total tokens/s over all ranks.

--workload prefill measures the batched forward pass instead (configs[4]: the 2B-shaped
model, --seq-len tokens, default 131072; --seq-len 8192 is configs[3]'s prompt): one step =
one qwc_prefill of the whole prompt (state seeded for decoding, last logits returned). Under
torchrun the N ranks run it tensor parallel (heads sharded, NCCL all-reduce inside the
library; strong scaling), value = prompt tokens / device time (max over ranks).

Defaults: N=1 runs the decode workload (the headline metric) and adds a `prefill_tp1`
object, the prefill workload timed on one GPU; N>1 (torchrun) runs the prefill workload
tensor parallel, so the scaling lines all measure the same prefill at tp1 (from the N=1
line's `prefill_tp1`), tp2, tp4 and tp8. Roofline: tensor, the algorithmic FLOPs of
the forward pass (2 x projection parameters per token, causal attention
4 NQ HD (t+1) per token per attention layer, GDN 7 DK DV per head per token per GDN layer,
the lm_head for the last token) against the measured bf16 peak.

--workload q8-gemv times the int8-weight GEMV (qwc_gemv_q8, no reference counterpart) on
the lm_head shape against the bf16 GEMV of the same shape.

--workload gdn-op / attn-op time the mixer ops of configs[1] and configs[2] through the
kernel-level C ABI on device buffers: the GDN core (16 heads, 128/128, conv K=4; seeded
N(0,1) inputs rounded to bf16 values, A_log ~ U(0, ln 16)) as a 4096-token chunked prefill
(qwc_gdn_prefill) followed by 256 single-token steps (qwc_gdn_decode_step); the gated
attention decode (8 q / 2 kv heads, HD 256, a bf16 KV cache of 32768 positions ~ N(0,1),
gates ~ N(0,1)) for 512 one-query steps (qwc_attention_decode). HBM roofline of a decode
step: GDN 2 MiB of state read + written; attention 64 MiB of K and V. The CPU baseline is
the oracle's C restatement of the same op on a bounded sample.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_PROMPT, N_NEW = 32, 128
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "k_decode_step_qwen35_0.8b.md")
SHAPE = "qwen3.5-0.8b-shaped"
METRIC = "decode tok/s"
UNIT = "tok/s"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


RANK, WORLD, LOCAL_RANK = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
HOST_CORES = os.cpu_count() or 1
os.environ.setdefault("OMP_NUM_THREADS", str(HOST_CORES))  # before any OpenMP library loads


def workload_config(args):
    return {"workload": "configs[0]: qwen3.5-0.8b-shaped greedy decode", "model": SHAPE,
            "prompt_tokens": N_PROMPT, "new_tokens": N_NEW,
            "tokens_per_step": N_PROMPT + N_NEW, "global_batch": 1,
            "seq_len": N_PROMPT + N_NEW, "kv_cache": "fp32", "parallelism": f"replicas{args.gpus}",
            "l2": "inputs larger than L2 (1.31 GB of weights streamed per token)"}


def model_dir():
    base = os.environ.get("QWC_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "qwc_models"))
    return os.path.join(base, f"{SHAPE}-s0")


def ensure_model(pkg):
    return pkg.synth.write_model(pkg.synth.SHAPES[SHAPE], model_dir(), seed=0)


def decode_bytes_per_token(cfg, ctx):
    """Algorithmic HBM bytes of one decode token at context length ctx (fp32 KV)."""
    H, I, V = cfg.hidden_size, cfg.ffn_intermediate, cfg.vocab_size
    L = cfg.n_layers_total
    n_attn = L // cfg.attn_interval
    n_gdn = L - n_attn
    KD = cfg.gdn_k_heads * cfg.gdn_k_head_dim
    VD = cfg.gdn_v_heads * cfg.gdn_v_head_dim
    C = 2 * KD + VD
    NQ, NKV, HD = cfg.attn_q_heads, cfg.attn_kv_heads, cfg.attn_head_dim
    w = 0
    w += n_gdn * ((C + VD + 2 * cfg.gdn_v_heads) * H + H * VD) * 2
    w += n_attn * ((2 * NQ * HD + 2 * NKV * HD) * H + H * NQ * HD) * 2
    w += L * 3 * H * I * 2
    w += V * H * 2 + H * 2  # lm_head (tied embedding read in full) + embedding row
    small = L * 2 * H * 4 + n_gdn * (C * 4 * 4 + 3 * cfg.gdn_v_heads * 4 + 128 * 4) + n_attn * 2 * HD * 4
    state = n_gdn * cfg.gdn_v_heads * cfg.gdn_k_head_dim * cfg.gdn_v_head_dim * 4 * 2
    conv = n_gdn * C * (16 + 4)  # ring: read 16 B, write 4 B per channel
    kv = n_attn * (ctx * NKV * HD * 4 * 2 + 2 * NKV * HD * 4)
    return w + small + state + conv + kv


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.path = tempfile.mktemp(prefix="qwc_clocks_", suffix=".csv")
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if not self.proc or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons, power = [], None, set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


_JSON_FD = None


def emit(line):
    """The one JSON line goes to the original stdout; everything else (the engine's
    load-time messages, library output) was redirected to stderr."""
    os.write(_JSON_FD if _JSON_FD is not None else 1, (json.dumps(line) + "\n").encode())


def ncu_traffic():
    """DRAM bytes per launch of k_decode_step from the committed ncu summary."""
    try:
        with open(TRAFFIC_FILE) as f:
            for ln in f:
                if ln.startswith("traffic_bytes_per_launch:"):
                    return int(ln.split(":", 1)[1].strip())
    except (OSError, ValueError):
        pass
    return None


def phase_shares(m):
    """Share of the persistent step spent in each phase kind (device timestamps)."""
    import numpy as np
    kinds, st = m.trace_step()
    t0 = st[:, 0, 0].min()
    end = (st[:, :, 3] - t0).max(0)
    dur = np.diff(np.concatenate([[0], end]))
    tot = float(dur.sum())
    out = {}
    for k, d in zip(kinds, dur):
        out[k] = out.get(k, 0.0) + float(d) / tot
    return {k: round(v, 4) for k, v in out.items()}, round(tot / 1e3, 2)


def prefill_flops(c, T):
    """Algorithmic FLOPs of a T-token forward pass (see the module docstring)."""
    H, I, V, L = c.hidden_size, c.ffn_intermediate, c.vocab_size, c.n_layers_total
    DK, DV, KH, VH = c.gdn_k_head_dim, c.gdn_v_head_dim, c.gdn_k_heads, c.gdn_v_heads
    KD, VD = KH * DK, VH * DV
    NQ, NKV, HD = c.attn_q_heads, c.attn_kv_heads, c.attn_head_dim
    n_attn = L // c.attn_interval
    n_gdn = L - n_attn
    gdn_proj = (2 * KD + VD + VD + 2 * VH) * H + H * VD
    attn_proj = (2 * NQ * HD + 2 * NKV * HD) * H + H * NQ * HD
    params = n_gdn * gdn_proj + n_attn * attn_proj + L * 3 * I * H
    f = 2.0 * params * T
    f += n_attn * 4.0 * NQ * HD * T * (T + 1) / 2
    f += n_gdn * 7.0 * DK * DV * VH * T
    f += 2.0 * V * H
    return f, params


def prefill_launches(c, T, world, chunk=4096):
    """Kernels the library launches for one qwc_prefill: per chunk the embedding, per
    layer two norms and four GEMMs, the mixer (attention: prep, V transpose, tensor-core
    attention; GDN: prep, conv ring, chunk factors, state pass, outputs, gated norm), with
    tensor parallelism one residual add per all-reduce; then final norm + lm_head."""
    L = c.n_layers_total
    n_attn = L // c.attn_interval
    per_chunk = 1 + n_attn * (6 + 3) + (L - n_attn) * (6 + 6) + (2 * L if world > 1 else 0)
    return ((T + chunk - 1) // chunk) * per_chunk + 2


def measured_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), "measured"
    return 1590.0, "fallback"


PREFILL_MODEL = "qwen3.5-2b-shaped"
PREFILL_T = 131072


def prefill_config(name, T, world, params=None):
    c = {"workload": f"prefill of {T} random ids, {name} (configs[4] shape and length)"
         if T == PREFILL_T else f"prefill of {T} random ids, {name} (configs[3]/[4] shape)",
         "model": name, "global_batch": 1, "seq_len": T, "parallelism": f"tp{world}", "kv_cache": "fp32",
         "l2": "inputs larger than L2 (weights and activations of every layer streamed)"}
    if params is not None:
        c["projection_params"] = params
    return c


def prefill_model(pkg, name, dist=None):
    shape = pkg.synth.SHAPES[name]
    base = os.environ.get("QWC_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "qwc_models"))
    mdir = os.path.join(base, f"{name}-s0")
    if RANK == 0:
        pkg.synth.write_model(shape, mdir, seed=0)
    if dist:
        dist.barrier()
    return shape, pkg.synth.write_model(shape, mdir, seed=0)


def gpu_index_of(local_rank):
    """nvidia-smi index of this rank's GPU (CUDA_VISIBLE_DEVICES may remap it)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids_v = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids_v) and ids_v[local_rank].strip().isdigit():
            return int(ids_v[local_rank])
    return local_rank


def time_prefill(m, ids, steps, warmup, dist=None):
    """Device time (max over ranks) and wall time of `steps` qwc_prefill calls."""
    import torch
    stream = torch.cuda.ExternalStream(m.stream())
    for _ in range(warmup):
        m.prefill(ids)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_index_of(LOCAL_RANK)) as clocks:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        w0 = time.perf_counter()
        for _ in range(steps):
            lg = m.prefill(ids)
        e1.record(stream)
        stream.synchronize()
        wall = time.perf_counter() - w0
        if dist:
            dist.barrier()
    dev_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([dev_ms, wall], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, wall = float(t[0]), float(t[1])
    return dev_ms, wall, lg, clocks.summary()


def prefill_fields(cfg, T, steps, dev_ms, wall, world, vocab):
    """value / roofline / e2e of a timed prefill (tensor roofline of the algorithmic FLOPs)."""
    flops, params = prefill_flops(cfg, T)
    tf, tf_src = measured_tflops()
    achieved = flops * steps / (dev_ms / 1000.0) / 1e12
    return params, {
        "value": round(T * steps / (dev_ms / 1000.0), 1), "unit": "tok/s",
        "ms_per_step": round(dev_ms / steps, 3),
        "roofline": {"bound": "tensor", "kernel": "whole forward pass (tcgen05 GEMMs + GDN + attention)",
                     "achieved": round(achieved, 1), "peak": tf, "unit": "TFLOP/s",
                     "frac": round(achieved / tf, 4), "peak_source": tf_src, "traffic": None,
                     "flops_per_step": flops},
        "e2e": {"value": round(T * steps / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * T,
                "d2h_bytes_per_step": 4 * vocab},
        "gpu_launches": steps * prefill_launches(cfg, T, world)}


def run_prefill(args):
    import numpy as np
    import torch
    import __graft_entry__
    torch.cuda.set_device(LOCAL_RANK)
    dist = None
    if WORLD > 1:
        import datetime
        import torch.distributed as dist
        # plumbing only (NCCL id, barriers, max over ranks); the all-reduces of the
        # forward pass run on the library's own NCCL communicator
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    pkg = __graft_entry__.load_package()
    name = args.model or PREFILL_MODEL
    shape, d = prefill_model(pkg, name, dist)
    T = args.seq_len
    box = [pkg.abi.tp_unique_id() if RANK == 0 and WORLD > 1 else None]
    if dist:
        dist.broadcast_object_list(box, src=0)
    m = pkg.abi.Model(d, max_context=T + 16, device=LOCAL_RANK, rank=RANK, world=WORLD, unique_id=box[0])
    ids = pkg.synth.random_prompt(shape.vocab_size, T, seed=1234)
    dev_ms, wall, lg, clk = time_prefill(m, ids, args.steps, args.warmup, dist)
    params, f = prefill_fields(m.cfg, T, args.steps, dev_ms, wall, WORLD, shape.vocab_size)
    line = {"metric": "prefill tok/s", "value": f["value"], "unit": "tok/s", "n_gpus": WORLD,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": f["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": prefill_config(name, T, WORLD, params),
            "roofline": f["roofline"], "e2e": f["e2e"], "gpu_launches": f["gpu_launches"], "clocks": clk,
            "last_argmax": int(np.argmax(lg))}
    if WORLD > 1:  # which all-reduce combined the ranks' residual partials
        line["config"]["allreduce"] = {1: "peer-memory (NVLink loads/stores)", 0: "nccl"}.get(m.tp_allreduce_path(),
                                                                                          "undecided")
    if RANK == 0 and WORLD == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = ref_prefill_sample(d, ids)
    m.close()
    if RANK == 0:
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def ref_prefill_sample(d, ids, n=32):
    """The reference's QwenForward::prefill (oracle/_ref) on the first n ids of the prompt."""
    from oracle import bindings
    n = min(len(ids), n)
    if bindings.ref_available():
        ref, kind = bindings.RefModel(d, n + 2), "reference"
    else:
        ref, kind = bindings.OracleModel(d, n + 2), "port"
    t0 = time.perf_counter()
    ref.prefill(ids[:n])
    secs = time.perf_counter() - t0
    return {"value": round(n / secs, 3), "unit": "tok/s", "cores": int(os.environ.get("OMP_NUM_THREADS", HOST_CORES)),
            "kind": kind, "sample": f"QwenForward::prefill of the first {n} ids ({secs:.1f} s)"}


def prefill_point(pkg, steps=3, warmup=1):
    """The prefill workload of the scaling lines timed on this one GPU (tp1)."""
    import torch
    shape, d = prefill_model(pkg, PREFILL_MODEL)
    m = pkg.abi.Model(d, max_context=PREFILL_T + 16, device=LOCAL_RANK)
    ids = pkg.synth.random_prompt(shape.vocab_size, PREFILL_T, seed=1234)
    dev_ms, wall, _, clk = time_prefill(m, ids, steps, warmup)
    params, f = prefill_fields(m.cfg, PREFILL_T, steps, dev_ms, wall, 1, shape.vocab_size)
    m.close()
    torch.cuda.empty_cache()
    out = {"metric": "prefill tok/s", "steps": steps, "warmup": warmup,
           "config": prefill_config(PREFILL_MODEL, PREFILL_T, 1, params), "clocks": clk}
    out.update(f)
    return out


def _op_line(args, metric, value, unit, config, extra):
    line = {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": config}
    line.update(extra)
    return line


def run_gdn_op(args):
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    abi = pkg.abi
    KH = VH = 16
    DK = DV = 128
    C = 2 * KH * DK + VH * DV
    T, ND = 4096, 256
    rng = np.random.default_rng(2)
    bf = lambda a: pkg.synth.bf16_bits_to_f32(pkg.synth.f32_to_bf16_bits(a.astype(np.float32)))
    mixed = bf(rng.standard_normal((T + ND, C)))
    a = rng.standard_normal((T + ND, VH)).astype(np.float32)
    b = rng.standard_normal((T + ND, VH)).astype(np.float32)
    conv_w = (rng.standard_normal((C, 4)) * 0.1).astype(np.float32)
    A_log = rng.uniform(0, np.log(16), VH).astype(np.float32)
    dt = np.zeros(VH, np.float32)
    neg = (-np.exp(A_log)).astype(np.float32)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    d_mixed, d_a, d_b, d_w, d_neg, d_dt = dev(mixed), dev(a), dev(b), dev(conv_w), dev(neg), dev(dt)
    d_ring = torch.zeros((C, 4), device="cuda")
    d_state = torch.zeros((VH, DK, DV), device="cuda")
    d_out = torch.empty((T + ND, VH * DV), device="cuda")
    ws_b = abi.gdn_prefill_workspace(KH, VH, T)
    ws = torch.empty(ws_b, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def prefill():
        abi.gdn_prefill(d_mixed.data_ptr(), d_a.data_ptr(), d_b.data_ptr(), d_w.data_ptr(), d_neg.data_ptr(),
                        d_dt.data_ptr(), d_ring.data_ptr(), d_state.data_ptr(), d_out.data_ptr(), KH, VH, T, 0,
                        ws.data_ptr(), ws_b, stream.cuda_stream)

    def decode(t, sh):
        abi.gdn_decode_step(d_mixed[t].data_ptr(), d_a[t].data_ptr(), d_b[t].data_ptr(), d_w.data_ptr(),
                            d_neg.data_ptr(), d_dt.data_ptr(), d_ring.data_ptr(), d_state.data_ptr(),
                            d_out[t].data_ptr(), KH, VH, t, sh)

    # the 256 single-token steps as one CUDA graph (one launch each, no host gaps)
    for t in range(T, T + 4):
        decode(t, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sh = torch.cuda.current_stream().cuda_stream
        for t in range(T, T + ND):
            decode(t, sh)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(args.warmup):
        d_ring.zero_(); d_state.zero_()
        prefill()
        graph.replay()
    pf_ms = dec_ms = 0.0
    for _ in range(args.steps):
        d_ring.zero_(); d_state.zero_()
        torch.cuda.synchronize()
        e[0].record(stream)
        prefill()
        e[1].record(stream)
        graph.replay()
        e[2].record(stream)
        torch.cuda.synchronize()
        pf_ms += e[0].elapsed_time(e[1])
        dec_ms += e[1].elapsed_time(e[2])
    pf_ms /= args.steps
    us_step = dec_ms / args.steps / ND * 1000
    peak, src = measured_peaks()
    dec_bytes = 2 * VH * DK * DV * 4 + C * 4 + 2 * VH * 4 + VH * DV * 4 + 2 * C * 4 * 4
    from oracle import bindings
    # the oracle's C restatement over the whole workload (4096-token prefill + 256 steps,
    # ~3 s on one core): the CPU baseline sample and the parity of every output row
    n = T + ND
    st, cs, want = np.zeros((VH, DK, DV), np.float32), np.zeros((C, 3), np.float32), np.empty((n, VH, DV), np.float32)
    t0 = time.perf_counter()
    bindings.orc_lib().orc_gdn_core(n, KH, VH, DK, DV, 4, np.ascontiguousarray(mixed[:n]), conv_w,
                                    np.ascontiguousarray(a[:n]), np.ascontiguousarray(b[:n]), A_log, dt, st, cs, want)
    cpu = n / (time.perf_counter() - t0)
    got = d_out.cpu().numpy().reshape(n, VH, DV).astype(np.float64)
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want.astype(np.float64)))
    rel_pf = float(np.linalg.norm(got[:T] - want[:T]) / np.linalg.norm(want[:T].astype(np.float64)))
    line = _op_line(args, "GDN op prefill tok/s", T / (pf_ms / 1000), "tok/s",
                    {"workload": "configs[1]: GDN mixer op, T=4096 prefill then 256 decode steps", "heads": VH,
                     "dk": DK, "dv": DV, "conv": 4, "l2": "state 1 MiB per head set, inputs 100+ MB"},
                    {"ms_per_step": round(pf_ms, 3),
                     "decode": {"us_per_step": round(us_step, 2), "achieved_gbs": round(dec_bytes / (us_step * 1e3), 1),
                                "peak_gbs": peak, "frac": round(dec_bytes / (us_step * 1e3) / peak, 4),
                                "bytes_per_step": dec_bytes, "peak_source": src},
                     "roofline": {"bound": "hbm", "kernel": "k_gdn_decode (decode step)",
                                  "achieved": round(dec_bytes / (us_step * 1e3), 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(dec_bytes / (us_step * 1e3) / peak, 4), "peak_source": src,
                                  "traffic": None},
                     "e2e": None, "gpu_launches": args.steps * (4 + ND),
                     "rel_l2_vs_oracle": rel, "rel_l2_vs_oracle_prefill": rel_pf,
                     "cpu_baseline": {"value": round(cpu, 1), "unit": "tok/s", "cores": 1, "kind": "port",
                                      "sample": f"orc_gdn_core over all {n} tokens (the oracle's C restatement)"}})
    emit(line)
    return 0


def run_attn_op(args):
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    abi = pkg.abi
    NQ, NKV, HD, CTX, NS = 8, 2, 256, 32768, 512
    g = torch.Generator(device="cuda").manual_seed(3)
    K = torch.randn(NKV, CTX, HD, device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn(NKV, CTX, HD, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(NS, NQ, HD, device="cuda", generator=g) * 0.0625
    gate = torch.randn(NS, NQ, HD, device="cuda", generator=g)
    out = torch.empty(NS, NQ, HD, device="cuda")
    stream = torch.cuda.current_stream()

    def one(i, sh):
        abi.attention_decode(q[i].data_ptr(), gate[i].data_ptr(), K.data_ptr(), V.data_ptr(), 1, NQ, NKV, CTX, CTX,
                             out[i].data_ptr(), sh)

    for i in range(8):  # first call sizes the split-K workspace (allocated once)
        one(i, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sh = torch.cuda.current_stream().cuda_stream
        for i in range(NS):
            one(i, sh)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms = 0.0
    for _ in range(args.steps):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms += e0.elapsed_time(e1)
    us = ms / args.steps / NS * 1000
    bytes_step = 2 * NKV * CTX * HD * 2 + 3 * NQ * HD * 4
    peak, src = measured_peaks()
    from oracle import bindings
    kc = K.float()[:, :CTX].transpose(0, 1).contiguous().cpu().numpy()
    vc = V.float()[:, :CTX].transpose(0, 1).contiguous().cpu().numpy()
    want = np.empty((NQ, HD), np.float32)
    qn, gn = q[0].cpu().numpy(), gate[0].cpu().numpy()
    reps = 4
    t0 = time.perf_counter()
    for _ in range(reps):
        bindings.orc_lib().orc_attention(NQ, NKV, HD, CTX, qn, gn, kc, vc, want)
    cpu = reps / (time.perf_counter() - t0)
    err = float(np.linalg.norm(out[0].cpu().numpy() - want) / np.linalg.norm(want))
    line = _op_line(args, "attention decode op steps/s", 1e6 / us, "steps/s",
                    {"workload": "configs[2]: gated attention decode, 8q/2kv, HD 256, bf16 KV 32768, 512 steps",
                     "kv_cache": "bf16", "context": CTX, "l2": "KV 64 MiB per step (inputs larger than L2 in total)"},
                    {"ms_per_step": round(us / 1000, 5),
                     "roofline": {"bound": "hbm", "kernel": "k_attn_long_st + k_attn_long_combine (split-K flash decode, cp.async-staged K/V)",
                                  "achieved": round(bytes_step / (us * 1e3), 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(bytes_step / (us * 1e3) / peak, 4), "peak_source": src,
                                  "traffic": None, "bytes_per_step": bytes_step},
                     "e2e": None, "gpu_launches": args.steps * NS, "rel_l2_vs_oracle": err,
                     "cpu_baseline": {"value": round(cpu, 3), "unit": "steps/s", "cores": 1, "kind": "port",
                                      "sample": f"orc_attention over {CTX} positions, {reps} steps"}})
    emit(line)
    return 0


def run_q8_gemv(args):
    """Int8-weight decode GEMV (qwc_gemv_q8) on the lm_head shape of the 0.8B-shaped model
    (151936 x 1024, the largest GEMV of a decode step), against the bf16 GEMV of the same
    shape: bytes per call, GB/s against the measured copy bandwidth, and the result against
    the format's dequantised product (oracle.q8_gemv)."""
    import numpy as np
    import torch
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    abi = pkg.abi
    from oracle import bindings
    rows, cols = 151936, 1024
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).astype(np.float32)
    wb = pkg.synth.f32_to_bf16_bits(w)
    x = rng.standard_normal(cols, dtype=np.float32)
    d_w = torch.from_numpy(wb.view(np.int16)).cuda()
    d_q = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    d_s = torch.empty((rows, cols // 128), dtype=torch.float32, device="cuda")
    d_x = torch.from_numpy(x).cuda()
    d_y, d_yb = torch.empty(rows, device="cuda"), torch.empty(rows, device="cuda")
    abi.quantize_q8(d_w.data_ptr(), d_q.data_ptr(), d_s.data_ptr(), rows, cols)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > L2 between timed calls
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ms = 0.0
        for _ in range(args.steps):
            flush.zero_()
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ms += e0.elapsed_time(e1)
        return ms / args.steps

    q_ms = timed(lambda: abi.gemv_q8(d_q.data_ptr(), d_s.data_ptr(), d_x.data_ptr(), d_y.data_ptr(), rows, cols))
    b_ms = timed(lambda: abi.gemv_bf16(d_w.data_ptr(), d_x.data_ptr(), d_yb.data_ptr(), rows, cols))
    q_bytes = rows * cols + rows * (cols // 128) * 4 + cols * 4 + rows * 4
    b_bytes = rows * cols * 2 + cols * 4 + rows * 4
    peak, src = measured_peaks()
    q, sc = d_q.cpu().numpy(), d_s.cpu().numpy()
    t0 = time.perf_counter()
    want = bindings.q8_gemv(q, sc, x)
    cpu_s = time.perf_counter() - t0
    got = d_y.cpu().numpy().astype(np.float64)
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    exact = w.astype(np.float64) @ x.astype(np.float64)
    qerr = float(np.linalg.norm(got - exact) / np.linalg.norm(exact))
    gbs = q_bytes / (q_ms * 1e6)
    line = _op_line(args, "int8 GEMV calls/s", 1000.0 / q_ms, "calls/s",
                    {"workload": "lm_head-shaped int8 GEMV (151936 x 1024), group-128 scales",
                     "l2": "flushed between timed calls (256 MB write)"},
                    {"ms_per_step": round(q_ms, 5),
                     "roofline": {"bound": "hbm", "kernel": "k_gemv_q8", "achieved": round(gbs, 1), "peak": peak,
                                  "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_source": src, "traffic": None,
                                  "bytes_per_step": q_bytes},
                     "bf16_gemv": {"ms": round(b_ms, 5), "gbs": round(b_bytes / (b_ms * 1e6), 1),
                                   "speedup_of_int8": round(b_ms / q_ms, 3)},
                     "e2e": None, "gpu_launches": args.steps, "rel_l2_vs_format": rel,
                     "rel_l2_vs_bf16_weights": qerr,
                     "cpu_baseline": {"value": round(1.0 / cpu_s, 3), "unit": "calls/s", "cores": 1, "kind": "port",
                                      "sample": "oracle.q8_gemv (numpy, float64) of one call"}})
    emit(line)
    return 0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def cpu_baseline(d, prompt, n_new):
    """The reference engine (oracle/_ref) on this host's cores: one full generation."""
    from oracle import bindings
    cores = int(os.environ.get("OMP_NUM_THREADS", HOST_CORES))
    if bindings.ref_available():
        ref, kind = bindings.RefModel(d, len(prompt) + n_new + 2), "reference"
        secs, toks = ref.time_generate(prompt, n_new)
    else:
        ref, kind = bindings.OracleModel(d, len(prompt) + n_new + 2), "port"
        t0 = time.perf_counter()
        toks = ref.generate_greedy(prompt, n_new)
        secs = time.perf_counter() - t0
    n = len(prompt) + n_new
    return {"value": round(n / secs, 3), "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"one generate_greedy: {len(prompt)} prompt + {n_new} new tokens "
                      f"({n} step() calls, {secs:.2f} s)"}, toks


def run_reference(args):
    """--impl reference: the reference's CPU path on this arm's workload, rank 0 only."""
    if RANK != 0:
        return 0
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    if args.workload == "prefill":
        return run_reference_prefill(args, pkg)
    from oracle import bindings
    d = ensure_model(pkg)
    prompt = pkg.synth.random_prompt(pkg.synth.SHAPES[SHAPE].vocab_size, N_PROMPT, seed=1234)
    if bindings.ref_available():
        ref, kind = bindings.RefModel(d, N_PROMPT + N_NEW + 2), "reference"
    else:
        ref, kind = bindings.OracleModel(d, N_PROMPT + N_NEW + 2), "port"
    # each step: one whole generation (32 prompt + 128 new tokens, ~4 s on 16 cores); only
    # a run of more than 30 steps is shortened, and the line's config then says so
    n_new = N_NEW if args.steps + args.warmup <= 30 else max(8, N_NEW * 30 // (args.steps + args.warmup))

    def one():
        t0 = time.perf_counter()
        ref.generate_greedy(prompt, n_new)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        one()
    secs = sum(one() for _ in range(args.steps))
    toks = args.steps * (N_PROMPT + n_new)
    val = toks / secs
    cores = int(os.environ.get("OMP_NUM_THREADS", HOST_CORES))
    config = workload_config(args)
    config["new_tokens"] = n_new
    config["tokens_per_step"] = N_PROMPT + n_new
    config["seq_len"] = N_PROMPT + n_new
    line = {"metric": METRIC, "value": round(val, 3), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000 * secs / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "cpu_baseline": {"value": round(val, 3), "unit": UNIT, "cores": cores, "kind": kind,
                             "sample": f"{args.steps} x generate_greedy({N_PROMPT} prompt + {n_new} new)"},
            "e2e": {"value": round(val, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


def run_reference_prefill(args, pkg):
    """The reference's QwenForward::prefill on the prefill workload's prompt: each step a
    32-id prefix (the reference's attention is O(T^2) scalar code and it materialises
    [T][vocab] fp32 logits, so the full 131072-id prompt does not run on the CPU)."""
    from oracle import bindings
    name = args.model or PREFILL_MODEL
    shape, d = prefill_model(pkg, name)
    T = args.seq_len
    n = min(T, 32)
    ids = pkg.synth.random_prompt(shape.vocab_size, T, seed=1234)
    if bindings.ref_available():
        ref, kind = bindings.RefModel(d, n + 2), "reference"
    else:
        ref, kind = bindings.OracleModel(d, n + 2), "port"

    def one():
        t0 = time.perf_counter()
        ref.prefill(ids[:n])
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        one()
    secs = sum(one() for _ in range(args.steps))
    val = args.steps * n / secs
    cores = int(os.environ.get("OMP_NUM_THREADS", HOST_CORES))
    line = {"metric": "prefill tok/s", "value": round(val, 3), "unit": "tok/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000 * secs / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": prefill_config(name, T, WORLD),
            "cpu_baseline": {"value": round(val, 3), "unit": "tok/s", "cores": cores, "kind": kind,
                             "sample": f"{args.steps} x QwenForward::prefill of the first {n} of the {T} ids"},
            "e2e": {"value": round(val, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


def run_ours(args):
    import numpy as np
    import torch
    import __graft_entry__
    torch.cuda.set_device(LOCAL_RANK)
    dist = None
    if WORLD > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", LOCAL_RANK))
    pkg = __graft_entry__.load_package()
    if RANK == 0:
        ensure_model(pkg)
    if dist:
        dist.barrier()
    d = ensure_model(pkg)
    shape = pkg.synth.SHAPES[SHAPE]
    prompt = pkg.synth.random_prompt(shape.vocab_size, N_PROMPT, seed=1234)
    max_ctx = N_PROMPT + N_NEW + 16
    m = pkg.abi.Model(d, max_context=max_ctx, device=LOCAL_RANK)
    stream = torch.cuda.ExternalStream(m.stream())
    n_tok = N_PROMPT + N_NEW

    # ---- value: device-resident generations
    m.set_prompt(prompt)
    for _ in range(args.warmup):
        m.enqueue_greedy(N_PROMPT, N_NEW)
    ref_tokens = m.read_tokens(N_PROMPT, N_NEW)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_index = LOCAL_RANK
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if LOCAL_RANK < len(ids) and ids[LOCAL_RANK].strip().isdigit():
            gpu_index = int(ids[LOCAL_RANK])
    with ClockSampler(gpu_index) as clocks:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            m.enqueue_greedy(N_PROMPT, N_NEW)
        e1.record(stream)
        stream.synchronize()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    dev_ms = e0.elapsed_time(e1)
    got = m.read_tokens(N_PROMPT, N_NEW)
    assert np.array_equal(got, ref_tokens), "generations differ between runs"
    if dist:
        t = torch.tensor([dev_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms = float(t.item())
    total_tokens = WORLD * args.steps * n_tok
    value = total_tokens / (dev_ms / 1000.0)
    clk = clocks.summary()

    # ---- e2e: the C ABI call with host buffers (H2D prompt, D2H ids inside the timed region)
    for _ in range(2):
        out = m.generate_greedy(prompt, N_NEW)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    w0 = time.perf_counter()
    for _ in range(args.steps):
        out = m.generate_greedy(prompt, N_NEW)
    e1.record(stream)
    stream.synchronize()
    wall = time.perf_counter() - w0
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    assert np.array_equal(out, ref_tokens), "e2e generation differs from the device-resident one"
    e2e = {"value": round(WORLD * args.steps * n_tok / (e2e_ms / 1000.0), 2), "unit": UNIT,
           "h2d_bytes_per_step": N_PROMPT * 4, "d2h_bytes_per_step": N_NEW * 4 + 4,
           "wall_clock_value": round(WORLD * args.steps * n_tok / wall, 2)}

    # ---- live per-launch timing of eager steps -> roofline of the dominant kernel
    m.generate_greedy(prompt, 8)  # position 40, mid-workload context
    prof = []
    for _ in range(4):
        prof += m.profile_step()
    launches_per_step = len(prof) // 4
    persistent = any(k == "decode_step" for k, _, _ in prof)
    shares, traced_us = phase_shares(m) if persistent else (None, None)
    by_kind = {}
    for k, ms, b in prof:
        e = by_kind.setdefault(k, [0.0, 0, 0])
        e[0] += ms
        e[1] += b
        e[2] += 1
    dom = max(by_kind, key=lambda k: by_kind[k][0])
    dms, dbytes, dn = by_kind[dom]
    peak, peak_src = measured_peaks()
    achieved = (dbytes / dn) / (dms / dn / 1000.0) / 1e9
    tot_ms = sum(v[0] for v in by_kind.values())
    share = {k: round(v[0] / tot_ms, 4) for k, v in by_kind.items()}
    kernel_gbs = {k: round((v[1] / v[2]) / (v[0] / v[2] / 1000.0) / 1e9, 1) for k, v in by_kind.items()}

    # step-level HBM roofline of the timed workload (context grows over the generation)
    cfg = m.cfg
    step_bytes = sum(decode_bytes_per_token(cfg, ctx) for ctx in range(1, n_tok + 1))
    step_gbs = step_bytes / ((dev_ms / args.steps) / 1000.0) / 1e9

    line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": WORLD,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args),
            "roofline": {"bound": "hbm",
                         "kernel": "k_decode_step (whole step)" if dom == "decode_step" else f"k_gemv ({dom})",
                         "achieved": round(achieved, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_src,
                         "traffic": ncu_traffic() if dom == "decode_step" else None,
                         "bytes_per_launch": int(dbytes / dn), "avg_launch_ms": round(dms / dn, 5),
                         "timing": "eager launches, CUDA events per launch"},
            "step_roofline": {"bytes_per_token": int(step_bytes / n_tok),
                              "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                              "frac": round(step_gbs / peak, 4), "peak_source": peak_src},
            "kernel_share": share, "kernel_gbs": kernel_gbs,
            "eager_step_ms": round(tot_ms / 4, 4),
            "phase_share": shares, "traced_step_us": traced_us,
            "e2e": e2e, "gpu_launches": int(args.steps * n_tok * launches_per_step),
            "clocks": clk}
    if RANK == 0 and WORLD == 1 and not args.no_cpu_baseline:
        cb, toks = cpu_baseline(d, prompt, N_NEW)
        cb["tokens_match"] = bool(np.array_equal(np.asarray(toks[:N_NEW]), ref_tokens))
        line["cpu_baseline"] = cb
    m.close()
    if WORLD == 1 and not args.no_prefill_point:
        # the scaling lines' prefill workload on this one GPU (their tp1 point)
        line["prefill_tp1"] = prefill_point(pkg)
    if RANK == 0:
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    global _JSON_FD
    _JSON_FD = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=("decode", "prefill", "gdn-op", "attn-op", "q8-gemv"), default=None,
                    help="default: decode on one GPU, prefill (tensor parallel) under torchrun")
    ap.add_argument("--seq-len", type=int, default=PREFILL_T, help="prefill workload: prompt length")
    ap.add_argument("--model", default=None, help="prefill workload: synthetic shape name")
    ap.add_argument("--no-prefill-point", action="store_true",
                    help="decode workload: skip the one-GPU prefill point (prefill_tp1)")
    args = ap.parse_args()
    if args.workload is None:
        args.workload = "prefill" if WORLD > 1 else "decode"
    if args.impl == "reference":
        return run_reference(args)
    args.warmup = max(args.warmup, 3)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "gdn-op":
        return run_gdn_op(args)
    if args.workload == "attn-op":
        return run_attn_op(args)
    if args.workload == "q8-gemv":
        return run_q8_gemv(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
