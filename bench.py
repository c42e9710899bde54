#!/usr/bin/env python
"""Benchmark of the INT8 decode step on B200.

Workload: Qwen3-ASR-0.6B decoder shapes (hidden
1024, intermediate 3072, 28 layers, 16/8 heads x 128, vocab 151936), random
N(0, 0.02) weights quantised per output channel to INT8, f32 embedding
table, M independent sequences (default 8) each at KV length 1024.  One
step = one greedy decode step of all M sequences: embedding gather, 28
layers, final norm, lm head, argmax.  Metric: decode tokens/s (whole job).

Data-parallel over GPUs with no collective on the data path: each rank runs
its own M sequences on its own weight replica (weak scaling); the only
collectives are the timing barrier and the max-over-ranks of the timings.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch M] [--impl ours|reference]

Prints one JSON line on rank 0.

    python bench.py --workload e2e [--gpus N]
    python bench.py --workload segments [--gpus N]

run the whole transcription path through qasr_transcribe_lanes: 30 s of
synthetic audio per segment -> log-mel -> encoder -> prompt -> prefill ->
greedy decode (e2e: Qwen3-ASR-0.6B shapes, one segment per GPU, 256 tokens;
segments: 1.7B shapes, 64 segments split evenly over the GPUs and decoded 8
at a time, 128 tokens each, over --lanes engine lanes per GPU that overlap
one another).  Metric: audio seconds per second (whole job).

    python bench.py --workload gemm [--steps K] [--warmup W]

measures the INT8 prefill/encoder projections instead (one GPU): one step =
the four projections of a decoder layer over a 404-token prompt plus the six
of an encoder layer over 390 tokens (Qwen3-ASR-0.6B shapes), through the
kernel-level linear_nobias_int8 / linear_int8 entries.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (INT8 decode step, Qwen3-ASR-0.6B decoder shapes)"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 50; 5 for e2e, 3 for segments)")
    ap.add_argument("--warmup", type=int, default=None, help="warm-up steps (default 5; 3 for e2e / segments)")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--kv-len", type=int, default=1024)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--step-kernel", type=int, choices=(0, 1), default=1,
                    help="decode step as one persistent kernel (0) or per-layer kernels (1, the default)")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode workload only: skip the configs[4]/[3] transcription objects of the line")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample length")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--segments", type=int, default=None,
                    help="segments of the whole job for --workload segments (default 64, the configuration's)")
    ap.add_argument("--lanes", type=int, default=None,
                    help="engine lanes (decoder + encoder pairs) per GPU for the transcription workloads "
                         "(default 1 for e2e, 4 for segments)")
    ap.add_argument("--workload", choices=("decode", "gemm", "encoder", "e2e", "segments", "pre_attn",
                                           "enc_elementwise"), default="decode")
    ap.add_argument("--model", choices=("0.6b", "1.7b"), default="0.6b",
                    help="decoder shapes of the decode workload (0.6b = BASELINE configs[2])")
    ap.add_argument("--layers", type=int, default=28,
                    help="decoder layers (28 = the configured workload; fewer only for profiler captures)")
    a = ap.parse_args()
    long_run = a.workload in ("e2e", "segments")
    if a.steps is None:
        a.steps = {"e2e": 5, "segments": 3, "pre_attn": 400, "enc_elementwise": 120}.get(a.workload, 50)
    if a.warmup is None:
        a.warmup = 3 if long_run else 5
    return a


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every few ms."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons = [], 0
        self.ok = False
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# --------------------------------------------------------- byte accounting --
# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each
# kernel class from one ncu capture of the 0.6B, M=8, KV-1024 step; see
# profiles/attn_decode_0p6b_m8_kv1024.md and
# profiles/int8_contraction_tcgen05_decode_0p6b_m8.md for the commands.
NCU_TRAFFIC_M8 = {"attn": 67960832 + 1236736, "qkv": 4317440, "oproj": 2247168, "gateup": 6412544,
                  "down": 3328512, "lmhead": 156295680 + 5308928}


def class_bytes(cfg, M, kv_len):
    """Algorithmic bytes per launch of each kernel class of the step (weights,
    scales, activations in/out, K/V rows read)."""
    H, I, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    q, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    f = 4
    return {
        "embed": M * H * f * 2,
        "norm": M * H * f * 2 + H * f,
        "qkv": (q + 2 * kv) * H + (q + 2 * kv) * f + M * H * f + M * (q + 2 * kv) * f,
        "qkv_post": M * (q + 2 * kv) * f * 2 + 2 * hd * f,
        "attn": M * 2 * kv_len * kv * f + 2 * M * q * f,
        "oproj": H * q + H * f + M * q * f + 2 * M * H * f,
        "gateup": 2 * I * H + 2 * I * f + M * H * f + M * I * f,
        "down": H * I + H * f + M * I * f + 2 * M * H * f,
        "lmhead": cfg["vocab"] * H + cfg["vocab"] * f + M * H * f,
        # the persistent kernel: the whole step but the embedding gather
        "step": decode_step_bytes(cfg, [kv_len - 1] * M),
    }


# ---------------------------------------------------------- CPU baseline ----
_CPU_STATE = {}


def cpu_decoder(cfg, seed):
    if "dec" not in _CPU_STATE:
        from oracle import pyoracle
        from qwenasr_b200 import synthetic
        w = synthetic.decoder_weights_np(cfg, seed)
        _CPU_STATE["w"] = w
        _CPU_STATE["dec"] = pyoracle.OracleDecoder(w)
        _CPU_STATE["orc"] = pyoracle
    return _CPU_STATE["dec"], _CPU_STATE["w"], _CPU_STATE["orc"]


def cpu_time_tokens(cfg, kv_len, n_tokens, seed, threads):
    """decoder_forward_int8 of the oracle on the host: n_tokens single-sequence
    steps at position kv_len-1.  Returns seconds per token."""
    dec, w, orc = cpu_decoder(cfg, seed)
    orc.set_threads(threads)
    if "kv" not in _CPU_STATE:
        k, v = dec.new_kv(kv_len)
        rng = np.random.default_rng(seed + 1)
        k[:, :kv_len - 1] = rng.standard_normal((k.shape[0], kv_len - 1, k.shape[2]), np.float32)
        v[:, :kv_len - 1] = rng.standard_normal((v.shape[0], kv_len - 1, v.shape[2]), np.float32)
        _CPU_STATE["kv"] = (k, v)
    k, v = _CPU_STATE["kv"]
    tok = 17
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        tok, _, _ = dec.forward(k, v, kv_len - 1, w["embed"][tok])
    return (time.perf_counter() - t0) / n_tokens


def cpu_threads():
    return max(1, min(16, os.cpu_count() or 1))  # the reference pool caps at MAX_THREADS = 16 (mod.rs:177)


def cpu_baseline(cfg, kv_len, seed, seconds):
    th = cpu_threads()
    per = cpu_time_tokens(cfg, kv_len, 1, seed, th)  # warm-up + estimate
    n = max(2, int(seconds / max(per, 1e-3)))
    per = cpu_time_tokens(cfg, kv_len, n, seed, th)
    return {"value": 1.0 / per, "unit": UNIT, "cores": th, "kind": "port",
            "sample": f"{n} single-sequence decode steps of the oracle restatement at KV length {kv_len} "
                      f"(0.6B shapes, 28 layers, 151936-row lm head), {th} threads of {os.cpu_count()} host cores"}


# ------------------------------------------------------------- reference ----
def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from qwenasr_b200 import synthetic
    cfg = synthetic.DEC_0_6B
    th = cpu_threads()
    est = cpu_time_tokens(cfg, a.kv_len, 1, a.seed, th)
    # one step = the M sequences decoded one after another (the reference has
    # no batching); shrink to fewer sequences per step when K steps of the full
    # batch would not finish within ~3 minutes
    per_step_seqs = a.batch
    budget = 180.0
    while per_step_seqs > 1 and est * per_step_seqs * (a.steps + a.warmup) > budget:
        per_step_seqs -= 1
    for _ in range(a.warmup):
        cpu_time_tokens(cfg, a.kv_len, per_step_seqs, a.seed, th)
    times = [cpu_time_tokens(cfg, a.kv_len, per_step_seqs, a.seed, th) * per_step_seqs for _ in range(a.steps)]
    step_s = sum(times) / len(times)
    value = per_step_seqs / step_s
    sample = (f"{per_step_seqs} of {a.batch} sequences per step, decoded sequentially like transcribe_segment; "
              f"oracle restatement of decoder_forward_int8 on {th} threads of {os.cpu_count()} host cores")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xf32", "data": "synthetic (seeded random-init weights, random KV history)",
            "impl": "reference",
            "hardware": (f"host CPU only: one process (rank 0 of {world}) on {th} threads; the reference has no "
                         f"GPU path, so this value does not grow with n_gpus"),
            "config": decode_config(a, cfg, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": th, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------- ours ----
def run_ours(a):
    import torch
    rank, local, world, dist = init_dist(600)
    from qwenasr_b200 import kernels as K
    from qwenasr_b200 import synthetic
    from qwenasr_b200.decoder import Decoder

    cfg = dict(synthetic.DEC_0_6B if a.model == "0.6b" else synthetic.DEC_1_7B, n_layers=a.layers)
    M, L = a.batch, a.kv_len
    dev = torch.device(f"cuda:{local}")
    dec = Decoder(cfg, device=local, max_batch=M, max_seq=L)
    dec.set_step_kernel(a.step_kernel)
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed)

    def qz(w):
        q = torch.empty(w.shape, dtype=torch.int8, device=dev)
        s = torch.empty(w.shape[0], dtype=torch.float32, device=dev)
        K.quantize_f32_to_int8(w, w.shape[0], w.shape[1], q, s)
        return q, s

    for i in range(cfg["n_layers"]):
        dec.set_layer(i, synthetic.layer_weights_gpu(cfg, gen, dev, qz))
    emb = torch.randn(cfg["vocab"], cfg["hidden"], generator=gen, device=dev) * 0.02
    lm, lms = qz(emb)
    norm = 1.0 + 0.02 * torch.randn(cfg["hidden"], generator=gen, device=dev)
    dec.set_globals(emb, norm, lm, lms)
    del lm, lms
    for m in range(M):
        k, v = dec.kv(m)
        k[:, :L - 1].normal_(generator=gen)
        v[:, :L - 1].normal_(generator=gen)
    torch.cuda.synchronize()

    tokens0 = torch.randint(0, cfg["vocab"], (M,), generator=gen, device=dev, dtype=torch.int32)
    positions = torch.full((M,), L - 1, dtype=torch.int32, device=dev)
    tok = tokens0.clone()
    st = dec.stream
    for _ in range(max(a.warmup, 3)):
        dec.step_device(tok, positions, tok)
    st.synchronize()

    def barrier():
        if dist:
            dist.barrier()

    # ---- device-timed region: K steps, inputs resident, tokens fed back ----
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev0.record(st)
        for _ in range(a.steps):
            dec.step_device(tok, positions, tok)
        ev1.record(st)
        st.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / a.steps
    ms_t = torch.tensor([ms], device=dev)
    if dist:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())

    # ---- e2e: the public host-buffer API, H2D ids+positions, D2H next ids ----
    host_tok = tokens0.cpu().numpy()
    host_pos = positions.cpu().numpy()
    for _ in range(max(a.warmup, 3)):
        host_tok = dec.step(host_tok, host_pos)
    barrier()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        host_tok = dec.step(host_tok, host_pos)
    e2e_s = (time.perf_counter() - t0) / a.steps
    barrier()
    e2e_t = torch.tensor([e2e_s], device=dev)
    if dist:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_s = float(e2e_t.item())

    # ---- live per-class kernel timing (eager step with events) ----
    prof = None
    for _ in range(3):
        prof = dec.profile_step(host_tok, host_pos)
    cb = class_bytes(cfg, M, L)
    # ---- in-step timing: the graph-replayed step with %globaltimer stamps
    # (first CTA past its dependency wait .. last CTA exit per launch), the
    # kernels as they overlap inside the timed region ----
    in_step = in_step_classes(dec, host_tok, host_pos, cfg["n_layers"]) if a.step_kernel != 0 else None
    src = in_step if in_step else prof
    dom = max(src, key=lambda k: src[k][0])
    dom_ms, dom_n = src[dom]
    per_launch_s = dom_ms / 1e3 / dom_n
    peak, peak_kind = peaks()
    achieved = cb[dom] / per_launch_s / 1e9
    launches_per_step = sum(n for _, n in prof.values())
    step_bytes = dec.step_bytes(host_pos)

    line = None
    if rank == 0:
        value = world * M / (ms / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xf32",
            "data": "synthetic (seeded random-init weights, random KV history)",
            "config": decode_config(a, cfg, world),
            "e2e": {"value": world * M / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 2 * 4 * M,
                    "d2h_bytes_per_step": 4 * M + 4},
            "gpu_launches": launches_per_step * a.steps,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (NCU_TRAFFIC_M8.get(dom)
                                     if (M, L, cfg["n_layers"], a.model) == (8, 1024, 28, "0.6b") else None),
                         "traffic_source": "committed constant (NCU_TRAFFIC_M8) copied from one earlier ncu capture of this "
                                           "workload (profiles/); not measured by this run", "peak_kind": peak_kind,
                         "bytes_per_launch": cb[dom], "us_per_launch": per_launch_s * 1e6,
                         "timing": ("in-step: %globaltimer stamps in the graph-replayed step, first CTA past its "
                                    "dependency wait to last CTA exit, mean over the class's launches"
                                    if in_step else "eager step, CUDA events around each launch")},
            "step_roofline": {"bytes": step_bytes, "achieved_gbs": step_bytes / (ms / 1e3) / 1e9,
                              "frac": step_bytes / (ms / 1e3) / 1e9 / peak},
            "kernel_ms_per_step": {k: round(v[0], 4) for k, v in prof.items()},
            "kernel_ms_in_step": ({k: round(v[0], 4) for k, v in in_step.items()} if in_step else None),
            "clocks": clk.summary(),
        }
    if dist:
        dist.barrier()
    dec.close()
    del dec
    torch.cuda.synchronize()
    if not a.no_extras and a.model == "0.6b" and a.layers == 28:
        # the transcription configurations, measured in the same run so that
        # every n_gpus of a scaling run records them
        # (64 segments split over the GPUs, the partitioned mode) and
        # configs[3] (one 30 s segment per GPU)
        seg = measure_transcribe(a, "segments", rank, local, world, dist, 2, 2, None, None, False)
        e2e4 = measure_transcribe(a, "e2e", rank, local, world, dist, 2, 2, None, None, False)
        if rank == 0:
            line["segments_cfg5"] = _sub_line(seg)
            line["e2e_cfg4"] = _sub_line(e2e4)
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, L, a.seed, a.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def in_step_classes(dec, tokens, positions, n_layers, reps=3):
    """{class: (ms summed over the step's launches, launches)} from the
    per-launch stamps of a graph-replayed step (Decoder.trace_step); the last
    of `reps` traced steps (the first re-captures the graph)."""
    t = None
    for _ in range(reps):
        t = dec.trace_step(tokens, positions)
    names = ("qkv", "attn", "oproj", "gateup", "down")
    out = {}
    for i in range(t.shape[0]):
        k = "lmhead" if i == 5 * n_layers else names[i % 5]
        s, e = int(t[i, 0]), int(t[i, 1])
        if e <= s or s == (1 << 64) - 1:
            return None  # a launch wrote no stamps
        ms, n = out.get(k, (0.0, 0))
        out[k] = (ms + (e - s) / 1e6, n + 1)
    return out


def _sub_line(line):
    keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "scaling", "config",
            "decode_tokens_per_s", "phase_ms_rank0", "e2e", "roofline", "gpu_launches", "clocks")
    return {k: line[k] for k in keep if k in line}


def decode_config(a, cfg, world):
    """The `config` of the decode line, shared by both arms."""
    return {"workload": ("INT8 decode step, Qwen3-ASR-0.6B decoder shapes (BASELINE configs[2])"
                         if a.model == "0.6b" else "INT8 decode step, Qwen3-ASR-1.7B decoder shapes"),
            "batch_per_gpu": a.batch, "kv_len": a.kv_len, "layers": cfg["n_layers"], "vocab": cfg["vocab"],
            "parallelism": f"replicas x{world} (no collective)",
            "decode_step": ("one persistent kernel per step" if a.step_kernel == 0
                            else "per-layer kernels (5 launches per layer)"),
            "l2": f"inputs larger than L2: "
                  f"{decode_step_bytes(cfg, [a.kv_len - 1] * a.batch) / 1e9:.2f} GB read per step"}


def decode_step_bytes(cfg, positions):
    """Algorithmic bytes of one decode step (qasr_decoder_step_bytes): every
    weight, scale and norm once, the lm head, K/V rows 0..pos per sequence."""
    H, I, hd, L = cfg["hidden"], cfg["inter"], cfg["head_dim"], cfg["n_layers"]
    q, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    w_layer = (q + 2 * kv) * H + H * q + 2 * I * H + H * I
    s_layer = 4 * ((q + 2 * kv) + H + 2 * I + H)
    n_layer = 4 * (2 * hd + 2 * H)
    b = L * (w_layer + s_layer + n_layer) + cfg["vocab"] * H + 4 * cfg["vocab"]
    return b + sum(L * 2 * (p + 1) * kv * 4 for p in positions)


# ------------------------------------------------------------ prefill GEMM --
GEMM_SHAPES = [  # (name, tokens, out, in, bias): 0.6B decoder layer prefill + encoder layer
    ("dec_qkv", 404, 4096, 1024, False), ("dec_o", 404, 1024, 2048, False),
    ("dec_gate_up", 404, 6144, 1024, False), ("dec_down", 404, 1024, 3072, False),
    ("enc_q", 390, 896, 896, True), ("enc_k", 390, 896, 896, True), ("enc_v", 390, 896, 896, True),
    ("enc_o", 390, 896, 896, True), ("enc_fc1", 390, 3584, 896, True), ("enc_fc2", 390, 896, 3584, True),
]


def run_gemm(a):
    import torch
    from qwenasr_b200 import kernels as K
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed)
    ops = []
    for name, T, O, I, bias in GEMM_SHAPES:
        wf = torch.randn(O, I, generator=gen, device=dev) * 0.02
        w = torch.empty(O, I, dtype=torch.int8, device=dev)
        sc = torch.empty(O, device=dev)
        K.quantize_f32_to_int8(wf, O, I, w, sc)
        x = torch.randn(T, I, generator=gen, device=dev)
        b = torch.randn(O, generator=gen, device=dev) * 0.1 if bias else None
        y = torch.empty(T, O, device=dev)
        ops.append((name, T, O, I, w, sc, x, b, y))
    flops = sum(2.0 * T * O * I for _, T, O, I, *_ in ops)
    weight_bytes = sum(O * I + 4 * O for _, T, O, I, *_ in ops)
    # L2 flush between steps by READING a buffer larger than L2: a write would
    # leave dirty lines whose write-back lands inside the next timed step
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def flush_l2():
        return flush_buf.sum()

    def step():
        for name, T, O, I, w, sc, x, b, y in ops:
            if b is None:
                K.linear_nobias_int8(y, x, w, sc, T, I, O)
            else:
                K.linear_int8(y, x, w, sc, b, T, I, O)

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with ClockSampler(0) as clk:
        for e0, e1 in evs:
            flush_l2()
            e0.record()
            step()
            e1.record()
        torch.cuda.synchronize()
    ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / a.steps
    # per-op timing, for the table in the design notes
    per_op = {}
    for name, T, O, I, w, sc, x, b, y in ops:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush_l2()
        e0.record()
        for _ in range(5):
            if b is None:
                K.linear_nobias_int8(y, x, w, sc, T, I, O)
            else:
                K.linear_int8(y, x, w, sc, b, T, I, O)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / 5
        per_op[name] = {"us": round(us, 2), "tflops": round(2.0 * T * O * I / us / 1e6, 1)}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        peak_kind = "measured bf16 x2 (int8 dense rate is twice bf16)"
    except Exception:
        bf16, peak_kind = 1590.0, "fallback bf16 x2"
    int8_tops = 3.0 * flops / (ms / 1e3) / 1e12  # three digit rows per activation row
    line = {
        "metric": "INT8 prefill/encoder projection throughput (f32-equivalent 2*T*in*out)", "value":
            flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "int8xf32",
        "data": "synthetic (seeded random-init weights and activations)",
        "config": {"workload": "decoder layer prefill (404 tokens) + encoder layer (390 tokens), 0.6B shapes",
                   "shapes": [list(sh) for sh in GEMM_SHAPES], "l2": "flushed before every step by reading 256 MB"},
        "roofline": {"bound": "tensor", "achieved": int8_tops, "peak": 2.0 * bf16, "unit": "TOPS (int8 MMA)",
                     "frac": int8_tops / (2.0 * bf16), "traffic": None, "peak_kind": peak_kind,
                     "weight_bytes_per_step": weight_bytes},
        "per_op": per_op,
        "clocks": clk.summary(),
    }
    if not a.no_cpu_baseline:
        # oracle (generic::int8_matvec_fused restated), all host threads, on 8 rows of every shape
        from oracle import pyoracle
        threads = cpu_threads()
        pyoracle.set_threads(threads)
        rng = np.random.default_rng(a.seed)
        t_cpu, f_cpu = 0.0, 0.0
        for name, T, O, I, w, sc, x, b, y in ops:
            xs = rng.standard_normal((8, I)).astype(np.float32)
            wn, sn = w.cpu().numpy(), sc.cpu().numpy()
            t0 = time.perf_counter()
            pyoracle.linear_nobias_int8(xs, wn, sn)
            t_cpu += time.perf_counter() - t0
            f_cpu += 2.0 * 8 * O * I
        line["cpu_baseline"] = {"value": f_cpu / t_cpu / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                "sample": "8 rows of each of the 10 projections (the reference runs seq_len "
                                          "sequential matvecs, so per-row cost is independent of T)"}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------ fused row kernels (cfg1/2) --
# the decoder pre-attention block at 0.6B shapes.
PRE_ATTN = dict(seq=512, hidden=1024, n_heads=16, n_kv=8, head_dim=128, capacity=4096, eps=1e-6, theta=1e6)
# the encoder elementwise steps, batch 8 x 375 frames.
ENC_ELEM = dict(rows=3000, d=896, n_pos=375, ffn=3584, eps=1e-5)


def pre_attn_bytes(c):
    """Algorithmic bytes of one config-1 block: x read, x_norm written, q read
    and written, k and v read, their cache rows written (norm weights and the
    RoPE rows are below 0.1 % and not counted)."""
    S, H, q, kv = c["seq"], c["hidden"], c["n_heads"] * c["head_dim"], c["n_kv"] * c["head_dim"]
    return 4 * S * (2 * H + 2 * q + 2 * kv + 2 * kv)


def enc_elem_bytes(c):
    """LN+PE: x read, out written; GELU: the FFN activation read and written."""
    return 4 * c["rows"] * c["d"] * 2 + 4 * c["rows"] * c["ffn"] * 2


class _Graph:
    """A CUDA graph of `fn` called once per input set (the sets together
    exceed L2, so every launch reads cold data)."""

    def __init__(self, torch, fn, n_sets):
        self.torch = torch
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for i in range(n_sets):  # warm-up outside the capture (attribute opt-ins)
                fn(i)
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        self.g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g):
            for i in range(n_sets):
                fn(i)
        self.n = n_sets

    def time_ms(self, reps):
        """Device time per launch: CUDA events around `reps` replays."""
        torch = self.torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            self.g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (reps * self.n)


def _row_kernel_line(a, metric, workload_cfg, bytes_step, ms, kernels, e2e_ms, h2d, d2h, cpu, clk, n_sets, set_bytes):
    peak, peak_kind = peaks()
    gbs = bytes_step / (ms / 1e3) / 1e9
    dom = max(kernels, key=lambda k: kernels[k]["us"])
    kd = kernels[dom]
    return {
        "metric": metric, "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, N(1,0.02) / N(0,0.02) norm weights)",
        "config": dict(workload_cfg, l2=f"{n_sets} input sets of {set_bytes / 1e6:.1f} MB used in turn "
                                        f"({n_sets * set_bytes / 1e6:.0f} MB > 126 MB L2): every launch reads "
                                        f"cold data"),
        "e2e": {"value": bytes_step / (e2e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": sum(k["launches_per_step"] for k in kernels.values()) * a.steps,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": kd["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": kd["gbs"] / peak, "traffic": None,
                     "traffic_note": "dram bytes of one launch are in profiles/ (ncu)", "peak_kind": peak_kind,
                     "bytes_per_launch": kd["bytes"], "us_per_launch": kd["us"]},
        "kernels": kernels,
        "cpu_baseline": cpu,
        "timing": "CUDA events around replays of a CUDA graph holding one launch per input set",
        "clocks": clk.summary(),
    }


def run_pre_attn(a):
    """BASELINE configs[0] through qasr_pre_attn_block (kernels.pre_attn_block)."""
    import torch
    from qwenasr_b200 import kernels as K
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    c = PRE_ATTN
    S, H, nh, nkv, hd, cap = c["seq"], c["hidden"], c["n_heads"], c["n_kv"], c["head_dim"], c["capacity"]
    q_dim, kv = nh * hd, nkv * hd
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed)
    cos = torch.empty(cap, hd, device=dev)
    sin = torch.empty(cap, hd, device=dev)
    K.rope_cache_table(cos, sin, cap, hd, c["theta"])
    w_in = 1 + 0.02 * torch.randn(H, generator=gen, device=dev)
    qw = 1 + 0.02 * torch.randn(hd, generator=gen, device=dev)
    kw = 1 + 0.02 * torch.randn(hd, generator=gen, device=dev)
    set_bytes = pre_attn_bytes(c)
    n_sets = 8
    sets = []
    for _ in range(n_sets):
        sets.append(dict(x=torch.randn(S, H, generator=gen, device=dev), xn=torch.empty(S, H, device=dev),
                         q=torch.randn(S, q_dim, generator=gen, device=dev),
                         k=torch.randn(S, kv, generator=gen, device=dev),
                         v=torch.randn(S, kv, generator=gen, device=dev),
                         kc=torch.zeros(cap, kv, device=dev), vc=torch.zeros(cap, kv, device=dev)))

    def call(i, s=None):
        s = s or sets[i]
        K.pre_attn_block(s["xn"], s["x"], w_in, S, H, s["q"], s["k"], s["v"], None, qw, kw, nh, nkv, hd, c["eps"],
                         cos, sin, 0, s["kc"], s["vc"], 0, cap)

    g = _Graph(torch, call, n_sets)
    reps = max(1, -(-a.steps // n_sets))
    for _ in range(max(a.warmup, 3)):
        g.time_ms(1)
    with ClockSampler(0) as clk:
        ms = g.time_ms(reps)
    kernels = {"pre_attn_block_kernel": {"us": ms * 1e3, "bytes": set_bytes, "gbs": set_bytes / (ms / 1e3) / 1e9,
                                         "launches_per_step": 1}}
    # e2e: pinned host inputs -> device, the C-ABI call, results -> pinned host
    hx = torch.randn(S, H).pin_memory()
    hq = torch.randn(S, q_dim).pin_memory()
    hk = torch.randn(S, kv).pin_memory()
    hv = torch.randn(S, kv).pin_memory()
    hxn = torch.empty(S, H).pin_memory()
    hqo = torch.empty(S, q_dim).pin_memory()
    hkc = torch.empty(S, kv).pin_memory()
    hvc = torch.empty(S, kv).pin_memory()
    s0 = sets[0]

    def e2e_step():
        s0["x"].copy_(hx, non_blocking=True)
        s0["q"].copy_(hq, non_blocking=True)
        s0["k"].copy_(hk, non_blocking=True)
        s0["v"].copy_(hv, non_blocking=True)
        call(0)
        hxn.copy_(s0["xn"], non_blocking=True)
        hqo.copy_(s0["q"], non_blocking=True)
        hkc.copy_(s0["kc"][:S], non_blocking=True)
        hvc.copy_(s0["vc"][:S], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / a.steps
    h2d = 4 * S * (H + q_dim + 2 * kv)
    d2h = 4 * S * (H + q_dim + 2 * kv)
    cpu = None
    if not a.no_cpu_baseline:
        from oracle import pyoracle as orc
        xs = [t.cpu().numpy() for t in (sets[0]["x"], w_in, sets[0]["q"], sets[0]["k"], sets[0]["v"], qw, kw)]
        ch, sh = cos.cpu().numpy(), sin.cpu().numpy()
        kc = np.zeros((cap, kv), np.float32)
        vc = np.zeros((cap, kv), np.float32)
        n, t_cpu = 0, 0.0
        while t_cpu < min(a.cpu_seconds, 10.0) or n < 3:
            t0 = time.perf_counter()
            orc.pre_attn_block(xs[0], xs[1], xs[2], xs[3], xs[4], xs[5], xs[6], nh, nkv, hd, c["eps"], ch, sh, 0,
                               kc, vc)
            t_cpu += time.perf_counter() - t0
            n += 1
        cpu = {"value": set_bytes * n / t_cpu / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{n} whole config-1 blocks of the oracle restatement (rms_norm, rms_norm_per_head, "
                         f"apply_rope_neox, KV append in the reference's order), 1 thread like the reference's "
                         f"norm kernels"}
    line = _row_kernel_line(
        a, "decoder pre-attention block HBM throughput (RMSNorm + q/k per-head norm + RoPE + KV append)",
        {"workload": "BASELINE configs[0]: S=512 rows at Qwen3-0.6B shapes, positions 0..511, KV capacity 4096",
         "seq": S, "hidden": H, "heads": [nh, nkv], "head_dim": hd}, set_bytes, ms, kernels, e2e_ms, h2d, d2h, cpu,
        clk, n_sets, set_bytes)
    print(json.dumps(line), flush=True)
    return 0


def run_enc_elementwise(a):
    """BASELINE configs[1] through qasr_ln_pe_gelu_erf (one launch), with the
    two separate entries qasr_ln_pe + qasr_gelu_erf timed beside it."""
    import torch
    from qwenasr_b200 import kernels as K
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    c = ENC_ELEM
    R, D, P, F = c["rows"], c["d"], c["n_pos"], c["ffn"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed)
    g_ = 1 + 0.02 * torch.randn(D, generator=gen, device=dev)
    b_ = 0.02 * torch.randn(D, generator=gen, device=dev)
    pe = torch.empty(P, D, device=dev)
    K.sinusoidal_pe(pe, P, D)
    set_bytes = enc_elem_bytes(c)
    n_sets = 3
    sets = [dict(x=torch.randn(R, D, generator=gen, device=dev), out=torch.empty(R, D, device=dev),
                 act=torch.randn(R * F, generator=gen, device=dev)) for _ in range(n_sets)]

    def fused(i):
        s = sets[i]
        K.ln_pe_gelu_erf(s["out"], s["x"], g_, b_, pe, R, D, P, c["eps"], s["act"], R * F)

    def ln_only(i):
        s = sets[i]
        K.ln_pe(s["out"], s["x"], g_, b_, pe, R, D, P, c["eps"])

    def gelu_only(i):
        K.gelu_erf(sets[i]["act"], R * F)

    graphs = {n: _Graph(torch, f, n_sets) for n, f in (("ln_pe_gelu_kernel", fused), ("layer_norm_kernel", ln_only),
                                                       ("gelu_erf_kernel", gelu_only))}
    reps = max(1, -(-a.steps // n_sets))
    for g in graphs.values():
        for _ in range(max(a.warmup, 3)):
            g.time_ms(1)
    with ClockSampler(0) as clk:
        ms = graphs["ln_pe_gelu_kernel"].time_ms(reps)
        ms_ln = graphs["layer_norm_kernel"].time_ms(reps)
        ms_ge = graphs["gelu_erf_kernel"].time_ms(reps)
    ln_b, ge_b = 4 * R * D * 2, 4 * R * F * 2
    kernels = {"ln_pe_gelu_kernel": {"us": ms * 1e3, "bytes": set_bytes, "gbs": set_bytes / (ms / 1e3) / 1e9,
                                     "launches_per_step": 1},
               "separate: layer_norm_kernel (qasr_ln_pe)": {"us": ms_ln * 1e3, "bytes": ln_b,
                                                            "gbs": ln_b / (ms_ln / 1e3) / 1e9,
                                                            "launches_per_step": 0},
               "separate: gelu_erf_kernel (qasr_gelu_erf)": {"us": ms_ge * 1e3, "bytes": ge_b,
                                                             "gbs": ge_b / (ms_ge / 1e3) / 1e9,
                                                             "launches_per_step": 0}}
    hx = torch.randn(R, D).pin_memory()
    ha = torch.randn(R * F).pin_memory()
    ho = torch.empty(R, D).pin_memory()
    hao = torch.empty(R * F).pin_memory()
    s0 = sets[0]

    def e2e_step():
        s0["x"].copy_(hx, non_blocking=True)
        s0["act"].copy_(ha, non_blocking=True)
        fused(0)
        ho.copy_(s0["out"], non_blocking=True)
        hao.copy_(s0["act"], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / a.steps
    h2d = d2h = 4 * (R * D + R * F)
    cpu = None
    if not a.no_cpu_baseline:
        from oracle import pyoracle as orc
        x_h, g_h, b_h, pe_h = (t.cpu().numpy() for t in (s0["x"], g_, b_, pe))
        act_h = s0["act"].cpu().numpy()
        pe_rows = pe_h[np.arange(R) % P]
        n, t_cpu = 0, 0.0
        while t_cpu < min(a.cpu_seconds, 10.0) or n < 2:
            t0 = time.perf_counter()
            _ = orc.layer_norm(x_h, g_h, b_h, c["eps"]) + pe_rows
            _ = orc.gelu_erf(act_h)
            t_cpu += time.perf_counter() - t0
            n += 1
        cpu = {"value": set_bytes * n / t_cpu / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"{n} whole config-2 passes of the oracle restatement (layer_norm_row AVX order + PE "
                         f"add + erff GELU), 1 thread like the reference's row kernels"}
    line = _row_kernel_line(
        a, "encoder elementwise HBM throughput (LayerNorm + sinusoidal PE, exact-erf GELU)",
        {"workload": "BASELINE configs[1]: LN + PE on [3000, 896] (8 items x 375 frames), erf GELU on "
                     "[3000, 3584]", "rows": R, "d_model": D, "ffn": F}, set_bytes, ms, kernels, e2e_ms, h2d, d2h,
        cpu, clk, n_sets, set_bytes)
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- encoder --
def encoder_flops(cfg, frames):
    """f32-equivalent multiply-adds x 2 of Encoder::forward for `frames` mel frames."""
    CH, D, F, O, cs = 480, cfg["d_model"], cfg["ffn_dim"], cfg["output_dim"], cfg["chunk_size"]
    fl, T = 0.0, 0
    for s0 in range(0, frames, cs):
        w = min(cs, frames - s0)
        h1, w1 = 64, (w - 1) // 2 + 1
        h2, w2 = 32, (w1 - 1) // 2 + 1
        h3, w3 = 16, (w2 - 1) // 2 + 1
        fl += 2.0 * CH * 9 * h1 * w1 + 2.0 * CH * CH * 9 * (h2 * w2 + h3 * w3) + 2.0 * w3 * CH * h3 * D
        T += w3
    wsize = 13 * (cfg["n_window_infer"] // cs)
    att = sum(2.0 * 2 * min(wsize, T - s0) ** 2 * D for s0 in range(0, T, wsize))
    fl += cfg["n_layers"] * (2.0 * T * (4 * D * D + 2 * D * F) + att) + 2.0 * T * (D * D + D * O)
    return fl, T


def run_encoder(a):
    import torch
    from qwenasr_b200 import synthetic
    from qwenasr_b200.encoder import Encoder
    torch.cuda.set_device(0)
    cfg = synthetic.ENC_0_6B
    frames = 3000  # one 30 s segment: 100 mel frames per second
    enc = Encoder(cfg, device=0)
    enc.set_weights(synthetic.encoder_weights_np(cfg, a.seed))
    mel_h = np.random.default_rng(a.seed).standard_normal((128, frames)).astype(np.float32)
    mel = torch.from_numpy(mel_h).cuda()
    for _ in range(max(a.warmup, 3)):
        enc.forward(mel)
    torch.cuda.synchronize()
    times = []
    with ClockSampler(0) as clk:
        for _ in range(a.steps):
            t0 = time.perf_counter()
            enc.forward(mel)  # synchronous: the engine waits for its stream
            times.append(time.perf_counter() - t0)
    # e2e: host mel in, host encoder rows out
    e2e = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        enc.forward(mel_h).cpu()
        e2e.append(time.perf_counter() - t0)
    s = statistics.median(times)
    fl, T = encoder_flops(cfg, frames)
    line = {"metric": "encoder audio seconds per second (Encoder::forward, Qwen3-ASR-0.6B encoder shapes)",
            "value": 30.0 / s, "unit": "audio-s/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": s * 1e3, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
            "dtype": "f32 (int8 digit planes on tcgen05)", "data": "synthetic (seeded weights, N(0,1) log-mel)",
            "config": {"workload": "one 30 s segment: 3000 mel frames -> %d tokens, 18 layers" % T},
            "tflops_f32_equivalent": fl / s / 1e12, "flops_per_step": fl,
            "e2e": {"value": 30.0 / statistics.median(e2e), "unit": "audio-s/s",
                    "h2d_bytes_per_step": 128 * frames * 4, "d2h_bytes_per_step": T * cfg["output_dim"] * 4},
            "timing": "host wall clock around the synchronous forward (median of steps)",
            "clocks": clk.summary()}
    enc.close()
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------- transcription --
TRANSCRIBE = {
    "e2e": dict(dec="DEC_0_6B", enc="ENC_0_6B", segments_per_rank=1, seconds=30.0, new=256, batch=1, lanes=1,
                scaling="weak", desc="BASELINE configs[3]: one 30 s segment per GPU, Qwen3-ASR-0.6B shapes "
                                     "(INT8 decoder, f32 encoder), 256 greedy tokens"),
    "segments": dict(dec="DEC_1_7B", enc="ENC_1_7B", segments=64, seconds=30.0, new=128, batch=8, lanes=4,
                     scaling="strong", desc="BASELINE configs[4]: 64 segments of 30 s split evenly over the GPUs, "
                                            "Qwen3-ASR-1.7B shapes (INT8 decoder, f32 encoder), 128 greedy tokens "
                                            "each, 8 segments per decode batch"),
}


def cpu_transcribe_baseline(dcfg, ecfg, seconds, new, seed, budget_s):
    """The oracle on the host cores, per segment: log-mel and encoder over the
    whole segment, prefill and decode on a sample of the positions, scaled to
    the segment's prompt and token counts."""
    from oracle import pyoracle as orc
    from qwenasr_b200 import synthetic
    th = cpu_threads()
    orc.set_threads(th)
    audio = synthetic.synthetic_audio(seconds, seed)
    t0 = time.perf_counter()
    mel = orc.mel_spectrogram(audio)
    t_mel = time.perf_counter() - t0
    we = synthetic.encoder_weights_np(ecfg, seed)
    t0 = time.perf_counter()
    rows = orc.encoder_forward(we, ecfg, mel)
    t_enc = time.perf_counter() - t0
    del we
    wd = synthetic.decoder_weights_np(dcfg, seed)
    od = orc.OracleDecoder(wd)
    prompt = 15 + rows.shape[0]
    k, v = od.new_kv(prompt + 8)
    n_pre = max(1, min(prompt - 1, int(budget_s / 4 / 0.05)))
    t0 = time.perf_counter()
    od.prefill(k, v, 0, rows[:n_pre])
    t_pre = (time.perf_counter() - t0) / n_pre * (prompt - 1)
    n_dec = 3
    t0 = time.perf_counter()
    tok = 198
    for i in range(n_dec):
        tok, _, _ = od.forward(k, v, n_pre + i, wd["embed"][tok])
    t_dec = (time.perf_counter() - t0) / n_dec * new
    total = t_mel + t_enc + t_pre + t_dec
    return {"value": seconds / total, "unit": "audio-s/s", "cores": th, "kind": "port",
            "sample": f"one {seconds:.0f} s segment: oracle log-mel and encoder over all of it "
                      f"({t_mel:.2f} s + {t_enc:.2f} s), prefill timed on {n_pre} of {prompt - 1} rows and "
                      f"decode on {n_dec} of {new} steps, both scaled linearly; {th} threads of "
                      f"{os.cpu_count()} host cores",
            "phase_s": {"mel": t_mel, "encoder": t_enc, "prefill_est": t_pre, "decode_est": t_dec}}


def init_dist(timeout_s):
    """One process per GPU (torchrun env); NCCL group for the timing barriers
    and max-over-ranks reductions only."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device(f"cuda:{local}"))
    return rank, local, world, dist


def run_transcribe(a):
    rank, local, world, dist = init_dist(600)
    line = measure_transcribe(a, a.workload, rank, local, world, dist, a.steps, a.warmup, a.lanes,
                              a.segments if a.workload == "segments" else None, not a.no_cpu_baseline)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def measure_transcribe(a, workload, rank, local, world, dist, steps, warmup, lanes_opt, segments_opt, with_cpu):
    """One transcription workload (TRANSCRIBE[workload]) on this rank's share
    of the segments; returns the JSON line on rank 0 (None elsewhere)."""
    import torch
    from qwenasr_b200 import kernels as K
    from qwenasr_b200 import synthetic
    from qwenasr_b200.decoder import Decoder
    from qwenasr_b200.encoder import Encoder
    from qwenasr_b200.segments import segment_range
    from qwenasr_b200.transcribe import prompt_len, transcribe_lanes

    spec = TRANSCRIBE[workload]
    dcfg = dict(getattr(synthetic, spec["dec"]), n_layers=a.layers)
    ecfg = getattr(synthetic, spec["enc"])
    n_seg = segments_opt or spec.get("segments", spec.get("segments_per_rank", 1) * world)
    mine = list(segment_range(n_seg, rank, world))
    new, batch, secs = spec["new"], spec["batch"], spec["seconds"]
    dev = torch.device(f"cuda:{local}")
    # lanes take full batches (qasr_transcribe_lanes): more lanes than batches would idle
    n_lanes = max(1, min(lanes_opt or spec["lanes"], -(-len(mine) // batch)))
    encs = [Encoder(ecfg, device=local) for _ in range(n_lanes)]
    enc_tokens = encs[0].tokens(K.mel_frames(int(secs * 16000)))
    max_seq = ((prompt_len(enc_tokens) - 1 + new + 63) // 64) * 64
    decs = [Decoder(dcfg, device=local, max_batch=batch, max_seq=max_seq) for _ in range(n_lanes)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(a.seed + 17 * rank)

    def qz(w):
        q = torch.empty(w.shape, dtype=torch.int8, device=dev)
        s = torch.empty(w.shape[0], dtype=torch.float32, device=dev)
        K.quantize_f32_to_int8(w, w.shape[0], w.shape[1], q, s)
        return q, s

    # every lane holds the same weights (its own copy)
    for i in range(dcfg["n_layers"]):
        lw = synthetic.layer_weights_gpu(dcfg, gen, dev, qz)
        for d in decs:
            d.set_layer(i, lw)
        del lw
    emb = torch.randn(dcfg["vocab"], dcfg["hidden"], generator=gen, device=dev) * 0.02
    lm, lms = qz(emb)
    norm = 1.0 + 0.02 * torch.randn(dcfg["hidden"], generator=gen, device=dev)
    for d in decs:
        d.set_globals(emb, norm, lm, lms)
    del lm, lms, emb
    we = synthetic.encoder_weights_gpu(ecfg, gen, dev)
    for e in encs:
        e.set_weights(we)
    del we
    lanes = list(zip(decs, encs))
    dec = decs[0]
    torch.cuda.synchronize()
    audio_h = [synthetic.synthetic_audio(secs, a.seed + s) for s in mine]
    audio_d = [torch.from_numpy(x).to(dev) for x in audio_h]
    torch.cuda.synchronize()

    def one_pass(src, n_new=new):
        return transcribe_lanes(lanes, src, n_new)

    def barrier():
        if dist:
            dist.barrier()

    for _ in range(max(warmup, 1)):
        one_pass(audio_d)
    st = dec.stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev0.record(st)
        for _ in range(steps):
            ids = one_pass(audio_d)
        ev1.record(st)
        st.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / steps
    # e2e: host samples in (H2D inside the call), host ids out
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_pass(audio_h)
    e2e_ms = (time.perf_counter() - t0) / steps * 1e3
    barrier()
    # phase split on this rank: everything but the decode loop (one token)
    t0 = time.perf_counter()
    one_pass(audio_d, 1)
    front_ms = (time.perf_counter() - t0) * 1e3
    t = torch.tensor([ms, e2e_ms], device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    n_batches = (len(mine) + batch - 1) // batch
    dec_step_ms = max(ms - front_ms, 1e-6) / max(1, n_batches * (new - 1))
    mid_pos = np.full(min(batch, len(mine)), prompt_len(enc_tokens) - 1 + new // 2, np.int32)
    step_bytes = dec.step_bytes(mid_pos)
    prof = None
    for _ in range(2):
        prof = dec.profile_step(np.full(len(mid_pos), 198, np.int32), mid_pos)
    launches = sum(n for _, n in prof.values()) * n_batches * new * steps
    peak, peak_kind = peaks()
    line = None
    if rank == 0:
        audio_s = n_seg * secs
        line = {
            "metric": "audio seconds per second (transcription: log-mel, encoder, prefill, greedy decode)",
            "value": audio_s / (ms / 1e3), "unit": "audio-s/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": spec["scaling"],
            "vs_baseline": None, "dtype": "int8xf32 decoder, f32 encoder (int8 digit planes on tcgen05)",
            "data": "synthetic (pink noise + 3 sinusoids at 16 kHz; seeded random-init weights)",
            "config": {"workload": spec["desc"], "segments": n_seg, "seconds_per_segment": secs,
                       "tokens_per_segment": new, "decode_batch": batch, "decoder_layers": dcfg["n_layers"],
                       "hidden": dcfg["hidden"], "encoder_layers": ecfg["n_layers"],
                       "parallelism": f"segments split over {world} GPU(s), no collective; {n_lanes} engine "
                                      f"lane(s) per GPU",
                       "lanes_per_gpu": n_lanes,
                       "l2": "decode steps read weights + KV above L2 size; no flush"},
            "decode_tokens_per_s": n_seg * new / (ms / 1e3),
            "phase_ms_rank0": {"audio_encoder_prefill_first_token": front_ms,
                               "decode_rest": ms - front_ms},
            "e2e": {"value": audio_s / (e2e_ms / 1e3), "unit": "audio-s/s",
                    "h2d_bytes_per_step": int(sum(x.nbytes for x in audio_h)) * world,
                    "d2h_bytes_per_step": n_seg * new * 4},
            "roofline": {"bound": "hbm", "kernel": "decode step (whole graph), estimated from the phase split: "
                                                   "decode-step bytes of all batches over the decode phase "
                                                   "(lanes overlap, so this is the aggregate rate)",
                         "achieved": step_bytes / (dec_step_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": step_bytes / (dec_step_ms / 1e3) / 1e9 / peak, "traffic": None,
                         "peak_kind": peak_kind, "bytes_per_step": step_bytes, "ms_per_decode_step": dec_step_ms},
            "gpu_launches": launches,
            "gpu_launches_note": "decode-step kernels of rank 0 only; mel, encoder and prefill launches come on top",
            "timing": "CUDA events on the decoder stream around whole passes (the call is synchronous)",
            "clocks": clk.summary(),
            "sample_ids": ids[0][:8],
        }
    if dist:
        dist.barrier()
    for d, e in lanes:
        d.close()
        e.close()
    if rank == 0 and world == 1 and with_cpu:
        line["cpu_baseline"] = cpu_transcribe_baseline(dcfg, ecfg, secs, new, a.seed, a.cpu_seconds)
    return line


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)
    if a.workload == "gemm":
        return run_gemm(a)
    if a.workload == "pre_attn":
        return run_pre_attn(a)
    if a.workload == "enc_elementwise":
        return run_enc_elementwise(a)
    if a.workload == "encoder":
        return run_encoder(a)
    if a.workload in TRANSCRIBE:
        return run_transcribe(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
