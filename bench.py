#!/usr/bin/env python
"""Decode benchmark: Qwen2.5-0.5B-shape Q8_0 greedy decode, batch 1, on B200.

Workload (synthetic, seeded): hidden 896, 24 layers, 14/2 heads, head_dim 64,
FFN 4864, vocab 151936, QKV bias, tied embeddings, N(0,0.02) weights
quantised to Q8_0; prompt = BOS + 128 ids uniform over the vocab (seed 0);
prefill, then greedy decode.  One step = one decode token.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload qwen05b|llama3-8b|qwen72b|matvec|attention]

value: decode tok/s over all ranks, device-timed with CUDA events on the
engine's stream (inputs resident in HBM).  e2e: the same tok/s through the C
ABI's per-token call (b2_forward_argmax) with the token id copied from pinned
host memory and the next id read back every step, wall-clock timed.  With
--gpus N > 1 every rank runs an independent replica (this model does not
shard), scaling "weak".  --impl reference times the reference's own CPU
implementation (its C++ engine compiled from the reference sources into
oracle/_ref, else the Go restatement in oracle/) on the host cores.

The other workloads (one GPU, one JSON line per case; not the driver's line):
  llama3-8b  Llama-3-8B-shape Q4_0 greedy decode at batch 1 (hidden 4096, 32
             layers, 32/8 heads, head_dim 128, FFN 14336, vocab 128256, untied),
             prompt 512 ids, then K decode tokens;
  qwen72b    Qwen2.5-72B-shape Q8_0 (hidden 8192, 64/8 heads of 128, FFN 29568,
             vocab 152064, untied) cut to 4 of its 80 layers, tensor-parallel
             over the --gpus N ranks (one process per GPU under torchrun,
             partial sums exchanged by peer stores over NVLink inside the
             decode kernel), prompt 256 ids; value = tok/s of the one model
             (strong scaling), ms_per_step = per-token latency;
  matvec     y = W x through b2_matvec (batch 1) and b2_matvec_batch (batch 8)
             for the Q8_0 and Q4_0 shapes 4096x4096, 14336x4096, 4096x14336,
             128256x4096 (GGUF block layout, W N(0,0.02), x N(0,1)), with
             >= 256 MB of distinct weight copies rotated so that L2 does not
             serve repeats;
  attention  b2_attention_decode, 32 query / 8 KV heads, head_dim 128, fp16 KV
             N(0,1), contexts 4096 / 16384 / 32768, batch 1 and 8, KV copies
             rotated past L2 in the same way;
  gemm       the tcgen05 tensor-core GEMM (b2_model_gemm) on one Llama-3-8B
             layer's Q4_0 matrices for --tokens tokens (512), TFLOP/s against
             the measured dense bf16 peak.
--case picks one case of a microbench (attention 32768x8, matvec
q8_0:128256x4096:1, gemm blk.0.ffn_up.weight).
With --batch B > 1 (qwen05b or llama3-8b, one GPU) the model workload runs as
batched greedy decode (b2_batch_*): B sequences, each prefilled with a prompt
of its own, then K steps of all of them; value = tokens of all sequences per
second.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ai-agent-framework_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

METRIC = "decode tok/s (B=1) and weight-stream HBM GB/s vs 8 TB/s peak"
WORKLOAD = "qwen2.5-0.5b-shape q8_0 greedy decode, batch 1, prompt 128+BOS"
FALLBACK_HBM_GBS = 6650.0


def measured_peaks() -> dict:
    """MEASURED_PEAKS.json as a dict ({} when absent)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """Samples the SM clock and the throttle reasons of this process's GPU
    every 5 ms through NVML (read-only queries) while the timed region runs;
    falls back to `nvidia-smi -lms 200` when NVML is unavailable."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.rows = []  # (sm_mhz, max_mhz, reasons bitmask)
        self.proc = None
        self.stop = threading.Event()
        self.t = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            u = pynvml.nvmlDeviceGetUUID(h)
            u = u.decode() if isinstance(u, bytes) else u
            if self.uuid is None or u == self.uuid:
                return pynvml, h
        raise RuntimeError("GPU not found by NVML")

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)

            def poll():
                while not self.stop.is_set():
                    try:
                        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.rows.append((float(sm), float(mx), int(rs)))
                    except Exception:
                        pass
                    self.stop.wait(0.005)

            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            pass
        try:
            fields = ("uuid,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                      "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                      "clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7 and (self.uuid is None or parts[0] == self.uuid):
                try:
                    mask = sum(bit for k, (_, bit) in enumerate(self.REASONS)
                               if parts[3 + k].lower().startswith("active"))
                    self.rows.append((float(parts[1]), float(parts[2]), mask))
                except ValueError:
                    pass

    def __exit__(self, *a):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=5)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [r[0] for r in self.rows]
        reasons = sorted({name for r in self.rows for name, bit in self.REASONS if r[2] & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": reasons, "samples": len(self.rows)}


def ensure_model(shape_name: str) -> str:
    from b2decode import gguf_writer as gw
    d = os.environ.get("B2_BENCH_DIR", os.path.join(tempfile.gettempdir(), "b2bench"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{shape_name}-s0.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        shape = gw.SHAPES[shape_name]
        if shape.hidden * shape.layers > 1 << 16:
            # multi-GB files: the writer's own process with one worker per host
            # core (fork + exec, so safe after CUDA initialisation)
            env = dict(os.environ, PYTHONPATH=os.path.join(ROOT, "ai-agent-framework_b200"))
            subprocess.run([sys.executable, "-m", "b2decode.gguf_writer", shape_name, tmp], check=True, env=env,
                           stdout=subprocess.DEVNULL)
        else:
            gw.write_model(tmp, shape, seed=0)
        os.replace(tmp, path)
    return path


# The decode workloads: shape, prompt length, description.
MODELS = {
    "qwen05b": ("qwen2.5-0.5b", 128, WORKLOAD),
    "llama3-8b": ("llama3-8b", 512, "llama-3-8b-shape q4_0 greedy decode, batch 1, prompt 512 ids"),
    "qwen72b": ("qwen2.5-72b-4l", 256, "qwen2.5-72b-shape q8_0 (4 of its 80 layers, full widths) tensor-parallel "
                "greedy decode, batch 1, prompt 256 ids"),
}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def profile_traffic(ms_per_step: float) -> tuple:
    """DRAM bytes (read + write) per launch of the decode kernel from the
    committed ncu summary (`dram_bytes_per_launch:`), used only when the
    launch it profiled (`kernel_ms:`) took within 10 % of the timed step;
    returns (bytes or None, a note naming the summary, its commit and time)."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_qwen05b_q8_0.md")
    if not os.path.exists(p):
        return None, "no profile summary"
    vals = {}
    for line in open(p):
        line = line.strip()
        for key in ("dram_bytes_per_launch", "kernel_ms", "commit"):
            if line.startswith(key + ":"):
                vals[key] = line.split(":", 1)[1].strip()
    if "dram_bytes_per_launch" not in vals or "kernel_ms" not in vals:
        return None, "profile summary without traffic or kernel time"
    kms = float(vals["kernel_ms"])
    note = (f"profiles/decode_kernel_qwen05b_q8_0.md (commit {vals.get('commit', '?')}, "
            f"profiled launch {kms:.3f} ms vs timed {ms_per_step:.3f} ms)")
    if abs(kms - ms_per_step) > 0.1 * ms_per_step:
        return None, note + ": more than 10 % apart, traffic not quoted"
    return int(vals["dram_bytes_per_launch"]), note


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), or the platform string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()


def cpu_baseline_goref(path: str, shape_name: str = "qwen2.5-0.5b", seconds: float = 12.0,
                       prefill: int = 16) -> dict:
    """Decode tok/s of the oracle (the Go engine restated, its worker pool with
    one thread per host core) on a bounded sample of the same workload."""
    import goref
    from b2decode import gguf_writer as gw
    shape = gw.SHAPES[shape_name]
    # Q4_0 models: the oracle's ggml-order Q4_0 (the Go engine reads Q4_0
    # matrices as Q8_0 rows and cannot run them)
    mode = goref.MODE_GGML_Q4 if shape.wtype == "q4_0" else goref.MODE_GO
    g = goref.GoRef(path, num_ctx=512, n_threads=0, mode=mode)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, prefill, seed=0)]).astype(np.int32)
    t = int(np.argmax(g.forward(prompt)))
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and n < 256:
        t = int(np.argmax(g.forward([t])))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": g.threads, "kind": "port", "cpu_model": cpu_model(),
            "logical_cpus": os.cpu_count(), "sample": f"{n} greedy decode tokens after a {len(prompt)}-token prefill, same synthetic GGUF, "
                      f"{dt:.1f} s, goref worker pool with {g.threads} threads"}


def run_reference(args) -> None:
    """The reference's own CPU implementation, same workload and metric."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import goref
    from b2decode import gguf_writer as gw
    shape = gw.SHAPES["qwen2.5-0.5b"]
    path = ensure_model("qwen2.5-0.5b")
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 128, seed=0)]).astype(np.int32)
    if goref.cppref_available():
        eng = goref.CppRef(path)
        kind, who = "reference", "the reference's C++ engine (Local-LLM) compiled from its sources"
        cores = os.cpu_count()
    else:
        eng = goref.GoRef(path, num_ctx=1024, n_threads=0)
        kind, who = "port", "goref, the Go engine restated in C++"
        cores = eng.threads
    t_pref = time.perf_counter()
    tok = int(np.argmax(eng.forward(prompt)))
    t_pref = time.perf_counter() - t_pref
    for _ in range(args.warmup):
        tok = int(np.argmax(eng.forward([tok])))
    n, t0 = 0, time.perf_counter()
    budget = float(os.environ.get("B2_REF_SECONDS", "60"))
    while n < args.steps and (time.perf_counter() - t0) < budget:
        tok = int(np.argmax(eng.forward([tok])))
        n += 1
    dt = time.perf_counter() - t0
    v = n / dt
    line = {
        "metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": ws, "steps": n,
        "warmup": args.warmup, "ms_per_step": 1000.0 * dt / max(n, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "prefill_s": t_pref, "engine": who},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "cpu_model": cpu_model(),
                         "logical_cpus": os.cpu_count(), "sample": f"{n} greedy decode tokens after the 129-token prefill ({dt:.1f} s)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    import b2decode
    from b2decode import gguf_writer as gw

    ws, rank, local = dist_env()
    if ws > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev_uuid = None
    try:
        u = torch.cuda.get_device_properties(local).uuid
        dev_uuid = "GPU-" + str(u)
    except Exception:
        pass

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if ws == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    shape_name, n_prompt, workload = MODELS[args.workload]
    shape = gw.SHAPES[shape_name]
    if rank == 0 or local == 0:
        path = ensure_model(shape_name)
    barrier()
    path = ensure_model(shape_name)
    K, W = args.steps, args.warmup
    e2e_steps = min(K, 64)
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, n_prompt, seed=0)]).astype(np.int32)
    num_ctx = len(prompt) + W + K + e2e_steps + 8
    tpn = ws if args.workload == "qwen72b" else 1  # tensor-parallel degree (else replicas)
    t_load = time.perf_counter()
    m = b2decode.Model(path, num_ctx=num_ctx, device=local, tp_size=tpn, tp_rank=rank if tpn > 1 else 0)
    load_s = time.perf_counter() - t_load
    load = _load_summary(m, load_s)
    if tpn > 1:
        from b2decode import tp as tpmod
        tpmod.connect(m)
    stream = torch.cuda.ExternalStream(m.stream_handle())
    cfg = m.cfg

    # prefill (timed for information)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    torch.cuda.nvtx.range_push("prefill")  # (lets a profiler keep to the prompt)
    first = m.forward_argmax(prompt)
    torch.cuda.nvtx.range_pop()
    prefill_s = time.perf_counter() - t0
    # warm-up decode steps
    warm = m.decode_greedy(first, W) if W > 0 else np.array([first])
    last = int(warm[-1]) if len(warm) else first

    # timed region: K device-resident decode steps
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev_uuid) as clk:
        torch.cuda.nvtx.range_push("timed")  # (lets a profiler keep to the timed steps)
        e0.record(stream)
        ids = m.decode_greedy(last, K)
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    barrier()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    if len(ids) != K:
        raise RuntimeError(f"decode produced {len(ids)} of {K} tokens")
    reps = ws // tpn  # independent model copies decoding at once
    value = reps * K / (ms_max / 1000.0)
    ms_tok = ms / K

    # e2e through the C ABI: one call per token, host in / host out
    tok = int(ids[-1])
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok = m.forward_argmax([tok])
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(e2e_s)
    e2e = reps * e2e_steps / e2e_s

    peak, peak_kind = peaks()
    bytes_tok = int(cfg["stream_bytes_per_token"])
    ctx_mid = len(prompt) + W + K // 2
    kv_bytes = 2 * cfg["num_layers"] * cfg["num_kv_heads"] * cfg["head_dim"] * 2 * ctx_mid
    achieved = bytes_tok / (ms_tok / 1000.0) / 1e9
    traffic, traffic_note = profile_traffic(ms_max / K) if args.workload == "qwen05b" else (None, "not profiled")
    clocks = clk.summary()
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            cpu = (cpu_baseline_goref(path) if args.workload == "qwen05b"
                   else cpu_baseline_goref(path, shape_name, seconds=20.0, prefill=0))
        except Exception as exc:  # the baseline must not sink the GPU line
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {exc}"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong" if tpn > 1 else "weak",
            "vs_baseline": None,
            "dtype": f"{shape.wtype.upper()} weights x int8 activation planes (3 per 32-block, |x - x'| <= "
                     f"2^-22 of the block maximum), exact int32 products, fp32 accumulate; fp16 KV cache",
            "data": "synthetic",
            "config": {"workload": workload, "weights": f"N(0,0.02) quantised {shape.wtype.upper()}, seed 0",
                       "prompt_tokens": int(len(prompt)), "decode_tokens_timed": K,
                       "ctx_range": [int(len(prompt) + W), int(len(prompt) + W + K)],
                       "l2": f"no flush needed: each token streams {bytes_tok / 1e6:.0f} MB of weights, > 126 MB L2",
                       "parallelism": (f"tp{tpn}" if tpn > 1 else (f"replicas x{ws}" if ws > 1 else "single gpu")),
                       "prefill_s": prefill_s,
                       "prefill_path": ("b2_forward_argmax: the prompt in chunks of up to 256 tokens on the tcgen05 GEMM path "
                                        "into the model's KV cache" if tpn == 1 else
                                        "b2_forward_argmax: the decode kernel once per prompt token (tensor parallel)"),
                       "load_s": load_s, "load": load,
                       "kv_cache": "fp16"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": traffic, "traffic_source": traffic_note,
                         "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" if peak_kind == "measured" else "fallback 6.65 TB/s",
                         "algorithmic_bytes_per_token": bytes_tok, "kv_bytes_per_token": kv_bytes},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "api": "b2_forward_argmax per token"},
            "gpu_launches": K,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
    m.close()
    if args.workload == "qwen05b" and not args.no_tp72b:
        tp = run_tp72b(args, ws, rank, local, barrier, max_over_ranks, peak, peak_kind)
        if rank == 0:
            line["tp72b"] = tp
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()


TP72B = "qwen2.5-72b-alias"


def run_tp72b(args, ws, rank, local, barrier, max_over_ranks, peak, peak_kind) -> dict:
    """The 72B shape (hidden 8192, 80 layers, 64/8 heads of 128, FFN 29568,
    vocab 152064, Q8_0, QKV bias, untied) tensor-parallel over all ranks:
    prompt BOS + 256 ids (seed 0), then greedy decode steps timed with CUDA
    events on each rank's stream, max over ranks.  The GGUF's 80 layers share
    one layer's data on disk; every rank still loads its share of all 80 as
    tensors of their own, so each step streams the full model's bytes."""
    import torch
    import torch.distributed as dist

    import b2decode
    from b2decode import gguf_writer as gw
    shape = gw.SHAPES[TP72B]
    if rank == 0 or local == 0:
        ensure_model(TP72B)
    barrier()
    path = ensure_model(TP72B)
    K, W = 32, 4
    prompt = np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, 256, seed=0)]).astype(np.int32)
    t0 = time.perf_counter()
    m = b2decode.Model(path, num_ctx=len(prompt) + W + K + 8, device=local, tp_size=ws if ws > 1 else 0,
                       tp_rank=rank if ws > 1 else 0)
    load_s = time.perf_counter() - t0
    load = _load_summary(m, load_s)
    if ws > 1:
        from b2decode import tp as tpmod
        tpmod.connect(m)
    stream = torch.cuda.ExternalStream(m.stream_handle())
    t0 = time.perf_counter()
    first = m.forward_argmax(prompt)
    prefill_s = time.perf_counter() - t0
    warm = m.decode_greedy(first, W)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ids = m.decode_greedy(int(warm[-1]), K)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    same = True
    if ws > 1:
        gathered = [None] * ws
        dist.all_gather_object(gathered, ids.tolist())
        same = all(g == gathered[0] for g in gathered)
    bytes_gpu = int(m.cfg["stream_bytes_per_token"])  # this rank's share
    bytes_all = int(max_over_ranks(float(bytes_gpu)))
    m.close()
    ms_tok = ms / K
    achieved = bytes_all / (ms_tok / 1000.0) / 1e9
    return {
        "workload": f"qwen2.5-72b-shape q8_0, all 80 layers, tensor-parallel over {ws} GPU(s), greedy decode, "
                    f"batch 1, prompt 256 ids + BOS",
        "weights": "N(0,0.02) quantised Q8_0, seed 0; the file's 80 layers share one layer's data, each rank "
                   "loads its share of all 80 layers as separate tensors",
        "tp": ws, "ms_per_token": ms_tok, "tok_s": 1000.0 / ms_tok, "steps": K, "warmup": W,
        "ctx_range": [int(len(prompt) + W), int(len(prompt) + W + K)],
        "bytes_per_token_per_gpu": bytes_all,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "per": "the most loaded rank's share"},
        "exchange": "after Wo and after down in every layer the ranks' partial rows go to every rank's buffer "
                    "by peer stores over NVLink inside the decode kernel (no collective library); argmax over "
                    "the vocab shares the same way" if ws > 1 else "none (one GPU)",
        "ids_first": [int(i) for i in ids[:8]], "ids_agree_across_ranks": bool(same),
        "load_s": load_s, "load": load, "prefill_s": prefill_s,
    }


def _load_summary(m, load_s: float) -> dict:
    """b2_get_load_stats of a loaded model: the load's phases and the upload
    rate (weight bytes / upload time)."""
    s = m.load_stats()
    up = s["upload_ns"] / 1e9
    return {"wall_s": load_s, "b2_load_s": s["total_ns"] / 1e9, "parse_s": s["parse_ns"] / 1e9, "upload_s": up,
            "host_copy_s": s["host_copy_ns"] / 1e9, "setup_s": s["setup_ns"] / 1e9, "weight_bytes": s["bytes_uploaded"],
            "upload_gbs": s["bytes_uploaded"] / up / 1e9 if up > 0 else None, "host_threads": s["host_threads"],
            "file": "memory-mapped" if s["mapped"] else "pread"}


def _rotations(nbytes: int) -> int:
    """Distinct copies so that one pass over them exceeds 256 MB (2x the L2)."""
    return max(1, -(-(256 << 20) // max(nbytes, 1)))


def _timed(torch, stream, fn, copies: int, iters: int) -> float:
    """Mean ms per call of fn(i) over `iters` calls cycling through the copies,
    CUDA events on `stream` after 3 warm-up passes."""
    for i in range(3 * copies):
        fn(i % copies)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(iters):
        fn(i % copies)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run_matvec(args) -> None:
    """Config-1 dequant-matvec microbench: b2_matvec (batch 1) and
    b2_matvec_batch (batch 8, one pass over W for all eight vectors)."""
    import torch

    import b2decode
    from b2decode import gguf_writer as gw
    torch.cuda.set_device(0)
    st = torch.cuda.Stream()
    peak, peak_kind = peaks()
    for batch in (1, 8):
        for kind, qt in (("q8_0", 8), ("q4_0", 2)):
            for rows, cols in ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)):
                if args.case and args.case != f"{kind}:{rows}x{cols}:{batch}":
                    continue
                rng = np.random.default_rng(rows * 7 + cols)
                base = gw.quantize(rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02),
                                   gw.TYPE_NAMES[kind])
                ncp = _rotations(base.nbytes)
                w0 = torch.from_numpy(base).cuda()
                ws = [w0] + [w0.clone() for _ in range(ncp - 1)]
                x = torch.from_numpy(rng.standard_normal((batch, cols), dtype=np.float32)).cuda()
                y = torch.empty((batch, rows), device="cuda")
                if batch == 1:
                    def call(i):
                        b2decode.matvec(qt, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, st.cuda_stream)
                else:
                    def call(i):
                        b2decode.matvec_batch(qt, ws[i].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, batch,
                                              st.cuda_stream)
                with torch.cuda.stream(st):
                    ms = _timed(torch, st, call, ncp, max(args.steps, 2 * ncp))
                nbytes = base.nbytes + 4 * batch * (rows + cols)
                gbs = nbytes / (ms / 1000.0) / 1e9
                print(json.dumps({
                    "metric": f"dequant-matvec GB/s (B={batch})", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                    "higher_is_better": True, "dtype": "fp32" if batch == 1 else "s8x3 planes, fp32 accumulate",
                    "data": "synthetic",
                    "config": {"workload": f"matvec {kind} {rows}x{cols}, batch {batch}", "us_per_call": ms * 1000.0,
                               "weight_bytes": int(base.nbytes), "l2": f"{ncp} weight copies rotated"},
                    "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                                 "peak_source": peak_kind},
                }), flush=True)
                del ws, w0
                torch.cuda.empty_cache()


def run_attention(args) -> None:
    """Config-3 GQA decode attention through b2_attention_decode."""
    import torch

    import b2decode
    torch.cuda.set_device(0)
    st = torch.cuda.Stream()
    peak, peak_kind = peaks()
    nh, nkv, hd = 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    for ctx in (4096, 16384, 32768):
        for B in (1, 8):
            if args.case and args.case != f"{ctx}x{B}":
                continue
            kvbytes = 2 * B * ctx * nkv * hd * 2
            ncp = _rotations(kvbytes)
            ks = [torch.randn(B * ctx * nkv * hd, generator=g, device="cuda").half() for _ in range(ncp)]
            vs = [torch.randn(B * ctx * nkv * hd, generator=g, device="cuda").half() for _ in range(ncp)]
            q = torch.randn(B * nh * hd, generator=g, device="cuda")
            out = torch.empty(B * nh * hd, device="cuda")
            with torch.cuda.stream(st):
                ms = _timed(torch, st, lambda i: b2decode.attention_decode(
                    q.data_ptr(), ks[i].data_ptr(), vs[i].data_ptr(), out.data_ptr(), B, nh, nkv, hd, ctx,
                    st.cuda_stream), ncp, max(args.steps, 2 * ncp))
            gbs = kvbytes / (ms / 1000.0) / 1e9
            print(json.dumps({
                "metric": "GQA decode attention GB/s", "value": gbs, "unit": "GB/s", "n_gpus": 1,
                "higher_is_better": True,
                "dtype": "fp16 KV; q and the probabilities split into two fp16 terms each on mma.m16n8k16, fp32 "
                         "accumulate and softmax",
                "data": "synthetic",
                "config": {"workload": f"attention nh {nh} nkv {nkv} hd {hd} ctx {ctx} batch {B}",
                           "us_per_call": ms * 1000.0, "kv_bytes": kvbytes, "l2": f"{ncp} KV copies rotated"},
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "peak_source": peak_kind},
            }), flush=True)
            del ks, vs
            torch.cuda.empty_cache()


def run_gemm(args) -> None:
    """The tcgen05 tensor-core GEMM (b2_model_gemm) on the matrices of one
    Llama-3-8B layer (Q4_0: Wq, Wk, Wv, Wo, gate, up, down; the 4-layer file
    of the real widths) for a prompt-sized token count (--tokens, 512 by
    default): TFLOP/s = 2 x rows x cols x tokens / time, against the measured
    dense bf16 peak (the fp16 kind runs at the same rate).  Gate and up are
    resident as one interleaved matrix: b2_model_gemm on ffn_gate computes
    the product of both halves (as the batched forward does) and gathers the
    gate half, so that line counts the flops of both."""
    import torch

    import b2decode
    from b2decode import gguf_writer as gw
    torch.cuda.set_device(0)
    shape = gw.SHAPES["llama3-8b-4l"]
    m = b2decode.Model(ensure_model("llama3-8b-4l"), num_ctx=64)
    st = torch.cuda.ExternalStream(m.stream_handle())
    H, FF, qd, kvd = shape.hidden, shape.ffn, shape.heads * shape.head_dim, shape.kv_dim
    mats = {"blk.0.attn_q.weight": (qd, H), "blk.0.attn_k.weight": (kvd, H), "blk.0.attn_v.weight": (kvd, H),
            "blk.0.attn_output.weight": (H, qd), "blk.0.ffn_gate.weight": (FF, H), "blk.0.ffn_down.weight": (H, FF)}
    mp = measured_peaks()
    peak = float(mp.get("bf16_tflops", 1590.0)) if mp else 1590.0
    ntok = args.tokens
    tot_flop, tot_ms = 0.0, 0.0
    for name, (rows, cols) in mats.items():
        if args.case and args.case != name:
            continue
        x = torch.randn(ntok, cols, device="cuda")
        y = torch.empty(ntok, rows, device="cuda")
        with torch.cuda.stream(st):
            ms = _timed(torch, st, lambda i: m.gemm(name, x.data_ptr(), y.data_ptr(), ntok), 1, max(args.steps, 8))
        both = name.endswith("ffn_gate.weight")  # the interleaved gate/up product
        flop = 2.0 * rows * cols * ntok * (2 if both else 1)
        label = f"{name} {rows}x{cols}" if not both else \
            f"{name[:-len('gate.weight')]}gate+up interleaved {2 * rows}x{cols} (gate half gathered)"
        tf = flop / (ms / 1000.0) / 1e12
        tot_flop += flop
        tot_ms += ms
        print(json.dumps({
            "metric": "tensor-core GEMM TFLOP/s (prefill product)", "value": tf, "unit": "TFLOP/s", "n_gpus": 1,
            "higher_is_better": True, "dtype": "Q4_0 weights -> fp16 (d*q rounded once) x fp16 activations "
                                               "(power-of-two scale per token), fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": f"{label} (Llama-3-8B widths, Q4_0) x {ntok} tokens",
                       "us_per_call": ms * 1000.0, "path": "b2_model_gemm: tcgen05.mma kind::f16, TMA-staged tiles"},
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_source": "MEASURED_PEAKS.json bf16_tflops" if mp else "fallback 1.59 PFLOP/s"},
        }), flush=True)
    if not args.case:
        tf = tot_flop / (tot_ms / 1000.0) / 1e12
        print(json.dumps({"metric": "tensor-core GEMM TFLOP/s, one Llama-3-8B layer's products", "value": tf,
                          "unit": "TFLOP/s", "n_gpus": 1, "higher_is_better": True,
                          "config": {"workload": f"q, k, v, o, gate+up, down x {ntok} tokens", "ms": tot_ms},
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                                       "frac": tf / peak}}), flush=True)
    m.close()


def run_sample(args) -> None:
    """Device-side sampling (b2_sample_device, one launch per token) on a
    Qwen2.5-vocabulary logits row (151936, N(0, 3)), per option set, against
    the host path it replaces: the 608 KB logits copy to the host plus
    sample() on the host (b2_sample_logits).  Each device call first restores
    the row (the sampler modifies it in place); that copy is timed alone and
    subtracted."""
    import time

    import numpy as np
    import torch

    import b2decode
    torch.cuda.set_device(0)
    V = 151936
    rng = np.random.default_rng(0)
    lg = (rng.standard_normal(V) * 3).astype(np.float32)
    gen = rng.integers(0, V, 64).astype(np.int32)
    src = torch.tensor(lg, device="cuda")
    work = torch.empty_like(src)
    scratch = torch.empty(b2decode.sample_scratch_bytes(V, 1), dtype=torch.uint8, device="cuda")
    dgen = torch.tensor(gen, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    host = torch.empty(V, dtype=torch.float32, pin_memory=True)
    st = torch.cuda.current_stream()
    sh = st.cuda_stream
    iters = max(args.steps, 50)
    copy_ms = _timed(torch, st, lambda i: work.copy_(src), 1, iters)
    d2h_ms = _timed(torch, st, lambda i: host.copy_(src, non_blocking=True), 1, iters)
    for temp, k, p, rp in ((0.8, 40, 0.9, 1.1), (1.0, 0, 0.9, 1.0), (0.7, 0, 0.0, 1.0), (0.001, 0, 0.0, 1.3)):
        opts = b2decode.sample_opts(temp, k, p, rp)

        def call(i):
            work.copy_(src)
            b2decode.sample_device(work.data_ptr(), V, 1, V, opts, dgen.data_ptr(), V, [len(gen)], [0.37],
                                   scratch.data_ptr(), out.data_ptr(), sh)

        dev_us = (_timed(torch, st, call, 1, iters) - copy_ms) * 1000.0
        t0 = time.perf_counter()
        n_host = 5
        for _ in range(n_host):
            b2decode.sample_logits(lg, opts, gen.tolist(), 0.37)
        host_us = (time.perf_counter() - t0) / n_host * 1e6 + d2h_ms * 1000.0
        print(json.dumps({
            "metric": "sampling latency per token (device sampler)", "value": dev_us, "unit": "us",
            "n_gpus": 1, "higher_is_better": False, "data": "synthetic",
            "config": {"workload": f"vocab {V}, temperature {temp}, top_k {k}, top_p {p}, repeat_penalty {rp} "
                                   f"over 64 ids",
                       "host_path_us": host_us, "host_path": "608 KB logits to the host + sample() there",
                       "d2h_us": d2h_ms * 1000.0, "speedup_vs_host_path": host_us / max(dev_us, 1e-9)},
        }), flush=True)


def run_batch(args) -> None:
    """Batched greedy decode (b2_batch_*) of --batch sequences of a model
    workload: each sequence prefilled with its own prompt (16-token chunks),
    then K steps of all sequences at once; value = tokens of all sequences
    per second."""
    import torch

    import b2decode
    from b2decode import gguf_writer as gw
    if dist_env()[0] > 1 or args.workload not in ("qwen05b", "llama3-8b"):
        raise SystemExit("--batch runs the qwen05b or llama3-8b workload on one GPU")
    torch.cuda.set_device(0)
    shape_name, n_prompt, _ = MODELS[args.workload]
    shape = gw.SHAPES[shape_name]
    path = ensure_model(shape_name)
    B, K, W = args.batch, args.steps, args.warmup
    m = b2decode.Model(path, num_ctx=n_prompt + 1 + W + K + 8)
    stream = torch.cuda.ExternalStream(m.stream_handle())
    bt = b2decode.Batch(m, B)
    if args.graph:
        bt.use_graph(True)  # captured after the first warm-up step
    t0 = time.perf_counter()
    nxt = [bt.prefill(b, np.concatenate([[shape.bos_id], gw.make_prompt(shape.vocab, n_prompt, seed=b)])
                      .astype(np.int32)) for b in range(B)]
    prefill_s = time.perf_counter() - t0
    for _ in range(W):
        nxt = bt.step(nxt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dev_uuid = None
    try:
        dev_uuid = "GPU-" + str(torch.cuda.get_device_properties(0).uuid)
    except Exception:
        pass
    with Clocks(dev_uuid) as clk:
        torch.cuda.nvtx.range_push("timed")  # (lets a profiler keep to the timed steps)
        e0.record(stream)
        t_host = time.perf_counter()
        for _ in range(K):
            nxt = bt.step(nxt)  # host ids in and out every step
        t_host = time.perf_counter() - t_host
        e1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    ms = e0.elapsed_time(e1)
    peak, peak_kind = peaks()
    bytes_step = int(m.cfg["stream_bytes_per_token"])
    cpu = None
    if not args.no_cpu_baseline:
        # the reference engine serves one sequence at a time: its rate over B
        # sequences is its single-sequence rate
        try:
            cpu = cpu_baseline_goref(path, shape_name, seconds=20.0, prefill=0)
        except Exception as exc:  # the baseline must not sink the GPU line
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {exc}"}
    achieved = bytes_step / (ms / K / 1000.0) / 1e9
    print(json.dumps({
        "metric": f"batched decode tok/s (B={B})", "value": B * K / (ms / 1000.0), "unit": "tok/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": (f"{shape.wtype.upper()} weights -> fp16 (d*q rounded once) x fp16 activations (power-of-two "
                  f"scale per token), fp32 accumulate (tcgen05 kind::f16)"),
        "data": "synthetic",
        "config": {"workload": f"{shape_name}-shape {shape.wtype} batched greedy decode, batch {B}, "
                               f"prompt {n_prompt} ids per sequence",
                   "launches": "one CUDA graph per step" if args.graph else "eager (11 per layer)",
                   "prompt_tokens": n_prompt + 1, "prefill_s": prefill_s,
                   "prefill_tok_s": B * (n_prompt + 1) / prefill_s,
                   # 2 flops per weight per token; weights = streamed bytes x 32 / (bytes per 32-block)
                   "prefill_tflops": 2.0 * bytes_step * 32 / (34 if shape.wtype == "q8_0" else 18)
                                     * B * (n_prompt + 1) / prefill_s / 1e12,
                   "prefill_path": "b2_batch_prefill: chunks of up to 256 prompt tokens, one weight pass each on "
                                   "the tcgen05 GEMM, the chunk's attention over the slot's cache",
                   "l2": f"no flush needed: each step streams {bytes_step / 1e6:.0f} MB of weights"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_kind, "algorithmic_bytes_per_step": bytes_step},
        "e2e": {"value": B * K / t_host, "unit": "tok/s", "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                "api": "b2_batch_step per step"},
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
    }), flush=True)
    bt.close()
    m.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp72b", action="store_true",
                    help="qwen05b: skip the tensor-parallel 72B-shape measurement added to the line")
    ap.add_argument("--workload", default="qwen05b",
                    choices=["qwen05b", "llama3-8b", "qwen72b", "matvec", "attention", "gemm", "sample"])
    ap.add_argument("--case", default="",
                    help="one case of a microbench: attention CTXxB (32768x8), matvec KIND:ROWSxCOLS:B "
                         "(q8_0:128256x4096:1), gemm tensor name (blk.0.ffn_up.weight)")
    ap.add_argument("--tokens", type=int, default=512, help="--workload gemm: tokens per product")
    ap.add_argument("--batch", type=int, default=1,
                    help="> 1: batched greedy decode of that many sequences (qwen05b / llama3-8b workloads)")
    ap.add_argument("--graph", action="store_true", help="--batch: replay each step from a captured CUDA graph")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "matvec":
        run_matvec(args)
    elif args.workload == "attention":
        run_attention(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "sample":
        run_sample(args)
    elif args.batch > 1:
        run_batch(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
