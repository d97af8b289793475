"""Decode throughput of the INT4 8B-class llama on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

One JSON line on rank 0.  A step = one greedy decode step of `batch` sequences
(a CUDA-graph replay: embedding, 32 x [QKV, flash-decode, O, gate|up, down], lm_head,
argmax) with the argmax fed back on the device.  Model: random-init (seeded) weights
of the llama-8b architecture, INT4 group-128 linears, fp16 embedding / lm_head /
KV cache, a 1024-token random prompt prefilled before timing.  Per step the kernels
stream ~4.8 GB of weights and KV (>> the 126 MB L2), so no L2 flush is needed.
With N > 1 the model is tensor-parallel (column/row split, NCCL allreduce after
o_proj and down_proj, vocab-sharded lm_head), one process per GPU.

--impl reference times the reference's CPU implementation of the same step (the C
restatement of DeepUnity's CPU module path in oracle/, on every host core) on a
bounded sample: one decoder layer plus 1/16 of the lm_head per step, scaled to a
full token.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = "llama-8b"
PROMPT = 1024
CAPACITY = 8192
PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=PROMPT)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", choices=["persistent", "per_stage"], default="per_stage",
                    help="decode step as one persistent kernel, or as a graph of per-stage kernels")
    ap.add_argument("--clock-sampler", choices=["nvml", "smi", "none"], default="nvml")
    ap.add_argument("--nccl-only", action="store_true", help="TP: decode reductions with ncclAllReduce only")
    ap.add_argument("--sweep", choices=["gemv", "attn"], default=None,
                    help="kernel sweeps (one JSON line per case): config-2 GEMV, config-3 flash-decode")
    ap.add_argument("--gemv-phases", action="store_true",
                    help="timing build (python -m deepunity_b200.build --stamps): per-CTA phase stamps of the "
                         "decode GEMVs over two decode steps, medians per stage boundary")
    ap.add_argument("--case", default=None, help="--sweep gemv: one cell quant:N:K:M, quant int4 / int8 / f16 (e.g. int4:14336:4096:1)")
    ap.add_argument("--reps", type=int, default=0, help="--sweep: timed launches per case (0 = auto)")
    ap.add_argument("--model", choices=["llama-8b", "llama-1.1b"], default="llama-8b",
                    help="llama-8b: BASELINE config 5 (INT4 g128); llama-1.1b: config 4 (INT8 per row)")
    ap.add_argument("--kv", choices=["fp16", "int8"], default="fp16",
                    help="KV cache format (KVQuant.FP16 / KVQuant.INT8)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: keep the first N decoder layers (smaller device footprint)")
    return ap.parse_args()


def tensor_peak():
    """Measured dense bf16 TFLOP/s (burst) of MEASURED_PEAKS.json, else the fallback."""
    try:
        with open(PEAKS) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def peaks():
    try:
        with open(PEAKS) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class NvmlClockSampler:
    """SM clock and clock-event (throttle) reasons read through NVML from a host
    thread every `period` seconds during the timed region (in-process: no
    nvidia-smi process competing for the driver)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, gpu: int, period: float = 0.05):
        self.gpu, self.period = gpu, period
        self.samples = []
        self.max_mhz = None

    def __enter__(self):
        import threading
        try:
            import pynvml as N
            N.nvmlInit()
            self.N = N
            self.h = N.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception:
            self.N = None
            return self
        self.stop = threading.Event()

        def run():
            while not self.stop.is_set():
                try:
                    mhz = self.N.nvmlDeviceGetClockInfo(self.h, self.N.NVML_CLOCK_SM)
                    r = self.N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.samples.append((mhz, r))
                except Exception:
                    pass
                self.stop.wait(self.period)

        self.t = threading.Thread(target=run, daemon=True)
        self.t.start()
        time.sleep(self.period)
        return self

    def __exit__(self, *a):
        if self.N is not None:
            self.stop.set()
            self.t.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        reasons = sorted({name for _, r in self.samples for name, attr in self.REASONS.items()
                          if r & getattr(self.N, attr, 0)})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "sampler": "nvml"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def summary(self):
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------- CPU baseline
def cpu_reference_sample(cfg, batch: int, prompt: int, steps: int, warmup: int):
    """Times the reference CPU path on a bounded sample; returns (tok/s, sample text, cores, per-step s)."""
    from oracle import oracle as orc
    import ctypes as C
    L = orc.lib()
    H, I, hq, hkv, hd = cfg.hidden_size, cfg.intermediate_size, cfg.num_heads_q, cfg.num_heads_kv, cfg.head_dim
    rng = np.random.default_rng(0)
    std = np.float32(0.02)
    mk = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std)
    Wqkv, Wo = mk((hq + 2 * hkv) * hd, H), mk(H, hq * hd)
    Wg, Wu, Wd = mk(I, H), mk(I, H), mk(H, I)
    ln = np.ones(H, np.float32)
    n_pos = prompt + warmup + steps + 2
    kc = np.ascontiguousarray(rng.standard_normal((n_pos, hkv, hd), dtype=np.float32))
    vc = np.ascontiguousarray(rng.standard_normal((n_pos, hkv, hd), dtype=np.float32))
    head_rows = cfg.vocab_size // 16
    Wh = mk(head_rows, H)
    x = rng.standard_normal(H).astype(np.float32)
    scratch = np.zeros(2 * H + (hq + 2 * hkv) * hd + 2 * hq * hd + 3 * I + hq * (n_pos + 1), np.float32)
    logits = np.empty(head_rows, np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    times = []
    for s in range(warmup + steps):
        pos = prompt + s
        t0 = time.perf_counter()
        L.orc_module_layer_decode(p(x), H, I, hq, hkv, hd, 1e-5, 10000.0, p(ln), p(ln), p(Wqkv), p(Wo), p(Wg),
                                  p(Wu), p(Wd), p(kc), p(vc), pos, p(scratch), 0)
        t1 = time.perf_counter()
        L.orc_dense_linear(p(x), 1, 0, H, head_rows, p(Wh), None, p(logits), 0)
        t2 = time.perf_counter()
        if s >= warmup:
            times.append(cfg.num_layers * (t1 - t0) + 16 * (t2 - t1))
    tok_s = steps / sum(times) if times else 0.0
    sample = (f"C restatement of the reference CPU module path (Dense.Linear / GroupedQueryAttention / RMSNorm / "
              f"GatedLinearUnit, fp32 weights, OpenMP over output rows); per step 1 of {cfg.num_layers} decoder "
              f"layers at kv {prompt}+ and 1/16 of the lm_head, scaled to a full token; batch 1")
    return tok_s, sample, orc.max_threads(), times


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from deepunity_b200.llm import CONFIGS
    cfg = CONFIGS[args.model]
    tok_s, sample, cores, times = cpu_reference_sample(cfg, args.batch, args.prompt, args.steps, args.warmup)
    mclass = "INT4 8B-class" if args.model == "llama-8b" else "INT8 1.1B-class"
    line = {"metric": f"decode tok/s ({mclass}, bs{args.batch})", "value": round(tok_s, 4), "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 / tok_s, 3) if tok_s else None, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.model} decode step, batch {args.batch}, kv {args.prompt} (CPU sample)",
                       "model": args.model, "global_batch": args.batch, "seq_len": args.prompt},
            "impl": "reference",
            "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from deepunity_b200 import _lib
    from deepunity_b200.llm import CONFIGS, KVQuant, LlamaForCausalLM, LLMQuant
    import ctypes as C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
    cfg = CONFIGS[args.model]
    quant = LLMQuant.INT4 if args.model == "llama-8b" else LLMQuant.INT8
    if args.layers:
        import dataclasses
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    B = args.batch
    need = args.prompt + args.warmup + 2 * args.steps + 4
    cap = max(CAPACITY if args.model == "llama-8b" else 0, need)
    m = LlamaForCausalLM(cfg, quant, kv_quant=KVQuant.INT8 if args.kv == "int8" else KVQuant.FP16,
                         max_context_length=cap, max_batch=B, seed=0,
                         device=local, tp_rank=rank, tp_size=world,
                         flags=_lib.FLAG_PERSISTENT if args.path == "persistent" else 0)
    if world > 1:
        uid = [None]
        if rank == 0:
            buf = C.create_string_buffer(128)
            _lib.call("du_nccl_unique_id", buf)
            uid[0] = buf.raw
        dist.broadcast_object_list(uid, src=0)
        m.init_tp(uid[0], timeout_ms=120000)
        if not args.nccl_only:      # decode reductions over NVLink peer memory
            hs = [None] * world
            dist.all_gather_object(hs, m.p2p_handle())
            m.init_p2p(hs)

    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (B, args.prompt)).astype(np.int32)
    _, nxt = m.forward(prompt, want_logits=False)
    ids = nxt.copy()
    # warm-up (captures the decode graph)
    toks = m.decode_loop(ids, args.warmup)
    ids = toks[-1].copy()
    kn, tn = C.c_int(), C.c_int()
    _lib.call("du_model_graph_info", m.handle, B, C.byref(kn), C.byref(tn))

    stream = torch.cuda.ExternalStream(m.stream(), device=local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed: K graph replays with the argmax fed back on the device
    sampler = {"nvml": NvmlClockSampler, "smi": ClockSampler}.get(args.clock_sampler)
    with (sampler(local) if sampler else contextlib.nullcontext()) as clk:
        barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_timed")      # ncu --nvtx-include decode_timed/ selects these launches
        ev0.record(stream)
        toks = m.decode_loop(ids, args.steps)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ids = toks[-1].copy()

    # ---- end to end through du_decode_step: host ids in, host ids out, every step
    barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    t0 = time.perf_counter()
    cur = ids
    for _ in range(args.steps):
        cur = m.decode_step(cur)
    ev1.record(stream)
    torch.cuda.synchronize()
    t_host = time.perf_counter() - t0
    barrier()
    ms_e2e = max_over_ranks(max(ev0.elapsed_time(ev1), 1000.0 * t_host))

    # ---- stage times of the last step when it ran as the persistent decode-step kernel:
    # globaltimer stamps at each grid-barrier exit (embed, L x [qkv, attn, o, gate|up, down], lm_head, argmax)
    L = cfg.num_layers
    st_buf = (C.c_float * (5 * L + 8))()
    n_st = C.c_int()
    _lib.call("du_model_stage_times", m.handle, st_buf, len(st_buf), C.byref(n_st))
    stage_us = None
    if n_st.value == 5 * L + 3:
        v = [float(x) for x in st_buf[:n_st.value]]
        per = [v[1 + 5 * l:1 + 5 * l + 5] for l in range(L)]
        avg = lambda i: sum(p[i] for p in per) / L
        stage_us = {"embed": round(v[0], 2), "qkv": round(avg(0), 2), "attn": round(avg(1), 2),
                    "o_proj": round(avg(2), 2), "gate_up": round(avg(3), 2), "down": round(avg(4), 2),
                    "lm_head": round(v[-2], 2), "argmax": round(v[-1], 2)}

    # ---- per-kernel device times of the per-stage path (CUDA events, all layers' weights)
    kt = (C.c_float * 6)()
    _lib.call("du_model_kernel_times", m.handle, B, 2, kt)
    kt = [float(v) for v in kt]

    value = B * args.steps / (ms / 1000.0)
    e2e = B * args.steps / (ms_e2e / 1000.0)
    peak, peak_kind = peaks()
    I_l, H = cfg.intermediate_size // world, cfg.hidden_size
    g = cfg.group_size

    def wbytes(n, k):      # algorithmic bytes of one linear's weights and scales
        return n * k // 2 + n * (k // g) * 2 if quant == LLMQuant.INT4 else n * k + 2 * n

    hq_l, hkv_l, hd = cfg.num_heads_q // world, cfg.num_heads_kv // world, cfg.head_dim
    gu_bytes = wbytes(2 * I_l, H) + B * H * 4 + B * I_l * 4
    # K and V rows read per step at the mean cache length of the timed steps
    kv_mean = args.prompt + args.warmup + args.steps // 2 + 1
    # (INT8 cache: one byte an element plus a 4-byte scale / zero-point word per position and kv head)
    kv_layer = 2 * B * kv_mean * hkv_l * (hd * 2 if args.kv == "fp16" else hd + 4)
    kv_read = cfg.num_layers * kv_layer
    step_bytes = m.weight_bytes() + kv_read
    step_ms = ms / args.steps
    # per-kernel algorithmic bytes (weights + the activations each reads and writes)
    stage_bytes = {"qkv": wbytes((hq_l + 2 * hkv_l) * hd, H) + B * H * 4 + B * hq_l * hd * 4,
                   "attn": kv_layer + 2 * B * hq_l * hd * 4,
                   "o_proj": wbytes(H, hq_l * hd) + B * hq_l * hd * 4 + 2 * B * H * 4,
                   "gate_up": gu_bytes,
                   "down": wbytes(H, I_l) + B * I_l * 4 + 2 * B * H * 4,
                   "lm_head": (cfg.vocab_size // world) * H * 2 + B * H * 4}
    if stage_us is not None:
        # one launch per step: the roofline is the whole persistent kernel
        roof_kernel = "decode_step_kernel (persistent; one launch = one decode step)"
        roof_bytes, roof_ms = step_bytes, step_ms
    else:
        roof_kernel = "qgemv_kernel gate|up INT4 GEMV (RMSNorm prologue, SiLU epilogue)"
        roof_bytes, roof_ms = gu_bytes, kt[3]
    achieved = roof_bytes / (roof_ms / 1000.0) / 1e9
    # DRAM bytes per launch of decode_step_kernel from ncu captures at two layer counts
    # (traffic = fixed + per_layer * layers), scaled to this run's layer count
    traffic = None
    if stage_us is not None:
        prof = os.path.join(ROOT, "profiles", "decode_step_traffic.json")
        key = None
    else:       # per-stage graph: DRAM bytes per launch of the gate|up GEMV (ncu, layer-independent)
        prof = os.path.join(ROOT, "profiles", "gateup_gemv_traffic.json")
    if os.path.exists(prof) and args.model == "llama-8b" and B == 1 and world == 1:
        try:
            tj = json.load(open(prof))
            traffic = int(tj["fixed_bytes"] + tj["per_layer_bytes"] * cfg.num_layers) if stage_us is not None \
                else int(tj["bytes_per_launch"])
        except Exception:
            traffic = None
    stage_roof = None
    if stage_us is not None:
        stage_roof = {"stage": "gate|up INT4 GEMV inside the persistent kernel (incl. its grid barrier)",
                      "bytes": gu_bytes, "us": stage_us["gate_up"],
                      "achieved_gbs": round(gu_bytes / (stage_us["gate_up"] * 1e-6) / 1e9, 1)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, sample, cores, _ = cpu_reference_sample(cfg, B, args.prompt, 6, 1)
        cpu = {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        mclass = "INT4 8B-class" if args.model == "llama-8b" else "INT8 1.1B-class"
        line = {
            "metric": f"decode tok/s ({mclass}, bs{B})",
            "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("int4" if quant == LLMQuant.INT4 else "int8") + f" weights x fp32 activations ({args.kv} KV)",
            "data": "synthetic (seeded random-init weights, random prompt ids)",
            "config": {"workload": f"{args.model} {'INT4-g128' if quant == LLMQuant.INT4 else 'INT8-row'} decode, "
                                   f"batch {B}, prompt {args.prompt}, "
                                   f"kv {args.prompt}..{args.prompt + args.warmup + args.steps}",
                       "model": args.model if not args.layers else f"{args.model} (first {args.layers} layers, profiling)",
                       "global_batch": B, "seq_len": args.prompt,
                       "parallelism": f"tp{world}",
                       "l2": f"no flush: {step_bytes / 1e9:.2f} GB streamed per step >> 126 MB L2"},
            "decode_path": "persistent decode-step kernel" if stage_us else "graph of per-stage kernels",
            "stage_us": stage_us,
            "roofline": {"bound": "hbm", "kernel": roof_kernel,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": roof_bytes, "launch_ms": round(roof_ms, 5)},
            "stage_roofline": stage_roof,
            "step_roofline": {"bound": "hbm", "what": "whole decode step: weights + K/V rows read per step "
                                                     "over the device-timed step",
                              "bytes_per_step": int(step_bytes), "ms_per_step": round(step_ms, 4),
                              "achieved": round(step_bytes / (step_ms / 1000.0) / 1e9, 1), "peak": peak,
                              "unit": "GB/s", "frac": round(step_bytes / (step_ms / 1000.0) / 1e9 / peak, 4),
                              "peak_kind": peak_kind},
            "kernel_ms": dict(zip(["qkv", "attn", "o_proj", "gate_up", "down", "lm_head"],
                                  [round(v, 5) for v in kt])),
            "kernel_frac_hbm": {k: round(stage_bytes[k] / (v / 1000.0) / 1e9 / peak, 4)
                                for k, v in zip(["qkv", "attn", "o_proj", "gate_up", "down", "lm_head"], kt)
                                if v > 0},
            "kernel_ms_note": "each stage kernel replayed back to back outside the decode graph (CUDA events, "
                              "all layers), averaged per launch; fractions are algorithmic bytes / time / peak",
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": int(kn.value) * args.steps,
            "clocks": clk.summary() if clk is not None else {"sm_mhz": None, "reasons": ["unsampled"]},
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    m.Release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _events_ms(fn, reps: int, stream=None):
    import torch
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record(stream)
    for i in range(reps):
        fn(i)
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def _graph_ms(fn, reps: int):
    """Device time per call of fn(i, stream) with `reps` calls captured in one CUDA graph
    (launch gaps of the host loop removed); CUDA events on the capturing stream."""
    import torch
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for i in range(2):          # first calls outside capture: attributes, grow-only scratch
            fn(i, s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i, s.cuda_stream)
    with torch.cuda.stream(s):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms


def run_sweep_gemv(args):
    """quant-GEMV HBM GB/s vs peak through du_gemv_q4 / du_gemv_q8.
    Distinct weight copies (>= 1 GB in total) rotate between launches so no launch
    finds its weights in the 126 MB L2."""
    import ctypes as C
    import torch
    from deepunity_b200 import _lib
    torch.cuda.set_device(0)
    _lib.call("du_init", 0)
    peak, kind = peaks()
    tpeak = tensor_peak()
    g = torch.Generator(device="cuda").manual_seed(0)
    only = None
    if args.case:   # "int4:14336:4096:1" -> one sweep cell (profiling)
        q_, n_, k_, m_ = args.case.split(":")
        only = (q_, int(n_), int(k_), int(m_))
    quants = (only[0],) if only else ("int4", "int8")
    shapes = [only[1:3]] if only else [(4096, 4096), (14336, 4096), (4096, 14336)]
    for quant in quants:
        for (N, K) in shapes:
            wbytes = N * K // 2 if quant == "int4" else N * K * (2 if quant == "f16" else 1)
            sbytes = N * (K // 128) * 2 if quant == "int4" else (N * 2 if quant == "int8" else 0)
            copies = max(2, int(np.ceil(1.1e9 / (wbytes + sbytes))))
            W = torch.randint(0, 256, (copies, wbytes), dtype=torch.uint8, device="cuda", generator=g)
            Sc = (torch.rand((copies, max(sbytes, 2) // 2), device="cuda", generator=g) * 1e-3).half()
            for M in (1, 4, 16, 64, 512):
                if only and M != only[3]:
                    continue
                x = torch.randn((M, K), device="cuda", generator=g).bfloat16()
                y = torch.empty((M, N), device="cuda")
                if quant == "int4":
                    f = lambda i, st: _lib.call("du_gemv_q4", C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()),
                                                _lib.DTYPE_BF16, C.c_void_p(W[i % copies].data_ptr()),
                                                C.c_void_p(Sc[i % copies].data_ptr()), 128, M, N, K, C.c_void_p(st))
                elif quant == "f16":
                    f = lambda i, st: _lib.call("du_gemv_f16", C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()),
                                                _lib.DTYPE_BF16, C.c_void_p(W[i % copies].data_ptr()), M, N, K,
                                                C.c_void_p(st))
                else:
                    f = lambda i, st: _lib.call("du_gemv_q8", C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()),
                                                _lib.DTYPE_BF16, C.c_void_p(W[i % copies].data_ptr()),
                                                C.c_void_p(Sc[i % copies].data_ptr()), _lib.DTYPE_F16, M, N, K,
                                                C.c_void_p(st))
                reps = args.reps or max(8, min(64, int(2e9 / (wbytes + sbytes))))
                ms = _graph_ms(f, reps)
                byts = wbytes + sbytes + M * K * 2 + M * N * 4
                gbs = byts / (ms / 1e3) / 1e9
                tflops = 2 * M * N * K / (ms / 1e3) / 1e12
                if M >= 16 and K % 64 == 0:
                    path = "tcgen05 GEMM (kind::f16, exact fp16 hi/lo operands)"
                elif (M <= 2 and quant == "int4" and K % 128 == 0 and (K // 128) % 8 == 0
                      and os.environ.get("DU_DECODE_GEMV") == "tcgen05"):
                    path = "tcgen05 GEMV (kind::i8, nibble x byte planes)"
                else:
                    path = "dp4a GEMV"
                print(json.dumps({"sweep": "gemv", "quant": quant + {"int4": "-g128", "int8": "-row"}.get(quant, ""),
                                  "N": N, "K": K, "M": M, "path": path, "us": round(ms * 1e3, 2),
                                  "GB_s": round(gbs, 1), "frac_hbm": round(gbs / peak, 4),
                                  "TFLOP_s": round(tflops, 2), "frac_tensor_bf16": round(tflops / tpeak, 4),
                                  "peak_kind": kind, "copies": copies,
                                  "timing": "CUDA graph of the launches, weights rotated over >= 1.1 GB"}), flush=True)
            del W, Sc


def run_sweep_attn(args):
    """split-K flash-decode over fp16 KV, 32 q / 8 kv heads, hd 128."""
    import ctypes as C
    import torch
    from deepunity_b200 import _lib
    torch.cuda.set_device(0)
    _lib.call("du_init", 0)
    peak, kind = peaks()
    g = torch.Generator(device="cuda").manual_seed(0)
    hq, hkv, hd = 32, 8, 128
    for kv in ("fp16", "int8"):
        for ctx in (512, 2048, 8192, 32768):
            for B in (1, 8, 32):
                # algorithmic bytes: K and V rows (2 bytes an element, or 1 + a 4-byte
                # scale / zero-point word per (position, kv head) for the INT8 cache)
                kv_bytes = B * ctx * hkv * (hd * 2 * 2 if kv == "fp16" else (hd + 4) * 2)
                copies = max(2, int(np.ceil(0.6e9 / kv_bytes)))
                if copies * kv_bytes > 40e9:
                    copies = 1
                q = torch.randn((B, hq, hd), device="cuda", generator=g)
                out = torch.empty((B, hq, hd), device="cuda")
                lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
                if kv == "fp16":
                    kc = [torch.randn((B, ctx, hkv, hd), device="cuda", generator=g).half() for _ in range(copies)]
                    vc = [torch.randn((B, ctx, hkv, hd), device="cuda", generator=g).half() for _ in range(copies)]
                    f = lambda i, st: _lib.call("du_flash_decode", C.c_void_p(out.data_ptr()), C.c_void_p(q.data_ptr()),
                                                C.c_void_p(kc[i % copies].data_ptr()),
                                                C.c_void_p(vc[i % copies].data_ptr()), C.c_void_p(lens.data_ptr()),
                                                B, hq, hkv, hd, ctx, C.c_float(hd ** -0.5), C.c_void_p(st))
                    kern = "flash_decode_cluster_kernel (du_flash_decode)"
                else:
                    kc = [torch.randint(0, 256, (B, ctx, hkv, hd), dtype=torch.uint8, device="cuda", generator=g)
                          for _ in range(copies)]
                    vc = [torch.randint(0, 256, (B, ctx, hkv, hd), dtype=torch.uint8, device="cuda", generator=g)
                          for _ in range(copies)]
                    # words: fp16 scale 0.01 (0x211F) | fp16 zero point 128 (0x5800) << 16
                    ksz = torch.full((B, ctx, hkv), 0x5800211F, dtype=torch.int32, device="cuda")
                    f = lambda i, st: _lib.call("du_flash_decode_kv8", C.c_void_p(out.data_ptr()),
                                                C.c_void_p(q.data_ptr()), C.c_void_p(kc[i % copies].data_ptr()),
                                                C.c_void_p(ksz.data_ptr()), C.c_void_p(vc[i % copies].data_ptr()),
                                                C.c_void_p(ksz.data_ptr()), C.c_void_p(lens.data_ptr()),
                                                B, hq, hkv, hd, ctx, C.c_float(hd ** -0.5), C.c_void_p(st))
                    kern = "flash_decode_cluster_kernel, INT8 cache (du_flash_decode_kv8)"
                ms = _graph_ms(f, max(8, min(64, int(2e9 / kv_bytes))))
                gbs = kv_bytes / (ms / 1e3) / 1e9
                print(json.dumps({"sweep": "flash_decode", "kv": kv, "ctx": ctx, "batch": B, "us": round(ms * 1e3, 2),
                                  "GB_s": round(gbs, 1), "frac_hbm": round(gbs / peak, 4), "peak_kind": kind,
                                  "copies": copies, "kernel": kern,
                                  "timing": "CUDA graph of the launches, caches rotated over >= 0.6 GB"}), flush=True)
                del kc, vc


def run_gemv_phases(args):
    """Where the time of a decode GEMV goes, from the timing build's per-CTA
    %globaltimer stamps (gemv_stamps.cuh): for each stage boundary (previous GEMV
    -> this GEMV; attention sits between QKV and O), medians over the layers of the
    second of two decode steps of: this launch's first / median / last CTA entry,
    the moment its dependency wait returned (one instant for every CTA), activation
    staging, the weight stream of the last warp and the last exit, all in ns after
    the previous GEMV's last stamp; and per SM the gap between the previous
    kernel's last stamp on that SM and this kernel's first CTA entry there."""
    import ctypes as C
    import torch
    from deepunity_b200 import _lib
    from deepunity_b200.build import STAMPS_LIB
    if not os.path.exists(STAMPS_LIB):
        raise SystemExit(f"{STAMPS_LIB} is missing: python -m deepunity_b200.build --stamps")
    _lib.LIB_PATH = STAMPS_LIB          # before the library is first loaded
    from deepunity_b200.llm import CONFIGS, KVQuant, LlamaForCausalLM, LLMQuant
    torch.cuda.set_device(0)
    cfg = CONFIGS[args.model]
    quant = LLMQuant.INT4 if args.model == "llama-8b" else LLMQuant.INT8
    m = LlamaForCausalLM(cfg, quant, kv_quant=KVQuant.INT8 if args.kv == "int8" else KVQuant.FP16,
                         max_context_length=args.prompt + 64, max_batch=1, seed=0, device=0)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (1, args.prompt)).astype(np.int32)
    _, nxt = m.forward(prompt, want_logits=False)
    toks = m.decode_loop(nxt.copy(), max(args.warmup, 3))
    L = C.CDLL(STAMPS_LIB)
    torch.cuda.synchronize()
    if L.du_gemv_stamps_reset() != 0:
        raise SystemExit("du_gemv_stamps_reset failed")
    m.decode_loop(toks[-1].copy(), 2)
    torch.cuda.synchronize()
    slots, ctas = C.c_int(), C.c_int()
    L.du_gemv_stamps_read(None, None, C.byref(slots), C.byref(ctas))
    buf = np.zeros(slots.value * ctas.value * 8, np.uint64)
    cnt = np.zeros(ctas.value, np.uint32)
    if L.du_gemv_stamps_read(buf.ctypes.data_as(C.c_void_p), cnt.ctypes.data_as(C.c_void_p),
                             C.byref(slots), C.byref(ctas)) != 0:
        raise SystemExit("du_gemv_stamps_read failed")
    buf = buf.reshape(slots.value, ctas.value, 8).astype(np.int64)
    n0 = int(cnt[0])
    if n0 < 4 or n0 > slots.value or n0 % 2:
        raise SystemExit(f"unexpected launch count {n0}")
    tag = lambda s_, c: (int(buf[s_, c, 7] >> 40), int((buf[s_, c, 7] >> 16) & 0xFFFFFF))
    # each CTA index's records are its launches in order; CTA 0 takes part in all of them
    seqs = [[tag(s_, c) for s_ in range(int(cnt[c]))] for c in range(ctas.value)]
    seq0 = seqs[0]
    part = []                                   # per launch: {cta: slot}
    for k in range(n0):
        part.append({})
    for c in range(ctas.value):
        j = 0
        for k in range(n0):
            if j < len(seqs[c]) and seqs[c][j] == seq0[k]:
                part[k][c] = j
                j += 1
    H, I = cfg.hidden_size, cfg.intermediate_size
    hd = cfg.head_dim
    names = {((cfg.num_heads_q + 2 * cfg.num_heads_kv) * hd, H): "qkv", (H, cfg.num_heads_q * hd): "o_proj",
             (2 * I, H): "gate_up", (H, I): "down"}
    def rec(k):
        cs = sorted(part[k])
        return np.array([buf[part[k][c], c, :] for c in cs])
    out = {}
    for k in range(n0 // 2 + 1, n0):
        a, b = rec(k - 1), rec(k)
        na, nb = names.get(seq0[k - 1], "lm_head"), names.get(seq0[k], "lm_head")
        if "lm_head" in (na, nb):
            continue
        a_last = np.maximum(a[:, 4], a[:, 5])
        t0 = a_last.max()
        a_sm, b_sm = a[:, 7] & 0xFFFF, b[:, 7] & 0xFFFF
        hand = [b[b_sm == s_, 0].min() - a_last[a_sm == s_].max() for s_ in np.unique(b_sm) if (a_sm == s_).any()]
        row = [b[:, 0].min() - t0, np.median(b[:, 0]) - t0, b[:, 0].max() - t0, b[:, 2].min() - t0,
               np.median(b[:, 3] - b[:, 2]), np.median(b[:, 4] - b[:, 3]), (b[:, 4] - b[:, 3]).max(),
               np.maximum(b[:, 4], b[:, 5]).max() - t0, np.median(hand) if hand else float("nan")]
        out.setdefault(f"{na} -> {nb}", []).append(row)
    keys = ["entry_first", "entry_median", "entry_last", "dependency_met", "staging_median", "stream_median",
            "stream_max", "last_exit", "sm_handoff_median"]
    for key, rows in out.items():
        med = np.median(np.array(rows, dtype=np.float64), axis=0)
        print(json.dumps({"gemv_phases": key, "layers": len(rows), "unit": "ns after the previous GEMV's last stamp",
                          **{k_: round(float(v), 0) for k_, v in zip(keys, med)},
                          "model": args.model, "kv": args.kv, "prompt": args.prompt}), flush=True)


def main():
    args = parse()
    if args.gemv_phases:
        return run_gemv_phases(args)
    if args.sweep == "gemv":
        return run_sweep_gemv(args)
    if args.sweep == "attn":
        return run_sweep_attn(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
