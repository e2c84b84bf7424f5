"""Benchmark: greedy Llama decode through libstb200.so (the BF16-weight Linear hot path of scala-torch).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload: SmolLM2-135M-shaped Llama, random-init BF16 weights
~N(0,0.02) generated on the device, RMSNorm weights 1, batch 1, a 128-token prompt of ids uniform
in [0,49152), greedy decode of 128 tokens with the KV cache resident in HBM.  One step = one
generate call (prefill + 128 decode tokens).  Metric: generated tokens per second of the whole
generation (prefill included).  With N GPUs every rank decodes its own sequence (independent
replicas, weak scaling); value = all ranks' tokens / the slowest rank's time.

Output: one JSON line on rank 0 (value from device events, e2e through the C-ABI with host
buffers, roofline of the dominant kernel, CPU baseline of the oracle restatement, clocks).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "scala-torch_b200"))
sys.path.insert(0, ROOT)

SMOL = dict(vocab_size=49152, hidden_size=576, intermediate_size=1536, num_layers=30, num_attention_heads=9,
            num_key_value_heads=3, max_positions=2048, tie_word_embeddings=True, rope_theta=10000.0,
            rms_norm_eps=1e-6, eos_token_ids=())
PROMPT, NEW, SEED = 128, 128, 2024


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit())
        mx = max((float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 3 + i and r[3 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.rows)}


def max_over_ranks(values, device=None):
    """Element-wise maximum over all ranks of the current process group (the slowest rank's
    times); `device` None keeps the tensor on the CPU (gloo)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def cpu_baseline_smol(seconds_budget: float = 20.0):
    """The oracle restatement of the reference CPU path (all host threads) on a bounded sample of the
    same workload: same model and prompt length, as many generated tokens as fit the budget."""
    import numpy as np

    import oracle
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from llama_fixtures import oracle_model
    from scalatorch.models import LlamaConfig
    cfg = LlamaConfig(**SMOL)
    model = oracle_model(cfg, seed=SEED)
    threads = oracle.max_threads()
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, PROMPT).tolist()
    t0 = time.perf_counter()
    model.generate(prompt[:PROMPT], 1)
    t_first = time.perf_counter() - t0
    # tokens after the first cost one decode step each; estimate how many fit the budget
    t0 = time.perf_counter()
    model.generate(prompt[:8], 2)
    t_small = time.perf_counter() - t0
    per_token = max(t_small / 2, 1e-3)
    n = int(max(1, min(NEW, (seconds_budget - t_first) / per_token)))
    t0 = time.perf_counter()
    out = model.generate(prompt, n)
    dt = time.perf_counter() - t0
    gen = len(out) - PROMPT
    return {"value": gen / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{PROMPT}-token prompt + {gen} greedy tokens (of {NEW}) on the oracle, {dt:.1f} s"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, world, rank)

    import numpy as np
    import torch
    import torch.distributed as dist
    from scalatorch import ffm
    from scalatorch.models import BackendLlama, LlamaConfig

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    hbm_peak, tc_peak, peak_kind = peaks()
    session = ffm.B200Session(local, 170 << 30)
    cfg = LlamaConfig(**SMOL)
    model = BackendLlama.prepare_random(session, cfg, seed=SEED)
    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, cfg.vocab_size, PROMPT).astype(np.int64)
    # pinned host buffers for the end-to-end path
    lib = ffm.library()
    import ctypes
    hp = ctypes.c_void_p()
    ffm.call("stb_host_alloc", PROMPT * 8, ctypes.byref(hp))
    pin_prompt = np.ctypeslib.as_array((ctypes.c_int64 * PROMPT).from_address(hp.value))
    pin_prompt[:] = prompt
    ho = ctypes.c_void_p()
    ffm.call("stb_host_alloc", (PROMPT + NEW) * 8, ctypes.byref(ho))
    pin_out = np.ctypeslib.as_array((ctypes.c_int64 * (PROMPT + NEW)).from_address(ho.value))
    gen = np.zeros(1, np.int32)
    tm = np.zeros(2, np.float32)

    def step():
        ffm.call("stb_llama_generate", model.handle, pin_prompt.ctypes.data, 1, PROMPT, NEW, None, 0,
                 pin_out.ctypes.data, gen.ctypes.data, tm.ctypes.data)
        return float(tm[0]) + float(tm[1]), float(tm[0]), float(tm[1])

    for _ in range(max(args.warmup, 3)):
        step()
    session.sync()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = session.launches
    dev_ms, pre_ms, dec_ms = [], [], []
    with Clocks(local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            d, p, q = step()
            dev_ms.append(d)
            pre_ms.append(p)
            dec_ms.append(q)
        session.sync()
        wall = time.perf_counter() - t0
    torch.cuda.synchronize()
    launches = session.launches - launches0
    assert int(gen[0]) == NEW, "generation stopped early"
    dev_total = sum(dev_ms) / 1000.0
    if world > 1:
        dev_total, wall = max_over_ranks([dev_total, wall], device="cuda")
        dist.barrier()
    tokens = NEW * args.steps * world
    value = tokens / dev_total
    e2e = tokens / wall

    roof = roofline_lm_head(session, cfg, hbm_peak, peak_kind)
    line = {
        "metric": "greedy decode tokens/s (SmolLM2-135M-shaped, BF16 weights, batch 1, 128-token prompt + 128 new)",
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_total * 1000 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16-weights/f32-compute", "data": "synthetic (device counter-RNG weights, random prompt ids)",
        "config": {"workload": "smollm2-135m-shaped greedy decode", "batch": 1, "prompt": PROMPT, "new_tokens": NEW,
                   "layers": 30, "hidden": 576, "vocab": 49152, "parallelism": f"replicas x{world}",
                   "prefill_ms": round(sum(pre_ms) / len(pre_ms), 3), "decode_ms": round(sum(dec_ms) / len(dec_ms), 3),
                   "decode_tok_s": round(NEW * 1000 / (sum(dec_ms) / len(dec_ms)), 1),
                   "weight_bytes_per_token": 268959744,
                   "l2": "inputs larger than L2: 269 MB of weights streamed per token vs 126 MB L2"},
        "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": PROMPT * 8,
                "d2h_bytes_per_step": (NEW * 8 + 8 * 3)},
        "gpu_launches": int(launches),
        "roofline": roof,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline_smol()
        except Exception as e:  # reported, never silently replaced
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    ffm.call("stb_host_free", hp)
    ffm.call("stb_host_free", ho)
    model.close()
    session.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def roofline_lm_head(session, cfg, hbm_peak, peak_kind):
    """The lm_head GEMV (49152 x 576 BF16, M = 1; the largest per-token kernel) timed alone with
    CUDA events on the session stream, L2 flushed (256 MB write) before every launch."""
    import ctypes

    import torch
    from scalatorch import ffm
    N, K = cfg.vocab_size, cfg.hidden_size
    stream = torch.cuda.ExternalStream(session.stream)
    w = torch.empty(N * K, dtype=torch.bfloat16, device="cuda")
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    wt = ffm.DeviceTensor(session, w.data_ptr(), (K, N), ffm.STB_BF16, N * K * 2, transposed_weight=True, owner=False)
    session.fill_normal(wt, 1, 1, 0.02)
    session.sync()
    torch.cuda.synchronize()
    times = []
    for i in range(23):
        with torch.cuda.stream(stream):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ffm.call("stb_linear", session.handle, x.data_ptr(), w.data_ptr(), ffm.STB_BF16, 0, y.data_ptr(), 1, N, K)
        e1.record(stream)
        e1.synchronize()
        if i >= 3:
            times.append(e0.elapsed_time(e1) / 1000.0)
    t = sorted(times)[len(times) // 2]
    algo = N * K * 2 + K * 4 + N * 4
    achieved = algo / t / 1e9
    return {"kernel": "gemv_kernel (lm_head 49152x576 BF16, M=1)", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
            "peak_source": f"{peak_kind} hbm_gbs", "algorithmic_bytes": algo, "launch_us": round(t * 1e6, 2),
            "traffic": None}


def reference_arm(args, world, rank):
    """The reference's CPU path (oracle restatement; the Scala/JVM reference cannot run here) on all host
    threads, same metric and config; bounded sample per step.  Rank 0 alone runs under torchrun."""
    if rank != 0:
        return
    import oracle
    samples = []
    for i in range(max(args.warmup, 0) + args.steps):
        r = cpu_baseline_smol(seconds_budget=15.0)
        if i >= args.warmup:
            samples.append(r)
    v = sum(s["value"] for s in samples) / len(samples)
    line = {"impl": "reference", "metric": "greedy decode tokens/s (SmolLM2-135M-shaped, BF16 weights, batch 1, 128-token prompt + 128 new)",
            "value": round(v, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "smollm2-135m-shaped greedy decode", "batch": 1,
                                            "prompt": PROMPT, "new_tokens": NEW},
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                             "sample": samples[-1]["sample"]},
            "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
