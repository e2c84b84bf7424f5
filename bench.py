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
        self.window = []  # [start, end) sample indices of the timed region (mark() twice)

    def mark(self):
        self.window.append(len(self.rows))

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
        rows = self.rows
        if len(self.window) == 2 and self.window[1] > self.window[0]:
            rows = rows[self.window[0]:self.window[1] + 1]  # samples taken during the timed region
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(r[0]) for r in rows if r[0].replace(".", "").isdigit())
        mx = max((float(r[1]) for r in rows if r[1].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 3 + i and r[3 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def max_over_ranks(values, device=None):
    """Element-wise maximum over all ranks of the current process group (the slowest rank's
    times); `device` None keeps the tensor on the CPU (gloo)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def cpu_baseline_smol(seconds_budget: float = 20.0, model=None, with_model: bool = False):
    """The oracle restatement of the reference CPU path (all host threads) on the same workload: the
    full 128 + 128 generation when it fits the budget, else the prompt plus as many greedy tokens as
    fit, with the remaining decode steps extrapolated at the measured per-token rate."""
    import numpy as np

    import oracle
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from llama_fixtures import oracle_model
    from scalatorch.models import LlamaConfig
    cfg = LlamaConfig(**SMOL)
    if model is None:
        model = oracle_model(cfg, seed=SEED)
    threads = oracle.max_threads()
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, PROMPT).tolist()
    t0 = time.perf_counter()
    model.generate(prompt, 1)  # prefill of the 128-token prompt + the first pick
    t_prefill = time.perf_counter() - t0
    n = 8
    t0 = time.perf_counter()
    model.generate(prompt, 1 + n)
    per_token = max((time.perf_counter() - t0 - t_prefill) / n, 1e-6)
    if t_prefill + NEW * per_token <= seconds_budget:
        t0 = time.perf_counter()
        out = model.generate(prompt, NEW)
        dt = time.perf_counter() - t0
        r = {"value": (len(out) - PROMPT) / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
             "sample": f"full {PROMPT}-token prompt + {len(out) - PROMPT} greedy tokens on the oracle, {dt:.2f} s"}
    else:
        dt = t_prefill + (NEW - 1) * per_token
        r = {"value": NEW / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
             "sample": f"{PROMPT}-token prefill {t_prefill:.2f} s + {per_token * 1000:.1f} ms/token measured over "
                       f"{n} tokens, extrapolated to {NEW} tokens"}
    # One host thread (numscala's ScalarF32Kernels run single-threaded): decode rate only, on a
    # 4-token prompt, so the sample stays a few seconds.
    model.threads = 1
    try:
        short = prompt[:4]
        t0 = time.perf_counter()
        model.generate(short, 1)
        t1 = time.perf_counter()
        model.generate(short, 3)
        per_token_1 = max((time.perf_counter() - t1 - (t1 - t0)) / 2, 1e-6)
    finally:
        model.threads = threads
    r["single_thread"] = {"decode_ms_per_token": round(per_token_1 * 1000, 1),
                          "decode_tokens_s": round(1.0 / per_token_1, 3)}
    r["host"] = host_cores()
    return (r, model) if with_model else r


LLAMA70B = dict(vocab_size=128256, hidden_size=8192, intermediate_size=28672, num_layers=80,
                num_attention_heads=64, num_key_value_heads=8, max_positions=8192, tie_word_embeddings=False,
                rope_theta=500000.0, rms_norm_eps=1e-5, eos_token_ids=())


class Generator:
    """One generate call through the C ABI with pinned host prompt/output buffers (the e2e path)."""

    def __init__(self, model, prompts, new):
        import ctypes

        import numpy as np
        from scalatorch import ffm
        self.ffm, self.model, self.new = ffm, model, new
        self.batch, self.plen = prompts.shape
        n_in, n_out = prompts.size, self.batch * (self.plen + new)
        self.hp, self.ho = ctypes.c_void_p(), ctypes.c_void_p()
        ffm.call("stb_host_alloc", n_in * 8, ctypes.byref(self.hp))
        ffm.call("stb_host_alloc", n_out * 8, ctypes.byref(self.ho))
        self.prompt = np.ctypeslib.as_array((ctypes.c_int64 * n_in).from_address(self.hp.value))
        self.prompt[:] = prompts.ravel()
        self.out = np.ctypeslib.as_array((ctypes.c_int64 * n_out).from_address(self.ho.value))
        self.gen = np.zeros(self.batch, np.int32)
        self.tm = np.zeros(2, np.float32)
        self.h2d, self.d2h = n_in * 8, self.batch * new * 8 + 8 * (2 + 2 * self.batch)

    def __call__(self):
        self.ffm.call("stb_llama_generate", self.model.handle, self.prompt.ctypes.data, self.batch, self.plen,
                      self.new, None, 0, self.out.ctypes.data, self.gen.ctypes.data, self.tm.ctypes.data)
        return float(self.tm[0]), float(self.tm[1])

    def close(self):
        self.ffm.call("stb_host_free", self.hp)
        self.ffm.call("stb_host_free", self.ho)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="smollm2",
                    choices=["smollm2", "llama70b", "linear", "prefill", "single", "roofline"],
                    help="single: the single-Linear configuration [16,576]x[1536,576]; roofline: only the "
                    "SmolLM2 lm_head roofline leg of the default line (for profiling)")
    ap.add_argument("--shapes", default="", help="linear/prefill: comma list of shape names to run (default all)")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"],
                    help="linear/prefill: weight type (F16 prefill rounds the activations to F16)")
    ap.add_argument("--ms", default="", help="linear/prefill: comma list of token-row counts M (default 1,4,16,32 "
                    "for linear, 2048,8192 for prefill)")
    ap.add_argument("--batch", type=int, default=1, help="llama70b: decode batch (1, 8, 32)")
    ap.add_argument("--prompt", type=int, default=512, help="llama70b: prompt tokens")
    ap.add_argument("--new", type=int, default=32, help="llama70b: generated tokens per step")
    ap.add_argument("--layers", type=int, default=0, help="llama70b: fewer layers (small profiling cases only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, world, rank)
    if args.workload in ("linear", "prefill"):
        return linear_sweep(args, world, rank, local)
    if args.workload == "single":
        return single_linear(args, local)
    if args.workload == "roofline":
        import torch
        from scalatorch import ffm
        from scalatorch.models import LlamaConfig
        torch.cuda.set_device(local)
        hbm_peak, _, peak_kind = peaks()
        session = ffm.B200Session(local, 8 << 30)
        print(json.dumps(roofline_lm_head(session, LlamaConfig(**SMOL), hbm_peak, peak_kind)), flush=True)
        session.close()
        return 0

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
    session = ffm.B200Session(local, 178 << 30)
    tp = args.workload == "llama70b"
    if tp:
        cfg = LlamaConfig(**(dict(LLAMA70B, num_layers=args.layers) if args.layers else LLAMA70B))
        batch, plen, new = args.batch, args.prompt, args.new
        if world > 1:  # one communicator for the tensor-parallel group
            uid = [ffm.B200Session.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(uid, src=0)
            session.init_tp(world, rank, uid[0])
        model = BackendLlama.prepare_random(session, cfg, seed=SEED, tp_rank=rank, tp_size=world)
        prompts = np.random.default_rng(SEED).integers(0, cfg.vocab_size, (batch, plen)).astype(np.int64)
    else:
        cfg = LlamaConfig(**SMOL)
        batch, plen, new = 1, PROMPT, NEW
        model = BackendLlama.prepare_random(session, cfg, seed=SEED)
        prompts = np.random.default_rng(SEED + rank).integers(0, cfg.vocab_size, (1, PROMPT)).astype(np.int64)
    step = Generator(model, prompts, new)

    with Clocks(local) as clocks:  # started before the warm-up so its start-up never overlaps the timing
        for _ in range(max(args.warmup, 3)):
            step()
        session.sync()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.mark()
        launches0 = session.launches
        pre_ms, dec_ms = [], []
        t0 = time.perf_counter()
        for _ in range(args.steps):
            p, q = step()
            pre_ms.append(p)
            dec_ms.append(q)
        session.sync()
        wall = time.perf_counter() - t0
        clocks.mark()
    torch.cuda.synchronize()
    launches = session.launches - launches0
    assert int(step.gen.min()) == new, "generation stopped early"
    pre_s, dec_s = sum(pre_ms) / 1000.0, sum(dec_ms) / 1000.0
    if world > 1:
        pre_s, dec_s, wall = max_over_ranks([pre_s, dec_s, wall], device="cuda")
        dist.barrier()

    if tp:
        # tensor parallel: the ranks produce one sequence batch together; metric = decode tokens/s,
        # the new - 1 tokens per row of the decode phase (the first comes out of the prefill)
        value = batch * max(new - 1, 1) * args.steps / dec_s
        e2e = batch * new * args.steps / wall  # whole generate calls, host buffers
        line = {
            "metric": "greedy decode tokens/s (Llama-3-70B-shaped, BF16 weights, tensor parallel)",
            "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round((pre_s + dec_s) * 1000 / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16-weights/f32-compute",
            "data": "synthetic (device counter-RNG weights, random prompt ids)",
            "config": {"workload": "llama3-70b-shaped greedy decode", "batch": batch, "prompt": plen,
                       "new_tokens": new, "layers": cfg.num_layers, "hidden": 8192, "vocab": 128256,
                       "parallelism": f"tp{world}", "prefill_ms": round(pre_s * 1000 / args.steps, 3),
                       "decode_ms": round(dec_s * 1000 / args.steps, 3),
                       "decode_ms_per_token": round(dec_s * 1000 / args.steps / max(new - 1, 1), 3),
                       "weight_bytes_per_rank": model.weight_bytes,
                       "l2": "inputs larger than L2: 141 GB of weights"},
            "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": step.h2d,
                    "d2h_bytes_per_step": step.d2h},
            "gpu_launches": int(launches), "clocks": clocks.summary(),
        }
        # HBM roofline of the decode step: every rank streams its weight shard once per token
        per_tok = dec_s / args.steps / max(new - 1, 1)
        achieved = model.weight_bytes / per_tok / 1e9
        line["roofline"] = {"kernel": "decode step (all kernels, per rank)", "bound": "hbm",
                            "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                            "frac": round(achieved / hbm_peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                            "algorithmic_bytes": model.weight_bytes, "traffic": None}
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline_70b_layer()
            except Exception as e:
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    else:
        tokens = new * args.steps * world
        value = tokens / (pre_s + dec_s)
        e2e = tokens / wall
        line = {
            "metric": "greedy decode tokens/s (SmolLM2-135M-shaped, BF16 weights, batch 1, 128-token prompt + 128 new)",
            "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round((pre_s + dec_s) * 1000 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16-weights/f32-compute",
            "data": "synthetic (device counter-RNG weights, random prompt ids)",
            "config": {"workload": "smollm2-135m-shaped greedy decode", "batch": 1, "prompt": PROMPT, "new_tokens": NEW,
                       "layers": 30, "hidden": 576, "vocab": 49152, "parallelism": f"replicas x{world}",
                       "prefill_ms": round(pre_s * 1000 / args.steps, 3),
                       "decode_ms": round(dec_s * 1000 / args.steps, 3),
                       "decode_tok_s": round((NEW - 1) * args.steps / dec_s, 1),
                       "weight_bytes_per_token": 268959744,
                       "l2": "inputs larger than L2: 269 MB of weights streamed per token vs 126 MB L2"},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": step.h2d,
                    "d2h_bytes_per_step": step.d2h},
            "gpu_launches": int(launches),
            "roofline": decode_step_roofline((NEW - 1) * args.steps / dec_s, hbm_peak, peak_kind,
                                             roofline_lm_head(session, cfg, hbm_peak, peak_kind)),
            "clocks": clocks.summary(),
        }
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline_smol()
            except Exception as e:  # reported, never silently replaced
                line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    step.close()
    model.close()
    session.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


LLAMA8B_SHAPES = {"q": (4096, 4096), "k": (1024, 4096), "v": (1024, 4096), "o": (4096, 4096),
                  "gate": (14336, 4096), "up": (14336, 4096), "down": (4096, 14336), "lm_head": (128256, 4096)}


def linear_sweep(args, world, rank, local):
    """The Linear sweeps (--workload linear: decode GEMV, FP32 activations, M = 1/4/16/32; --workload
    prefill: tcgen05 GEMM, M = 2048/8192) on Llama-3-8B projection shapes with
    device-generated BF16 weights ~N(0,0.02).  Each launch is timed alone with CUDA events on the
    session stream after a 256 MB L2 flush; the median of the timed launches is reported."""
    import numpy as np
    import torch
    from scalatorch import ffm
    torch.cuda.set_device(local)
    hbm_peak, tc_peak, peak_kind = peaks()
    s = ffm.B200Session(local, 100 << 30)
    stream = torch.cuda.ExternalStream(s.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    prefill = args.workload == "prefill"
    wdt = ffm.STB_F16 if args.dtype == "f16" else ffm.STB_BF16
    tdt = torch.float16 if args.dtype == "f16" else torch.bfloat16
    wname = args.dtype.upper()
    ms = (2048, 8192) if prefill else (1, 4, 16, 32)
    if args.ms:
        ms = tuple(int(v) for v in args.ms.split(","))
    names = [n for n in LLAMA8B_SHAPES if not args.shapes or n in args.shapes.split(",")]
    fn = "stb_linear_prefill" if prefill else "stb_linear"
    results, clocks = [], Clocks(local)
    launches0 = s.launches
    with clocks:
        clocks.mark()
        for si, name in enumerate(names):
            n, k = LLAMA8B_SHAPES[name]
            w = torch.empty(n * k, dtype=tdt, device="cuda")
            wt = ffm.DeviceTensor(s, w.data_ptr(), (k, n), wdt, n * k * 2, transposed_weight=True, owner=False)
            s.fill_normal(wt, SEED, 100 + si, 0.02)
            for m in ms:
                x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(m))
                y = torch.empty(m, n, device="cuda")
                torch.cuda.synchronize()
                s.sync()
                times = []
                for it in range(args.warmup + args.steps):
                    with torch.cuda.stream(stream):
                        flush.zero_()
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(stream)
                    ffm.call(fn, s.handle, x.data_ptr(), w.data_ptr(), wdt, 0, y.data_ptr(), m, n, k)
                    e1.record(stream)
                    e1.synchronize()
                    if it >= args.warmup:
                        times.append(e0.elapsed_time(e1) / 1000.0)
                t = sorted(times)[len(times) // 2]
                algo = n * k * 2 + m * k * 4 + m * n * 4
                results.append({"shape": name, "M": m, "N": n, "K": k, "us": round(t * 1e6, 2),
                                "GB_s": round(algo / t / 1e9, 1), "TFLOP_s": round(2 * m * n * k / t / 1e12, 2),
                                "hbm_frac": round(algo / t / 1e9 / hbm_peak, 4),
                                "tensor_frac": round(2 * m * n * k / t / 1e12 / tc_peak, 4)})
                del x, y
            del w
            torch.cuda.empty_cache()
        clocks.mark()
    launches = s.launches - launches0
    # end-to-end through the host-buffer C ABI on the first shape at the smallest M
    n, k = LLAMA8B_SHAPES[names[0]]
    m = ms[0]
    w = torch.empty(n * k, dtype=tdt, device="cuda")
    wt = ffm.DeviceTensor(s, w.data_ptr(), (k, n), wdt, n * k * 2, transposed_weight=True, owner=False)
    s.fill_normal(wt, SEED, 100, 0.02)
    s.sync()
    hx = np.random.default_rng(0).standard_normal((m, k)).astype(np.float32)
    hy = np.empty((m, n), np.float32)
    e2e_t = None
    if not prefill:
        for it in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            ffm.call("stb_linear_host", s.handle, hx.ctypes.data, w.data_ptr(), wdt, 0, hy.ctypes.data, m, n, k)
            dt = time.perf_counter() - t0
            e2e_t = dt if e2e_t is None or it < args.warmup else min(e2e_t, dt)
    s.close()
    if prefill:
        flops = sum(2 * r["M"] * r["N"] * r["K"] for r in results)
        secs = sum(r["us"] for r in results) / 1e6
        value, unit = flops / secs / 1e12, "TFLOP/s"
        top = max(results, key=lambda r: r["us"])
        roof = {"kernel": f"gemm_tc2_kernel, CTA pairs ({top['shape']} M={top['M']})", "bound": "tensor",
                "achieved": top["TFLOP_s"], "peak": tc_peak, "unit": "TFLOP/s", "frac": top["tensor_frac"],
                "peak_source": f"{peak_kind} bf16_tflops (burst)", "traffic": None}
        metric = f"prefill GEMM TFLOP/s (Llama-3-8B projections, {wname} weights, activations rounded to {wname})"
    else:
        m1 = [r for r in results if r["M"] == min(ms)]
        byts = sum(r["N"] * r["K"] * 2 + r["K"] * 4 + r["N"] * 4 for r in m1)
        secs = sum(r["us"] for r in m1) / 1e6
        value, unit = byts / secs / 1e9, "GB/s"
        top = max(m1, key=lambda r: r["us"])
        roof = {"kernel": f"gemv_kernel ({top['shape']} M={top['M']})", "bound": "hbm", "achieved": top["GB_s"],
                "peak": hbm_peak, "unit": "GB/s", "frac": top["hbm_frac"], "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_bytes": top["N"] * top["K"] * 2 + top["K"] * 4 + top["N"] * 4, "traffic": None}
        metric = f"decode GEMV GB/s at M={min(ms)} (Llama-3-8B projections, {wname} weights, FP32 activations)"
    line = {"metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(secs * 1000 / max(len(results), 1), 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"{args.dtype}-weights/f32-accumulate",
            "data": "synthetic (device counter-RNG weights, N(0,1) activations)",
            "config": {"workload": f"llama3-8b {args.workload} sweep", "l2": "flushed (256 MB write) before every launch",
                       "shapes": results},
            "gpu_launches": int(launches), "roofline": roof, "clocks": clocks.summary()}
    if e2e_t:
        line["e2e"] = {"value": round((n * k * 2 + m * k * 4 + m * n * 4) / e2e_t / 1e9, 2), "unit": "GB/s",
                       "h2d_bytes_per_step": m * k * 4, "d2h_bytes_per_step": m * n * 4,
                       "note": f"stb_linear_host on {names[0]} M={m} (host x in, host y out)"}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_linear_shapes([(LLAMA8B_SHAPES[r] + (r,)) for r in names], min(ms), prefill)
    print(json.dumps(line), flush=True)


SINGLE_M, SINGLE_N, SINGLE_K = 16, 1536, 576
SINGLE_BYTES = SINGLE_N * SINGLE_K * 2 + SINGLE_M * SINGLE_K * 4 + SINGLE_M * SINGLE_N * 4  # 1,904,640 B


def host_cores() -> dict:
    """Host CPUs visible to this process (nproc) and in its affinity mask."""
    try:
        affinity = len(os.sched_getaffinity(0))
    except AttributeError:
        affinity = os.cpu_count()
    return {"nproc": os.cpu_count(), "affinity": affinity}


def _seconds_per_call(fn, seconds: float) -> tuple:
    fn()  # first call outside the clock (page faults of the output)
    t0, reps = time.perf_counter(), 0
    while True:
        fn()
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            return dt / reps, reps


def cpu_single_linear(seconds: float = 3.0):
    """The reference CPU nn.Linear on the single-Linear configuration (weights widened to F32 once, as
    SafeTensors.readFloat does at load; numscala's transposed-right order), on all host threads and
    on one thread (numscala's ScalarF32Kernels are single-threaded)."""
    import numpy as np

    import oracle
    x = np.random.default_rng(1).standard_normal((SINGLE_M, SINGLE_K)).astype(np.float32)
    wf = oracle.widen(oracle.normal_bf16(SINGLE_N * SINGLE_K, 1, 1, 0.02), oracle.BF16).reshape(SINGLE_N, SINGLE_K)
    threads = oracle.max_threads()
    dt, reps = _seconds_per_call(lambda: oracle.matmul_tr(x, wf, threads), seconds)
    dt1, reps1 = _seconds_per_call(lambda: oracle.matmul_tr(x, wf, 1), seconds / 2)
    return {"value": round(SINGLE_BYTES / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"single-Linear x[16,576].W[1536,576]^T: {reps} calls on {threads} threads, "
                      f"{reps1} on 1 thread", "us_per_call": round(dt * 1e6, 2),
            "single_thread": {"value": round(SINGLE_BYTES / dt1 / 1e9, 3), "us_per_call": round(dt1 * 1e6, 2)},
            "host": host_cores()}


def cpu_linear_shapes(shapes, m: int, prefill: bool, seconds: float = 1.0):
    """The reference CPU path on each Llama-3-8B projection shape at M = m rows (weights widened to F32,
    numscala order, all host threads), each on a bounded sample of output rows: up to 512 MB of
    widened weights for decode shapes (larger than a host's last-level cache, so the sample streams
    from DRAM as the full shape does), 128 rows for prefill (compute-bound).  The CPU cost is linear
    in the output rows, so the time is scaled to the full N.  value aggregates the shapes as the GPU
    line does: total algorithmic bytes (decode) or FLOPs (prefill) / total scaled time."""
    import numpy as np

    import oracle
    threads = oracle.max_threads()
    out, total_work, total_t = [], 0, 0.0
    for i, (n, k, name) in enumerate(shapes):
        rows = min(n, 128 if prefill else max(1, (512 << 20) // (4 * k)))
        wf = oracle.widen(oracle.normal_bf16(rows * k, SEED, 100 + i, 0.02), oracle.BF16).reshape(rows, k)
        x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
        if prefill:  # activations rounded to BF16, as on the tensor-core path
            x = oracle.widen(oracle.round_bf16(x), oracle.BF16)
        dt, reps = _seconds_per_call(lambda: oracle.matmul_tr(x, wf, threads), seconds)
        t_full = dt * n / rows
        work = 2 * m * n * k if prefill else n * k * 2 + m * k * 4 + m * n * 4
        total_work += work
        total_t += t_full
        out.append({"shape": name, "M": m, "rows_sampled": rows, "calls": reps, "ms_full": round(t_full * 1e3, 3)})
    value = total_work / total_t / (1e12 if prefill else 1e9)
    return {"value": round(value, 4), "unit": "TFLOP/s" if prefill else "GB/s", "cores": threads, "kind": "port",
            "sample": f"each shape at M={m} on {'128 output rows' if prefill else 'up to 512 MB of F32 weight rows'}"
                      " (or all), time scaled to the full N",
            "shapes": out, "host": host_cores()}


def single_linear(args, local):
    """The single-Linear configuration (x F32 [16,576] ~N(0,1), W BF16 [1536,576] ~N(0,0.02), no bias)
    through stb_linear.  One step = CALLS forwards.  Cold: a 256 MB L2 flush before every call and
    CUDA events around each call alone (the reported value, against HBM); warm: CALLS back-to-back
    calls between one event pair (the 1.8 MB weight stays in L2).  e2e: stb_linear_host with host
    x and y, wall clock per call."""
    import numpy as np
    import torch
    from scalatorch import ffm
    CALLS = 100
    torch.cuda.set_device(local)
    hbm_peak, _, peak_kind = peaks()
    s = ffm.B200Session(local, 4 << 30)
    stream = torch.cuda.ExternalStream(s.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    M, N, K = SINGLE_M, SINGLE_N, SINGLE_K
    w = torch.empty(N * K, dtype=torch.bfloat16, device="cuda")
    wt = ffm.DeviceTensor(s, w.data_ptr(), (K, N), ffm.STB_BF16, N * K * 2, transposed_weight=True, owner=False)
    s.fill_normal(wt, 1, 1, 0.02)
    hx = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
    hy = np.empty((M, N), np.float32)
    x = torch.from_numpy(hx).cuda()
    y = torch.empty(M, N, device="cuda")
    s.sync()
    torch.cuda.synchronize()

    def call():
        ffm.call("stb_linear", s.handle, x.data_ptr(), w.data_ptr(), ffm.STB_BF16, 0, y.data_ptr(), M, N, K)

    cold, warm, e2e, clocks = [], [], [], Clocks(local)
    launches0 = s.launches
    with clocks:
        for step in range(args.warmup + args.steps):
            if step == args.warmup:
                clocks.mark()
                launches0 = s.launches
            ts = []
            for _ in range(CALLS):
                with torch.cuda.stream(stream):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                call()
                e1.record(stream)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) / 1000.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(CALLS):
                call()
            e1.record(stream)
            e1.synchronize()
            if step >= args.warmup:
                cold.extend(ts)
                warm.append(e0.elapsed_time(e1) / 1000.0 / CALLS)
        clocks.mark()
        launches = s.launches - launches0
    for step in range(args.warmup + args.steps):
        ts = []
        for _ in range(CALLS):
            t0 = time.perf_counter()
            ffm.call("stb_linear_host", s.handle, hx.ctypes.data, w.data_ptr(), ffm.STB_BF16, 0, hy.ctypes.data, M, N, K)
            ts.append(time.perf_counter() - t0)
        if step >= args.warmup:
            e2e.extend(ts)
    s.close()
    med = lambda v: sorted(v)[len(v) // 2]
    t_cold, t_warm, t_e2e = med(cold), med(warm), med(e2e)
    achieved = SINGLE_BYTES / t_cold / 1e9
    line = {"metric": "single-Linear GB/s (x F32 [16,576] . W BF16 [1536,576]^T, L2 flushed before each call)",
            "value": round(achieved, 2), "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_cold * CALLS * 1000, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16-weights/f32-accumulate",
            "data": "synthetic (device counter-RNG weights seed 1 stream 1, N(0,1) activations seed 1)",
            "config": {"workload": "single Linear", "M": M, "N": N, "K": K, "calls_per_step": CALLS,
                       "l2": "flushed (256 MB write) before every cold call; warm calls back to back",
                       "cold_us": round(t_cold * 1e6, 2), "warm_us": round(t_warm * 1e6, 2),
                       "warm_GB_s": round(SINGLE_BYTES / t_warm / 1e9, 1)},
            "gpu_launches": int(launches),
            "roofline": {"kernel": "stb_linear (prep + gemm_skinny_kernel + fixup, M=16)", "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes": SINGLE_BYTES, "traffic": None},
            "e2e": {"value": round(SINGLE_BYTES / t_e2e / 1e9, 3), "unit": "GB/s", "us_per_call": round(t_e2e * 1e6, 2),
                    "h2d_bytes_per_step": CALLS * M * K * 4, "d2h_bytes_per_step": CALLS * M * N * 4,
                    "note": "stb_linear_host (host x in, host y out), median wall clock per call"},
            "clocks": clocks.summary()}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_single_linear()
    print(json.dumps(line), flush=True)


def cpu_baseline_70b_layer():
    """The reference CPU path on ONE Llama-3-70B-shaped decoder layer (weights generated by the same
    counter-based streams, widened to F32 as SafeTensors.readFloat does), decode at batch 1 after a
    16-token context, scaled to 80 layers.  The tiny vocabulary of the probe model keeps the
    lm_head out of the measurement."""
    import numpy as np

    import oracle
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from llama_fixtures import oracle_model
    from scalatorch.models import LlamaConfig
    cfg = LlamaConfig(**dict(LLAMA70B, num_layers=1, vocab_size=256))
    model = oracle_model(cfg, seed=SEED)
    ctx = list(range(1, 17))
    cache = model.new_cache(1, 64)
    model.decode(cache, np.array([ctx]))
    t0 = time.perf_counter()
    n = 3
    for i in range(n):
        model.decode(cache, np.array([[i + 20]]))
    per_layer = (time.perf_counter() - t0) / n
    model.threads = 1  # one host thread, as numscala's ScalarF32Kernels
    t0 = time.perf_counter()
    model.decode(cache, np.array([[n + 20]]))
    per_layer_1 = time.perf_counter() - t0
    model.free_cache(cache)
    return {"value": round(1.0 / (per_layer * 80), 5), "unit": "tokens/s", "cores": oracle.max_threads(),
            "kind": "port", "sample": f"1 of 80 decoder layers, batch 1, {n} decode steps after a 16-token context: "
                                      f"{per_layer * 1000:.0f} ms/layer/token x 80 layers",
            "single_thread": {"value": round(1.0 / (per_layer_1 * 80), 5),
                              "ms_per_layer_token": round(per_layer_1 * 1e3, 1)},
            "host": host_cores()}


LM_HEAD_TRAFFIC_BYTES = 56_646_400
SMOL_WEIGHT_BYTES_PER_TOKEN = 268_959_744  # 30 x 3,538,944 x 2 + 49,152 x 576 x 2
# DRAM read + write of one decode step (all 153 kernels) in one ncu capture
# (profiles/decode_step_smollm2_launch_list.md)
SMOL_STEP_TRAFFIC_BYTES = 279_862_272


def decode_step_roofline(decode_tok_s, hbm_peak, peak_kind, lm_head):
    """The SmolLM2 line's roofline in the benchmark's own unit: weight bytes per decode token x
    decode tokens/s (CUDA events around the decode phase of the timed steps) against the measured
    HBM copy bandwidth.  The step is a graph of ~150 short kernels and is latency-bound; the
    largest single kernel (the lm_head GEMV, timed alone) is attached for the kernel-level view."""
    achieved = SMOL_WEIGHT_BYTES_PER_TOKEN * decode_tok_s / 1e9
    return {"kernel": "decode step (graph of per-layer GEMV / attention kernels, 153 launches per token)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes": SMOL_WEIGHT_BYTES_PER_TOKEN, "units": "weight bytes per decode token",
            "traffic": SMOL_STEP_TRAFFIC_BYTES, "traffic_unit": "B per decode token", "lm_head_gemv": lm_head}


def roofline_lm_head(session, cfg, hbm_peak, peak_kind):
    """The lm_head GEMV (49152 x 576 BF16, M = 1; the largest per-token kernel) timed alone with
    CUDA events on the session stream, L2 flushed (256 MB write) before every launch."""
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
            # dram__bytes_read.sum + dram__bytes_write.sum per launch of this kernel, one ncu capture
            # (profiles/gemv_kernel_smollm2_lm_head_m1.md)
            "traffic": LM_HEAD_TRAFFIC_BYTES, "traffic_unit": "B"}


def reference_arm(args, world, rank):
    """The reference's CPU path (oracle restatement; the Scala/JVM reference cannot run here) on all host
    threads, same metric and config; bounded sample per step.  Rank 0 alone runs under torchrun."""
    if rank != 0:
        return
    import oracle
    samples = []
    unit = "tokens/s"
    if args.workload == "single":
        for i in range(max(args.warmup, 0) + args.steps):
            r = cpu_single_linear(seconds=2.0)
            if i >= args.warmup:
                samples.append(r)
        metric = "single-Linear GB/s (x F32 [16,576] . W BF16 [1536,576]^T, L2 flushed before each call)"
        config = {"workload": "single Linear", "M": SINGLE_M, "N": SINGLE_N, "K": SINGLE_K}
        scaling, unit = "weak", "GB/s"
    elif args.workload in ("linear", "prefill"):
        prefill = args.workload == "prefill"
        ms = tuple(int(v) for v in args.ms.split(",")) if args.ms else ((2048, 8192) if prefill else (1, 4, 16, 32))
        names = [n for n in LLAMA8B_SHAPES if not args.shapes or n in args.shapes.split(",")]
        for i in range(max(args.warmup, 0) + args.steps):
            r = cpu_linear_shapes([(LLAMA8B_SHAPES[n] + (n,)) for n in names], min(ms), prefill, seconds=0.5)
            if i >= args.warmup:
                samples.append(r)
        metric = ("prefill GEMM TFLOP/s (Llama-3-8B projections, BF16 weights, activations rounded to BF16)"
                  if prefill else f"decode GEMV GB/s at M={min(ms)} (Llama-3-8B projections, BF16 weights, FP32 "
                  "activations)")
        config = {"workload": f"llama3-8b {args.workload} sweep", "M": min(ms), "shapes": names}
        scaling, unit = "weak", samples[0]["unit"]
    elif args.workload == "llama70b":
        for i in range(max(args.warmup, 0) + args.steps):
            r = cpu_baseline_70b_layer()
            if i >= args.warmup:
                samples.append(r)
        metric = "greedy decode tokens/s (Llama-3-70B-shaped, BF16 weights, tensor parallel)"
        config = {"workload": "llama3-70b-shaped greedy decode", "batch": args.batch, "prompt": args.prompt,
                  "new_tokens": args.new}
        scaling = "strong"
    else:
        model = None
        for i in range(max(args.warmup, 0) + args.steps):
            r, model = cpu_baseline_smol(seconds_budget=10.0, model=model, with_model=True)
            if i >= args.warmup:
                samples.append(r)
        metric = "greedy decode tokens/s (SmolLM2-135M-shaped, BF16 weights, batch 1, 128-token prompt + 128 new)"
        config = {"workload": "smollm2-135m-shaped greedy decode", "batch": 1, "prompt": PROMPT, "new_tokens": NEW}
        scaling = "weak"
    v = sum(s["value"] for s in samples) / len(samples)
    line = {"impl": "reference", "metric": metric,
            "value": round(v, 5), "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(v, 5), "unit": unit, "cores": oracle.max_threads(), "kind": "port",
                             "sample": samples[-1]["sample"]},
            "e2e": {"value": round(v, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
