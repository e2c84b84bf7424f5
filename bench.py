"""Benchmark: the BF16-weight Linear hot path of scala-torch's Llama runtime, through libstb200.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload, at every N (1, 2, 4, 8 GPUs of one box; one process per GPU under torchrun):
Llama-3-70B-shaped greedy decode, tensor parallel over the N GPUs (Megatron column / row / vocabulary
split; the row-split projections of decode steps exchange their partial sums over NVLink peer stores,
prompt chunks use one NCCL allreduce per row-split projection).  Random-init BF16 weights ~N(0,0.02)
generated on the device, RMSNorm weights 1, batch 8, 512-token prompts of ids uniform in [0,128256),
32 greedy tokens per row, KV cache resident in HBM.  One step = one generate call (prefill + decode).
Metric: decode tokens/s -- the 31 tokens per row that follow the one the prefill picks, all rows,
over the decode phase's CUDA-event time, max over ranks.  The job is fixed, so scaling is "strong".
`e2e` is whole generate calls through the C ABI (stb_llama_generate) with host prompt and id
buffers, wall clock.  `parity`: every rank's greedy ids agree (`ranks_agree`); how many leading ids
of each row equal the recorded single-GPU ids (`tp1_prefix_match_per_row`, `tp_ids_match` when all
do); and `tp_small`: a small 8-head model generated with the same tensor-parallel runtime at this N,
id for id against the CPU oracle (a mismatch makes the run exit non-zero).

At N = 1 the line also carries the other BASELINE configurations, measured in the same run (`sweeps`):
  smollm2  SmolLM2-135M-shaped, batch 1, 128-token prompt + 128 greedy tokens, with parity against the
           CPU oracle on the same seed (ids identical, logits after the prompt within 1e-5 (1+|e|));
           a mismatch makes the run exit non-zero
  single   the single Linear x F32 [16,576] . W BF16 [1536,576]^T
  decode   Llama-3-8B projections at M = 1, 4, 16, 32 (GB/s and fraction of measured HBM)
  prefill  Llama-3-8B projections at M = 2048 and 8192 (TFLOP/s and fraction of measured dense BF16)
Every fraction is computed at run time against MEASURED_PEAKS.json.

Output: one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "scala-torch_b200"))
sys.path.insert(0, ROOT)

SEED = 2024
SMOL = dict(vocab_size=49152, hidden_size=576, intermediate_size=1536, num_layers=30, num_attention_heads=9,
            num_key_value_heads=3, max_positions=2048, tie_word_embeddings=True, rope_theta=10000.0,
            rms_norm_eps=1e-6, eos_token_ids=())
SMOL_PROMPT, SMOL_NEW = 128, 128
SMOL_WEIGHT_BYTES_PER_TOKEN = 268_959_744  # 30 x 3,538,944 x 2 + 49,152 x 576 x 2
LLAMA70B = dict(vocab_size=128256, hidden_size=8192, intermediate_size=28672, num_layers=80,
                num_attention_heads=64, num_key_value_heads=8, max_positions=8192, tie_word_embeddings=False,
                rope_theta=500000.0, rms_norm_eps=1e-5, eos_token_ids=())
LLAMA8B_SHAPES = {"q": (4096, 4096), "k": (1024, 4096), "v": (1024, 4096), "o": (4096, 4096),
                  "gate": (14336, 4096), "up": (14336, 4096), "down": (4096, 14336), "lm_head": (128256, 4096)}
SINGLE_M, SINGLE_N, SINGLE_K = 16, 1536, 576
SINGLE_BYTES = SINGLE_N * SINGLE_K * 2 + SINGLE_M * SINGLE_K * 4 + SINGLE_M * SINGLE_N * 4  # 1,904,640 B

# The greedy ids (batch rows x new tokens) of the default workload on one GPU, seed 2024, recorded from
# `python bench.py` on a B200 (TP1); keyed by batch/prompt/new/layers.  The tensor-parallel runs report
# how many leading ids of each row they reproduce: on an 80-layer random-weight model the argmax over
# 128,256 near-tied logits can flip under the Float32 reassociation of a row-split sum, after which the
# sequences diverge.  The exact check at every N is `parity.tp_small` (ids against the CPU oracle).
TP1_IDS = {"8/512/32/80": [
    [89289, 122223, 57117, 84874, 118673, 75253, 107876, 30747, 29566, 71866, 54375, 89189, 37853, 21649, 73888, 23536, 121691, 89094, 29020, 3133, 18731, 22227, 104517, 28954, 9324, 57596, 84645, 105391, 125094, 97141, 60628, 23650],
    [118140, 102482, 117568, 110555, 101663, 2358, 118303, 109816, 124562, 102501, 112788, 16848, 18777, 46650, 40017, 8232, 109038, 6153, 61757, 43578, 8334, 82436, 110740, 85112, 112328, 105851, 114037, 77759, 34152, 97490, 42193, 87570],
    [104271, 236, 20488, 1499, 70293, 38267, 69268, 73015, 32637, 82579, 106803, 28214, 95798, 49450, 70693, 24705, 95016, 99018, 32255, 30057, 64208, 77279, 63674, 103519, 20146, 126965, 26746, 28320, 31865, 29761, 58455, 79292],
    [108529, 86287, 122692, 128030, 95374, 82016, 97715, 12170, 93104, 56973, 72629, 7061, 17348, 41548, 56687, 100415, 113228, 89077, 68058, 49080, 79181, 52486, 82643, 22568, 20011, 35784, 100791, 83208, 88724, 72817, 59760, 108916],
    [107238, 127209, 107064, 123617, 98148, 117116, 3661, 109219, 48042, 117645, 40355, 33644, 57150, 46225, 67544, 92541, 41344, 42441, 37728, 74953, 32725, 66692, 32783, 34587, 82604, 72114, 122215, 24193, 105889, 78118, 46280, 102713],
    [35970, 96088, 114821, 88599, 33238, 61588, 32914, 126558, 42798, 95006, 41477, 101455, 45135, 59187, 13370, 77939, 81696, 82121, 88417, 88827, 61297, 91242, 85456, 82660, 95758, 88201, 107377, 20348, 62777, 90903, 40787, 93173],
    [58516, 28655, 113392, 68354, 66956, 127783, 24561, 4985, 100096, 119608, 66697, 97699, 54441, 101205, 31142, 34658, 60427, 84129, 8379, 37124, 44213, 23165, 88, 92379, 121439, 55649, 110081, 110210, 118406, 63133, 82297, 24909],
    [99947, 45951, 112512, 109489, 91634, 2425, 122818, 111101, 46513, 63257, 3381, 60326, 125064, 89171, 9448, 100665, 89718, 11610, 68435, 87116, 109200, 98680, 88122, 120993, 106525, 122549, 124297, 15406, 123923, 122750, 16513, 49903]]}
# A small model every tensor-parallel size up to 8 divides (8 heads, 8 KV heads), generated with the
# same tensor-parallel runtime at every N and compared id for id with the CPU oracle.
TP_SMALL = dict(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_layers=2, num_attention_heads=8,
                num_key_value_heads=8, max_positions=64, tie_word_embeddings=False, eos_token_ids=())

# DRAM read + write bytes of one gemm_skinny_kernel launch on the dominant decode shape (70B gate/up
# shard, M = 8, TP1: 57344 x 8192 BF16 = 939.5 MB of weights): dram__bytes_read.sum 942,707,712 +
# dram__bytes_write.sum 6,144,512 from one ncu capture (--set full, --clock-control none) of
# `bench.py --workload kernel --steps 2 --warmup 0` on a B200 with the current kernel (two CTAs per SM).
# Keyed by the tensor-parallel size (the other sizes' shard shapes were not captured).
SKINNY_GATE_UP_TRAFFIC = {1: 948_852_224}


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


def host_cores() -> dict:
    """Host CPUs visible to this process (nproc) and in its affinity mask."""
    try:
        affinity = len(os.sched_getaffinity(0))
    except AttributeError:
        affinity = os.cpu_count()
    return {"nproc": os.cpu_count(), "affinity": affinity}


def median(v):
    v = sorted(v)
    return v[len(v) // 2]


# ---------------------------------------------------------------- workload descriptions (both arms)

def describe(args, world: int) -> tuple:
    """(metric, unit, scaling, config) of a workload: the same dict in the device and the reference arm."""
    w = args.workload
    if w == "llama70b":
        layers = args.layers or LLAMA70B["num_layers"]
        return ("greedy decode tokens/s (Llama-3-70B-shaped, BF16 weights, tensor parallel; batch "
                f"{args.batch}, {args.prompt}-token prompts + {args.new} new)", "tokens/s", "strong",
                {"workload": "llama3-70b-shaped greedy decode", "batch": args.batch, "prompt": args.prompt,
                 "new_tokens": args.new, "layers": layers, "hidden": 8192, "vocab": 128256,
                 "parallelism": f"tp{world}", "l2": "inputs larger than L2: 141 GB of weights / TP streamed per token"})
    if w == "smollm2":
        return ("greedy decode tokens/s (SmolLM2-135M-shaped, BF16 weights, batch 1, 128-token prompt + 128 new)",
                "tokens/s", "weak",
                {"workload": "smollm2-135m-shaped greedy decode", "batch": 1, "prompt": SMOL_PROMPT,
                 "new_tokens": SMOL_NEW, "layers": 30, "hidden": 576, "vocab": 49152,
                 "parallelism": f"replicas x{world}",
                 "l2": "inputs larger than L2: 269 MB of weights streamed per token vs 126 MB L2"})
    if w == "single":
        return ("single-Linear GB/s (x F32 [16,576] . W BF16 [1536,576]^T, L2 flushed before each call)", "GB/s",
                "weak", {"workload": "single Linear", "M": SINGLE_M, "N": SINGLE_N, "K": SINGLE_K,
                         "l2": "flushed before every call (256 MB write, then 256 MB read of another buffer)"})
    prefill = w == "prefill"
    ms = sweep_ms(args)
    names = sweep_names(args)
    wname = args.dtype.upper()
    if prefill:
        metric = f"prefill GEMM TFLOP/s (Llama-3-8B projections, {wname} weights, activations rounded to {wname})"
    else:
        metric = f"decode GEMV GB/s at M={min(ms)} (Llama-3-8B projections, {wname} weights, FP32 activations)"
    return (metric, "TFLOP/s" if prefill else "GB/s", "weak",
            {"workload": f"llama3-8b {w} sweep", "M": list(ms), "shapes": names,
             "l2": "flushed before every launch (256 MB write, then 256 MB read of another buffer)"})


def sweep_ms(args):
    if args.ms:
        return tuple(int(v) for v in args.ms.split(","))
    return (2048, 8192) if args.workload == "prefill" else (1, 4, 16, 32)


def sweep_names(args):
    return [n for n in LLAMA8B_SHAPES if not args.shapes or n in args.shapes.split(",")]


# ---------------------------------------------------------------- device helpers

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

    def generated(self):
        """(batch, new) int64 copy of the ids the last call generated."""
        return self.out.reshape(self.batch, self.plen + self.new)[:, self.plen:].copy()

    def close(self):
        self.ffm.call("stb_host_free", self.hp)
        self.ffm.call("stb_host_free", self.ho)


def ids_digest(ids) -> str:
    import numpy as np
    return hashlib.sha256(np.ascontiguousarray(ids, np.int64).tobytes()).hexdigest()[:16]


class L2Flush:
    """Evicts the timed kernel's data from the 126 MB L2 before each call: a 256 MB write (the timing
    rule), then a 256 MB read of a second buffer, so the write's dirty lines are written back before
    the timed kernel starts instead of during it (they would add up to 126 MB of DRAM writes that
    are not the kernel's own)."""

    def __init__(self):
        import torch
        self.write = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.read = torch.ones(64 << 20, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.write.zero_()
        self.read.sum()


def timed_linear(session, fn, x_addr, w_addr, wdt, y_addr, m, n, k, reps, warm, flush):
    """Each call alone between CUDA events on the session stream, L2 flushed (L2Flush, on the same
    stream) before every call; returns the median seconds of the `reps` calls after `warm`."""
    import torch
    from scalatorch import ffm
    stream = torch.cuda.ExternalStream(session.stream)
    times = []
    for it in range(warm + reps):
        with torch.cuda.stream(stream):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ffm.call(fn, session.handle, x_addr, w_addr, wdt, 0, y_addr, m, n, k)
        e1.record(stream)
        e1.synchronize()
        if it >= warm:
            times.append(e0.elapsed_time(e1) / 1000.0)
    return median(times)


def device_weight(session, n, k, dtype, seed, stream, std=0.02):
    """A resident (out,in) half weight of the device generator (torch owns the memory)."""
    import torch
    from scalatorch import ffm
    tdt = torch.float16 if dtype == ffm.STB_F16 else torch.bfloat16
    w = torch.empty(n * k, dtype=tdt, device="cuda")
    wt = ffm.DeviceTensor(session, w.data_ptr(), (k, n), dtype, n * k * 2, transposed_weight=True, owner=False)
    session.fill_normal(wt, seed, stream, std)
    return w


def linear_roofline(session, name, m, n, k, hbm_peak, peak_kind, reps=10, warm=3):
    """One projection shape timed alone (stb_linear: the decode family; for M >= 2 the skinny
    tensor-core form = prologue + gemm_skinny_kernel + fixup, three PDL-chained launches)."""
    import torch
    from scalatorch import ffm
    flush = L2Flush()
    w = device_weight(session, n, k, ffm.STB_BF16, SEED, 900)
    x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(m))
    y = torch.empty(m, n, device="cuda")
    session.sync()
    torch.cuda.synchronize()
    t = timed_linear(session, "stb_linear", x.data_ptr(), w.data_ptr(), ffm.STB_BF16, y.data_ptr(), m, n, k, reps,
                     warm, flush)
    algo = n * k * 2 + m * k * 4 + m * n * 4
    del w, x, y, flush
    torch.cuda.empty_cache()
    return {"kernel": name, "bound": "hbm", "achieved": round(algo / t / 1e9, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(algo / t / 1e9 / hbm_peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes": algo, "launch_us": round(t * 1e6, 2), "M": m, "N": n, "K": k}


# ---------------------------------------------------------------- the default workload

def run_llama70b(args, world, rank, local):
    import numpy as np
    import torch
    import torch.distributed as dist
    from scalatorch import ffm
    from scalatorch.models import BackendLlama, LlamaConfig

    torch.cuda.set_device(local)
    hbm_peak, tc_peak, peak_kind = peaks()
    sweeps, failures = {}, []
    if world == 1 and not args.no_sweeps:
        sweeps, failures = run_sweeps(args, local, hbm_peak, tc_peak, peak_kind)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    metric, unit, scaling, config = describe(args, world)
    cfg = LlamaConfig(**(dict(LLAMA70B, num_layers=args.layers) if args.layers else LLAMA70B))
    batch, plen, new = args.batch, args.prompt, args.new
    session = ffm.B200Session(local, 178 << 30)
    if world > 1:  # one communicator for the tensor-parallel group
        uid = [ffm.B200Session.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        session.init_tp(world, rank, uid[0])
    model = BackendLlama.prepare_random(session, cfg, seed=SEED, tp_rank=rank, tp_size=world)
    prompts = np.random.default_rng(SEED).integers(0, cfg.vocab_size, (batch, plen)).astype(np.int64)
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
    gen_ids = step.generated()
    digest = ids_digest(gen_ids)
    pre_s, dec_s = sum(pre_ms) / 1000.0, sum(dec_ms) / 1000.0
    agree = True
    if world > 1:
        pre_s, dec_s, wall = max_over_ranks([pre_s, dec_s, wall], device="cuda")
        h = torch.tensor([int(digest, 16) >> 1], dtype=torch.int64, device="cuda")
        lo, hi = h.clone(), h.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        agree = int(lo.item()) == int(hi.item())
    # the dominant kernel of the decode step: the gate/up projection (55 % of the weight bytes), this
    # rank's shard at M = batch, timed alone
    gu_n = 2 * cfg.intermediate_size // world
    roof = linear_roofline(session, f"stb_linear gate/up shard (prologue + gemm_skinny_kernel + fixup), "
                           f"{gu_n}x{cfg.hidden_size} BF16, M={batch}", batch, gu_n, cfg.hidden_size, hbm_peak,
                           peak_kind)
    roof["traffic"] = SKINNY_GATE_UP_TRAFFIC.get(world) if batch == 8 else None
    per_tok = dec_s / args.steps / max(new - 1, 1)
    step_gbs = model.weight_bytes / per_tok / 1e9
    roof["step"] = {"what": "decode step, all kernels: this rank's weight bytes per token / decode time per token",
                    "achieved": round(step_gbs, 1), "frac": round(step_gbs / hbm_peak, 4),
                    "weight_bytes_per_rank": model.weight_bytes}
    small = tp_small_parity(session, world, rank)
    if world > 1:
        dist.barrier()

    value = batch * max(new - 1, 1) * args.steps / dec_s
    e2e = batch * new * args.steps / wall
    key = f"{batch}/{plen}/{new}/{cfg.num_layers}"
    tp1 = TP1_IDS.get(key)
    expected = ids_digest(tp1) if tp1 else None
    prefix = None
    if tp1:
        prefix = [next((i for i, (a, b) in enumerate(zip(row, ref)) if int(a) != int(b)), len(ref))
                  for row, ref in zip(gen_ids.tolist(), tp1)]
    line = {
        "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round((pre_s + dec_s) * 1000 / args.steps, 3),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16-weights/f32-compute",
        "data": "synthetic (device counter-RNG weights, random prompt ids)", "config": config,
        "e2e": {"value": round(e2e, 3), "unit": unit, "h2d_bytes_per_step": step.h2d, "d2h_bytes_per_step": step.d2h,
                "what": "whole generate calls (prefill + decode) through stb_llama_generate, host buffers, wall clock"},
        "gpu_launches": int(launches), "roofline": roof, "clocks": clocks.summary(),
        "detail": {"prefill_ms": round(pre_s * 1000 / args.steps, 3), "decode_ms": round(dec_s * 1000 / args.steps, 3),
                   "decode_ms_per_token": round(per_tok * 1000, 3), "weight_bytes_per_rank": model.weight_bytes,
                   "launches_per_step": round(launches / args.steps, 1)},
        "parity": {"ids_digest": digest, "ranks_agree": agree, "tp1_digest": expected,
                   "tp_ids_match": (agree and digest == expected) if expected else None,
                   "tp1_prefix_match_per_row": prefix, "tp_small": small,
                   "ids": gen_ids.tolist()},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline_70b_layer(batch)
        except Exception as e:  # reported, never silently replaced
            line["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if sweeps:
        line["sweeps"] = sweeps
        line["parity"]["smollm2"] = sweeps.get("smollm2", {}).get("parity")
    step.close()
    model.close()
    session.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if small is not None and not small["ids_identical_to_oracle"]:
        failures.append(f"tensor-parallel small-model ids differ from the oracle: {small}")
    if failures:
        print("parity failures: " + "; ".join(failures), file=sys.stderr, flush=True)
        return 1
    return 0


def tp_small_parity(session, world, rank):
    """TP_SMALL generated with the tensor-parallel runtime over the current group (every rank takes
    part) and, on rank 0, compared id for id with the CPU oracle on the same seed and prompts (2 rows x
    12 prompt tokens, 12 greedy tokens: Float32 activations, so the decode tolerance applies)."""
    import numpy as np
    from scalatorch.models import BackendLlama, LlamaConfig
    cfg = LlamaConfig(**TP_SMALL)
    prompts = np.random.default_rng(11).integers(0, cfg.vocab_size, (2, 12))
    with BackendLlama.prepare_random(session, cfg, seed=SEED, tp_rank=rank, tp_size=world) as m:
        got = m.generate_ids(prompts, 12)
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from llama_fixtures import oracle_model
    ref = oracle_model(cfg, seed=SEED)
    want = [ref.generate(prompts[b].tolist(), 12) for b in range(2)]
    return {"model": "2 layers, hidden 512, 8 heads / 8 KV heads, vocab 1024, batch 2, 12 + 12 tokens",
            "tp": world, "ids_identical_to_oracle": [list(map(int, r)) for r in got] == want}


# ---------------------------------------------------------------- the other configurations

def run_sweeps(args, local, hbm_peak, tc_peak, peak_kind):
    """configs 1-4 of BASELINE, each time-bounded, before the 70B model takes the device."""
    import torch
    out, failures = {}, []
    t0 = time.perf_counter()
    rec = smollm2_record(local, steps=5, warmup=3, hbm_peak=hbm_peak, peak_kind=peak_kind, parity=True,
                         cpu=not args.no_cpu_baseline)
    if not rec["parity"]["ok"]:
        failures.append(f"smollm2 parity: {rec['parity']}")
    out["smollm2"] = rec
    out["single"] = single_record(local, steps=3, warmup=2, hbm_peak=hbm_peak, peak_kind=peak_kind,
                                  cpu=not args.no_cpu_baseline)
    names = list(LLAMA8B_SHAPES)
    out["decode"] = linear_sweep_record(local, False, (1, 4, 16, 32), names, "bf16", 5, 2, hbm_peak, tc_peak,
                                        peak_kind, cpu=not args.no_cpu_baseline)
    out["prefill"] = linear_sweep_record(local, True, (2048, 8192), names, "bf16", 5, 2, hbm_peak, tc_peak,
                                         peak_kind, cpu=not args.no_cpu_baseline)
    out["prefill_f16"] = linear_sweep_record(local, True, (2048,), names, "f16", 3, 1, hbm_peak, tc_peak,
                                             peak_kind, cpu=False)
    out["seconds"] = round(time.perf_counter() - t0, 1)
    torch.cuda.empty_cache()
    return out, failures


def smollm2_record(local, steps, warmup, hbm_peak, peak_kind, parity=True, cpu=True):
    """SmolLM2-shaped 128 + 128 greedy generation: tokens/s, decode tokens/s, decode-step HBM fraction,
    and (parity) the same seed and prompt on the CPU oracle: ids identical and the logits after the
    prompt within 1e-5 (1 + |e|)."""
    import numpy as np
    import torch
    from scalatorch import ffm
    from scalatorch.models import BackendLlama, LlamaConfig
    torch.cuda.set_device(local)
    cfg = LlamaConfig(**SMOL)
    session = ffm.B200Session(local, 8 << 30)
    model = BackendLlama.prepare_random(session, cfg, seed=SEED)
    prompts = np.random.default_rng(SEED).integers(0, cfg.vocab_size, (1, SMOL_PROMPT)).astype(np.int64)
    step = Generator(model, prompts, SMOL_NEW)
    for _ in range(warmup):
        step()
    session.sync()
    l0 = session.launches
    pre, dec = [], []
    t0 = time.perf_counter()
    for _ in range(steps):
        p, q = step()
        pre.append(p)
        dec.append(q)
    session.sync()
    wall = time.perf_counter() - t0
    launches = session.launches - l0
    ids = step.generated()[0]
    logits = None
    if parity:
        cache = model.new_cache(1, SMOL_PROMPT + 1)
        got, _ = cache.decode(prompts)
        logits = got[0, -1].astype(np.float64)
        cache.close()
    step.close()
    model.close()
    session.close()
    pre_s, dec_s = sum(pre) / 1000, sum(dec) / 1000
    dec_tok_s = (SMOL_NEW - 1) * steps / dec_s
    achieved = SMOL_WEIGHT_BYTES_PER_TOKEN * dec_tok_s / 1e9
    rec = {"tokens_s": round(SMOL_NEW * steps / (pre_s + dec_s), 2), "e2e_tokens_s": round(SMOL_NEW * steps / wall, 2),
           "decode_tokens_s": round(dec_tok_s, 1), "prefill_ms": round(pre_s * 1000 / steps, 3),
           "decode_ms_per_token": round(dec_s * 1000 / steps / (SMOL_NEW - 1), 4),
           "launches_per_step": round(launches / steps, 1),
           "decode_step_roofline": {"achieved": round(achieved, 1), "unit": "GB/s", "peak": hbm_peak,
                                    "frac": round(achieved / hbm_peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                                    "algorithmic_bytes": SMOL_WEIGHT_BYTES_PER_TOKEN,
                                    "units": "weight bytes per decode token"},
           "steps": steps, "warmup": warmup}
    if parity:
        import oracle
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from llama_fixtures import oracle_model
        ref = oracle_model(cfg, seed=SEED)
        t0 = time.perf_counter()
        want = ref.generate(prompts[0], SMOL_NEW)[SMOL_PROMPT:]
        dt = time.perf_counter() - t0
        oc = ref.new_cache(1, SMOL_PROMPT + 1)
        e = ref.decode(oc, prompts)[0, -1].astype(np.float64)
        ref.free_cache(oc)
        ratio = float(np.max(np.abs(logits - e) / (1e-5 * (1 + np.abs(e)))))
        same = [int(v) for v in ids] == [int(v) for v in want]
        first_diff = next((i for i, (a, b) in enumerate(zip(ids, want)) if int(a) != int(b)), -1)
        rec["parity"] = {"ids_identical": same, "first_differing_id": first_diff, "ids": len(want),
                         "max_logit_err": float(np.max(np.abs(logits - e))), "worst_ratio_to_1e-5(1+|e|)": round(ratio, 4),
                         "ok": bool(same and ratio <= 1.0)}
        if cpu:
            rec["cpu_baseline"] = {"value": round(SMOL_NEW / dt, 3), "unit": "tokens/s", "cores": oracle.max_threads(),
                                   "kind": "port", "sample": f"full {SMOL_PROMPT} + {SMOL_NEW} generation on the oracle "
                                                             f"(the parity run), {dt:.2f} s", "host": host_cores()}
    return rec


def single_record(local, steps, warmup, hbm_peak, peak_kind, cpu=True, calls=100):
    """The single-Linear configuration (x F32 [16,576] ~N(0,1), W BF16 [1536,576] ~N(0,0.02), no bias)
    through stb_linear.  Cold: an L2 flush (L2Flush) before every call and CUDA events around each call
    alone (the reported value, against HBM); warm: `calls` back-to-back calls between one event pair
    (the 1.8 MB weight stays in L2).  e2e: stb_linear_host with host x and y, wall clock per call."""
    import numpy as np
    import torch
    from scalatorch import ffm
    torch.cuda.set_device(local)
    s = ffm.B200Session(local, 4 << 30)
    stream = torch.cuda.ExternalStream(s.stream)
    flush = L2Flush()
    M, N, K = SINGLE_M, SINGLE_N, SINGLE_K
    w = device_weight(s, N, K, ffm.STB_BF16, 1, 1)
    hx = np.random.default_rng(1).standard_normal((M, K)).astype(np.float32)
    hy = np.empty((M, N), np.float32)
    x = torch.from_numpy(hx).cuda()
    y = torch.empty(M, N, device="cuda")
    s.sync()
    torch.cuda.synchronize()
    cold, warm, e2e = [], [], []
    l0 = s.launches
    for st in range(warmup + steps):
        t = [timed_linear(s, "stb_linear", x.data_ptr(), w.data_ptr(), ffm.STB_BF16, y.data_ptr(), M, N, K, 1, 0,
                          flush) for _ in range(calls)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(calls):
            ffm.call("stb_linear", s.handle, x.data_ptr(), w.data_ptr(), ffm.STB_BF16, 0, y.data_ptr(), M, N, K)
        e1.record(stream)
        e1.synchronize()
        if st >= warmup:
            cold.extend(t)
            warm.append(e0.elapsed_time(e1) / 1000.0 / calls)
    launches = s.launches - l0
    for st in range(warmup + steps):
        for _ in range(calls):
            t0 = time.perf_counter()
            ffm.call("stb_linear_host", s.handle, hx.ctypes.data, w.data_ptr(), ffm.STB_BF16, 0, hy.ctypes.data, M, N, K)
            if st >= warmup:
                e2e.append(time.perf_counter() - t0)
    s.close()
    del w, x, y, flush
    torch.cuda.empty_cache()
    t_cold, t_warm, t_e2e = median(cold), median(warm), median(e2e)
    rec = {"GB_s": round(SINGLE_BYTES / t_cold / 1e9, 2), "hbm_frac": round(SINGLE_BYTES / t_cold / 1e9 / hbm_peak, 4),
           "peak_source": f"{peak_kind} hbm_gbs", "cold_us": round(t_cold * 1e6, 2), "warm_us": round(t_warm * 1e6, 2),
           "warm_GB_s": round(SINGLE_BYTES / t_warm / 1e9, 1), "e2e_us": round(t_e2e * 1e6, 2),
           "e2e_GB_s": round(SINGLE_BYTES / t_e2e / 1e9, 3), "algorithmic_bytes": SINGLE_BYTES,
           "launches_per_call": round(launches / ((warmup + steps) * 2 * calls), 2), "calls_per_step": calls}
    if cpu:
        rec["cpu_baseline"] = cpu_single_linear(seconds=2.0)
    return rec


def linear_sweep_record(local, prefill, ms, names, dtype, steps, warmup, hbm_peak, tc_peak, peak_kind, cpu=True):
    """Llama-3-8B projection shapes: stb_linear (decode family, FP32 activations) or stb_linear_prefill
    (tcgen05 GEMM, activations rounded to the weight type), each launch timed alone with CUDA events
    on the session stream after an L2 flush (L2Flush); the median of the timed launches per shape."""
    import torch
    from scalatorch import ffm
    torch.cuda.set_device(local)
    s = ffm.B200Session(local, 100 << 30)
    flush = L2Flush()
    wdt = ffm.STB_F16 if dtype == "f16" else ffm.STB_BF16
    fn = "stb_linear_prefill" if prefill else "stb_linear"
    results = []
    for si, name in enumerate(names):
        n, k = LLAMA8B_SHAPES[name]
        w = device_weight(s, n, k, wdt, SEED, 100 + si)
        for m in ms:
            x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(m))
            y = torch.empty(m, n, device="cuda")
            torch.cuda.synchronize()
            s.sync()
            t = timed_linear(s, fn, x.data_ptr(), w.data_ptr(), wdt, y.data_ptr(), m, n, k, steps, warmup, flush)
            algo = n * k * 2 + m * k * 4 + m * n * 4
            r = {"shape": name, "M": m, "N": n, "K": k, "us": round(t * 1e6, 2)}
            if prefill:
                r.update({"TFLOP_s": round(2 * m * n * k / t / 1e12, 1),
                          "tensor_frac": round(2 * m * n * k / t / 1e12 / tc_peak, 4)})
            else:
                r.update({"GB_s": round(algo / t / 1e9, 1), "hbm_frac": round(algo / t / 1e9 / hbm_peak, 4)})
            results.append(r)
            del x, y
        del w
        torch.cuda.empty_cache()
    s.close()
    del flush
    torch.cuda.empty_cache()
    rec = {"shapes": results, "dtype": dtype, "timing": f"median of {steps} launches after {warmup}, L2 flushed"}
    if prefill:
        flops = sum(2 * r["M"] * r["N"] * r["K"] for r in results)
        secs = sum(r["us"] for r in results) / 1e6
        rec.update({"TFLOP_s": round(flops / secs / 1e12, 1), "tensor_frac": round(flops / secs / 1e12 / tc_peak, 4),
                    "peak": tc_peak, "peak_source": f"{peak_kind} bf16_tflops (burst)",
                    "what": "total 2MNK of the sweep / total time"})
    else:
        for m in ms:
            sel = [r for r in results if r["M"] == m]
            byts = sum(r["N"] * r["K"] * 2 + m * r["K"] * 4 + m * r["N"] * 4 for r in sel)
            secs = sum(r["us"] for r in sel) / 1e6
            rec[f"M{m}"] = {"GB_s": round(byts / secs / 1e9, 1), "hbm_frac": round(byts / secs / 1e9 / hbm_peak, 4)}
        rec.update({"peak": hbm_peak, "peak_source": f"{peak_kind} hbm_gbs",
                    "what": "per M: total algorithmic bytes of the shapes / total time"})
    if cpu:
        rec["cpu_baseline"] = cpu_linear_shapes([(LLAMA8B_SHAPES[n] + (n,)) for n in names], min(ms), prefill,
                                                seconds=0.5)
    return rec


def run_smollm2(args, world, rank, local):
    """--workload smollm2: the SmolLM2-shaped generation as the line's own value (N independent
    replicas at N > 1), with the oracle parity check at N = 1."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    hbm_peak, _, peak_kind = peaks()
    metric, unit, scaling, config = describe(args, world)
    with Clocks(local) as clocks:
        clocks.mark()
        rec = smollm2_record(local, args.steps, max(args.warmup, 3), hbm_peak, peak_kind,
                             parity=world == 1, cpu=world == 1 and not args.no_cpu_baseline)
        clocks.mark()
    tok = rec["tokens_s"]
    if world > 1:
        tok = world * min(-max_over_ranks([-tok], device="cuda")[0], tok)
        dist.destroy_process_group()
    line = {"metric": metric, "value": tok, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(SMOL_NEW * 1000 / rec["tokens_s"], 3), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "bf16-weights/f32-compute",
            "data": "synthetic (device counter-RNG weights, random prompt ids)", "config": config,
            "e2e": {"value": rec["e2e_tokens_s"], "unit": unit, "h2d_bytes_per_step": SMOL_PROMPT * 8,
                    "d2h_bytes_per_step": SMOL_NEW * 8 + 32},
            "gpu_launches": int(rec["launches_per_step"] * args.steps),
            "roofline": dict(rec["decode_step_roofline"], kernel="decode step (all kernels)", bound="hbm",
                             traffic=None),
            "clocks": clocks.summary(), "detail": rec}
    if "cpu_baseline" in rec:
        line["cpu_baseline"] = rec["cpu_baseline"]
    if "parity" in rec:
        line["parity"] = rec["parity"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0 if rec.get("parity", {"ok": True})["ok"] else 1


def run_linear_line(args, local):
    """--workload linear / prefill / single: one configuration as the line's own value."""
    import torch
    torch.cuda.set_device(local)
    hbm_peak, tc_peak, peak_kind = peaks()
    metric, unit, scaling, config = describe(args, 1)
    with Clocks(local) as clocks:
        clocks.mark()
        if args.workload == "single":
            rec = single_record(local, args.steps, args.warmup, hbm_peak, peak_kind, cpu=not args.no_cpu_baseline)
        else:
            rec = linear_sweep_record(local, args.workload == "prefill", sweep_ms(args), sweep_names(args), args.dtype,
                                      args.steps, args.warmup, hbm_peak, tc_peak, peak_kind,
                                      cpu=not args.no_cpu_baseline)
        clocks.mark()
    if args.workload == "single":
        value = rec["GB_s"]
        roof = {"kernel": "stb_linear x[16,576] (one gemv_kernel launch)", "bound": "hbm", "achieved": value,
                "peak": hbm_peak, "unit": "GB/s", "frac": rec["hbm_frac"], "peak_source": f"{peak_kind} hbm_gbs",
                "algorithmic_bytes": SINGLE_BYTES, "traffic": None}
        e2e = {"value": rec["e2e_GB_s"], "unit": unit, "h2d_bytes_per_step": SINGLE_M * SINGLE_K * 4,
               "d2h_bytes_per_step": SINGLE_M * SINGLE_N * 4, "what": "stb_linear_host, median wall clock per call"}
    elif args.workload == "prefill":
        value = rec["TFLOP_s"]
        top = max(rec["shapes"], key=lambda r: r["us"])
        roof = {"kernel": f"gemm_tc2_kernel, CTA pairs ({top['shape']} M={top['M']})", "bound": "tensor",
                "achieved": top["TFLOP_s"], "peak": tc_peak, "unit": "TFLOP/s", "frac": top["tensor_frac"],
                "peak_source": f"{peak_kind} bf16_tflops (burst)", "traffic": None}
        e2e = None
    else:
        m1 = min(sweep_ms(args))
        value = rec[f"M{m1}"]["GB_s"]
        top = max([r for r in rec["shapes"] if r["M"] == m1], key=lambda r: r["us"])
        roof = {"kernel": f"stb_linear ({top['shape']} M={top['M']})", "bound": "hbm", "achieved": top["GB_s"],
                "peak": hbm_peak, "unit": "GB/s", "frac": top["hbm_frac"], "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": None}
        e2e = None
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": f"{args.dtype}-weights/f32-accumulate", "data": "synthetic (device counter-RNG weights)",
            "config": config, "roofline": roof, "clocks": clocks.summary(), "detail": rec}
    if e2e:
        line["e2e"] = e2e
    if "cpu_baseline" in rec:
        line["cpu_baseline"] = rec["cpu_baseline"]
    print(json.dumps(line), flush=True)
    return 0


def run_kernel(args, local):
    """--workload kernel: the headline's dominant kernel alone (70B gate/up shard of --gpus ranks at
    M = --batch), a few launches; the case the committed ncu capture covers."""
    import torch
    from scalatorch import ffm
    torch.cuda.set_device(local)
    hbm_peak, _, peak_kind = peaks()
    s = ffm.B200Session(local, 8 << 30)
    n = 2 * LLAMA70B["intermediate_size"] // args.gpus
    r = linear_roofline(s, "stb_linear gate/up shard", args.batch, n, LLAMA70B["hidden_size"], hbm_peak, peak_kind,
                        reps=args.steps, warm=args.warmup)
    s.close()
    print(json.dumps(r), flush=True)
    return 0


# ---------------------------------------------------------------- CPU baselines (the oracle port)

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


class Cpu70bLayer:
    """The reference CPU path on ONE Llama-3-70B-shaped decoder layer (weights from the same counter-based
    streams, widened to F32 as SafeTensors.readFloat does), decoding a batch of `batch` rows after a
    one-token context; the per-layer time is scaled to 80 layers.  A probe vocabulary of 256 keeps
    the lm_head (1.3 % of the weights) out of the sample; attention over a 512-key context costs
    0.5 % of a layer's multiply-adds at batch 8, so the short context does not flatter the CPU."""

    def __init__(self, batch: int):
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from llama_fixtures import oracle_model
        from scalatorch.models import LlamaConfig
        cfg = LlamaConfig(**dict(LLAMA70B, num_layers=1, vocab_size=256))
        self.model = oracle_model(cfg, seed=SEED)
        self.batch = batch
        self.cache = self.model.new_cache(batch, 4096)
        self.model.decode(self.cache, np.arange(1, batch + 1).reshape(batch, 1))
        self.pos = 1

    def step(self) -> float:
        """Seconds of one decode step of the layer (batch rows, one token each)."""
        import numpy as np
        if self.pos >= 4095:
            self.model.free_cache(self.cache)
            self.cache = self.model.new_cache(self.batch, 4096)
            self.model.decode(self.cache, np.arange(1, self.batch + 1).reshape(self.batch, 1))
            self.pos = 1
        t0 = time.perf_counter()
        self.model.decode(self.cache, np.full((self.batch, 1), 20 + self.pos % 200))
        self.pos += 1
        return time.perf_counter() - t0

    def close(self):
        self.model.free_cache(self.cache)


def cpu_baseline_70b_layer(batch: int, steps: int = 3):
    import oracle
    probe = Cpu70bLayer(batch)
    try:
        per_layer = median([probe.step() for _ in range(steps)])
        probe.model.threads = 1  # one host thread, as numscala's ScalarF32Kernels
        per_layer_1 = probe.step()
        probe.model.threads = oracle.max_threads()
    finally:
        probe.close()
    return {"value": round(batch / (per_layer * 80), 5), "unit": "tokens/s", "cores": oracle.max_threads(),
            "kind": "port", "sample": f"1 of 80 decoder layers, batch {batch}, median of {steps} decode steps after "
                                      f"a 1-token context: {per_layer * 1000:.0f} ms/layer/step x 80 layers",
            "single_thread": {"value": round(batch / (per_layer_1 * 80), 6),
                              "ms_per_layer_step": round(per_layer_1 * 1e3, 1)},
            "host": host_cores()}


# ---------------------------------------------------------------- reference arm

def reference_arm(args, world, rank):
    """The reference's CPU path (the oracle restatement; the Scala/JVM reference cannot run here) on all
    host threads, same metric, unit and config as the device arm; a bounded sample per step.  Rank 0
    alone runs under torchrun; the other ranks exit without work."""
    if rank != 0:
        return 0
    import oracle
    metric, unit, scaling, config = describe(args, world)
    samples = []
    if args.workload == "single":
        for i in range(max(args.warmup, 0) + args.steps):
            r = cpu_single_linear(seconds=2.0)
            if i >= args.warmup:
                samples.append(r)
    elif args.workload in ("linear", "prefill"):
        prefill = args.workload == "prefill"
        for i in range(max(args.warmup, 0) + args.steps):
            r = cpu_linear_shapes([(LLAMA8B_SHAPES[n] + (n,)) for n in sweep_names(args)], min(sweep_ms(args)),
                                  prefill, seconds=0.5)
            if i >= args.warmup:
                samples.append(r)
        unit = samples[0]["unit"]
    elif args.workload == "llama70b":
        probe = Cpu70bLayer(args.batch)
        try:
            for i in range(max(args.warmup, 0) + args.steps):
                per_layer = probe.step()
                if i >= args.warmup:
                    samples.append({"value": args.batch / (per_layer * 80),
                                    "sample": f"1 of 80 decoder layers, batch {args.batch}, one decode step per "
                                              f"bench step after a 1-token context ({per_layer * 1000:.0f} ms per "
                                              f"layer step) x 80 layers"})
        finally:
            probe.close()
    else:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        import numpy as np
        from llama_fixtures import oracle_model
        from scalatorch.models import LlamaConfig
        cfg = LlamaConfig(**SMOL)
        model = oracle_model(cfg, seed=SEED)
        prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, SMOL_PROMPT).tolist()
        for i in range(max(args.warmup, 0) + args.steps):
            t0 = time.perf_counter()
            out = model.generate(prompt, SMOL_NEW)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                samples.append({"value": (len(out) - SMOL_PROMPT) / dt,
                                "sample": f"full {SMOL_PROMPT}-token prompt + {SMOL_NEW} greedy tokens, {dt:.2f} s"})
    v = sum(s["value"] for s in samples) / len(samples)
    line = {"impl": "reference", "metric": metric,
            "value": round(v, 5), "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(v, 5), "unit": unit, "cores": oracle.max_threads(), "kind": "port",
                             "sample": samples[-1]["sample"]},
            "e2e": {"value": round(v, 5), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama70b",
                    choices=["llama70b", "smollm2", "linear", "prefill", "single", "kernel"],
                    help="llama70b (default): the tensor-parallel 70B-shaped decode with the other configurations "
                    "as sweeps at N = 1; smollm2 / single / linear / prefill: one configuration as the line's value; "
                    "kernel: the headline's dominant kernel alone (for profiling)")
    ap.add_argument("--shapes", default="", help="linear/prefill: comma list of shape names to run (default all)")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"],
                    help="linear/prefill: weight type (F16 prefill rounds the activations to F16)")
    ap.add_argument("--ms", default="", help="linear/prefill: comma list of token-row counts M (default 1,4,16,32 "
                    "for linear, 2048,8192 for prefill)")
    ap.add_argument("--batch", type=int, default=8, help="llama70b / kernel: decode batch (1, 8, 32)")
    ap.add_argument("--prompt", type=int, default=512, help="llama70b: prompt tokens")
    ap.add_argument("--new", type=int, default=32, help="llama70b: generated tokens per step")
    ap.add_argument("--layers", type=int, default=0, help="llama70b: fewer layers (small profiling cases only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweeps", action="store_true", help="llama70b: skip the other configurations at N = 1")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, world, rank)
    if args.workload == "llama70b":
        return run_llama70b(args, world, rank, local)
    if args.workload == "smollm2":
        return run_smollm2(args, world, rank, local)
    if args.workload == "kernel":
        return run_kernel(args, local)
    return run_linear_line(args, local)


if __name__ == "__main__":
    sys.exit(main())
