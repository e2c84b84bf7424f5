"""Generate tests/golden/reference_vectors.json from scala-torch's own tests and fixtures.

Run in a container where the scala-torch source tree is mounted (pass its root as argv[1]).
The reference's known-answer tests are Scala munit suites that cannot run without a JVM, so
this script does two things:

* it reads the binary fixture io/src/test/resources/safetensors/upstream-0.6.2.safetensors
  (written by the official Rust safetensors 0.6.2 serializer) and records its raw tensor bits;
* it records the known answers of the cited test lines and, for each, checks that the cited
  Scala source still contains the literal the answer was transcribed from, so a drift in the
  reference shows up as a failure here rather than as a silently stale fixture.

The output is small JSON; tests read only that file, never the reference tree.
"""
from __future__ import annotations

import json
import math
import os
import struct
import sys


def read_safetensors(path):
    raw = open(path, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        b, e = info["data_offsets"]
        out[name] = {"dtype": info["dtype"], "shape": info["shape"], "bytes": data[b:e]}
    return out, header.get("__metadata__", {})


def check_literal(root, rel, needle):
    text = open(os.path.join(root, rel), encoding="utf-8").read()
    if needle not in text:
        raise SystemExit(f"{rel} no longer contains {needle!r}; re-derive the golden vector")
    return rel


def f32bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def main(root):
    out = {"source": "scala-torch reference tests and fixtures", "cases": {}}
    cases = out["cases"]

    # --- binary fixture written by Rust safetensors 0.6.2
    fx = "io/src/test/resources/safetensors/upstream-0.6.2.safetensors"
    tensors, meta = read_safetensors(os.path.join(root, fx))
    u16 = lambda b: list(struct.unpack(f"<{len(b)//2}H", b))
    f32 = lambda b: list(struct.unpack(f"<{len(b)//4}f", b))
    cases["upstream_safetensors"] = {
        "cite": fx + "; nn/src/test/scala/scalatorch/nn/SafeWeightsSuite.scala:10-24",
        # the whole archive, so the header reader is checked against the Rust serializer's layout
        "archive_hex": open(os.path.join(root, fx), "rb").read().hex(),
        "tensors": {n: {"dtype": t["dtype"], "shape": t["shape"]} for n, t in sorted(tensors.items())},
        "metadata": meta,
        "weight": f32(tensors["weight"]["bytes"]), "weight_shape": tensors["weight"]["shape"],
        "bias": f32(tensors["bias"]["bytes"]),
        "half_bits": u16(tensors["half"]["bytes"]), "bfloat_bits": u16(tensors["bfloat"]["bytes"]),
        "input": [1.0, 2.0, 3.0], "expected": [24.0, 52.0],
    }
    check_literal(root, "nn/src/test/scala/scalatorch/nn/SafeWeightsSuite.scala", "Seq(24f, 52f)")

    # --- F16 / BF16 decode tables (SafeTensorsSuite.scala:36-53, 135-148)
    st = "io/src/test/scala/scalatorch/io/SafeTensorsSuite.scala"
    check_literal(root, st, "0x0000, 0x8000, 0x0001, 0x03ff, 0x0400, 0x3c00, 0xc000, 0x7bff, 0x7c00, 0xfc00, 0x7e01")
    check_literal(root, st, "0x3f80, 0xc000, 0x0001, 0x8000, 0x7f80, 0xff80, 0x7fc1")
    check_literal(root, st, "Array(0x3f80, 0xc000, 0x0001, 0x7f7f)")
    cases["f16_decode"] = {
        "cite": st + ":36-53",
        "bits": [0x0000, 0x8000, 0x0001, 0x03ff, 0x0400, 0x3c00, 0xc000, 0x7bff, 0x7c00, 0xfc00, 0x7e01],
        "expected_f32_bits": [f32bits(v) for v in
                              [0.0, -0.0, 2.0 ** -24, 1023 * 2.0 ** -24, 2.0 ** -14, 1.0, -2.0, 65504.0,
                               math.inf, -math.inf]] + ["nan"],
    }
    cases["bf16_decode"] = {
        "cite": st + ":36-53",
        "bits": [0x3f80, 0xc000, 0x0001, 0x8000, 0x7f80, 0xff80, 0x7fc1],
        "expected_f32_bits": [f32bits(v) for v in [1.0, -2.0, 2.0 ** -133, -0.0, math.inf, -math.inf]] + ["nan"],
    }
    cases["chunked_decode"] = {
        "cite": st + ":135-148",
        "count": 40000,
        "f16_words": [0x3c00, 0xc000, 0x0001, 0x7bff],
        "f16_expected": [1.0, -2.0, 2.0 ** -24, 65504.0],
        "bf16_words": [0x3f80, 0xc000, 0x0001, 0x7f7f],
        "bf16_expected": [1.0, -2.0, 2.0 ** -133, (2.0 - 1.0 / 128) * 2.0 ** 127],
    }

    # --- GEMM known answers
    bs = "cpu/src/test/scala/scalatorch/cpu/BackendSuite.scala"
    check_literal(root, bs, "Seq(58f, 64f, 139f, 154f)")
    cases["gemm_small"] = {
        "cite": bs + ":22-43; ffm/src/main/scala/scalatorch/ffm/CudaProbe.scala:65-67",
        "a": [[1, 2, 3], [4, 5, 6]], "b": [[7, 8], [9, 10], [11, 12]],
        "expected": [[58, 64], [139, 154]],
    }
    cf = "cpu/src/test/scala/scalatorch/cpu/CpuFloatBackendSuite.scala"
    check_literal(root, cf, "Vector(10f,13f,22f,29f)")
    cases["gemm_2x2"] = {"cite": cf + ":29-41", "a": [[1, 2], [3, 4]], "b": [[2, 3], [4, 5]],
                         "expected": [[10, 13], [22, 29]]}
    check_literal(root, bs, "Seq.fill(6)(0f)")
    cases["gemm_empty_inner"] = {"cite": bs + ":34", "M": 2, "N": 3, "K": 0, "expected": [0.0] * 6}
    cases["gemm_nan_zero"] = {"cite": bs + ":38-43", "a": 0.0, "b": "nan", "expected": "nan"}

    # CudaProbeSuite patterns: values are multiples of 1/8 and 1/4 so every sum is exact.
    cp = "ffm/src/test/scala/scalatorch/ffm/CudaProbeSuite.scala"
    check_literal(root, cp, "(i % 11 - 5).toFloat / 8")
    check_literal(root, cp, "(i % 7 - 3).toFloat / 4")
    probe = []
    for m, n, k in [(2, 2, 3), (5, 17, 7), (3, 4, 0)]:
        a = [(i % 11 - 5) / 8 for i in range(m * k)]
        b = [(i % 7 - 3) / 4 for i in range(k * n)]
        c = [sum(a[i * k + p] * b[p * n + j] for p in range(k)) for i in range(m) for j in range(n)]
        probe.append({"m": m, "n": n, "k": k, "expected": c})
    cases["gemm_probe_patterns"] = {"cite": cp + ":17-28", "cases": probe}

    # --- decode-step ops
    check_literal(root, cf, "(6/math.sqrt(13)).toFloat")
    cases["rmsnorm"] = {"cite": cf + ":29-41", "x": [[3, 4], [0, 0]], "w": [2, 3], "eps": 0.5,
                        "expected_f32_bits": [f32bits(6 / math.sqrt(13)), f32bits(12 / math.sqrt(13)), 0, 0]}
    check_literal(root, cf, "-.26894142137")
    cases["silu"] = {"cite": cf + ":43-50", "x": [-1.0, 1.0], "expected": [-0.26894142137, 0.73105857863],
                     "tol": 1e-7, "neg_inf_bits": 0x80000000}
    check_literal(root, cf, "Vector(5f,6f,1f,2f,5f,6f,3f,4f)")
    cases["embedding"] = {"cite": cf + ":60-70", "table": [[1, 2], [3, 4], [5, 6]], "ids": [[2, 0], [2, 1]],
                          "expected": [5, 6, 1, 2, 5, 6, 3, 4]}
    ca = "cpu/src/test/scala/scalatorch/cpu/CpuAttentionSuite.scala"
    check_literal(root, ca, "Vector(2f,4f,6f,5f,7f,9f,2f,4f,6f,5f,7f,9f)")
    cases["rope"] = {"cite": ca + ":6-11", "x": [1, 2, 3, 4], "start": 1, "theta": 10000.0,
                     "expected": [1 * math.cos(1.0) - 3 * math.sin(1.0), 2 * math.cos(0.01) - 4 * math.sin(0.01)],
                     "tol": 1e-6}
    cases["attention"] = {
        "cite": ca + ":12-18", "q_shape": [1, 2, 2, 2], "k_shape": [1, 1, 2, 2], "v": [2, 4, 6, 8, 10, 12],
        "v_shape": [1, 1, 2, 3],
        "expected_start0": [2, 4, 6, 5, 7, 9, 2, 4, 6, 5, 7, 9],
        "expected_start1": [5, 7, 9, 5, 7, 9, 5, 7, 9, 5, 7, 9]}
    ss = "models/src/test/scala/scalatorch/models/SamplerSuite.scala"
    check_literal(root, ss, "Array(2f,2f,1f)")
    cases["greedy_ties"] = {"cite": ss + ":7-9; models/src/main/scala/scalatorch/models/TokenSampler.scala:32-38",
                            "logits": [2.0, 2.0, 1.0], "expected": 0}
    wr = "io/src/main/scala/scalatorch/io/SafeTensorsWriter.scala"
    check_literal(root, wr, "((bits+0x7fff+((bits>>>16)&1))>>>16)")
    cases["bf16_rne_rule"] = {"cite": wr + ":58-61",
                              "note": "NaN -> (bits>>>16)|0x40; else (bits+0x7fff+((bits>>>16)&1))>>>16"}

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_vectors.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SCALA_TORCH_ROOT", "."))
