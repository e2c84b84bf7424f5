"""Host-side safetensors validation of the raw-upload path (no GPU).

Behaviour follows the reference's io suites (io/src/test/scala/scalatorch/io/SafeTensorsSuite.scala,
ShardSuite.scala) and LlamaModel.load's checkpoint checks (LlamaModel.scala:158-173): every invalid
archive is rejected at open with IllegalArgumentException, before any payload read or device work.
"""
from __future__ import annotations

import json
import math
import os
import struct
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "scala-torch_b200"))

from scalatorch.ffm import IllegalArgumentException, IllegalStateException  # noqa: E402
from scalatorch.io import (ReadLimits, SafeTensors, SafeTensorSet, ShardLimits, write_index,  # noqa: E402
                           write_safetensors)
from scalatorch.models import LlamaConfig, check_llama_archive, llama_weight_shapes  # noqa: E402
from scalatorch.ffm import STB_BF16, STB_F16  # noqa: E402

GOLDEN = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_vectors.json")))["cases"]


def archive(tmp_path, header: str | bytes, payload: bytes = b"", name: str = "x.safetensors") -> str:
    h = header.encode("utf-8", "surrogatepass") if isinstance(header, str) else header
    path = os.path.join(str(tmp_path), name)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + payload)
    return path


def entry(dtype: str, shape: str, begin: int, end: int) -> str:
    return f'{{"dtype":"{dtype}","shape":{shape},"data_offsets":[{begin},{end}]}}'


def bad(tmp_path, header, payload=b"", **limits):
    path = archive(tmp_path, header, payload)
    with pytest.raises(IllegalArgumentException):
        SafeTensors(path, ReadLimits(**limits))


def test_upstream_rust_archive_reads_exactly(tmp_path):
    """The Rust safetensors 0.6.2 fixture (SafeTensorsSuite.scala:106-124) through the raw and typed
    readers."""
    g = GOLDEN["upstream_safetensors"]
    path = os.path.join(str(tmp_path), "upstream.safetensors")
    open(path, "wb").write(bytes.fromhex(g["archive_hex"]))
    with SafeTensors(path) as f:
        assert {n: (t.dtype, list(t.shape)) for n, t in f.tensors.items()} == \
            {n: (t["dtype"], t["shape"]) for n, t in g["tensors"].items()}
        assert f.read_raw("weight").ravel().tolist() == [1, 2, 3, 4, 5, 6]
        assert f.read_raw("bias").tolist() == [10, 20]
        assert f.read_raw("half").view(np.float16).astype(np.float32).tolist() == [1, -2, 2.0 ** -24, 65504]
        assert math.isnan((f.read_raw("bfloat").astype(np.uint32) << 16).view(np.float32)[-1])
        assert f.read_raw("long").tolist() == [9007199254740993, -7]
        assert f.read_raw("double").tolist() == [1.25, -2.5]
        assert f.read_raw("bool").tolist() == [0, 1]
        assert f.read_raw("empty").shape == (0, 3)
        assert f.read_float("weight").ravel().tolist() == [1, 2, 3, 4, 5, 6]
        assert f.read_float("half").tolist() == [1, -2, 2.0 ** -24, 65504]
        assert math.isnan(f.read_float("bfloat")[-1])
        assert f.read_long("long").tolist() == [9007199254740993, -7]
        assert f.read_double("double").tolist() == [1.25, -2.5]
        assert f.read_boolean("bool").tolist() == [False, True]
        assert f.read_float("empty").shape == (0, 3)


def test_typed_scalars_empty_tensors_and_metadata(tmp_path):
    payload = struct.pack("<fdqB", 1.5, -2.25, 9007199254740993, 1)
    header = ('{"__metadata__":{"format":"pt"},"f":' + entry("F32", "[]", 0, 4) + ',"d":' + entry("F64", "[]", 4, 12)
              + ',"l":' + entry("I64", "[]", 12, 20) + ',"b":' + entry("BOOL", "[]", 20, 21)
              + ',"z":' + entry("F32", "[2,0]", 21, 21) + "}   ")
    with SafeTensors(archive(tmp_path, header, payload)) as f:
        assert f.metadata == {"format": "pt"}
        assert f.read_raw("f").tolist() == 1.5 and f.read_raw("d").tolist() == -2.25
        assert f.read_raw("l").tolist() == 9007199254740993 and f.read_raw("b").tolist() == 1
        assert f.read_raw("z").shape == (2, 0)
        # typed reads (SafeTensorsSuite.scala:21-35)
        assert f.read_float("f").tolist() == 1.5 and f.read_double("d").tolist() == -2.25
        assert f.read_long("l").tolist() == 9007199254740993 and f.read_boolean("b").tolist() is True
        assert f.read_float("z").shape == (2, 0)
        for bad_read in (lambda: f.read_float("l"), lambda: f.read_float("missing"), lambda: f.read_raw("missing"),
                         lambda: f.read_double("f"), lambda: f.read_long("d"), lambda: f.read_boolean("f")):
            with pytest.raises(IllegalArgumentException):
                bad_read()


def _bits_of(values):
    return [int(v) for v in np.asarray(values, np.float32).view(np.uint32)]


def test_f16_and_bf16_widen_subnormals_signed_zero_and_nonfinite(tmp_path):
    """SafeTensorsSuite.scala:36-53, through read_float."""
    half = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xC000, 0x7BFF, 0x7C00, 0xFC00, 0x7E01]
    bf = [0x3F80, 0xC000, 0x0001, 0x8000, 0x7F80, 0xFF80, 0x7FC1]
    payload = np.array(half + bf, np.uint16).tobytes()
    header = ('{"h":' + entry("F16", f"[{len(half)}]", 0, 2 * len(half)) + ',"b":'
              + entry("BF16", f"[{len(bf)}]", 2 * len(half), len(payload)) + '}')
    with SafeTensors(archive(tmp_path, header, payload)) as f:
        h = f.read_float("h")
        assert _bits_of(h[:8]) == _bits_of([0.0, -0.0, 2.0 ** -24, 1023 * 2.0 ** -24, 2.0 ** -14, 1, -2, 65504])
        assert h[8] == np.inf and h[9] == -np.inf and math.isnan(h[10])
        b = f.read_float("b")
        assert b[:3].tolist() == [1.0, -2.0, 2.0 ** -133] and _bits_of(b[3:4]) == [0x80000000]
        assert b[4] == np.inf and b[5] == -np.inf and math.isnan(b[6])


def test_typed_reads_count_their_float32_output_against_the_limit(tmp_path):
    """SafeTensorsSuite.scala:75-95: a typed read counts the widened output (4 bytes per F16 word)."""
    half = archive(tmp_path, '{"x":' + entry("F16", "[1]", 0, 2) + '}', bytes([0, 0x3C]), name="h.safetensors")
    with SafeTensors(half, ReadLimits(max_tensor_bytes=2)) as f:
        assert f.tensors["x"].end == 2
        with pytest.raises(IllegalArgumentException):
            f.read_float("x")  # decoded Float32 needs 4 bytes
        assert f.read_raw("x").view(np.float16).tolist() == [1.0]
    with SafeTensors(half, ReadLimits(max_tensor_bytes=4)) as f:
        assert f.read_float("x").tolist() == [1.0]


def test_typed_decoders_cross_read_chunks(tmp_path):
    """SafeTensorsSuite.scala:96-105, 135-157."""
    n = 20000
    vals = (np.arange(n) / 8).astype(np.float32)
    with SafeTensors(archive(tmp_path, '{"x":' + entry("F32", f"[{n}]", 0, 4 * n) + '}', vals.tobytes())) as f:
        assert np.array_equal(f.read_float("x"), vals)
    n = 40000
    for dtype, words, expected in (("F16", [0x3C00, 0xC000, 0x0001, 0x7BFF], [1.0, -2.0, 2.0 ** -24, 65504.0]),
                                   ("BF16", [0x3F80, 0xC000, 0x0001, 0x7F7F],
                                    [1.0, -2.0, 2.0 ** -133, (2.0 - 1.0 / 128) * 2.0 ** 127])):
        payload = np.array(words * (n // 4), np.uint16).tobytes()
        path = archive(tmp_path, '{"x":' + entry(dtype, f"[{n}]", 0, 2 * n) + '}', payload,
                       name=f"{dtype}.safetensors")
        with SafeTensors(path) as f:
            assert np.array_equal(f.read_float("x"), np.array(expected * (n // 4), np.float32))
    count = 10000
    doubles = np.arange(count) + 0.125
    path = archive(tmp_path, '{"x":' + entry("F64", f"[{count}]", 0, 8 * count) + '}', doubles.tobytes(),
                   name="d.safetensors")
    with SafeTensors(path) as f:
        assert np.array_equal(f.read_double("x"), doubles)


@pytest.mark.parametrize("header,payload", [
    # duplicates, wrong types, unknown dtype, fractional integers (SafeTensorsSuite.scala:54-63)
    ('{"a":' + entry("F32", "[0]", 0, 0) + ',"a":' + entry("F32", "[0]", 0, 0) + '}', b""),
    ('{"a":{"dtype":"F32","dtype":"F16","shape":[0],"data_offsets":[0,0]}}', b""),
    ('{"__metadata__":{"x":1}}', b""),
    ('{"x":' + entry("F8_UNKNOWN", "[0]", 0, 0) + '}', b""),
    ('{"x":{"dtype":"F32","shape":[0.0],"data_offsets":[0,0]}}', b""),
    ('{"x":{"dtype":"F32","shape":[0],"data_offsets":[0,0.0]}}', b""),
    ("{} {}", b""),
    (" {}", b""),
    # offsets, shapes and file length (SafeTensorsSuite.scala:64-74)
    ('{"x":' + entry("F32", "[-1]", 0, 0) + '}', b""),
    ('{"x":' + entry("F32", "[9223372036854775807,2]", 0, 0) + '}', b""),
    ('{"x":' + entry("F64", "[9223372036854775807]", 0, 0) + '}', b""),
    ('{"x":' + entry("F32", "[1]", 0, 3) + '}', bytes(3)),
    ('{"a":' + entry("F32", "[1]", 0, 4) + ',"b":' + entry("F32", "[1]", 0, 4) + '}', bytes(4)),
    ('{"x":' + entry("F32", "[1]", 1, 5) + '}', bytes(5)),
    ('{"x":' + entry("F32", "[1]", 0, 4) + '}', bytes(3)),
    ("{}", bytes(1)),
    ('{"x":{"dtype":"F32","shape":[0],"data_offsets":[9007199254740993,9007199254740993]}}', b""),
    # unpaired surrogates, unsigned lengths, nesting (SafeTensorsSuite.scala:125-134)
    ('{"\\ud800":{"dtype":"F32","shape":[0],"data_offsets":[0,0]}}', b""),
    ('{"x":{"dtype":"F32","shape":[18446744073709551615],"data_offsets":[0,0]}}', b""),
    ('{"x":{"dtype":"F32","shape":[[[[0]]]],"data_offsets":[0,0]}}', b""),
    # metadata duplicates (SafeTensorsSuite.scala:158-169)
    ('{"__metadata__":{"a":"1","a":"2"}}', b""),
    ('{"__metadata__":{},"__metadata__":{}}', b""),
    # JSON forms the reference's parser has no token for: booleans as integers, NaN, reversed offsets
    ('{"x":{"dtype":"F32","shape":[true],"data_offsets":[0,4]}}', bytes(4)),
    ('{"x":{"dtype":"F32","shape":[0],"data_offsets":[NaN,0]}}', b""),
    ('{"x":' + entry("F32", "[0]", 4, 0) + '}', b""),
    ('{"x":{"dtype":"F32","shape":[0],"data_offsets":[0,0],"extra":1}}', b""),
    ('{"x":{"dtype":"F32","shape":[0]}}', b""),
])
def test_invalid_headers_reject_at_open(tmp_path, header, payload):
    bad(tmp_path, header, payload)


def test_malformed_prefixes_and_utf8_reject(tmp_path):
    path = os.path.join(str(tmp_path), "p.safetensors")
    for raw in (b"", b"\xff" * 8, bytes([2, 0, 0, 0, 0, 0, 0, 0, 0xC0, 0xAF])):
        open(path, "wb").write(raw)
        with pytest.raises(IllegalArgumentException):
            SafeTensors(path)
    raw = bytearray(open(archive(tmp_path, '{"__metadata__":{"a":"X"}}'), "rb").read())
    raw[raw.index(b"X", 8)] = 0xFF
    open(path, "wb").write(bytes(raw))
    with pytest.raises(IllegalArgumentException):
        SafeTensors(path)


def test_limits_lifetime_and_owned_results(tmp_path):
    """ReadLimits and close (SafeTensorsSuite.scala:75-95); raw reads count on-disk bytes."""
    path = archive(tmp_path, '{"x":' + entry("F32", "[2]", 0, 8) + '}', bytes(8))
    for limits in (dict(max_header_bytes=2), dict(max_tensors=0), dict(max_rank=0)):
        with pytest.raises(IllegalArgumentException):
            SafeTensors(path, ReadLimits(**limits))
    with pytest.raises(IllegalArgumentException):
        ReadLimits(max_header_bytes=1)
    with SafeTensors(path, ReadLimits(max_tensor_bytes=4)) as limited:
        with pytest.raises(IllegalArgumentException):
            limited.read_raw("x")
    f = SafeTensors(path)
    x = f.read_raw("x")
    f.close()
    f.close()
    with pytest.raises(IllegalStateException):
        f.read_raw("x")
    assert x.tolist() == [0.0, 0.0]
    half = archive(tmp_path, '{"x":' + entry("F16", "[1]", 0, 2) + '}', bytes([0, 0x3C]), name="h.safetensors")
    with SafeTensors(half, ReadLimits(max_tensor_bytes=2)) as f:
        assert f.read_raw("x").view(np.float16).tolist() == [1.0]  # 2 raw bytes: nothing is widened


def test_payloads_cross_read_chunks_and_shapes_stay_exact(tmp_path):
    n = 40000
    words = np.array([0x3C00, 0xC000, 0x0001, 0x7BFF] * (n // 4), np.uint16)
    path = archive(tmp_path, '{"x":' + entry("F16", f"[{n}]", 0, 2 * n) + '}', words.tobytes())
    with SafeTensors(path) as f:
        assert np.array_equal(f.read_raw("x"), words)
    big = 9007199254740993  # above double precision (SafeTensorsSuite.scala:170-178)
    with SafeTensors(archive(tmp_path, '{"x":' + entry("F32", f"[{big},0]", 0, 0) + '}', name="b.safetensors")) as f:
        assert f.tensors["x"].shape == (big, 0) and f.read_raw("x").shape == (big, 0)


def _shard(d, file, name, value):
    write_safetensors(os.path.join(d, file), {name: ("F32", (1,), np.array([value], np.float32))})


def _fixture(d):
    _shard(d, "a.safetensors", "a", 1.25)
    _shard(d, "b.safetensors", "b", -2.0)
    write_index(d, {"a": "a.safetensors", "b": "b.safetensors"}, total_size=8)


def test_indexed_sets_route_reads_and_close(tmp_path):
    """ShardSuite.scala:36-51."""
    d = str(tmp_path)
    _fixture(d)
    s = SafeTensorSet.open(d)
    assert set(s.tensors) == {"a", "b"}
    a = s.read_float("a")
    assert s.read_float("b").tolist() == [-2.0] and s.read_raw("b").tolist() == [-2.0]
    with pytest.raises(IllegalArgumentException):
        s.read_float("missing")
    with pytest.raises(IllegalArgumentException):
        s.read_long("a")
    s.close()
    s.close()
    assert a.tolist() == [1.25]
    with pytest.raises(IllegalStateException):
        s.read_raw("a")
    assert all(x.closed for x in s.archives)
    write_index(d, {"a": "a.safetensors", "b": "b.safetensors"})  # no total_size
    with SafeTensorSet.open(d) as s:
        assert len(s.tensors) == 2
        assert sorted(os.path.basename(p) for p in s.source_files) == \
            ["a.safetensors", "b.safetensors", "model.safetensors.index.json"]


def test_single_archive_and_ambiguity(tmp_path):
    """ShardSuite.scala:52-60; explicit archive names (ShardSuite.scala:8-19)."""
    d = str(tmp_path)
    _shard(d, "model.safetensors", "a", 3.0)
    with SafeTensorSet.open(d) as s:
        assert s.read_raw("a").tolist() == [3.0]
    write_index(d, {"a": "a.safetensors"})
    with pytest.raises(IllegalArgumentException):
        SafeTensorSet.open(d)
    for name in ("../model.safetensors", "a/b.safetensors", "C:model.safetensors", "bad.bin", "", ".safetensors"):
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d, filename=name)
    with SafeTensorSet.open_file(os.path.join(d, "model.safetensors")) as s:
        assert s.names() == ["a"]


def test_index_assignments_totals_and_limits(tmp_path):
    """ShardSuite.scala:75-92."""
    d = str(tmp_path)
    _fixture(d)
    for weight_map in ({"a": "a.safetensors", "b": "a.safetensors"}, {"a": "b.safetensors", "b": "a.safetensors"},
                       {"x": "a.safetensors", "b": "b.safetensors"}, {"a": "missing.safetensors"}):
        write_index(d, weight_map, total_size=8)
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d)
    write_index(d, {"a": "a.safetensors", "b": "b.safetensors"}, total_size=9)
    with pytest.raises(IllegalArgumentException):
        SafeTensorSet.open(d)
    write_index(d, {"a": "a.safetensors", "b": "b.safetensors"}, total_size=8)
    for kwargs in (dict(read_limits=ReadLimits(max_tensors=1)), dict(shard_limits=ShardLimits(max_shards=1)),
                   dict(shard_limits=ShardLimits(max_index_bytes=8))):
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d, **kwargs)
    _shard(d, "b.safetensors", "a", 2.0)
    with pytest.raises(IllegalArgumentException):
        SafeTensorSet.open(d)


def test_index_rejects_malformed_json_and_escaping_paths(tmp_path):
    """ShardSuite.scala:93-103."""
    d = str(tmp_path)
    _fixture(d)
    index = os.path.join(d, "model.safetensors.index.json")
    for shard in ("../a.safetensors", "/tmp/a.safetensors", "x/a.safetensors", "x\\a.safetensors", "C:a.safetensors",
                  "bad.bin", ""):
        write_index(d, {"a": shard})
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d)
    for raw in ("{}", "{", '{"weight_map":{}}', '{"weight_map":{"a":1}}',
                '{"weight_map":{"a":"a.safetensors","a":"a.safetensors"}}',
                '{"metadata":{"total_size":8.0},"weight_map":{}}', '{"metadata":{"total_size":-1},"weight_map":{}}',
                '{"weight_map":{"a":"a.safetensors"},"extra":{}}', '{"weight_map":{"":"a.safetensors"}}'):
        open(index, "w").write(raw)
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d)


def test_failed_open_keeps_no_descriptors(tmp_path):
    """ShardSuite.scala:104-118: a later shard's failure closes the shards already opened."""
    d = str(tmp_path)
    _fixture(d)
    open(os.path.join(d, "b.safetensors"), "w").write("bad")

    def open_here():
        fds = "/proc/self/fd"
        n = 0
        for fd in os.listdir(fds):
            try:
                n += os.readlink(os.path.join(fds, fd)).startswith(d)
            except OSError:
                pass
        return n

    if not os.path.isdir("/proc/self/fd"):
        pytest.skip("Linux descriptor table")
    before = open_here()
    for _ in range(12):
        with pytest.raises(IllegalArgumentException):
            SafeTensorSet.open(d)
    assert open_here() == before


TINY = dict(vocab_size=40, hidden_size=16, intermediate_size=24, num_layers=2, num_attention_heads=4,
            num_key_value_heads=2, max_positions=32, eos_token_ids=())


def _llama_dir(d, cfg: LlamaConfig, dtype="BF16", drop=(), extra=None, override=None):
    rng = np.random.default_rng(0)
    tensors = {}
    for name, shape in llama_weight_shapes(cfg).items():
        if name in drop or (cfg.tie_word_embeddings and name == "lm_head.weight"):
            continue
        dt = "F32" if len(shape) == 1 else dtype
        arr = rng.standard_normal(shape).astype(np.float32)
        arr = arr.view(np.uint32) >> 16 if dt == "BF16" else arr.astype(np.float16) if dt == "F16" else arr
        tensors[name] = (dt, shape, np.asarray(arr, {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}[dt]))
    tensors.update(extra or {})
    for name, spec in (override or {}).items():
        tensors[name] = spec
    write_safetensors(os.path.join(d, "model.safetensors"), tensors)
    return tensors


def test_llama_checkpoint_checks_before_device_work(tmp_path):
    """LlamaModel.load's name / shape / dtype checks (LlamaModel.scala:158-167), host only."""
    cfg = LlamaConfig(**TINY)
    cases = [
        (dict(), None),
        (dict(drop=("model.layers.1.mlp.up_proj.weight",)), "names mismatch"),
        (dict(extra={"model.layers.2.mlp.up_proj.weight": ("BF16", (24, 16), np.zeros((24, 16), np.uint16))}),
         "names mismatch"),
        (dict(override={"model.layers.0.self_attn.k_proj.weight": ("BF16", (16, 16), np.zeros((16, 16), np.uint16))}),
         "metadata mismatch"),
        (dict(override={"model.norm.weight": ("I32", (16,), np.zeros(16, np.int32))}), "metadata mismatch"),
        (dict(override={"model.layers.0.self_attn.q_proj.weight": ("F16", (16, 16), np.zeros((16, 16), np.float16))}),
         "share one"),
        (dict(dtype="F32"), "share one"),
    ]
    for i, (kwargs, error) in enumerate(cases):
        d = os.path.join(str(tmp_path), str(i))
        os.makedirs(d)
        _llama_dir(d, cfg, **kwargs)
        with SafeTensorSet.open(d) as s:
            if error is None:
                assert check_llama_archive(cfg, s) == (STB_BF16, False)
            else:
                with pytest.raises(IllegalArgumentException, match=error):
                    check_llama_archive(cfg, s)
    d = os.path.join(str(tmp_path), "f16")
    os.makedirs(d)
    _llama_dir(d, cfg, dtype="F16")
    with SafeTensorSet.open(d) as s:
        assert check_llama_archive(cfg, s) == (STB_F16, False)


def test_tied_head_must_equal_the_embeddings(tmp_path):
    """LlamaModel.scala:169-173: a stored lm_head beside tied embeddings must match bit for bit."""
    cfg = LlamaConfig(**dict(TINY, tie_word_embeddings=True))
    d = os.path.join(str(tmp_path), "absent")
    os.makedirs(d)
    _llama_dir(d, cfg)
    with SafeTensorSet.open(d) as s:
        assert check_llama_archive(cfg, s) == (STB_BF16, False)
    emb = _llama_dir(d, cfg)["model.embed_tokens.weight"][2]
    for name, head, ok in (("same", emb.copy(), True), ("f32", (emb.astype(np.uint32) << 16).view(np.float32), True),
                           ("other", emb ^ np.uint16(1), False)):
        d = os.path.join(str(tmp_path), name)
        os.makedirs(d)
        dt = "F32" if head.dtype == np.float32 else "BF16"
        _llama_dir(d, cfg, extra={"lm_head.weight": (dt, head.shape, head)})
        with SafeTensorSet.open(d) as s:
            if ok:
                assert check_llama_archive(cfg, s) == (STB_BF16, True)
            else:
                with pytest.raises(IllegalArgumentException, match="conflicting tied"):
                    check_llama_archive(cfg, s)


def test_indexed_set_keeps_the_upstream_fixture_dtypes(tmp_path):
    """ShardSuite.scala:61-74: typed reads through an index over the Rust-written archive."""
    d = str(tmp_path)
    g = GOLDEN["upstream_safetensors"]
    open(os.path.join(d, "typed.safetensors"), "wb").write(bytes.fromhex(g["archive_hex"]))
    write_index(d, {n: "typed.safetensors" for n in g["tensors"]})
    with SafeTensorSet.open(d) as s:
        assert s.read_double("double").tolist() == [1.25, -2.5]
        assert s.read_long("long").tolist() == [9007199254740993, -7]
        assert s.read_boolean("bool").tolist() == [False, True]
        assert s.read_float("half")[0] == 1.0


def test_random_header_values_fail_only_as_invalid_arguments(tmp_path):
    """Any JSON value in any field of a tensor entry either opens consistently or is rejected with
    IllegalArgumentException (never another exception type), as the reference's parser does."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    scalars = st.one_of(st.none(), st.booleans(), st.integers(-2 ** 70, 2 ** 70), st.floats(allow_nan=False),
                        st.text(max_size=6))
    values = st.recursive(scalars, lambda c: st.one_of(st.lists(c, max_size=3),
                                                       st.dictionaries(st.text(max_size=4), c, max_size=3)),
                          max_leaves=6)
    fields = st.fixed_dictionaries({}, optional={"dtype": st.one_of(st.sampled_from(["F32", "BF16", "I64"]), values),
                                                 "shape": st.one_of(st.lists(st.integers(0, 3), max_size=3), values),
                                                 "data_offsets": st.one_of(st.lists(st.integers(0, 16), max_size=3),
                                                                           values),
                                                 "extra": values})

    @settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(fields, st.integers(0, 16))
    def check(entry_obj, payload_len):
        path = archive(tmp_path, json.dumps({"x": entry_obj}), bytes(payload_len), name="fuzz.safetensors")
        try:
            with SafeTensors(path) as f:
                info = f.tensors["x"]
                assert info.end - info.begin == payload_len and f.read_raw("x").nbytes == payload_len
        except IllegalArgumentException:
            pass

    check()


def test_random_index_documents_fail_only_as_invalid_arguments(tmp_path):
    """Any JSON document as model.safetensors.index.json either opens or is rejected with
    IllegalArgumentException (SafeTensorsIndex.read's contract)."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    d = str(tmp_path)
    _shard(d, "a.safetensors", "a", 1.25)
    scalars = st.one_of(st.none(), st.booleans(), st.integers(-5, 10), st.floats(allow_nan=False),
                        st.sampled_from(["a", "a.safetensors", "b.safetensors", "../a.safetensors", ""]))
    values = st.recursive(scalars, lambda c: st.one_of(st.lists(c, max_size=3),
                                                       st.dictionaries(st.sampled_from(["a", "b", "total_size"]), c,
                                                                       max_size=3)),
                          max_leaves=6)
    docs = st.one_of(values, st.fixed_dictionaries({}, optional={"weight_map": values, "metadata": values,
                                                                 "other": values}))

    @settings(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
    @given(docs)
    def check(doc):
        with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
            json.dump(doc, f)
        try:
            with SafeTensorSet.open(d) as s:
                assert set(s.tensors) == {"a"} and s.read_float("a").tolist() == [1.25]
        except IllegalArgumentException:
            pass

    check()
