"""Device Llama runtime against the CPU oracle on the same synthetic BF16 weights.

Tolerances: logits |a - e| <= 1e-5 * (1 + |e|) (the reference holds 3e-6*(1+|e|) between its
own CUDA and CPU paths, BackendLlamaSuite.scala:18, for a 1-layer model; deeper models add
per-layer Float32 reassociation); greedy token ids identical for the small models.
"""
import os
import tempfile

import numpy as np
import pytest

from llama_fixtures import SMOL, TINY, named_bf16_weights, oracle_model
from scalatorch import ffm
from scalatorch.io import write_index, write_safetensors
from scalatorch.models import BackendLlama, LlamaConfig, load_safetensors

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-5


def close(a, e, tol=LOGIT_TOL):
    err = np.abs(a.astype(np.float64) - e.astype(np.float64))
    lim = tol * (1 + np.abs(e.astype(np.float64)))
    assert np.all(err <= lim), f"max err {err.max()}, worst ratio {np.max(err / lim)}"


@pytest.fixture(scope="module")
def tiny():
    return LlamaConfig(**TINY)


def test_tiny_cached_decode_matches_oracle(session, tiny):
    ref = oracle_model(tiny, seed=3)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, tiny.vocab_size, (2, 5))
    with BackendLlama.prepare_random(session, tiny, seed=3) as m:
        cache = m.new_cache(batch_size=2, capacity=12)
        oc = ref.new_cache(2, 12)
        got, nxt = cache.decode(prompt)
        want = ref.decode(oc, prompt)
        close(got, want)
        assert cache.position == 5
        for step in range(4):
            tok = rng.integers(0, tiny.vocab_size, (2, 1))
            got, nxt = cache.decode(tok)
            want = ref.decode(oc, tok)
            close(got, want)
            assert nxt == [int(np.argmax(want[b, -1])) for b in range(2)]
        assert cache.position == 9
        ref.free_cache(oc)
        cache.close()


def test_tiny_generate_ids_match_oracle(session, tiny):
    ref = oracle_model(tiny, seed=5)
    prompt = [1, 17, 400, 999, 3]
    with BackendLlama.prepare_random(session, tiny, seed=5) as m:
        assert m.generate_ids(prompt, 20) == ref.generate(prompt, 20)
        # EOS stop: stop at the 4th generated id of the unconstrained run
        full = ref.generate(prompt, 20)
        eos = full[len(prompt) + 3]
        got = m.generate_ids(prompt, 20, eos_token_ids=[eos])
        assert got == ref.generate(prompt, 20, eos=[eos])
        assert got[-1] == eos and len(got) <= len(full)
        assert m.generate_ids(prompt, 0) == prompt


def test_repeated_generation_reuses_the_cache_and_graph(session, tiny):
    """A generate call of the same shape as the previous one reuses its cache, buffers and decode
    graph: identical ids, no growth of the session's allocations; a different shape rebuilds."""
    ref = oracle_model(tiny, seed=21)
    prompts = np.array([[5, 6, 7, 8], [900, 1, 2, 3]])
    with BackendLlama.prepare_random(session, tiny, seed=21) as m:
        first = m.generate_ids(prompts, 9)
        held = session.allocated_bytes
        for _ in range(3):
            assert m.generate_ids(prompts, 9) == first
            assert session.allocated_bytes == held
        assert m.generate_ids(prompts[:1], 5) == [ref.generate(prompts[0].tolist(), 5)]
        assert m.generate_ids(prompts, 9) == first
    for b in range(2):
        assert first[b] == ref.generate(prompts[b].tolist(), 9)


def test_batched_generation_rows_are_independent(session, tiny):
    ref = oracle_model(tiny, seed=9)
    prompts = np.array([[5, 6, 7, 8], [900, 1, 2, 3], [42, 42, 42, 42]])
    with BackendLlama.prepare_random(session, tiny, seed=9) as m:
        rows = m.generate_ids(prompts, 10)
        for b in range(3):
            assert rows[b] == ref.generate(prompts[b].tolist(), 10)


def test_safetensors_raw_upload_equals_device_init(session, tiny):
    named = named_bf16_weights(tiny, seed=11)
    with tempfile.TemporaryDirectory() as d:
        cfg = ('{"model_type":"llama","vocab_size":1000,"hidden_size":64,"intermediate_size":128,'
               '"num_hidden_layers":2,"num_attention_heads":4,"num_key_value_heads":2,'
               '"max_position_embeddings":64,"tie_word_embeddings":false,"eos_token_id":null}')
        open(os.path.join(d, "config.json"), "w").write(cfg)
        names = sorted(named)
        half = len(names) // 2
        weight_map = {}
        for i, part in enumerate((names[:half], names[half:])):  # a two-shard indexed set
            write_safetensors(os.path.join(d, f"model-{i}.safetensors"),
                              {n: ("BF16", named[n].shape, named[n]) for n in part})
            weight_map.update({n: f"model-{i}.safetensors" for n in part})
        write_index(d, weight_map, total_size=sum(named[n].nbytes for n in names))
        loaded = load_safetensors(session, d)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    with loaded, BackendLlama.prepare_random(session, tiny, seed=11) as gen:
        a = loaded.new_cache(1, 16)
        b = gen.new_cache(1, 16)
        la, _ = a.decode([prompt])
        lb, _ = b.decode([prompt])
        assert np.array_equal(la, lb)  # identical bits: raw upload == device generator
        # resident bytes: half matrices (never widened), F32 norms, the double rotary table
        H, V, I, L, hd, pos = 64, 1000, 128, 2, 16, 64
        half_matrices = 2 * V * H + L * ((4 + 2 * 2) * hd * H + H * H + 2 * I * H + H * I)
        assert loaded.weight_bytes == 2 * half_matrices + 4 * H * (2 * L + 1) + pos * (hd // 2) * 16


def test_tied_checkpoint_with_a_stored_head_loads_once(session):
    """A tied checkpoint that also stores lm_head.weight (equal to the embeddings) passes
    LlamaModel.load's check (LlamaModel.scala:169-173), uploads the embeddings once and decodes as
    the device-initialised tied model; a differing stored head is rejected before any upload."""
    cfg = LlamaConfig(**dict(TINY, tie_word_embeddings=True))
    named = named_bf16_weights(cfg, seed=17)
    text = ('{"model_type":"llama","vocab_size":1000,"hidden_size":64,"intermediate_size":128,'
            '"num_hidden_layers":2,"num_attention_heads":4,"num_key_value_heads":2,'
            '"max_position_embeddings":64,"tie_word_embeddings":true,"eos_token_id":null}')
    prompt = [7, 1, 8, 2, 8]
    for head, ok in ((named["model.embed_tokens.weight"].copy(), True),
                     (named["model.embed_tokens.weight"] ^ np.uint16(1), False)):
        with tempfile.TemporaryDirectory() as d:
            open(os.path.join(d, "config.json"), "w").write(text)
            tensors = {n: ("BF16", v.shape, v) for n, v in named.items()}
            tensors["lm_head.weight"] = ("BF16", head.shape, head)
            write_safetensors(os.path.join(d, "model.safetensors"), tensors)
            if not ok:
                held = session.allocated_bytes
                with pytest.raises(ffm.IllegalArgumentException, match="conflicting tied"):
                    load_safetensors(session, d)
                assert session.allocated_bytes == held
                continue
            loaded = load_safetensors(session, d)
        with loaded, BackendLlama.prepare_random(session, cfg, seed=17) as gen:
            assert loaded.weight_bytes == gen.weight_bytes
            la, _ = loaded.new_cache(1, 16).decode([prompt])
            lb, _ = gen.new_cache(1, 16).decode([prompt])
            assert np.array_equal(la, lb)


def test_tied_head_is_stored_once(session):
    cfg = LlamaConfig(**dict(TINY, tie_word_embeddings=True))
    untied = LlamaConfig(**TINY)
    with BackendLlama(session, cfg) as a, BackendLlama(session, untied) as b:
        assert b.weight_bytes - a.weight_bytes == 2 * cfg.vocab_size * cfg.hidden_size


def test_chunked_prefill_matches_oracle(session, tiny, monkeypatch):
    """Prompts prefilled in several chunks (STB_PREFILL_CHUNK_ROWS) give the same greedy ids."""
    ref = oracle_model(tiny, seed=13)
    prompts = np.array([[3, 1, 4, 1, 5, 9, 2], [6, 5, 3, 5, 8, 9, 7]])
    monkeypatch.setenv("STB_PREFILL_CHUNK_ROWS", "4")  # 2 tokens per chunk for batch 2
    with BackendLlama.prepare_random(session, tiny, seed=13) as m:
        rows = m.generate_ids(prompts, 8)
    for b in range(2):
        assert rows[b] == ref.generate(prompts[b].tolist(), 8)


def test_tensor_core_prefill_within_prefill_tolerance(session, tiny):
    """Chunks of >= tc_prefill_rows rows run the projections on tcgen05 with activations rounded to
    BF16.  Each rounded GEMM is within 2e-3 normwise (test_prefill_gpu.py); a model chains four of
    them per layer, so the model-level logits tolerance is 1e-2 normwise per row (observed ~3e-3 for
    two layers).  The single-token decode steps after it keep Float32 activations."""
    ref = oracle_model(tiny, seed=17)
    rng = np.random.default_rng(17)
    prompt = rng.integers(0, tiny.vocab_size, (2, 6))
    with BackendLlama.prepare_random(session, tiny, seed=17, tc_prefill_rows=4) as m:
        c = m.new_cache(2, 12)
        oc = ref.new_cache(2, 12)
        got, _ = c.decode(prompt)  # 12 rows -> tensor cores
        want = ref.decode(oc, prompt)
        for b in range(2):
            for t in range(6):
                rel = np.linalg.norm(got[b, t] - want[b, t]) / np.linalg.norm(want[b, t])
                assert rel <= 1e-2, (b, t, rel)
        got, _ = c.decode([[7], [8]])  # 2 rows -> Float32 GEMV path over the tensor-core-built cache
        want = ref.decode(oc, np.array([[7], [8]]))
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert rel <= 1e-2, rel
        ref.free_cache(oc)
        c.close()


@pytest.mark.parametrize("heads,kv,chunks", [(8, 2, ((0, 100), (100, 150))), (4, 1, ((0, 100), (100, 150))),
                                             (4, 1, ((0, 300),)), (8, 8, ((0, 40), (40, 300)))])
def test_tiled_prefill_attention_on_long_chunks(session, heads, kv, chunks):
    """Tensor-core prefill chunks use the tcgen05 flash attention (128-query x 128-key tiles, BF16 Q / K
    / V / P, online softmax in FP32).  Head sizes 64 and 128, grouped and ungrouped heads, two batch
    rows, several query and key tiles with the causal diagonal inside a tile, and a second chunk that
    attends to the first chunk's cached keys (ragged tiles on both axes): logits within the
    tensor-core prefill tolerance, 1e-2 normwise per row."""
    cfg = LlamaConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_layers=1,
                      num_attention_heads=heads, num_key_value_heads=kv, max_positions=512,
                      tie_word_embeddings=False, eos_token_ids=())
    ref = oracle_model(cfg, seed=23)
    rng = np.random.default_rng(23)
    end = chunks[-1][1]
    prompt = rng.integers(0, cfg.vocab_size, (2, end))
    with BackendLlama.prepare_random(session, cfg, seed=23, tc_prefill_rows=64) as m:
        c = m.new_cache(2, end + 10)
        oc = ref.new_cache(2, end + 10)
        for lo, hi in chunks:
            got, _ = c.decode(prompt[:, lo:hi])
            want = ref.decode(oc, prompt[:, lo:hi])
            rel = np.linalg.norm(got - want, axis=-1) / np.linalg.norm(want, axis=-1)
            assert rel.max() <= 1e-2, (lo, rel.max())
        assert c.position == end
        ref.free_cache(oc)
        c.close()


def test_cache_rejects_and_keeps_position(session, tiny):
    with BackendLlama.prepare_random(session, tiny, seed=1) as m:
        c = m.new_cache(1, 6)
        c.decode([[1, 2, 3, 4]])
        with pytest.raises(ffm.IllegalArgumentException):
            c.decode([[1, 2, 3]])  # capacity 6 exceeded
        assert c.position == 4
        with pytest.raises(ffm.IllegalArgumentException):
            c.decode([[1000]])  # outside the vocabulary
        assert c.position == 4
        c.reset()
        assert c.position == 0
        with pytest.raises(ffm.IllegalArgumentException):
            m.generate_ids([1], 64)  # prompt + new > max_positions
        c.close()


def test_smollm2_shaped_greedy_ids_and_logits(session):
    """SmolLM2-135M shape (30 layers, vocab 49152, 9/3 heads) with a shortened prompt and
    decode so the CPU oracle finishes in seconds; ids must be identical."""
    cfg = LlamaConfig(**SMOL)
    ref = oracle_model(cfg, seed=2024)
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, cfg.vocab_size, 12).tolist()
    with BackendLlama.prepare_random(session, cfg, seed=2024) as m:
        assert m.generate_ids(prompt, 12) == ref.generate(prompt, 12)
        c = m.new_cache(1, 32)
        oc = ref.new_cache(1, 32)
        got, _ = c.decode([prompt])
        close(got, ref.decode(oc, np.array([prompt])))
        got, _ = c.decode([[17]])
        close(got, ref.decode(oc, np.array([[17]])))
        ref.free_cache(oc)
        c.close()


def test_smollm2_full_bench_configuration_ids_and_logits(session):
    """The benchmarked SmolLM2 configuration itself: seed 2024, a 128-token prompt of ids uniform in
    [0, 49152) (numpy default_rng(2024)), 128 greedy tokens -- ids identical to the oracle's, and the
    logits after the prompt within 1e-5 (1 + |e|)."""
    cfg = LlamaConfig(**SMOL)
    ref = oracle_model(cfg, seed=2024)
    prompt = np.random.default_rng(2024).integers(0, cfg.vocab_size, 128).tolist()
    with BackendLlama.prepare_random(session, cfg, seed=2024) as m:
        assert m.generate_ids(prompt, 128) == ref.generate(prompt, 128)
        c = m.new_cache(1, 129)
        oc = ref.new_cache(1, 129)
        got, _ = c.decode([prompt])
        close(got[0, -1], ref.decode(oc, np.array([prompt]))[0, -1])
        ref.free_cache(oc)
        c.close()


# head size 128 and a query group of 8 (the 70B shape's attention) on a small model
HD128 = dict(vocab_size=512, hidden_size=1024, intermediate_size=256, num_layers=2, num_attention_heads=8,
             num_key_value_heads=1, max_positions=512, tie_word_embeddings=False, eos_token_ids=())


@pytest.mark.parametrize("stream,impl,kps,hd128,heads,kvh,g8", [
    (1, 1, 0, 1, 8, 1, 1), (1, 1, 32, 1, 8, 1, 1), (1, 1, 64, 1, 6, 1, 1), (1, 1, 96, 1, 5, 1, 1),
    (1, 1, 40, 1, 8, 1, 1), (1, 1, 72, 1, 8, 2, 1),
    (1, 1, 32, 1, 8, 1, 0), (1, 1, 64, 1, 8, 2, 1), (1, 1, 96, 1, 6, 2, 1), (1, 1, 32, 1, 4, 4, 1),
    (0, 1, 32, 1, 8, 1, 1), (0, 1, 64, 1, 8, 1, 1), (0, 1, 128, 1, 8, 1, 1), (0, 1, 64, 0, 8, 1, 1),
    (0, 0, 0, 1, 8, 1, 1), (0, 1, 64, 1, 8, 2, 1), (0, 1, 32, 1, 6, 2, 1)])
def test_decode_attention_splits_head128(stream, impl, kps, hd128, heads, kvh, g8):
    """The decode attention on head size 128 with 8, 6, 5, 4, 3 and 1 query heads per KV head: the streamed
    form (decode_attention_stream_g8_kernel for 5 to 8 heads per KV head, or decode_attention_stream_kernel
    with STB_DS_G8=0 and for smaller groups, + the merge in the o projection's prologue) with its keys per
    split left to the plan or forced to 32 / 40 / 64 / 72 / 96 (STB_DS_KPS; 40 and 72 end splits inside a
    32-key chunk), and with STB_DECODE_STREAM=0 the split forms
    (decode_attention_hd128_kernel, and decode_attention_kernel with STB_DA_HD128=0) with keys per split
    forced to 32 / 64 / 128 (STB_DA_KPS) and the register form (STB_DA_IMPL) -- variables read once per
    process: a child process each -- over 127 prompt tokens
    (254 rows: below the tensor-core prefill threshold, so the whole run keeps Float32 activations) and 8
    decode steps for 2 rows, so splits merge: greedy ids identical to the oracle and the logits of a
    cached step within 1e-5 (1 + |e|)."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{root!r}, {os.path.join(root, 'scala-torch_b200')!r}, {os.path.join(root, 'tests')!r}]\n"
        "from llama_fixtures import oracle_model\n"
        "from test_llama_gpu import HD128, close\n"
        "from scalatorch import ffm\n"
        "from scalatorch.models import BackendLlama, LlamaConfig\n"
        f"cfg = LlamaConfig(**dict(HD128, hidden_size={heads * 128}, num_attention_heads={heads}, "
        f"num_key_value_heads={kvh}))\n"
        "ref = oracle_model(cfg, seed=9)\n"
        "rng = np.random.default_rng(3)\n"
        "prompts = rng.integers(0, cfg.vocab_size, (2, 127))\n"
        "s = ffm.B200Session(0, 8 << 30)\n"
        "with BackendLlama.prepare_random(s, cfg, seed=9) as m:\n"
        "    got = m.generate_ids(prompts, 8)\n"
        "    for b in range(2):\n"
        "        assert got[b] == ref.generate(prompts[b].tolist(), 8), b\n"
        "    c = m.new_cache(2, 140)\n"
        "    oc = ref.new_cache(2, 140)\n"
        "    c.decode(prompts)\n"
        "    ref.decode(oc, prompts)\n"
        "    lg, _ = c.decode([[7], [300]])\n"
        "    close(lg, ref.decode(oc, np.array([[7], [300]])))\n"
        "    ref.free_cache(oc)\n"
        "    c.close()\n"
        "s.close()\n"
        "print('ok')\n")
    env = dict(os.environ, STB_DECODE_STREAM=str(stream), STB_DS_KPS=str(kps if stream else 0),
               STB_DA_KPS=str(0 if stream else kps), STB_DA_IMPL=str(impl), STB_DA_HD128=str(hd128), STB_DS_G8=str(g8))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]



@pytest.mark.parametrize("batch,fuse,heads,kvh", [(3, 1, 8, 2), (3, 0, 8, 2), (20, 1, 8, 2), (40, 1, 8, 2),
                                                 (40, 0, 8, 2), (3, 1, 8, 1), (3, 0, 8, 1), (20, 1, 6, 1),
                                                 (40, 1, 8, 1)])
def test_skinny_decode_with_fused_prologues(batch, fuse, heads, kvh):
    """Decode steps whose every projection takes the tensor-core skinny form (STB_SKINNY_MIN_WORK=0, batch
    rows 3 / 20 / 40: 16-, 32- and 64-row term tiles), with the next projection's prologue done by the
    fixups (STB_FUSE_NEXT=1: o -> RMSNorm + split for gate/up, SiLU*up -> split for down, down -> RMSNorm
    + split for the next layer's q/k/v) or by their own prologue kernels (0); with 8 or 6 query heads per
    KV head (head size 128) the attention also adds the QKV projection's pieces (RoPE, cache append) and
    merges its own splits (STB_FUSE_ATT=1) instead of the QKV fixup and merge kernels (0).  RMSNorm weights are
    random, not ones, so each fused norm must use its own layer's weights.  The prompt pass stays on the
    Float32 path (tensor-core prefill off).  Child processes (variables read
    once per process): greedy ids identical to the oracle and the logits of a cached step within
    1e-5 (1 + |e|)."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{root!r}, {os.path.join(root, 'scala-torch_b200')!r}, {os.path.join(root, 'tests')!r}]\n"
        "import oracle\n"
        "from llama_fixtures import oracle_model\n"
        "from test_llama_gpu import HD128, close\n"
        "from scalatorch import ffm\n"
        "from scalatorch.models import BackendLlama, LlamaConfig\n"
        f"cfg = LlamaConfig(**dict(HD128, hidden_size={heads * 128}, num_attention_heads={heads}, "
        f"num_key_value_heads={kvh}, intermediate_size=384, max_positions=64))\n"
        "rng = np.random.default_rng(5)\n"
        "H = cfg.hidden_size\n"
        "norms = {'model.norm.weight': oracle.round_bf16((1 + 0.25 * rng.standard_normal(H)).astype(np.float32))}\n"
        "for l in range(cfg.num_layers):\n"
        "    for n in ('input_layernorm', 'post_attention_layernorm'):\n"
        "        norms[f'model.layers.{l}.{n}.weight'] = oracle.round_bf16("
        "(1 + 0.25 * rng.standard_normal(H)).astype(np.float32))\n"
        "ref = oracle_model(cfg, seed=9, replace=norms)\n"
        f"prompts = rng.integers(0, cfg.vocab_size, ({batch}, 20))\n"
        "s = ffm.B200Session(0, 8 << 30)\n"
        "with BackendLlama.prepare_random(s, cfg, seed=9, tc_prefill_rows=-1) as m:\n"
        "    for name, bits in norms.items():\n"
        "        m.set_weight(name, bits, ffm.STB_BF16)\n"
        "    got = m.generate_ids(prompts, 6)\n"
        f"    for b in range({batch}):\n"
        "        assert got[b] == ref.generate(prompts[b].tolist(), 6), b\n"
        f"    c = m.new_cache({batch}, 40)\n"
        f"    oc = ref.new_cache({batch}, 40)\n"
        "    c.decode(prompts)\n"
        "    ref.decode(oc, prompts)\n"
        f"    nxt = rng.integers(0, cfg.vocab_size, ({batch}, 1))\n"
        "    lg, _ = c.decode(nxt)\n"
        "    close(lg, ref.decode(oc, nxt))\n"
        "    lg, _ = c.decode(nxt[::-1].copy())\n"
        "    close(lg, ref.decode(oc, nxt[::-1].copy()))\n"
        "    ref.free_cache(oc)\n"
        "    c.close()\n"
        "s.close()\n"
        "print('ok')\n")
    env = dict(os.environ, STB_SKINNY_MIN_WORK="0", STB_FUSE_NEXT=str(fuse), STB_FUSE_ATT=str(fuse))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
