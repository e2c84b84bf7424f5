"""Tensor-parallel Llama decode on 2 GPUs (Megatron splits, one NCCL allreduce per row-split
projection) against the CPU oracle.  Skipped when fewer than two GPUs are visible.

Each rank is a spawned process bound to its own GPU; rank 0 creates the NCCL unique id and hands
it to the others through a queue.  Every rank must produce the single-GPU oracle's greedy ids.
A rank that fails reports its error through the result queue; the parent kills ranks that do not
finish in time, so a broken collective cannot hang the run.
"""
import multiprocessing as mp
import os
import queue
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# Wide enough that every projection of a 2-row decode step can take the tensor-core skinny form
# (local N >= 128; the ranks set STB_SKINNY_MIN_WORK=0), including the row-split o / down projections
# with the peer-exchange epilogue.
WIDE = dict(vocab_size=1000, hidden_size=256, intermediate_size=512, num_layers=2, num_attention_heads=8,
            num_key_value_heads=4, max_positions=64, tie_word_embeddings=False, eos_token_ids=())
# Head size 128 with 8 query heads per KV head on each rank: the fused decode attention (QKV pieces,
# RoPE, cache append and split merge in one kernel), the peer reduces that also do the next RMSNorm
# and split, and the SiLU split -- with random RMSNorm weights (NORM_SEED), so each fused norm must use
# its own layer's weights.
G8 = dict(vocab_size=1000, hidden_size=2048, intermediate_size=512, num_layers=2, num_attention_heads=16,
          num_key_value_heads=2, max_positions=64, tie_word_embeddings=False, eos_token_ids=())
NORM_SEED = 17
CONFIGS = {"wide": WIDE, "g8": G8}


def random_norms(cfg: dict) -> dict:
    """name -> BF16 bits of random RMSNorm weights (1 + N(0, 0.25^2)) for every norm of the model."""
    import oracle
    rng = np.random.default_rng(NORM_SEED)
    H = cfg["hidden_size"]
    out = {"model.norm.weight": oracle.round_bf16((1 + 0.25 * rng.standard_normal(H)).astype(np.float32))}
    for l in range(cfg["num_layers"]):
        for n in ("input_layernorm", "post_attention_layernorm"):
            out[f"model.layers.{l}.{n}.weight"] = oracle.round_bf16((1 + 0.25 * rng.standard_normal(H)).astype(np.float32))
    return out


def _rank_main(rank, world, id_q, res_q, prompts, max_new, seed, peer, cfg):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "scala-torch_b200"), os.path.join(ROOT, "tests")]
    os.environ["STB_TP_PEER"] = "1" if peer else "0"
    os.environ["STB_PEER_WAIT_MS"] = "20000"
    os.environ["STB_SKINNY_MIN_WORK"] = "0"
    try:
        from llama_fixtures import TINY
        from scalatorch import ffm
        from scalatorch.models import BackendLlama, LlamaConfig
        if rank == 0:
            uid = ffm.B200Session.nccl_unique_id()
            for _ in range(world - 1):
                id_q.put(uid)
        else:
            uid = id_q.get(timeout=120)
        s = ffm.B200Session(rank, 1 << 30)
        s.init_tp(world, rank, uid)
        import ctypes
        enabled, elems = ctypes.c_int(), ctypes.c_uint64()
        ffm.library().stb_session_tp_peer.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        ffm.call("stb_session_tp_peer", s.handle, ctypes.byref(enabled), ctypes.byref(elems))
        assert bool(enabled.value) == peer, (enabled.value, peer)
        conf = TINY if cfg == "tiny" else CONFIGS[cfg]
        m = BackendLlama.prepare_random(s, LlamaConfig(**conf), seed=seed, tp_rank=rank, tp_size=world)
        if cfg == "g8":
            for name, bits in random_norms(conf).items():
                m.set_weight(name, bits, ffm.STB_BF16)
        out = m.generate_ids(np.array(prompts), max_new)
        single = m.generate_ids(prompts[0], max_new)
        m.close()
        s.close()
        res_q.put((rank, "ok", (out, single)))
    except Exception as e:  # reported to the parent, never swallowed
        res_q.put((rank, "error", repr(e)))


def _gpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("cfg", ["tiny", "wide", "g8"])
@pytest.mark.parametrize("peer", [True, False], ids=["nvlink-peer-exchange", "nccl-allreduce"])
def test_tp2_generation_matches_oracle(peer, cfg):
    from llama_fixtures import TINY, oracle_model
    from scalatorch.models import LlamaConfig
    ctx = mp.get_context("spawn")
    id_q, res_q = ctx.Queue(), ctx.Queue()
    prompts = [[5, 6, 7, 8], [900, 1, 2, 3]]
    procs = [ctx.Process(target=_rank_main, args=(r, 2, id_q, res_q, prompts, 12, 9, peer, cfg)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, status, payload = res_q.get(timeout=300)
            results[rank] = (status, payload)
    except queue.Empty:
        pass
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert set(results) == {0, 1}, f"ranks finished: {sorted(results)}"
    for rank, (status, payload) in results.items():
        assert status == "ok", f"rank {rank}: {payload}"
    conf = TINY if cfg == "tiny" else CONFIGS[cfg]
    ref = oracle_model(LlamaConfig(**conf), seed=9, replace=random_norms(conf) if cfg == "g8" else None)
    want = [ref.generate(p, 12) for p in prompts]
    for rank in (0, 1):
        batch_ids, single_ids = results[rank][1]
        assert batch_ids == want
        assert single_ids == want[0]
