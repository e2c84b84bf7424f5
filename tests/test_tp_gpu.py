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


# Wide enough that every projection of a 2-row decode step takes the tensor-core skinny form
# (local N >= 128), including the row-split o / down projections with the peer-exchange epilogue.
WIDE = dict(vocab_size=1000, hidden_size=256, intermediate_size=512, num_layers=2, num_attention_heads=8,
            num_key_value_heads=4, max_positions=64, tie_word_embeddings=False, eos_token_ids=())


def _rank_main(rank, world, id_q, res_q, prompts, max_new, seed, peer, cfg):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "scala-torch_b200"), os.path.join(ROOT, "tests")]
    os.environ["STB_TP_PEER"] = "1" if peer else "0"
    os.environ["STB_PEER_WAIT_MS"] = "20000"
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
        m = BackendLlama.prepare_random(s, LlamaConfig(**(TINY if cfg == "tiny" else WIDE)), seed=seed,
                                        tp_rank=rank, tp_size=world)
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
@pytest.mark.parametrize("cfg", ["tiny", "wide"])
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
    ref = oracle_model(LlamaConfig(**(TINY if cfg == "tiny" else WIDE)), seed=9)
    want = [ref.generate(p, 12) for p in prompts]
    for rank in (0, 1):
        batch_ids, single_ids = results[rank][1]
        assert batch_ids == want
        assert single_ids == want[0]
