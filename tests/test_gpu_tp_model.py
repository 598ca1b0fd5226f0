"""Tensor-parallel dense Qwen3 inside the library on 2 GPUs: each rank holds its heads, FFN units
and vocab rows (tp.shard_model); the wo and ffn_down partial sums are all-reduced over the
library's NCCL communicator and the greedy id is the first maximum over the vocab shards
(qwen3-engine.js:115-245, tensor.js:231-237).  A batched prefill, then multi-sequence steps of
4 sequences, against the oracle with the whole model: logits within 1e-2, greedy ids identical."""
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        if str(ROOT) not in sys.path:
            sys.path.insert(0, str(ROOT))
        import datetime
        import os

        import torch.distributed as dist

        from __graft_entry__ import load_oracle, load_package

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        qq3 = load_package()
        orc = load_oracle()
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        spec = qq3.synth.qwen3_0p6b(seed=47)
        spec.n_layers = 3
        g = qq3.synth.memory_model(spec)
        ctx = qq3.runtime.Context(rank)
        ctx.comm_init_from_torch(timeout_ms=60000)
        n = 4
        eng = qq3.Qwen3CudaEngine(g, ctx=ctx, max_ctx=96, n_seq=n, tp_world=world)
        refs = [orc.OracleModel(g, max_ctx=96, threads=4) for _ in range(n)]
        cur, pos = [], []
        worst = 0.0
        for s in range(n):  # the same sequences on every rank (their shards of the same work)
            toks = qq3.synth.uniform_tokens(70 + 3 * s, 300 + s, spec.n_vocab)
            got = eng.forward(int(toks[0]), 0, False).copy() if s == 0 else None  # one-row step, logits
            if s == 0:
                want = refs[0].forward(int(toks[0]), 0, False)
                worst = max(worst, float(np.abs(got - want).max() / np.abs(want).max()))
                assert int(np.argmax(got)) == int(np.argmax(want))
                eng.prefill(toks[1:-1].tolist(), pos0=1, seq=0)
                for p, t in enumerate(toks[1:-1]):
                    refs[0].forward(int(t), p + 1, True)
            else:
                eng.prefill(toks[:-1].tolist(), pos0=0, seq=s)
                for p, t in enumerate(toks[:-1]):
                    refs[s].forward(int(t), p, True)
            cur.append(int(toks[-1]))
            pos.append(len(toks) - 1)
        ok = True
        for step in range(3):
            logits, am = eng.forward_batch(list(range(n)), cur, pos)
            for s in range(n):
                want = refs[s].forward(cur[s], pos[s], False)
                worst = max(worst, float(np.abs(logits[s] - want).max() / np.abs(want).max()))
                ok = ok and int(am[s]) == int(np.argmax(want)) == int(np.argmax(logits[s]))
                cur[s] = int(np.argmax(want))
                pos[s] += 1
        q.put((rank, (worst, ok)))
        eng.close()
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
    except Exception as e:  # report instead of leaving the parent waiting
        import traceback

        q.put((rank, repr(e) + traceback.format_exc()))


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_model_two_gpus(qq3):
    import torch.multiprocessing as mp

    qq3.build.build_all()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert isinstance(res[r], tuple), res[r]
        worst, ok = res[r]
        assert worst < 1e-2, (r, worst)
        assert ok, r
