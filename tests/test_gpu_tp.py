"""Tensor-parallel dense Qwen3 on GPUs (qwenqwen3.js_b200/tp.py, GPURank): the per-rank token
step bound to the library's kernels (Q8_0 GEMVs, RMSNorm, RoPE, split attention over the rank's
K/V cache, SwiGLU, residual add) against the unsharded CPU oracle (qwen3-engine.js:115-301):
logits within 1e-2 max relative error, greedy ids identical.  World 1 runs on one GPU (every
step on the device, no exchange); world 2 adds the NCCL all-reduces and needs two GPUs."""
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
TOL = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_rank(qq3, orc, rank, world, device, gather_pairs, gather_logits):
    """Five tokens of a seeded tiny Qwen3 (one without logits) on this rank; returns the worst
    logits error against the oracle and the number of greedy-id mismatches."""
    spec = qq3.synth.tiny_qwen3(seed=41)
    g = qq3.synth.memory_model(spec)
    plan = qq3.tp.TPPlan(spec.n_head, spec.n_head_kv, spec.head_dim, spec.n_embd, spec.n_ff, spec.n_vocab, world,
                         rank)
    ctx = qq3.runtime.Context(device)
    stream = torch.cuda.Stream(device=device)
    r = qq3.tp.GPURank(ctx, plan, qq3.tp.shard_model(g, plan), spec.head_dim, spec.rope_base, 8, spec.n_layers,
                       stream)
    ops = r.ops()
    ref = orc.OracleModel(g, max_ctx=8)
    worst, mismatches = 0.0, 0
    with torch.cuda.stream(stream):
        for p, t in enumerate(qq3.synth.uniform_tokens(5, 17, spec.n_vocab)):
            skip = p == 1
            logits, greedy = qq3.tp.tp_forward(int(t), p, plan, r.shards, ops, spec.eps, spec.n_layers,
                                               r.nccl_all_reduce, gather_pairs, want_logits=not skip)
            want = ref.forward(int(t), p, skip)
            if skip:
                continue
            full = gather_logits(logits)
            worst = max(worst, float(np.abs(full - want).max() / np.abs(want).max()))
            mismatches += int(greedy != orc.sample_greedy(want))
    stream.synchronize()
    r.close()
    ctx.close()
    return worst, mismatches


def test_tp_gpu_world1_vs_oracle(qq3, orc):
    worst, mismatches = _run_rank(qq3, orc, 0, 1, 0, lambda pair: [pair], lambda x: x)
    assert worst < TOL, f"logits rel err {worst:.3e}"
    assert mismatches == 0


def _worker(rank, world, port, q):
    try:
        if str(ROOT) not in sys.path:
            sys.path.insert(0, str(ROOT))
        import datetime
        import os

        import torch.distributed as dist

        from __graft_entry__ import load_oracle, load_package

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        qq3, orc = load_package(), load_oracle()
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))

        def gather_pairs(pair):
            out = [None] * world
            dist.all_gather_object(out, pair)
            return out

        def gather_logits(x):
            out = [None] * world
            dist.all_gather_object(out, x)
            return np.concatenate(out)

        q.put((rank, _run_rank(qq3, orc, rank, world, rank, gather_pairs, gather_logits)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_gpu_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], tuple), res[r]
        worst, mismatches = res[r]
        assert worst < TOL, f"rank {r}: logits rel err {worst:.3e}"
        assert mismatches == 0, f"rank {r}: greedy ids differ"
