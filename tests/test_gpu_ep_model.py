"""Expert-parallel LFM2-MoE model on 2 GPUs: each rank holds half of every MoE layer's experts
and decodes its own sequence; every MoE layer exchanges token rows over the library's NCCL
communicator (dispatch once per destination rank, grouped expert GEMMs on the owner, partial
sums back).  Each rank's batched prefill (prompt > 64 tokens), the logits after it and the next
greedy tokens match the oracle run with all experts (lfm2-engine.js:413-487)."""
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
        spec = qq3.synth.lfm2_8b_a1b(seed=83)
        spec.n_layers, spec.attn_layers, spec.n_expert = 4, (2,), 8
        g = qq3.synth.memory_model(spec)
        ctx = qq3.runtime.Context(rank)
        ctx.comm_init_from_torch(timeout_ms=60000)
        eng = qq3.Lfm2CudaEngine(g, ctx=ctx, max_ctx=96, ep_world=world)
        prompt = qq3.synth.uniform_tokens(72, 200 + rank, spec.n_vocab)  # each rank its own sequence
        eng.prefill(prompt[:-1].tolist())  # batched, with the expert exchange per MoE layer
        logits = eng.forward(int(prompt[-1]), 71, False).copy()
        toks = eng.model.decode_loop(int(np.argmax(logits)), 72, 6).tolist()
        ref = orc.OracleModel(g, max_ctx=96, threads=8)
        for p, t in enumerate(prompt[:-1]):
            ref.forward(int(t), p, True)
        want = ref.forward(int(prompt[-1]), 71, False)
        err = float(np.abs(logits - want).max() / np.abs(want).max())
        cur, pos, want_toks = int(np.argmax(want)), 72, []
        for _ in range(6):
            cur = int(np.argmax(ref.forward(cur, pos, False)))
            want_toks.append(cur)
            pos += 1
        q.put((rank, (err, int(np.argmax(logits)) == int(np.argmax(want)), toks == want_toks, toks, want_toks)))
        eng.close()
        dist.barrier()
        ctx.close()
        dist.destroy_process_group()
    except Exception as e:  # report instead of leaving the parent waiting
        import traceback

        q.put((rank, repr(e) + traceback.format_exc()))


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_model_two_gpus(qq3):
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
        err, same_argmax, same_tokens, got, want = res[r]
        assert err < 1e-2, (r, err)
        assert same_argmax and same_tokens, (r, got, want)
