"""Expert-parallel LFM2-MoE block on 2 GPUs (NCCL all-to-all dispatch/combine, experts sharded):
every rank's output matches the single-GPU block (all experts) on the same token rows."""
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


def _worker(rank, world, port, T, q):
    try:
        if str(ROOT) not in sys.path:
            sys.path.insert(0, str(ROOT))
        import datetime
        import os

        import torch.distributed as dist

        from __graft_entry__ import load_package

        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        qq3 = load_package()
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        spec = qq3.synth.lfm2_8b_a1b(seed=61)
        spec.n_expert = 8
        prefix = "blk.2."
        names = {prefix + n for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                      "ffn_down_exps.weight", "exp_probs_b.bias")}
        tensors = qq3.synth.build_tensors(spec, only=names)
        ctx = qq3.runtime.Context(rank)
        block = qq3.ep.EPMoEBlock(ctx, tensors, prefix, spec.n_expert, 4, rank, world)
        Tr = T + 7 * rank  # ragged token counts per rank
        x = torch.from_numpy(qq3.synth.normal_f32(Tr * 2048, seed=40 + rank).reshape(Tr, 2048)).cuda()
        got = block.forward(x)
        torch.cuda.synchronize()
        # the unsharded block on this rank (all experts)
        full = qq3.runtime.LayerDesc()
        full.is_moe = 1
        keep = []
        for slot in ("ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps", "exp_probs_b"):
            t, ne, raw = tensors[prefix + qq3.runtime.SLOT_TENSOR_NAMES[slot]]
            h = ctx.upload(raw, t, ne)
            keep.append(h)
            full.t[qq3.runtime.SLOT[slot]] = h.h.value
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        want = torch.empty_like(x)
        ctx.moe_block(full, spec.n_expert, 4, x, Tr, want)
        torch.cuda.synchronize()
        err = float((got - want).abs().max() / want.abs().max())
        q.put((rank, err))
        for h in keep:
            h.free()
        block.close()
        dist.barrier()
        dist.destroy_process_group()
        ctx.close()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_moe_block_two_gpus(qq3):
    import torch.multiprocessing as mp

    qq3.build.build_all()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, 48, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-4, res[r]
