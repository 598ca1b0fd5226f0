"""Expert-parallel MoE exchange (qwenqwen3.js_b200/ep.py) on CPU: gloo ranks, a toy MoE whose
experts are elementwise functions, checked on every rank against the unsharded block."""
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent
N_EXPERT, TOP_K, K = 8, 4, 16


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _toy(seed, T):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32))
    # distinct experts per token (as a top-k gives), weights summing to 1
    idx = torch.from_numpy(np.stack([rng.permutation(N_EXPERT)[:TOP_K] for _ in range(T)]).astype(np.int32))
    w = torch.from_numpy(rng.dirichlet(np.ones(TOP_K), size=T).astype(np.float32))
    return x, idx, w


def _expert(e, rows):  # a different elementwise function per global expert id
    return torch.tanh(rows * (e + 1) / 4.0) + 0.1 * e


def _worker(rank, world, port, T, q):
    try:
        if str(ROOT) not in sys.path:
            sys.path.insert(0, str(ROOT))
        import torch.distributed as dist

        from __graft_entry__ import load_package

        ep = load_package().ep
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        x, idx, w = _toy(100 + rank, T + 3 * rank)  # ragged: the ranks own different token counts
        n_local = N_EXPERT // world

        def experts(rows, eid):
            out = torch.empty_like(rows)
            for r in range(rows.shape[0]):
                out[r] = _expert(rank * n_local + int(eid[r]), rows[r])
            return out

        def combine(rows, pos, ww):
            return (ww.unsqueeze(-1) * rows[pos.long()]).sum(1)

        got = ep.ep_forward(x, lambda xx: (idx, w), experts, combine, N_EXPERT, TOP_K)
        want = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for s in range(TOP_K):
                want[t] += w[t, s] * _expert(int(idx[t, s]), x[t])
        q.put((rank, float((got - want).abs().max())))
        dist.destroy_process_group()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_gloo(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 5, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-6, res[r]


def test_plan_dispatch_positions(qq3):
    _, idx, _ = _toy(5, 9)
    order, counts, pos, eid = qq3.ep.plan_dispatch(idx, 2, 4)
    flat = idx.reshape(-1).long()
    assert counts.tolist() == np.bincount((flat // 2).numpy(), minlength=4).tolist()
    # pos inverts order; destinations never decrease along order; eid is the destination-local id
    assert torch.equal(order[pos.reshape(-1).long()], torch.arange(flat.numel()))
    assert bool(((flat[order] // 2)[1:] >= (flat[order] // 2)[:-1]).all())
    assert torch.equal(eid.long(), flat[order] % 2)


def test_expert_slice_bytes(qq3):
    K, N, E = 64, 3, 4
    stride = N * (K // 32) * 34
    raw = np.arange(E * stride, dtype=np.int64).astype(np.uint8)
    part, ne = qq3.ep.expert_slice(raw, [K, N, E], 1, 2)
    assert ne == [K, N, 2] and part.nbytes == 2 * stride
    assert np.array_equal(part, raw[stride:3 * stride])
