"""Tensor-parallel dense Qwen3 (qwenqwen3.js_b200/tp.py) on CPU: gloo ranks that each hold
their shards of a seeded Qwen3 model and run its layers with the CPU oracle's arithmetic and the
two all-reduces and the greedy-id gather of the tensor-parallel step; checked against the
unsharded oracle model (qwen3-engine.js:115-301): logits within 1e-2 max relative error, greedy
ids identical."""
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent
TOL = 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spec(qq3, world):
    if world == 2:
        return qq3.synth.tiny_qwen3(seed=41)  # 4 query / 2 KV heads of 128, FFN 512, vocab 1024
    # 8 query / 4 KV heads of 64, so that 4 ranks own one KV head each
    return qq3.synth.ModelSpec("qwen3", 2, 256, 8, 4, 64, 1000, 512, 1e6, 1e-6, seed=43, name="tiny-qwen3-tp4")


def _oracle_ops(orc, tp, plan, shards, hd, base, max_ctx, n_layers):
    """TPOps backed by the CPU restatement; attention as _selfAttentionCore (qwen3-engine.js:249-291)
    over this rank's heads with a local K/V cache."""
    nq, nkv = len(plan.q_heads), len(plan.kv_heads)
    kc = np.zeros((n_layers, nkv, max_ctx, hd), np.float32)
    vc = np.zeros_like(kc)
    emb = shards["token_embd.weight"]

    def f32w(entry):
        return np.asarray(entry[2]).view(np.float32)

    def attention(layer, pos, q):
        out = np.zeros(nq * hd, np.float32)
        for j, h in enumerate(plan.q_heads):
            kv = h * plan.n_kv // plan.n_head - plan.kv_heads.start  # GQA map (qwen3-engine.js:260)
            qh = q[j * hd:(j + 1) * hd].astype(np.float64)
            scores = (kc[layer, kv, :pos + 1].astype(np.float64) @ qh).astype(np.float32) * np.float32(1 / np.sqrt(hd))
            w = orc.softmax(scores.astype(np.float32))
            acc = np.zeros(hd, np.float32)
            for p in range(pos + 1):
                if w[p] != 0:
                    acc += vc[layer, kv, p] * w[p]
            out[j * hd:(j + 1) * hd] = acc
        return out

    def kv_store(layer, pos, k, v):
        kc[layer, :, pos] = k.reshape(nkv, hd)
        vc[layer, :, pos] = v.reshape(nkv, hd)

    return tp.TPOps(
        embed=lambda t: orc.embedding(emb[2], emb[1], t),
        rmsnorm=lambda x, e, eps: orc.rmsnorm(x, f32w(e), eps),
        matmul=lambda e, x: orc.matmul(e[2], e[0], e[1], np.asarray(x, np.float32)[None, :])[0],
        head_rmsnorm=lambda x, n, e, eps: orc.rmsnorm(np.asarray(x).reshape(n, hd), f32w(e), eps).reshape(-1),
        rope=lambda x, n, pos: orc.rope(x, n, hd, pos, base),
        kv_store=kv_store,
        attention=attention,
        silu_mul=lambda g, u: (orc.silu(g) * np.asarray(u, np.float32)).astype(np.float32),
        add=lambda a, b: (a + b).astype(np.float32),
        to_host=lambda a: np.asarray(a, np.float32),
    )


def _worker(rank, world, port, q):
    try:
        if str(ROOT) not in sys.path:
            sys.path.insert(0, str(ROOT))
        import torch.distributed as dist

        from __graft_entry__ import load_oracle, load_package

        qq3 = load_package()
        orc = load_oracle()
        orc.set_threads(1)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        spec = _spec(qq3, world)
        g = qq3.synth.memory_model(spec)
        plan = qq3.tp.TPPlan(spec.n_head, spec.n_head_kv, spec.head_dim, spec.n_embd, spec.n_ff, spec.n_vocab, world,
                             rank)
        shards = qq3.tp.shard_model(g, plan)
        max_ctx = 8
        ops = _oracle_ops(orc, qq3.tp, plan, shards, spec.head_dim, spec.rope_base, max_ctx, spec.n_layers)

        def all_reduce(x):
            t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def gather_pairs(pair):
            out = [None] * world
            dist.all_gather_object(out, pair)
            return out

        ref = orc.OracleModel(g, max_ctx=max_ctx)
        toks = qq3.synth.uniform_tokens(5, 17, spec.n_vocab)
        worst, mismatches = 0.0, 0
        for p, t in enumerate(toks):
            skip = p == 1  # one prefill-style step without logits
            logits, greedy = qq3.tp.tp_forward(int(t), p, plan, shards, ops, spec.eps, spec.n_layers, all_reduce,
                                               gather_pairs, want_logits=not skip)
            want = ref.forward(int(t), p, skip)
            if skip:
                continue
            parts = [None] * world
            dist.all_gather_object(parts, logits)
            full = np.concatenate(parts)
            worst = max(worst, float(np.abs(full - want).max() / np.abs(want).max()))
            mismatches += int(greedy != orc.sample_greedy(want))
        q.put((rank, (worst, mismatches)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_qwen3_gloo(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], tuple), res[r]
        worst, mismatches = res[r]
        assert worst < TOL, f"rank {r}: logits rel err {worst:.3e}"
        assert mismatches == 0, f"rank {r}: greedy ids differ"


def test_q8_shards_reassemble(qq3):
    """Row shards concatenate to the tensor; column shards interleave back block by block."""
    K, N = 96, 5
    raw = qq3.synth.q8_0_blocks(K * N, seed=3)
    rows = [qq3.tp.q8_rows(raw, K, a, b) for a, b in ((0, 2), (2, 5))]
    assert np.array_equal(np.concatenate(rows), raw)
    cols = [qq3.tp.q8_cols(raw, K, N, a, b).reshape(N, -1, 34) for a, b in ((0, 32), (32, 96))]
    assert np.array_equal(np.concatenate(cols, axis=1).reshape(-1), raw)
    with pytest.raises(ValueError):
        qq3.tp.q8_cols(raw, K, N, 16, 48)


def test_merge_greedy_is_sample_greedy(qq3):
    """The merged id equals sampleGreedy on the whole row (tensor.js:231-237): ties across shard
    boundaries go to the lower index, NaN never wins, a NaN first logit wins outright."""
    rng = np.random.default_rng(5)
    tp = qq3.tp

    def js_greedy(x):
        m = 0
        for i in range(1, len(x)):
            if x[i] > x[m]:
                m = i
        return m

    cases = []
    for _ in range(40):
        x = rng.integers(-3, 4, size=37).astype(np.float32)  # many equal values: ties everywhere
        if rng.random() < 0.3:
            x[rng.integers(0, 37, size=3)] = np.nan
        cases.append(x)
    tie = np.zeros(37, np.float32)
    tie[20] = tie[5] = 2.0
    cases += [tie, np.full(37, np.nan, np.float32)]
    first_nan = np.arange(37, dtype=np.float32)
    first_nan[0] = np.nan
    cases.append(first_nan)
    for x in cases:
        for world in (1, 2, 3, 4):
            v = [r * len(x) // world for r in range(world + 1)]
            pairs = [tp.local_greedy(x[v[r]:v[r + 1]], v[r]) for r in range(world)]
            assert tp.merge_greedy(pairs) == js_greedy(x), (x, world)


def test_plan_checks(qq3):
    tp = qq3.tp
    p = tp.TPPlan(32, 8, 128, 4096, 12288, 151936, 8, 3)  # Qwen3-8B at 8 ranks
    assert p.q_heads == range(12, 16) and p.kv_heads == range(3, 4) and p.ff_units == range(4608, 6144)
    assert p.vocab_offsets()[-1] == 151936 and p.vocab_rows == range(56976, 75968)
    with pytest.raises(ValueError):
        tp.TPPlan(16, 8, 128, 1024, 3072, 151936, 16, 0)  # 8 KV heads over 16 ranks
    with pytest.raises(ValueError):
        tp.TPPlan(16, 8, 128, 1024, 3000, 151936, 2, 0)  # FFN not in whole blocks per rank
