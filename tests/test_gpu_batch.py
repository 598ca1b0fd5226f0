"""Multi-sequence decode (qq_forward_batch): one step of several independent sequences at once.

The reference serves one sequence per engine; a batched step must give each sequence what n
separate forward() calls give it (qwen3-engine.js:115-245, lfm2-engine.js:228-269).  Checked
against the CPU oracle run sequence by sequence, and against the engine's own per-token decode
steps at Qwen3-8B widths (the 16-sequence decode of that configuration).  Bars as everywhere:
logits within 1e-2 max relative error, greedy ids identical, router top-k identical except
near-ties (selection-score gap < 1e-5).
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _router_gap(g, spec, rec):
    """Smallest k-th vs (k+1)-th selection-score gap over the MoE layers of one oracle record."""
    gap = np.inf
    k = spec.n_expert_used
    for m, layer in enumerate([i for i in range(spec.n_layers) if spec.is_moe(i)]):
        bias = g.getTensorMetaByName(f"blk.{layer}.exp_probs_b.bias").raw().view(np.float32)
        sel = np.sort((rec[m][2 * k:] + bias).astype(np.float32))[::-1]
        gap = min(gap, float(sel[k - 1] - sel[k]))
    return gap


@pytest.mark.parametrize("arch", ["qwen3", "lfm2"])
def test_forward_batch_vs_oracle(qq3, orc, arch):
    """Four sequences with ragged prompts decode together; one step runs a subset of them out of
    order; the last step of sequence 0 goes through the per-token path, which must continue from
    the state the batched steps left (K/V rows, conv state)."""
    spec = qq3.synth.tiny_lfm2(seed=31) if arch == "lfm2" else qq3.synth.tiny_qwen3(seed=31)
    n_seq = 4
    g = qq3.synth.memory_model(spec)
    eng = qq3.engine_for(g, device=0, max_ctx=32, n_seq=n_seq)
    refs = [orc.OracleModel(g, max_ctx=32, threads=8) for _ in range(n_seq)]
    cur, pos = [], []
    for s, n in enumerate([3, 6, 1, 4]):
        toks = qq3.synth.uniform_tokens(n, 40 + s, spec.n_vocab)
        if n > 1:
            eng.prefill(toks[:-1].tolist(), pos0=0, seq=s)
            for p, t in enumerate(toks[:-1]):
                refs[s].forward(int(t), p, True)
        cur.append(int(toks[-1]))
        pos.append(n - 1)
    exempt = set()  # sequences whose routing met a near-tie: their states may differ from here on
    k, E = spec.n_expert_used, spec.n_expert
    for step in range(5):
        rows = [3, 1] if step == 2 else list(range(n_seq))
        logits, am = eng.forward_batch(rows, [cur[s] for s in rows], [pos[s] for s in rows])
        assert logits.shape == (len(rows), spec.n_vocab)
        for i, s in enumerate(rows):
            want, _, rec = refs[s].forward(cur[s], pos[s], False, routing=True)
            if arch == "lfm2" and _router_gap(g, spec, rec) < 1e-5:
                exempt.add(s)
            if s not in exempt:
                assert rel_err(logits[i], want) < TOL, f"step {step}, sequence {s}: logits"
                assert int(am[i]) == int(np.argmax(want)), f"step {step}, sequence {s}: greedy id"
                assert int(am[i]) == int(np.argmax(logits[i]))
            if arch == "lfm2" and i == len(rows) - 1 and s not in exempt:
                # the routing record kept for onRouterUpdate is the last row's
                for m in range(rec.shape[0]):
                    got = eng.model.read_routing(m, 2 * k + E)
                    assert np.array_equal(got[:k], rec[m][:k]), f"step {step}: routing ids, moe layer {m}"
                    assert rel_err(got[2 * k:], rec[m][2 * k:]) < 1e-3
            cur[s] = int(np.argmax(want))  # teacher forcing: both sides see the oracle's ids
            pos[s] += 1
    got = eng.forward(cur[0], pos[0], False)
    want = refs[0].forward(cur[0], pos[0], False)
    if 0 not in exempt:
        assert rel_err(got, want) < TOL
        assert int(np.argmax(got)) == int(np.argmax(want))
    eng.close()


def test_forward_batch_skip_logits_and_errors(qq3):
    """skipLogits steps advance the state like forward(t, pos, true); a sequence named twice, an
    id beyond n_seq or a position beyond the KV capacity is refused before any work."""
    spec = qq3.synth.tiny_qwen3(seed=33)
    g = qq3.synth.memory_model(spec)
    eng = qq3.engine_for(g, device=0, max_ctx=16, n_seq=3)
    toks = qq3.synth.uniform_tokens(6, 77, spec.n_vocab)
    # sequences 0 and 1 get the same tokens: 0 by batched skip-logit steps, 1 by per-token steps
    for p in range(3):
        assert eng.forward_batch([0, 2], [int(toks[p]), int(toks[5 - p])], [p, p], skipLogits=True) == (None, None)
        eng.forward(int(toks[p]), p, True, seq=1)
    a, _ = eng.forward_batch([0], [int(toks[3])], [3])
    b = eng.forward(int(toks[3]), 3, False, seq=1)
    assert rel_err(a[0], b) < TOL and int(np.argmax(a[0])) == int(np.argmax(b))
    for bad in (([0, 0], [1, 2], [4, 4]), ([3], [1], [0]), ([1], [1], [16])):
        with pytest.raises(RuntimeError):
            eng.forward_batch(*bad)
    eng.close()


def test_forward_batch_qwen3_8b_width_16_sequences(qq3, orc):
    """Qwen3-8B widths (hidden 4096, 32/8 heads of 128, FFN 12288, vocab 151936, untied output),
    two layers, 16 sequences at mixed positions: the batched steps against the same sequences run
    by the per-token decode step (sequences 16..31 of the same engine), and four of them against
    the oracle."""
    spec = qq3.synth.qwen3_8b(seed=35)
    spec.n_layers = 2
    g = qq3.synth.memory_model(spec)
    n = 16
    eng = qq3.engine_for(g, device=0, max_ctx=8, n_seq=2 * n)
    checked = (0, 5, 10, 15)
    refs = {s: orc.OracleModel(g, max_ctx=8, threads=8) for s in checked}
    cur, pos = [], []
    for s in range(n):
        toks = qq3.synth.uniform_tokens(1 + s % 3, 60 + s, spec.n_vocab)
        for p, t in enumerate(toks[:-1]):
            eng.forward(int(t), p, True, seq=s)
            eng.forward(int(t), p, True, seq=n + s)
            if s in refs:
                refs[s].forward(int(t), p, True)
        cur.append(int(toks[-1]))
        pos.append(len(toks) - 1)
    for step in range(2):
        logits, am = eng.forward_batch(list(range(n)), cur, pos)
        for s in range(n):
            single = eng.forward(cur[s], pos[s], False, seq=n + s)
            assert rel_err(logits[s], single) < TOL, f"step {step}, sequence {s}: batched vs per-token"
            assert int(am[s]) == int(np.argmax(single)), f"step {step}, sequence {s}: greedy id"
            if s in refs:
                want = refs[s].forward(cur[s], pos[s], False)
                assert rel_err(logits[s], want) < TOL, f"step {step}, sequence {s}: vs oracle"
                assert int(am[s]) == int(np.argmax(want))
            cur[s] = int(am[s])
            pos[s] += 1
    eng.close()


@pytest.mark.parametrize("arch", ["qwen3", "lfm2"])
def test_forward_batch_long_context(qq3, orc, arch):
    """Rows at 40, 150 and 90 positions: the batched attention splits positions over CTAs (64 per
    split) and merges the splits, for head_dim 128 (Qwen3) and 64 (LFM2)."""
    spec = qq3.synth.tiny_lfm2(seed=37) if arch == "lfm2" else qq3.synth.tiny_qwen3(seed=37)
    g = qq3.synth.memory_model(spec)
    lens = [40, 150, 90]
    eng = qq3.engine_for(g, device=0, max_ctx=160, n_seq=len(lens))
    refs = [orc.OracleModel(g, max_ctx=160, threads=8) for _ in lens]
    cur, pos = [], []
    for s, n in enumerate(lens):
        toks = qq3.synth.uniform_tokens(n, 90 + s, spec.n_vocab)
        for p, t in enumerate(toks[:-1]):  # per-token steps: no batched prefill in this test
            eng.forward(int(t), p, True, seq=s)
            refs[s].forward(int(t), p, True)
        cur.append(int(toks[-1]))
        pos.append(n - 1)
    exempt = set()
    for step in range(3):
        logits, am = eng.forward_batch([0, 1, 2], cur, pos)
        for s in range(len(lens)):
            want, _, rec = refs[s].forward(cur[s], pos[s], False, routing=True)
            if arch == "lfm2" and _router_gap(g, spec, rec) < 1e-5:
                exempt.add(s)
            if s not in exempt:
                assert rel_err(logits[s], want) < TOL, f"step {step}, sequence {s}: logits"
                assert int(am[s]) == int(np.argmax(want)), f"step {step}, sequence {s}: greedy id"
            cur[s] = int(np.argmax(want))
            pos[s] += 1
    eng.close()
