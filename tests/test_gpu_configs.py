"""Parity of the benchmarked configurations themselves, run the way bench.py runs them.

* Benchmark config 4 (LFM2-8B-A1B shapes, all 24 layers, 32 experts): the 512-token prompt goes
  through the batched prefill (tensor-core projections, grouped MoE), then 128 greedy tokens come
  from the device decode loop -- bench.py's exact sequence of calls, seed and prompt.  The tokens
  must equal the CPU oracle's (the restated JS path, lfm2-engine.js:523-583 with thinking
  suppression, which is a no-op here: LFM2's think id is beyond this vocabulary).
* Benchmark config 5 at long context (Qwen3-8B widths, 2 of its 36 layers): 16 sequences with
  ragged prompts of 4096-4141 tokens, prefilled through the batched path, then multi-sequence
  decode steps past 4096 positions (beyond the reference's own 4096 cap, qwen3-engine.js:10,
  which is why the oracle's KV cache is uncapped), checked against the oracle.

Bars (north star): greedy tokens identical; logits within 1e-2 max relative error.
"""
import os

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2
SEED = 1234          # bench.py SEED
THINK_LFM2 = 124901  # bench.py THINK_ID (lfm2-engine.js:539)


def _threads():
    return max(1, os.cpu_count() or 1)


def _router_gap(g, spec, rec):
    """Smallest k-th vs (k+1)-th selection-score gap over the MoE layers of one oracle record."""
    gap = np.inf
    k = spec.n_expert_used
    for m, layer in enumerate([i for i in range(spec.n_layers) if spec.is_moe(i)]):
        bias = g.getTensorMetaByName(f"blk.{layer}.exp_probs_b.bias").raw().view(np.float32)
        sel = np.sort((rec[m][2 * k:] + bias).astype(np.float32))[::-1]
        gap = min(gap, float(sel[k - 1] - sel[k]))
    return gap


def test_lfm2_8b_a1b_config4_as_benched(qq3, orc):
    """512-token batched prefill + 128 greedy decode-loop tokens, token-exact against the oracle."""
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    g = qq3.synth.MemoryGGUF(spec, qq3.synth.build_tensors(spec))
    prompt = qq3.synth.uniform_tokens(512, SEED, spec.n_vocab)  # bench.py: seed SEED + rank, rank 0
    steps = 128
    suppress = THINK_LFM2 if THINK_LFM2 < spec.n_vocab else -1
    eng = qq3.Lfm2CudaEngine(g, device=0, max_ctx=512 + steps + 8)
    eng.prefill(prompt[:-1].tolist())  # 511 tokens: the batched tensor-core path (>= 64 tokens)
    got = eng.model.decode_loop(int(prompt[-1]), 511, steps, suppress_id=suppress).tolist()
    eng.close()

    ref = orc.OracleModel(g, max_ctx=512 + steps + 8, threads=_threads())
    gaps = []
    for p, t in enumerate(prompt[:-1]):
        _, _, rec = ref.forward(int(t), p, True, routing=True)
        gaps.append(_router_gap(g, spec, rec))
    want, top2 = [], []
    cur, pos = int(prompt[-1]), 511
    for _ in range(steps):
        logits, _, rec = ref.forward(cur, pos, False, routing=True)
        gaps.append(_router_gap(g, spec, rec))
        srt = np.sort(logits)
        top2.append(float(srt[-1] - srt[-2]) / max(float(np.abs(logits).max()), 1e-30))
        cur = int(np.argmax(logits))
        want.append(cur)
        pos += 1
    if got != want:
        first = next(i for i, (a, b) in enumerate(zip(got, want)) if a != b)
        pytest.fail(f"greedy tokens differ from step {first} on: got {got[first:first + 4]}, want "
                    f"{want[first:first + 4]}; smallest router gap in the prompt {min(gaps[:511]):.3e}, in the "
                    f"decode {min(gaps[511:]):.3e}; relative top-2 logit gap at that step {top2[first]:.3e}")


def test_qwen3_8b_width_long_context_batch(qq3, orc):
    """Config 5 at long context: 16 sequences, ragged 4096-4141-token prompts through the batched
    prefill, then three multi-sequence steps (each row attending 4096-4144 positions); sequence 0 (placed mid-batch)
    against the oracle's uncapped KV cache, every row's greedy id against its own logits."""
    spec = qq3.synth.qwen3_8b(seed=36)
    spec.n_layers = 2
    g = qq3.synth.memory_model(spec)
    n = 16
    lens = [4096 + 3 * s for s in range(n)]
    max_ctx = max(lens) + 8
    eng = qq3.engine_for(g, device=0, max_ctx=max_ctx, n_seq=n)
    prompts = [qq3.synth.uniform_tokens(L, 500 + s, spec.n_vocab) for s, L in enumerate(lens)]
    for s in range(n):
        eng.prefill(prompts[s][:-1].tolist(), pos0=0, seq=s)
    order = [5, 11, 2, 14, 0, 7, 9, 1, 15, 3, 12, 6, 10, 4, 13, 8]  # sequence 0 is row 4
    cur = {s: int(prompts[s][-1]) for s in range(n)}
    pos = {s: lens[s] - 1 for s in range(n)}
    ref = orc.OracleModel(g, max_ctx=max_ctx, threads=_threads())
    for p, t in enumerate(prompts[0][:-1]):
        ref.forward(int(t), p, True)
    for step in range(3):
        logits, am = eng.forward_batch(order, [cur[s] for s in order], [pos[s] for s in order])
        for i, s in enumerate(order):
            assert np.isfinite(logits[i]).all(), f"step {step}, sequence {s}: non-finite logits"
            assert int(am[i]) == int(np.argmax(logits[i])), f"step {step}, sequence {s}: device argmax"
        i0 = order.index(0)
        want = ref.forward(cur[0], pos[0], False)
        assert rel_err(logits[i0], want) < TOL, f"step {step} (position {pos[0]}): logits vs oracle"
        assert int(am[i0]) == int(np.argmax(want)), f"step {step} (position {pos[0]}): greedy id vs oracle"
        for i, s in enumerate(order):
            cur[s] = int(am[i])
            pos[s] += 1
    eng.close()
