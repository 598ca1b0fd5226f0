"""Next-token sampling on the device (qq_sample_logits, qq_forward_sample, qq_generate_sample)
against the JS sampling loops (tensor.js:188-265) on the same uniform draws.

The reference draws Math.random(); the device draws r = sample_uniform(seed, sequence, position)
and the host reproduces every draw, so the comparison is exact: the same token id for the same r.
"""
import numpy as np
import pytest

from test_host import _js_top_p_top_k

pytestmark = pytest.mark.gpu


def _js_think(logits, temperature, top_p, top_k, mode, think_id, end_id, done, r):
    """sampleWithThinkControl (tensor.js:244-265) with Math.random() = r."""
    x = np.asarray(logits, np.float32).copy()
    n = len(x)
    if mode == "suppress" and 0 <= think_id < n:
        x[think_id] = -np.inf
    elif mode == "shorten" and not done and 0 <= end_id < n:
        end = x[end_id]
        if int(np.count_nonzero(x > end)) < top_k:
            return end_id
    if temperature <= 0:
        return int(np.argmax(x)) if not np.isnan(x[0]) else 0
    return _js_top_p_top_k(x, temperature, top_p, top_k, r)


def test_sample_logits_matches_js_loops(qq3, gpu_ctx, torch):
    rt = qq3.runtime
    rng = np.random.default_rng(5)
    cases = 0
    for n in (7, 1000, 65536, 151936):
        for trial in range(10 if n > 1000 else 25):
            scale = float(rng.choice([0.5, 2.0, 6.0]))
            logits = (rng.standard_normal(n) * scale).astype(np.float32)
            if trial % 4 == 1:
                logits = np.round(logits * 2) / 2  # many exact ties
            if trial % 7 == 3:
                logits[rng.integers(0, n, 3)] = -np.inf
            t = float(rng.choice([0.0, 0.3, 0.7, 1.0, 2.0]))
            top_p = float(rng.choice([0.5, 0.9, 0.95, 1.0]))
            top_k = int(rng.choice([1, 2, 40, 1000, 1024]))
            mode = ["suppress", "shorten", "full"][trial % 3]
            think_id, end_id = int(rng.integers(0, n)), int(rng.integers(0, n))
            done = bool(trial % 2)
            r = float(rng.random()) if trial % 9 else (0.0 if trial % 2 else 0.999999)
            want = _js_think(logits, t, top_p, top_k, mode, think_id, end_id, done, r)
            p = rt.sample_params(t, top_p, top_k, mode, think_id, end_id, seed=0)
            got = gpu_ctx.sample_logits(torch.from_numpy(logits).cuda(), n, p, r, done)
            assert got == want, (n, trial, t, top_p, top_k, mode, r)
            cases += 1
    assert cases == 70


def test_sample_refuses_unserved_options(qq3, gpu_ctx, torch):
    x = torch.zeros(16, device="cuda")
    for k in (0, 1025):
        with pytest.raises(qq3.runtime.QQError):
            gpu_ctx.sample_logits(x, 16, qq3.runtime.sample_params(0.7, 0.9, k), 0.5)


@pytest.mark.parametrize("arch", ["lfm2", "qwen3"])
def test_generate_sample_matches_oracle_with_js_sampler(qq3, orc, arch):
    """Sampled generate() on the device -- the whole continuation as device steps with the sampler
    in the step's graph -- gives the tokens the oracle's logits give through the JS sampling loops
    with the same draws; the host-driven engine loop (qq_forward_sample per token) gives them too."""
    spec = qq3.synth.tiny_lfm2(seed=61) if arch == "lfm2" else qq3.synth.tiny_qwen3(seed=61)
    g = qq3.synth.memory_model(spec)
    eng = qq3.engine_for(g, device=0, max_ctx=64)
    ref = orc.OracleModel(g, max_ctx=64, threads=8)
    prompt = qq3.synth.uniform_tokens(6, 13, spec.n_vocab).tolist()
    seed, steps = 0xC0FFEE1234, 24
    for t, top_p, top_k, mode in ((0.8, 0.9, 40, "suppress"), (1.5, 0.95, 1000, "full"), (0.0, 0.9, 5, "shorten")):
        params = qq3.runtime.sample_params(t, top_p, top_k, mode, eng.THINK_ID, eng.END_THINK_ID, seed)
        got = eng.model.generate_sample(prompt, steps, params).tolist()
        # oracle logits + the JS loops, draws r = sample_uniform(seed, 0, position of the logits)
        ref.reset()
        for p, tok in enumerate(prompt[:-1]):
            ref.forward(tok, p, True)
        done = mode == "suppress"
        cur, pos, want = prompt[-1], len(prompt) - 1, []
        nxt = None
        for s in range(steps + 1):
            logits = ref.forward(cur, pos, False)
            nxt = _js_think(logits, t, top_p, top_k, mode, eng.THINK_ID, eng.END_THINK_ID, done,
                            qq3.runtime.sample_uniform(seed, 0, pos))
            if s == steps:
                break
            want.append(nxt)
            if nxt == eng.END_THINK_ID:
                done = True
            cur, pos = nxt, pos + 1
        assert got == want, (arch, t, top_p, top_k, mode)
        # the engine's host loop with device sampling per token
        got2 = eng.generate(prompt, maxSteps=steps, temperature=t, topP=top_p, topK=top_k, thinkingMode=mode,
                            seed=seed)
        stop = next((i for i, v in enumerate(want) if v == eng.eosTokenId), len(want))
        assert got2 == want[:stop]
    eng.close()
