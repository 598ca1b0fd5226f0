"""Host-side logic and the C ABI boundary, without a GPU."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_library_exports_every_declared_symbol(qq3):
    qq3.build.build_cuda()
    header = (ROOT / "include" / "qq3.h").read_text()
    declared = sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(qq_\w+)\s*\(", header, re.M)))
    assert len(declared) >= 20
    lib = qq3.runtime.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(qq3.runtime.exported_symbols()) == declared


def test_init_without_gpu_fails_loudly(qq3):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(qq3.runtime.QQError) as e:
        qq3.runtime.Context(0)
    assert e.value.code in (qq3.runtime.QQ_ERR_CUDA, qq3.runtime.QQ_ERR_INVALID)
    assert str(e.value)


def test_gguf_round_trip(qq3, tmp_path):
    spec = qq3.synth.tiny_lfm2(seed=2)
    path = tmp_path / "m.gguf"
    qq3.synth.write_gguf(spec, path)
    r = qq3.gguf.GGUFReader.fromFile(path)
    arch = r.getArch()
    assert arch["architecture"] == "lfm2moe" and arch["blockCount"] == spec.n_layers
    assert arch["headCountKV"] == spec.n_head_kv  # per-layer array, max of the non-zero entries
    assert r.getKeyValue("general.alignment") == 32
    mem = qq3.synth.build_tensors(spec)
    for name, (t, ne, raw) in mem.items():
        m = r.getTensorMetaByName(name)
        assert m.type == t and m.shape == ne
        assert m.offset % 32 == 0 and m.nbytes % 256 == 0
        assert np.array_equal(m.raw(), raw)
    assert len(r.getKeyValue("tokenizer.ggml.tokens")) == spec.n_vocab
    assert r.getKeyValue("tokenizer.ggml.merges") == []


def test_synth_is_deterministic_and_sliceable(qq3):
    a = qq3.synth.q8_0_blocks(32 * 100, seed=9)
    b = qq3.synth.q8_0_blocks(32 * 100, seed=9)
    assert np.array_equal(a, b)
    c = qq3.synth.q8_0_blocks(32 * 40, seed=9, block0=60)
    assert np.array_equal(a[60 * 34:], c)
    q = a.reshape(-1, 34)[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127
    d = a.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float64)
    assert np.all(d > 0) and abs(d.mean() - 0.02 / 127) < 0.1 * 0.02 / 127


def test_f16_conversion_matches_numpy(qq3):
    vals = np.concatenate([qq3.synth.normal_f32(5000, seed=1) * 1e-3, qq3.synth.normal_f32(5000, seed=2) * 1e-6,
                           np.array([65504, 65519, 65520, 1e-8, 3e-8, 6e-8, 5.96e-8, 2.98e-8, 0.0, -0.0], np.float32),
                           qq3.synth.normal_f32(5000, seed=3) * 3e4])
    ours = np.array([qq3.synth.f32_to_f16_bits(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, want)


def test_zipf_bias_calibration(qq3):
    spec = qq3.synth.lfm2_8b_a1b(seed=5)
    t = qq3.synth.build_tensors(spec, only={"blk.2.ffn_gate_inp.weight", "blk.2.exp_probs_b.bias"})
    alpha = spec.extra["zipf_alpha"]["blk.2.exp_probs_b.bias"]
    assert 0.0 < alpha < 0.5
    bias = t["blk.2.exp_probs_b.bias"][2].view(np.float32)
    assert bias.shape == (32,) and np.all(bias <= 0)


def test_engine_hparams_mirror_js(qq3):
    """Lfm2Engine / Qwen3Engine constructor derivations, without binding a device."""
    spec = qq3.synth.lfm2_8b_a1b()
    g = qq3.synth.MemoryGGUF(spec, {n: (t, ne, np.zeros(1, np.uint8)) for n, t, ne in qq3.synth.tensor_specs(spec)})
    e = object.__new__(qq3.Lfm2CudaEngine)
    e.gguf = g
    e._read_hparams(g)
    assert (e.nLayers, e.nEmb, e.nHeads, e.nHeadKV, e.headDim) == (24, 2048, 32, 8, 64)
    assert (e.nExperts, e.nExpertsUsed, e.nVocab, e.maxCtx) == (32, 4, 65536, 4096)
    assert [i for i in range(24) if e._is_attn(i)] == list(qq3.synth.LFM2_8B_ATTN_LAYERS)
    assert [i for i in range(24) if e._is_moe(i)] == list(range(2, 24))
    assert abs(e.eps - 1e-5) < 1e-12 and e.ropeFreqBase == 1e6
    spec = qq3.synth.qwen3_0p6b()
    g = qq3.synth.MemoryGGUF(spec, {n: (t, ne, np.zeros(1, np.uint8)) for n, t, ne in qq3.synth.tensor_specs(spec)})
    q = object.__new__(qq3.Qwen3CudaEngine)
    q._read_hparams(g)
    assert (q.nLayers, q.nEmb, q.nHeads, q.nHeadKV, q.headDim, q.nVocab, q.maxCtx) == (28, 1024, 16, 8, 128, 151936, 4096)
    # a Qwen3-MoE file: expert counts from its metadata, MoE layers where a router exists
    spec = qq3.synth.ModelSpec("qwen3moe", 2, 64, 2, 1, 64, 96, 64, 1e6, 1e-6, n_expert=8, n_expert_used=2,
                               n_ff_exp=32)
    g = qq3.synth.MemoryGGUF(spec, {n: (t, ne, np.zeros(1, np.uint8)) for n, t, ne in qq3.synth.tensor_specs(spec)})
    m = object.__new__(qq3.Qwen3CudaEngine)
    m._read_hparams(g)
    assert (m.nExperts, m.nExpertsUsed) == (8, 2) and [m._is_moe(i) for i in range(2)] == [True, True]


def test_host_sampling_mirrors_tensor_js(qq3):
    from qq3.engine import sample_top_p_top_k, sample_with_think_control

    logits = np.array([0.1, 2.0, 2.0, -1.0, 0.5], np.float32)
    assert sample_with_think_control(logits.copy(), 0.0, 0.9, 40, dict(mode="full", thinkId=1, endThinkId=4)) == 1
    assert sample_with_think_control(logits.copy(), 0.0, 0.9, 40, dict(mode="suppress", thinkId=1, endThinkId=4)) == 2
    # 'shorten': </think> forced when fewer than topK logits beat it
    assert sample_with_think_control(logits.copy(), 0.0, 0.9, 3, dict(mode="shorten", thinkId=1, endThinkId=4,
                                                                       thinkingDone=False)) == 4
    # top-k = 1: a draw inside the kept mass returns the most probable id; the JS does not
    # renormalise after the cut, so a draw above it falls through to the last sorted id
    assert sample_top_p_top_k(logits, 0.7, 0.9, 1, rng=lambda: 0.1) == 1
    assert sample_top_p_top_k(logits, 0.7, 0.9, 1, rng=lambda: 0.999) == 3


def _js_top_p_top_k(logits, temperature, top_p, top_k, r):
    """sampleTopPTopK (tensor.js:188-228) transcribed loop for loop: f64 arithmetic (JS numbers),
    f32 rounding where the JS stores into the Float32Array, a stable sort, Math.random() = r."""
    x = [float(v) for v in np.asarray(logits, np.float32)]
    n = len(x)
    mx = -np.inf
    for v in x:
        if v > mx:
            mx = v
    s = 0.0
    for i in range(n):
        x[i] = float(np.float32(np.exp((x[i] - mx) / temperature)))
        s += x[i]
    inv = 1.0 / s
    for i in range(n):
        x[i] = float(np.float32(x[i] * inv))
    idx = sorted(([x[i], i] for i in range(n)), key=lambda a: -a[0])  # Python's sort is stable
    k_limit = min(top_k, n) if top_k > 0 else n
    for i in range(k_limit, n):
        idx[i][0] = 0.0
    cum = 0.0
    for i in range(n):
        cum += idx[i][0]
        if cum >= top_p:
            for j in range(i + 1, n):
                idx[j][0] = 0.0
            break
    cum = 0.0
    for i in range(n):
        cum += idx[i][0]
        if r <= cum:
            return idx[i][1]
    return idx[n - 1][1]


def test_top_p_top_k_matches_js_transcription(qq3):
    """The host sampler picks the same id as the literal JS loops on random logits (with ties),
    temperatures, top-p, top-k and random draws.  (A NaN logit makes every JS probability NaN and
    the result then depends on the JS engine's sort, so it is not a case here.)"""
    from qq3.engine import sample_top_p_top_k

    rng = np.random.default_rng(11)
    for case in range(300):
        n = int(rng.integers(1, 60))
        logits = (rng.standard_normal(n) * rng.choice([0.5, 3.0, 20.0])).astype(np.float32)
        if case % 5 == 0:
            logits = np.round(logits)  # ties
        t = float(rng.choice([0.3, 0.7, 1.0, 1.5]))
        top_p = float(rng.choice([0.5, 0.9, 0.95, 1.0]))
        top_k = int(rng.choice([0, 1, 5, 40]))
        r = float(rng.random())
        want = _js_top_p_top_k(logits, t, top_p, top_k, r)
        assert sample_top_p_top_k(logits.copy(), t, top_p, top_k, rng=lambda: r) == want, case


def test_gguf_reads_k_quant_and_legacy_tensors(qq3, tmp_path):
    """A GGUF holding k-quant and legacy quantised tensors parses, and every tensor reads back its
    own bytes (block sizes: 84/110/144/176/210 per 256 values, 18/20/22/24/36 per 32)."""
    G = qq3.gguf
    w = G.GGUFWriter()
    w.add_kv("general.architecture", G.KV_TYPES["STRING"], "qwen3")
    rng = np.random.default_rng(3)
    want = {}
    for t in (2, 3, 6, 7, 9, 10, 11, 12, 13, 14):
        shape = [512, 3]
        raw = rng.integers(0, 256, size=G.tensor_nbytes(shape, t), dtype=np.uint8)
        w.add_tensor(f"t{t}", shape, t, raw)
        want[f"t{t}"] = (t, raw)
    path = tmp_path / "k.gguf"
    w.write(path)
    r = G.GGUFReader.fromFile(path)
    for name, (t, raw) in want.items():
        m = r.getTensorMetaByName(name)
        assert m.type == t and m.shape == [512, 3]
        assert np.array_equal(m.raw(), raw), name
    assert G.tensor_nbytes([512, 3], 12) == 6 * 144 and G.tensor_nbytes([64], 2) == 2 * 18
    with pytest.raises(ValueError):
        G.tensor_nbytes([32], 15)


def test_sample_uniform_twin_matches_library(qq3):
    """The device sampler's draws (qq_sample_uniform, a host function of the library) and their
    Python twin agree bit for bit, so a host can reproduce every Math.random() replacement."""
    import ctypes as C

    lib = qq3.runtime.load()
    rng = np.random.default_rng(3)
    for _ in range(200):
        seed = int(rng.integers(0, 2 ** 63)) * 2 + int(rng.integers(0, 2))
        seq, pos = int(rng.integers(0, 64)), int(rng.integers(0, 1 << 20))
        r = C.c_double(-1.0)
        qq3.runtime.check(lib.qq_sample_uniform(C.c_uint64(seed), seq, pos, C.byref(r)))
        assert r.value == qq3.runtime.sample_uniform(seed, seq, pos)
        assert 0.0 <= r.value < 1.0


def _fake_engine(qq3, script, eos=2, stops=(7,)):
    """A Qwen3 engine object without a device: the token that follows forward(t, pos) is
    script[pos] (greedy on the device, or the only finite logit on the host path)."""
    eng_mod = qq3.engine

    class Fake(eng_mod.Qwen3CudaEngine):
        def __init__(self):  # no GGUF, no context
            self.nVocab = 64
            self.eosTokenId = eos
            self.stopTokenIds = set(stops)
            self.calls = []
            self.prefilled = []

        def resetKVCache(self, seq=0):
            self.calls.clear()

        def prefill(self, tokenIds, pos0=0, seq=0):
            self.prefilled = list(tokenIds)

        def forward_argmax(self, tokenId, position, suppress_id=-1, seq=0):
            self.calls.append((int(tokenId), int(position), int(suppress_id)))
            return int(script[position])

        def forward(self, tokenId, position, skipLogits=False, seq=0):
            self.calls.append((int(tokenId), int(position), -2))
            logits = np.full(self.nVocab, -1e30, dtype=np.float32)
            logits[int(script[position])] = 0.0
            return logits

    return Fake()


def _js_generate(token_ids, max_steps, eos, stops, next_after):
    # qwen3-engine.js:397-457: sample after the last prompt token, then per step: stop on EOS or
    # a stop id, forward the current token at position n + step, emit it, sample the next
    cur = next_after(token_ids[-1], len(token_ids) - 1)
    out = []
    for step in range(max_steps):
        if cur == eos or cur in stops:
            break
        nxt = next_after(cur, len(token_ids) + step)
        out.append(cur)
        cur = nxt
    return out


@pytest.mark.parametrize("case", ["eos", "stop_id", "max_steps", "host_sampler"])
def test_generate_loop_mirrors_js(qq3, case):
    rng = np.random.default_rng(11)
    script = rng.integers(10, 60, size=256)
    prompt = [3, 5, 8, 13]
    n = len(prompt)
    if case == "eos":
        script[n + 4] = 2
    elif case == "stop_id":
        script[n + 2] = 7
    eng = _fake_engine(qq3, script)
    max_steps = 9 if case == "max_steps" else 40
    want = _js_generate(prompt, max_steps, 2, {7}, lambda t, p: int(script[p]))
    seen, finished = [], []
    kw = dict(temperature=0.7, topP=0.9, topK=0) if case == "host_sampler" else dict(temperature=0)
    got = eng.generate(prompt, maxSteps=max_steps, onToken=seen.append, onFinish=finished.append, **kw)
    assert got == want
    assert seen == want and finished == [want]
    assert eng.prefilled == prompt[:-1]
    # positions: the last prompt token at n - 1, then generated token s at n + s
    assert [c[1] for c in eng.calls] == list(range(n - 1, n - 1 + len(eng.calls)))
    assert [c[0] for c in eng.calls] == [prompt[-1]] + want[: len(eng.calls) - 1]
    if case != "host_sampler":  # greedy on the device with the think id suppressed
        assert all(c[2] == (eng.THINK_ID if eng.THINK_ID < eng.nVocab else -1) for c in eng.calls)
    # script[n - 1] is the first generated token, script[n + s] the one after generated token s
    if case == "eos":
        assert len(want) == 5
    elif case == "stop_id":
        assert len(want) == 3
    elif case == "max_steps":
        assert len(want) == max_steps


def test_generate_abort_returns_none(qq3):
    script = np.full(64, 20)
    eng = _fake_engine(qq3, script)

    class Signal:
        aborted = False

    sig = Signal()

    def on_token(t):
        if len(eng.calls) >= 3:
            sig.aborted = True

    assert eng.generate([1, 4], maxSteps=20, temperature=0, onToken=on_token, abortSignal=sig) is None
    assert len(eng.calls) == 3
    sig.aborted = True
    assert eng.generate([1, 4], maxSteps=20, temperature=0, abortSignal=sig) is None


def test_cpu_baseline_leg_on_a_tiny_model(qq3, orc):
    """bench.py's CPU baseline leg (the oracle on the host cores) on a tiny model: its record
    carries the fields the JSON line reports, the single-thread sample included."""
    import sys

    sys.path.insert(0, str(ROOT))
    import bench

    spec = qq3.synth.tiny_lfm2(seed=5)
    g = qq3.synth.MemoryGGUF(spec, qq3.synth.build_tensors(spec))
    prompt = qq3.synth.uniform_tokens(12, 5, spec.n_vocab)
    cb = bench.cpu_decode(g, spec, prompt, steps=3, warmup=1, single_s=0.05, label="tiny LFM2")
    assert cb["unit"] == "tok/s" and cb["kind"] == "port" and cb["value"] > 0
    assert cb["cores"] >= 1 and cb["nproc"] == cb["cores"]
    assert "12-token prompt" in cb["sample"] and "1 warm-up + 3 timed greedy steps" in cb["sample"]
    assert cb["single_thread"]["cores"] == 1 and cb["single_thread"]["value"] > 0
