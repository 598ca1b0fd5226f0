"""The C oracle (oracle/qq3_oracle.c) against the golden vectors of the independent
pure-Python restatement (tests/golden/gen_golden.py).  CPU only."""
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return dict(np.load(GOLD / name))


def test_ops_golden(orc):
    g = _load("ops.npz")
    K, N = 96, 10
    y = orc.matmul(g["mm_raw"], 8, [K, N], g["mm_x"])
    assert np.array_equal(y, g["mm_y"])
    assert np.array_equal(orc.embedding(g["mm_raw"], [K, N], 7), g["emb"])
    v, w = g["vec"], g["w"]
    rms = np.concatenate([orc.rmsnorm(v[:64], w, float(np.float32(1e-6))), orc.rmsnorm(v[64:], w, float(np.float32(1e-6)))])
    assert np.array_equal(rms, g["rms"])
    assert np.array_equal(orc.rope(v, 2, 64, 37, 1e6), g["rope"])
    assert np.array_equal(orc.softmax(v), g["softmax"])
    assert np.array_equal(orc.silu(v), g["silu"])
    assert orc.sample_greedy(v) == int(g["greedy"][0])


class _Npz:
    """GGUF-lookup view over a golden .npz (tensors stored raw)."""

    def __init__(self, g, kv):
        self.g, self.kv = g, kv

    def getKeyValue(self, k, d=None):
        return self.kv.get(k, d)

    def getTensorMetaByName(self, name):
        if "w:" + name not in self.g:
            return None
        from qq3.gguf import TensorMeta

        ne = [int(v) for v in self.g["ne:" + name]]
        raw = self.g["w:" + name]
        return TensorMeta(raw, 0, raw.nbytes, ne[:-1], ne[-1], name)


def _micro(qq3, which):
    from tests.golden.gen_golden import micro_specs  # noqa: F401  (same specs as the generator)

    from tests.golden.gen_golden import micro_qwen3kq_spec, micro_qwen3moe_spec

    _, lfm, qw = micro_specs()
    spec = {"lfm2": lfm, "qwen3": qw, "qwen3moe": micro_qwen3moe_spec(qq3), "qwen3kq": micro_qwen3kq_spec(qq3)}[which]
    kv = qq3.synth.kv_values(spec)
    return spec, _Npz(_load(f"micro_{which}.npz"), kv)


@pytest.mark.parametrize("which", ["lfm2", "qwen3", "qwen3moe", "qwen3kq"])
def test_micro_model_golden(qq3, orc, which):
    spec, g = _micro(qq3, which)
    m = orc.OracleModel(g, max_ctx=32, threads=1)
    for p, t in enumerate(g.g["tokens"]):
        logits, hidden, rec = m.forward(int(t), p, False, dump=True, routing=True)
        assert np.array_equal(logits, g.g["logits"][p]), f"pos {p} logits"
        assert np.array_equal(hidden, g.g["hidden"][p]), f"pos {p} hidden"
        if "routing" in g.g:
            assert np.array_equal(rec, g.g["routing"][p]), f"pos {p} routing"
    cur = int(np.argmax(logits))
    gen = []
    pos = len(g.g["tokens"])
    for _ in range(len(g.g["generated"])):
        lg = m.forward(cur, pos, False)
        gen.append(cur)
        cur = int(np.argmax(lg))
        pos += 1
    assert gen == g.g["generated"].tolist()


def test_oracle_threads_do_not_change_results(qq3, orc):
    spec = qq3.synth.tiny_lfm2(seed=9)
    g = qq3.synth.memory_model(spec)
    a = orc.OracleModel(g, max_ctx=16, threads=1)
    outs1 = [a.forward(t, p) for p, t in enumerate([3, 9, 27])]
    b = orc.OracleModel(g, max_ctx=16, threads=4)
    outs4 = [b.forward(t, p) for p, t in enumerate([3, 9, 27])]
    for x, y in zip(outs1, outs4):
        assert np.array_equal(x, y)


def test_oracle_matches_numpy_float64(qq3, orc):
    """Dequantised matmul in float64 (numpy) agrees with the oracle to f32 rounding."""
    K, N = 256, 40
    raw = qq3.synth.q8_0_blocks(K * N, seed=5, mode=1)
    x = qq3.synth.normal_f32(3 * K, seed=6).reshape(3, K)
    W = qq3.synth.dequant_q8_0(raw, K * N).reshape(N, K).astype(np.float64)
    want = (x.astype(np.float64) @ W.T).astype(np.float32)
    got = orc.matmul(raw, 8, [K, N], x)
    assert np.allclose(got, want, rtol=0, atol=1e-6 * np.abs(want).max())
    assert np.array_equal(orc.dequant(raw, 8, [K, N]), qq3.synth.dequant_q8_0(raw, K * N))


@pytest.mark.parametrize("t", [10, 11, 12, 13, 14])
def test_kquants_golden(orc, t):
    """k-quant matmuls, column lookups and dequantisation (Q2_K..Q6_K, tensor.js:267-664) of the
    C oracle against the independent transcription's vectors, bit for bit (K = 512 and a ragged
    K = 300 whose last superblock is partly used)."""
    g = _load("kquants.npz")
    for K in (512, 300):
        key = f"t{t}_k{K}"
        raw, x, y, cols = g[key + "_raw"], g[key + "_x"], g[key + "_y"], g[key + "_cols"]
        N = cols.shape[0]
        assert np.array_equal(orc.matmul(raw, t, [K, N], x), y), key
        for c in range(N):
            assert np.array_equal(_column(orc, raw, t, K, N, c), cols[c]), (key, c)
        assert np.array_equal(orc.dequant(raw, t, [K, N]), cols.reshape(-1)), key


def _column(orc, raw, t, K, N, c):
    """embeddingLookupGeneric of a k-quant tensor (tensor.js:511-549): column c."""
    import ctypes as C

    tens = orc.make_tensor(raw, t, [K, N])
    out = np.empty(K, dtype=np.float32)
    orc.lib().orc_embedding(C.byref(tens), c, out.ctypes.data)
    return out
