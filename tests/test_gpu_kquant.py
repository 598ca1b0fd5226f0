"""k-quant weights (Q2_K..Q6_K) on the device against the reference's arithmetic
(tensor.js:267-664): dequantisation bit-exact, matmuls within the f32-accumulation bound, and
dense Qwen3 models whose embedding, lm_head and projections are k-quants (real GGUF mixes such as
Q4_K_M) token-exact against the oracle."""
from pathlib import Path

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TIGHT = 2e-5  # f32 accumulation against the f64 sums of a single matmul
TOL = 1e-2


@pytest.mark.parametrize("t", [10, 11, 12, 13, 14])
def test_kquant_dequant_matmul_embed_golden(qq3, gpu_ctx, torch, t):
    g = np.load(GOLDEN / "kquants.npz")
    raw, x, y, cols = (g[f"t{t}_k512_{k}"] for k in ("raw", "x", "y", "cols"))
    K, N = 512, cols.shape[0]
    W = gpu_ctx.upload(raw, t, [K, N])
    out = torch.empty(N * K, dtype=torch.float32, device="cuda")
    W.dequant(out)
    gpu_ctx.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), cols.reshape(-1).view(np.uint32))  # bit-exact
    yd = torch.empty((x.shape[0], N), dtype=torch.float32, device="cuda")
    gpu_ctx.q8_matmul(W, torch.from_numpy(np.ascontiguousarray(x)).cuda(), x.shape[0], yd)
    gpu_ctx.synchronize()
    assert rel_err(yd.cpu().numpy(), y) < TIGHT
    row = torch.empty((2, K), dtype=torch.float32, device="cuda")
    gpu_ctx.embed(W, [3, 0], row)
    gpu_ctx.synchronize()
    assert np.array_equal(row.cpu().numpy()[0].view(np.uint32), cols[3].view(np.uint32))
    # a tensor whose rows are not whole superblocks is refused (the reference pads its last one)
    with pytest.raises(qq3.runtime.QQError):
        gpu_ctx.upload(g[f"t{t}_k300_raw"], t, [300, N])
    W.free()


def _npz_model(qq3, name, spec):
    g = np.load(GOLDEN / name)
    tensors = {}
    for k in g.files:
        if k.startswith("w:"):
            n = k[2:]
            ne = [int(v) for v in g["ne:" + n]]
            tensors[n] = (ne[-1], ne[:-1], g[k])
    return g, qq3.synth.MemoryGGUF(spec, tensors)


def test_micro_qwen3_kquant_model_golden(qq3):
    """The golden micro Qwen3 whose embedding (also the tied lm_head), attn_q, attn_output,
    ffn_gate / up / down are Q6_K, Q4_K, Q5_K, Q2_K, Q3_K and Q6_K."""
    from tests.golden.gen_golden import micro_qwen3kq_spec

    g, gg = _npz_model(qq3, "micro_qwen3kq.npz", micro_qwen3kq_spec(qq3))
    eng = qq3.Qwen3CudaEngine(gg, device=0, max_ctx=32)
    for p, t in enumerate(g["tokens"]):
        got = eng.forward(int(t), p, False)
        assert rel_err(got, g["logits"][p]) < TOL, f"pos {p}"
        assert int(np.argmax(got)) == int(np.argmax(g["logits"][p]))
    cur, pos, gen = int(np.argmax(g["logits"][-1])), len(g["tokens"]), []
    for _ in range(len(g["generated"])):
        gen.append(cur)
        cur = eng.forward_argmax(cur, pos)
        pos += 1
    assert gen == g["generated"].tolist()
    eng.close()


def test_qwen3_0p6b_width_kquant_model_vs_oracle(qq3, orc):
    """Qwen3-0.6B widths (hidden 1024, 16/8 heads of 128, FFN 3072), 2 layers, a 4096-token
    vocabulary: k-quant embedding / lm_head and projections as in the golden micro model, 12
    prompt tokens then 8 greedy tokens, against the oracle."""
    from tests.golden.gen_golden import kquantize

    spec = qq3.synth.qwen3_0p6b(seed=53)
    spec.n_layers, spec.n_vocab = 2, 4096
    g = qq3.synth.MemoryGGUF(spec, kquantize(qq3.synth.build_tensors(spec), 54))
    eng = qq3.Qwen3CudaEngine(g, device=0, max_ctx=32)
    ref = orc.OracleModel(g, max_ctx=32, threads=8)
    prompt = qq3.synth.uniform_tokens(12, 55, spec.n_vocab)
    for p, t in enumerate(prompt):
        got = eng.forward(int(t), p, False)
        want = ref.forward(int(t), p, False)
        assert rel_err(got, want) < TOL, f"pos {p}"
        assert int(np.argmax(got)) == int(np.argmax(want))
    assert eng.model.generate(prompt, 8).tolist() == ref.generate(prompt, 8).tolist()
    eng.close()
