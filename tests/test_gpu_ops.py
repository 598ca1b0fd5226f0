"""Op-level parity of the CUDA path (through the C ABI) against the CPU oracle.

Tolerances: dequantised weights are bit-exact; floating-point outputs must be within the
north-star bar of 1e-2 max relative error (max|got-want| / max|want|), and the f32-vs-f64
accumulation gap is additionally held to TIGHT so that a dropped block or row shows up.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2      # north-star bar for activations / logits
TIGHT = 2e-5    # f32 accumulation vs the oracle's f64 on a single matmul
TC = 1e-4       # M >= 2 rows run on the tensor cores: x and w = q*d split into fp16 hi/lo pairs,
                # three products accumulated in f32 (~2^-22 per product, like the f32 GEMV)

SWEEP = [(1024, 1024), (3072, 1024), (1024, 3072), (151936, 1024), (7168, 2048)]


@pytest.fixture(scope="module")
def torch():
    import torch as t

    assert t.cuda.is_available()
    return t


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_streaming_upload_bit_exact(qq3, orc, gpu_ctx, torch):
    """Tensors uploaded through the pinned staging ring (qq_upload_begin/_async/_finish) equal the
    oracle's dequantisation bit for bit: a small staging ring (4 slots of 68 KB) splits the larger
    tensors into many chunks whose boundaries fall mid-row, and F32 tensors ride along."""
    shapes = [(8, [1024, 1792]), (8, [32, 96]), (0, [2048]), (8, [2048, 1792, 3]), (0, [3, 2048]), (8, [64, 5])]
    raws = []
    for i, (t, ne) in enumerate(shapes):
        n = int(np.prod(ne))
        raws.append(qq3.synth.q8_0_blocks(n, seed=300 + i, mode=1) if t == 8 else
                    qq3.synth.normal_f32(n, seed=300 + i).view(np.uint8))
    with gpu_ctx.streaming_upload(staging_bytes=4 * 68 * 1024) as up:
        tensors = [up.upload(raw, t, ne) for (t, ne), raw in zip(shapes, raws)]
    assert up.bytes == sum(r.nbytes for r in raws)
    for (t, ne), raw, W in zip(shapes, raws, tensors):
        n = int(np.prod(ne))
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        W.dequant(out)
        gpu_ctx.synchronize()
        want = orc.dequant(raw, 8, ne) if t == 8 else raw.view(np.float32)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32)), ne
        W.free()


@pytest.mark.parametrize("N,K", SWEEP + [(1792, 2048 * 32), (96, 32)])
def test_dequant_bit_exact(qq3, orc, gpu_ctx, torch, N, K):
    raw = qq3.synth.q8_0_blocks(N * K, seed=100 + N + K, mode=1)
    W = gpu_ctx.upload(raw, 8, [K, N])
    out = torch.empty(N * K, dtype=torch.float32, device="cuda")
    W.dequant(out)
    gpu_ctx.synchronize()
    want = orc.dequant(raw, 8, [K, N])
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    W.free()


@pytest.mark.parametrize("N,K", SWEEP)
@pytest.mark.parametrize("M", [1, 16])
def test_q8_matmul_vs_oracle(qq3, orc, gpu_ctx, torch, N, K, M):
    orc.set_threads(8)
    raw = qq3.synth.q8_0_blocks(N * K, seed=7 + N * 3 + K, mode=1)
    x = qq3.synth.normal_f32(M * K, seed=M + N).reshape(M, K)
    W = gpu_ctx.upload(raw, 8, [K, N])
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    xd = _dev(torch, x)
    torch.cuda.synchronize()
    gpu_ctx.q8_matmul(W, xd, M, y)
    gpu_ctx.synchronize()
    got = y.cpu().numpy()
    want = orc.matmul(raw, 8, [K, N], x)
    bar = TIGHT if M == 1 else TC
    for r in range(M):
        e = rel_err(got[r], want[r])
        assert e < bar, f"row {r}: rel err {e:.3e}"
    W.free()


@pytest.mark.parametrize("M", [512, 4096])
def test_q8_matmul_large_m_sampled_rows(qq3, orc, gpu_ctx, torch, M):
    """Large-M sweep points: every row on the GPU, a seeded sample of rows on the oracle."""
    orc.set_threads(8)
    N, K = 7168, 2048
    raw = qq3.synth.q8_0_blocks(N * K, seed=900 + M, mode=1)
    x = qq3.synth.normal_f32(M * K, seed=M).reshape(M, K)
    W = gpu_ctx.upload(raw, 8, [K, N])
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    gpu_ctx.q8_matmul(W, _dev(torch, x), M, y)
    gpu_ctx.synchronize()
    got = y.cpu().numpy()
    rows = np.unique(np.concatenate([[0, M - 1], qq3.synth.uniform_tokens(6, M, M)]))
    want = orc.matmul(raw, 8, [K, N], x[rows])
    for i, r in enumerate(rows):
        assert rel_err(got[r], want[i]) < TC
    assert np.isfinite(got).all()
    W.free()


@pytest.mark.parametrize("M,N,K", [(2, 96, 32), (3, 1000, 96), (17, 1000, 4096), (32, 3072, 12288),
                                   (130, 257, 2048), (129, 4096, 1024)])
def test_q8_matmul_tensor_core_ragged(qq3, orc, gpu_ctx, torch, M, N, K):
    """Ragged tiles of the tensor-core paths: M and N off the tiles, K % 64 == 32; M <= 32 takes
    the few-row kernel (16- and 32-row operand tiles, K split over CTAs), larger M the 128-row one."""
    orc.set_threads(8)
    raw = qq3.synth.q8_0_blocks(N * K, seed=31 * N + K, mode=1)
    x = qq3.synth.normal_f32(M * K, seed=5 * M + 1).reshape(M, K)
    W = gpu_ctx.upload(raw, 8, [K, N])
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.q8_matmul(W, _dev(torch, x), M, y)
    gpu_ctx.synchronize()
    got = y.cpu().numpy()
    want = orc.matmul(raw, 8, [K, N], x)
    assert np.isfinite(got).all()
    for r in range(M):
        assert rel_err(got[r], want[r]) < TC, f"row {r}"
    W.free()


def test_rope_vs_oracle(qq3, orc, gpu_ctx, torch):
    """qq_rope against applyRoPE (tensor.js:132-147): rows at consecutive positions."""
    rows, heads, hd, pos0, base = 3, 4, 128, 37, 1e6
    x = qq3.synth.normal_f32(rows * heads * hd, seed=61).reshape(rows, heads * hd)
    xd = _dev(torch, x)
    gpu_ctx.rope(xd, rows, heads, hd, pos0, base)
    gpu_ctx.synchronize()
    got = xd.cpu().numpy()
    for r in range(rows):
        want = orc.rope(x[r], heads, hd, pos0 + r, base)
        assert rel_err(got[r], want) < 1e-5, f"row {r}"


@pytest.mark.parametrize("n_head,n_kv,hd,pos", [(4, 2, 128, 150), (8, 2, 64, 0), (32, 8, 64, 700)])
def test_attention_decode_vs_f64(qq3, gpu_ctx, torch, n_head, n_kv, hd, pos):
    """qq_attention_decode against _selfAttentionCore (qwen3-engine.js:249-291) evaluated in f64:
    query head h reads KV head floor(h n_kv / n_head), softmax over positions 0..pos."""
    max_ctx = 768
    q = qq3.synth.normal_f32(n_head * hd, seed=62).reshape(n_head, hd)
    kc = qq3.synth.normal_f32(n_kv * max_ctx * hd, seed=63).reshape(n_kv, max_ctx, hd)
    vc = qq3.synth.normal_f32(n_kv * max_ctx * hd, seed=64).reshape(n_kv, max_ctx, hd)
    out = torch.full((n_head, hd), float("nan"), dtype=torch.float32, device="cuda")
    gpu_ctx.attention_decode(_dev(torch, q), _dev(torch, kc), _dev(torch, vc), n_head, n_kv, hd, max_ctx, pos, out)
    gpu_ctx.synchronize()
    got = out.cpu().numpy()
    for h in range(n_head):
        kv = h * n_kv // n_head
        s = kc[kv, :pos + 1].astype(np.float64) @ q[h].astype(np.float64) / np.sqrt(hd)
        w = np.exp(s - s.max())
        want = (w / w.sum()) @ vc[kv, :pos + 1].astype(np.float64)
        assert rel_err(got[h], want) < 1e-4, f"head {h}"


def test_embed_and_swiglu(qq3, orc, gpu_ctx, torch):
    """qq_embed is embeddingLookupQ80 bit for bit (tensor.js:56-77); qq_swiglu is silu(g) * u
    (tensor.js:168-180)."""
    K, V = 256, 1000
    raw = qq3.synth.q8_0_blocks(K * V, seed=65, mode=1)
    E = gpu_ctx.upload(raw, 8, [K, V])
    toks = [0, 7, V - 1, 7]
    out = torch.empty((len(toks), K), dtype=torch.float32, device="cuda")
    gpu_ctx.embed(E, toks, out)
    got = out.cpu().numpy()
    for i, t in enumerate(toks):
        assert np.array_equal(got[i], orc.embedding(raw, [K, V], t)), f"token {t}"
    with pytest.raises(RuntimeError):
        gpu_ctx.embed(E, [V], out)
    E.free()
    n = 3000
    g = qq3.synth.normal_f32(n, seed=66) * 4
    u = qq3.synth.normal_f32(n, seed=67)
    h = torch.empty(n, dtype=torch.float32, device="cuda")
    gpu_ctx.swiglu(_dev(torch, g), _dev(torch, u), n, h)
    gpu_ctx.synchronize()
    want = orc.silu(g) * u
    assert rel_err(h.cpu().numpy(), want) < 1e-6


def test_rmsnorm_vs_oracle(qq3, orc, gpu_ctx, torch):
    n, rows = 2048, 5
    x = qq3.synth.normal_f32(n * rows, seed=3).reshape(rows, n) * 3
    w = qq3.synth.normal_f32(n, seed=4)
    wt = gpu_ctx.upload(w.view(np.uint8), 0, [n])
    xd = _dev(torch, x)
    yd = torch.empty_like(xd)
    gpu_ctx.rmsnorm(xd, rows, n, wt, 1e-5, yd)
    gpu_ctx.synchronize()
    want = orc.rmsnorm(x, w, float(np.float32(1e-5)))
    assert rel_err(yd.cpu().numpy(), want) < 1e-6


def _moe_layer(qq3, E=2048, F=1792, NE=32, seed=5):
    spec = qq3.synth.lfm2_8b_a1b(seed=seed)
    names = [f"blk.2.{n}" for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                    "ffn_down_exps.weight", "exp_probs_b.bias")]
    t = qq3.synth.build_tensors(spec, only=set(names))
    return {k.split(".", 2)[2]: v for k, v in t.items()}


def _upload_layer(qq3, gpu_ctx, tensors):
    rt = qq3.runtime
    L = rt.LayerDesc()
    keep = []
    for name, (t, ne, raw) in tensors.items():
        slot = rt.SLOT[[s for s, n in rt.SLOT_TENSOR_NAMES.items() if n == name][0]]
        h = gpu_ctx.upload(raw, t, ne)
        keep.append(h)
        L.t[slot] = h.h.value
    L.is_moe = 1
    return L, keep


@pytest.mark.parametrize("T", [1, 15, 16, 64])
def test_moe_block_vs_oracle(qq3, orc, gpu_ctx, torch, T):
    """T < 16: per-token expert GEMVs; T >= 16: rows regrouped by expert on the tensor cores."""
    orc.set_threads(8)
    tensors = _moe_layer(qq3)
    L, keep = _upload_layer(qq3, gpu_ctx, tensors)
    x = qq3.synth.normal_f32(T * 2048, seed=T).reshape(T, 2048)
    out = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
    rec = torch.empty((T, 2 * 4 + 32), dtype=torch.float32, device="cuda")
    gpu_ctx.moe_block(L, 32, 4, _dev(torch, x), T, out, rec)
    gpu_ctx.synchronize()
    want, want_rec = orc.lfm2_moe(tensors, 2048, 32, 4, x)
    got_rec = rec.cpu().numpy()
    # router: identical top-k ids except near-ties (selection-score gap < 1e-5)
    sel_ids_ok = np.array_equal(got_rec[:, :4], want_rec[:, :4])
    if not sel_ids_ok:
        bias = tensors["exp_probs_b.bias"][2].view(np.float32)
        for t in range(T):
            if not np.array_equal(got_rec[t, :4], want_rec[t, :4]):
                s = np.sort(want_rec[t, 8:] + bias)[::-1]
                assert abs(s[3] - s[4]) < 1e-5, f"token {t}: top-k differs without a near-tie"
    assert rel_err(got_rec[:, 8:], want_rec[:, 8:]) < 1e-6  # sigmoid probs
    assert rel_err(got_rec[:, 4:8], want_rec[:, 4:8]) < 1e-5  # normalised weights
    for t in range(T):
        assert rel_err(out.cpu().numpy()[t], want[t]) < TOL
    for k in keep:
        k.free()


def test_moe_block_t2048_sampled_rows(qq3, orc, gpu_ctx, torch):
    """benchmark config 3 at T = 2048 (grouped tensor-core path): every row on the GPU, a seeded
    sample of rows on the oracle (the block is row-independent)."""
    orc.set_threads(8)
    T = 2048
    tensors = _moe_layer(qq3, seed=9)
    L, keep = _upload_layer(qq3, gpu_ctx, tensors)
    x = qq3.synth.normal_f32(T * 2048, seed=77).reshape(T, 2048)
    out = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
    rec = torch.empty((T, 2 * 4 + 32), dtype=torch.float32, device="cuda")
    gpu_ctx.moe_block(L, 32, 4, _dev(torch, x), T, out, rec)
    gpu_ctx.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    rows = np.unique(np.concatenate([[0, T - 1], qq3.synth.uniform_tokens(14, 5, T)]))
    want, want_rec = orc.lfm2_moe(tensors, 2048, 32, 4, x[rows])
    got_rec = rec.cpu().numpy()[rows]
    bias = tensors["exp_probs_b.bias"][2].view(np.float32)
    for i, t in enumerate(rows):
        if np.array_equal(got_rec[i, :4], want_rec[i, :4]):
            assert rel_err(got[t], want[i]) < TOL, f"token {t}"
        else:  # routing may differ only at a near-tie (selection-score gap < 1e-5)
            s = np.sort(want_rec[i, 8:] + bias)[::-1]
            assert abs(s[3] - s[4]) < 1e-5, f"token {t}: top-k {got_rec[i, :4]} vs {want_rec[i, :4]} without a near-tie"
    for k in keep:
        k.free()
