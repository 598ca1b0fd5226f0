"""The allocation-free MoE block (qq_moe_block_noalloc) against the allocating entry point.

Some callers cannot let the library call cudaMalloc while a layer runs: a host that owns all
device memory through its own pool or budget (an embedding runtime such as a JS engine's addon,
or a serving process that pre-plans its memory), or code that issues the block while recording
its own stream work.  For them qq_moe_block_noalloc keeps its scratch in one fixed device array
of the library.  This file is collected last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the north-star bar used by the other parity tests


def _layer(qq3, ctx):
    spec = qq3.synth.lfm2_8b_a1b(seed=99)
    names = {f"blk.2.{n}" for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                    "ffn_down_exps.weight", "exp_probs_b.bias")}
    rt = qq3.runtime
    L = rt.LayerDesc()
    keep = []
    for name, (t, ne, raw) in qq3.synth.build_tensors(spec, only=names).items():
        suffix = name.split(".", 2)[2]
        slot = [k for k, v in rt.SLOT_TENSOR_NAMES.items() if v == suffix][0]
        h = ctx.upload(raw, t, ne)
        keep.append(h)
        L.t[rt.SLOT[slot]] = h.h.value
    L.is_moe = 1
    return L, keep


def _layer_tensors(qq3):
    spec = qq3.synth.lfm2_8b_a1b(seed=99)
    names = {f"blk.2.{n}" for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                    "ffn_down_exps.weight", "exp_probs_b.bias")}
    return {k.split(".", 2)[2]: v for k, v in qq3.synth.build_tensors(spec, only=names).items()}


def test_moe_block_noalloc_matches_allocating_entry_point(qq3, orc, gpu_ctx):
    """Three calls in a row -- 6 rows with routing records, 3 rows without (the records then live
    in the library's array), and 1024 rows, the stated maximum (where qq_moe_block regroups the
    rows by expert on the tensor cores while this entry point serves them token by token) --
    against qq_moe_block on every row and record, and against the CPU oracle on a sample of rows."""
    import torch

    L, keep = _layer(qq3, gpu_ctx)
    tensors = _layer_tensors(qq3)
    bias = tensors["exp_probs_b.bias"][2].view(np.float32)
    orc.set_threads(8)
    limit = qq3.runtime.QQ_NOALLOC_MAX_TOKENS
    for call, (T, with_records) in enumerate([(6, True), (3, False), (limit, True)]):
        x_host = qq3.synth.normal_f32(T * 2048, seed=100 + call).reshape(T, 2048)
        x = torch.from_numpy(x_host).cuda()
        want = torch.empty((T, 2048), dtype=torch.float32, device="cuda")
        want_rec = torch.empty((T, 40), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        gpu_ctx.moe_block(L, 32, 4, x, T, want, want_rec)
        gpu_ctx.synchronize()
        got = torch.full((T, 2048), float("nan"), dtype=torch.float32, device="cuda")
        got_rec = torch.full((T, 40), float("nan"), dtype=torch.float32, device="cuda") if with_records else None
        torch.cuda.synchronize()
        gpu_ctx.moe_block_noalloc(L, 32, 4, x, T, got, got_rec)
        gpu_ctx.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all(), f"call {call}: non-finite output"
        for t in range(T):
            assert rel_err(g[t], w[t]) < TOL, f"call {call}, token {t}"
        if with_records:
            # the same router kernel on both paths: ids, weights and probabilities agree exactly
            assert np.array_equal(got_rec.cpu().numpy(), want_rec.cpu().numpy()), f"call {call}: routing records"
        # the CPU oracle (the restated _moEFFN) on every row of the small calls, 12 rows of the large
        rows = np.arange(T) if T <= 8 else np.unique(np.concatenate([[0, T - 1], qq3.synth.uniform_tokens(10, 7, T)]))
        ref, ref_rec = orc.lfm2_moe(tensors, 2048, 32, 4, x_host[rows])
        ids = want_rec.cpu().numpy()[:, :4]  # equal to the no-alloc call's (checked above when it returns them)
        for i, t in enumerate(rows):
            if not np.array_equal(ids[t], ref_rec[i, :4]):
                s = np.sort(ref_rec[i, 8:] + bias)[::-1]
                assert abs(s[3] - s[4]) < 1e-5, f"call {call}, token {t}: top-k differs without a near-tie"
                continue
            assert rel_err(g[t], ref[i]) < TOL, f"call {call}, token {t}: vs oracle"
    # beyond the stated limit the call is refused before any GPU work
    with pytest.raises(qq3.runtime.QQError) as e:
        gpu_ctx.moe_block_noalloc(L, 32, 4, 16, limit + 1, 16, None)
    assert "exceeds the limit" in str(e.value)
    for k in keep:
        k.free()
