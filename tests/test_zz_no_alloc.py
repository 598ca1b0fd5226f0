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


def test_moe_block_noalloc_matches_allocating_entry_point(qq3, gpu_ctx):
    import torch

    L, keep = _layer(qq3, gpu_ctx)
    # two calls in a row; the second is smaller and takes the records from the scratch array
    for call, (T, with_records) in enumerate([(6, True), (3, False)]):
        x = torch.from_numpy(qq3.synth.normal_f32(T * 2048, seed=100 + call).reshape(T, 2048)).cuda()
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
            assert np.array_equal(got_rec.cpu().numpy()[:, :4], want_rec.cpu().numpy()[:, :4])
    # beyond the stated limit the call is refused before any GPU work
    big = qq3.runtime.QQ_NOALLOC_MAX_TOKENS + 1
    with pytest.raises(qq3.runtime.QQError) as e:
        gpu_ctx.moe_block_noalloc(L, 32, 4, 16, big, 16, None)
    assert "exceeds the limit" in str(e.value)
    for k in keep:
        k.free()
