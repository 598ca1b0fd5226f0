"""Parity of the per-phase decode kernels (one launch per phase, QQ3_PERSISTENT=0) against the
CPU oracle, with the same bars as the default persistent step (logits within 1e-2 max relative
error, router top-k identical except near-ties, greedy tokens identical)."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_models import TOL, _check_routing, _pair

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def phase_kernels(monkeypatch):
    monkeypatch.setenv("QQ3_PERSISTENT", "0")


def _assert_phases(qq3, eng):
    # more than one kernel node per decode step means the per-phase kernels ran
    assert eng.model.stat(qq3.runtime.QQ_STAT_STEP_KERNELS) > 1


@pytest.mark.parametrize("arch", ["lfm2", "qwen3"])
def test_phases_per_token_parity(qq3, orc, arch):
    spec = qq3.synth.tiny_lfm2(seed=51) if arch == "lfm2" else qq3.synth.tiny_qwen3(seed=52)
    g, eng, ref = _pair(qq3, orc, spec)
    toks = qq3.synth.uniform_tokens(12, 9, spec.n_vocab)
    for p, t in enumerate(toks):
        want, _, rec = ref.forward(int(t), p, False, dump=True, routing=True)
        got = eng.forward(int(t), p, False)
        assert rel_err(got, want) < TOL
        assert int(np.argmax(got)) == int(np.argmax(want))
        if arch == "lfm2":
            _check_routing(eng, rec)
    _assert_phases(qq3, eng)
    eng.close()


def test_phases_decode_loop_and_mask(qq3, orc):
    spec = qq3.synth.tiny_lfm2(seed=53)
    g, eng, ref = _pair(qq3, orc, spec)
    masked = {1, 6}
    eng.expertMask = masked
    ref.set_expert_mask(masked)
    prompt = qq3.synth.uniform_tokens(7, 3, spec.n_vocab).tolist()
    eng.prefill(prompt[:-1])
    dev = eng.model.decode_loop(prompt[-1], len(prompt) - 1, 16)
    for p, t in enumerate(prompt[:-1]):
        ref.forward(t, p, True)
    cur, pos, want = prompt[-1], len(prompt) - 1, []
    for _ in range(16):
        cur = int(np.argmax(ref.forward(cur, pos, False)))
        want.append(cur)
        pos += 1
    assert dev.tolist() == want
    _assert_phases(qq3, eng)
    eng.close()


def test_phases_lfm2_8b_a1b_truncated_full_width(qq3, orc):
    spec = qq3.synth.lfm2_8b_a1b(seed=78)
    spec.n_layers = 4
    spec.attn_layers = (2,)
    g, eng, ref = _pair(qq3, orc, spec, max_ctx=96)
    toks = qq3.synth.uniform_tokens(40, 6, spec.n_vocab)
    for p, t in enumerate(toks):
        want, _, rec = ref.forward(int(t), p, False, dump=True, routing=True)
        got = eng.forward(int(t), p, False)
        assert rel_err(got, want) < TOL
        assert int(np.argmax(got)) == int(np.argmax(want))
        _check_routing(eng, rec)
    _assert_phases(qq3, eng)
    eng.close()


def test_phases_lfm2_8b_a1b_config_greedy_slice(qq3, orc):
    spec = qq3.synth.lfm2_8b_a1b(seed=1235)
    g, eng, ref = _pair(qq3, orc, spec, max_ctx=64)
    prompt = qq3.synth.uniform_tokens(16, 4322, spec.n_vocab)
    want = ref.generate(prompt, 8, think_id=124901)
    got = eng.model.generate(prompt, 8, think_id=124901)
    assert got.tolist() == want.tolist()
    _assert_phases(qq3, eng)
    eng.close()


def test_phases_qwen3_0p6b_config_greedy(qq3, orc):
    spec = qq3.synth.qwen3_0p6b(seed=1236)
    g, eng, ref = _pair(qq3, orc, spec, max_ctx=96)
    prompt = qq3.synth.uniform_tokens(24, 1236, spec.n_vocab)
    want = ref.generate(prompt, 32, think_id=151667)
    got = eng.model.generate(prompt, 32, think_id=151667)
    assert got.tolist() == want.tolist()
    _assert_phases(qq3, eng)
    eng.close()
