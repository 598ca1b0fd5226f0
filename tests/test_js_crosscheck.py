"""Cross-check of the golden vectors against the reference's own JavaScript, where a JS runtime
exists.

The golden vectors (tests/golden/) come from a Python transcription of the reference's CPU path,
and the C oracle reproduces them bit for bit; nothing here checks them against the reference's
own code, because no JS runtime is installed on these machines.  This test closes that gap on a
machine that has one: it loads the reference's `src/tensor.js` into Node (its functions are
plain globals) and runs `matmulGeneric` and `embeddingLookupGeneric` on the golden inputs, which
must reproduce the golden outputs bit for bit (Q8_0 and the five k-quants).

Needs `node` on PATH with `DataView.prototype.getFloat16` (ES2025; tensor.js:21-23) and the
reference's `src` directory in the environment variable QQ3_REFERENCE_SRC; skipped otherwise.
"""
import json
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"

_DRIVER = r"""
const fs = require('fs'), vm = require('vm');
vm.runInThisContext(fs.readFileSync(process.env.QQ3_REFERENCE_SRC + '/tensor.js', 'utf8'));
const job = JSON.parse(fs.readFileSync(0, 'utf8'));
const buf = new Uint8Array(job.raw).buffer;
const meta = {buffer: buf, offset: 0, nbytes: buf.byteLength, shape: [job.K, job.N], type: job.type};
const out = {rows: job.x.map(r => Array.from(matmulGeneric(meta, Float32Array.from(r)))),
             cols: job.cols.map(c => Array.from(embeddingLookupGeneric(meta, c)))};
process.stdout.write(JSON.stringify(out));
"""


def _runtime():
    node = shutil.which("node")
    src = os.environ.get("QQ3_REFERENCE_SRC")
    if not node or not src or not (Path(src) / "tensor.js").exists():
        pytest.skip("no JS runtime, or QQ3_REFERENCE_SRC does not name the reference's src directory")
    probe = subprocess.run([node, "-e", "process.exit(typeof DataView.prototype.getFloat16 === 'function' ? 0 : 3)"])
    if probe.returncode != 0:
        pytest.skip("this JS runtime has no DataView.prototype.getFloat16")
    return node, src


def _run(node, src, raw, t, K, N, x, cols):
    job = dict(raw=[int(v) for v in raw], type=t, K=K, N=N, x=[[float(v) for v in r] for r in x], cols=cols)
    env = dict(os.environ, QQ3_REFERENCE_SRC=src)
    r = subprocess.run([node, "-e", _DRIVER], input=json.dumps(job), capture_output=True, text=True, timeout=300,
                       check=True, env=env)
    out = json.loads(r.stdout)
    return np.asarray(out["rows"], np.float32), np.asarray(out["cols"], np.float32)


def test_q8_0_golden_against_reference_js():
    node, src = _runtime()
    g = dict(np.load(GOLD / "ops.npz"))
    rows, cols = _run(node, src, g["mm_raw"], 8, 96, 10, g["mm_x"], [7])
    assert np.array_equal(rows, g["mm_y"])
    assert np.array_equal(cols[0], g["emb"])


@pytest.mark.parametrize("t", [10, 11, 12, 13, 14])
def test_kquant_golden_against_reference_js(t):
    node, src = _runtime()
    g = dict(np.load(GOLD / "kquants.npz"))
    for K in (512, 300):
        key = f"t{t}_k{K}"
        n = g[key + "_cols"].shape[0]
        rows, cols = _run(node, src, g[key + "_raw"], t, K, n, g[key + "_x"], list(range(n)))
        assert np.array_equal(rows, g[key + "_y"]), key
        assert np.array_equal(cols, g[key + "_cols"]), key
