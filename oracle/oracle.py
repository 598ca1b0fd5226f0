"""ctypes wrapper of liboracle.so -- the CPU restatement of the QwenQwen3.js CPU path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg, never by the product.  Parity status: UNPINNED (the reference is JavaScript
without tests or golden vectors and no JS runtime exists here); see qq3_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

SLOTS = [
    "attn_norm.weight", "ffn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
    "attn_q_norm.weight", "attn_k_norm.weight", "shortconv.conv.weight", "shortconv.in_proj.weight",
    "shortconv.out_proj.weight", "ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "ffn_gate_inp.weight",
    "ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight", "exp_probs_b.bias",
]
(ATTN_NORM, FFN_NORM, WQ, WK, WV, WO, Q_NORM, K_NORM, CONV, IN_PROJ, OUT_PROJ, FFN_GATE, FFN_UP, FFN_DOWN, ROUTER,
 GATE_EXPS, UP_EXPS, DOWN_EXPS, EXP_BIAS) = range(19)


class Tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4)]


class Layer(C.Structure):
    _fields_ = [("is_attn", C.c_int32), ("is_moe", C.c_int32), ("t", Tensor * len(SLOTS))]


class ModelDesc(C.Structure):
    _fields_ = [("arch", C.c_int32), ("n_layers", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
                ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("n_vocab", C.c_int32), ("n_expert", C.c_int32),
                ("n_expert_used", C.c_int32), ("max_ctx", C.c_int32), ("rms_eps", C.c_double),
                ("rope_base", C.c_double), ("tok_embd", Tensor), ("output_norm", Tensor), ("output", Tensor),
                ("layers", C.POINTER(Layer))]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        L = C.CDLL(str(LIB))
        P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.POINTER(C.c_float)
        sigs = {
            "orc_set_threads": (None, [I]), "orc_get_threads": (I, []),
            "orc_f16_to_double": (C.c_double, [C.c_uint16]),
            "orc_matmul": (None, [C.POINTER(Tensor), P, P]),
            "orc_matmul_rows": (None, [C.POINTER(Tensor), P, I64, P]),
            "orc_embedding": (None, [C.POINTER(Tensor), C.c_int32, P]),
            "orc_dequant": (None, [C.POINTER(Tensor), P]),
            "orc_rmsnorm": (None, [P, I64, C.POINTER(Tensor), C.c_double]),
            "orc_per_head_rmsnorm": (None, [P, I, I, C.POINTER(Tensor), C.c_double]),
            "orc_rope": (None, [P, I, I, I, C.c_double]),
            "orc_softmax": (None, [P, I64, I64]),
            "orc_silu": (None, [P, I64]), "orc_mul": (None, [P, P, I64]), "orc_add": (None, [P, P, I64]),
            "orc_sample_greedy": (C.c_int32, [P, I64]),
            "orc_sample_suppress": (C.c_int32, [P, I64, C.c_int32]),
            "orc_lfm2_moe": (None, [C.POINTER(Layer), I, I, I, P, I64, P, P, P]),
            "orc_model_create": (I, [C.POINTER(ModelDesc), C.POINTER(P)]),
            "orc_model_destroy": (None, [P]), "orc_reset": (None, [P]),
            "orc_set_expert_mask": (I, [P, C.POINTER(C.c_int32), I]),
            "orc_forward": (I, [P, C.c_int32, C.c_int32, I, P, P, P]),
            "orc_generate": (I, [P, C.POINTER(C.c_int32), I, I, C.c_int32, C.c_int32, C.POINTER(C.c_int32)]),
            "orc_n_moe_layers": (I, [P]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def make_tensor(raw: np.ndarray | None, ggml_type: int = 0, ne=(1,)) -> Tensor:
    t = Tensor()
    if raw is None:
        t.data = None
        return t
    t.data = raw.ctypes.data
    t.type = ggml_type
    t.n_dims = len(ne)
    for i in range(4):
        t.ne[i] = int(ne[i]) if i < len(ne) else 1
    return t


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- per-op wrappers ---------------------------------------------------------------

def matmul(raw: np.ndarray, ggml_type: int, ne, x: np.ndarray) -> np.ndarray:
    """M independent matmulGeneric calls: x [M, K] -> [M, N]."""
    t = make_tensor(raw, ggml_type, ne)
    x = _f32(x).reshape(-1, int(ne[0]))
    y = np.empty((x.shape[0], int(ne[1])), dtype=np.float32)
    lib().orc_matmul_rows(C.byref(t), x.ctypes.data, x.shape[0], y.ctypes.data)
    return y


def dequant(raw: np.ndarray, ggml_type: int, ne) -> np.ndarray:
    t = make_tensor(raw, ggml_type, ne)
    out = np.empty(int(np.prod(ne)), dtype=np.float32)
    lib().orc_dequant(C.byref(t), out.ctypes.data)
    return out


def embedding(raw, ne, token: int) -> np.ndarray:
    t = make_tensor(raw, 8, ne)
    out = np.empty(int(ne[0]), dtype=np.float32)
    lib().orc_embedding(C.byref(t), token, out.ctypes.data)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = _f32(x).copy()
    w = _f32(w)
    t = make_tensor(w.view(np.uint8), 0, (w.size,))
    for r in x.reshape(-1, w.size):
        lib().orc_rmsnorm(r.ctypes.data, w.size, C.byref(t), eps)
    return x


def rope(x: np.ndarray, n_heads: int, head_dim: int, pos: int, base: float) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_rope(x.ctypes.data, n_heads, head_dim, pos, base)
    return x


def softmax(x: np.ndarray) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_softmax(x.ctypes.data, 0, x.size)
    return x


def silu(x):
    x = _f32(x).copy()
    lib().orc_silu(x.ctypes.data, x.size)
    return x


def sample_greedy(logits) -> int:
    x = _f32(logits)
    return int(lib().orc_sample_greedy(x.ctypes.data, x.size))


def lfm2_moe(layer_tensors: dict, n_embd: int, n_expert: int, top_k: int, x: np.ndarray, mask=None):
    """Lfm2Engine._moEFFN on rows of x (already ffn-normalised). Returns (out, routing)."""
    L = Layer()
    keep = []
    for slot, name in enumerate(SLOTS):
        if name in layer_tensors:
            t, ne, raw = layer_tensors[name]
            keep.append(raw)
            L.t[slot] = make_tensor(raw, t, ne)
    x = _f32(x).reshape(-1, n_embd)
    T = x.shape[0]
    out = np.empty_like(x)
    rec = np.empty((T, 2 * top_k + n_expert), dtype=np.float32)
    m = None
    if mask:
        m = np.zeros(n_expert, dtype=np.uint8)
        m[list(mask)] = 1
    lib().orc_lfm2_moe(C.byref(L), n_embd, n_expert, top_k, x.ctypes.data, T, out.ctypes.data, rec.ctypes.data,
                       m.ctypes.data if m is not None else None)
    return out, rec


# ---- model -------------------------------------------------------------------------

class OracleModel:
    """Qwen3Engine / Lfm2Engine restated in C, bound to the tensors of a GGUF reader."""

    def __init__(self, gguf, max_ctx: int = 4096, threads: int | None = None):
        if threads is not None:
            set_threads(threads)
        arch = gguf.getKeyValue("general.architecture", "")
        self.lfm2 = arch.startswith("lfm2")
        a = arch + "."
        kv = lambda k, d=None: gguf.getKeyValue(a + k, d)  # noqa: E731
        n_layers = int(kv("block_count"))
        emb = gguf.getTensorMetaByName("token_embd.weight")
        n_embd, n_vocab = int(emb.shape[0]), int(emb.shape[1])
        n_head = int(kv("attention.head_count"))
        hkv = kv("attention.head_count_kv")
        n_head_kv = max(v for v in hkv if v > 0) if isinstance(hkv, list) else int(hkv or n_head)
        self._keep = []

        def T(name):
            m = gguf.getTensorMetaByName(name)
            if m is None:
                return make_tensor(None)
            raw = np.ascontiguousarray(m.raw())
            self._keep.append(raw)
            return make_tensor(raw, m.type, m.shape)

        layers = (Layer * n_layers)()
        head_dim = None
        n_expert = int(kv("expert_count", 0) or 0)
        n_used = int(kv("expert_used_count", 0) or 0)
        for i in range(n_layers):
            L = layers[i]
            for s, name in enumerate(SLOTS):
                L.t[s] = T(f"blk.{i}.{name}")
            L.is_attn = 0 if L.t[CONV].data else 1
            L.is_moe = 1 if L.t[ROUTER].data else 0
            if L.is_attn and head_dim is None:
                head_dim = int(L.t[WQ].ne[1]) // n_head
        d = ModelDesc()
        d.arch = 1 if self.lfm2 else 0
        d.n_layers, d.n_embd, d.n_head, d.n_head_kv = n_layers, n_embd, n_head, n_head_kv
        d.head_dim = head_dim or 64
        d.n_vocab = n_vocab
        d.n_expert, d.n_expert_used = n_expert, n_used
        d.max_ctx = max_ctx
        d.rms_eps = float(kv("attention.layer_norm_rms_epsilon") or (1e-5 if self.lfm2 else 1e-6))
        d.rope_base = float(kv("rope.freq_base") or kv("rope_freq_base") or (5e6 if self.lfm2 else 1e4))
        d.tok_embd = T("token_embd.weight")
        d.output_norm = T("token_embd_norm.weight" if self.lfm2 else "output_norm.weight")
        d.output = T("output.weight")
        d.layers = C.cast(layers, C.POINTER(Layer))
        self._layers = layers
        self.desc = d
        h = C.c_void_p()
        rc = lib().orc_model_create(C.byref(d), C.byref(h))
        if rc:
            raise RuntimeError(f"orc_model_create failed: {rc}")
        self.h = h
        self.n_layers, self.n_embd, self.n_vocab = n_layers, n_embd, n_vocab
        self.n_expert, self.n_used = n_expert, n_used
        self.n_moe = lib().orc_n_moe_layers(h)

    def __del__(self):
        try:
            if getattr(self, "h", None) and _lib is not None:
                _lib.orc_model_destroy(self.h)
        except Exception:
            pass
        self.h = None

    def reset(self):
        lib().orc_reset(self.h)

    def set_expert_mask(self, ids):
        a = np.asarray(sorted(ids), dtype=np.int32)
        lib().orc_set_expert_mask(self.h, a.ctypes.data_as(C.POINTER(C.c_int32)), len(a))

    def forward(self, token: int, pos: int, skip_logits: bool = False, dump: bool = False, routing: bool = False):
        logits = None if skip_logits else np.empty(self.n_vocab, dtype=np.float32)
        hd = np.empty((self.n_layers, self.n_embd), dtype=np.float32) if dump else None
        rec = np.empty((max(self.n_moe, 1), 2 * self.n_used + self.n_expert), dtype=np.float32) if routing else None
        rc = lib().orc_forward(self.h, token, pos, 1 if skip_logits else 0,
                               logits.ctypes.data if logits is not None else None,
                               hd.ctypes.data if hd is not None else None,
                               rec.ctypes.data if rec is not None else None)
        if rc:
            raise RuntimeError(f"orc_forward failed: {rc}")
        if dump or routing:
            return logits, hd, rec
        return logits

    def generate(self, prompt, max_steps: int, think_id: int = -1, eos_id: int = -1) -> np.ndarray:
        p = np.asarray(prompt, dtype=np.int32)
        out = np.empty(max(max_steps, 1), dtype=np.int32)
        n = lib().orc_generate(self.h, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p), max_steps, think_id, eos_id,
                               out.ctypes.data_as(C.POINTER(C.c_int32)))
        if n < 0:
            raise RuntimeError(f"orc_generate failed: {n}")
        return out[:n]
