"""ctypes binding of libqq3cuda.so (declared in include/qq3.h).

This is the Python twin of the N-API addon a Node host would load: it calls the C ABI
with plain pointers and sizes.  There is no CPU fallback -- if the library or a B200 is
missing, opening a context raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import build as _build

QQ_OK = 0
QQ_ERR_INVALID = -1
QQ_ERR_CUDA = -2
QQ_ERR_OOM = -3
QQ_ERR_UNSUPPORTED = -4

QQ_TYPE_F32 = 0
QQ_TYPE_Q8_0 = 8

QQ_ARCH_QWEN3 = 0
QQ_ARCH_LFM2 = 1

# per-layer tensor slots (include/qq3.h)
SLOTS = [
    "attn_norm", "ffn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm",
    "shortconv.conv", "shortconv.in_proj", "shortconv.out_proj", "ffn_gate", "ffn_up", "ffn_down",
    "ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps", "exp_probs_b",
]
SLOT_COUNT = len(SLOTS)
SLOT = {name: i for i, name in enumerate(SLOTS)}

# GGUF tensor name of each slot for layer N (qwen3-engine.js:46-75, lfm2-engine.js:88-140)
SLOT_TENSOR_NAMES = {
    "attn_norm": "attn_norm.weight", "ffn_norm": "ffn_norm.weight", "attn_q": "attn_q.weight",
    "attn_k": "attn_k.weight", "attn_v": "attn_v.weight", "attn_output": "attn_output.weight",
    "attn_q_norm": "attn_q_norm.weight", "attn_k_norm": "attn_k_norm.weight",
    "shortconv.conv": "shortconv.conv.weight", "shortconv.in_proj": "shortconv.in_proj.weight",
    "shortconv.out_proj": "shortconv.out_proj.weight", "ffn_gate": "ffn_gate.weight", "ffn_up": "ffn_up.weight",
    "ffn_down": "ffn_down.weight", "ffn_gate_inp": "ffn_gate_inp.weight", "ffn_gate_exps": "ffn_gate_exps.weight",
    "ffn_up_exps": "ffn_up_exps.weight", "ffn_down_exps": "ffn_down_exps.weight", "exp_probs_b": "exp_probs_b.bias",
}


class QQError(RuntimeError):
    """A failed qq_* call: .code is the QQ_ERR_* status, the message is qq_last_error()."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


QQ_COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """A new NCCL unique id for qq_comm_init (made on one rank, shared with the others)."""
    buf = C.create_string_buffer(QQ_COMM_ID_BYTES)
    check(load().qq_comm_unique_id(buf))
    return buf.raw


class SampleParams(C.Structure):
    """qq_sample_params: generate()'s sampling options (tensor.js:188-265)."""
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_int32), ("think_mode", C.c_int32),
                ("think_id", C.c_int32), ("end_think_id", C.c_int32), ("seed", C.c_uint64)]


QQ_THINK_SUPPRESS = 0
QQ_THINK_SHORTEN = 1
QQ_THINK_FULL = 2
QQ_SAMPLE_MAX_TOP_K = 1024
THINK_MODES = {"suppress": QQ_THINK_SUPPRESS, "shorten": QQ_THINK_SHORTEN, "full": QQ_THINK_FULL}


def sample_params(temperature: float, top_p: float, top_k: int, think_mode: str = "suppress", think_id: int = -1,
                  end_think_id: int = -1, seed: int = 0) -> SampleParams:
    return SampleParams(float(temperature), float(top_p), int(top_k), THINK_MODES[think_mode], int(think_id),
                        int(end_think_id), int(seed) & 0xFFFFFFFFFFFFFFFF)


def sample_uniform(seed: int, seq: int, pos: int) -> float:
    """The device sampler's uniform draw after the logits of position pos of sequence seq (the
    same splitmix64 finaliser and 53-bit scaling as sample_uniform in csrc/kernels.h)."""
    M = 0xFFFFFFFFFFFFFFFF
    z = (seed & M) ^ ((0x9E3779B97F4A7C15 * ((pos + 1) & 0xFFFFFFFF)) & M) ^ ((0xD1B54A32D192ED03 * ((seq + 1) & 0xFFFFFFFF)) & M)
    z = (z + 0x9E3779B97F4A7C15) & M
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
    z ^= z >> 31
    return (z >> 11) * (1.0 / 9007199254740992.0)


class LayerDesc(C.Structure):
    _fields_ = [("is_attn", C.c_int32), ("is_moe", C.c_int32), ("t", C.c_void_p * SLOT_COUNT)]


class ModelDesc(C.Structure):
    _fields_ = [
        ("arch", C.c_int32), ("n_layers", C.c_int32), ("n_embd", C.c_int32), ("n_head", C.c_int32),
        ("n_head_kv", C.c_int32), ("head_dim", C.c_int32), ("n_vocab", C.c_int32), ("n_expert", C.c_int32),
        ("n_expert_used", C.c_int32), ("max_ctx", C.c_int32), ("n_seq", C.c_int32), ("rms_eps", C.c_float),
        ("rope_base", C.c_double), ("tok_embd", C.c_void_p), ("output_norm", C.c_void_p), ("output", C.c_void_p),
        ("layers", C.POINTER(LayerDesc)), ("ep_world", C.c_int32), ("tp_world", C.c_int32),
    ]


_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64
_SIGS = {
    "qq_last_error": (C.c_char_p, []),
    "qq_init": (_I, [C.POINTER(_I), _I, C.POINTER(_P)]),
    "qq_destroy": (_I, [_P]),
    "qq_set_stream": (_I, [_P, _P]),
    "qq_synchronize": (_I, [_P]),
    "qq_upload_tensor": (_I, [_P, _P, C.c_size_t, _I, C.POINTER(_I64), _I, C.POINTER(_P)]),
    "qq_free_tensor": (_I, [_P]),
    "qq_tensor_info": (_I, [_P, C.POINTER(_I), C.POINTER(_I64), C.POINTER(_I)]),
    "qq_dequant": (_I, [_P, _P]),
    "qq_q8_matmul": (_I, [_P, _P, _P, _I, _P]),
    "qq_rmsnorm": (_I, [_P, _P, _I64, _I, _P, C.c_float, _P]),
    "qq_rope": (_I, [_P, _P, _I, _I, _I, _I, C.c_double]),
    "qq_attention_decode": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "qq_embed": (_I, [_P, _P, C.POINTER(C.c_int32), _I, _P]),
    "qq_swiglu": (_I, [_P, _P, _P, _I64, _P]),
    "qq_add": (_I, [_P, _P, _P, _I64]),
    "qq_model_create": (_I, [_P, C.POINTER(ModelDesc), C.POINTER(_P)]),
    "qq_model_destroy": (_I, [_P]),
    "qq_forward": (_I, [_P, C.POINTER(C.c_int32), _I, _I, _I, _I, _P, C.POINTER(C.c_int32), _I]),
    "qq_forward_batch": (_I, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int32), _I, _I, _P,
                              C.POINTER(C.c_int32), _I]),
    "qq_generate": (_I, [_P, _I, C.POINTER(C.c_int32), _I, _I, _I, _I, C.POINTER(C.c_int32), C.POINTER(_I)]),
    "qq_reset": (_I, [_P, _I]),
    "qq_read_routing": (_I, [_P, _I, _P]),
    "qq_set_expert_mask": (_I, [_P, C.POINTER(C.c_int32), _I]),
    "qq_forward_dump": (_I, [_P, C.c_int32, _I, _I, _P]),
    "qq_decode_loop": (_I, [_P, _I, _I, _I, _I, _I, C.POINTER(C.c_int32)]),
    "qq_moe_block": (_I, [_P, C.POINTER(LayerDesc), _I, _I, _P, _I, _P, _P]),
    "qq_model_stat": (_I, [_P, _I, C.POINTER(_I64)]),
    "qq_bench_kernel": (_I, [_P, _I, _I, C.POINTER(C.c_float)]),
    "qq_moe_block_noalloc": (_I, [_P, C.POINTER(LayerDesc), _I, _I, _P, _I, _P, _P]),
    "qq_comm_unique_id": (_I, [_P]),
    "qq_comm_init": (_I, [_P, _P, _I, _I, _I]),
    "qq_comm_destroy": (_I, [_P]),
    "qq_ep_profile": (_I, [_P, _I, _P]),
    "qq_decode_trace": (_I, [_P, _I, _P, _P, C.POINTER(_I), C.POINTER(_I)]),
    "qq_decode_trace_sub": (_I, [_P, _P, C.POINTER(_I)]),
    "qq_upload_begin": (_I, [_P, C.c_size_t, C.POINTER(_P)]),
    "qq_upload_tensor_async": (_I, [_P, _P, C.c_size_t, _I, C.POINTER(_I64), _I, C.POINTER(_P)]),
    "qq_upload_finish": (_I, [_P, C.POINTER(C.c_size_t)]),
    "qq_forward_sample": (_I, [_P, C.c_int32, _I, _I, C.POINTER(SampleParams), _I, C.POINTER(C.c_int32)]),
    "qq_generate_sample": (_I, [_P, _I, C.POINTER(C.c_int32), _I, _I, C.POINTER(SampleParams), _I,
                                C.POINTER(C.c_int32), C.POINTER(_I)]),
    "qq_sample_logits": (_I, [_P, _P, _I, C.POINTER(SampleParams), C.c_double, _I, C.POINTER(C.c_int32)]),
    "qq_sample_uniform": (_I, [C.c_uint64, _I, _I, C.POINTER(C.c_double)]),
    "qq_moe_route": (_I, [_P, C.POINTER(LayerDesc), _I, _I, _P, _I, _P, _P, _P]),
    "qq_moe_experts": (_I, [_P, C.POINTER(LayerDesc), _I, _P, _P, _I, _P]),
    "qq_moe_combine": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
}

QQ_NOALLOC_MAX_TOKENS = 1024
QQ_NOALLOC_MAX_FF = 4096

QQ_STAT_STEP_KERNELS = 0
QQ_STAT_N_MOE = 1
QQ_STAT_STEP_PHASES = 2
QQ_STAT_MOE_FUSED = 3
QQ_KERN_MOE_LAYER = 0
QQ_KERN_MOE_GATEUP = 1
QQ_KERN_MOE_DOWN = 2

_lib = None


def library_path() -> Path:
    return _build.CUDA_LIB


def load(build_if_missing: bool = False) -> C.CDLL:
    """Load libqq3cuda.so (raises if it is absent: there is no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        if not build_if_missing:
            raise RuntimeError(f"{path} is missing; run qwenqwen3.js_b200/build.py (no CPU fallback exists)")
        _build.build_cuda()
    lib = C.CDLL(str(path))
    for name, (res, args) in _SIGS.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(rc: int) -> None:
    if rc != QQ_OK:
        msg = load().qq_last_error().decode("utf-8", "replace")
        raise QQError(rc, msg)


def _ptr(a) -> int | None:
    """Device pointer of a torch tensor / int, or host pointer of a numpy array."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    raise TypeError(f"cannot take a pointer of {type(a)}")


class Context:
    """qq_ctx on one device."""

    def __init__(self, device: int = 0):
        self.lib = load()
        dev = (C.c_int * 1)(device)
        h = C.c_void_p()
        check(self.lib.qq_init(dev, 1, C.byref(h)))
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            check(self.lib.qq_destroy(self.h))
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # cudaStreamLegacy: the legacy default stream, which torch reports as handle 0
    CUDA_STREAM_LEGACY = 0x1

    def set_stream(self, cuda_stream: int | None) -> None:
        """Run later work on a caller's stream: a cudaStream_t handle (torch's `cuda_stream`),
        where 0 means the legacy default stream (torch's default stream reports 0) and None the
        context's own stream.  (The C ABI reads NULL as the context's own stream.)"""
        if cuda_stream == 0:
            cuda_stream = self.CUDA_STREAM_LEGACY
        check(self.lib.qq_set_stream(self.h, cuda_stream))

    def synchronize(self) -> None:
        check(self.lib.qq_synchronize(self.h))

    def upload(self, raw: np.ndarray, ggml_type: int, ne) -> "Tensor":
        raw = np.ascontiguousarray(raw)
        ne = list(int(v) for v in ne)
        arr = (C.c_int64 * len(ne))(*ne)
        h = C.c_void_p()
        check(self.lib.qq_upload_tensor(self.h, raw.ctypes.data, raw.nbytes, ggml_type, arr, len(ne), C.byref(h)))
        return Tensor(self, h, ggml_type, ne)

    # --- multi-GPU: the context's NCCL communicator (qq_comm_*)
    def comm_init(self, comm_id: bytes, rank: int, world: int, timeout_ms: int = 0) -> None:
        buf = C.create_string_buffer(bytes(comm_id), QQ_COMM_ID_BYTES)
        check(self.lib.qq_comm_init(self.h, buf, rank, world, timeout_ms))
        self._comm = (rank, world)

    def comm_rank(self) -> int:
        if not getattr(self, "_comm", None):
            raise QQError(QQ_ERR_INVALID, "this context has no communicator (comm_init)")
        return self._comm[0]

    def comm_init_from_torch(self, timeout_ms: int = 0) -> None:
        """Communicator over the ranks of the default torch.distributed group: rank 0 makes the
        id, torch.distributed broadcasts it."""
        import torch.distributed as dist

        obj = [comm_unique_id() if dist.get_rank() == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        self.comm_init(obj[0], dist.get_rank(), dist.get_world_size(), timeout_ms)

    def comm_destroy(self) -> None:
        check(self.lib.qq_comm_destroy(self.h))
        self._comm = None

    def streaming_upload(self, staging_bytes: int = 0) -> "Uploader":
        """Upload many tensors through a pinned staging ring (qq_upload_begin .. qq_upload_finish);
        use as a context manager, the tensors are ready when it exits."""
        return Uploader(self, staging_bytes)

    def q8_matmul(self, W: "Tensor", x_dev, M: int, y_dev) -> None:
        check(self.lib.qq_q8_matmul(self.h, W.h, _ptr(x_dev), M, _ptr(y_dev)))

    def rmsnorm(self, x_dev, n_rows: int, n: int, w: "Tensor", eps: float, y_dev) -> None:
        check(self.lib.qq_rmsnorm(self.h, _ptr(x_dev), n_rows, n, w.h, eps, _ptr(y_dev)))

    def rope(self, x_dev, n_rows: int, n_heads: int, head_dim: int, pos0: int, base: float) -> None:
        check(self.lib.qq_rope(self.h, _ptr(x_dev), n_rows, n_heads, head_dim, pos0, base))

    def attention_decode(self, q_dev, k_cache_dev, v_cache_dev, n_head: int, n_kv: int, head_dim: int, max_ctx: int,
                         pos: int, out_dev) -> None:
        check(self.lib.qq_attention_decode(self.h, _ptr(q_dev), _ptr(k_cache_dev), _ptr(v_cache_dev), n_head, n_kv,
                                           head_dim, max_ctx, pos, _ptr(out_dev)))

    def embed(self, E: "Tensor", tokens, out_dev) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        check(self.lib.qq_embed(self.h, E.h, t.ctypes.data_as(C.POINTER(C.c_int32)), len(t), _ptr(out_dev)))

    def swiglu(self, g_dev, u_dev, n: int, h_dev) -> None:
        check(self.lib.qq_swiglu(self.h, _ptr(g_dev), _ptr(u_dev), n, _ptr(h_dev)))

    def add(self, x_dev, d_dev, n: int) -> None:
        check(self.lib.qq_add(self.h, _ptr(x_dev), _ptr(d_dev), n))

    def moe_block(self, layer: LayerDesc, n_expert: int, top_k: int, x_dev, T: int, out_dev, routing_dev=None) -> None:
        check(self.lib.qq_moe_block(self.h, C.byref(layer), n_expert, top_k, _ptr(x_dev), T, _ptr(out_dev),
                                    _ptr(routing_dev)))


    def moe_block_noalloc(self, layer: LayerDesc, n_expert: int, top_k: int, x_dev, T: int, out_dev,
                          routing_dev=None) -> None:
        """qq_moe_block without device allocation (scratch in the library's fixed device array)."""
        check(self.lib.qq_moe_block_noalloc(self.h, C.byref(layer), n_expert, top_k, _ptr(x_dev), T, _ptr(out_dev),
                                            _ptr(routing_dev)))

    def sample_logits(self, logits_dev, n: int, params: SampleParams, r: float, think_done: bool = False) -> int:
        """sampleWithThinkControl on device logits with the uniform draw r (qq_sample_logits)."""
        tok = C.c_int32(-1)
        check(self.lib.qq_sample_logits(self.h, _ptr(logits_dev), n, C.byref(params), float(r),
                                        1 if think_done else 0, C.byref(tok)))
        return tok.value

    # expert-parallel pieces of the MoE block (device pointers; see include/qq3.h)
    def moe_route(self, layer: LayerDesc, n_expert: int, top_k: int, x_dev, T: int, idx_dev, w_dev,
                  routing_dev=None) -> None:
        check(self.lib.qq_moe_route(self.h, C.byref(layer), n_expert, top_k, _ptr(x_dev), T, _ptr(idx_dev),
                                    _ptr(w_dev), _ptr(routing_dev)))

    def moe_experts(self, layer: LayerDesc, n_local: int, x_dev, eid_dev, R: int, y_dev) -> None:
        check(self.lib.qq_moe_experts(self.h, C.byref(layer), n_local, _ptr(x_dev), _ptr(eid_dev), R, _ptr(y_dev)))

    def moe_combine(self, y_dev, pos_dev, w_dev, T: int, top_k: int, K: int, out_dev) -> None:
        check(self.lib.qq_moe_combine(self.h, _ptr(y_dev), _ptr(pos_dev), _ptr(w_dev), T, top_k, K, _ptr(out_dev)))


class Tensor:
    """An uploaded tensor (qq_tensor)."""

    def __init__(self, ctx: Context, h, ggml_type: int, ne):
        self.ctx = ctx
        self.h = h
        self.type = ggml_type
        self.ne = list(ne)

    @property
    def numel(self) -> int:
        return int(np.prod(self.ne))

    def info(self):
        t = C.c_int()
        ne = (C.c_int64 * 4)()
        nd = C.c_int()
        check(self.ctx.lib.qq_tensor_info(self.h, C.byref(t), ne, C.byref(nd)))
        return t.value, list(ne)[: nd.value]

    def dequant(self, out_dev) -> None:
        check(self.ctx.lib.qq_dequant(self.h, _ptr(out_dev)))

    def free(self) -> None:
        if self.h:
            check(self.ctx.lib.qq_free_tensor(self.h))
            self.h = C.c_void_p()

    def __del__(self):
        try:
            if self.h and self.ctx.h:
                self.free()
        except Exception:
            pass


class Uploader:
    """qq_uploader: streaming upload of many tensors (see Context.streaming_upload)."""

    def __init__(self, ctx: "Context", staging_bytes: int = 0):
        self.ctx = ctx
        self.h = C.c_void_p()
        self.bytes = 0
        check(ctx.lib.qq_upload_begin(ctx.h, staging_bytes, C.byref(self.h)))

    def upload(self, raw: np.ndarray, ggml_type: int, ne) -> "Tensor":
        raw = np.ascontiguousarray(raw)
        ne = list(int(v) for v in ne)
        arr = (C.c_int64 * len(ne))(*ne)
        h = C.c_void_p()
        check(self.ctx.lib.qq_upload_tensor_async(self.h, raw.ctypes.data, raw.nbytes, ggml_type, arr, len(ne),
                                                  C.byref(h)))
        return Tensor(self.ctx, h, ggml_type, ne)

    def finish(self) -> int:
        if self.h:
            n = C.c_size_t(0)
            h, self.h = self.h, C.c_void_p()
            check(self.ctx.lib.qq_upload_finish(h, C.byref(n)))
            self.bytes = n.value
        return self.bytes

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.finish()


class Model:
    """qq_model: an engine over uploaded tensors."""

    def __init__(self, ctx: Context, desc: ModelDesc, layers_arr, keepalive):
        self.ctx = ctx
        self.desc = desc
        self._layers = layers_arr
        self._keep = keepalive
        h = C.c_void_p()
        check(ctx.lib.qq_model_create(ctx.h, C.byref(desc), C.byref(h)))
        self.h = h
        self.n_vocab = desc.n_vocab
        self.n_layers = desc.n_layers
        self.n_embd = desc.n_embd
        # reusable ctypes arguments of forward_argmax (one greedy token per call)
        self._tok1 = (C.c_int32 * 1)()
        self._am1 = C.c_int32(-1)
        self._am1_ref = C.byref(self._am1)

    def close(self) -> None:
        if self.h:
            check(self.ctx.lib.qq_model_destroy(self.h))
            self.h = C.c_void_p()

    def __del__(self):
        try:
            if self.h and self.ctx.h:
                self.close()
        except Exception:
            pass

    def forward(self, tokens, seq: int = 0, pos0: int = 0, want_logits: bool = True, logits: bool = True,
                suppress_id: int = -1):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32).reshape(-1))
        out = np.empty(self.n_vocab, dtype=np.float32) if (want_logits and logits) else None
        am = C.c_int32(-1)
        check(self.ctx.lib.qq_forward(self.h, toks.ctypes.data_as(C.POINTER(C.c_int32)), len(toks), seq, pos0,
                                      1 if want_logits else 0, _ptr(out), C.byref(am) if want_logits else None,
                                      suppress_id))
        return out, am.value

    def forward_argmax(self, token: int, seq: int = 0, pos: int = 0, suppress_id: int = -1) -> int:
        """One token with the device greedy id (qq_forward with want_logits and no logits copy),
        without per-call array allocations."""
        self._tok1[0] = token
        check(self.ctx.lib.qq_forward(self.h, self._tok1, 1, seq, pos, 1, None, self._am1_ref, suppress_id))
        return self._am1.value

    def forward_batch(self, seqs, tokens, positions, want_logits: bool = True, logits: bool = True,
                      suppress_id: int = -1):
        """One step of each sequence seqs[i] (token tokens[i] at positions[i]); returns
        (logits [n][n_vocab] or None, greedy ids [n] or None)."""
        i32 = lambda a: np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))  # noqa: E731
        sq, tk, ps = i32(seqs), i32(tokens), i32(positions)
        n = len(sq)
        if len(tk) != n or len(ps) != n:
            raise ValueError("forward_batch: seqs, tokens and positions differ in length")
        out = np.empty((n, self.n_vocab), dtype=np.float32) if (want_logits and logits) else None
        am = np.full(n, -1, dtype=np.int32) if want_logits else None
        p32 = lambda a: a.ctypes.data_as(C.POINTER(C.c_int32))  # noqa: E731
        check(self.ctx.lib.qq_forward_batch(self.h, p32(sq), p32(tk), p32(ps), n, 1 if want_logits else 0,
                                            _ptr(out), p32(am) if am is not None else None, suppress_id))
        return out, am

    def forward_dump(self, token: int, seq: int, pos: int) -> np.ndarray:
        out = np.empty((self.n_layers, self.n_embd), dtype=np.float32)
        check(self.ctx.lib.qq_forward_dump(self.h, token, seq, pos, out.ctypes.data))
        return out

    def decode_loop(self, first_token: int, pos0: int, n_steps: int, seq: int = 0, suppress_id: int = -1,
                    want_tokens: bool = True):
        out = np.empty(max(n_steps, 1), dtype=np.int32) if want_tokens else None
        check(self.ctx.lib.qq_decode_loop(self.h, seq, first_token, pos0, n_steps, suppress_id,
                                          out.ctypes.data_as(C.POINTER(C.c_int32)) if want_tokens else None))
        return out[:n_steps] if want_tokens else None

    def generate(self, prompt, max_steps: int, think_id: int = -1, eos_id: int = -1, seq: int = 0) -> np.ndarray:
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.empty(max(max_steps, 1), dtype=np.int32)
        n = C.c_int(0)
        check(self.ctx.lib.qq_generate(self.h, seq, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p), max_steps,
                                       think_id, eos_id, out.ctypes.data_as(C.POINTER(C.c_int32)), C.byref(n)))
        return out[: n.value]

    def generate_sample(self, prompt, max_steps: int, params: SampleParams, eos_id: int = -1,
                        seq: int = 0) -> np.ndarray:
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.empty(max(max_steps, 1), dtype=np.int32)
        n = C.c_int(0)
        check(self.ctx.lib.qq_generate_sample(self.h, seq, p.ctypes.data_as(C.POINTER(C.c_int32)), len(p), max_steps,
                                              C.byref(params), eos_id, out.ctypes.data_as(C.POINTER(C.c_int32)),
                                              C.byref(n)))
        return out[: n.value]

    def forward_sample(self, token: int, pos: int, params: SampleParams, think_done: bool = False,
                       seq: int = 0) -> int:
        tok = C.c_int32(-1)
        check(self.ctx.lib.qq_forward_sample(self.h, int(token), seq, pos, C.byref(params), 1 if think_done else 0,
                                             C.byref(tok)))
        return tok.value

    def reset(self, seq: int = 0) -> None:
        check(self.ctx.lib.qq_reset(self.h, seq))

    def read_routing(self, moe_layer: int, rec_len: int) -> np.ndarray:
        out = np.empty(rec_len, dtype=np.float32)
        check(self.ctx.lib.qq_read_routing(self.h, moe_layer, out.ctypes.data))
        return out

    def stat(self, what: int) -> int:
        v = C.c_int64(0)
        check(self.ctx.lib.qq_model_stat(self.h, what, C.byref(v)))
        return v.value

    def bench_kernel(self, what: int, iters: int) -> float:
        ms = C.c_float(0)
        check(self.ctx.lib.qq_bench_kernel(self.h, what, iters, C.byref(ms)))
        return ms.value

    def decode_trace(self, enable: bool, read: bool = False):
        """Switch the per-phase %globaltimer trace of the persistent step; with read, return
        (stamps [n_ctas][n_phases + 1] ns of the last traced step, phase kinds [n_phases])."""
        np_, nc = C.c_int(0), C.c_int(0)
        check(self.ctx.lib.qq_decode_trace(self.h, 1 if enable else 0, None, None, C.byref(np_), C.byref(nc)))
        if not read:
            return None
        st = np.zeros((nc.value, np_.value + 1), dtype=np.uint64)
        kinds = np.zeros(np_.value, dtype=np.int32)
        check(self.ctx.lib.qq_decode_trace(self.h, 1 if enable else 0, st.ctypes.data, kinds.ctypes.data,
                                           C.byref(np_), C.byref(nc)))
        return st, kinds

    def decode_trace_sub(self):
        """Sub-phase stamps of the last traced step: [n_ctas][n_phases][n_sub] ns (0 where a phase
        does not reach a point; the points are listed at qq_decode_trace_sub in qq3.h)."""
        np_, nc, ns = C.c_int(0), C.c_int(0), C.c_int(0)
        check(self.ctx.lib.qq_decode_trace(self.h, 0, None, None, C.byref(np_), C.byref(nc)))
        check(self.ctx.lib.qq_decode_trace_sub(self.h, None, C.byref(ns)))
        out = np.zeros((nc.value, np_.value, ns.value), dtype=np.uint64)
        check(self.ctx.lib.qq_decode_trace_sub(self.h, out.ctypes.data, C.byref(ns)))
        return out

    def ep_profile(self, enable: bool):
        """Switch the per-exchange CUDA-event split on/off; returns the split summed since the
        last call: dict(dispatch, experts, ret, combine) in ms and the exchange count."""
        out = (C.c_float * 5)()
        check(self.ctx.lib.qq_ep_profile(self.h, 1 if enable else 0, out))
        return dict(dispatch=out[0], experts=out[1], ret=out[2], combine=out[3], exchanges=int(out[4]))

    def set_expert_mask(self, ids) -> None:
        ids = np.ascontiguousarray(np.asarray(sorted(ids), dtype=np.int32))
        check(self.ctx.lib.qq_set_expert_mask(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), len(ids)))
