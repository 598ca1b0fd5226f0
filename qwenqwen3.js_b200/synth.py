"""Seeded random-init Q8_0 models in the GGUF layout the reference engines read.

No checkpoints exist on these machines, so every model is generated from a seed:
  * Q8_0 weights: qs ~ U{-127..127}; fp16 scale d = 0.02/127 * |N(1, 0.1)| (model configs)
    or |N(0, 0.02)|/127 (the isolated matmul sweep);
  * norm weights: F32 ones;
  * LFM2 short-conv kernels: F32 N(0, 0.1) (stored F32: ggml Q8_0 needs ne0 % 32 == 0 and
    the kernel's ne0 is 3, lfm2-engine.js:146-179);
  * LFM2 expert-selection bias exp_probs_b: alpha * log(zipf_pmf(rank(e))) over a seeded
    rank permutation, alpha calibrated per layer so that the top-k selection frequencies of
    2048 N(0,1) tokens through that layer's router fit Zipf(s=1.1).
Tensor names, shapes and metadata keys are the ones qwen3-engine.js:31-76,
lfm2-engine.js:15-141 and gguf.js getArch (:264-291) look up.

The byte generator is libqq3synth.so (counter-based, any slice reproducible).
"""
from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass, field

import numpy as np

from . import build as _build
from .gguf import KV_TYPES, TYPE_F32, TYPE_Q8_0, GGUFWriter, TensorMeta, tensor_nbytes

_synth = None


def _lib():
    global _synth
    if _synth is None:
        path = _build.SYNTH_LIB
        if not path.exists():
            _build.build_synth()
        lib = C.CDLL(str(path))
        lib.qq_synth_q8_0.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_uint64, C.c_int, C.c_double, C.c_double]
        lib.qq_synth_normal_f32.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_uint64, C.c_double, C.c_double]
        lib.qq_synth_uniform_i32.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_int64, C.c_int64]
        lib.qq_synth_f32_to_f16.argtypes = [C.c_float]
        lib.qq_synth_f32_to_f16.restype = C.c_uint16
        _synth = lib
    return _synth


def q8_0_blocks(n_elems: int, seed: int, mode: int = 0, block0: int = 0) -> np.ndarray:
    """Raw Q8_0 stream for n_elems values (n_elems % 32 == 0), as uint8 [n_blocks*34]."""
    assert n_elems % 32 == 0
    nb = n_elems // 32
    out = np.empty(nb * 34, dtype=np.uint8)
    if mode == 0:
        _lib().qq_synth_q8_0(out.ctypes.data, nb, block0, seed, 0, 0.02, 0.1)
    else:
        _lib().qq_synth_q8_0(out.ctypes.data, nb, block0, seed, 1, 0.02, 0.0)
    return out


def normal_f32(n: int, seed: int, mean: float = 0.0, std: float = 1.0, i0: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _lib().qq_synth_normal_f32(out.ctypes.data, n, i0, seed, mean, std)
    return out


def uniform_tokens(n: int, seed: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    _lib().qq_synth_uniform_i32(out.ctypes.data, n, seed, 0, vocab)
    return out


def f32_to_f16_bits(x: float) -> int:
    return int(_lib().qq_synth_f32_to_f16(float(x)))


def dequant_q8_0(raw: np.ndarray, n_elems: int) -> np.ndarray:
    """q*d in storage order (float32, exact) -- numpy twin of the device dequant."""
    blk = raw[: (n_elems // 32) * 34].reshape(-1, 34)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    q = blk[:, 2:].view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)


def tensor_seed(base: int, name: str) -> int:
    return (base * 1000003 + zlib.crc32(name.encode())) & 0xFFFFFFFFFFFFFFFF


@dataclass
class ModelSpec:
    arch: str  # "qwen3" | "lfm2moe"
    n_layers: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_vocab: int
    n_ff: int
    rope_base: float
    eps: float
    context_length: int = 40960
    tied: bool = True
    attn_layers: tuple = ()
    n_expert: int = 0
    n_expert_used: int = 0
    n_ff_exp: int = 0
    n_dense_lead: int = 0
    seed: int = 1234
    zipf_s: float = 1.1
    router_f32: bool = False  # Qwen3-MoE GGUFs store the router as F32
    name: str = ""
    extra: dict = field(default_factory=dict)

    def is_attn(self, i: int) -> bool:
        return self.arch in ("qwen3", "qwen3moe") or i in self.attn_layers

    def is_moe(self, i: int) -> bool:
        return self.arch in ("lfm2moe", "qwen3moe") and self.n_expert > 0 and i >= self.n_dense_lead


def qwen3_0p6b(seed: int = 1234) -> ModelSpec:
    """benchmark config 1: Qwen3-0.6B architecture."""
    return ModelSpec("qwen3", 28, 1024, 16, 8, 128, 151936, 3072, 1e6, 1e-6, seed=seed, name="Qwen3-0.6B")


def qwen3_8b(seed: int = 1234) -> ModelSpec:
    """benchmark config 5: Qwen3-8B-shaped, untied embeddings."""
    return ModelSpec("qwen3", 36, 4096, 32, 8, 128, 151936, 12288, 1e6, 1e-6, tied=False, seed=seed, name="Qwen3-8B")


LFM2_8B_ATTN_LAYERS = (2, 6, 10, 14, 18, 21)


def lfm2_8b_a1b(seed: int = 1234) -> ModelSpec:
    """benchmark config 4: LFM2-8B-A1B-shaped hybrid MoE (18 short-conv + 6 attention layers)."""
    return ModelSpec("lfm2moe", 24, 2048, 32, 8, 64, 65536, 7168, 1e6, 1e-5, context_length=128000,
                     attn_layers=LFM2_8B_ATTN_LAYERS, n_expert=32, n_expert_used=4, n_ff_exp=1792, n_dense_lead=2,
                     seed=seed, name="LFM2-8B-A1B")


def tiny_qwen3(seed: int = 7) -> ModelSpec:
    return ModelSpec("qwen3", 3, 256, 4, 2, 128, 1024, 512, 1e6, 1e-6, seed=seed, name="tiny-qwen3")


def tiny_qwen3moe(seed: int = 7, router_f32: bool = False) -> ModelSpec:
    """A small Qwen3-MoE (softmax-routed): 128 experts, top-8, as Qwen3-30B-A3B routes."""
    return ModelSpec("qwen3moe", 3, 256, 4, 2, 64, 1024, 512, 1e6, 1e-6, n_expert=128, n_expert_used=8, n_ff_exp=64,
                     router_f32=router_f32, seed=seed, name="tiny-qwen3moe")


def tiny_lfm2(seed: int = 7, n_layers: int = 6) -> ModelSpec:
    return ModelSpec("lfm2moe", n_layers, 256, 4, 2, 64, 768, 512, 1e6, 1e-5, context_length=128000,
                     attn_layers=(2, 5), n_expert=8, n_expert_used=4, n_ff_exp=128, n_dense_lead=2, seed=seed,
                     name="tiny-lfm2")


def tensor_specs(spec: ModelSpec) -> list[tuple[str, int, list]]:
    """(name, ggml type, ne) of every tensor, in file order."""
    E, V, hd = spec.n_embd, spec.n_vocab, spec.head_dim
    nq, nkv = spec.n_head * hd, spec.n_head_kv * hd
    out = [("token_embd.weight", TYPE_Q8_0, [E, V])]
    if spec.arch in ("qwen3", "qwen3moe"):
        out.append(("output_norm.weight", TYPE_F32, [E]))
    else:
        out.append(("token_embd_norm.weight", TYPE_F32, [E]))
    if not spec.tied:
        out.append(("output.weight", TYPE_Q8_0, [E, V]))
    for i in range(spec.n_layers):
        b = f"blk.{i}."
        out += [(b + "attn_norm.weight", TYPE_F32, [E]), (b + "ffn_norm.weight", TYPE_F32, [E])]
        if spec.is_attn(i):
            out += [(b + "attn_q.weight", TYPE_Q8_0, [E, nq]), (b + "attn_k.weight", TYPE_Q8_0, [E, nkv]),
                    (b + "attn_v.weight", TYPE_Q8_0, [E, nkv]), (b + "attn_output.weight", TYPE_Q8_0, [nq, E]),
                    (b + "attn_q_norm.weight", TYPE_F32, [hd]), (b + "attn_k_norm.weight", TYPE_F32, [hd])]
        else:
            out += [(b + "shortconv.conv.weight", TYPE_F32, [3, E]),
                    (b + "shortconv.in_proj.weight", TYPE_Q8_0, [E, 3 * E]),
                    (b + "shortconv.out_proj.weight", TYPE_Q8_0, [E, E])]
        if spec.is_moe(i):
            F, NE = spec.n_ff_exp, spec.n_expert
            out += [(b + "ffn_gate_inp.weight", TYPE_F32 if spec.router_f32 else TYPE_Q8_0, [E, NE]),
                    (b + "ffn_gate_exps.weight", TYPE_Q8_0, [E, F, NE]),
                    (b + "ffn_up_exps.weight", TYPE_Q8_0, [E, F, NE]),
                    (b + "ffn_down_exps.weight", TYPE_Q8_0, [F, E, NE])]
            if spec.arch == "lfm2moe":  # the Qwen3-MoE router has no selection bias
                out.append((b + "exp_probs_b.bias", TYPE_F32, [NE]))
        else:
            F = spec.n_ff
            out += [(b + "ffn_gate.weight", TYPE_Q8_0, [E, F]), (b + "ffn_up.weight", TYPE_Q8_0, [E, F]),
                    (b + "ffn_down.weight", TYPE_Q8_0, [F, E])]
    return out


def zipf_bias(router_raw: np.ndarray, n_embd: int, n_expert: int, top_k: int, seed: int, s: float = 1.1,
              n_tokens: int = 2048) -> tuple[np.ndarray, float]:
    """exp_probs_b for one layer: alpha * log(zipf_pmf(rank)), alpha fitted to Zipf(s) top-k frequencies."""
    W = dequant_q8_0(router_raw, n_embd * n_expert).reshape(n_expert, n_embd).astype(np.float64)
    X = normal_f32(n_tokens * n_embd, seed ^ 0x5EED).reshape(n_tokens, n_embd).astype(np.float64)
    X /= np.sqrt((X * X).mean(axis=1, keepdims=True))  # tokens as RMS-normalised router inputs
    p = 1.0 / (1.0 + np.exp(-(X @ W.T)))
    ranks = np.argsort(normal_f32(n_expert, seed ^ 0xA11CE)).argsort() + 1  # seeded permutation, ranks 1..E
    pmf = ranks.astype(np.float64) ** (-s)
    pmf /= pmf.sum()
    logpmf = np.log(pmf)
    best = (np.inf, 0.0)
    for alpha in np.linspace(0.0, 0.5, 201):
        sel = (p + alpha * logpmf).astype(np.float32)
        top = np.argsort(-sel, axis=1, kind="stable")[:, :top_k]
        freq = np.bincount(top.reshape(-1), minlength=n_expert) / top.size
        err = np.abs(freq - pmf).sum()
        if err < best[0]:
            best = (err, alpha)
    alpha = best[1]
    return (alpha * logpmf).astype(np.float32), float(alpha)


def generate_tensor(spec: ModelSpec, name: str, ggml_type: int, ne, cache: dict | None = None) -> np.ndarray:
    """Raw bytes of one tensor."""
    seed = tensor_seed(spec.seed, name)
    n = int(np.prod(ne))
    if name.endswith("exp_probs_b.bias"):
        layer = name.split(".")[1]
        rname = f"blk.{layer}.ffn_gate_inp.weight"
        rraw = cache.get(rname) if cache else None
        if rraw is None:
            rraw = q8_0_blocks(spec.n_embd * spec.n_expert, tensor_seed(spec.seed, rname))
        bias, alpha = zipf_bias(rraw, spec.n_embd, spec.n_expert, spec.n_expert_used, seed, spec.zipf_s)
        spec.extra.setdefault("zipf_alpha", {})[name] = alpha
        return bias.view(np.uint8)
    if ggml_type == TYPE_Q8_0:
        return q8_0_blocks(n, seed, 0)
    if name.endswith("ffn_gate_inp.weight"):  # an F32 router
        return normal_f32(n, seed, 0.0, 0.05).view(np.uint8)
    if "shortconv.conv" in name:
        return normal_f32(n, seed, 0.0, 0.1).view(np.uint8)
    return np.ones(n, dtype=np.float32).view(np.uint8)  # RMSNorm weights


def kv_metadata(spec: ModelSpec) -> list[tuple[str, int, object, int | None]]:
    a = spec.arch + "."
    U32, F32, STR, ARR = KV_TYPES["UINT32"], KV_TYPES["FLOAT32"], KV_TYPES["STRING"], KV_TYPES["ARRAY"]
    kv = [("general.architecture", STR, spec.arch, None), ("general.name", STR, spec.name or spec.arch, None),
          (a + "block_count", U32, spec.n_layers, None), (a + "context_length", U32, spec.context_length, None),
          (a + "embedding_length", U32, spec.n_embd, None), (a + "feed_forward_length", U32, spec.n_ff, None),
          (a + "attention.head_count", U32, spec.n_head, None),
          (a + "attention.layer_norm_rms_epsilon", F32, spec.eps, None),
          (a + "rope.freq_base", F32, spec.rope_base, None), (a + "vocab_size", U32, spec.n_vocab, None),
          (a + "attention.key_length", U32, spec.head_dim, None),
          (a + "attention.value_length", U32, spec.head_dim, None)]
    if spec.arch == "qwen3":
        kv.append((a + "attention.head_count_kv", U32, spec.n_head_kv, None))
    elif spec.arch == "qwen3moe":  # the keys Qwen3Engine reads for MoE layers (qwen3-engine.js:40-41, 89-94)
        kv += [(a + "attention.head_count_kv", U32, spec.n_head_kv, None),
               (a + "expert_count", U32, spec.n_expert, None), (a + "expert_used_count", U32, spec.n_expert_used, None),
               (a + "expert_feed_forward_length", U32, spec.n_ff_exp, None)]
    else:
        per_layer = [spec.n_head_kv if spec.is_attn(i) else 0 for i in range(spec.n_layers)]
        kv += [(a + "attention.head_count_kv", ARR, per_layer, U32), (a + "expert_count", U32, spec.n_expert, None),
               (a + "expert_used_count", U32, spec.n_expert_used, None),
               (a + "expert_feed_forward_length", U32, spec.n_ff_exp, None),
               (a + "leading_dense_block_count", U32, spec.n_dense_lead, None),
               (a + "shortconv.l_cache", U32, 3, None), (a + "expert_gating_func", U32, 2, None)]
    # tokenizer.js:36-44 throws without tokens and merges; ids are all this path needs
    kv += [("tokenizer.ggml.model", STR, "gpt2", None),
           ("tokenizer.ggml.tokens", ARR, [f"<t{i}>" for i in range(spec.n_vocab)], STR),
           ("tokenizer.ggml.merges", ARR, [], STR)]
    return kv


def kv_values(spec: ModelSpec) -> dict:
    """Metadata as a GGUF reader returns it: FLOAT32 values come back rounded to f32."""
    out = {}
    for k, t, v, at in kv_metadata(spec):
        if t == KV_TYPES["FLOAT32"]:
            v = float(np.float32(v))
        out[k] = v
    return out


class MemoryGGUF:
    """In-memory stand-in with the GGUFReader lookup API (for models too large to write out)."""

    def __init__(self, spec: ModelSpec, tensors: dict[str, tuple[int, list, np.ndarray]]):
        self.spec = spec
        self._kv = kv_values(spec)
        self._t = tensors

    def getKeyValue(self, key, default=None):
        return self._kv.get(key, default)

    def getTensorMetaByName(self, name):
        if name not in self._t:
            return None
        t, ne, raw = self._t[name]
        return TensorMeta(raw, 0, -(-raw.nbytes // 256) * 256, list(ne), t, name)

    def getArch(self):
        from .gguf import GGUFReader
        return GGUFReader.getArch(self)


def build_tensors(spec: ModelSpec, only=None) -> dict[str, tuple[int, list, np.ndarray]]:
    out: dict[str, tuple[int, list, np.ndarray]] = {}
    raw_cache: dict[str, np.ndarray] = {}
    for name, t, ne in tensor_specs(spec):
        if only is not None and name not in only:
            continue
        raw = generate_tensor(spec, name, t, ne, raw_cache)
        if name.endswith("ffn_gate_inp.weight"):
            raw_cache[name] = raw
        out[name] = (t, ne, raw)
    return out


def memory_model(spec: ModelSpec) -> MemoryGGUF:
    return MemoryGGUF(spec, build_tensors(spec))


def write_gguf(spec: ModelSpec, path) -> None:
    w = GGUFWriter()
    for k, t, v, at in kv_metadata(spec):
        w.add_kv(k, t, v, at)
    for name, (t, ne, raw) in build_tensors(spec).items():
        assert raw.nbytes == tensor_nbytes(ne, t)
        w.add_tensor(name, ne, t, raw)
    w.write(path)
