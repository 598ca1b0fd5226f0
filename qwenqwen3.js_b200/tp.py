"""Tensor-parallel dense Qwen3 over a torch.distributed process group (one process per GPU).

Qwen3Engine.forward (qwen3-engine.js:115-245) runs every head and every FFN unit of a layer in
one process.  Here a layer is split over G ranks:

* wq / wk / wv are column-parallel by heads: rank r owns the query heads [r nH/G, (r+1) nH/G)
  and the KV heads [r nKV/G, (r+1) nKV/G).  The GQA map kvHead = floor(h nKV / nH)
  (qwen3-engine.js:260) then keeps every query head with its KV head on one rank, so the
  per-head RMSNorm, RoPE, the KV cache and attention stay local;
* wo is row-parallel (its input dimension is the heads): each rank's product is a partial sum
  of the full output, all-reduced before the residual add (qwen3-engine.js:185);
* ffn_gate / ffn_up are column-parallel over the FFN units, ffn_down row-parallel and
  all-reduced (qwen3-engine.js:207-214);
* the lm_head is vocab-parallel: rank r owns the vocab rows [v_r, v_r+1).  The greedy id is
  sampleGreedy's first maximum (tensor.js:231-237) over the ranks' (maximum, first index) pairs;
* the embedding and the norms are replicated.

That is two all-reduces of one hidden row per token per layer plus one gather of G pairs per
token.  Q8_0 tensors shard on whole 34-byte blocks, so the weights stay raw GGUF bytes: rows
for the column-parallel tensors, block columns for the row-parallel ones.

`tp_forward` takes the arithmetic as callables (`ops`) and the two collectives as functions, as
`ep.py` does, so the sharding and the exchange are testable on CPU (gloo ranks, the CPU oracle
as arithmetic); GPU ranks bind the same steps to the library's kernels and NCCL.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

Q8_0 = 8
F32 = 0
Q8_BLOCK_BYTES = 34


@dataclass
class TPPlan:
    """Which heads, FFN units and vocab rows rank `rank` of `world` owns."""

    n_head: int
    n_kv: int
    head_dim: int
    n_embd: int
    n_ff: int
    n_vocab: int
    world: int
    rank: int

    def __post_init__(self):
        G = self.world
        if not 0 <= self.rank < G:
            raise ValueError(f"rank {self.rank} outside a world of {G}")
        if self.n_head % G or self.n_kv % G:
            raise ValueError(f"{self.n_head} query / {self.n_kv} KV heads do not shard over {G} ranks")
        if (self.n_head // G * self.head_dim) % 32:
            raise ValueError("wo's per-rank input width is not a whole number of Q8_0 blocks")
        if self.n_ff % G or (self.n_ff // G) % 32:
            raise ValueError(f"FFN width {self.n_ff} does not shard over {G} ranks in whole Q8_0 blocks")
        if self.n_vocab < G:
            raise ValueError("fewer vocab rows than ranks")

    @property
    def q_heads(self) -> range:
        n = self.n_head // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    @property
    def kv_heads(self) -> range:
        n = self.n_kv // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    @property
    def ff_units(self) -> range:
        n = self.n_ff // self.world
        return range(self.rank * n, (self.rank + 1) * n)

    def vocab_offsets(self) -> list[int]:
        """v_0 = 0 < v_1 < ... < v_G = n_vocab: rank r owns rows [v_r, v_r+1)."""
        return [r * self.n_vocab // self.world for r in range(self.world + 1)]

    @property
    def vocab_rows(self) -> range:
        v = self.vocab_offsets()
        return range(v[self.rank], v[self.rank + 1])


# ---- raw Q8_0 slicing (the byte layout of src/gguf.js:307-309, 344-345) --------------------

def q8_rows(raw: np.ndarray, K: int, r0: int, r1: int) -> np.ndarray:
    """Output rows [r0, r1) of a Q8_0 tensor [K, N]: each row is K/32 contiguous blocks."""
    row = K // 32 * Q8_BLOCK_BYTES
    return np.ascontiguousarray(raw[r0 * row: r1 * row])


def q8_cols(raw: np.ndarray, K: int, N: int, k0: int, k1: int) -> np.ndarray:
    """Input columns [k0, k1) (whole blocks) of every row of a Q8_0 tensor [K, N]: a [k1-k0, N]
    tensor."""
    if k0 % 32 or k1 % 32:
        raise ValueError("Q8_0 columns shard on 32-value blocks")
    blocks = np.asarray(raw[: N * (K // 32) * Q8_BLOCK_BYTES]).reshape(N, K // 32, Q8_BLOCK_BYTES)
    return np.ascontiguousarray(blocks[:, k0 // 32: k1 // 32, :]).reshape(-1)


def shard_model(gguf, plan: TPPlan) -> dict:
    """This rank's tensors, name -> (ggml type, ne, raw bytes), under the reference's tensor
    names.  Replicated: token_embd, the norms.  `output.weight` (or the tied token_embd,
    qwen3-engine.js:47-49) becomes this rank's vocab rows."""
    E, hd = plan.n_embd, plan.head_dim
    out = {}

    def meta(name):
        m = gguf.getTensorMetaByName(name)
        if m is None:
            raise KeyError(f"missing tensor {name}")
        return m

    def keep(name):
        m = meta(name)
        out[name] = (m.type, list(m.shape), np.asarray(m.raw()))

    def need_q8(m, name):
        if m.type != Q8_0:
            raise ValueError(f"{name}: tensor parallelism shards Q8_0 weights only (type {m.type})")

    keep("token_embd.weight")
    keep("output_norm.weight")
    n_layers = int(gguf.getArch()["blockCount"])
    qh, kvh, ff = plan.q_heads, plan.kv_heads, plan.ff_units
    for i in range(n_layers):
        p = f"blk.{i}."
        for n in ("attn_norm.weight", "ffn_norm.weight", "attn_q_norm.weight", "attn_k_norm.weight"):
            keep(p + n)
        for n, rows in (("attn_q.weight", (qh.start * hd, qh.stop * hd)),
                        ("attn_k.weight", (kvh.start * hd, kvh.stop * hd)),
                        ("attn_v.weight", (kvh.start * hd, kvh.stop * hd)),
                        ("ffn_gate.weight", (ff.start, ff.stop)),
                        ("ffn_up.weight", (ff.start, ff.stop))):
            m = meta(p + n)
            need_q8(m, p + n)
            K = int(m.shape[0])
            out[p + n] = (Q8_0, [K, rows[1] - rows[0]], q8_rows(m.raw(), K, *rows))
        for n, cols in (("attn_output.weight", (qh.start * hd, qh.stop * hd)),
                        ("ffn_down.weight", (ff.start, ff.stop))):
            m = meta(p + n)
            need_q8(m, p + n)
            K, N = int(m.shape[0]), int(m.shape[1])
            out[p + n] = (Q8_0, [cols[1] - cols[0], N], q8_cols(m.raw(), K, N, *cols))
    lm = gguf.getTensorMetaByName("output.weight") or meta("token_embd.weight")
    need_q8(lm, "lm_head")
    vr = plan.vocab_rows
    out["output.weight"] = (Q8_0, [E, vr.stop - vr.start], q8_rows(lm.raw(), E, vr.start, vr.stop))
    return out


# ---- greedy id over vocab shards ------------------------------------------------------------

def local_greedy(logits: np.ndarray, v0: int) -> tuple[float, int, bool]:
    """sampleGreedy's view of one vocab shard starting at global row v0: (max, its first
    global index, whether the shard's first logit is NaN).  NaN never wins a comparison in the
    JS loop (`logits[i] > logits[maxIdx]`), so it is skipped; a shard of all NaN reports -inf."""
    x = np.asarray(logits, dtype=np.float32)
    finite = np.where(np.isnan(x), -np.inf, x)
    i = int(np.argmax(finite))  # first occurrence of the maximum
    return float(finite[i]), v0 + i, bool(x.size and np.isnan(x[0]))


def merge_greedy(pairs: list[tuple[float, int, bool]]) -> int:
    """The global first maximum from the ranks' local_greedy results, ranks in vocab order.
    sampleGreedy starts from index 0 and replaces it only with a strictly larger logit, so a NaN
    logit 0 wins outright and equal maxima resolve to the lowest index."""
    if pairs and pairs[0][2]:
        return 0
    best_v, best_i = -np.inf, 0
    for v, i, _ in pairs:
        if v > best_v:
            best_v, best_i = v, i
    return best_i


# ---- one token through the tensor-parallel layers -------------------------------------------

@dataclass
class TPOps:
    """The arithmetic a rank runs.  Vectors are whatever the ops use (numpy on CPU, device tensors
    on a GPU); weights are shard entries (ggml type, ne, raw) or what the ops made of them:
    embed(token) -> [E]; rmsnorm(x, w, eps) -> x'; matmul(w, x) -> [N];
    head_rmsnorm(x, n_heads, w, eps) -> x'; rope(x, n_heads, pos) -> x';
    kv_store(layer, pos, k, v); attention(layer, pos, q) -> [local heads * hd] over this rank's
    query/KV heads; silu_mul(g, u) -> h; add(x, d) -> x + d; to_host(x) -> numpy float32."""

    embed: object
    rmsnorm: object
    matmul: object
    head_rmsnorm: object
    rope: object
    kv_store: object
    attention: object
    silu_mul: object
    add: object
    to_host: object


def tp_forward(token: int, pos: int, plan: TPPlan, shards: dict, ops: TPOps, eps: float, n_layers: int,
               all_reduce, gather_pairs, want_logits: bool = True):
    """Qwen3Engine.forward(token, pos, !want_logits) on this rank's shards.  all_reduce(x) returns
    the element-wise sum over the ranks; gather_pairs(pair) returns every rank's local_greedy
    pair in rank order.  Returns (this rank's vocab-shard logits as numpy, global greedy id) or
    (None, None) without logits."""
    nq, nkv = len(plan.q_heads), len(plan.kv_heads)
    x = ops.embed(token)
    for i in range(n_layers):
        p = f"blk.{i}."
        xn = ops.rmsnorm(x, shards[p + "attn_norm.weight"], eps)
        q = ops.matmul(shards[p + "attn_q.weight"], xn)
        k = ops.matmul(shards[p + "attn_k.weight"], xn)
        v = ops.matmul(shards[p + "attn_v.weight"], xn)
        q = ops.rope(ops.head_rmsnorm(q, nq, shards[p + "attn_q_norm.weight"], eps), nq, pos)
        k = ops.rope(ops.head_rmsnorm(k, nkv, shards[p + "attn_k_norm.weight"], eps), nkv, pos)
        ops.kv_store(i, pos, k, v)
        att = ops.attention(i, pos, q)
        x = ops.add(x, all_reduce(ops.matmul(shards[p + "attn_output.weight"], att)))
        xn = ops.rmsnorm(x, shards[p + "ffn_norm.weight"], eps)
        h = ops.silu_mul(ops.matmul(shards[p + "ffn_gate.weight"], xn), ops.matmul(shards[p + "ffn_up.weight"], xn))
        x = ops.add(x, all_reduce(ops.matmul(shards[p + "ffn_down.weight"], h)))
    if not want_logits:
        return None, None
    xn = ops.rmsnorm(x, shards["output_norm.weight"], eps)
    logits = ops.to_host(ops.matmul(shards["output.weight"], xn))
    return logits, merge_greedy(gather_pairs(local_greedy(logits, plan.vocab_rows.start)))


# ---- the GPU binding -------------------------------------------------------------------------

class GPURank:
    """One rank's shards on its GPU and the TPOps that run them through the library
    (runtime.Context: Q8_0 GEMVs, RMSNorm, RoPE, split attention over a local f32 K/V cache
    [layer][local KV head][max_ctx][head_dim], SwiGLU, residual add).  Device vectors are torch
    tensors on `stream`, which the context also runs on, so no operation needs another stream's
    results.  all_reduce for tp_forward: `GPURank.nccl_all_reduce` (torch.distributed, NCCL)."""

    def __init__(self, ctx, plan: TPPlan, shards: dict, head_dim: int, rope_base: float, max_ctx: int,
                 n_layers: int, stream):
        import torch

        self.torch = torch
        self.ctx, self.plan, self.hd = ctx, plan, head_dim
        self.stream = stream
        ctx.set_stream(stream.cuda_stream)
        self.dev = torch.device("cuda", ctx.device)
        self.w = {name: ctx.upload(raw, t, ne) for name, (t, ne, raw) in shards.items()}
        self.shards = {name: self.w[name] for name in shards}  # tp_forward looks weights up by name
        nkv = len(plan.kv_heads)
        self.kc = torch.zeros((n_layers, nkv, max_ctx, head_dim), dtype=torch.float32, device=self.dev)
        self.vc = torch.zeros_like(self.kc)
        self.max_ctx, self.base = max_ctx, rope_base

    def _new(self, n):
        with self.torch.cuda.stream(self.stream):  # allocations belong to the stream that uses them
            return self.torch.empty(n, dtype=self.torch.float32, device=self.dev)

    def ops(self) -> TPOps:
        ctx, hd, plan = self.ctx, self.hd, self.plan
        nq, nkv = len(plan.q_heads), len(plan.kv_heads)
        E = plan.n_embd

        def embed(token):
            out = self._new(E)
            ctx.embed(self.w["token_embd.weight"], [token], out)
            return out

        def rmsnorm(x, w, eps):
            y = self._new(x.numel())
            ctx.rmsnorm(x, 1, x.numel(), w, eps, y)
            return y

        def matmul(w, x):
            y = self._new(int(w.ne[1]))
            ctx.q8_matmul(w, x, 1, y)
            return y

        def head_rmsnorm(x, n, w, eps):
            y = self._new(x.numel())
            ctx.rmsnorm(x, n, hd, w, eps, y)
            return y

        def rope(x, n, pos):
            ctx.rope(x, 1, n, hd, pos, self.base)
            return x

        def kv_store(layer, pos, k, v):
            with self.torch.cuda.stream(self.stream):
                self.kc[layer, :, pos].copy_(k.view(nkv, hd))
                self.vc[layer, :, pos].copy_(v.view(nkv, hd))

        def attention(layer, pos, q):
            out = self._new(nq * hd)
            ctx.attention_decode(q, self.kc[layer], self.vc[layer], nq, nkv, hd, self.max_ctx, pos, out)
            return out

        def silu_mul(g, u):
            h = self._new(g.numel())
            ctx.swiglu(g, u, g.numel(), h)
            return h

        def add(x, d):
            ctx.add(x, d, x.numel())
            return x

        def to_host(x):
            self.stream.synchronize()
            return x.cpu().numpy()

        return TPOps(embed, rmsnorm, matmul, head_rmsnorm, rope, kv_store, attention, silu_mul, add, to_host)

    def nccl_all_reduce(self, x):
        """Sum of x over the ranks of the default process group, in place (NCCL over NVLink)."""
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_world_size() > 1:
            with self.torch.cuda.stream(self.stream):
                dist.all_reduce(x)
        return x

    def close(self):
        for t in self.w.values():
            t.free()
        self.w.clear()
