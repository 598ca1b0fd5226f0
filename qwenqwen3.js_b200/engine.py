"""Qwen3CudaEngine / Lfm2CudaEngine: the reference engine API over libqq3cuda.so.

They mirror Qwen3GPUEngine / Lfm2GPUEngine (webgpu.js:495-1103, 1467-2124) and the CPU
engines they extend (qwen3-engine.js, lfm2-engine.js): same constructor inputs (a GGUF
reader), same hyper-parameter derivation, ``forward(tokenId, position, skipLogits)``
returning the logits array (or None), ``generate(tokenIds, options)`` with the same
options and callbacks, ``resetKVCache()``, ``onRouterUpdate`` and ``expertMask``.  The
arithmetic runs on the B200 through the C ABI; sampling with temperature > 0 and the
'shorten' thinking mode stay on the host exactly as in tensor.js:188-265.
"""
from __future__ import annotations

import ctypes as C
import math
import random

import numpy as np

from . import runtime as rt

# ---------------------------------------------------------------------------------------
# host-side sampling (tensor.js:188-265)


def sample_greedy(logits: np.ndarray) -> int:
    """sampleGreedy (tensor.js:231-237): first maximum wins."""
    return int(np.argmax(logits))  # numpy returns the first occurrence of the maximum


def sample_top_p_top_k(logits: np.ndarray, temperature: float, top_p: float, top_k: int, rng=random.random) -> int:
    """sampleTopPTopK (tensor.js:188-228)."""
    x = logits.astype(np.float64)
    mx = float(np.max(np.where(np.isnan(x), -np.inf, x)))  # `logits[i] > maxVal` skips NaN
    e = np.exp((x - mx) / temperature).astype(np.float32)  # stored into the Float32Array
    s = float(np.cumsum(e.astype(np.float64))[-1])  # sumExp: a sequential f64 sum, as the JS loop
    p = (e.astype(np.float64) * (1.0 / s)).astype(np.float32)
    order = np.argsort(-p, kind="stable")
    probs = p[order].astype(np.float64)
    n = len(probs)
    k_limit = min(top_k, n) if top_k > 0 else n
    probs[k_limit:] = 0.0
    cum = np.cumsum(probs)
    cut = np.searchsorted(cum, top_p, side="left")
    if cut < n:
        probs[cut + 1:] = 0.0
    r = rng()
    cum = 0.0
    for i in range(n):
        cum += probs[i]
        if r <= cum:
            return int(order[i])
    return int(order[-1])


def sample_with_think_control(logits: np.ndarray, temperature: float, top_p: float, top_k: int, think: dict) -> int:
    """sampleWithThinkControl (tensor.js:244-265)."""
    mode = think.get("mode", "suppress")
    if mode == "suppress":
        logits[think["thinkId"]] = -np.inf
    elif mode == "shorten" and not think.get("thinkingDone"):
        end_logit = logits[think["endThinkId"]]
        rank = int(np.count_nonzero(logits > end_logit))
        if rank < top_k:
            return int(think["endThinkId"])
    return sample_greedy(logits) if temperature <= 0 else sample_top_p_top_k(logits, temperature, top_p, top_k)


# ---------------------------------------------------------------------------------------


def _num(v, default):
    try:
        f = float(v)
    except (TypeError, ValueError):
        return default
    return default if (f == 0 or math.isnan(f)) else f


class _CudaEngine:
    ARCH = rt.QQ_ARCH_QWEN3
    THINK_ID = 151667
    END_THINK_ID = 151668

    EXPERT_TENSORS = ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight")

    def __init__(self, gguf, *, ctx: rt.Context | None = None, device: int = 0, max_ctx: int | None = None,
                 n_seq: int = 1, ep_world: int = 1, tp_world: int = 1):
        """ep_world > 1: expert parallelism -- ctx carries a communicator of ep_world ranks
        (Context.comm_init) and this engine uploads only its rank's share of every expert tensor;
        every rank then makes the same forward calls with the same token counts.
        tp_world > 1 (dense Qwen3): tensor parallelism over the communicator's ranks -- this engine
        uploads its rank's shards (tp.shard_model: its heads, FFN units and vocab rows); steps go
        through forward / forward_batch, made by every rank alike."""
        self.gguf = gguf
        self.ctx = ctx or rt.Context(device)
        self.epWorld = int(ep_world)
        self.epRank = 0
        self.tpWorld = int(tp_world)
        self._shards = None
        self._read_hparams(gguf)
        if max_ctx is not None:
            self.maxCtx = int(max_ctx)
        self.nSeq = n_seq
        self.onRouterUpdate = None
        self._expert_mask: set | None = None
        self.eosTokenId = int(gguf.getKeyValue("tokenizer.ggml.eos_token_id", -1))
        self.stopTokenIds: set = set()
        self._tensors: dict = {}
        self._uploader = None
        self.uploadBytes = 0
        self._build()
        self.bufLogits = np.zeros(self.nVocab, dtype=np.float32)

    @classmethod
    def create(cls, gguf, **kw):
        """Mirrors ``static async create(gguf)`` (webgpu.js:498, 1470)."""
        return cls(gguf, **kw)

    # --- upload + model binding
    def _upload(self, name):
        if self._shards is not None:  # tensor-parallel: this rank's shard of the tensor
            if name not in self._shards:
                return None
            if name not in self._tensors:
                t, ne, raw = self._shards[name]
                up = self._uploader
                self._tensors[name] = (up.upload if up is not None else self.ctx.upload)(raw, t, ne)
            return self._tensors[name]
        meta = self.gguf.getTensorMetaByName(name)
        if meta is None:
            return None
        if name not in self._tensors:
            up = self._uploader
            raw, shape = meta.raw(), list(meta.shape)
            if self.epWorld > 1 and name.endswith(self.EXPERT_TENSORS):
                # this rank's experts: a contiguous run of the packed [ne0, ne1, E] tensor
                # (_expertSlice, lfm2-engine.js:490-505)
                per = shape[2] // self.epWorld
                stride = raw.nbytes // shape[2]
                raw = raw[self.epRank * per * stride:(self.epRank + 1) * per * stride]
                shape = shape[:2] + [per]
            self._tensors[name] = (up.upload if up is not None else self.ctx.upload)(raw, meta.type, shape)
        return self._tensors[name]

    def _build(self):
        """Upload every tensor the engine reads (streamed through a pinned ring: the host copy, the
        DMA and the device-side Q8_0 split of consecutive chunks overlap), then bind the model."""
        self._uploader = self.ctx.streaming_upload()
        try:
            self._bind()
        finally:
            if self._uploader is not None:  # an upload failed part-way
                up, self._uploader = self._uploader, None
                up.finish()

    def _bind(self):
        if self.epWorld > 1:
            self.epRank = self.ctx.comm_rank()
        if self.tpWorld > 1:
            from .tp import TPPlan, shard_model

            n_ff = int(self.gguf.getTensorMetaByName("blk.0.ffn_gate.weight").shape[1])
            plan = TPPlan(self.nHeads, self.nHeadKV, self.headDim, self.nEmb, n_ff, self.nVocab, self.tpWorld,
                          self.ctx.comm_rank())
            self._shards = shard_model(self.gguf, plan)
        layers = (rt.LayerDesc * self.nLayers)()
        for i in range(self.nLayers):
            L = layers[i]
            L.is_attn = 1 if self._is_attn(i) else 0
            L.is_moe = 1 if self._is_moe(i) else 0
            for slot, suffix in rt.SLOT_TENSOR_NAMES.items():
                t = self._upload(f"blk.{i}.{suffix}")
                L.t[rt.SLOT[slot]] = t.h.value if t is not None else None
        d = rt.ModelDesc()
        d.arch = self.ARCH
        d.n_layers = self.nLayers
        d.n_embd = self.nEmb
        d.n_head = self.nHeads
        d.n_head_kv = self.nHeadKV
        d.head_dim = self.headDim
        d.n_vocab = self.nVocab
        d.n_expert = self.nExperts
        d.n_expert_used = self.nExpertsUsed
        d.max_ctx = self.maxCtx
        d.n_seq = self.nSeq
        d.rms_eps = self.eps
        d.rope_base = self.ropeFreqBase
        d.tok_embd = self._upload("token_embd.weight").h.value
        d.output_norm = self._upload(self.OUTPUT_NORM).h.value
        out = self._upload("output.weight")
        d.output = out.h.value if out is not None else None
        d.layers = C.cast(layers, C.POINTER(rt.LayerDesc))
        d.ep_world = self.epWorld
        d.tp_world = self.tpWorld
        up, self._uploader = self._uploader, None
        self.uploadBytes = up.finish() if up is not None else 0  # tensors are ready from here on
        self.model = rt.Model(self.ctx, d, layers, list(self._tensors.values()))

    # --- reference API
    def forward(self, tokenId: int, position: int, skipLogits: bool = False, seq: int = 0):
        """forward(tokenId, position, skipLogits) (qwen3-engine.js:115-245, lfm2-engine.js:228-269)."""
        if skipLogits:
            self.model.forward([tokenId], seq=seq, pos0=position, want_logits=False)
            self._emit_routing()
            return None
        logits, _ = self.model.forward([tokenId], seq=seq, pos0=position, want_logits=True, logits=True)
        self.bufLogits[:] = logits
        self._emit_routing()
        return self.bufLogits

    def forward_argmax(self, tokenId: int, position: int, suppress_id: int = -1, seq: int = 0) -> int:
        """forward() + device greedy argmax (4-byte readback instead of the logits)."""
        am = self.model.forward_argmax(tokenId, seq=seq, pos=position, suppress_id=suppress_id)
        self._emit_routing()
        return am

    def forward_batch(self, seqs, tokenIds, positions, skipLogits: bool = False, suppress_id: int = -1,
                      want_logits_array: bool = True):
        """forward(tokenIds[i], positions[i], skipLogits) of sequence seqs[i] for every i in one
        step (the engine was created with n_seq > max(seqs)).  Returns the logits rows
        [len(seqs)][nVocab] and the device greedy ids (suppress_id excluded), or (None, None) with
        skipLogits.  onRouterUpdate sees the routing of the last row."""
        if skipLogits:
            self.model.forward_batch(seqs, tokenIds, positions, want_logits=False)
            self._emit_routing()
            return None, None
        logits, am = self.model.forward_batch(seqs, tokenIds, positions, want_logits=True,
                                              logits=want_logits_array, suppress_id=suppress_id)
        self._emit_routing()
        return logits, am

    def prefill(self, tokenIds, pos0: int = 0, seq: int = 0) -> None:
        """forward(t, pos, true) for each token, in one C-ABI call."""
        self.model.forward(tokenIds, seq=seq, pos0=pos0, want_logits=False)

    def resetKVCache(self, seq: int = 0) -> None:
        self.model.reset(seq)

    resetState = resetKVCache

    @property
    def expertMask(self):
        return self._expert_mask

    @expertMask.setter
    def expertMask(self, ids):
        self._expert_mask = set(ids) if ids else None
        self.model.set_expert_mask(sorted(self._expert_mask) if self._expert_mask else [])

    def _emit_routing(self):
        if not self.onRouterUpdate or self.nExperts == 0:
            return
        k, E = self.nExpertsUsed, self.nExperts
        m = 0
        for i in range(self.nLayers):
            if not self._is_moe(i):
                continue
            rec = self.model.read_routing(m, 2 * k + E)
            self.onRouterUpdate(dict(layer=i, probs=rec[2 * k:].tolist(), selected=[int(round(v)) for v in rec[:k]],
                                     weights=rec[k:2 * k].tolist()))
            m += 1

    def generate(self, tokenIds, maxSteps=512, temperature=0.7, topP=0.9, topK=40, thinkingMode="suppress",
                 onToken=None, onPrefill=None, onFinish=None, abortSignal=None, seed=None):
        """generate(tokenIds, options) (qwen3-engine.js:397-457, lfm2-engine.js:523-583).

        Sampling runs on the device (qq_forward_sample: one 4-byte readback a token) for every
        option set the device sampler serves -- greedy, and top-k/top-p with 1 <= topK <= 1024
        (the JS default is 40).  Math.random() is replaced by the device's seeded draws (seed:
        default a random 64-bit value).  topK = 0 ("no limit") with temperature > 0 samples the
        logits on the host, exactly as tensor.js:188-228."""
        think = dict(mode=thinkingMode, thinkId=self.THINK_ID, endThinkId=self.END_THINK_ID,
                     thinkingDone=thinkingMode == "suppress")
        aborted = (lambda: bool(abortSignal and getattr(abortSignal, "aborted", False)))
        self.resetKVCache()
        n = len(tokenIds)
        device_greedy = temperature <= 0 and thinkingMode in ("suppress", "full")
        suppress = self.THINK_ID if thinkingMode == "suppress" and self.THINK_ID < self.nVocab else -1
        dev_params = None
        if not device_greedy and (temperature <= 0 or 1 <= topK <= rt.QQ_SAMPLE_MAX_TOP_K):
            dev_params = rt.sample_params(temperature, topP, max(0, min(int(topK), rt.QQ_SAMPLE_MAX_TOP_K)),
                                          thinkingMode, self.THINK_ID, self.END_THINK_ID,
                                          random.getrandbits(64) if seed is None else seed)
        if aborted():
            return None
        if n > 1:
            if onPrefill is None:
                self.prefill(tokenIds[:-1])
            else:
                for i in range(n - 1):
                    if aborted():
                        return None
                    self.forward(tokenIds[i], i, True)
                    onPrefill(i + 1, n)
        if aborted():
            return None

        def step(tok, pos):
            if device_greedy:
                return self.forward_argmax(tok, pos, suppress)
            if dev_params is not None:
                nxt = self.model.forward_sample(tok, pos, dev_params, think["thinkingDone"])
                self._emit_routing()
                return nxt
            logits = self.forward(tok, pos, False).copy()
            if think["thinkId"] >= self.nVocab:
                think_local = dict(think, mode="full")
                return sample_with_think_control(logits, temperature, topP, topK, think_local)
            return sample_with_think_control(logits, temperature, topP, topK, think)

        cur = step(tokenIds[-1], n - 1)
        generated = []
        for s in range(maxSteps):
            if cur == self.eosTokenId or cur in self.stopTokenIds:
                break
            if cur == think["endThinkId"]:
                think["thinkingDone"] = True
            if aborted():
                return None
            nxt = step(cur, n + s)
            generated.append(cur)
            if onToken:
                onToken(cur)
            cur = nxt
        if onFinish:
            onFinish(generated)
        return generated

    def close(self):
        self.model.close()
        for t in self._tensors.values():
            t.free()
        self._tensors.clear()


class Qwen3CudaEngine(_CudaEngine):
    """Hyper-parameters as Qwen3Engine (qwen3-engine.js:2-29, 78-111)."""

    ARCH = rt.QQ_ARCH_QWEN3
    THINK_ID = 151667
    END_THINK_ID = 151668
    OUTPUT_NORM = "output_norm.weight"

    def _read_hparams(self, gguf):
        a = gguf.getArch()
        self.nLayers = int(a["blockCount"])
        self.nEmb = int(a["embeddingLength"])
        self.nHeads = int(a["headCount"])
        self.nHeadKV = int(a["headCountKV"] or a["headCount"])
        self.eps = _num(a["layerNormRmsEps"], 1e-6)
        self.ropeFreqBase = _num(a["ropeFreqBase"], 10000.0)
        self.maxCtx = min(int(_num(a["contextLength"], 8192)), 4096)
        self.nVocab = int(gguf.getTensorMetaByName("token_embd.weight").shape[1])
        self.nQ = int(gguf.getTensorMetaByName("blk.0.attn_q.weight").shape[1])
        self.headDim = self.nQ // self.nHeads
        self._moe = [gguf.getTensorMetaByName(f"blk.{i}.ffn_gate_inp.weight") is not None
                     for i in range(self.nLayers)]
        if any(self._moe):
            # Qwen3-MoE (qwen3-engine.js:37-41): softmax-routed experts, counts from the metadata
            arch = gguf.getKeyValue("general.architecture", "qwen3")
            self.nExperts = int(_num(gguf.getKeyValue(f"{arch}.expert_count"), 128))
            self.nExpertsUsed = int(_num(gguf.getKeyValue(f"{arch}.expert_used_count"), 8))
        else:
            self.nExperts = 0
            self.nExpertsUsed = 0

    def _is_attn(self, i):
        return True

    def _is_moe(self, i):
        return self._moe[i]


class Lfm2CudaEngine(_CudaEngine):
    """Hyper-parameters as Lfm2Engine (lfm2-engine.js:15-74)."""

    ARCH = rt.QQ_ARCH_LFM2
    THINK_ID = 124901
    END_THINK_ID = 124902
    OUTPUT_NORM = "token_embd_norm.weight"

    def _read_hparams(self, gguf):
        arch = gguf.getKeyValue("general.architecture", "lfm2moe")
        p = arch + "."
        g = lambda k, d: _num(gguf.getKeyValue(p + k), d)  # noqa: E731  (Number(x) || default)
        self.nLayers = int(g("block_count", 24))
        self.nEmb = int(g("embedding_length", 2048))
        self.nHeads = int(g("attention.head_count", 32))
        self.eps = g("attention.layer_norm_rms_epsilon", 1e-5)
        self.nExperts = int(g("expert_count", 32))
        self.nExpertsUsed = int(g("expert_used_count", 4))
        self.nFFExp = int(g("expert_feed_forward_length", 1792))
        self.nDenseLead = int(g("leading_dense_block_count", 2))
        self.lCache = int(g("shortconv.l_cache", 3))
        self.maxCtx = min(int(g("context_length", 4096)), 4096)
        rope = gguf.getKeyValue(p + "rope.freq_base") or gguf.getKeyValue(p + "rope_freq_base")
        self.ropeFreqBase = _num(rope, 5_000_000.0)
        hkv = gguf.getKeyValue(p + "attention.head_count_kv")
        self.nHeadKV = max(v for v in hkv if v > 0) if isinstance(hkv, list) else int(_num(hkv, 8))
        self.nVocab = int(gguf.getTensorMetaByName("token_embd.weight").shape[1])
        self._recurrent = [gguf.getTensorMetaByName(f"blk.{i}.shortconv.conv.weight") is not None
                           for i in range(self.nLayers)]
        first_attn = next((i for i in range(self.nLayers) if not self._recurrent[i]), None)
        if first_attn is not None:
            self.headDim = gguf.getTensorMetaByName(f"blk.{first_attn}.attn_q.weight").shape[1] // self.nHeads
        else:
            self.headDim = 64
        if not any(self._is_moe(i) for i in range(self.nLayers)):
            self.nExperts = 0
            self.nExpertsUsed = 0

    def _is_attn(self, i):
        return not self._recurrent[i]

    def _is_moe(self, i):
        return i >= self.nDenseLead and self.gguf.getTensorMetaByName(f"blk.{i}.ffn_gate_inp.weight") is not None


def engine_for(gguf, **kw) -> _CudaEngine:
    arch = gguf.getKeyValue("general.architecture", "")
    if arch.startswith("lfm2"):
        return Lfm2CudaEngine(gguf, **kw)
    return Qwen3CudaEngine(gguf, **kw)
