// qq3-cuda-engine.js -- Qwen3CudaEngine / Lfm2CudaEngine for the QwenQwen3.js page or a Node host.
//
// Drop-in twins of Qwen3GPUEngine / Lfm2GPUEngine (src/webgpu.js:495-1103, 1467-2124): same
// `static async create(gguf)`, `async forward(tokenId, position, skipLogits)`, `async
// generate(tokenIds, options)`, `resetKVCache()`, `onRouterUpdate`, `expertMask`.  The CPU
// engine (Qwen3Engine / Lfm2Engine) is still constructed for its metadata and tokenizer, as
// the WebGPU engines do; the arithmetic runs in libqq3cuda.so through the N-API addon
// (qq3_addon.cc).  gguf.js meta objects are uploaded raw: new Uint8Array(meta.buffer,
// meta.offset, meta.nbytes), exactly the bytes GPUDevice.uploadBuffer receives today.
'use strict';

const qq3 = require('./build/Release/qq3.node');

const SLOTS = [
    'attn_norm.weight', 'ffn_norm.weight', 'attn_q.weight', 'attn_k.weight', 'attn_v.weight',
    'attn_output.weight', 'attn_q_norm.weight', 'attn_k_norm.weight', 'shortconv.conv.weight',
    'shortconv.in_proj.weight', 'shortconv.out_proj.weight', 'ffn_gate.weight', 'ffn_up.weight',
    'ffn_down.weight', 'ffn_gate_inp.weight', 'ffn_gate_exps.weight', 'ffn_up_exps.weight',
    'ffn_down_exps.weight', 'exp_probs_b.bias',
];

function upload(ctx, meta) {
    if (!meta) return null;
    return qq3.uploadTensor(ctx, new Uint8Array(meta.buffer, meta.offset, meta.nbytes), meta.type, meta.shape);
}

class CudaEngineBase {
    static async _create(gguf, cpu, arch, outputNormName, opts = {}) {
        const e = new this();
        e._cpu = cpu;
        e.tokenizer = cpu.tokenizer;
        e.ctx = qq3.init(opts.device ?? 0);
        e.nVocab = cpu.nVocab;
        e.nLayers = cpu.nLayers;
        e.nExperts = cpu.nExperts ?? 0;
        e.nExpertsUsed = cpu.nExpertsUsed ?? 0;
        e.onRouterUpdate = null;
        e.batchRouterUpdate = true;
        e._mask = null;
        const t = (name) => upload(e.ctx, gguf.getTensorMetaByName(name));
        const layers = [];
        e._moeLayers = [];
        for (let i = 0; i < cpu.nLayers; i++) {
            const isAttn = gguf.getTensorMetaByName(`blk.${i}.shortconv.conv.weight`) === null ? 1 : 0;
            const isMoE = gguf.getTensorMetaByName(`blk.${i}.ffn_gate_inp.weight`) !== null ? 1 : 0;
            if (isMoE) e._moeLayers.push(i);
            layers.push({ isAttn, isMoE, t: SLOTS.map((s) => t(`blk.${i}.${s}`)) });
        }
        e.model = qq3.modelCreate(e.ctx, {
            arch, nLayers: cpu.nLayers, nEmb: cpu.nEmb, nHeads: cpu.nHeads, nHeadKV: cpu.nHeadKV,
            headDim: cpu.headDim ?? cpu.headDimQ, nVocab: cpu.nVocab, nExperts: e.nExperts,
            nExpertsUsed: e.nExpertsUsed, maxCtx: opts.maxCtx ?? cpu.maxCtx, nSeq: 1, eps: cpu.eps,
            ropeFreqBase: cpu.ropeFreqBase, tokEmbd: t('token_embd.weight'), outputNorm: t(outputNormName),
            output: t('output.weight'), layers,
        });
        e.bufLogits = new Float32Array(cpu.nVocab);
        return e;
    }

    set expertMask(set) {
        this._mask = set;
        qq3.setExpertMask(this.model, Int32Array.from(set ? [...set] : []));
    }
    get expertMask() { return this._mask; }

    resetKVCache() { qq3.reset(this.model, 0); }
    resetState() { this.resetKVCache(); }

    // forward(tokenId, position, skipLogits): Float32Array logits or null (webgpu.js:806-875, 1954-2034)
    async forward(tokenId, position, skipLogits = false) {
        const r = await qq3.forward(this.model, Int32Array.of(tokenId), 0, position, skipLogits ? 0 : 1, -1, this.nVocab);
        if (this.onRouterUpdate) this._readbackRoutingData();
        if (skipLogits) return null;
        this.bufLogits.set(r.logits);
        return this.bufLogits;
    }

    // One step of several sequences (qq_forward_batch; the engine was created with nSeq > max(seqs)):
    // forward(tokenIds[i], positions[i], skipLogits) of sequence seqs[i].  Resolves to
    // {logits: Float32Array(n * nVocab), argmax: Int32Array(n)}, or null with skipLogits.
    async forwardBatch(seqs, tokenIds, positions, skipLogits = false) {
        const r = await qq3.forwardBatch(this.model, Int32Array.from(seqs), Int32Array.from(tokenIds),
                                         Int32Array.from(positions), skipLogits ? 0 : 1, -1, this.nVocab);
        if (this.onRouterUpdate) this._readbackRoutingData();
        return skipLogits ? null : r;
    }

    // routing records [topK ids | topK weights | nExperts probs] (webgpu.js:1922-1945)
    _readbackRoutingData() {
        const k = this.nExpertsUsed, n = this.nExperts;
        this._moeLayers.forEach((layer, m) => {
            const res = qq3.readRouting(this.model, m, 2 * k + n);
            this.onRouterUpdate({
                layer, probs: Array.from(res.subarray(2 * k)),
                selected: Array.from(res.subarray(0, k), Math.round), weights: Array.from(res.subarray(k, 2 * k)),
            });
        });
    }

    // generate(): the CPU engine's loop (lfm2-engine.js:523-583) over the CUDA forward()
    async generate(tokenIds, options = {}) {
        const { maxSteps = 512, temperature = 0.7, topP = 0.9, topK = 40, thinkingMode = 'suppress',
                onToken, onPrefill, onFinish, abortSignal } = options;
        const thinkOpts = { mode: thinkingMode, thinkId: this.THINK_ID, endThinkId: this.END_THINK_ID,
                            thinkingDone: thinkingMode === 'suppress' };
        this.resetKVCache();
        for (let i = 0; i < tokenIds.length - 1; i++) {
            if (abortSignal?.aborted) return;
            await this.forward(tokenIds[i], i, true);
            if (onPrefill) onPrefill(i + 1, tokenIds.length);
        }
        if (abortSignal?.aborted) return;
        await this.forward(tokenIds[tokenIds.length - 1], tokenIds.length - 1, false);
        let cur = sampleWithThinkControl(this.bufLogits, temperature, topP, topK, thinkOpts);
        const out = [];
        for (let step = 0; step < maxSteps; step++) {
            if (cur === this.tokenizer.eosTokenId || this.tokenizer.stopTokenIds?.has(cur)) break;
            if (cur === thinkOpts.endThinkId) thinkOpts.thinkingDone = true;
            if (abortSignal?.aborted) return;
            await this.forward(cur, tokenIds.length + step);
            out.push(cur);
            if (onToken) onToken(cur);
            cur = sampleWithThinkControl(this.bufLogits, temperature, topP, topK, thinkOpts);
        }
        if (onFinish) onFinish(out);
    }

    formatChat(...a) { return this._cpu.formatChat(...a); }
}

class Qwen3CudaEngine extends CudaEngineBase {
    static async create(gguf, opts) {
        const e = await super._create(gguf, new Qwen3Engine(gguf), 0, 'output_norm.weight', opts);
        e.THINK_ID = 151667; e.END_THINK_ID = 151668;
        return e;
    }
}

class Lfm2CudaEngine extends CudaEngineBase {
    static async create(gguf, opts) {
        const e = await super._create(gguf, new Lfm2Engine(gguf), 1, 'token_embd_norm.weight', opts);
        e.THINK_ID = 124901; e.END_THINK_ID = 124902;
        return e;
    }
}

if (typeof module !== 'undefined') module.exports = { Qwen3CudaEngine, Lfm2CudaEngine };
