/*
 * qq3.h -- C ABI of libqq3cuda.so, the sm_100a (B200) backend for the QwenQwen3.js
 * quantised inference path.
 *
 * The reference engines (src/qwen3-engine.js, src/lfm2-engine.js, and their WebGPU
 * twins in src/webgpu.js) call an ops layer with GGUF tensor-meta objects and host
 * Float32Arrays.  This header is what a binding (N-API addon, ctypes, cgo, ...) calls
 * instead: plain pointers and sizes, no framework types.
 *
 * Conventions
 *   - Every function returns QQ_OK (0) or a negative QQ_ERR_* code; qq_last_error()
 *     returns a thread-local description of the last failure on the calling thread
 *     (the JS engines throw; webgpu.js:443).
 *   - Pointers named *_dev are device pointers on the context's device; every other
 *     buffer is host memory, copied by the call (the caller keeps ownership, as with
 *     GPUDevice.uploadBuffer, webgpu.js:370-383).
 *   - Calls that take or return host buffers are synchronous.  Calls on *_dev buffers
 *     are enqueued on the context stream (qq_set_stream) and complete in stream order;
 *     qq_synchronize() waits for them.
 *   - There is no CPU fallback: without a usable sm_100 device qq_init fails.
 */
#ifndef QQ3_H
#define QQ3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QQ_OK 0
#define QQ_ERR_INVALID -1     /* bad argument, shape or state */
#define QQ_ERR_CUDA -2        /* CUDA runtime error */
#define QQ_ERR_OOM -3         /* device allocation failed */
#define QQ_ERR_UNSUPPORTED -4 /* valid request this build does not implement */

/* ggml tensor types accepted by qq_upload_tensor (gguf.js:25-34) */
#define QQ_TYPE_F32 0
#define QQ_TYPE_Q8_0 8
/* k-quants (tensor.js:267-664): 256-value superblocks of 84 / 110 / 144 / 176 / 210 bytes; kept
 * raw on the device.  qq_dequant, qq_q8_matmul and qq_embed accept them, and a dense Qwen3 model
 * may use them for any projection, the embedding and the lm_head (ne0 % 256 == 0). */
#define QQ_TYPE_Q2_K 10
#define QQ_TYPE_Q3_K 11
#define QQ_TYPE_Q4_K 12
#define QQ_TYPE_Q5_K 13
#define QQ_TYPE_Q6_K 14

typedef struct qq_ctx qq_ctx;
typedef struct qq_tensor qq_tensor;
typedef struct qq_model qq_model;

/* ---------------------------------------------------------------- context */

/* Thread-local message of the last failed call on this thread ("" if none). */
const char* qq_last_error(void);

/* Open a context on devices[0..n_devices).  Replaces GPUDevice.create (webgpu.js:355-367).
 * This build drives one device per context (n_devices == 1); multi-GPU runs use one
 * process and one context per GPU. */
int qq_init(const int* devices, int n_devices, qq_ctx** out);
int qq_destroy(qq_ctx* ctx);
/* ---- multi-GPU: one NCCL communicator per context (one process per GPU) ----
 * The expert-parallel and tensor-parallel paths enqueue their exchanges on the context stream
 * through this communicator.  Rank 0 makes the id (qq_comm_unique_id), the host distributes it,
 * every rank calls qq_comm_init; a rank that does not join within timeout_ms (0 = 120 s) turns
 * into QQ_ERR_CUDA on the others and an aborted communicator, not a hang.  No reference
 * counterpart: the reference runs on one device. */
#define QQ_COMM_ID_BYTES 128
int qq_comm_unique_id(void* id_out);
int qq_comm_init(qq_ctx* ctx, const void* id, int rank, int world, int timeout_ms);
int qq_comm_destroy(qq_ctx* ctx);
/* Make subsequent work of this context run on a caller-owned cudaStream_t (NULL = the
 * context's own stream). */
int qq_set_stream(qq_ctx* ctx, void* cuda_stream);
int qq_synchronize(qq_ctx* ctx);

/* ---------------------------------------------------------------- tensors */

/* Upload one GGUF tensor from its raw file bytes.  Replaces GPUDevice.uploadBuffer of
 * new Uint8Array(meta.buffer, meta.offset, meta.nbytes) (webgpu.js:370-383, 569-624,
 * 1538-1629).  Q8_0 data is the 34-byte block stream (fp16 d + 32 int8, tensor.js:1-2);
 * ne[0] must be a multiple of 32.  nbytes may exceed the exact size (gguf.js pads each
 * tensor slice to 256 bytes, gguf.js:78-79).  n_dims in 1..3. */
int qq_upload_tensor(qq_ctx* ctx, const void* host, size_t nbytes, int ggml_type, const int64_t* ne, int n_dims,
                     qq_tensor** out);
int qq_free_tensor(qq_tensor* t);
/* Streaming upload of a whole model (GGUFReader.fromFile's per-tensor slices, gguf.js:350-374,
 * each uploaded raw as GPUDevice.uploadBuffer does, webgpu.js:370-383, 569-624): the bytes go
 * through a ring of pinned staging slots (staging_bytes in all; 0 = 128 MiB) so that the host
 * copy of one chunk, the DMA of the previous one and the device-side Q8_0 split of the one
 * before overlap.  qq_upload_tensor_async returns once the caller's bytes are copied (the caller
 * keeps ownership, as with qq_upload_tensor); the tensors it creates may be used after
 * qq_upload_finish, which waits for the device work, frees the ring and the uploader (also on
 * failure) and reports the bytes uploaded. */
typedef struct qq_uploader qq_uploader;
int qq_upload_begin(qq_ctx* ctx, size_t staging_bytes, qq_uploader** out);
int qq_upload_tensor_async(qq_uploader* u, const void* host, size_t nbytes, int ggml_type, const int64_t* ne,
                           int n_dims, qq_tensor** out);
int qq_upload_finish(qq_uploader* u, size_t* bytes_out);
/* Shape/type of an uploaded tensor (the meta.shape / meta.type fields, gguf.js:235-254). */
int qq_tensor_info(const qq_tensor* t, int* ggml_type, int64_t* ne4, int* n_dims);
/* out_dev[i] = element i in storage order, dequantised as q*d (bit-exact; the column
 * readers of tensor.js:56-77 and _readWeightF32, tensor.js:80-100). */
int qq_dequant(const qq_tensor* t, float* out_dev);

/* ---------------------------------------------------------------- ops */

/* y_dev[m][c] = sum_k x_dev[m][k] * W[k, c] for m < M: M independent calls of
 * matmulQ80xF32 / matmulGeneric (tensor.js:26-53, 485-496); W is [K, N] Q8_0 and a 3-D
 * tensor is taken as its first [K, N] matrix, as the JS does. */
int qq_q8_matmul(qq_ctx* ctx, const qq_tensor* W, const float* x_dev, int M, float* y_dev);
/* Row-wise RMSNorm, y = w * x / sqrt(mean(x^2) + eps) (rmsnorm, tensor.js:103-114; per
 * head, perHeadRMSNorm, tensor.js:117-129).  w is an F32 tensor of length n. y may equal x. */
int qq_rmsnorm(qq_ctx* ctx, const float* x_dev, int64_t n_rows, int n, const qq_tensor* w, float eps,
               float* y_dev);
/* applyRoPE (tensor.js:132-147) in place on n_rows rows of n_heads x head_dim floats, row r at
 * position pos0 + r: split-half rotation by theta = position / base^(i / (head_dim/2)), cos and
 * sin computed in double and rounded to f32 (the table the model's RoPE kernels read). */
int qq_rope(qq_ctx* ctx, float* x_dev, int n_rows, int n_heads, int head_dim, int pos0, double base);
/* The attention core of one decode step, _selfAttentionCore (qwen3-engine.js:249-291,
 * lfm2-engine.js:329-378): GQA attention of q_dev [n_head][head_dim] (already normalised and
 * rotated) over positions 0..pos of a K/V cache laid out [n_kv][max_ctx][head_dim] (f32, the
 * kv-cache.js:8-11 layout), query head h reading KV head floor(h n_kv / n_head); out_dev
 * [n_head][head_dim].  Positions split over CTAs, merged in split order.  head_dim 64 or 128. */
int qq_attention_decode(qq_ctx* ctx, const float* q_dev, const float* k_cache_dev, const float* v_cache_dev,
                        int n_head, int n_kv, int head_dim, int max_ctx, int pos, float* out_dev);
/* embeddingLookupQ80 (tensor.js:56-77) of n host token ids: out_dev [n][ne0], exact. */
int qq_embed(qq_ctx* ctx, const qq_tensor* E, const int32_t* tokens, int n, float* out_dev);
/* SwiGLU pieces siluInPlace + mulInPlace (tensor.js:168-180): h = silu(g) * u over n floats. */
int qq_swiglu(qq_ctx* ctx, const float* g_dev, const float* u_dev, int64_t n, float* h_dev);
/* addVec (tensor.js:181-185): x += d over n floats (the residual add). */
int qq_add(qq_ctx* ctx, float* x_dev, const float* d_dev, int64_t n);

/* ---------------------------------------------------------------- model */

/* Per-layer tensor slots; names as the engines look them up (qwen3-engine.js:46-75,
 * lfm2-engine.js:88-140). */
enum {
    QQ_ATTN_NORM = 0, /* blk.N.attn_norm.weight */
    QQ_FFN_NORM,      /* blk.N.ffn_norm.weight */
    QQ_WQ,            /* blk.N.attn_q.weight */
    QQ_WK,            /* blk.N.attn_k.weight */
    QQ_WV,            /* blk.N.attn_v.weight */
    QQ_WO,            /* blk.N.attn_output.weight */
    QQ_Q_NORM,        /* blk.N.attn_q_norm.weight */
    QQ_K_NORM,        /* blk.N.attn_k_norm.weight */
    QQ_CONV,          /* blk.N.shortconv.conv.weight (F32 [3, E]) */
    QQ_IN_PROJ,       /* blk.N.shortconv.in_proj.weight */
    QQ_OUT_PROJ,      /* blk.N.shortconv.out_proj.weight */
    QQ_FFN_GATE,      /* blk.N.ffn_gate.weight */
    QQ_FFN_UP,        /* blk.N.ffn_up.weight */
    QQ_FFN_DOWN,      /* blk.N.ffn_down.weight */
    QQ_ROUTER,        /* blk.N.ffn_gate_inp.weight */
    QQ_GATE_EXPS,     /* blk.N.ffn_gate_exps.weight [E_in, F, n_expert] */
    QQ_UP_EXPS,       /* blk.N.ffn_up_exps.weight */
    QQ_DOWN_EXPS,     /* blk.N.ffn_down_exps.weight [F, E_in, n_expert] */
    QQ_EXP_BIAS,      /* blk.N.exp_probs_b.bias (F32 [n_expert]) */
    QQ_SLOT_COUNT
};

typedef struct qq_layer_desc {
    int32_t is_attn; /* 1 = GQA attention; 0 = LFM2 short-conv (shortconv.conv.weight present, lfm2-engine.js:90-91) */
    int32_t is_moe;  /* 1 = MoE FFN (Lfm2Engine._moEFFN); 0 = dense SwiGLU */
    qq_tensor* t[QQ_SLOT_COUNT]; /* NULL where a slot does not apply */
} qq_layer_desc;

#define QQ_ARCH_QWEN3 0
#define QQ_ARCH_LFM2 1

/* The hyper-parameters the engine constructors read (gguf.js getArch :264-291,
 * qwen3-engine.js:2-29, lfm2-engine.js:15-74) plus the tensors they bind. */
typedef struct qq_model_desc {
    int32_t arch;
    int32_t n_layers;
    int32_t n_embd;
    int32_t n_head;
    int32_t n_head_kv;
    int32_t head_dim;
    int32_t n_vocab;
    int32_t n_expert;      /* 0 for dense models */
    int32_t n_expert_used;
    int32_t max_ctx;       /* KV capacity in positions (the JS default is min(ctx, 4096)) */
    int32_t n_seq;         /* independent sequences (KV caches / conv states) */
    float rms_eps;
    double rope_base;
    qq_tensor* tok_embd;    /* token_embd.weight */
    qq_tensor* output_norm; /* output_norm.weight (Qwen3) / token_embd_norm.weight (LFM2) */
    qq_tensor* output;      /* output.weight, or NULL for tied embeddings */
    const qq_layer_desc* layers;
    /* Expert parallelism (no reference counterpart): > 1 splits the experts of every MoE layer
     * evenly over ep_world ranks -- this rank (its context's communicator rank, qq_comm_init with
     * world ep_world) holds experts [rank E/ep_world, (rank+1) E/ep_world), so the expert tensors
     * have ne[2] = E/ep_world -- and every MoE layer exchanges token rows with the other ranks.
     * Every rank then makes the same forward calls with the same token counts (the calls are
     * collective).  0 or 1: one rank holds every expert. */
    int32_t ep_world;
    /* Tensor parallelism for dense Qwen3 (no reference counterpart): > 1 splits every layer over
     * tp_world ranks (the context's communicator, world tp_world).  The hyper-parameters above stay
     * the whole model's; the tensors are this rank's shards: wq/wk/wv the rows of its query heads
     * [r nH/G, (r+1) nH/G) and KV heads, wo the matching input columns, ffn_gate/up the rows of
     * its FFN units [r F/G, (r+1) F/G) and ffn_down those input columns, output (required) the
     * vocab rows [r V/G, (r+1) V/G); token_embd and the norms whole.  wo and ffn_down partial
     * sums are all-reduced; the greedy id is the first maximum over the ranks' shards.  Steps run
     * through qq_forward / qq_forward_batch (collective: every rank makes the same calls).
     * 0 or 1: no split. */
    int32_t tp_world;
} qq_model_desc;

/* Bind uploaded tensors into an engine.  Replaces Qwen3GPUEngine.create /
 * Lfm2GPUEngine.create (webgpu.js:498-567, 1470-1536).  Tensors stay owned by the caller
 * and must outlive the model. */
int qq_model_create(qq_ctx* ctx, const qq_model_desc* desc, qq_model** out);
int qq_model_destroy(qq_model* m);

/* forward(tokenId, position, skipLogits) for n_tokens consecutive tokens of sequence
 * seq_id starting at position pos0 (qwen3-engine.js:115-245, lfm2-engine.js:228-269,
 * webgpu.js:806-875, 1954-2034); n_tokens > 1 is exactly n sequential forward() calls.
 * Only the last token produces logits, and only when want_logits != 0:
 *   logits_out (nullable) receives n_vocab floats,
 *   argmax_out (nullable) receives the greedy id (sampleGreedy, tensor.js:231-237) with
 *   suppress_id (>= 0) excluded first (thinking suppression, tensor.js:247-248). */
int qq_forward(qq_model* m, const int32_t* token_ids, int n_tokens, int seq_id, int pos0, int want_logits,
               float* logits_out, int32_t* argmax_out, int suppress_id);
/* One forward(tokenId, position, false) step for each of n independent sequences at once:
 * token_ids[i] at position positions[i] of sequence seq_ids[i] (distinct ids, each < n_seq),
 * the same as n separate qq_forward calls (qwen3-engine.js:115-245, lfm2-engine.js:228-269) up to
 * the tensor-core GEMM's f32 accumulation order.  The reference serves one sequence per engine;
 * this is the batched decode of the 16-sequence Qwen3-8B configuration: each weight streams from
 * HBM once for all n rows.  With want_logits != 0:
 *   logits_out (nullable) receives n x n_vocab floats (row i for sequence seq_ids[i]),
 *   argmax_out (nullable) receives n greedy ids (sampleGreedy, tensor.js:231-237) with
 *   suppress_id (>= 0) excluded (tensor.js:247-248).
 * The routing record of each MoE layer (qq_read_routing) is that of row n-1. */
int qq_forward_batch(qq_model* m, const int32_t* seq_ids, const int32_t* token_ids, const int32_t* positions, int n,
                     int want_logits, float* logits_out, int32_t* argmax_out, int suppress_id);
/* Greedy generate(): reset, prefill, then up to max_steps decode steps, stopping at
 * eos_id (qwen3-engine.js:397-457, lfm2-engine.js:523-583, webgpu.js:1032-1098,
 * 2047-2117 with temperature 0 and thinkingMode 'suppress').  out_tokens gets the
 * generated ids; *n_out their count. */
int qq_generate(qq_model* m, int seq_id, const int32_t* prompt, int n_prompt, int max_steps, int think_id,
                int eos_id, int32_t* out_tokens, int* n_out);
/* ---------------------------------------------------------------- sampling on the device */

/* thinkingMode (tensor.js:240-243) */
#define QQ_THINK_SUPPRESS 0 /* logits[think_id] = -Infinity before sampling */
#define QQ_THINK_SHORTEN 1  /* until end_think_id was produced, force it while it ranks in the top_k */
#define QQ_THINK_FULL 2     /* no control */
#define QQ_SAMPLE_MAX_TOP_K 1024

/* The generate() sampling options (qwen3-engine.js:397-405, lfm2-engine.js:523-542).  temperature
 * <= 0 is greedy; otherwise sampleTopPTopK (tensor.js:188-228) with 1 <= top_k <= 1024 (the JS
 * default is 40; top_k = 0, "no limit", is not served on the device).  Think ids outside the
 * vocabulary disable think control.  seed picks the stream of uniform draws that replaces
 * Math.random(): the draw after the logits of position p of sequence s is
 * qq_sample_uniform(seed, s, p). */
typedef struct qq_sample_params {
    double temperature;
    double top_p;
    int32_t top_k;
    int32_t think_mode; /* QQ_THINK_* */
    int32_t think_id, end_think_id;
    uint64_t seed;
} qq_sample_params;

/* forward(token_id, pos, false) then sampleWithThinkControl on the device: *token_out is the
 * next token (4-byte readback instead of the logits).  think_done is the caller's
 * thinkOpts.thinkingDone.  Replaces the logits readback + host sampling of generate()
 * (webgpu.js:2030, 2092). */
int qq_forward_sample(qq_model* m, int32_t token_id, int seq_id, int pos, const qq_sample_params* params,
                      int think_done, int32_t* token_out);
/* generate() with sampling (qwen3-engine.js:397-457, lfm2-engine.js:523-583): prefill, then up
 * to max_steps sampled tokens; without a stop token (eos_id < 0) every step and its sampling run
 * on the device with no host round trip. */
int qq_generate_sample(qq_model* m, int seq_id, const int32_t* prompt, int n_prompt, int max_steps,
                       const qq_sample_params* params, int eos_id, int32_t* out_tokens, int* n_out);
/* Op level: sampleWithThinkControl over logits_dev[n] with the given uniform draw r in [0, 1)
 * (tensor.js:244-265 with Math.random() = r). */
int qq_sample_logits(qq_ctx* ctx, const float* logits_dev, int n, const qq_sample_params* params, double r,
                     int think_done, int32_t* token_out);
/* The uniform draw the device sampler uses after the logits of position pos of sequence seq_id. */
int qq_sample_uniform(uint64_t seed, int seq_id, int pos, double* r_out);

/* resetState()/resetKVCache() (lfm2-engine.js:216-224, kv-cache.js:50-52): zero the
 * conv states of seq_id; the KV cache is overwritten before it is read. */
int qq_reset(qq_model* m, int seq_id);
/* Routing record of the most recent token for MoE layer moe_layer (0-based among MoE
 * layers): [top_k ids | top_k normalised weights | n_expert sigmoid probs] as floats, the
 * buffer read by _readbackRoutingData (webgpu.js:1617-1618, 1922-1945). */
int qq_read_routing(qq_model* m, int moe_layer, float* out);
/* expertMask (lfm2-engine.js:464, router-viz.html:274): masked experts are skipped in
 * the combine without renormalising.  n == 0 clears the mask. */
int qq_set_expert_mask(qq_model* m, const int32_t* ids, int n);
/* Hidden state after every layer for the last token of a qq_forward call, [n_layers][n_embd]
 * (the parity probe used by the tests; the JS logs per-layer maxima, qwen3-engine.js:189-215). */
int qq_forward_dump(qq_model* m, int32_t token_id, int seq_id, int pos, float* hidden_out);
/* Device-resident greedy decode: starting from token first_token at position pos0, run
 * n_steps forward+argmax steps with the next token fed back on the device (no host round
 * trip).  tokens_out (nullable, host) receives the n_steps generated ids. */
int qq_decode_loop(qq_model* m, int seq_id, int first_token, int pos0, int n_steps, int suppress_id,
                   int32_t* tokens_out);

/* ---------------------------------------------------------------- diagnostics */

/* Per-phase trace of the persistent decode step (no reference counterpart; the breakdown behind
 * the decode-step profile): enable = 1 makes every later step's CTAs stamp %globaltimer at their
 * start and at the end of each phase (the last step's stamps are kept); enable = 0 stops it.
 * stamps_out (nullable) receives the stamps of the last traced step, [n_ctas][n_phases + 1] ns;
 * kinds_out (nullable, n_phases ints) each phase's type | epilogue << 8 | routed << 16. */
int qq_decode_trace(qq_model* m, int enable, uint64_t* stamps_out, int32_t* kinds_out, int* n_phases, int* n_ctas);
/* Sub-phase stamps of the last traced step: out (nullable) receives [n_ctas][n_phases][*n_sub] ns
 * stamps of thread 0 of each CTA at fixed points of a phase (0 where a phase does not reach one):
 * 0 input wait over, 1 input staged, 2 token routed, 3 first weight stage landed, 4 first part
 * done (gate/up + SwiGLU; all GEMV rows; attention keys), 5 second part done (down / out_proj),
 * 6 bulk reduction performed (attention: split counter taken), 7 output published, 8 router stage
 * landed, 9 router logits complete, 10 the producer thread saw the routing, 11 the producer thread
 * issued the phase's first weight stage, 12-14 the top-k warp starts / has the ranks / has the ids
 * and weights, 15 the CTA starts routing. */
int qq_decode_trace_sub(qq_model* m, uint64_t* out, int* n_sub);
/* Expert-parallel models: switch the CUDA-event split of every MoE exchange on (enable = 1) or
 * off, and read (ms_out, nullable, 5 floats) the time summed since the last call over the
 * exchanges recorded: [dispatch (plan + gather + NCCL send/recv), experts (owner GEMMs),
 * return (NCCL send/recv back), combine, number of exchanges]. */
int qq_ep_profile(qq_model* m, int enable, float* ms_out);

/* Statistics of a model (no reference counterpart; used by the benchmark):
 *   QQ_STAT_STEP_KERNELS  kernels launched by one decode step with logits
 *   QQ_STAT_N_MOE         number of MoE layers
 *   QQ_STAT_STEP_PHASES   phases of the persistent decode step with logits (0: per-phase kernels)
 *   QQ_STAT_MOE_FUSED     MoE layers the persistent step runs as one fused phase */
#define QQ_STAT_STEP_KERNELS 0
#define QQ_STAT_N_MOE 1
#define QQ_STAT_STEP_PHASES 2
#define QQ_STAT_MOE_FUSED 3
int qq_model_stat(qq_model* m, int what, int64_t* value);
/* Time one kernel class over every MoE layer in turn (so no layer's weights are still in
 * L2 when it is read again), iters rounds, using the routing of the latest token; returns
 * the mean duration of one launch in *ms (CUDA events on the context stream).  Clobbers the
 * hidden state of the current step.  No reference counterpart.
 *   QQ_KERN_MOE_LAYER   router + expert gate/up + expert down-combine of one layer
 *   QQ_KERN_MOE_GATEUP  the expert gate/up SwiGLU GEMV
 *   QQ_KERN_MOE_DOWN    the expert down GEMV + weighted combine */
#define QQ_KERN_MOE_LAYER 0
#define QQ_KERN_MOE_GATEUP 1
#define QQ_KERN_MOE_DOWN 2
int qq_bench_kernel(qq_model* m, int what, int iters, float* ms);

/* ---------------------------------------------------------------- MoE block */

/* The LFM2-MoE FFN (Lfm2Engine._moEFFN, lfm2-engine.js:413-487; WGSL_MOE_SIGMOID_TOPK +
 * WGSL_MATMUL_EXPERT_Q80 + WGSL_AXPY_EXPERT, webgpu.js:1243-1283, 1290-1324, 1441-1454) on
 * T token rows: x_dev [T][E_in] is the ffn-normalised input, out_dev [T][E_in] receives
 * sum_k w_k * expert_k(x); routing_dev (nullable) [T][2*top_k + n_expert] the records.
 * layer->t[QQ_ROUTER], [QQ_GATE_EXPS], [QQ_UP_EXPS], [QQ_DOWN_EXPS], [QQ_EXP_BIAS] are used. */
int qq_moe_block(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k, const float* x_dev, int T,
                 float* out_dev, float* routing_dev);

/* ---------------------------------------------------------------- expert-parallel MoE pieces */

/* No reference counterpart (the JS runs every expert in one process): the three parts of
 * qq_moe_block a rank of an expert-parallel group calls around its own row exchange (NCCL
 * all-to-all in the caller), with experts sharded evenly over the ranks.
 *  qq_moe_route    router logits, sigmoid, top-k and weights of T token rows
 *                  (lfm2-engine.js:417-447): idx_dev [T][top_k] global expert ids, w_dev
 *                  [T][top_k], routing_dev (nullable) [T][2*top_k + n_expert] the records.  Uses
 *                  layer->t[QQ_ROUTER] and [QQ_EXP_BIAS].
 *  qq_moe_experts  y_dev[r] = down_e(silu(gate_e . x_r) * (up_e . x_r)) for R rows x_dev [R][K],
 *                  e = eid_dev[r] in 0..n_local-1, the rank's own experts: layer->t[QQ_GATE_EXPS],
 *                  [QQ_UP_EXPS], [QQ_DOWN_EXPS] hold n_local experts (GGUF [K, F, n_local],
 *                  [F, K, n_local]).  Unweighted (the weights stay with the token's owner).
 *  qq_moe_combine  out_dev[t] = sum over slots s (in order) of w_dev[t][s] * y_dev[pos_dev[t][s]]
 *                  (lfm2-engine.js:459-486), rows of K floats. */
int qq_moe_route(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k, const float* x_dev, int T,
                 int32_t* idx_dev, float* w_dev, float* routing_dev);
int qq_moe_experts(qq_ctx* ctx, const qq_layer_desc* layer, int n_local, const float* x_dev, const int32_t* eid_dev,
                   int R, float* y_dev);
int qq_moe_combine(qq_ctx* ctx, const float* y_dev, const int32_t* pos_dev, const float* w_dev, int T, int top_k,
                   int K, float* out_dev);

/* ---------------------------------------------------------------- allocation-free MoE block */

/* No counterpart in the reference.  qq_moe_block without any device allocation, for callers
 * that cannot let the library call cudaMalloc while a layer runs: a host that owns all device
 * memory through its own pool or budget (an embedding runtime such as a JS engine's addon, or a
 * serving process that pre-plans its memory), or code that issues the block while recording
 * its own stream work.  Inputs and outputs are the caller's, exactly as for qq_moe_block; the
 * scratch is one fixed device array of the library module (256 KiB, held by every GPU that
 * loads the library until the process exits).
 * Limits: T <= QQ_NOALLOC_MAX_TOKENS, expert FFN width <= QQ_NOALLOC_MAX_FF, top_k == 4,
 * n_expert <= 32; beyond them the call fails with QQ_ERR_INVALID and does no GPU work.
 * The first call on a device resolves the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  All calls on a device share the array and it
 * keeps the last call's contents: calls whose GPU work overlaps race.
 * Cost: the rows are served token by token (two expert GEMV launches per row, 2T launches for T
 * rows), where qq_moe_block regroups T >= 16 rows by expert on the tensor cores, so large T is
 * much slower here than there. */
#define QQ_NOALLOC_MAX_TOKENS 1024
#define QQ_NOALLOC_MAX_FF 4096
int qq_moe_block_noalloc(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k, const float* x_dev,
                         int T, float* out_dev, float* routing_dev);

#ifdef __cplusplus
}
#endif
#endif /* QQ3_H */
