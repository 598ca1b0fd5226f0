/*
 * qq3_oracle.h -- CPU restatement of the QwenQwen3.js CPU inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * The product (libqq3cuda.so) never calls it.
 *
 * Parity status: UNPINNED.  The reference is browser JavaScript (the src directory) with no
 * tests, fixtures or golden vectors, and no JavaScript runtime exists on this
 * machine or on the GPU box, so the reference itself cannot be executed to pin
 * this restatement.  It follows the JS arithmetic line by line instead:
 *   - accumulators are IEEE doubles (JS numbers),
 *   - values are rounded to float exactly where the JS stores into a Float32Array,
 *   - products keep the JS evaluation order (e.g. (x*q)*d in matmulQ80xF32),
 *   - built with -ffp-contract=off so no fused multiply-add changes a rounding.
 * libm's exp/sin/cos/pow may differ from V8's by at most 1 ulp of a double.
 *
 * Every function cites the reference file:line it restates.
 */
#ifndef QQ3_ORACLE_H
#define QQ3_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor types used on this path (gguf.js:25-34) */
#define ORC_TYPE_F32 0
#define ORC_TYPE_F16 1
#define ORC_TYPE_Q8_0 8
/* k-quants (tensor.js:267-664): 256-value superblocks */
#define ORC_TYPE_Q2_K 10
#define ORC_TYPE_Q3_K 11
#define ORC_TYPE_Q4_K 12
#define ORC_TYPE_Q5_K 13
#define ORC_TYPE_Q6_K 14

/* A raw GGUF tensor: host bytes exactly as stored in the file, plus its ggml shape
 * (ne[0] fastest-varying), i.e. the meta object of gguf.js:235-254. */
typedef struct orc_tensor {
    const uint8_t* data;   /* NULL = tensor absent */
    int32_t type;
    int32_t n_dims;
    int64_t ne[4];
} orc_tensor;

/* Per-layer tensor slots (names as read by qwen3-engine.js:46-75, lfm2-engine.js:88-140) */
enum {
    ORC_ATTN_NORM = 0,  /* blk.N.attn_norm.weight            */
    ORC_FFN_NORM,       /* blk.N.ffn_norm.weight             */
    ORC_WQ,             /* blk.N.attn_q.weight               */
    ORC_WK,             /* blk.N.attn_k.weight               */
    ORC_WV,             /* blk.N.attn_v.weight               */
    ORC_WO,             /* blk.N.attn_output.weight          */
    ORC_Q_NORM,         /* blk.N.attn_q_norm.weight          */
    ORC_K_NORM,         /* blk.N.attn_k_norm.weight          */
    ORC_CONV,           /* blk.N.shortconv.conv.weight       */
    ORC_IN_PROJ,        /* blk.N.shortconv.in_proj.weight    */
    ORC_OUT_PROJ,       /* blk.N.shortconv.out_proj.weight   */
    ORC_FFN_GATE,       /* blk.N.ffn_gate.weight             */
    ORC_FFN_UP,         /* blk.N.ffn_up.weight               */
    ORC_FFN_DOWN,       /* blk.N.ffn_down.weight             */
    ORC_ROUTER,         /* blk.N.ffn_gate_inp.weight         */
    ORC_GATE_EXPS,      /* blk.N.ffn_gate_exps.weight        */
    ORC_UP_EXPS,        /* blk.N.ffn_up_exps.weight          */
    ORC_DOWN_EXPS,      /* blk.N.ffn_down_exps.weight        */
    ORC_EXP_BIAS,       /* blk.N.exp_probs_b.bias            */
    ORC_SLOT_COUNT
};

typedef struct orc_layer {
    int32_t is_attn;    /* 1 = GQA attention, 0 = LFM2 short-conv */
    int32_t is_moe;     /* 1 = MoE FFN, 0 = dense SwiGLU */
    orc_tensor t[ORC_SLOT_COUNT];
} orc_layer;

#define ORC_ARCH_QWEN3 0
#define ORC_ARCH_LFM2 1

typedef struct orc_model_desc {
    int32_t arch;
    int32_t n_layers;
    int32_t n_embd;
    int32_t n_head;
    int32_t n_head_kv;
    int32_t head_dim;
    int32_t n_vocab;
    int32_t n_expert;
    int32_t n_expert_used;
    int32_t max_ctx;      /* KV capacity (the JS caps at 4096; larger values are an uncapped extension) */
    double rms_eps;       /* the f32 GGUF value widened to double, as JS Number() does */
    double rope_base;
    orc_tensor tok_embd;
    orc_tensor output_norm;
    orc_tensor output;    /* data NULL => tied to tok_embd */
    const orc_layer* layers;
} orc_model_desc;

typedef struct orc_model orc_model;

void orc_set_threads(int n);
int orc_get_threads(void);

/* ---- per-op restatements ---- */
double orc_f16_to_double(uint16_t h);
void orc_matmul(const orc_tensor* w, const float* x, float* y);
void orc_matmul_rows(const orc_tensor* w, const float* x, int64_t m, float* y);
void orc_embedding(const orc_tensor* w, int32_t token, float* out);
void orc_dequant(const orc_tensor* w, float* out);
void orc_rmsnorm(float* x, int64_t n, const orc_tensor* w, double eps);
void orc_per_head_rmsnorm(float* x, int n_heads, int head_dim, const orc_tensor* w, double eps);
void orc_rope(float* x, int n_heads, int head_dim, int position, double base);
void orc_softmax(float* a, int64_t start, int64_t end);
void orc_silu(float* a, int64_t n);
void orc_mul(float* a, const float* b, int64_t n);
void orc_add(float* a, const float* b, int64_t n);
int32_t orc_sample_greedy(const float* logits, int64_t n);
int32_t orc_sample_suppress(float* logits, int64_t n, int32_t think_id);

/* LFM2 MoE FFN on T independent token rows (lfm2-engine.js:413-487).
 * normed: [T][n_embd] (post ffn_norm), out: [T][n_embd] = sum_k w_k * expert_k(normed)
 * routing (nullable): [T][2*top_k + n_expert] = [top-k ids | normalised weights | sigmoid probs]
 * mask (nullable): n_expert flags, 1 = skip that expert (expertMask). */
void orc_lfm2_moe(const orc_layer* layer, int n_embd, int n_expert, int top_k,
                  const float* normed, int64_t T, float* out, float* routing,
                  const uint8_t* mask);

/* ---- full engines ---- */
int orc_model_create(const orc_model_desc* desc, orc_model** out);
void orc_model_destroy(orc_model* m);
void orc_reset(orc_model* m);
int orc_set_expert_mask(orc_model* m, const int32_t* ids, int n);
/* One forward(tokenId, position, skipLogits) call.
 * logits (nullable, ignored when skip_logits): n_vocab floats.
 * hidden_dump (nullable): [n_layers][n_embd] hidden state after each layer.
 * routing (nullable): [n_moe_layers][2*top_k + n_expert], in layer order. */
int orc_forward(orc_model* m, int32_t token, int32_t position, int skip_logits,
                float* logits, float* hidden_dump, float* routing);
/* generate() with temperature 0 and thinkingMode 'suppress' (greedy).
 * out_tokens receives at most max_steps ids; returns how many were produced. */
int orc_generate(orc_model* m, const int32_t* prompt, int n_prompt, int max_steps,
                 int32_t think_id, int32_t eos_id, int32_t* out_tokens);
int orc_n_moe_layers(const orc_model* m);

#ifdef __cplusplus
}
#endif
#endif
