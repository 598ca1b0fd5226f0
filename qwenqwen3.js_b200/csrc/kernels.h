// kernels.h -- host-side launchers of the sm_100a kernels (internal to libqq3cuda.so).
#pragma once
#include "common.cuh"

namespace qq3 {

// Input staging of a GEMV launch: nvec input vectors of length K (K % 32 == 0) are copied
// into shared memory once per CTA.  With norm_w set (nvec == 1) the copy is the
// RMSNorm of x (tensor.js:103-114) so the norm is fused into the consumer.
struct XStage {
    const float* x[8] = {nullptr};
    int nvec = 1;
    int K = 0;
    const float* norm_w = nullptr;
    float eps = 0.f;
};

// y[i] (+)= W[row0 + i] . x for i < n
void launch_gemv_rows(const DTensor& W, int64_t row0, int64_t n, const XStage& st, float* y, bool residual,
                      cudaStream_t s);
// Q|K|V projections into one buffer qkv = [wq rows | wk rows | wv rows]
void launch_gemv_qkv(const DTensor& wq, const DTensor& wk, const DTensor& wv, const XStage& st, float* qkv,
                     cudaStream_t s);
// h[j] = silu(gate[j] . x) * (up[j] . x)
void launch_gemv_swiglu(const DTensor& gate, const DTensor& up, const XStage& st, float* h, cudaStream_t s);
// LFM2 short-conv: in_proj rows (j, E+j, 2E+j) -> B, C, x; depthwise causal conv with the
// rolling state (updated in place); y[j] = C * conv_out (lfm2-engine.js:282-321)
void launch_gemv_conv(const DTensor& in_proj, const float* conv_w, float* state, const XStage& st, float* y,
                      cudaStream_t s);
// logits = W . x and a fused first-max argmax into *best (packed key, see argmax_key).
// *suppress_dev >= 0 is excluded from the argmax (thinking suppression, tensor.js:247-248).
void launch_gemv_logits_argmax(const DTensor& W, const XStage& st, float* logits, unsigned long long* best,
                               const int* suppress_dev, cudaStream_t s);
// MoE expert gate/up for one token: h[k][j] = silu(gate_e . x) * (up_e . x), e = idx[k]
void launch_moe_gateup(const DTensor& gate_exps, const DTensor& up_exps, const int* idx, const uint32_t* mask,
                       int top_k, const XStage& st, float* h, cudaStream_t s);
// MoE down + weighted combine + residual: hidden[j] += sum_k w[k] * (down_e[k] . h[k])
void launch_moe_down_combine(const DTensor& down_exps, const int* idx, const float* w, const uint32_t* mask,
                             int top_k, const float* h, float* hidden, cudaStream_t s);

// ---- misc kernels (kernels_misc.cu) ----
void launch_repack_q8(const uint8_t* raw, int64_t n_blocks, int8_t* qs, __half* d, cudaStream_t s);
void launch_dequant_q8(const DTensor& W, float* out, cudaStream_t s);
// hidden = dequantised row `token` of the embedding (tensor.js:56-77); token read from device
void launch_embed(const DTensor& E, const int* token, float* hidden, unsigned long long* argmax_reset,
                  cudaStream_t s);
// in place RMSNorm over n_rows rows of length n (tensor.js:103-114 / 117-129)
void launch_rmsnorm(float* x, int64_t n_rows, int n, const float* w, float eps, float* y, cudaStream_t s);
// ctl = [token, pos]: token <- argmax, pos <- pos + 1, trace[pos] <- token (device-driven decode)
void launch_argmax_finish(const unsigned long long* best, int* ctl, int* trace, cudaStream_t s);

// ---- attention (kernels_attn.cu) ----
struct AttnArgs {
    const float* qkv;      // [n_head*hd | n_kv*hd | n_kv*hd] raw projections (pre norm/rope)
    const float* q_norm;   // [hd]
    const float* k_norm;   // [hd]
    const float* rope_cs;  // [max_ctx][hd/2][2] cos, sin
    float* k_cache;        // [n_kv][max_ctx][hd] for this layer (and sequence)
    float* v_cache;
    float* out;            // [n_head*hd]
    float* part;           // scratch: [n_head][n_split][hd + 2]
    unsigned int* counter; // scratch: [n_kv] arrival counters (self-resetting)
    const int* pos;        // device position
    int n_head, n_kv, hd, max_ctx, n_split;
    float eps;
};
void launch_attention_decode(const AttnArgs& a, cudaStream_t s);
int attention_splits(int max_ctx);

// ---- MoE routing (kernels_moe.cu) ----
// LFM2 sigmoid router for T tokens (lfm2-engine.js:417-447).  x: [T][K] hidden rows,
// RMS-normalised in the prologue when norm_w is set.  Outputs per token t:
// record[t] = [ids | normalised weights | sigmoid probs] (2k+E floats), idx[t][k], w[t][k].
void launch_lfm2_router(const DTensor& router, const float* bias, const float* x, int T, const float* norm_w,
                        float eps, int n_expert, int top_k, float* record, int* idx, float* w, cudaStream_t s);
// The router of either family for T rows: softmax = true is the Qwen3-MoE rule
// (qwen3-engine.js:304-321), false the LFM2 rule above.  <= 128 experts, top_k <= 8, Q8_0 or F32 rows.
void launch_router(const DTensor& router, const float* bias, const float* x, int T, const float* norm_w, float eps,
                   int n_expert, int top_k, bool softmax, float* record, int* idx, float* w, cudaStream_t s);

int num_sms();

// ---- tensor-core Q8_0 matmul for M >= 2 rows (kernels_gemm.cu) ----
// y[M][N] = x[M][K] . W^T with x f32 row-major; x16 = scratch of gemm_q8_scratch_bytes(M, K).
bool gemm_q8_supported(const DTensor& W);
// true (default): three-product fp16 split, ~2^-22 relative like the f32 GEMV; QQ3_GEMM_FAST=1:
// one fp16 product (~1e-3).  Operand buffers then hold hi rows followed by lo rows.
bool gemm_exact();
size_t gemm_q8_scratch_bytes(int64_t M, int64_t K);
// x16_ready: x16 already holds x split into fp16 (the previous product had the same input)
void launch_gemm_q8(const DTensor& W, const float* x, int M, __half* x16, float* y, cudaStream_t s,
                    bool x16_ready = false);
// Few-row form for 2 <= M <= kGemmFewMax rows (multi-sequence decode): weights on the MMA's
// 128-row side, activation rows on its N side, K split over CTAs; rows_scratch holds
// gemm_rows_scratch_bytes(M) bytes whose first 1 KB (arrival tickets) is zero before the first
// launch and stays zero after each.  Other shapes (or rows_scratch null, or QQ3_GEMM_FAST) take
// launch_gemm_q8.
constexpr int kGemmFewMax = 32;
size_t gemm_rows_scratch_bytes(int M);
void gemm_rows_reset(void* rows_scratch, cudaStream_t s);
void launch_gemm_q8_few(const DTensor& W, const float* x, int M, __half* x16, void* rows_scratch, float* y,
                        cudaStream_t s, bool x16_ready = false);
// Grouped form: W holds groups of group_rows rows (e.g. the experts of a packed tensor); work
// item i = tiles[i] = (group, first row of a16, rows <= 128), *n_tiles items, max_tiles >= it.
struct GemmGroups {
    const int4* tiles;
    const int* n_tiles;
    int max_tiles;
};
// y[r][c] (row stride ldc) = a16[r] . W[group * group_rows + c] for c < group_rows
void launch_gemm_q8_f16(const DTensor& W, int64_t group_rows, const __half* a16, int M, float* y, int ldc,
                        const GemmGroups* groups, cudaStream_t s);
void launch_f32_to_f16(const float* x, __half* y, size_t n, cudaStream_t s);

// Per expert e of a packed Q8_0 tensor (rows = n_expert x R, K): t_qs[e][k][r] = qs[e R + r][k]
// and t_d[e][k/32][r] = d[e R + r][k/32] (the fused decode MoE reads down columns as rows).
void launch_transpose_experts(const DTensor& W, int n_expert, int8_t* t_qs, __half* t_d, cudaStream_t s);

// ---- MoE block for T rows regrouped by expert on the tensor cores (kernels_moe_grouped.cu) ----
// out[t] = sum_s w[t][s] * y[pos[t][s]] (w nullable: weight 1), rows of K floats
void launch_moe_combine_rows(const float* y, const int* pos, const float* w, int T, int top_k, int K, float* out,
                             cudaStream_t s);
size_t moe_grouped_scratch_bytes(int T, int top_k, int n_expert, int64_t K, int64_t F);
// idx/w: routed ids and weights [T][top_k]; out[T][K] = sum_s w[t][s] * down_e(silu(gate_e x) * up_e x)
// over the slots whose expert is not set in mask (nullable bitset)
void launch_moe_grouped(const DTensor& gate, const DTensor& up, const DTensor& down, const int* idx, const float* w,
                        const uint32_t* mask, const float* x, int T, int top_k, int n_expert, void* scratch, float* out,
                        cudaStream_t s);

// ---- batched prefill pieces (kernels_prefill.cu) ----
void launch_embed_rows(const DTensor& E, const int* tok, int T, int n_vocab, float* out, cudaStream_t s);
void launch_rope_rows(float* x, int T, int n_heads, int hd, const float* cs, int pos0, cudaStream_t s);
void launch_kv_append(const float* k, const float* v, int T, int n_kv, int hd, int max_ctx, int pos0, float* kc,
                      float* vc, cudaStream_t s);
void launch_conv_prefill(const float* bcx, const float* w, float* state, int T, int E, float* y, cudaStream_t s);
void launch_add_rows(float* x, const float* d, size_t n, cudaStream_t s);
void launch_swiglu_rows(const float* g, const float* u, size_t n, float* h, cudaStream_t s);
void launch_attn_prefill(const float* q, const float* kc, const float* vc, int T, int pos0, int n_head, int n_kv,
                         int hd, int max_ctx, float* out, cudaStream_t s);
// the same on the tensor cores (kernels_attn_tc.cu): hd 64 or 128, 128 % (n_head / n_kv) == 0
bool attn_prefill_tc_supported(int n_head, int n_kv, int hd);
void launch_attn_prefill_tc(const float* q, const float* kc, const float* vc, int T, int pos0, int n_head, int n_kv,
                            int hd, int max_ctx, float* out, cudaStream_t s);
// multi-sequence decode rows (kernels_prefill.cu): row t is sequence seq[t] (device) at position
// pos[t] (device); the KV cache / conv state of sequence s start seq_stride / state_stride floats
// after the given base pointer
void launch_rope_rows_at(float* x, int T, int n_heads, int hd, const float* cs, const int* pos, cudaStream_t s);
void launch_kv_append_at(const float* k, const float* v, int T, int n_kv, int hd, int max_ctx, const int* seq,
                         const int* pos, size_t seq_stride, float* kc, float* vc, cudaStream_t s);
void launch_conv_rows_at(const float* bcx, const float* w, float* state, size_t state_stride, const int* seq, int T,
                         int E, float* y, cudaStream_t s);
// out[t] = first-max argmax of logits row t, *suppress (nullable; < 0: none) left out;
// scratch: argmax_rows_scratch_bytes(T) bytes
size_t argmax_rows_scratch_bytes(int T);
void launch_argmax_rows(const float* logits, int T, int V, const int* suppress, void* scratch, int* out,
                        cudaStream_t s);
// attention of the rows split over positions (chunks of attn_rows_chunk()), partial states in
// part (attn_rows_part_floats(T, n_head, hd, max_ctx) floats), merged in split order into out;
// max_len = the longest row's length (positions attended, pos + 1)
int attn_rows_chunk();
size_t attn_rows_part_floats(int T, int n_head, int hd, int max_ctx);
void launch_attn_rows_split(const float* q, const float* kc, const float* vc, int T, const int* seq, const int* pos,
                            int max_len, size_t seq_stride, int n_head, int n_kv, int hd, int max_ctx, float* part,
                            float* out, cudaStream_t s, __half* out16 = nullptr);
// ---- fused row pieces (kernels_prefill.cu); y16 / out16: the fp16 operand planes of the next
// tensor-core product (what launch_f32_to_f16 writes for it), so that product runs x16_ready ----
// SwiGLU of n values into the operand planes only
void launch_swiglu_rows_f16(const float* g, const float* u, size_t n, __half* y16, cudaStream_t s);
// x += d (d nullable), then y = RMS norm of each row of n values (launch_rmsnorm's result) and,
// when y16 is non-null, y's operand planes
void launch_add_rmsnorm_rows(float* x, const float* d, int64_t n_rows, int n, const float* w, float eps, float* y,
                             __half* y16, cudaStream_t s);
// per-head norms and RoPE of the rows' query heads (in place) and key heads, and the keys and
// values stored into the cache (cache layout and row map as launch_kv_append_at; seq nullable:
// kc / vc are the sequence's own; pos nullable: positions pos0 + t)
void launch_qk_norm_rope_rows(float* q, const float* k, const float* v, int T, int n_head, int n_kv, int hd,
                              const float* qw, const float* kw, float eps, const float* cs, const int* seq,
                              const int* pos, int pos0, size_t seq_stride, int max_ctx, float* kc, float* vc,
                              cudaStream_t s);

// ---- bulk-copy streamed GEMV path (kernels_gemv2.cu) ----
// Each returns false when the shape is outside the streamed path (the caller then uses the
// kernels above).  Launched with programmatic dependent launch unless set_pdl(0).
bool launch2_rows(const DTensor& W, int64_t row0, int64_t n, const XStage& st, float* y, bool residual,
                  cudaStream_t s);
bool launch2_qkv(const DTensor& wq, const DTensor& wk, const DTensor& wv, const XStage& st, float* qkv,
                 cudaStream_t s);
bool launch2_swiglu(const DTensor& gate, const DTensor& up, const XStage& st, float* h, cudaStream_t s);
bool launch2_conv(const DTensor& in_proj, const float* conv_w, float* state, const XStage& st, float* y,
                  cudaStream_t s);
bool launch2_logits_argmax(const DTensor& W, const XStage& st, float* logits, unsigned long long* best,
                           const int* suppress_dev, cudaStream_t s);
bool launch2_moe_gateup(const DTensor& gate_exps, const DTensor& up_exps, const int* idx, const uint32_t* mask,
                        int top_k, const XStage& st, float* h, cudaStream_t s);
bool launch2_moe_down_combine(const DTensor& down_exps, const int* idx, const float* w, const uint32_t* mask,
                              int top_k, const float* h, float* hidden, cudaStream_t s);
// router for ONE token: logits_tmp [n_expert] and counter (zero, self-resetting) are scratch
bool launch2_router(const DTensor& router, const float* bias, const XStage& st, int n_expert, int top_k,
                    float* logits_tmp, unsigned int* counter, float* record, int* idx, float* w, cudaStream_t s);
void set_pdl(int on);
// 0 forces the register-streamed kernels of kernels_gemv.cu everywhere (A/B measurements)
void set_stream_path(int on);
int stream_path();
// ---- k-quant weights, raw superblocks in DTensor::qs (kernels_kquant.cu) ----
int kq_block_bytes(int type);  // 0 for a type that is not a k-quant
// rows [row0, row0 + n_rows) dequantised bit-exactly (the reference's f64 value rounded to f32)
void launch_kq_dequant(const DTensor& W, int64_t row0, int64_t n_rows, float* out, cudaStream_t s);
// y[m][n] = W[n] . x[m] for m < M (x [M][K], 16-byte aligned), y row stride ldy
void launch_kq_matmul(const DTensor& W, const float* x, int M, float* y, int ldy, cudaStream_t s);
// out[0..K) = the embedding row of the token *tok_dev (k-quant column reader)
void launch_kq_embed(const DTensor& W, const int* tok_dev, int n_vocab, float* out, cudaStream_t s);
// ctl = [*tok, ctl[1] + 1], trace[ctl[1]] = *tok (a decode step's last word)
void launch_finish_token(const int* tok, int* ctl, int* trace, cudaStream_t s);

// ---- tensor-parallel greedy id over vocab shards (kernels_prefill.cu) ----
// keys [T][32] of a vocab shard whose row 0 is global row idx0 (suppress: a shard-local id or -1)
void launch_argmax_rows_keys(const float* logits, int T, int V, const int* suppress, int idx0, void* keys,
                             cudaStream_t s);
// out[t] = first global maximum over the G shards' keys [G][T][32]
void launch_argmax_merge(const void* keys, int G, int T, int* out, cudaStream_t s);

// ---- expert-parallel exchange, token side (kernels_ep.cu) ----
// per destination rank r of W: pos[r][t] (token t's row in r's block, or -1), tok_of[r][q] (the
// token of row q, or -1), ids[r][q][s] (owner-local expert of slot s, or -1) and wts[r][q][s]
void launch_ep_plan(const int* idx, const float* w, const uint32_t* mask, int T, int top_k, int n_expert, int W, int C,
                    int* pos, int* tok_of, int* ids, float* wts, cudaStream_t s);
// send rows: out[r][q] = x[tok_of[r][q]] (zero where there is no token)
void launch_ep_gather(const float* x, const int* tok_of, int W, int C, int E, float* out, cudaStream_t s);
// hidden[t] += sum over r (rank order) of back[r][pos[r][t]]
void launch_ep_combine(const float* back, const int* pos, int W, int T, int C, int E, float* hidden, cudaStream_t s);

// ---- next-token sampling (kernels_sample.cu) ----
constexpr int kSampleMaxTopK = 1024;
constexpr int kThinkSuppress = 0, kThinkShorten = 1, kThinkFull = 2;
struct SampleArgs {
    double temperature, top_p;  // JS numbers
    int top_k;                  // 1..kSampleMaxTopK
    int think_mode;             // kThink*
    int think_id, end_think_id;
    unsigned long long seed;
};
// The uniform draw in [0, 1) for (seed, sequence, position): a splitmix64 finaliser over the
// three, top 53 bits.  Host code reproduces it bit for bit.
__host__ __device__ inline double sample_uniform(unsigned long long seed, int seq, int pos) {
    unsigned long long z = seed ^ (0x9E3779B97F4A7C15ull * (unsigned long long)(unsigned)(pos + 1)) ^
                           (0xD1B54A32D192ED03ull * (unsigned long long)(unsigned)(seq + 1));
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}
// sampleWithThinkControl over logits[n] into out[0].  r >= 0 is the uniform draw; r < 0 draws
// sample_uniform(seed, seq, pos), pos < 0 meaning ctl[1] - 1.  With ctl set the token also
// becomes ctl[0] and trace[ctl[1]] (the step's greedy id is replaced).  think_done (nullable) is
// the per-sequence "thinking done" flag of the 'shorten' mode; set when endThinkId is produced.
// scratch: n words.
void launch_sample(const float* logits, int n, const SampleArgs* args_dev, int* think_done, double r, int seq,
                   int pos, int* ctl, int* trace, int* out, uint32_t* scratch, cudaStream_t s);

// error word written by bounded waits that gave up (0 = none); read-and-clear.  The address is
// that of the current device's copy of the word (resolved once per device).
int* kernel_err_ptr();
// true the first time it is called for (key, current device): per-device one-time set-up such as
// cudaFuncSetAttribute, which applies to the current device only
bool first_use_on_device(const void* key);
int take_kernel_error(cudaStream_t s);

}  // namespace qq3
