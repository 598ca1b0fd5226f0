// api.cu -- the extern "C" boundary of libqq3cuda.so and the decode runtime behind it.
//
// Runtime design (one B200, one sequence per decode step):
//   * weights are uploaded raw (GGUF Q8_0 blocks) and split on the device into qs/d planes;
//   * a decode step is a fixed sequence of ~5 launches per layer (see enqueue_step), every
//     kernel reading the token id and position from device memory, so the whole step is
//     captured once per (sequence, with/without logits) as a CUDA graph and replayed;
//   * greedy decode can run entirely on the device: the step's last kernel writes the
//     argmax back as the next step's token (qq_decode_loop).
#include <algorithm>
#include <array>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

#include <numeric>

#include "api_internal.h"
#include "comm.h"
#include "decode_prog.h"

namespace qq3 {
static thread_local std::string g_err;
void set_error(const std::string& msg) { g_err = msg; }
const char* last_error_cstr() { return g_err.c_str(); }
}  // namespace qq3

using namespace qq3api;

namespace {

void* dmalloc(size_t bytes) {
    void* p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Error{QQ_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + " bytes) failed: " + cudaGetErrorString(e)};
    }
    return p;
}

template <class T>
T* dalloc(size_t n) {
    return static_cast<T*>(dmalloc(n * sizeof(T)));
}

bool getenv_flag(const char* name) {
    const char* v = getenv(name);
    return v && atoi(v) != 0;
}

// a switch that is on unless set to 0
bool getenv_flag_zero(const char* name) {
    const char* v = getenv(name);
    return v && atoi(v) == 0;
}

void* ctx_scratch(qq_ctx* c, size_t bytes) {
    if (bytes > c->scratch_bytes) {
        if (c->scratch) {
            QQ_CUDA_TRY(cudaStreamSynchronize(c->stream));
            cudaFree(c->scratch);
            c->scratch = nullptr;
            c->scratch_bytes = 0;
        }
        c->scratch = dmalloc(bytes);
        c->scratch_bytes = bytes;
    }
    return c->scratch;
}

}  // namespace

// =====================================================================================
// Model

struct Layer {
    bool attn = false, moe = false;
    const DTensor* t[QQ_SLOT_COUNT] = {nullptr};
    int attn_slot = -1, moe_slot = -1;
    // the FFN down tensor (experts) and the short-conv out_proj transposed for the fused phases
    // of the persistent decode step (owned; built on first use)
    int8_t* dt_qs = nullptr;
    __half* dt_d = nullptr;
    int8_t* ot_qs = nullptr;
    __half* ot_d = nullptr;
};

struct qq_model {
    qq_ctx* ctx = nullptr;
    qq_model_desc d{};
    std::vector<Layer> layers;
    const DTensor* tok_embd = nullptr;
    const DTensor* out_norm = nullptr;
    const DTensor* output = nullptr;
    int n_attn = 0, n_moe = 0, n_ff_max = 0, n_split = 1, rec_len = 0;
    // activations
    float *hidden = nullptr, *qkv = nullptr, *attn_out = nullptr, *y = nullptr, *h = nullptr, *logits = nullptr;
    // per-sequence state
    float *k_cache = nullptr, *v_cache = nullptr, *conv_state = nullptr;
    int* trace = nullptr;  // [n_seq][max_ctx + 1] greedy ids produced by device-driven steps
    // tables / scratch
    float* rope_cs = nullptr;
    float* attn_part = nullptr;
    unsigned int* attn_counter = nullptr;
    float* rec = nullptr;
    float* rlogits = nullptr;          // router logits scratch [n_expert]
    unsigned int* rcounter = nullptr;  // router last-CTA ticket (self-resetting)
    int* ridx = nullptr;
    float* rw = nullptr;
    uint32_t* mask = nullptr;
    int* ctl = nullptr;       // [token, pos, error word copy, pad]: the persistent step's token
    int* suppress = nullptr;  // [1]
    unsigned long long* best = nullptr;
    float* dump = nullptr;    // [n_layers][n_embd] for qq_forward_dump
    int* h_ctl = nullptr;     // pinned staging [2 * h_ctl_cap]
    size_t h_ctl_cap = 0;
    int* h_small = nullptr;   // pinned [8]: suppress id, argmax, token, pos, kernel error word, think flag
    int* h_io = nullptr;      // pinned [8]: one host step's token, pos in; argmax, pos, error word out
    int suppress_set = INT32_MIN;  // the suppress id last copied to the device
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
    // captured multi-sequence steps, per (rows, want_logits): valid for the attention split count
    // nz and the buffers it was captured with
    struct BatchGraph {
        cudaGraphExec_t exec = nullptr;
        int nz = 0;
        bool seen = false;  // the key ran once eagerly (kernel attributes are set)
        const void* ptrs[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    };
    std::map<std::pair<int, int>, BatchGraph> bgraphs;
    cudaStream_t cap = nullptr;
    // persistent decode kernel programs, per (sequence, with logits)
    struct Prog {
        qq3::PhaseDesc* d_prog = nullptr;
        int n = 0;
    };
    std::map<std::pair<int, int>, Prog> progs;
    qq3::DecodeCtl* dctl = nullptr;  // model-wide control block of the persistent kernel
    unsigned long long* trace_buf = nullptr;  // per-CTA phase stamps (qq_decode_trace)
    // batched prefill / multi-sequence buffers (grow-only, pf_bytes allocated)
    size_t pf_bytes = 0;
    void* pf_arena = nullptr;
    // multi-sequence decode rows (qq_forward_batch) for up to bt_cap rows (grow-only):
    // device [token | seq | pos | argmax] x bt_cap ints, logits [bt_cap][n_vocab], pinned staging
    int bt_cap = 0;
    int* bt_i = nullptr;
    float* bt_logits = nullptr;
    float* bt_attn = nullptr;  // split-attention partial states of the rows
    void* bt_keys = nullptr;   // row-argmax partial keys
    int* h_bt = nullptr;
    qq3::tword* tarena = nullptr;    // tagged activations: one buffer per phase output
    size_t tarena_len = 0;
    float* aarena = nullptr;         // accumulated vectors + counters, two halves of aarena_half words
    size_t aarena_half = 0;
    // device sampling (allocated on first use): arguments, per-sequence 'thinking done' flags,
    // probability keys [n_vocab], the sampled id; pinned staging for the arguments
    qq3::SampleArgs* sargs = nullptr;
    int* think_done = nullptr;
    uint32_t* spk = nullptr;
    int* sout = nullptr;
    qq3::SampleArgs* h_sargs = nullptr;
    // expert parallelism: this rank's share of the experts, and the exchange buffers (grow-only,
    // for ep_cap rows per destination rank)
    int ep_world = 1, ep_rank = 0, n_expert_local = 0;
    int ep_cap = 0;
    void* ep_arena = nullptr;
    float* ep_xn = nullptr;  // the normalised FFN input of a decode step [n_embd]
    // optional CUDA-event split of every exchange (qq_ep_profile): dispatch, experts, return, combine
    bool ep_prof = false;
    std::vector<std::array<cudaEvent_t, 5>> ep_evs;
    // tensor parallelism (dense Qwen3): this rank's vocab rows [v0, v0 + v_local) of the lm_head;
    // d.n_head / d.n_head_kv hold this rank's head counts; greedy keys of all ranks [G][cap][32],
    // gathered logits [G][cap][v_local], the shard-local suppressed id
    int tp_world = 1, tp_rank = 0, v_local = 0, v0 = 0;
    void* tp_keys = nullptr;
    float* tp_logits = nullptr;
    int* tp_suppress = nullptr;
    int tp_cap = 0;
    // a model with k-quant weights: decode steps op by op (enqueue_step_generic); its buffers:
    // gate, up [n_ff_max] and a hidden-sized partial; greedy scratch and the step's id
    bool generic = false;
    float* gen_buf = nullptr;
    void* gen_keys = nullptr;
    int* gen_tok = nullptr;
    int mega = -1;  // -1 unknown, 0 no (a phase does not fit or disabled), 1 yes
    int64_t step_kernels = 0;  // kernel nodes in the decode-step graph (with logits)

    size_t kv_stride_seq() const { return (size_t)n_attn * d.n_head_kv * d.max_ctx * d.head_dim; }
    size_t kv_stride_layer() const { return (size_t)d.n_head_kv * d.max_ctx * d.head_dim; }
    float* conv(int seq, int l) const { return conv_state + ((size_t)seq * d.n_layers + l) * 2 * d.n_embd; }
};

namespace {

void free_model(qq_model* m) {
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    for (auto& kv : m->bgraphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    m->bgraphs.clear();
    m->graphs.clear();
    for (auto& kv : m->progs)
        if (kv.second.d_prog) cudaFree(kv.second.d_prog);
    m->progs.clear();
    if (m->dctl) cudaFree(m->dctl);
    if (m->trace_buf) cudaFree(m->trace_buf);
    if (m->pf_arena) cudaFree(m->pf_arena);
    if (m->bt_i) cudaFree(m->bt_i);
    if (m->bt_logits) cudaFree(m->bt_logits);
    if (m->bt_attn) cudaFree(m->bt_attn);
    if (m->bt_keys) cudaFree(m->bt_keys);
    if (m->h_bt) cudaFreeHost(m->h_bt);
    if (m->tarena) cudaFree(m->tarena);
    if (m->ep_arena) cudaFree(m->ep_arena);
    if (m->gen_buf) cudaFree(m->gen_buf);
    if (m->gen_keys) cudaFree(m->gen_keys);
    if (m->gen_tok) cudaFree(m->gen_tok);
    if (m->tp_keys) cudaFree(m->tp_keys);
    if (m->tp_logits) cudaFree(m->tp_logits);
    if (m->tp_suppress) cudaFree(m->tp_suppress);
    for (auto& ev : m->ep_evs)
        for (auto e : ev) cudaEventDestroy(e);
    m->ep_evs.clear();
    if (m->ep_xn) cudaFree(m->ep_xn);
    if (m->aarena) cudaFree(m->aarena);
    for (Layer& L : m->layers) {
        for (void* q : {(void*)L.dt_qs, (void*)L.dt_d, (void*)L.ot_qs, (void*)L.ot_d})
            if (q) cudaFree(q);
        L.dt_qs = nullptr;
        L.dt_d = nullptr;
        L.ot_qs = nullptr;
        L.ot_d = nullptr;
    }
    void* bufs[] = {m->hidden, m->qkv, m->attn_out, m->y, m->h, m->logits, m->k_cache, m->v_cache, m->conv_state,
                    m->trace, m->rope_cs, m->attn_part, m->attn_counter, m->rec, m->rlogits, m->rcounter, m->ridx, m->rw,
                    m->mask, m->ctl,
                    m->suppress, m->best, m->dump, m->sargs, m->think_done, m->spk, m->sout};
    for (void* p : bufs)
        if (p) cudaFree(p);
    if (m->h_ctl) cudaFreeHost(m->h_ctl);
    if (m->h_small) cudaFreeHost(m->h_small);
    if (m->h_io) cudaFreeHost(m->h_io);
    if (m->h_sargs) cudaFreeHost(m->h_sargs);
    if (m->cap) cudaStreamDestroy(m->cap);
}

// ---- expert-parallel MoE -------------------------------------------------------------------
// The MoE of layer L for T rows xn (normalised FFN inputs) routed to idx / w (global expert ids,
// T x top_k), with this rank holding n_expert_local experts: plan + gather the rows per owner
// rank (kernels_ep.cu), NCCL exchange, the grouped expert GEMMs over the rows received (each
// owner's weighted partial sum of the slots it serves), NCCL exchange back, and
// hidden[t] += the partial sums in rank order.  Collective: every rank calls it with the same T.
struct EpBufs {
    int *pos, *tok_of, *sids, *rids;
    float *swts, *rwts, *sx, *rx, *y, *back;
    void* moe;
};

EpBufs ep_bufs(qq_model* m, int C) {
    const qq_model_desc& d = m->d;
    const size_t W = m->ep_world, E = d.n_embd, k = d.n_expert_used;
    size_t F = 0;
    for (const Layer& L : m->layers)
        if (L.moe) F = std::max<size_t>(F, L.t[QQ_GATE_EXPS]->ne[1]);
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    auto sizes = [&](size_t c) {
        return std::vector<size_t>{al(W * c * 4),     al(W * c * 4),      al(W * c * k * 4), al(W * c * k * 4),
                                   al(W * c * k * 4), al(W * c * k * 4), al(W * c * E * 4), al(W * c * E * 4),
                                   al(W * c * E * 4), al(W * c * E * 4),
                                   al(qq3::moe_grouped_scratch_bytes((int)(W * c), (int)k, m->n_expert_local, E, F))};
    };
    if (C > m->ep_cap) {
        if (m->ep_arena) {
            QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
            cudaFree(m->ep_arena);
            m->ep_arena = nullptr;
            m->ep_cap = 0;
        }
        size_t total = 0;
        for (size_t v : sizes(C)) total += v;
        m->ep_arena = dmalloc(total);
        m->ep_cap = C;
    }
    const std::vector<size_t> sz = sizes(m->ep_cap);
    char* b = static_cast<char*>(m->ep_arena);
    size_t i = 0;
    auto take = [&]() {
        char* r = b;
        b += sz[i++];
        return r;
    };
    EpBufs e;
    e.pos = reinterpret_cast<int*>(take());
    e.tok_of = reinterpret_cast<int*>(take());
    e.sids = reinterpret_cast<int*>(take());
    e.rids = reinterpret_cast<int*>(take());
    e.swts = reinterpret_cast<float*>(take());
    e.rwts = reinterpret_cast<float*>(take());
    e.sx = reinterpret_cast<float*>(take());
    e.rx = reinterpret_cast<float*>(take());
    e.y = reinterpret_cast<float*>(take());
    e.back = reinterpret_cast<float*>(take());
    e.moe = take();
    return e;
}

void ep_moe(qq_model* m, const Layer& L, const float* xn, int T, const int* idx, const float* w, float* hidden,
            cudaStream_t s) {
    const qq_model_desc& d = m->d;
    const int W = m->ep_world, E = d.n_embd, k = d.n_expert_used, C = T;
    qq_ctx* c = m->ctx;
    EpBufs b = ep_bufs(m, C);
    std::array<cudaEvent_t, 5> ev{};
    if (m->ep_prof) {
        for (auto& e : ev) QQ_CUDA_TRY(cudaEventCreate(&e));
        QQ_CUDA_TRY(cudaEventRecord(ev[0], s));
    }
    qq3::launch_ep_plan(idx, w, m->mask, T, k, d.n_expert, W, C, b.pos, b.tok_of, b.sids, b.swts, s);
    qq3::launch_ep_gather(xn, b.tok_of, W, C, E, b.sx, s);
    const size_t rowb = (size_t)C * E * 4, slotb = (size_t)C * k * 4;
    qq3::comm_group_start();
    for (int r = 0; r < W; r++) {
        qq3::comm_send(c, b.sx + (size_t)r * C * E, rowb, r, s);
        qq3::comm_send(c, b.sids + (size_t)r * C * k, slotb, r, s);
        qq3::comm_send(c, b.swts + (size_t)r * C * k, slotb, r, s);
        qq3::comm_recv(c, b.rx + (size_t)r * C * E, rowb, r, s);
        qq3::comm_recv(c, b.rids + (size_t)r * C * k, slotb, r, s);
        qq3::comm_recv(c, b.rwts + (size_t)r * C * k, slotb, r, s);
    }
    qq3::comm_group_end(c);
    if (m->ep_prof) QQ_CUDA_TRY(cudaEventRecord(ev[1], s));
    // the owner side: weighted partial sums of the slots this rank serves, row by received row
    qq3::launch_moe_grouped(*L.t[QQ_GATE_EXPS], *L.t[QQ_UP_EXPS], *L.t[QQ_DOWN_EXPS], b.rids, b.rwts, nullptr, b.rx,
                            W * C, k, m->n_expert_local, b.moe, b.y, s);
    if (m->ep_prof) QQ_CUDA_TRY(cudaEventRecord(ev[2], s));
    qq3::comm_group_start();
    for (int r = 0; r < W; r++) {
        qq3::comm_send(c, b.y + (size_t)r * C * E, rowb, r, s);
        qq3::comm_recv(c, b.back + (size_t)r * C * E, rowb, r, s);
    }
    qq3::comm_group_end(c);
    if (m->ep_prof) QQ_CUDA_TRY(cudaEventRecord(ev[3], s));
    qq3::launch_ep_combine(b.back, b.pos, W, T, C, E, hidden, s);
    if (m->ep_prof) {
        QQ_CUDA_TRY(cudaEventRecord(ev[4], s));
        m->ep_evs.push_back(ev);
    }
}

// y = W . x for one row, whatever W's type (Q8_0: the streamed GEMV; k-quant: raw superblocks)
void gemv_any(const DTensor& W, const float* x, float* y, cudaStream_t s) {
    if (qq3::kq_block_bytes(W.type)) {
        qq3::launch_kq_matmul(W, x, 1, y, (int)W.rows, s);
        return;
    }
    qq3::XStage st;
    st.x[0] = x;
    st.K = (int)W.K;
    qq3::launch_gemv_rows(W, 0, W.rows, st, y, false, s);
}

// Qwen3Engine.forward (qwen3-engine.js:115-245) op by op, for models with k-quant weights (real
// GGUF mixes such as Q4_K_M): RMSNorm, each projection as its own matmul of whatever type the
// tensor has, the decode attention (QK-norm, RoPE, KV append fused), SwiGLU, residual adds;
// then the output norm, lm_head and the first-max greedy id into the control words.
void enqueue_step_generic(qq_model* m, int seq, bool want_logits, cudaStream_t s, bool dump) {
    const qq_model_desc& d = m->d;
    const int E = d.n_embd, hd = d.head_dim;
    const int nq = d.n_head * hd, nkv = d.n_head_kv * hd;
    float* g = m->gen_buf;
    float* u = g + m->n_ff_max;
    float* part = u + m->n_ff_max;
    if (qq3::kq_block_bytes(m->tok_embd->type)) qq3::launch_kq_embed(*m->tok_embd, m->ctl, d.n_vocab, m->hidden, s);
    else qq3::launch_embed(*m->tok_embd, m->ctl, m->hidden, nullptr, s);
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        qq3::launch_rmsnorm(m->hidden, 1, E, L.t[QQ_ATTN_NORM]->f32, d.rms_eps, m->y, s);
        gemv_any(*L.t[QQ_WQ], m->y, m->qkv, s);
        gemv_any(*L.t[QQ_WK], m->y, m->qkv + nq, s);
        gemv_any(*L.t[QQ_WV], m->y, m->qkv + nq + nkv, s);
        qq3::AttnArgs a;
        a.qkv = m->qkv;
        a.q_norm = L.t[QQ_Q_NORM]->f32;
        a.k_norm = L.t[QQ_K_NORM]->f32;
        a.rope_cs = m->rope_cs;
        a.k_cache = m->k_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
        a.v_cache = m->v_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
        a.out = m->attn_out;
        a.part = m->attn_part;
        a.counter = m->attn_counter;
        a.pos = m->ctl + 1;
        a.n_head = d.n_head;
        a.n_kv = d.n_head_kv;
        a.hd = hd;
        a.max_ctx = d.max_ctx;
        a.n_split = m->n_split;
        a.eps = d.rms_eps;
        qq3::launch_attention_decode(a, s);
        gemv_any(*L.t[QQ_WO], m->attn_out, part, s);
        qq3::launch_add_rows(m->hidden, part, E, s);
        qq3::launch_rmsnorm(m->hidden, 1, E, L.t[QQ_FFN_NORM]->f32, d.rms_eps, m->y, s);
        const size_t F = L.t[QQ_FFN_GATE]->ne[1];
        gemv_any(*L.t[QQ_FFN_GATE], m->y, g, s);
        gemv_any(*L.t[QQ_FFN_UP], m->y, u, s);
        qq3::launch_swiglu_rows(g, u, F, m->h, s);
        gemv_any(*L.t[QQ_FFN_DOWN], m->h, part, s);
        qq3::launch_add_rows(m->hidden, part, E, s);
        if (dump)
            QQ_CUDA_TRY(cudaMemcpyAsync(m->dump + (size_t)l * E, m->hidden, sizeof(float) * E,
                                        cudaMemcpyDeviceToDevice, s));
    }
    if (!want_logits) return;
    qq3::launch_rmsnorm(m->hidden, 1, E, m->out_norm->f32, d.rms_eps, m->y, s);
    gemv_any(m->output ? *m->output : *m->tok_embd, m->y, m->logits, s);
    qq3::launch_argmax_rows(m->logits, 1, d.n_vocab, m->suppress, m->gen_keys, m->gen_tok, s);
    qq3::launch_finish_token(m->gen_tok, m->ctl, m->trace + (size_t)seq * (d.max_ctx + 1), s);
}

// One decode step for sequence `seq` (token/position in m->ctl), as the fixed kernel
// sequence of Qwen3Engine.forward / Lfm2Engine.forward.
void enqueue_step(qq_model* m, int seq, bool want_logits, cudaStream_t s, bool dump) {
    if (m->generic) {
        enqueue_step_generic(m, seq, want_logits, s, dump);
        return;
    }
    const qq_model_desc& d = m->d;
    const int E = d.n_embd, hd = d.head_dim;
    const int nq = d.n_head * hd;
    qq3::launch_embed(*m->tok_embd, m->ctl, m->hidden, want_logits ? m->best : nullptr, s);
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        qq3::XStage st;
        st.x[0] = m->hidden;
        st.K = E;
        st.norm_w = L.t[QQ_ATTN_NORM]->f32;
        st.eps = d.rms_eps;
        if (L.attn) {
            qq3::launch_gemv_qkv(*L.t[QQ_WQ], *L.t[QQ_WK], *L.t[QQ_WV], st, m->qkv, s);
            qq3::AttnArgs a;
            a.qkv = m->qkv;
            a.q_norm = L.t[QQ_Q_NORM]->f32;
            a.k_norm = L.t[QQ_K_NORM]->f32;
            a.rope_cs = m->rope_cs;
            a.k_cache = m->k_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            a.v_cache = m->v_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            a.out = m->attn_out;
            a.part = m->attn_part;
            a.counter = m->attn_counter;
            a.pos = m->ctl + 1;
            a.n_head = d.n_head;
            a.n_kv = d.n_head_kv;
            a.hd = hd;
            a.max_ctx = d.max_ctx;
            a.n_split = m->n_split;
            a.eps = d.rms_eps;
            qq3::launch_attention_decode(a, s);
            qq3::XStage so;
            so.x[0] = m->attn_out;
            so.K = nq;
            qq3::launch_gemv_rows(*L.t[QQ_WO], 0, E, so, m->hidden, true, s);
        } else {
            qq3::launch_gemv_conv(*L.t[QQ_IN_PROJ], L.t[QQ_CONV]->f32, m->conv(seq, l), st, m->y, s);
            qq3::XStage so;
            so.x[0] = m->y;
            so.K = E;
            qq3::launch_gemv_rows(*L.t[QQ_OUT_PROJ], 0, E, so, m->hidden, true, s);
        }
        qq3::XStage sf;
        sf.x[0] = m->hidden;
        sf.K = E;
        sf.norm_w = L.t[QQ_FFN_NORM]->f32;
        sf.eps = d.rms_eps;
        if (L.moe && m->ep_world > 1) {
            const int k = d.n_expert_used;
            float* rec = m->rec + (size_t)L.moe_slot * m->rec_len;
            int* idx = m->ridx + (size_t)L.moe_slot * k;
            float* w = m->rw + (size_t)L.moe_slot * k;
            const float* bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            qq3::launch_rmsnorm(m->hidden, 1, E, sf.norm_w, sf.eps, m->ep_xn, s);
            qq3::launch_router(*L.t[QQ_ROUTER], bias, m->ep_xn, 1, nullptr, 0.f, d.n_expert, k, d.arch == QQ_ARCH_QWEN3,
                               rec, idx, w, s);
            ep_moe(m, L, m->ep_xn, 1, idx, w, m->hidden, s);
        } else if (L.moe) {
            const int k = d.n_expert_used;
            float* rec = m->rec + (size_t)L.moe_slot * m->rec_len;
            int* idx = m->ridx + (size_t)L.moe_slot * k;
            float* w = m->rw + (size_t)L.moe_slot * k;
            const float* bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            if (d.arch == QQ_ARCH_QWEN3)
                qq3::launch_router(*L.t[QQ_ROUTER], nullptr, m->hidden, 1, sf.norm_w, sf.eps, d.n_expert, k, true, rec,
                                   idx, w, s);
            else if (!(qq3::stream_path() && qq3::launch2_router(*L.t[QQ_ROUTER], bias, sf, d.n_expert, k, m->rlogits,
                                                                 m->rcounter, rec, idx, w, s)))
                qq3::launch_lfm2_router(*L.t[QQ_ROUTER], bias, m->hidden, 1, sf.norm_w, sf.eps, d.n_expert, k, rec,
                                        idx, w, s);
            qq3::launch_moe_gateup(*L.t[QQ_GATE_EXPS], *L.t[QQ_UP_EXPS], idx, m->mask, k, sf, m->h, s);
            qq3::launch_moe_down_combine(*L.t[QQ_DOWN_EXPS], idx, w, m->mask, k, m->h, m->hidden, s);
        } else {
            qq3::launch_gemv_swiglu(*L.t[QQ_FFN_GATE], *L.t[QQ_FFN_UP], sf, m->h, s);
            qq3::XStage sd;
            sd.x[0] = m->h;
            sd.K = (int)L.t[QQ_FFN_GATE]->ne[1];
            qq3::launch_gemv_rows(*L.t[QQ_FFN_DOWN], 0, E, sd, m->hidden, true, s);
        }
        if (dump)
            QQ_CUDA_TRY(cudaMemcpyAsync(m->dump + (size_t)l * E, m->hidden, sizeof(float) * E,
                                        cudaMemcpyDeviceToDevice, s));
    }
    if (want_logits) {
        qq3::XStage so;
        so.x[0] = m->hidden;
        so.K = E;
        so.norm_w = m->out_norm->f32;
        so.eps = d.rms_eps;
        const DTensor* out = m->output ? m->output : m->tok_embd;
        qq3::launch_gemv_logits_argmax(*out, so, m->logits, m->best, m->suppress, s);
        qq3::launch_argmax_finish(m->best, m->ctl, m->trace + (size_t)seq * (d.max_ctx + 1), s);
    }
}

// Tagged-activation words the persistent program of this model needs: a bound on the sum of
// all phase outputs (at most three vectors per layer, plus the embedding).
size_t tarena_bound(const qq_model* m) {
    const qq_model_desc& d = m->d;
    size_t v = (size_t)d.n_embd;
    v = std::max(v, (size_t)(d.n_head + 2 * d.n_head_kv) * d.head_dim);
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        if (L.moe) v = std::max(v, (size_t)d.n_expert_used * L.t[QQ_GATE_EXPS]->ne[1]);
        else if (L.t[QQ_FFN_GATE]) v = std::max(v, (size_t)L.t[QQ_FFN_GATE]->ne[1]);
    }
    v = (v + 31) & ~(size_t)31;
    return (size_t)(3 * d.n_layers + 2) * v;
}

// Whether the FFN of layer L runs as one fused phase of the persistent step (router, gate/up,
// SwiGLU, down and combine; outputs accumulated): an MoE layer, or a dense FFN as a single
// expert.  QQ3_MOE_FUSED=0 selects the two-phase forms (gate/up, then down).
bool ffn_fused(const qq_model* m, const Layer& L) {
    const char* env = getenv("QQ3_MOE_FUSED");
    if (env && atoi(env) == 0) return false;
    const qq_model_desc& d = m->d;
    const DTensor* gate = L.t[L.moe ? QQ_GATE_EXPS : QQ_FFN_GATE];
    const DTensor* down = L.t[L.moe ? QQ_DOWN_EXPS : QQ_FFN_DOWN];
    if (!gate || !down) return false;
    const int F = (int)gate->ne[1];
    return (int)down->K == F && (L.moe ? qq3::decode_moe_fits(d.n_embd, F, d.n_embd, d.n_expert, d.n_expert_used)
                                       : qq3::decode_moe_fits(d.n_embd, F, d.n_embd, 1, 1));
}

// Whether the short-conv block of layer L (in_proj, conv, out_proj) runs as one fused phase;
// QQ3_CONV_FUSED=0 keeps two phases (in_proj + conv, then out_proj).
bool conv_fused(const qq_model* m, const Layer& L) {
    const char* env = getenv("QQ3_CONV_FUSED");
    if ((env && atoi(env) == 0) || L.attn || !L.t[QQ_IN_PROJ] || !L.t[QQ_OUT_PROJ] || !L.t[QQ_CONV]) return false;
    const int E = m->d.n_embd;
    return L.t[QQ_IN_PROJ]->ne[1] == 3 * E && L.t[QQ_OUT_PROJ]->K == E && L.t[QQ_OUT_PROJ]->rows == E &&
           qq3::decode_moe_fits(E, E, E, 1, 1, 3);
}

// The decode step as a phase program for the persistent kernel (kernels_decode.cu); the same
// sequence of operations as enqueue_step.  Each phase writes its own tagged output buffer and
// names the phase that wrote each vector it reads.
std::vector<qq3::PhaseDesc> build_program(qq_model* m, int seq, bool want_logits) {
    using namespace qq3;
    const qq_model_desc& d = m->d;
    const int E = d.n_embd, hd = d.head_dim, nq = d.n_head * hd, nkv = d.n_head_kv * hd;
    bool fuse = false;  // any fused FFN phase (they need the accumulator arena)
    for (const Layer& L : m->layers) fuse = fuse || ffn_fused(m, L) || conv_fused(m, L);
    if (!m->tarena) {
        m->tarena_len = tarena_bound(m);
        m->tarena = dalloc<tword>(m->tarena_len);
        // tag 0 never matches a step's tags
        QQ_CUDA_TRY(cudaMemsetAsync(m->tarena, 0, sizeof(tword) * m->tarena_len, m->ctx->stream));
    }
    if (!m->dctl) {
        m->dctl = dalloc<DecodeCtl>(1);
        QQ_CUDA_TRY(cudaMemsetAsync(m->dctl, 0, sizeof(DecodeCtl), m->ctx->stream));
    }
    // fused MoE: one accumulated vector (E floats) + counter (padded to 32 words) per MoE layer
    const size_t aslot = ((size_t)qq3::kAccCopies * E + 32 + 31) & ~(size_t)31;
    if (fuse && !m->aarena) {
        m->aarena_half = aslot * (size_t)d.n_layers * 2;  // up to two fused phases per layer
        m->aarena = dalloc<float>(2 * m->aarena_half);
        cudaStream_t s = m->ctx->stream;
        QQ_CUDA_TRY(cudaMemsetAsync(m->aarena, 0, sizeof(float) * 2 * m->aarena_half, s));
        float* a = m->aarena;
        long long h = (long long)m->aarena_half;
        QQ_CUDA_TRY(cudaMemcpyAsync(&m->dctl->arena, &a, sizeof(a), cudaMemcpyHostToDevice, s));
        QQ_CUDA_TRY(cudaMemcpyAsync(&m->dctl->arena_half, &h, sizeof(h), cudaMemcpyHostToDevice, s));
        for (Layer& L : m->layers) {
            if (ffn_fused(m, L) && !L.dt_qs) {
                const DTensor& W = *L.t[L.moe ? QQ_DOWN_EXPS : QQ_FFN_DOWN];
                L.dt_qs = dalloc<int8_t>((size_t)W.rows * W.K);
                L.dt_d = dalloc<__half>((size_t)W.rows * (W.K / 32));
                qq3::launch_transpose_experts(W, L.moe ? d.n_expert : 1, L.dt_qs, L.dt_d, s);
            }
            if (conv_fused(m, L) && !L.ot_qs) {
                const DTensor& W = *L.t[QQ_OUT_PROJ];
                L.ot_qs = dalloc<int8_t>((size_t)W.rows * W.K);
                L.ot_d = dalloc<__half>((size_t)W.rows * (W.K / 32));
                qq3::launch_transpose_experts(W, 1, L.ot_qs, L.ot_d, s);
            }
        }
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // the pointers above are host locals
    }
    size_t cursor = 0;
    auto take = [&](size_t n) {
        tword* t = m->tarena + cursor;
        cursor += (n + 31) & ~(size_t)31;
        QQ_CHECK(cursor <= m->tarena_len, QQ_ERR_INVALID, "persistent program: activation arena too small");
        return t;
    };
    std::vector<PhaseDesc> prog;
    auto blank = [] {
        PhaseDesc p;
        std::memset(&p, 0, sizeof(p));
        p.S = 1;
        return p;
    };
    // a vector between phases: tagged words and the phase that wrote them, or an accumulated
    // vector with its counter and the count that completes it
    struct Ref {
        const tword* t = nullptr;
        int ph = -1;
        const float* a = nullptr;
        const unsigned* c = nullptr;
        int n = 0;
    };
    Ref hid;  // the residual stream
    {
        PhaseDesc p = blank();
        p.type = PH_EMBED;
        p.emb_qs = m->tok_embd->qs;
        p.emb_d = m->tok_embd->d;
        p.emb_K = (int)m->tok_embd->K;
        p.n_vocab = d.n_vocab;
        p.ctl = m->ctl;
        p.y = take(E);
        hid.t = p.y;
        hid.ph = 0;
        prog.push_back(p);
    }
    auto tagged = [](const tword* t, int ph) {
        Ref r;
        r.t = t;
        r.ph = ph;
        return r;
    };
    auto gemv = [&](int map, int epi, int S, int K, int n_items, const Ref& in, const float* norm_w) {
        PhaseDesc p = blank();
        p.type = PH_GEMV;
        p.map = map;
        p.epi = epi;
        p.S = S;
        p.K = K;
        p.n_items = n_items;
        p.x = in.t;
        p.x_ph = in.ph;
        p.xa = in.a;
        p.xa_cnt = in.c;
        p.xa_n = in.n;
        p.norm_w = norm_w;
        p.eps = d.rms_eps;
        p.G = qq3::decode_stage_items(S, K, n_items, n_items);
        return p;
    };
    auto resid = [&](PhaseDesc& p) {  // y = hid + acc: a new version of the residual stream
        p.res = hid.t;
        p.res_ph = hid.ph;
        p.ra = hid.a;
        p.ra_cnt = hid.c;
        p.ra_n = hid.n;
        p.y = take(E);
    };
    auto push_hid = [&](PhaseDesc& p) {
        prog.push_back(p);
        hid = tagged(p.y, (int)prog.size() - 1);
    };
    int n_acc = 0;  // accumulated vectors handed out
    auto set_src = [](PhaseDesc& p, int i, const DTensor* t) {
        p.qs[i] = t->qs;
        p.d[i] = t->d;
    };
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        const float* an = L.t[QQ_ATTN_NORM]->f32;
        const float* fn = L.t[QQ_FFN_NORM]->f32;
        auto take_acc = [&](PhaseDesc& g) {
            QQ_CHECK((size_t)(n_acc + 1) * aslot <= m->aarena_half, QQ_ERR_INVALID,
                     "persistent program: accumulator arena too small");
            g.acc = m->aarena + (size_t)n_acc * aslot;
            g.acc_cnt = reinterpret_cast<unsigned*>(g.acc + (size_t)qq3::kAccCopies * E);
            ++n_acc;
        };
        auto set_hid_acc = [&](const PhaseDesc& g) {
            hid = Ref();
            hid.a = g.acc;
            hid.c = g.acc_cnt;
            hid.n = qq3::num_sms();  // every CTA of the grid counts once
        };
        if (L.attn) {
            PhaseDesc q = gemv(MK_CONCAT3, EK_STORE, 1, E, nq + 2 * nkv, hid, an);
            set_src(q, 0, L.t[QQ_WQ]);
            set_src(q, 1, L.t[QQ_WK]);
            set_src(q, 2, L.t[QQ_WV]);
            q.n0 = nq;
            q.n1 = nkv;
            q.G = qq3::decode_stage_items(1, E, std::gcd(nq, nkv), nq + 2 * nkv);  // groups must not straddle q|k|v
            q.y = take(nq + 2 * nkv);
            prog.push_back(q);
            PhaseDesc a = blank();
            a.type = PH_ATTN;
            a.a_qkv = q.y;
            a.a_qkv_ph = (int)prog.size() - 1;
            a.a_out = take(nq);
            a.attn.q_norm = L.t[QQ_Q_NORM]->f32;
            a.attn.k_norm = L.t[QQ_K_NORM]->f32;
            a.attn.rope_cs = m->rope_cs;
            a.attn.k_cache = m->k_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            a.attn.v_cache = m->v_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            a.attn.part = m->attn_part;
            a.attn.counter = m->attn_counter;
            a.attn.pos = m->ctl + 1;
            a.attn.n_head = d.n_head;
            a.attn.n_kv = d.n_head_kv;
            a.attn.hd = hd;
            a.attn.max_ctx = d.max_ctx;
            a.attn.n_split = m->n_split;
            a.attn.eps = d.rms_eps;
            prog.push_back(a);
            PhaseDesc o = gemv(MK_ROWS, EK_RESID, 1, nq, E, tagged(a.a_out, (int)prog.size() - 1), nullptr);
            set_src(o, 0, L.t[QQ_WO]);
            resid(o);
            push_hid(o);
        } else if (conv_fused(m, L) && L.ot_qs) {
            // in_proj + conv + out_proj as one phase over channels, accumulated (+ residual)
            PhaseDesc c = gemv(MK_STRIDE3, EK_CONV, 3, E, E, hid, an);
            c.type = PH_FUSED;
            set_src(c, 0, L.t[QQ_IN_PROJ]);
            c.stride = E;
            c.conv_w = L.t[QQ_CONV]->f32;
            c.state = m->conv(seq, l);
            c.E = E;
            c.N = E;
            c.n_expert = 1;
            c.top_k = 1;
            c.dt_qs = L.ot_qs;
            c.dt_d = L.ot_d;
            c.n_out = E;
            take_acc(c);
            prog.push_back(c);
            set_hid_acc(c);
        } else {
            PhaseDesc c = gemv(MK_STRIDE3, EK_CONV, 3, E, E, hid, an);
            set_src(c, 0, L.t[QQ_IN_PROJ]);
            c.stride = E;
            c.conv_w = L.t[QQ_CONV]->f32;
            c.state = m->conv(seq, l);
            c.E = E;
            c.y = take(E);
            prog.push_back(c);
            PhaseDesc o = gemv(MK_ROWS, EK_RESID, 1, E, E, tagged(c.y, (int)prog.size() - 1), nullptr);
            set_src(o, 0, L.t[QQ_OUT_PROJ]);
            resid(o);
            push_hid(o);
        }
        if (!L.moe && ffn_fused(m, L) && L.dt_qs) {
            const int F = (int)L.t[QQ_FFN_GATE]->ne[1];
            PhaseDesc g = gemv(MK_PAIR, EK_STORE, 2, E, F, hid, fn);
            g.type = PH_FUSED;  // without a router (r_qs null): one expert of weight 1
            g.G = kMoeG;
            set_src(g, 0, L.t[QQ_FFN_GATE]);
            set_src(g, 1, L.t[QQ_FFN_UP]);
            g.n_expert = 1;
            g.top_k = 1;
            g.N = F;
            g.dt_qs = L.dt_qs;
            g.dt_d = L.dt_d;
            g.n_out = E;
            take_acc(g);
            prog.push_back(g);
            set_hid_acc(g);
        } else if (L.moe && ffn_fused(m, L) && L.dt_qs) {
            const int k = d.n_expert_used;
            const int F = (int)L.t[QQ_GATE_EXPS]->ne[1];
            PhaseDesc g = gemv(MK_EXPERT_PAIR, EK_STORE, 2, E, k * F, hid, fn);
            g.type = PH_FUSED;
            g.G = kMoeG;
            set_src(g, 0, L.t[QQ_GATE_EXPS]);
            set_src(g, 1, L.t[QQ_UP_EXPS]);
            g.r_qs = L.t[QQ_ROUTER]->qs;
            g.r_d = L.t[QQ_ROUTER]->d;
            g.bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            g.rec = m->rec + (size_t)L.moe_slot * m->rec_len;
            g.ridx = m->ridx + (size_t)L.moe_slot * k;
            g.rw = m->rw + (size_t)L.moe_slot * k;
            g.n_expert = d.n_expert;
            g.top_k = k;
            g.mask = m->mask;
            g.N = F;
            g.dt_qs = L.dt_qs;
            g.dt_d = L.dt_d;
            g.n_out = E;
            take_acc(g);
            prog.push_back(g);
            set_hid_acc(g);
        } else if (L.moe) {
            // the down + combine phase reads its residual as tagged words
            QQ_CHECK(hid.t != nullptr, QQ_ERR_UNSUPPORTED, "persistent program: MoE after an accumulated vector");
            const int k = d.n_expert_used;
            const int F = (int)L.t[QQ_GATE_EXPS]->ne[1];
            PhaseDesc g = gemv(MK_EXPERT_PAIR, EK_SWIGLU, 2, E, k * F, hid, fn);
            g.G = qq3::decode_stage_items(2, E, F, k * F);  // groups must not straddle experts
            set_src(g, 0, L.t[QQ_GATE_EXPS]);
            set_src(g, 1, L.t[QQ_UP_EXPS]);
            g.r_qs = L.t[QQ_ROUTER]->qs;  // the router runs inside this phase, in every CTA
            g.r_d = L.t[QQ_ROUTER]->d;
            g.bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            g.rec = m->rec + (size_t)L.moe_slot * m->rec_len;
            g.ridx = m->ridx + (size_t)L.moe_slot * k;
            g.rw = m->rw + (size_t)L.moe_slot * k;
            g.n_expert = d.n_expert;
            g.top_k = k;
            g.mask = m->mask;
            g.N = F;
            g.y = take((size_t)k * F);
            prog.push_back(g);
            PhaseDesc dn = blank();
            dn.type = PH_DOWN4;
            dn.map = MK_DOWN4;
            dn.G = 4;
            dn.S = 4;
            dn.K = F;
            dn.n_items = E;
            dn.x = g.y;
            dn.x_ph = (int)prog.size() - 1;
            set_src(dn, 0, L.t[QQ_DOWN_EXPS]);
            dn.top_k = k;
            dn.mask = m->mask;
            dn.N = E;
            resid(dn);
            push_hid(dn);
        } else {
            const int F = (int)L.t[QQ_FFN_GATE]->ne[1];
            PhaseDesc g = gemv(MK_PAIR, EK_SWIGLU, 2, E, F, hid, fn);
            set_src(g, 0, L.t[QQ_FFN_GATE]);
            set_src(g, 1, L.t[QQ_FFN_UP]);
            g.y = take(F);
            prog.push_back(g);
            PhaseDesc dn = gemv(MK_ROWS, EK_RESID, 1, F, E, tagged(g.y, (int)prog.size() - 1), nullptr);
            set_src(dn, 0, L.t[QQ_FFN_DOWN]);
            resid(dn);
            push_hid(dn);
        }
    }
    if (want_logits) {
        const DTensor* out = m->output ? m->output : m->tok_embd;
        PhaseDesc h = gemv(MK_ROWS, EK_ARGMAX, 1, E, d.n_vocab, hid, m->out_norm->f32);
        set_src(h, 0, out);
        h.logits = m->logits;
        h.best = &m->dctl->best;
        h.suppress = m->suppress;
        prog.push_back(h);
        PhaseDesc f = blank();
        f.type = PH_FINISH;
        f.best = &m->dctl->best;
        f.ctl = m->ctl;
        f.trace = m->trace + (size_t)seq * (d.max_ctx + 1);
        prog.push_back(f);
    }
    QQ_CHECK((int)prog.size() <= qq3::kMaxPhases, QQ_ERR_UNSUPPORTED, "persistent program: too many phases");
    return prog;
}

bool mega_enabled(qq_model* m) {
    if (m->mega < 0) {
        // the persistent step is the default; QQ3_PERSISTENT=0 selects the per-phase kernels
        const char* env = getenv("QQ3_PERSISTENT");
        // the persistent step's fused FFN phase routes with the LFM2 rule only: a softmax-routed
        // (Qwen3-MoE) model takes the per-phase kernels
        bool ok = !(env && atoi(env) == 0) && qq3::stream_path() && !(m->d.arch == QQ_ARCH_QWEN3 && m->n_moe > 0) &&
                  m->ep_world <= 1;  // expert-parallel steps exchange rows between ranks: per-phase kernels
        if (ok) {
            std::vector<qq3::PhaseDesc> prog;
            try {
                prog = build_program(m, 0, true);
            } catch (const qq3::Error&) {
                ok = false;  // e.g. more phases than a tag can name: use the per-phase kernels
            }
            for (const auto& p : prog)
                if (!qq3::decode_phase_fits(p)) { ok = false; break; }
        }
        m->mega = ok ? 1 : 0;
    }
    return m->mega == 1;
}

qq_model::Prog& get_prog(qq_model* m, int seq, bool want_logits) {
    auto key = std::make_pair(seq, want_logits ? 1 : 0);
    auto it = m->progs.find(key);
    if (it != m->progs.end()) return it->second;
    std::vector<qq3::PhaseDesc> host = build_program(m, seq, want_logits);
    qq_model::Prog pr;
    pr.n = (int)host.size();
    pr.d_prog = dalloc<qq3::PhaseDesc>(host.size());
    cudaStream_t s = m->ctx->stream;
    QQ_CUDA_TRY(cudaMemcpyAsync(pr.d_prog, host.data(), sizeof(qq3::PhaseDesc) * host.size(), cudaMemcpyHostToDevice, s));
    QQ_CUDA_TRY(cudaStreamSynchronize(s));  // host vector goes out of scope
    return m->progs[key] = pr;
}

cudaGraphExec_t get_graph(qq_model* m, int seq, bool want_logits) {
    auto key = std::make_pair(seq, want_logits ? 1 : 0);
    auto it = m->graphs.find(key);
    if (it != m->graphs.end()) return it->second;
    cudaGraph_t g = nullptr;
    const bool mega = mega_enabled(m);
    qq_model::Prog* pr = mega ? &get_prog(m, seq, want_logits) : nullptr;
    QQ_CUDA_TRY(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeRelaxed));
    try {
        if (mega) qq3::launch_decode_step(pr->d_prog, pr->n, m->dctl, qq3::kernel_err_ptr(), m->cap);
        else enqueue_step(m, seq, want_logits, m->cap, false);
    } catch (...) {
        cudaStreamEndCapture(m->cap, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw;
    }
    QQ_CUDA_TRY(cudaStreamEndCapture(m->cap, &g));
    if (want_logits && !mega) {
        size_t n = 0;
        cudaGraphGetNodes(g, nullptr, &n);
        std::vector<cudaGraphNode_t> nodes(n);
        cudaGraphGetNodes(g, nodes.data(), &n);
        int64_t k = 0;
        for (auto nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
        }
        m->step_kernels = k;
    }
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    QQ_CUDA_TRY(e);
    if (mega) m->step_kernels = 1;
    m->graphs[key] = ge;
    return ge;
}

// One host-driven greedy step of the persistent kernel as one graph (key (seq, 3)): the token
// and position copied in from h_io[0..1], the step, and the argmax token, the next position and the
// kernel error word (which the step's closing CTA copies into ctl[2]) copied out to h_io[2..4], so
// that a step is one launch and one synchronisation.
cudaGraphExec_t get_io_graph(qq_model* m, int seq) {
    auto key = std::make_pair(seq, 3);
    auto it = m->graphs.find(key);
    if (it != m->graphs.end()) return it->second;
    qq_model::Prog& pr = get_prog(m, seq, true);
    cudaGraph_t g = nullptr;
    QQ_CUDA_TRY(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeRelaxed));
    try {
        QQ_CUDA_TRY(cudaMemcpyAsync(m->ctl, m->h_io, 2 * sizeof(int), cudaMemcpyHostToDevice, m->cap));
        qq3::launch_decode_step(pr.d_prog, pr.n, m->dctl, qq3::kernel_err_ptr(), m->cap);
        QQ_CUDA_TRY(cudaMemcpyAsync(m->h_io + 2, m->ctl, 3 * sizeof(int), cudaMemcpyDeviceToHost, m->cap));
    } catch (...) {
        cudaStreamEndCapture(m->cap, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw;
    }
    QQ_CUDA_TRY(cudaStreamEndCapture(m->cap, &g));
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    QQ_CUDA_TRY(e);
    m->graphs[key] = ge;
    return ge;
}

// One decode step of sequence seq on stream s: its captured graph, or, for an expert-parallel
// model (whose NCCL exchanges the host enqueues between the kernels), the kernel sequence itself.
void launch_step(qq_model* m, int seq, bool want_logits, cudaStream_t s) {
    if (m->ep_world > 1) enqueue_step(m, seq, want_logits, s, false);
    else QQ_CUDA_TRY(cudaGraphLaunch(get_graph(m, seq, want_logits), s));
}

void ensure_h_ctl(qq_model* m, size_t n) {
    if (n <= m->h_ctl_cap) return;
    if (m->h_ctl) {
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
        cudaFreeHost(m->h_ctl);
        m->h_ctl = nullptr;
    }
    size_t cap = 64;
    while (cap < n) cap *= 2;
    QQ_CUDA_TRY(cudaMallocHost(&m->h_ctl, cap * 2 * sizeof(int)));
    m->h_ctl_cap = cap;
}

void check_seq_pos(qq_model* m, int seq, int pos0, int n) {
    need(seq >= 0 && seq < m->d.n_seq, "seq_id out of range");
    need(pos0 >= 0 && n >= 0 && (int64_t)pos0 + n <= m->d.max_ctx,
         "positions [" + std::to_string(pos0) + ", " + std::to_string(pos0 + n) + ") exceed the KV capacity " +
             std::to_string(m->d.max_ctx));
}

void check_kernel_error(cudaStream_t s) {
    const int e = qq3::take_kernel_error(s);
    QQ_CHECK(e == 0, QQ_ERR_CUDA, "a kernel pipeline wait timed out (code " + std::to_string(e) + ")");
}

void set_suppress(qq_model* m, int id) {
    if (id == m->suppress_set) return;  // the device copy already holds it
    m->h_small[0] = id;
    QQ_CUDA_TRY(cudaMemcpyAsync(m->suppress, m->h_small, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
    if (m->tp_world > 1) {
        m->h_small[6] = (id >= m->v0 && id < m->v0 + m->v_local) ? id - m->v0 : -1;
        QQ_CUDA_TRY(cudaMemcpyAsync(m->tp_suppress, m->h_small + 6, sizeof(int), cudaMemcpyHostToDevice,
                                    m->ctx->stream));
    }
    m->suppress_set = id;
}

// ---- device sampling ------------------------------------------------------------------
// sampleWithThinkControl (tensor.js:244-265) after a decode step, on the step's logits.

qq3::SampleArgs sample_args(const qq_sample_params* p) {
    need(p != nullptr, "sampling parameters are required");
    need(p->think_mode >= QQ_THINK_SUPPRESS && p->think_mode <= QQ_THINK_FULL, "unknown thinking mode");
    // top_k ranks the end-of-thinking id in 'shorten' mode and limits top-k sampling; sampling
    // (temperature > 0) needs at least one candidate
    need(p->top_k >= (p->temperature > 0.0 ? 1 : 0) && p->top_k <= QQ_SAMPLE_MAX_TOP_K,
         "top_k must be in [1, " + std::to_string(QQ_SAMPLE_MAX_TOP_K) + "] for device sampling");
    need(!(p->temperature > 0.0) || p->top_p == p->top_p, "top_p is NaN");
    qq3::SampleArgs a;
    a.temperature = p->temperature;
    a.top_p = p->top_p;
    a.top_k = p->top_k;
    a.think_mode = p->think_mode;
    a.think_id = p->think_id;
    a.end_think_id = p->end_think_id;
    a.seed = p->seed;
    return a;
}

void ensure_sampling(qq_model* m) {
    if (m->sargs) return;
    m->sargs = dalloc<qq3::SampleArgs>(1);
    m->think_done = dalloc<int>((size_t)m->d.n_seq);
    m->spk = dalloc<uint32_t>((size_t)m->d.n_vocab);
    m->sout = dalloc<int>(1);
    QQ_CUDA_TRY(cudaMallocHost(&m->h_sargs, sizeof(qq3::SampleArgs)));
}

// the arguments and the sequence's 'thinking done' flag, in stream order
void put_sample_state(qq_model* m, const qq3::SampleArgs& a, int seq, int think_done) {
    cudaStream_t s = m->ctx->stream;
    QQ_CUDA_TRY(cudaStreamSynchronize(s));  // the pinned staging may still feed an earlier copy
    *m->h_sargs = a;
    m->h_small[5] = think_done ? 1 : 0;
    QQ_CUDA_TRY(cudaMemcpyAsync(m->sargs, m->h_sargs, sizeof(qq3::SampleArgs), cudaMemcpyHostToDevice, s));
    QQ_CUDA_TRY(cudaMemcpyAsync(m->think_done + seq, m->h_small + 5, sizeof(int), cudaMemcpyHostToDevice, s));
}

int* trace_of(qq_model* m, int seq) { return m->trace + (size_t)seq * (m->d.max_ctx + 1); }

// the decode step followed by the sampler, as one graph per sequence (key (seq, 2))
cudaGraphExec_t get_sample_graph(qq_model* m, int seq) {
    auto key = std::make_pair(seq, 2);
    auto it = m->graphs.find(key);
    if (it != m->graphs.end()) return it->second;
    const bool mega = mega_enabled(m);
    qq_model::Prog* pr = mega ? &get_prog(m, seq, true) : nullptr;
    cudaGraph_t g = nullptr;
    QQ_CUDA_TRY(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeRelaxed));
    try {
        if (mega) qq3::launch_decode_step(pr->d_prog, pr->n, m->dctl, qq3::kernel_err_ptr(), m->cap);
        else enqueue_step(m, seq, true, m->cap, false);
        qq3::launch_sample(m->logits, m->d.n_vocab, m->sargs, m->think_done + seq, -1.0, seq, -1, m->ctl,
                           trace_of(m, seq), m->sout, m->spk, m->cap);
    } catch (...) {
        cudaStreamEndCapture(m->cap, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw;
    }
    QQ_CUDA_TRY(cudaStreamEndCapture(m->cap, &g));
    cudaGraphExec_t ge = nullptr;
    cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    QQ_CUDA_TRY(e);
    m->graphs[key] = ge;
    return ge;
}

// sample after the logits of position pos (already computed), into ctl[0] and *m->sout
void sample_after(qq_model* m, int seq, int pos) {
    qq3::launch_sample(m->logits, m->d.n_vocab, m->sargs, m->think_done + seq, -1.0, seq, pos, m->ctl,
                       trace_of(m, seq), m->sout, m->spk, m->ctx->stream);
}

int read_sampled(qq_model* m) {
    cudaStream_t s = m->ctx->stream;
    QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->sout, sizeof(int), cudaMemcpyDeviceToHost, s));
    QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 4, qq3::kernel_err_ptr(), sizeof(int), cudaMemcpyDeviceToHost, s));
    QQ_CUDA_TRY(cudaStreamSynchronize(s));
    if (m->h_small[4]) check_kernel_error(s);
    return m->h_small[1];
}

// ---- batched prefill -------------------------------------------------------------------
// T prompt tokens at positions pos0.. through the layers at once: projections as tensor-core
// GEMMs, the MoE regrouped by expert, causal attention and the short-conv recurrence over the
// T rows (kernels_prefill.cu).  Same semantics as T sequential forward(t, pos, true) calls
// (qwen3-engine.js:397-457, lfm2-engine.js:523-583); the routing record of each MoE layer is
// that of the last token, as after the sequential calls.

constexpr int kPrefillChunk = 1024;  // tokens per pass (bounds the buffers)
// Shorter prompts take the per-token decode step.  Both meet the parity bar, but the tensor-core
// projections carry ~3e-6 relative error at K = 2048 (the tensor core's f32 accumulation) against
// ~1e-7 for the GEMV, so a router near-tie (selection-score gap < 1e-5, which the bar exempts)
// can resolve the other way in a batched prefill and change later tokens.
constexpr int kBatchedPrefillMin = 64;

struct PrefillBufs {
    int* tok;
    float *hidden, *xn, *y, *tmp, *bcx, *q, *k, *v, *attn, *g, *u, *h, *rec, *w;
    int* idx;
    __half* x16;
    void* moe;
    void* rows;  // few-row GEMM scratch (T <= kGemmFewMax), else null
};

PrefillBufs prefill_bufs(qq_model* m, int T) {
    const qq_model_desc& d = m->d;
    const size_t E = d.n_embd, nq = (size_t)d.n_head * d.head_dim, nkv = (size_t)d.n_head_kv * d.head_dim;
    size_t F = 0, Fe = 0;
    for (const Layer& L : m->layers) {
        if (L.moe) Fe = std::max<size_t>(Fe, L.t[QQ_GATE_EXPS]->ne[1]);
        else if (L.t[QQ_FFN_GATE]) F = std::max<size_t>(F, L.t[QQ_FFN_GATE]->ne[1]);
    }
    const int k = std::max(d.n_expert_used, 1);
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t C = (size_t)T;
    const size_t sizes[] = {al(C * 4),                                            // tok
                            al(C * E * 4), al(C * E * 4), al(C * E * 4), al(C * E * 4),  // hidden xn y tmp
                            al(C * 3 * E * 4), al(C * nq * 4), al(C * nkv * 4), al(C * nkv * 4),
                            al(C * nq * 4),                                        // attn
                            al(C * F * 4), al(C * F * 4), al(C * F * 4),           // g u h
                            al(C * (2 * k + d.n_expert) * 4), al(C * k * 4), al(C * k * 4),  // rec w idx
                            al(C * std::max({E, nq, F}) * 2 * (qq3::gemm_exact() ? 2 : 1)),  // x16 (hi, lo)
                            Fe ? al(qq3::moe_grouped_scratch_bytes(T, k, d.n_expert, E, Fe)) : 0,
                            T <= qq3::kGemmFewMax ? al(qq3::gemm_rows_scratch_bytes(T)) : 0};  // few-row GEMM
    size_t total = 0;
    for (size_t v : sizes) total += v;
    if (total > m->pf_bytes) {
        if (m->pf_arena) {
            QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
            cudaFree(m->pf_arena);
            m->pf_arena = nullptr;
            m->pf_bytes = 0;
        }
        m->pf_arena = dmalloc(total);
        m->pf_bytes = total;
    }
    char* b = static_cast<char*>(m->pf_arena);
    size_t i = 0;
    auto take = [&]() {
        char* r = b;
        b += sizes[i++];
        return r;
    };
    PrefillBufs p;
    p.tok = reinterpret_cast<int*>(take());
    p.hidden = reinterpret_cast<float*>(take());
    p.xn = reinterpret_cast<float*>(take());
    p.y = reinterpret_cast<float*>(take());
    p.tmp = reinterpret_cast<float*>(take());
    p.bcx = reinterpret_cast<float*>(take());
    p.q = reinterpret_cast<float*>(take());
    p.k = reinterpret_cast<float*>(take());
    p.v = reinterpret_cast<float*>(take());
    p.attn = reinterpret_cast<float*>(take());
    p.g = reinterpret_cast<float*>(take());
    p.u = reinterpret_cast<float*>(take());
    p.h = reinterpret_cast<float*>(take());
    p.rec = reinterpret_cast<float*>(take());
    p.w = reinterpret_cast<float*>(take());
    p.idx = reinterpret_cast<int*>(take());
    p.x16 = reinterpret_cast<__half*>(take());
    p.moe = take();
    p.rows = T <= qq3::kGemmFewMax ? take() : nullptr;
    return p;
}

void prefill_chunk(qq_model* m, const int32_t* tokens, int T, int seq, int pos0) {
    const qq_model_desc& d = m->d;
    cudaStream_t s = m->ctx->stream;
    const int E = d.n_embd, hd = d.head_dim;
    PrefillBufs b = prefill_bufs(m, T);
    QQ_CUDA_TRY(cudaMemcpyAsync(b.tok, tokens, sizeof(int) * T, cudaMemcpyHostToDevice, s));
    qq3::launch_embed_rows(*m->tok_embd, b.tok, T, d.n_vocab, b.hidden, s);
    const size_t TE = (size_t)T * E;
    // the residual of the previous layer's FFN / MoE, added by the next norm; the last layer's is
    // not added: nothing reads the rows' hidden state once the prompt's caches are written
    const float* pend = nullptr;
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        qq3::launch_add_rmsnorm_rows(b.hidden, pend, T, E, L.t[QQ_ATTN_NORM]->f32, d.rms_eps, b.xn, b.x16, s);
        pend = nullptr;
        if (L.attn) {
            qq3::launch_gemm_q8(*L.t[QQ_WQ], b.xn, T, b.x16, b.q, s, true);  // operand planes of the norm
            qq3::launch_gemm_q8(*L.t[QQ_WK], b.xn, T, b.x16, b.k, s, true);
            qq3::launch_gemm_q8(*L.t[QQ_WV], b.xn, T, b.x16, b.v, s, true);
            float* kc = m->k_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            float* vc = m->v_cache + seq * m->kv_stride_seq() + L.attn_slot * m->kv_stride_layer();
            qq3::launch_qk_norm_rope_rows(b.q, b.k, b.v, T, d.n_head, d.n_head_kv, hd, L.t[QQ_Q_NORM]->f32,
                                          L.t[QQ_K_NORM]->f32, d.rms_eps, m->rope_cs, nullptr, nullptr, pos0, 0,
                                          d.max_ctx, kc, vc, s);
            qq3::launch_attn_prefill(b.q, kc, vc, T, pos0, d.n_head, d.n_head_kv, hd, d.max_ctx, b.attn, s);
            qq3::launch_gemm_q8(*L.t[QQ_WO], b.attn, T, b.x16, b.tmp, s);
            if (m->tp_world > 1) qq3::comm_allreduce_sum_f32(m->ctx, b.tmp, b.tmp, TE, s);
        } else {
            qq3::launch_gemm_q8(*L.t[QQ_IN_PROJ], b.xn, T, b.x16, b.bcx, s, true);
            qq3::launch_conv_prefill(b.bcx, L.t[QQ_CONV]->f32, m->conv(seq, l), T, E, b.y, s);
            qq3::launch_gemm_q8(*L.t[QQ_OUT_PROJ], b.y, T, b.x16, b.tmp, s);
        }
        qq3::launch_add_rmsnorm_rows(b.hidden, b.tmp, T, E, L.t[QQ_FFN_NORM]->f32, d.rms_eps, b.xn, b.x16, s);
        if (L.moe) {
            const int k = d.n_expert_used;
            const float* bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            qq3::launch_router(*L.t[QQ_ROUTER], bias, b.xn, T, nullptr, 0.f, d.n_expert, k, d.arch == QQ_ARCH_QWEN3,
                               b.rec, b.idx, b.w, s);
            // the layer's routing record / ids / weights: those of the last token
            QQ_CUDA_TRY(cudaMemcpyAsync(m->rec + (size_t)L.moe_slot * m->rec_len, b.rec + (size_t)(T - 1) * m->rec_len,
                                        sizeof(float) * m->rec_len, cudaMemcpyDeviceToDevice, s));
            QQ_CUDA_TRY(cudaMemcpyAsync(m->ridx + (size_t)L.moe_slot * k, b.idx + (size_t)(T - 1) * k,
                                        sizeof(int) * k, cudaMemcpyDeviceToDevice, s));
            QQ_CUDA_TRY(cudaMemcpyAsync(m->rw + (size_t)L.moe_slot * k, b.w + (size_t)(T - 1) * k, sizeof(float) * k,
                                        cudaMemcpyDeviceToDevice, s));
            if (m->ep_world > 1) {
                ep_moe(m, L, b.xn, T, b.idx, b.w, b.hidden, s);  // adds the MoE output to the rows
                continue;
            }
            qq3::launch_moe_grouped(*L.t[QQ_GATE_EXPS], *L.t[QQ_UP_EXPS], *L.t[QQ_DOWN_EXPS], b.idx, b.w, m->mask,
                                    b.xn, T, k, d.n_expert, b.moe, b.tmp, s);
        } else {
            const size_t F = L.t[QQ_FFN_GATE]->ne[1];
            qq3::launch_gemm_q8(*L.t[QQ_FFN_GATE], b.xn, T, b.x16, b.g, s, true);
            qq3::launch_gemm_q8(*L.t[QQ_FFN_UP], b.xn, T, b.x16, b.u, s, true);
            qq3::launch_swiglu_rows_f16(b.g, b.u, (size_t)T * F, b.x16, s);
            qq3::launch_gemm_q8(*L.t[QQ_FFN_DOWN], b.h, T, b.x16, b.tmp, s, true);
            if (m->tp_world > 1) qq3::comm_allreduce_sum_f32(m->ctx, b.tmp, b.tmp, TE, s);
        }
        pend = b.tmp;
    }
}

// ---- multi-sequence decode step -----------------------------------------------------------
// One forward() step of each of T independent sequences at once: row t is token tok[t] of
// sequence seq[t] at position pos[t] (distinct sequences).  The layer pieces are those of the
// batched prefill -- projections as tensor-core GEMMs over the T rows (each weight streams once
// for all the sequences), the MoE regrouped by expert -- with a row map for RoPE, the K/V
// append, attention and the short-conv state; then the output norm, the lm_head GEMM and a
// first-max argmax per row.  The MoE routing record kept for onRouterUpdate is that of the last
// row.  Same results as T separate forward() calls up to the GEMM's f32 accumulation order.
// the tensor-parallel gather buffers for T rows (grow-only): keys of all ranks + this rank's, and
// all ranks' logits shards
void ensure_tp_bufs(qq_model* m, int T) {
    if (T <= m->tp_cap) return;
    QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    if (m->tp_keys) cudaFree(m->tp_keys);
    if (m->tp_logits) cudaFree(m->tp_logits);
    m->tp_keys = nullptr;
    m->tp_logits = nullptr;
    int cap = 16;
    while (cap < T) cap *= 2;
    m->tp_keys = dmalloc((size_t)(m->tp_world + 1) * cap * 32 * sizeof(unsigned long long));
    m->tp_logits = static_cast<float*>(dmalloc((size_t)m->tp_world * cap * m->v_local * sizeof(float)));
    m->tp_cap = cap;
}

void batch_step_on(qq_model* m, int T, int max_len, bool want_logits, cudaStream_t s) {
    const qq_model_desc& d = m->d;
    const int E = d.n_embd, hd = d.head_dim;
    PrefillBufs b = prefill_bufs(m, T);
    const int* tok = m->bt_i;
    const int* seq = m->bt_i + m->bt_cap;
    const int* pos = m->bt_i + 2 * m->bt_cap;
    QQ_CUDA_TRY(cudaMemcpyAsync(m->bt_i, m->h_bt, sizeof(int) * 3 * m->bt_cap, cudaMemcpyHostToDevice, s));
    if (b.rows) qq3::gemm_rows_reset(b.rows, s);
    qq3::launch_embed_rows(*m->tok_embd, tok, T, d.n_vocab, b.hidden, s);
    const size_t TE = (size_t)T * E;
    // the norms write the fp16 operand planes of the products that follow them (x16_ready), and
    // the residual of the previous layer's FFN / MoE is added by the next norm
    const float* pend = nullptr;
    for (int l = 0; l < d.n_layers; l++) {
        const Layer& L = m->layers[l];
        qq3::launch_add_rmsnorm_rows(b.hidden, pend, T, E, L.t[QQ_ATTN_NORM]->f32, d.rms_eps, b.xn, b.x16, s);
        pend = nullptr;
        if (L.attn) {
            qq3::launch_gemm_q8_few(*L.t[QQ_WQ], b.xn, T, b.x16, b.rows, b.q, s, true);
            qq3::launch_gemm_q8_few(*L.t[QQ_WK], b.xn, T, b.x16, b.rows, b.k, s, true);
            qq3::launch_gemm_q8_few(*L.t[QQ_WV], b.xn, T, b.x16, b.rows, b.v, s, true);
            float* kc = m->k_cache + L.attn_slot * m->kv_stride_layer();
            float* vc = m->v_cache + L.attn_slot * m->kv_stride_layer();
            qq3::launch_qk_norm_rope_rows(b.q, b.k, b.v, T, d.n_head, d.n_head_kv, hd, L.t[QQ_Q_NORM]->f32,
                                          L.t[QQ_K_NORM]->f32, d.rms_eps, m->rope_cs, seq, pos, 0, m->kv_stride_seq(),
                                          d.max_ctx, kc, vc, s);
            qq3::launch_attn_rows_split(b.q, kc, vc, T, seq, pos, max_len, m->kv_stride_seq(), d.n_head, d.n_head_kv,
                                        hd, d.max_ctx, m->bt_attn, b.attn, s, b.x16);
            qq3::launch_gemm_q8_few(*L.t[QQ_WO], b.attn, T, b.x16, b.rows, b.tmp, s, true);
            if (m->tp_world > 1) qq3::comm_allreduce_sum_f32(m->ctx, b.tmp, b.tmp, TE, s);  // heads' partial sums
        } else {
            qq3::launch_gemm_q8_few(*L.t[QQ_IN_PROJ], b.xn, T, b.x16, b.rows, b.bcx, s, true);
            qq3::launch_conv_rows_at(b.bcx, L.t[QQ_CONV]->f32, m->conv(0, l), (size_t)d.n_layers * 2 * E, seq, T, E,
                                     b.y, s);
            qq3::launch_gemm_q8_few(*L.t[QQ_OUT_PROJ], b.y, T, b.x16, b.rows, b.tmp, s);
        }
        qq3::launch_add_rmsnorm_rows(b.hidden, b.tmp, T, E, L.t[QQ_FFN_NORM]->f32, d.rms_eps, b.xn, b.x16, s);
        if (L.moe) {
            const int k = d.n_expert_used;
            const float* bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
            qq3::launch_router(*L.t[QQ_ROUTER], bias, b.xn, T, nullptr, 0.f, d.n_expert, k, d.arch == QQ_ARCH_QWEN3,
                               b.rec, b.idx, b.w, s);
            QQ_CUDA_TRY(cudaMemcpyAsync(m->rec + (size_t)L.moe_slot * m->rec_len, b.rec + (size_t)(T - 1) * m->rec_len,
                                        sizeof(float) * m->rec_len, cudaMemcpyDeviceToDevice, s));
            QQ_CUDA_TRY(cudaMemcpyAsync(m->ridx + (size_t)L.moe_slot * k, b.idx + (size_t)(T - 1) * k,
                                        sizeof(int) * k, cudaMemcpyDeviceToDevice, s));
            QQ_CUDA_TRY(cudaMemcpyAsync(m->rw + (size_t)L.moe_slot * k, b.w + (size_t)(T - 1) * k, sizeof(float) * k,
                                        cudaMemcpyDeviceToDevice, s));
            if (m->ep_world > 1) {
                ep_moe(m, L, b.xn, T, b.idx, b.w, b.hidden, s);  // adds the MoE output to the rows
                continue;
            }
            qq3::launch_moe_grouped(*L.t[QQ_GATE_EXPS], *L.t[QQ_UP_EXPS], *L.t[QQ_DOWN_EXPS], b.idx, b.w, m->mask,
                                    b.xn, T, k, d.n_expert, b.moe, b.tmp, s);
        } else {
            const size_t F = L.t[QQ_FFN_GATE]->ne[1];
            qq3::launch_gemm_q8_few(*L.t[QQ_FFN_GATE], b.xn, T, b.x16, b.rows, b.g, s, true);
            qq3::launch_gemm_q8_few(*L.t[QQ_FFN_UP], b.xn, T, b.x16, b.rows, b.u, s, true);
            qq3::launch_swiglu_rows_f16(b.g, b.u, (size_t)T * F, b.x16, s);
            qq3::launch_gemm_q8_few(*L.t[QQ_FFN_DOWN], b.h, T, b.x16, b.rows, b.tmp, s, true);
            if (m->tp_world > 1) qq3::comm_allreduce_sum_f32(m->ctx, b.tmp, b.tmp, TE, s);  // units' partial sums
        }
        pend = b.tmp;
    }
    if (!want_logits) return;  // the last residual add is left out with the logits: nothing reads it
    qq3::launch_add_rmsnorm_rows(b.hidden, pend, T, E, m->out_norm->f32, d.rms_eps, b.xn, b.x16, s);
    const DTensor* out = m->output ? m->output : m->tok_embd;
    qq3::launch_gemm_q8_few(*out, b.xn, T, b.x16, b.rows, m->bt_logits, s, true);
    if (m->tp_world > 1) {
        // this shard's greedy keys (global ids), all ranks' keys, then the first global maximum
        ensure_tp_bufs(m, T);
        const size_t kb = (size_t)T * 32 * sizeof(unsigned long long);
        char* keys_all = static_cast<char*>(m->tp_keys);
        char* mine = keys_all + (size_t)m->tp_world * m->tp_cap * 32 * sizeof(unsigned long long);
        qq3::launch_argmax_rows_keys(m->bt_logits, T, m->v_local, m->tp_suppress, m->v0, mine, s);
        qq3::comm_allgather(m->ctx, mine, keys_all, kb, s);
        qq3::launch_argmax_merge(keys_all, m->tp_world, T, m->bt_i + 3 * m->bt_cap, s);
        return;
    }
    qq3::launch_argmax_rows(m->bt_logits, T, d.n_vocab, m->suppress, m->bt_keys, m->bt_i + 3 * m->bt_cap, s);
}

// One multi-sequence step (rows in m->h_bt).  A dense single-GPU model replays it as a CUDA graph
// (per rows and want_logits; re-captured when the attention split count ceil(max_len / 64) or a
// buffer changes), which removes the launch gaps of its ~15 kernels per layer; the first step of
// a key runs eagerly (it sets the kernels' attributes).  QQ3_BATCH_GRAPH=0 always runs eagerly.
void batch_step(qq_model* m, int T, int max_len, bool want_logits) {
    cudaStream_t s = m->ctx->stream;
    static const bool graph_off = getenv_flag_zero("QQ3_BATCH_GRAPH");
    bool dense = true;
    for (const Layer& L : m->layers) dense = dense && !L.moe;
    if (graph_off || !dense || m->tp_world > 1 || m->ep_world > 1) {
        batch_step_on(m, T, max_len, want_logits, s);
        return;
    }
    prefill_bufs(m, T);  // any growth of the row buffers happens before a capture
    const int chunk = qq3::attn_rows_chunk();
    const int nz = (max_len + chunk - 1) / chunk;
    qq_model::BatchGraph& g = m->bgraphs[std::make_pair(T, want_logits ? 1 : 0)];
    const void* ptrs[5] = {m->pf_arena, m->bt_i, m->h_bt, m->bt_attn, m->bt_logits};
    const bool same_bufs = std::equal(ptrs, ptrs + 5, g.ptrs);
    if (g.exec && (g.nz != nz || !same_bufs)) {
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        cudaGraphExecDestroy(g.exec);
        g.exec = nullptr;
    }
    if (!g.seen) {
        g.seen = true;
        batch_step_on(m, T, max_len, want_logits, s);
        return;
    }
    if (!g.exec) {
        // captured with the longest length of this split count: the grid is the same
        const int cap_len = std::min(nz * chunk, m->d.max_ctx);
        cudaGraph_t gr = nullptr;
        QQ_CUDA_TRY(cudaStreamBeginCapture(m->cap, cudaStreamCaptureModeRelaxed));
        try {
            batch_step_on(m, T, cap_len, want_logits, m->cap);
        } catch (...) {
            cudaStreamEndCapture(m->cap, &gr);
            if (gr) cudaGraphDestroy(gr);
            cudaGetLastError();
            throw;
        }
        QQ_CUDA_TRY(cudaStreamEndCapture(m->cap, &gr));
        cudaGraphExec_t ge = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&ge, gr, 0);
        cudaGraphDestroy(gr);
        QQ_CUDA_TRY(e);
        g.exec = ge;
        g.nz = nz;
        std::copy(ptrs, ptrs + 5, g.ptrs);
    }
    QQ_CUDA_TRY(cudaGraphLaunch(g.exec, s));
}

// the vocab shards' logits of T rows from every rank into host logits [T][n_vocab]
void tp_logits_to_host(qq_model* m, int T, float* host) {
    cudaStream_t s = m->ctx->stream;
    ensure_tp_bufs(m, T);
    const size_t per = (size_t)T * m->v_local;
    qq3::comm_allgather(m->ctx, m->bt_logits, m->tp_logits, per * sizeof(float), s);
    for (int g = 0; g < m->tp_world; g++)
        QQ_CUDA_TRY(cudaMemcpy2DAsync(host + (size_t)g * m->v_local, sizeof(float) * m->d.n_vocab,
                                      m->tp_logits + (size_t)g * per, sizeof(float) * m->v_local,
                                      sizeof(float) * m->v_local, T, cudaMemcpyDeviceToHost, s));
}

// grow the multi-sequence row buffers to hold T rows (device and pinned staging)
void ensure_batch_rows(qq_model* m, int T) {
    if (T <= m->bt_cap) return;
    QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    if (m->bt_i) cudaFree(m->bt_i);
    if (m->bt_logits) cudaFree(m->bt_logits);
    if (m->bt_attn) cudaFree(m->bt_attn);
    if (m->bt_keys) cudaFree(m->bt_keys);
    if (m->h_bt) cudaFreeHost(m->h_bt);
    m->bt_i = nullptr;
    m->bt_logits = nullptr;
    m->bt_attn = nullptr;
    m->bt_keys = nullptr;
    m->h_bt = nullptr;
    m->bt_cap = 0;
    int cap = 16;
    while (cap < T) cap *= 2;
    m->bt_i = static_cast<int*>(dmalloc(sizeof(int) * 4 * cap));
    m->bt_logits = static_cast<float*>(dmalloc(sizeof(float) * (size_t)cap * m->d.n_vocab));
    m->bt_keys = dmalloc(qq3::argmax_rows_scratch_bytes(cap));
    if (m->n_attn > 0)
        m->bt_attn = static_cast<float*>(
            dmalloc(sizeof(float) * qq3::attn_rows_part_floats(cap, m->d.n_head, m->d.head_dim, m->d.max_ctx)));
    QQ_CUDA_TRY(cudaMallocHost(&m->h_bt, sizeof(int) * 4 * cap));
    m->bt_cap = cap;
}

bool batched_prefill_ok(qq_model* m) {
    if (getenv_flag("QQ3_NO_TCGEN05") || m->generic) return false;
    if (const char* v = getenv("QQ3_PREFILL_BATCH"))
        if (atoi(v) == 0) return false;
    const qq_model_desc& d = m->d;
    if (d.head_dim != 64 && d.head_dim != 128) return false;
    for (const Layer& L : m->layers)
        for (int sl = 0; sl < QQ_SLOT_COUNT; sl++)
            if (L.t[sl] && L.t[sl]->type == QQ_TYPE_Q8_0 && !qq3::gemm_q8_supported(*L.t[sl])) return false;
    return true;
}

// host-driven steps: token_ids[i] at pos0 + i; logits graph for the last one if requested
void run_tokens(qq_model* m, const int32_t* token_ids, int n, int seq, int pos0, bool want_logits) {
    cudaStream_t s = m->ctx->stream;
    for (int i = 0; i < n; i++) need(token_ids[i] >= 0 && token_ids[i] < m->d.n_vocab, "token id out of range");
    if (m->tp_world > 1) {
        // tensor-parallel: the prompt through the batched layers, the token with logits as a
        // one-row multi-sequence step (its greedy id and vocab shard in bt_i / bt_logits)
        const int n_batch = want_logits ? n - 1 : n;
        for (int c = 0; c < n_batch; c += kPrefillChunk)
            prefill_chunk(m, token_ids + c, std::min(kPrefillChunk, n_batch - c), seq, pos0 + c);
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // the host token array is read asynchronously above
        if (!want_logits) return;
        ensure_batch_rows(m, 1);
        m->h_bt[0] = token_ids[n - 1];
        m->h_bt[m->bt_cap] = seq;
        m->h_bt[2 * m->bt_cap] = pos0 + n - 1;
        batch_step(m, 1, pos0 + n, true);
        return;
    }
    // a long prefix runs batched; the token that needs logits takes the decode step below
    const int n_batch = want_logits ? n - 1 : n;
    if (n_batch >= kBatchedPrefillMin && batched_prefill_ok(m)) {
        for (int c = 0; c < n_batch; c += kPrefillChunk)
            prefill_chunk(m, token_ids + c, std::min(kPrefillChunk, n_batch - c), seq, pos0 + c);
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // the host token array is read asynchronously above
        token_ids += n_batch;
        pos0 += n_batch;
        n -= n_batch;
        if (n == 0) return;
    }
    ensure_h_ctl(m, (size_t)n);
    for (int i = 0; i < n; i++) {
        need(token_ids[i] >= 0 && token_ids[i] < m->d.n_vocab, "token id out of range");
        m->h_ctl[2 * i] = token_ids[i];
        m->h_ctl[2 * i + 1] = pos0 + i;
    }
    for (int i = 0; i < n; i++) {
        const bool logits = want_logits && i == n - 1;
        QQ_CUDA_TRY(cudaMemcpyAsync(m->ctl, m->h_ctl + 2 * i, 2 * sizeof(int), cudaMemcpyHostToDevice, s));
        launch_step(m, seq, logits, s);
    }
}

}  // namespace

// =====================================================================================
// C ABI

extern "C" {

const char* qq_last_error(void) { return qq3::last_error_cstr(); }

int qq_init(const int* devices, int n_devices, qq_ctx** out) {
    return guard([&] {
        need(out != nullptr, "qq_init: out is NULL");
        need(n_devices == 1 && devices != nullptr,
             "qq_init: this build drives one device per context (run one process per GPU)");
        int count = 0;
        QQ_CUDA_TRY(cudaGetDeviceCount(&count));
        need(devices[0] >= 0 && devices[0] < count, "qq_init: device index out of range");
        cudaDeviceProp p;
        QQ_CUDA_TRY(cudaGetDeviceProperties(&p, devices[0]));
        QQ_CHECK(p.major == 10 && p.minor == 0, QQ_ERR_UNSUPPORTED,
                 std::string("qq_init: libqq3cuda.so is built for sm_100a (B200); device is ") + p.name);
        DeviceGuard dg(devices[0]);
        qq_ctx* c = new qq_ctx;
        c->device = devices[0];
        cudaError_t e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete c;
            QQ_CUDA_TRY(e);
        }
        c->stream = c->own;
        if (const char* v = getenv("QQ3_STREAM_GEMV")) qq3::set_stream_path(atoi(v));
        if (const char* v = getenv("QQ3_PDL")) qq3::set_pdl(atoi(v));
        *out = c;
    });
}

int qq_destroy(qq_ctx* ctx) {
    return guard([&] {
        if (!ctx) return;
        DeviceGuard dg(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        if (ctx->scratch) cudaFree(ctx->scratch);
        qq3::comm_destroy(ctx);
        if (ctx->own) cudaStreamDestroy(ctx->own);
        delete ctx;
    });
}

int qq_set_stream(qq_ctx* ctx, void* cuda_stream) {
    return guard([&] {
        need(ctx != nullptr, "qq_set_stream: ctx is NULL");
        ctx->stream = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : ctx->own;
    });
}

int qq_synchronize(qq_ctx* ctx) {
    return guard([&] {
        need(ctx != nullptr, "qq_synchronize: ctx is NULL");
        DeviceGuard dg(ctx->device);
        QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        check_kernel_error(ctx->stream);
    });
}

int qq_upload_tensor(qq_ctx* ctx, const void* host, size_t nbytes, int ggml_type, const int64_t* ne, int n_dims,
                     qq_tensor** out) {
    return guard([&] {
        need(ctx && host && ne && out, "qq_upload_tensor: NULL argument");
        need(n_dims >= 1 && n_dims <= 4, "qq_upload_tensor: n_dims must be 1..4");
        QQ_CHECK(ggml_type == QQ_TYPE_F32 || ggml_type == QQ_TYPE_Q8_0 || qq3::kq_block_bytes(ggml_type) > 0,
                 QQ_ERR_UNSUPPORTED, "qq_upload_tensor: F32 (0), Q8_0 (8) and Q2_K..Q6_K (10..14) tensors only");
        DTensor t;
        t.type = ggml_type;
        t.n_dims = n_dims;
        int64_t n = 1;
        for (int i = 0; i < n_dims; i++) {
            need(ne[i] >= 1, "qq_upload_tensor: every ne[i] must be >= 1");
            t.ne[i] = ne[i];
            n *= ne[i];
        }
        t.K = t.ne[0];
        t.rows = n / t.ne[0];
        t.device = ctx->device;
        DeviceGuard dg(ctx->device);
        if (const int bs = qq3::kq_block_bytes(ggml_type)) {
            // k-quant superblocks stay raw (kernels_kquant.cu reads them in place)
            need(t.ne[0] % 256 == 0, "qq_upload_tensor: k-quant tensors need ne[0] % 256 == 0");
            const size_t bytes = (size_t)(n / 256) * bs;
            need(nbytes >= bytes, "qq_upload_tensor: buffer shorter than the k-quant superblocks");
            t.qs = dalloc<int8_t>(bytes + 256);
            QQ_CUDA_TRY(cudaMemcpyAsync(t.qs, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
            QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        } else if (ggml_type == QQ_TYPE_F32) {
            need(nbytes >= (size_t)n * 4, "qq_upload_tensor: buffer shorter than ne0*ne1*... floats");
            t.f32 = dalloc<float>((size_t)n);
            // ordered on the context stream: a pageable cudaMemcpy may return before its DMA
            // lands and only orders against the legacy stream, not this non-blocking one
            QQ_CUDA_TRY(cudaMemcpyAsync(t.f32, host, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->stream));
            QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        } else {
            need(t.ne[0] % 32 == 0, "qq_upload_tensor: Q8_0 needs ne[0] % 32 == 0");
            const int64_t nb = n / 32;
            need(nbytes >= (size_t)nb * 34, "qq_upload_tensor: buffer shorter than the Q8_0 block stream");
            uint8_t* raw = dalloc<uint8_t>((size_t)nb * 34);
            try {
                // +256 bytes: the streamed GEMV rounds the last group's scale copy up to 16 bytes
                t.qs = dalloc<int8_t>((size_t)n + 256);
                t.d = dalloc<__half>((size_t)nb + 128);
                QQ_CUDA_TRY(cudaMemcpyAsync(raw, host, (size_t)nb * 34, cudaMemcpyHostToDevice, ctx->stream));
                qq3::launch_repack_q8(raw, nb, t.qs, t.d, ctx->stream);
                QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
            } catch (...) {
                cudaFree(raw);
                if (t.qs) cudaFree(t.qs);
                if (t.d) cudaFree(t.d);
                throw;
            }
            cudaFree(raw);
        }
        qq_tensor* r = new qq_tensor;
        r->ctx = ctx;
        r->t = t;
        *out = r;
    });
}

int qq_free_tensor(qq_tensor* t) {
    return guard([&] {
        if (!t) return;
        DeviceGuard dg(t->t.device);
        if (t->t.qs) cudaFree(t->t.qs);
        if (t->t.d) cudaFree(t->t.d);
        if (t->t.f32) cudaFree(t->t.f32);
        delete t;
    });
}

int qq_tensor_info(const qq_tensor* t, int* ggml_type, int64_t* ne4, int* n_dims) {
    return guard([&] {
        need(t != nullptr, "qq_tensor_info: NULL tensor");
        if (ggml_type) *ggml_type = t->t.type;
        if (n_dims) *n_dims = t->t.n_dims;
        if (ne4)
            for (int i = 0; i < 4; i++) ne4[i] = t->t.ne[i];
    });
}

int qq_dequant(const qq_tensor* t, float* out_dev) {
    return guard([&] {
        need(t && out_dev, "qq_dequant: NULL argument");
        DeviceGuard dg(t->t.device);
        cudaStream_t s = t->ctx->stream;
        if (t->t.type == QQ_TYPE_F32)
            QQ_CUDA_TRY(cudaMemcpyAsync(out_dev, t->t.f32, sizeof(float) * t->t.K * t->t.rows,
                                        cudaMemcpyDeviceToDevice, s));
        else if (qq3::kq_block_bytes(t->t.type))
            qq3::launch_kq_dequant(t->t, 0, t->t.rows, out_dev, s);
        else
            qq3::launch_dequant_q8(t->t, out_dev, s);
    });
}

int qq_q8_matmul(qq_ctx* ctx, const qq_tensor* W, const float* x_dev, int M, float* y_dev) {
    return guard([&] {
        need(ctx && W && x_dev && y_dev, "qq_q8_matmul: NULL argument");
        need(M >= 0, "qq_q8_matmul: M < 0");
        QQ_CHECK(W->t.type == QQ_TYPE_Q8_0 || qq3::kq_block_bytes(W->t.type), QQ_ERR_UNSUPPORTED,
                 "qq_q8_matmul: W must be Q8_0 or a k-quant");
        DeviceGuard dg(ctx->device);
        const int64_t K = W->t.ne[0], N = W->t.ne[1];
        if (qq3::kq_block_bytes(W->t.type)) {  // k-quant: raw superblocks, CUDA-core matmul
            qq3::launch_kq_matmul(W->t, x_dev, M, y_dev, (int)N, ctx->stream);
            return;
        }
        if (M >= 2 && qq3::gemm_q8_supported(W->t) && !getenv_flag("QQ3_NO_TCGEN05")) {
            // tensor cores: fp16 operands, f32 accumulation in TMEM (kernels_gemm.cu)
            const size_t xb = (qq3::gemm_q8_scratch_bytes(M, K) + 255) & ~(size_t)255;
            if (M <= qq3::kGemmFewMax) {  // few rows: weights on the MMA's 128-row side, split-K
                char* sc = static_cast<char*>(ctx_scratch(ctx, xb + qq3::gemm_rows_scratch_bytes(M)));
                qq3::gemm_rows_reset(sc + xb, ctx->stream);
                qq3::launch_gemm_q8_few(W->t, x_dev, M, reinterpret_cast<__half*>(sc), sc + xb, y_dev, ctx->stream);
                return;
            }
            __half* x16 = static_cast<__half*>(ctx_scratch(ctx, xb));
            qq3::launch_gemm_q8(W->t, x_dev, M, x16, y_dev, ctx->stream);
            return;
        }
        for (int r = 0; r < M; r++) {
            qq3::XStage st;
            st.x[0] = x_dev + (size_t)r * K;
            st.K = (int)K;
            qq3::launch_gemv_rows(W->t, 0, N, st, y_dev + (size_t)r * N, false, ctx->stream);
        }
    });
}

int qq_rmsnorm(qq_ctx* ctx, const float* x_dev, int64_t n_rows, int n, const qq_tensor* w, float eps, float* y_dev) {
    return guard([&] {
        need(ctx && x_dev && w && y_dev, "qq_rmsnorm: NULL argument");
        need(w->t.type == QQ_TYPE_F32 && w->t.K * w->t.rows == n, "qq_rmsnorm: w must be F32 of length n");
        DeviceGuard dg(ctx->device);
        qq3::launch_rmsnorm(const_cast<float*>(x_dev), n_rows, n, w->t.f32, eps, y_dev, ctx->stream);
    });
}

int qq_rope(qq_ctx* ctx, float* x_dev, int n_rows, int n_heads, int head_dim, int pos0, double base) {
    return guard([&] {
        need(ctx && x_dev && n_rows >= 0 && n_heads >= 1 && pos0 >= 0, "qq_rope: bad argument");
        need(head_dim >= 2 && head_dim % 2 == 0, "qq_rope: head_dim must be even");
        if (n_rows == 0) return;
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        // cos/sin of (pos0 + r) * base^(-i/half) in double, stored f32 (tensor.js:137-140), the
        // table layout of the model's RoPE rows
        const int half = head_dim / 2;
        std::vector<float> tab((size_t)n_rows * head_dim);
        for (int r = 0; r < n_rows; r++)
            for (int i = 0; i < half; i++) {
                const double th = (double)(pos0 + r) * (1.0 / std::pow(base, (double)i / (double)half));
                tab[(size_t)r * head_dim + 2 * i] = (float)std::cos(th);
                tab[(size_t)r * head_dim + 2 * i + 1] = (float)std::sin(th);
            }
        float* cs = static_cast<float*>(ctx_scratch(ctx, tab.size() * sizeof(float)));
        QQ_CUDA_TRY(cudaMemcpyAsync(cs, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice, s));
        qq3::launch_rope_rows(x_dev, n_rows, n_heads, head_dim, cs, 0, s);
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // tab is a local buffer
    });
}

int qq_attention_decode(qq_ctx* ctx, const float* q_dev, const float* k_cache_dev, const float* v_cache_dev,
                        int n_head, int n_kv, int head_dim, int max_ctx, int pos, float* out_dev) {
    return guard([&] {
        need(ctx && q_dev && k_cache_dev && v_cache_dev && out_dev, "qq_attention_decode: NULL argument");
        need(n_kv >= 1 && n_head >= n_kv && n_head % n_kv == 0, "qq_attention_decode: n_head must be a multiple of n_kv");
        need(pos >= 0 && pos < max_ctx, "qq_attention_decode: pos outside the cache");
        QQ_CHECK(head_dim == 64 || head_dim == 128, QQ_ERR_UNSUPPORTED, "qq_attention_decode: head_dim must be 64 or 128");
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        // scratch: [sequence 0, position] | split partial states
        const size_t part = qq3::attn_rows_part_floats(1, n_head, head_dim, max_ctx) * sizeof(float);
        char* sc = static_cast<char*>(ctx_scratch(ctx, 256 + part));
        const int rowmap[2] = {0, pos};
        QQ_CUDA_TRY(cudaMemcpyAsync(sc, rowmap, sizeof(rowmap), cudaMemcpyHostToDevice, s));
        const int* dev = reinterpret_cast<const int*>(sc);
        qq3::launch_attn_rows_split(q_dev, k_cache_dev, v_cache_dev, 1, dev, dev + 1, pos + 1, 0, n_head, n_kv,
                                    head_dim, max_ctx, reinterpret_cast<float*>(sc + 256), out_dev, s);
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // rowmap is a local buffer
    });
}

int qq_embed(qq_ctx* ctx, const qq_tensor* E, const int32_t* tokens, int n, float* out_dev) {
    return guard([&] {
        need(ctx && E && tokens && out_dev && n >= 0, "qq_embed: bad argument");
        QQ_CHECK(E->t.type == QQ_TYPE_Q8_0 || qq3::kq_block_bytes(E->t.type), QQ_ERR_UNSUPPORTED,
                 "qq_embed: the embedding must be Q8_0 or a k-quant");
        for (int i = 0; i < n; i++) need(tokens[i] >= 0 && tokens[i] < E->t.rows, "qq_embed: token id out of range");
        if (n == 0) return;
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        if (qq3::kq_block_bytes(E->t.type)) {  // embeddingLookupGeneric -> the k-quant column reader
            for (int i = 0; i < n; i++) qq3::launch_kq_dequant(E->t, tokens[i], 1, out_dev + (size_t)i * E->t.K, s);
            QQ_CUDA_TRY(cudaStreamSynchronize(s));
            return;
        }
        int* tok = static_cast<int*>(ctx_scratch(ctx, sizeof(int) * (size_t)n));
        QQ_CUDA_TRY(cudaMemcpyAsync(tok, tokens, sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, s));
        qq3::launch_embed_rows(E->t, tok, n, (int)E->t.rows, out_dev, s);
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // tokens is the caller's host buffer
    });
}

int qq_swiglu(qq_ctx* ctx, const float* g_dev, const float* u_dev, int64_t n, float* h_dev) {
    return guard([&] {
        need(ctx && g_dev && u_dev && h_dev && n >= 0, "qq_swiglu: bad argument");
        DeviceGuard dg(ctx->device);
        qq3::launch_swiglu_rows(g_dev, u_dev, (size_t)n, h_dev, ctx->stream);
    });
}

int qq_add(qq_ctx* ctx, float* x_dev, const float* d_dev, int64_t n) {
    return guard([&] {
        need(ctx && x_dev && d_dev && n >= 0, "qq_add: bad argument");
        DeviceGuard dg(ctx->device);
        qq3::launch_add_rows(x_dev, d_dev, (size_t)n, ctx->stream);
    });
}

int qq_model_create(qq_ctx* ctx, const qq_model_desc* desc, qq_model** out) {
    return guard([&] {
        need(ctx && desc && out && desc->layers, "qq_model_create: NULL argument");
        // with tensor parallelism the model below is this rank's share: its heads, its vocab rows
        qq_model_desc dl = *desc;
        const int G = std::max(desc->tp_world, 1);
        if (G > 1) {
            need(desc->arch == QQ_ARCH_QWEN3, "qq_model_create: tensor parallelism is for dense Qwen3 models");
            need(ctx->comm != nullptr && ctx->comm_world == G,
                 "qq_model_create: tensor parallelism over tp_world ranks needs a communicator of that size");
            need(desc->ep_world <= 1, "qq_model_create: expert and tensor parallelism do not combine");
            need(desc->n_head % G == 0 && desc->n_head_kv % G == 0 && desc->n_vocab % G == 0,
                 "qq_model_create: heads and vocab must split evenly over tp_world ranks");
            need(desc->output != nullptr, "qq_model_create: tensor parallelism needs the rank's output rows");
            dl.n_head /= G;
            dl.n_head_kv /= G;
        }
        const qq_model_desc& d = dl;
        need(d.arch == QQ_ARCH_QWEN3 || d.arch == QQ_ARCH_LFM2, "qq_model_create: unknown arch");
        need(d.n_layers >= 1 && d.n_embd >= 32 && d.n_embd % 32 == 0, "qq_model_create: bad n_layers/n_embd");
        need(d.n_head >= 1 && d.n_head_kv >= 1 && d.n_head % d.n_head_kv == 0, "qq_model_create: bad head counts");
        QQ_CHECK(d.head_dim == 64 || d.head_dim == 128, QQ_ERR_UNSUPPORTED, "qq_model_create: head_dim must be 64/128");
        QQ_CHECK(d.n_head / d.n_head_kv <= 8, QQ_ERR_UNSUPPORTED, "qq_model_create: GQA group larger than 8");
        need(d.max_ctx >= 1 && d.n_seq >= 1 && d.n_vocab >= 1, "qq_model_create: bad max_ctx/n_seq/n_vocab");
        if (d.ep_world > 1) {
            need(ctx->comm != nullptr && ctx->comm_world == d.ep_world,
                 "qq_model_create: expert parallelism over ep_world ranks needs a communicator of that size (qq_comm_init)");
            need(d.n_expert > 0 && d.n_expert % d.ep_world == 0,
                 "qq_model_create: the experts must split evenly over ep_world ranks");
        }
        const int E = d.n_embd, hd = d.head_dim;
        const int nq = d.n_head * hd, nkv = d.n_head_kv * hd;
        DeviceGuard dg(ctx->device);
        qq_model* m = new qq_model;
        m->ctx = ctx;
        m->d = d;
        m->d.layers = nullptr;
        try {
            // k-quant weights (a dense Qwen3 on one GPU) run the op-by-op step: the type a check accepts
            bool any_moe = false;
            for (int l = 0; l < d.n_layers; l++) any_moe = any_moe || d.layers[l].is_moe;
            const bool kq_ok = d.arch == QQ_ARCH_QWEN3 && !any_moe && G <= 1 && d.ep_world <= 1;
            auto wt = [&](const DTensor* t) {
                if (t && qq3::kq_block_bytes(t->type) && kq_ok) {
                    m->generic = true;
                    return t->type;
                }
                return (int)QQ_TYPE_Q8_0;
            };
            m->tok_embd = dt(d.tok_embd);
            check_shape(m->tok_embd, wt(m->tok_embd), E, d.n_vocab, 1, "token_embd.weight");
            m->out_norm = dt(d.output_norm);
            check_shape(m->out_norm, QQ_TYPE_F32, E, 1, 1, "output norm");
            m->output = dt(d.output);
            if (m->output) check_shape(m->output, wt(m->output), E, d.n_vocab / G, 1, "output.weight");
            m->layers.resize(d.n_layers);
            for (int l = 0; l < d.n_layers; l++) {
                const qq_layer_desc& ld = d.layers[l];
                Layer& L = m->layers[l];
                L.attn = ld.is_attn != 0;
                L.moe = ld.is_moe != 0;
                for (int s = 0; s < QQ_SLOT_COUNT; s++) {
                    L.t[s] = dt(ld.t[s]);
                    if (ld.t[s]) need(ld.t[s]->ctx == ctx, "qq_model_create: tensor from another context");
                }
                const std::string b = "blk." + std::to_string(l) + ".";
                check_shape(L.t[QQ_ATTN_NORM], QQ_TYPE_F32, E, 1, 1, (b + "attn_norm.weight").c_str());
                check_shape(L.t[QQ_FFN_NORM], QQ_TYPE_F32, E, 1, 1, (b + "ffn_norm.weight").c_str());
                if (L.attn) {
                    L.attn_slot = m->n_attn++;
                    check_shape(L.t[QQ_WQ], wt(L.t[QQ_WQ]), E, nq, 1, (b + "attn_q.weight").c_str());
                    check_shape(L.t[QQ_WK], wt(L.t[QQ_WK]), E, nkv, 1, (b + "attn_k.weight").c_str());
                    check_shape(L.t[QQ_WV], wt(L.t[QQ_WV]), E, nkv, 1, (b + "attn_v.weight").c_str());
                    check_shape(L.t[QQ_WO], wt(L.t[QQ_WO]), nq, E, 1, (b + "attn_output.weight").c_str());
                    check_shape(L.t[QQ_Q_NORM], QQ_TYPE_F32, hd, 1, 1, (b + "attn_q_norm.weight").c_str());
                    check_shape(L.t[QQ_K_NORM], QQ_TYPE_F32, hd, 1, 1, (b + "attn_k_norm.weight").c_str());
                } else {
                    need(d.arch == QQ_ARCH_LFM2, "qq_model_create: short-conv layers exist only in LFM2");
                    check_shape(L.t[QQ_CONV], QQ_TYPE_F32, 3, E, 1, (b + "shortconv.conv.weight").c_str());
                    check_shape(L.t[QQ_IN_PROJ], QQ_TYPE_Q8_0, E, 3 * E, 1, (b + "shortconv.in_proj.weight").c_str());
                    check_shape(L.t[QQ_OUT_PROJ], QQ_TYPE_Q8_0, E, E, 1, (b + "shortconv.out_proj.weight").c_str());
                }
                if (L.moe) {
                    if (d.arch == QQ_ARCH_LFM2)
                        QQ_CHECK(d.n_expert_used == 4 && d.n_expert <= 32, QQ_ERR_UNSUPPORTED,
                                 "qq_model_create: LFM2 MoE layers need top-4 of <= 32 experts in this build");
                    else  // Qwen3-MoE: softmax router (qwen3-engine.js:304-363)
                        QQ_CHECK(d.n_expert_used >= 1 && d.n_expert_used <= 8 && d.n_expert <= 128 &&
                                     d.n_expert_used <= d.n_expert,
                                 QQ_ERR_UNSUPPORTED,
                                 "qq_model_create: Qwen3-MoE layers need top-k <= 8 of <= 128 experts in this build");
                    L.moe_slot = m->n_moe++;
                    const int64_t F = L.t[QQ_GATE_EXPS] ? L.t[QQ_GATE_EXPS]->ne[1] : 0;
                    const int rtype = (d.arch == QQ_ARCH_QWEN3 && L.t[QQ_ROUTER] && L.t[QQ_ROUTER]->type == QQ_TYPE_F32)
                                          ? QQ_TYPE_F32 : QQ_TYPE_Q8_0;
                    check_shape(L.t[QQ_ROUTER], rtype, E, d.n_expert, 1, (b + "ffn_gate_inp.weight").c_str());
                    const int nl = d.n_expert / std::max(d.ep_world, 1);  // experts this rank holds
                    check_shape(L.t[QQ_GATE_EXPS], QQ_TYPE_Q8_0, E, F, nl, (b + "ffn_gate_exps.weight").c_str());
                    check_shape(L.t[QQ_UP_EXPS], QQ_TYPE_Q8_0, E, F, nl, (b + "ffn_up_exps.weight").c_str());
                    check_shape(L.t[QQ_DOWN_EXPS], QQ_TYPE_Q8_0, F, E, nl, (b + "ffn_down_exps.weight").c_str());
                    if (L.t[QQ_EXP_BIAS])
                        check_shape(L.t[QQ_EXP_BIAS], QQ_TYPE_F32, d.n_expert, 1, 1, (b + "exp_probs_b.bias").c_str());
                    need(F % 32 == 0, "expert FFN width must be a multiple of 32");
                    if (d.n_expert_used * F > m->n_ff_max) m->n_ff_max = (int)(d.n_expert_used * F);
                } else {
                    const int64_t F = L.t[QQ_FFN_GATE] ? L.t[QQ_FFN_GATE]->ne[1] : 0;
                    check_shape(L.t[QQ_FFN_GATE], wt(L.t[QQ_FFN_GATE]), E, F, 1, (b + "ffn_gate.weight").c_str());
                    check_shape(L.t[QQ_FFN_UP], wt(L.t[QQ_FFN_UP]), E, F, 1, (b + "ffn_up.weight").c_str());
                    check_shape(L.t[QQ_FFN_DOWN], wt(L.t[QQ_FFN_DOWN]), F, E, 1, (b + "ffn_down.weight").c_str());
                    need(F % 32 == 0, "FFN width must be a multiple of 32");
                    if (F > m->n_ff_max) m->n_ff_max = (int)F;
                }
            }
            if (G > 1) {
                m->tp_world = G;
                m->tp_rank = ctx->comm_rank;
                m->v_local = d.n_vocab / G;
                m->v0 = m->tp_rank * m->v_local;
                m->tp_suppress = dalloc<int>(1);
                QQ_CUDA_TRY(cudaMemsetAsync(m->tp_suppress, 0xff, 4, ctx->stream));
                m->mega = 0;  // steps run through the multi-row path (batch_step)
            }
            if (d.ep_world > 1) {
                m->ep_world = d.ep_world;
                m->ep_rank = ctx->comm_rank;
                m->ep_xn = dalloc<float>(E);
            }
            m->n_expert_local = d.n_expert / std::max(m->ep_world, 1);
            if (m->generic) {
                m->mega = 0;
                m->gen_buf = dalloc<float>(2 * (size_t)std::max(m->n_ff_max, 32) + E);
                m->gen_keys = dmalloc(qq3::argmax_rows_scratch_bytes(1));
                m->gen_tok = dalloc<int>(1);
            }
            m->n_split = qq3::attention_splits(d.max_ctx);
            m->rec_len = 2 * d.n_expert_used + d.n_expert;
            m->hidden = dalloc<float>(E);
            m->qkv = dalloc<float>((size_t)nq + 2 * nkv);
            m->attn_out = dalloc<float>(nq);
            m->y = dalloc<float>(E);
            m->h = dalloc<float>((size_t)std::max(m->n_ff_max, 32));
            m->logits = dalloc<float>(d.n_vocab);
            const size_t kv = (size_t)d.n_seq * std::max(m->n_attn, 1) * nkv * d.max_ctx;
            m->k_cache = dalloc<float>(kv);
            m->v_cache = dalloc<float>(kv);
            QQ_CUDA_TRY(cudaMemsetAsync(m->k_cache, 0, kv * 4, ctx->stream));
            QQ_CUDA_TRY(cudaMemsetAsync(m->v_cache, 0, kv * 4, ctx->stream));
            const size_t cs = (size_t)d.n_seq * d.n_layers * 2 * E;
            m->conv_state = dalloc<float>(cs);
            QQ_CUDA_TRY(cudaMemsetAsync(m->conv_state, 0, cs * 4, ctx->stream));
            m->trace = dalloc<int>((size_t)d.n_seq * (d.max_ctx + 1));
            // RoPE table: cos/sin of position * base^(-i/half) in double (tensor.js:137-140)
            {
                const int half = hd / 2;
                std::vector<float> tab((size_t)d.max_ctx * hd);
                for (int p = 0; p < d.max_ctx; p++)
                    for (int i = 0; i < half; i++) {
                        const double freq = 1.0 / std::pow(d.rope_base, (double)i / (double)half);
                        const double th = (double)p * freq;
                        tab[(size_t)p * hd + 2 * i] = (float)std::cos(th);
                        tab[(size_t)p * hd + 2 * i + 1] = (float)std::sin(th);
                    }
                m->rope_cs = dalloc<float>(tab.size());
                QQ_CUDA_TRY(cudaMemcpyAsync(m->rope_cs, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, ctx->stream));
                QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));  // tab is a local buffer
            }
            m->attn_part = dalloc<float>((size_t)d.n_head * m->n_split * (hd + 2));
            m->attn_counter = dalloc<unsigned int>(d.n_head_kv);
            QQ_CUDA_TRY(cudaMemsetAsync(m->attn_counter, 0, sizeof(unsigned int) * d.n_head_kv, ctx->stream));
            const int nm = std::max(m->n_moe, 1);
            m->rec = dalloc<float>((size_t)nm * std::max(m->rec_len, 1));
            m->rlogits = dalloc<float>(std::max(d.n_expert, 1));
            m->rcounter = dalloc<unsigned int>(1);
            QQ_CUDA_TRY(cudaMemsetAsync(m->rcounter, 0, sizeof(unsigned int), ctx->stream));
            m->ridx = dalloc<int>((size_t)nm * std::max(d.n_expert_used, 1));
            m->rw = dalloc<float>((size_t)nm * std::max(d.n_expert_used, 1));
            QQ_CUDA_TRY(cudaMemsetAsync(m->rec, 0, sizeof(float) * nm * std::max(m->rec_len, 1), ctx->stream));
            QQ_CUDA_TRY(cudaMemsetAsync(m->ridx, 0, sizeof(int) * nm * std::max(d.n_expert_used, 1), ctx->stream));
            m->mask = dalloc<uint32_t>(8);
            QQ_CUDA_TRY(cudaMemsetAsync(m->mask, 0, 32, ctx->stream));
            m->ctl = dalloc<int>(4);
            QQ_CUDA_TRY(cudaMemsetAsync(m->ctl, 0, 16, ctx->stream));
            m->suppress = dalloc<int>(1);
            QQ_CUDA_TRY(cudaMemsetAsync(m->suppress, 0xff, 4, ctx->stream));
            m->best = dalloc<unsigned long long>(1);
            m->dump = dalloc<float>((size_t)d.n_layers * E);
            QQ_CUDA_TRY(cudaMallocHost(&m->h_small, 8 * sizeof(int)));
            QQ_CUDA_TRY(cudaMallocHost(&m->h_io, 8 * sizeof(int)));
            QQ_CUDA_TRY(cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking));
            QQ_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        } catch (...) {
            free_model(m);
            delete m;
            throw;
        }
        *out = m;
    });
}

int qq_model_destroy(qq_model* m) {
    return guard([&] {
        if (!m) return;
        DeviceGuard dg(m->ctx->device);
        cudaStreamSynchronize(m->ctx->stream);
        free_model(m);
        delete m;
    });
}

int qq_forward(qq_model* m, const int32_t* token_ids, int n_tokens, int seq_id, int pos0, int want_logits,
               float* logits_out, int32_t* argmax_out, int suppress_id) {
    return guard([&] {
        need(m && token_ids && n_tokens >= 1, "qq_forward: NULL argument or n_tokens < 1");
        check_seq_pos(m, seq_id, pos0, n_tokens);
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        const bool logits = want_logits != 0;
        if (logits) set_suppress(m, suppress_id);
        if (n_tokens == 1 && logits && !logits_out && argmax_out && m->tp_world <= 1 && m->ep_world <= 1 &&
            mega_enabled(m)) {
            // one greedy token of the persistent step: one graph launch and one synchronisation
            need(token_ids[0] >= 0 && token_ids[0] < m->d.n_vocab, "token id out of range");
            cudaGraphExec_t ge = get_io_graph(m, seq_id);
            m->h_io[0] = token_ids[0];
            m->h_io[1] = pos0;
            QQ_CUDA_TRY(cudaGraphLaunch(ge, s));
            QQ_CUDA_TRY(cudaStreamSynchronize(s));
            if (m->h_io[4]) check_kernel_error(s);  // reads the word again, clears it and throws
            *argmax_out = m->h_io[2];
            return;
        }
        run_tokens(m, token_ids, n_tokens, seq_id, pos0, logits);
        if (m->tp_world > 1) {
            if (logits && logits_out) tp_logits_to_host(m, 1, logits_out);
            if (logits) QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->bt_i + 3 * m->bt_cap, sizeof(int),
                                                    cudaMemcpyDeviceToHost, s));
            QQ_CUDA_TRY(cudaStreamSynchronize(s));
            check_kernel_error(s);
            if (logits && argmax_out) *argmax_out = m->h_small[1];
            return;
        }
        if (logits && logits_out)
            QQ_CUDA_TRY(cudaMemcpyAsync(logits_out, m->logits, sizeof(float) * m->d.n_vocab, cudaMemcpyDeviceToHost, s));
        if (logits && argmax_out)
            QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->ctl, sizeof(int), cudaMemcpyDeviceToHost, s));
        // the kernels' error word rides along: one synchronisation per call
        QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 4, qq3::kernel_err_ptr(), sizeof(int), cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        if (m->h_small[4]) check_kernel_error(s);  // reads it again, clears it and throws
        if (logits && argmax_out) *argmax_out = m->h_small[1];
    });
}

int qq_forward_batch(qq_model* m, const int32_t* seq_ids, const int32_t* token_ids, const int32_t* positions, int n,
                     int want_logits, float* logits_out, int32_t* argmax_out, int suppress_id) {
    return guard([&] {
        need(m && seq_ids && token_ids && positions && n >= 1, "qq_forward_batch: NULL argument or n < 1");
        std::vector<char> seen((size_t)m->d.n_seq, 0);
        for (int i = 0; i < n; i++) {
            check_seq_pos(m, seq_ids[i], positions[i], 1);
            need(!seen[(size_t)seq_ids[i]], "qq_forward_batch: a sequence appears twice in one call");
            seen[(size_t)seq_ids[i]] = 1;
            need(token_ids[i] >= 0 && token_ids[i] < m->d.n_vocab, "token id out of range");
        }
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        const bool logits = want_logits != 0;
        const size_t V = (size_t)m->d.n_vocab;
        if (logits) set_suppress(m, suppress_id);
        if (m->tp_world <= 1 && (n == 1 || !batched_prefill_ok(m))) {
            // one sequence (or no tensor-core path): the per-token decode step, row by row
            for (int i = 0; i < n; i++) {
                run_tokens(m, token_ids + i, 1, seq_ids[i], positions[i], logits);
                if (logits && logits_out)
                    QQ_CUDA_TRY(cudaMemcpyAsync(logits_out + i * V, m->logits, sizeof(float) * V,
                                                cudaMemcpyDeviceToHost, s));
                if (logits && argmax_out) {
                    QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->ctl, sizeof(int), cudaMemcpyDeviceToHost, s));
                    QQ_CUDA_TRY(cudaStreamSynchronize(s));
                    argmax_out[i] = m->h_small[1];
                }
            }
            QQ_CUDA_TRY(cudaStreamSynchronize(s));
            check_kernel_error(s);
            return;
        }
        ensure_batch_rows(m, n);
        int max_len = 1;
        for (int i = 0; i < n; i++) {
            m->h_bt[i] = token_ids[i];
            m->h_bt[m->bt_cap + i] = seq_ids[i];
            m->h_bt[2 * m->bt_cap + i] = positions[i];
            max_len = std::max(max_len, positions[i] + 1);
        }
        batch_step(m, n, max_len, logits);
        if (logits && logits_out) {
            if (m->tp_world > 1) tp_logits_to_host(m, n, logits_out);
            else QQ_CUDA_TRY(cudaMemcpyAsync(logits_out, m->bt_logits, sizeof(float) * V * n, cudaMemcpyDeviceToHost, s));
        }
        if (logits && argmax_out)
            QQ_CUDA_TRY(cudaMemcpyAsync(m->h_bt + 3 * m->bt_cap, m->bt_i + 3 * m->bt_cap, sizeof(int) * n,
                                        cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));  // also: the pinned staging is read asynchronously above
        check_kernel_error(s);
        if (logits && argmax_out)
            for (int i = 0; i < n; i++) argmax_out[i] = m->h_bt[3 * m->bt_cap + i];
    });
}

int qq_forward_dump(qq_model* m, int32_t token_id, int seq_id, int pos, float* hidden_out) {
    return guard([&] {
        need(m && m->tp_world <= 1, "qq_forward_dump: not available for a tensor-parallel model (use qq_forward / qq_forward_batch)");
        need(m && hidden_out, "qq_forward_dump: NULL argument");
        check_seq_pos(m, seq_id, pos, 1);
        need(token_id >= 0 && token_id < m->d.n_vocab, "token id out of range");
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        m->h_small[2] = token_id;
        m->h_small[3] = pos;
        QQ_CUDA_TRY(cudaMemcpyAsync(m->ctl, m->h_small + 2, 2 * sizeof(int), cudaMemcpyHostToDevice, s));
        enqueue_step(m, seq_id, false, s, true);
        QQ_CUDA_TRY(cudaMemcpyAsync(hidden_out, m->dump, sizeof(float) * m->d.n_layers * m->d.n_embd,
                                    cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        check_kernel_error(s);
    });
}

int qq_decode_loop(qq_model* m, int seq_id, int first_token, int pos0, int n_steps, int suppress_id,
                   int32_t* tokens_out) {
    return guard([&] {
        need(m && m->tp_world <= 1, "qq_decode_loop: not available for a tensor-parallel model (use qq_forward / qq_forward_batch)");
        need(m != nullptr && n_steps >= 0, "qq_decode_loop: bad argument");
        check_seq_pos(m, seq_id, pos0, n_steps);
        need(first_token >= 0 && first_token < m->d.n_vocab, "token id out of range");
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        set_suppress(m, suppress_id);
        m->h_small[2] = first_token;
        m->h_small[3] = pos0;
        QQ_CUDA_TRY(cudaMemcpyAsync(m->ctl, m->h_small + 2, 2 * sizeof(int), cudaMemcpyHostToDevice, s));
        for (int i = 0; i < n_steps; i++) launch_step(m, seq_id, true, s);
        if (tokens_out && n_steps > 0)
            QQ_CUDA_TRY(cudaMemcpyAsync(tokens_out, m->trace + (size_t)seq_id * (m->d.max_ctx + 1) + pos0 + 1,
                                        sizeof(int) * n_steps, cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        check_kernel_error(s);
    });
}

int qq_generate(qq_model* m, int seq_id, const int32_t* prompt, int n_prompt, int max_steps, int think_id,
                int eos_id, int32_t* out_tokens, int* n_out) {
    return guard([&] {
        need(m && m->tp_world <= 1, "qq_generate: not available for a tensor-parallel model (use qq_forward / qq_forward_batch)");
        need(m && prompt && n_prompt >= 1 && max_steps >= 0 && n_out, "qq_generate: bad argument");
        check_seq_pos(m, seq_id, 0, n_prompt + max_steps);
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        // resetState(): conv states to zero; KV positions are rewritten before use
        QQ_CUDA_TRY(cudaMemsetAsync(m->conv(seq_id, 0), 0, sizeof(float) * m->d.n_layers * 2 * m->d.n_embd, s));
        set_suppress(m, think_id);
        run_tokens(m, prompt, n_prompt, seq_id, 0, true);
        QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->ctl, sizeof(int), cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        int cur = m->h_small[1];
        int n = 0;
        if (eos_id < 0) {
            // no stop token: the whole continuation runs on the device
            if (max_steps > 0) {
                std::vector<int32_t> tail(max_steps);
                for (int i = 0; i < max_steps; i++) launch_step(m, seq_id, true, s);
                QQ_CUDA_TRY(cudaMemcpyAsync(tail.data(), m->trace + (size_t)seq_id * (m->d.max_ctx + 1) + n_prompt + 1,
                                            sizeof(int) * max_steps, cudaMemcpyDeviceToHost, s));
                QQ_CUDA_TRY(cudaStreamSynchronize(s));
                // generated = [cur, tail[0], ..., tail[max_steps-2]] (the last id is sampled, not fed)
                for (int i = 0; i < max_steps; i++) out_tokens[n++] = i == 0 ? cur : tail[i - 1];
            }
        } else {
            for (int step = 0; step < max_steps; step++) {
                if (cur == eos_id) break;
                int32_t t = cur;
                run_tokens(m, &t, 1, seq_id, n_prompt + step, true);
                QQ_CUDA_TRY(cudaMemcpyAsync(m->h_small + 1, m->ctl, sizeof(int), cudaMemcpyDeviceToHost, s));
                QQ_CUDA_TRY(cudaStreamSynchronize(s));
                out_tokens[n++] = cur;
                cur = m->h_small[1];
            }
        }
        *n_out = n;
    });
}

int qq_forward_sample(qq_model* m, int32_t token_id, int seq_id, int pos, const qq_sample_params* params,
                      int think_done, int32_t* token_out) {
    return guard([&] {
        need(m && m->tp_world <= 1, "qq_forward_sample: not available for a tensor-parallel model (use qq_forward / qq_forward_batch)");
        need(m && token_out, "qq_forward_sample: NULL argument");
        check_seq_pos(m, seq_id, pos, 1);
        const qq3::SampleArgs a = sample_args(params);
        DeviceGuard dg(m->ctx->device);
        ensure_sampling(m);
        put_sample_state(m, a, seq_id, think_done);
        run_tokens(m, &token_id, 1, seq_id, pos, true);
        sample_after(m, seq_id, pos);
        *token_out = read_sampled(m);
    });
}

int qq_generate_sample(qq_model* m, int seq_id, const int32_t* prompt, int n_prompt, int max_steps,
                       const qq_sample_params* params, int eos_id, int32_t* out_tokens, int* n_out) {
    return guard([&] {
        need(m && m->tp_world <= 1, "qq_generate_sample: not available for a tensor-parallel model (use qq_forward / qq_forward_batch)");
        need(m && prompt && n_prompt >= 1 && max_steps >= 0 && n_out && (out_tokens || max_steps == 0),
             "qq_generate_sample: bad argument");
        check_seq_pos(m, seq_id, 0, n_prompt + max_steps);
        const qq3::SampleArgs a = sample_args(params);
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        ensure_sampling(m);
        // resetState(): conv states to zero; KV positions are rewritten before use
        QQ_CUDA_TRY(cudaMemsetAsync(m->conv(seq_id, 0), 0, sizeof(float) * m->d.n_layers * 2 * m->d.n_embd, s));
        // thinkingDone starts true only in 'suppress' mode (lfm2-engine.js:537-542)
        put_sample_state(m, a, seq_id, a.think_mode == QQ_THINK_SUPPRESS);
        run_tokens(m, prompt, n_prompt, seq_id, 0, true);
        sample_after(m, seq_id, n_prompt - 1);
        int cur = read_sampled(m);
        int n = 0;
        if (eos_id < 0) {
            // no stop token: the whole continuation runs on the device (step + sampler graph)
            if (max_steps > 0) {
                std::vector<int32_t> tail(max_steps);
                for (int i = 0; i < max_steps; i++) {
                    if (m->ep_world > 1) {  // host-enqueued steps (see launch_step), then the sampler
                        enqueue_step(m, seq_id, true, s, false);
                        qq3::launch_sample(m->logits, m->d.n_vocab, m->sargs, m->think_done + seq_id, -1.0, seq_id, -1,
                                           m->ctl, trace_of(m, seq_id), m->sout, m->spk, s);
                    } else {
                        QQ_CUDA_TRY(cudaGraphLaunch(get_sample_graph(m, seq_id), s));
                    }
                }
                QQ_CUDA_TRY(cudaMemcpyAsync(tail.data(), trace_of(m, seq_id) + n_prompt + 1,
                                            sizeof(int) * max_steps, cudaMemcpyDeviceToHost, s));
                QQ_CUDA_TRY(cudaStreamSynchronize(s));
                check_kernel_error(s);
                for (int i = 0; i < max_steps; i++) out_tokens[n++] = i == 0 ? cur : tail[i - 1];
            }
        } else {
            for (int step = 0; step < max_steps; step++) {
                if (cur == eos_id) break;
                int32_t t = cur;
                run_tokens(m, &t, 1, seq_id, n_prompt + step, true);
                sample_after(m, seq_id, n_prompt + step);
                out_tokens[n++] = cur;
                cur = read_sampled(m);
            }
        }
        *n_out = n;
    });
}

int qq_sample_logits(qq_ctx* ctx, const float* logits_dev, int n, const qq_sample_params* params, double r,
                     int think_done, int32_t* token_out) {
    return guard([&] {
        need(ctx && logits_dev && token_out && n >= 1, "qq_sample_logits: bad argument");
        need(r >= 0.0 && r < 1.0, "qq_sample_logits: r must be a uniform draw in [0, 1)");
        const qq3::SampleArgs a = sample_args(params);
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        // scratch: [args | out, flag | keys]
        char* sc = static_cast<char*>(ctx_scratch(ctx, 256 + sizeof(uint32_t) * (size_t)n));
        auto* dargs = reinterpret_cast<qq3::SampleArgs*>(sc);
        int* dout = reinterpret_cast<int*>(sc + 128);
        int* dflag = dout + 1;
        struct {
            qq3::SampleArgs a;
            int flag;
        } h{a, think_done ? 1 : 0};
        QQ_CUDA_TRY(cudaMemcpyAsync(dargs, &h.a, sizeof(h.a), cudaMemcpyHostToDevice, s));
        QQ_CUDA_TRY(cudaMemcpyAsync(dflag, &h.flag, sizeof(int), cudaMemcpyHostToDevice, s));
        qq3::launch_sample(logits_dev, n, dargs, dflag, r, 0, 0, nullptr, nullptr, dout,
                           reinterpret_cast<uint32_t*>(sc + 256), s);
        int v = -1;
        QQ_CUDA_TRY(cudaMemcpyAsync(&v, dout, sizeof(int), cudaMemcpyDeviceToHost, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        *token_out = v;
    });
}

int qq_sample_uniform(uint64_t seed, int seq_id, int pos, double* r_out) {
    return guard([&] {
        need(r_out != nullptr, "qq_sample_uniform: NULL argument");
        *r_out = qq3::sample_uniform(seed, seq_id, pos);
    });
}

int qq_reset(qq_model* m, int seq_id) {
    return guard([&] {
        need(m != nullptr, "qq_reset: NULL model");
        need(seq_id >= 0 && seq_id < m->d.n_seq, "seq_id out of range");
        DeviceGuard dg(m->ctx->device);
        QQ_CUDA_TRY(cudaMemsetAsync(m->conv(seq_id, 0), 0, sizeof(float) * m->d.n_layers * 2 * m->d.n_embd,
                                    m->ctx->stream));
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    });
}

int qq_read_routing(qq_model* m, int moe_layer, float* out) {
    return guard([&] {
        need(m && out, "qq_read_routing: NULL argument");
        need(moe_layer >= 0 && moe_layer < m->n_moe, "qq_read_routing: moe_layer out of range");
        DeviceGuard dg(m->ctx->device);
        QQ_CUDA_TRY(cudaMemcpyAsync(out, m->rec + (size_t)moe_layer * m->rec_len, sizeof(float) * m->rec_len,
                                    cudaMemcpyDeviceToHost, m->ctx->stream));
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    });
}

int qq_set_expert_mask(qq_model* m, const int32_t* ids, int n) {
    return guard([&] {
        need(m != nullptr && n >= 0 && (n == 0 || ids), "qq_set_expert_mask: bad argument");
        uint32_t bits[8] = {0};
        for (int i = 0; i < n; i++) {
            need(ids[i] >= 0 && ids[i] < m->d.n_expert, "qq_set_expert_mask: expert id out of range");
            bits[ids[i] >> 5] |= 1u << (ids[i] & 31);
        }
        DeviceGuard dg(m->ctx->device);
        QQ_CUDA_TRY(cudaMemcpyAsync(m->mask, bits, sizeof(bits), cudaMemcpyHostToDevice, m->ctx->stream));
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    });
}

int qq_model_stat(qq_model* m, int what, int64_t* value) {
    return guard([&] {
        need(m && value, "qq_model_stat: NULL argument");
        if (what == QQ_STAT_STEP_KERNELS) {
            get_graph(m, 0, true);
            *value = m->step_kernels;
        } else if (what == QQ_STAT_N_MOE) {
            *value = m->n_moe;
        } else if (what == QQ_STAT_STEP_PHASES || what == QQ_STAT_MOE_FUSED) {
            int64_t n = 0;
            if (mega_enabled(m)) {
                const qq_model::Prog& pr = get_prog(m, 0, true);
                if (what == QQ_STAT_STEP_PHASES) {
                    n = pr.n;
                } else {
                    std::vector<qq3::PhaseDesc> h(pr.n);
                    QQ_CUDA_TRY(cudaMemcpy(h.data(), pr.d_prog, sizeof(qq3::PhaseDesc) * pr.n, cudaMemcpyDeviceToHost));
                    for (const auto& p : h) n += p.type == qq3::PH_FUSED && p.r_qs ? 1 : 0;
                }
            }
            *value = n;
        } else {
            need(false, "qq_model_stat: unknown statistic");
        }
    });
}

int qq_decode_trace(qq_model* m, int enable, uint64_t* stamps_out, int32_t* kinds_out, int* n_phases,
                    int* n_ctas) {
    return guard([&] {
        need(m && n_phases && n_ctas, "qq_decode_trace: NULL argument");
        DeviceGuard dg(m->ctx->device);
        need(mega_enabled(m), "qq_decode_trace: the model does not run the persistent decode step");
        cudaStream_t s = m->ctx->stream;
        qq_model::Prog& pr = get_prog(m, 0, true);
        const int np = pr.n, nc = qq3::num_sms();
        *n_phases = np;
        *n_ctas = nc;
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
        if (stamps_out && m->trace_buf)
            QQ_CUDA_TRY(cudaMemcpy(stamps_out, m->trace_buf, sizeof(uint64_t) * (size_t)nc * (np + 1),
                                   cudaMemcpyDeviceToHost));
        if (kinds_out) {
            // per phase: type | epi << 8 | (routed ? 1 << 16 : 0)
            std::vector<qq3::PhaseDesc> host((size_t)np);
            QQ_CUDA_TRY(cudaMemcpy(host.data(), pr.d_prog, sizeof(qq3::PhaseDesc) * np, cudaMemcpyDeviceToHost));
            for (int i = 0; i < np; i++)
                kinds_out[i] = host[i].type | (host[i].epi << 8) | (host[i].r_qs ? 1 << 16 : 0);
        }
        // phase stamps [nc][np + 1], then the sub-stamps [nc][np][kSubStamps] (zeroed: a point a
        // phase does not reach reads 0)
        const size_t n_main = (size_t)nc * (np + 1), n_sub = (size_t)nc * np * qq3::kSubStamps;
        if (enable && !m->trace_buf) m->trace_buf = dalloc<unsigned long long>(n_main + n_sub);
        if (enable) QQ_CUDA_TRY(cudaMemsetAsync(m->trace_buf + n_main, 0, sizeof(uint64_t) * n_sub, s));
        unsigned long long* ptrs[2] = {enable ? m->trace_buf : nullptr, enable ? m->trace_buf + n_main : nullptr};
        static_assert(offsetof(qq3::DecodeCtl, sub) == offsetof(qq3::DecodeCtl, trace) + sizeof(void*),
                      "trace and sub pointers are adjacent");
        QQ_CUDA_TRY(cudaMemcpyAsync(&m->dctl->trace, ptrs, sizeof(ptrs), cudaMemcpyHostToDevice, s));
        QQ_CUDA_TRY(cudaStreamSynchronize(s));
    });
}

int qq_decode_trace_sub(qq_model* m, uint64_t* out, int* n_sub) {
    return guard([&] {
        need(m && n_sub, "qq_decode_trace_sub: NULL argument");
        DeviceGuard dg(m->ctx->device);
        need(mega_enabled(m), "qq_decode_trace_sub: the model does not run the persistent decode step");
        qq_model::Prog& pr = get_prog(m, 0, true);
        const int np = pr.n, nc = qq3::num_sms();
        *n_sub = qq3::kSubStamps;
        if (!out) return;
        need(m->trace_buf != nullptr, "qq_decode_trace_sub: no traced step (qq_decode_trace)");
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
        QQ_CUDA_TRY(cudaMemcpy(out, m->trace_buf + (size_t)nc * (np + 1),
                               sizeof(uint64_t) * (size_t)nc * np * qq3::kSubStamps, cudaMemcpyDeviceToHost));
    });
}

int qq_ep_profile(qq_model* m, int enable, float* ms_out) {
    return guard([&] {
        need(m != nullptr, "qq_ep_profile: NULL model");
        need(m->ep_world > 1, "qq_ep_profile: not an expert-parallel model");
        DeviceGuard dg(m->ctx->device);
        QQ_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
        float acc[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
        for (auto& ev : m->ep_evs) {
            for (int i = 0; i < 4; i++) {
                float v = 0.f;
                QQ_CUDA_TRY(cudaEventElapsedTime(&v, ev[i], ev[i + 1]));
                acc[i] += v;
            }
            for (auto e : ev) cudaEventDestroy(e);
        }
        acc[4] = (float)m->ep_evs.size();
        m->ep_evs.clear();
        if (ms_out)
            for (int i = 0; i < 5; i++) ms_out[i] = acc[i];
        m->ep_prof = enable != 0;
    });
}

int qq_bench_kernel(qq_model* m, int what, int iters, float* ms) {
    return guard([&] {
        need(m && ms && iters >= 1, "qq_bench_kernel: bad argument");
        need(m->n_moe > 0, "qq_bench_kernel: the model has no MoE layer");
        need(what >= QQ_KERN_MOE_LAYER && what <= QQ_KERN_MOE_DOWN, "qq_bench_kernel: unknown kernel class");
        DeviceGuard dg(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        const qq_model_desc& d = m->d;
        const int k = d.n_expert_used;
        cudaEvent_t e0, e1;
        QQ_CUDA_TRY(cudaEventCreate(&e0));
        QQ_CUDA_TRY(cudaEventCreate(&e1));
        int64_t launches = 0;
        auto run = [&](bool timed) {
            for (int it = 0; it < (timed ? iters : 1); it++)
                for (const Layer& L : m->layers) {
                    if (!L.moe) continue;
                    qq3::XStage sf;
                    sf.x[0] = m->hidden;
                    sf.K = d.n_embd;
                    sf.norm_w = L.t[QQ_FFN_NORM]->f32;
                    sf.eps = d.rms_eps;
                    float* rec = m->rec + (size_t)L.moe_slot * m->rec_len;
                    int* idx = m->ridx + (size_t)L.moe_slot * k;
                    float* w = m->rw + (size_t)L.moe_slot * k;
                    const float* bias = L.t[QQ_EXP_BIAS] ? L.t[QQ_EXP_BIAS]->f32 : nullptr;
                    if (what == QQ_KERN_MOE_LAYER)
                        qq3::launch_lfm2_router(*L.t[QQ_ROUTER], bias, m->hidden, 1, sf.norm_w, sf.eps, d.n_expert, k,
                                                rec, idx, w, s);
                    if (what != QQ_KERN_MOE_DOWN)
                        qq3::launch_moe_gateup(*L.t[QQ_GATE_EXPS], *L.t[QQ_UP_EXPS], idx, m->mask, k, sf, m->h, s);
                    if (what != QQ_KERN_MOE_GATEUP)
                        qq3::launch_moe_down_combine(*L.t[QQ_DOWN_EXPS], idx, w, m->mask, k, m->h, m->hidden, s);
                    if (timed) launches++;
                }
        };
        run(false);  // warm-up round
        QQ_CUDA_TRY(cudaEventRecord(e0, s));
        run(true);
        QQ_CUDA_TRY(cudaEventRecord(e1, s));
        QQ_CUDA_TRY(cudaEventSynchronize(e1));
        float t = 0.f;
        QQ_CUDA_TRY(cudaEventElapsedTime(&t, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *ms = t / (float)launches;
    });
}

// T at and above which qq_moe_block regroups the rows by expert (tensor-core GEMMs) instead of
// running the per-token expert GEMVs
constexpr int kGroupedMoeRows = 16;

int qq_moe_block(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k, const float* x_dev, int T,
                 float* out_dev, float* routing_dev) {
    return guard([&] {
        need(ctx && layer && x_dev && out_dev && T >= 0, "qq_moe_block: bad argument");
        const DTensor* router = dt(layer->t[QQ_ROUTER]);
        const DTensor* gate = dt(layer->t[QQ_GATE_EXPS]);
        const DTensor* up = dt(layer->t[QQ_UP_EXPS]);
        const DTensor* down = dt(layer->t[QQ_DOWN_EXPS]);
        const DTensor* bias = dt(layer->t[QQ_EXP_BIAS]);
        need(router && gate && up && down, "qq_moe_block: router and expert tensors are required");
        QQ_CHECK(top_k == 4 && n_expert >= 4 && n_expert <= 32, QQ_ERR_UNSUPPORTED,
                 "qq_moe_block: this build routes top-4 of <= 32 experts");
        const int64_t K = router->ne[0], F = gate->ne[1];
        check_shape(router, QQ_TYPE_Q8_0, K, n_expert, 1, "ffn_gate_inp.weight");
        check_shape(gate, QQ_TYPE_Q8_0, K, F, n_expert, "ffn_gate_exps.weight");
        check_shape(up, QQ_TYPE_Q8_0, K, F, n_expert, "ffn_up_exps.weight");
        check_shape(down, QQ_TYPE_Q8_0, F, K, n_expert, "ffn_down_exps.weight");
        if (bias) check_shape(bias, QQ_TYPE_F32, n_expert, 1, 1, "exp_probs_b.bias");
        if (T == 0) return;
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        const int rec_len = 2 * top_k + n_expert;
        // scratch: idx [T][k] | w [T][k] | record [T][rec_len] (unless the caller wants it) | h [k][F]
        const size_t b_idx = (size_t)T * top_k * 4, b_w = b_idx, b_rec = routing_dev ? 0 : (size_t)T * rec_len * 4;
        const bool grouped = T >= kGroupedMoeRows && qq3::gemm_q8_supported(*gate) && qq3::gemm_q8_supported(*down) &&
                             !getenv_flag("QQ3_NO_TCGEN05");
        const size_t b_h = grouped ? qq3::moe_grouped_scratch_bytes(T, top_k, n_expert, K, F) : (size_t)top_k * F * 4;
        auto align = [](size_t v) { return (v + 255) & ~(size_t)255; };
        char* base = static_cast<char*>(ctx_scratch(ctx, align(b_idx) + align(b_w) + align(b_rec) + align(b_h)));
        int* idx = reinterpret_cast<int*>(base);
        float* w = reinterpret_cast<float*>(base + align(b_idx));
        float* rec = routing_dev ? routing_dev : reinterpret_cast<float*>(base + align(b_idx) + align(b_w));
        float* h = reinterpret_cast<float*>(base + align(b_idx) + align(b_w) + align(b_rec));
        qq3::launch_lfm2_router(*router, bias ? bias->f32 : nullptr, x_dev, T, nullptr, 0.f, n_expert, top_k, rec, idx,
                                w, s);
        if (grouped) {  // rows regrouped by expert: each expert's weights stream once (tensor cores)
            qq3::launch_moe_grouped(*gate, *up, *down, idx, w, nullptr, x_dev, T, top_k, n_expert, h, out_dev, s);
            return;
        }
        QQ_CUDA_TRY(cudaMemsetAsync(out_dev, 0, sizeof(float) * (size_t)T * K, s));
        for (int t = 0; t < T; t++) {
            qq3::XStage st;
            st.x[0] = x_dev + (size_t)t * K;
            st.K = (int)K;
            qq3::launch_moe_gateup(*gate, *up, idx + (size_t)t * top_k, nullptr, top_k, st, h, s);
            qq3::launch_moe_down_combine(*down, idx + (size_t)t * top_k, w + (size_t)t * top_k, nullptr, top_k, h,
                                         out_dev + (size_t)t * K, s);
        }
    });
}

int qq_moe_route(qq_ctx* ctx, const qq_layer_desc* layer, int n_expert, int top_k, const float* x_dev, int T,
                 int32_t* idx_dev, float* w_dev, float* routing_dev) {
    return guard([&] {
        need(ctx && layer && x_dev && idx_dev && w_dev && T >= 0, "qq_moe_route: bad argument");
        const DTensor* router = dt(layer->t[QQ_ROUTER]);
        const DTensor* bias = dt(layer->t[QQ_EXP_BIAS]);
        need(router != nullptr, "qq_moe_route: the router tensor is required");
        check_shape(router, QQ_TYPE_Q8_0, router->ne[0], n_expert, 1, "ffn_gate_inp.weight");
        if (bias) check_shape(bias, QQ_TYPE_F32, n_expert, 1, 1, "exp_probs_b.bias");
        if (T == 0) return;
        DeviceGuard dg(ctx->device);
        cudaStream_t s = ctx->stream;
        float* rec = routing_dev;
        if (!rec) rec = static_cast<float*>(ctx_scratch(ctx, (size_t)T * (2 * top_k + n_expert) * 4));
        qq3::launch_lfm2_router(*router, bias ? bias->f32 : nullptr, x_dev, T, nullptr, 0.f, n_expert, top_k, rec,
                                idx_dev, w_dev, s);
    });
}

int qq_moe_experts(qq_ctx* ctx, const qq_layer_desc* layer, int n_local, const float* x_dev, const int32_t* eid_dev,
                   int R, float* y_dev) {
    return guard([&] {
        need(ctx && layer && R >= 0 && n_local >= 1 && (R == 0 || (x_dev && eid_dev && y_dev)),
             "qq_moe_experts: bad argument");
        const DTensor* gate = dt(layer->t[QQ_GATE_EXPS]);
        const DTensor* up = dt(layer->t[QQ_UP_EXPS]);
        const DTensor* down = dt(layer->t[QQ_DOWN_EXPS]);
        need(gate && up && down, "qq_moe_experts: expert tensors are required");
        const int64_t K = gate->ne[0], F = gate->ne[1];
        check_shape(gate, QQ_TYPE_Q8_0, K, F, n_local, "ffn_gate_exps.weight");
        check_shape(up, QQ_TYPE_Q8_0, K, F, n_local, "ffn_up_exps.weight");
        check_shape(down, QQ_TYPE_Q8_0, F, K, n_local, "ffn_down_exps.weight");
        QQ_CHECK(n_local <= 256 && qq3::gemm_q8_supported(*gate) && qq3::gemm_q8_supported(*down) &&
                     !getenv_flag("QQ3_NO_TCGEN05"),
                 QQ_ERR_UNSUPPORTED, "qq_moe_experts: needs the tensor-core grouped GEMM");
        if (R == 0) return;
        DeviceGuard dg(ctx->device);
        // each row is its own (token, slot) pair: top_k 1, weight 1
        void* scratch = ctx_scratch(ctx, qq3::moe_grouped_scratch_bytes(R, 1, n_local, K, F));
        qq3::launch_moe_grouped(*gate, *up, *down, eid_dev, nullptr, nullptr, x_dev, R, 1, n_local, scratch, y_dev,
                                ctx->stream);
    });
}

int qq_moe_combine(qq_ctx* ctx, const float* y_dev, const int32_t* pos_dev, const float* w_dev, int T, int top_k,
                   int K, float* out_dev) {
    return guard([&] {
        need(ctx && T >= 0 && top_k >= 1 && K >= 1 && (T == 0 || (y_dev && pos_dev && w_dev && out_dev)),
             "qq_moe_combine: bad argument");
        DeviceGuard dg(ctx->device);
        qq3::launch_moe_combine_rows(y_dev, pos_dev, w_dev, T, top_k, K, out_dev, ctx->stream);
    });
}

}  // extern "C"
