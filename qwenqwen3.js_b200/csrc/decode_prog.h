// decode_prog.h -- the decode step as a device-side program of phases, run by one persistent
// kernel (kernels_decode.cu).  Built once per (model, sequence) by the runtime (api.cu).
//
// Activations between phases are tagged words: (tag << 32 | float bits), written once per step
// with one 64-bit store, tag = step epoch * 256 + writing phase + 1.  A reader spins until the
// words it needs carry the tag of their producer phase, so data arrival is the only
// synchronisation between CTAs; every phase writes its own output buffer, so no word is
// written twice in one step.
//
// A fused phase (PH_FUSED) instead sums partial outputs of every CTA into an accumulated
// vector (a bulk f32 add-reduction at L2 per CTA) and counts the CTAs that are done in a
// counter next to it; a reader waits for the counter before it reads the vector.  Accumulated vectors and counters live in
// an arena of two halves: step `epoch` uses half (epoch & 1) and zeroes the other half, which
// the previous step used and the next step will use.
#pragma once
#include "kernels.h"

namespace qq3 {

typedef unsigned long long tword;  // tagged activation word

constexpr int kMaxPhases = 255;  // phase index fits the low byte of a tag

enum PhaseType : int {
    PH_EMBED = 0,   // hidden = dequantised embedding row of the token; argmax key reset
    PH_GEMV = 1,    // streamed Q8_0 GEMV, one shared input (consumer mode A)
    PH_DOWN4 = 2,   // MoE down + combine + residual over the 4 routed experts (consumer mode B)
    PH_ATTN = 3,    // GQA decode attention with QK-norm, RoPE and KV append
    PH_FINISH = 4,  // token = argmax, pos += 1, trace
    PH_FUSED = 5,   // a layer half split over units, outputs accumulated: an FFN (router + expert
                    // gate/up + SwiGLU + down + combine + residual; a dense FFN as one expert of
                    // weight 1), or a short-conv block (in_proj + conv + out_proj + residual)
};

enum MapKind : int { MK_ROWS = 0, MK_CONCAT3 = 1, MK_PAIR = 2, MK_STRIDE3 = 3, MK_EXPERT_PAIR = 4, MK_DOWN4 = 5 };

enum EpiKind : int { EK_STORE = 0, EK_RESID = 1, EK_SWIGLU = 2, EK_CONV = 3, EK_ARGMAX = 4 };

// 16-byte aligned and sized: the persistent kernel copies descriptors into shared memory
struct alignas(16) PhaseDesc {
    int type, map, epi, S;
    int K;        // inner dimension (input length)
    int n_items;  // outputs of the phase
    int pad0;
    int G;        // items per stage (multiple of 4; stages are sized to ~16 KB for the bulk-copy stream)
    // input
    const tword* x;       // mode A input, or the 4 expert inputs h[0..3] (stride K) for PH_DOWN4
    int x_ph;             // phase that writes x
    int res_ph;           // phase that writes res
    const tword* res;     // residual stream read by EK_RESID and PH_DOWN4 (own items)
    const float* norm_w;  // fused RMSNorm weight (nullable)
    float eps;
    int n0, n1;           // MK_CONCAT3 boundaries
    int N;                // rows per expert (expert maps)
    int64_t stride;       // MK_STRIDE3
    const int8_t* qs[3];
    const __half* d[3];
    int* ridx;            // routed expert ids / weights / record, written by CTA 0 for the host
    float* rw;
    float* rec;
    const uint32_t* mask;
    // epilogue
    tword* y;             // output (tagged with this phase)
    const float* conv_w;
    float* state;
    int E;
    int n_expert, top_k;
    int pad1;
    float* logits;
    unsigned long long* best;
    const int* suppress;
    const int8_t* r_qs;     // router rows fused into the expert gate/up phase (nullable)
    const __half* r_d;
    const float* bias;
    // attention / embed / finish
    AttnArgs attn;        // qkv and out are unused: the tagged forms below replace them
    const tword* a_qkv;
    int a_qkv_ph;
    int pad2;
    tword* a_out;
    const int8_t* emb_qs;
    const __half* emb_d;
    int emb_K, n_vocab;
    int* ctl;    // [token, pos]
    int* trace;  // per-sequence greedy ids by position
    // accumulated vectors (addresses in arena half 0; the kernel adds the half of the step)
    const float* xa;         // input read instead of x (nullable)
    const unsigned* xa_cnt;  // its counter and the count that completes it
    int xa_n;
    int ra_n;
    const float* ra;         // residual read instead of res by EK_RESID (nullable)
    const unsigned* ra_cnt;
    // PH_FUSED: the expert down tensor transposed, and the accumulated output
    const int8_t* dt_qs;     // [n_expert][N][n_out] int8: row j of expert e = column j of its down
    const __half* dt_d;      // [n_expert][N/32][n_out] block scales
    float* acc;              // [n_out] sum over CTAs (+ the residual), zero at the start of the step
    unsigned* acc_cnt;       // CTAs done (gridDim.x completes it)
    int n_out;
    int pad3;
};

static_assert(sizeof(PhaseDesc) % 16 == 0, "phase descriptors are copied in 16-byte units");

// Control block of the persistent kernel, one per model (shared by all its programs).
struct DecodeCtl {
    unsigned int epoch;       // steps run; tags of the current step derive from it
    unsigned int end_ticket;  // CTAs done with the current step (the last one closes the step)
    unsigned long long best;  // argmax key of the logits (reset by the CTA that closes the step)
    float* arena;             // accumulated vectors and counters: two halves of arena_half words
    long long arena_half;
    // per-phase trace (nullable): CTA c writes the %globaltimer at its start to
    // trace[c * (n_phases + 1)] and at the end of phase ph to trace[c * (n_phases + 1) + ph + 1]
    unsigned long long* trace;
    // per-phase sub-stamps (nullable): thread 0 of CTA c writes %globaltimer at the points of
    // DecSub to sub[(c * n_phases + ph) * kSubStamps + k]; a point a phase does not reach is left
    unsigned long long* sub;
    unsigned int pad[20];
};

// Points of a phase that the sub-stamps record (for thread 0 of each CTA).
enum DecSub : int {
    SUB_INPUT = 0,      // its input wait is over (the counter complete, or its tagged words carry the tag)
    SUB_STAGED = 1,     // the input is staged (RMSNorm, digits) and the CTA's warps met
    SUB_ROUTED = 2,     // the CTA has routed the token (routed FFN phases)
    SUB_FIRST = 3,      // the first weight stage of the phase has landed (thread 0's set)
    SUB_PART1 = 4,      // the first part is done: gate/up + SwiGLU (fused), all rows (GEMV), the keys (attention)
    SUB_PART2 = 5,      // the down / out_proj stages are done (fused)
    SUB_REDUCED = 6,    // the bulk reduction is performed (fused); the split counter is taken (attention)
    SUB_PUBLISHED = 7,  // the counter is raised (fused); the merged head outputs are written (attention)
    SUB_ROUTE_STAGE = 8,  // the first router stage of thread 0's set has landed (routed phases)
    SUB_ROUTE_DOTS = 9,   // the router logits are complete (routed phases)
    SUB_PROD_ROUTED = 10, // the producer thread has seen the routing (routed phases)
    SUB_PROD_ISSUE = 11,  // the producer thread has issued the phase's first weight stage
    SUB_TOPK_START = 12,  // the top-k warp starts (routed phases)
    SUB_TOPK_RANKS = 13,  // the top-k warp has the ranks
    SUB_TOPK_DONE = 14,   // the top-k warp has the ids and weights (before it releases the producer)
    SUB_ROUTE_START = 15,  // the CTA starts routing (after the RMSNorm factor of the staged input)
};
constexpr int kSubStamps = 16;

// Shared-memory plan of the persistent kernel: a byte ring of kDecRingBytes holding up to
// kDecSlots in-flight stages of any size (so bytes in flight fill the ring whatever the phase),
// the input digits of the current phase, and attention scratch.
constexpr int kDecSlots = 16;
constexpr int kDecRingBytes = 176 * 1024;
constexpr int kDecMaxStageBytes = 72 * 1024;
constexpr int kDecDigitBytes = 24 * 1024;
constexpr int kDecAttnBytes = 20 * 1024;

// Fused MoE phase: hidden units per gate/up stage and per down stage, rows of the output per
// consumer thread (the 128 threads of a consumer set cover n_out = 2048).
constexpr int kMoeG = 8;  // measured (us/step): 16 units (69.6 KB stages) 760, 8 units 724, 4 units 814
constexpr int kConvG = 8;  // units per first-part stage of a fused short-conv phase (3 rows each)
constexpr int kMoeDU = 16;
constexpr int kMoeRows = 16;
constexpr int kMoeOut = 128 * kMoeRows;
constexpr int kMoeMaxUnits = 512;  // hidden units one CTA may own
// Copies of each accumulated vector: CTA c adds into copy c % kAccCopies (fewer same-line
// reductions contend at L2); a reader sums the copies.  A slot is [kAccCopies][n] floats, then
// the counter.
constexpr int kAccCopies = 1;

// Launch one decode step (grid = one CTA per SM).
void launch_decode_step(const PhaseDesc* prog, int n_phases, DecodeCtl* ctl, int* err, cudaStream_t s);
// Items per stage for a streamed phase (a power of two >= 4 dividing n_div when possible).
int decode_stage_items(int S, int K, int n_div, int n_total);
// Whether a fused phase of these shapes fits (input K, N units per expert, n_out outputs; S = 2
// sources per unit for an FFN, 3 for a short-conv layer).
bool decode_moe_fits(int K, int N, int n_out, int n_expert, int top_k, int S = 2);
// Whether a phase fits the persistent kernel's shared-memory plan.
bool decode_phase_fits(const PhaseDesc& p);

}  // namespace qq3
