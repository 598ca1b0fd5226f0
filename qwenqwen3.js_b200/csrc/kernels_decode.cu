// kernels_decode.cu -- one persistent kernel per decode step (sm_100a).
//
// The decode step of Qwen3Engine.forward / Lfm2Engine.forward (qwen3-engine.js:115-245,
// lfm2-engine.js:228-269) is a chain of ~100 dependent phases: embedding, per layer the
// operator (short-conv or attention) and the FFN (dense, or router -> experts -> down), then
// lm_head + argmax.  Launched as separate kernels, every phase pays a launch, a DRAM ramp and
// a tail (about 3.5 us each on this part, measured), which is more than the data time of the
// whole step.  Here one grid (one CTA per SM) runs all phases:
//
//  * the producer warp of each CTA walks the whole phase list and streams the weight rows of
//    the groups this CTA owns into a ring of shared-memory slots with 1-D bulk copies.  Weights
//    never depend on activations, so it runs ahead across phase boundaries; it only stops on
//    a full ring, or before an expert gate/up phase until its own CTA has routed the token;
//  * the consumer warps run the phases in order.  There is no grid-wide barrier: activations
//    are tagged words (decode_prog.h) and a CTA waits only for the words it reads to carry the
//    tag of their producer phase; a CTA with no work in a phase skips it;
//  * the MoE router is not a phase of its own: every CTA computes the 32 router logits and
//    the top-k itself at the start of the expert gate/up phase (identical arithmetic in every
//    CTA, so every CTA routes identically), which saves a grid-wide barrier per MoE layer;
//  * a warp dots up to four rows at once, reading the activation digits of a chunk once for
//    all of them;
//  * every wait is bounded: on timeout the kernel records an error, raises an abort flag that
//    all waits poll, drains its in-flight copies (bounded) and returns.
#include "decode_prog.h"
#include "gemv2_core.cuh"

namespace qq3 {

constexpr int kDecThreads = kThreads2;  // 8 consumer warps + 1 producer warp
constexpr int kMaxRoutes = 32;          // experts the fused router handles
constexpr int kMaxStageK = 8192;        // largest K of a streamed phase (4 staging passes)
constexpr int kMaxRowsPerWarp = 8;      // rows a consumer warp dots per stage
constexpr uint32_t kProducerBackoffNs = 0;  // producer ring waits poll tightly (see slot_wait)
constexpr int kRouteWarp = 1;           // consumer warp that computes the top-k
constexpr int kStageTarget = 64 * 1024; // stage size the item count per stage aims for
// L2 prefetch, per CTA, of the rows of the phases after an MoE layer (which do not depend on
// the routing), issued while the CTA routes: DRAM is otherwise idle then
constexpr uint32_t kRoutePrefetchBytes = 0;
// Weight rows are read once per step (1.66 GB through a 126 MB L2): copy them evict-first so
// that activations, norms, K/V rows and the shared router rows stay in L2
constexpr bool kWeightsEvictFirst = true;

// bulk copy of weight rows into a ring stage
__device__ __forceinline__ void weight_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    if (kWeightsEvictFirst) bulk_g2s_hint(dst, src, bytes, bar, pol);
    else bulk_g2s(dst, src, bytes, bar);
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Loads issued where they stand: a volatile asm keeps the compiler from sinking a prefetch of
// data that does not depend on this step below a spin wait on data that does.
__device__ __forceinline__ float4 ld_early_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ld_early_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_early_f32(const float* p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// The sub-stamps of the current phase of this CTA (thread 0 only sets and reads it; null when
// the step is not traced).
__shared__ unsigned long long* s_sub;

__device__ __forceinline__ void sub_stamp(int k) {
    if (threadIdx.x == 0 && s_sub) s_sub[k] = globaltimer_ns();
}
// The same from lane 0 of any consumer warp (s_sub is published by the barrier at the phase top).
__device__ __forceinline__ void sub_stamp_lane0(int k) {
    if ((threadIdx.x & 31) == 0 && s_sub) s_sub[k] = globaltimer_ns();
}

__device__ __forceinline__ uint32_t step_tag(uint32_t epoch, int ph) { return epoch * 256u + (uint32_t)ph + 1u; }

__device__ __forceinline__ void st_tw(tword* p, float v, uint32_t tag) {
    const tword w = ((tword)tag << 32) | (tword)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ tword ld_tw(const tword* p) {
    tword w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ bool tw_is(tword w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float tw_val(tword w) { return __uint_as_float((uint32_t)w); }

// the value of *p once it carries `tag` (bounded; 0 on timeout or abort)
__device__ __forceinline__ float wait_tw(const tword* p, uint32_t tag, int* err) {
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        const tword w = ld_tw(p);
        if (tw_is(w, tag)) return tw_val(w);
        if ((it & 255u) == 255u && ld_volatile(err)) return 0.f;
    }
    set_err(err, 4);
    return 0.f;
}

// eight consecutive words once all carry `tag` (bounded)
__device__ __forceinline__ void wait_tw8(const tword* p, uint32_t tag, int* err, float (&v)[8]) {
    tword w[8];
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        bool ok = true;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            w[j] = ld_tw(p + j);
            ok = ok && tw_is(w[j], tag);
        }
        if (ok) break;
        if ((it & 255u) == 255u && ld_volatile(err)) break;
        if (it + 1 == kSpinLimit) set_err(err, 4);
    }
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = tw_val(w[j]);
}

// Bounded wait on a ring / routing mbarrier, polling tightly unless backoff_ns is given (then
// __nanosleep between polls after the first few).  Measured on the decode step: a backoff in
// the consumers cost ~1.3% of the step, a 200 ns backoff in the producer ~1.6%.
__device__ __forceinline__ bool slot_wait(uint64_t* bar, uint32_t parity, int* err, uint32_t backoff_ns = 0) {
    const uint32_t a = smem_u32(bar);
    for (uint32_t it = 0; it < kWaitPolls; ++it) {
        if (mbar_try_wait(a, parity)) return true;
        if ((it & 63u) == 63u && ld_volatile(err)) return false;
        if (backoff_ns && it >= 4) __nanosleep(backoff_ns);
    }
    set_err(err, kErrFullWait);
    return false;
}

__device__ __forceinline__ bool streamed(int type) { return type == PH_GEMV || type == PH_DOWN4 || type == PH_FUSED; }

// Bounded wait until the counter of an accumulated vector reaches n (acquire: the vector's
// reductions, published by the writers' fences before they counted, are visible afterwards).
__device__ __forceinline__ void wait_cnt(const unsigned* c, unsigned n, int* err) {
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
        if (v >= n) return;
        if ((it & 255u) == 255u && ld_volatile(err)) return;
    }
    set_err(err, 4);
}

// Count one arrival with release semantics (this thread's earlier writes, and those ordered
// before it by a CTA barrier, are visible to a reader that acquires the count).
__device__ __forceinline__ void red_release_add(unsigned* c, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(c), "r"(v) : "memory");
}
// The same as an acquire-release read-modify-write that returns the previous count.
__device__ __forceinline__ unsigned atom_acq_rel_add(unsigned* c, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(c), "r"(v) : "memory");
    return old;
}

// The hidden units [u0, u1) of the fused MoE phase this CTA owns: the U = top_k * N units of
// the routed experts (slot-major) split into nearly equal runs of whole quads.
__device__ __forceinline__ void moe_range(int U, int& u0, int& u1) {
    const uint32_t nq = (uint32_t)U >> 2;  // nq * gridDim.x < 2^32 for every phase that fits
    u0 = 4 * (int)(nq * blockIdx.x / gridDim.x);
    u1 = 4 * (int)(nq * (blockIdx.x + 1) / gridDim.x);
}

// Units of the next stage at u: at most cap, within the run, and within one expert.
__device__ __forceinline__ int moe_stage_len(int u, int u1, int N, int cap) {
    return min(min(cap, u1 - u), (u / N + 1) * N - u);
}

__device__ __forceinline__ bool dec_masked(const uint32_t* mask, int e) {
    return mask && ((mask[e >> 5] >> (e & 31)) & 1u);
}

struct DecRing {
    uint8_t* base;       // kDecRingBytes
    uint64_t* full;      // [kDecSlots]
    uint64_t* empty;     // [kDecSlots]
    uint32_t* off;       // [kDecSlots] ring offset of the stage in each descriptor
    uint32_t* charge;    // [kDecSlots] ring bytes the stage holds (its size + any skipped ring end)
};

// Routing of the current MoE layer, computed by the CTA itself (shared memory).
struct DecRoute {
    int id[4];
    int skip[4];  // the expert of slot s is masked (its rows are skipped)
    float w[4];
    float logit[kMaxRoutes];
    float prob[kMaxRoutes];  // sigmoid of the logits
    __align__(16) float sel[kMaxRoutes];  // selection scores (prob + bias; -inf past n_expert)
    int top_i[4];            // the selected experts in selection order, and their probabilities
    float top_p[4];
    uint64_t bar;  // completes once per MoE layer: the producer may read id[]
};

// Per-phase values the hot loops need, loaded once into registers (the descriptor lives in
// global memory and every asm memory clobber would otherwise force it to be re-read).
struct PhaseRegs {
    int K, S, map, n_items, N, n0, n1, G;
    int64_t stride;
    const int8_t* q[3];
    const __half* d[3];
    int e[4];     // routed expert ids (expert maps)
    bool on[4];   // source active (expert not masked)
};

__device__ __forceinline__ void load_phase(const PhaseDesc* pp, PhaseRegs& R, const DecRoute* route) {
    R.K = pp->K; R.S = pp->S; R.map = pp->map; R.n_items = pp->n_items; R.N = pp->N;
    R.n0 = pp->n0; R.n1 = pp->n1; R.stride = pp->stride; R.G = pp->G;
    for (int s = 0; s < 3; s++) { R.q[s] = pp->qs[s]; R.d[s] = pp->d[s]; }
    for (int s = 0; s < 4; s++) { R.e[s] = 0; R.on[s] = s < R.S; }
    if (route) {
        const uint32_t* mask = pp->mask;
        for (int s = 0; s < 4; s++) {
            R.e[s] = route->id[s];
            R.on[s] = !dec_masked(mask, R.e[s]);
        }
    }
}

__device__ __forceinline__ bool expert_map(int map) { return map == MK_EXPERT_PAIR || map == MK_DOWN4; }

// Element k (runtime, < 4) of a 4-array held in registers (a dynamic index would move the
// whole struct to local memory).
template <typename T>
__device__ __forceinline__ T pick4(const T (&a)[4], int k) {
    return k == 0 ? a[0] : (k == 1 ? a[1] : (k == 2 ? a[2] : a[3]));
}

// Row pointers of the group starting at item0 (registers only).
__device__ __forceinline__ void group_ptrs(const PhaseRegs& R, int item0, const int8_t* (&q)[4],
                                           const __half* (&d)[4], bool (&on)[4]) {
    const int64_t K = R.K, KS = R.K >> 5;
    switch (R.map) {
        case MK_ROWS:
            q[0] = R.q[0] + item0 * K; d[0] = R.d[0] + item0 * KS; on[0] = true;
            break;
        case MK_CONCAT3: {
            const int t = item0 >= R.n0 + R.n1 ? 2 : (item0 >= R.n0 ? 1 : 0);
            const int row = item0 - (t == 2 ? R.n0 + R.n1 : (t == 1 ? R.n0 : 0));
            q[0] = R.q[t] + row * K; d[0] = R.d[t] + row * KS; on[0] = true;
            break;
        }
        case MK_PAIR:
            q[0] = R.q[0] + item0 * K; d[0] = R.d[0] + item0 * KS;
            q[1] = R.q[1] + item0 * K; d[1] = R.d[1] + item0 * KS;
            on[0] = on[1] = true;
            break;
        case MK_STRIDE3:
            for (int s = 0; s < 3; s++) {
                const int64_t row = item0 + s * R.stride;
                q[s] = R.q[0] + row * K; d[s] = R.d[0] + row * KS; on[s] = true;
            }
            break;
        case MK_EXPERT_PAIR: {
            const int k = item0 / R.N, j0 = item0 - k * R.N;
            const int64_t row = (int64_t)pick4(R.e, k) * R.N + j0;
            q[0] = R.q[0] + row * K; d[0] = R.d[0] + row * KS;
            q[1] = R.q[1] + row * K; d[1] = R.d[1] + row * KS;
            on[0] = on[1] = pick4(R.on, k);
            break;
        }
        case MK_DOWN4:
            for (int s = 0; s < 4; s++) {
                const int64_t row = (int64_t)R.e[s] * R.N + item0;
                q[s] = R.q[0] + row * K; d[s] = R.d[0] + row * KS; on[s] = R.on[s];
            }
            break;
    }
}

__device__ __forceinline__ uint32_t qs_stride(int G, int K) { return (uint32_t)G * K; }
__device__ __forceinline__ uint32_t d_stride(int G, int K) { return round16((uint32_t)G * (K >> 4)); }
__device__ __forceinline__ uint32_t stage_bytes(int S, int G, int K) {
    return (S * (qs_stride(G, K) + d_stride(G, K)) + 127u) & ~127u;
}

// ---- producer ------------------------------------------------------------------------------

// Splits of the context used this step: at most one (kv head, split) item per CTA.
__device__ __forceinline__ int dec_attn_splits(const AttnArgs& a) {
    int n = (int)gridDim.x / a.n_kv;
    if (n > a.n_split) n = a.n_split;
    return n < 1 ? 1 : n;
}

// Positions [p0, p1) of the context that split `split` of n_split covers at length len.
__device__ __forceinline__ void dec_attn_range(int len, int n_split, int split, int& p0, int& p1) {
    int chunk = (len + n_split - 1) / n_split;
    if (chunk < 32) chunk = 32;
    p0 = split * chunk;
    p1 = min(len, p0 + chunk);
}

// Ring bookkeeping of the producer thread: stages are issued in consumption order into a byte
// ring; a stage that does not fit before the ring end starts at offset 0 and is charged the
// skipped bytes too.
struct ProdRing {
    uint32_t i = 0;         // stages issued
    uint32_t tail = 0;      // oldest stage not yet known to be released
    uint32_t head = 0;      // next free ring offset
    uint32_t inflight = 0;  // ring bytes held by stages tail..i-1

    // Reserve `need` bytes for stage i; false on a timeout or abort.
    __device__ __forceinline__ bool alloc(const DecRing& r, uint32_t need, int* err, int& slot, uint8_t*& sb) {
        const bool wrap = head + need > (uint32_t)kDecRingBytes;
        const uint32_t charge = need + (wrap ? kDecRingBytes - head : 0u);
        while (tail < i && (i - tail >= (uint32_t)kDecSlots || inflight + charge > (uint32_t)kDecRingBytes)) {
            if (!slot_wait(&r.empty[tail % kDecSlots], (tail / kDecSlots) & 1u, err, kProducerBackoffNs)) return false;
            inflight -= r.charge[tail % kDecSlots];
            ++tail;
        }
        slot = i % kDecSlots;
        const uint32_t off = wrap ? 0u : head;
        head = off + need;
        inflight += charge;
        r.charge[slot] = charge;
        r.off[slot] = off;
        sb = r.base + off;
        return true;
    }
};

// L2 prefetch of this CTA's groups of a streamed phase, up to `budget` bytes; returns the rest.
__device__ uint32_t prefetch_phase_l2(const PhaseDesc* pp, uint32_t budget) {
    PhaseRegs R;
    load_phase(pp, R, nullptr);
    const int K = R.K, S = R.S, G = R.G;
    const int n_groups = (R.n_items + G - 1) / G;
    for (int g = blockIdx.x; g < n_groups && budget > 0; g += gridDim.x) {
        const int item0 = g * G;
        const int rows = min(G, R.n_items - item0);
        const int8_t* q[4];
        const __half* d[4];
        bool on[4] = {false, false, false, false};
        group_ptrs(R, item0, q, d, on);
        const uint32_t qb = (uint32_t)rows * K, db = round16((uint32_t)rows * (K >> 4));
#pragma unroll
        for (int s = 0; s < 4; s++) {
            if (s >= S || !on[s]) continue;
            bulk_prefetch_l2(q[s], qb);
            bulk_prefetch_l2(d[s], db);
            budget = qb + db >= budget ? 0u : budget - (qb + db);
        }
    }
    return budget;
}

// Expert of slot s of a fused FFN phase, and whether its rows are skipped: the routed expert
// (masked ones skipped), or the single dense FFN "expert" 0 of a phase without a router.
__device__ __forceinline__ int ffn_expert(const PhaseDesc* pp, const DecRoute* route, int s) {
    return pp->r_qs ? route->id[s] : 0;
}
__device__ __forceinline__ bool ffn_skip(const PhaseDesc* pp, const DecRoute* route, int s) {
    return pp->r_qs && route->skip[s];
}

// First-part sources of a fused phase: the SwiGLU form (an FFN) dots a unit's gate and up rows,
// the short-conv form its B, C and x rows of in_proj (rows j, j + E, j + 2E).
__device__ __forceinline__ int fused_sources(const PhaseDesc* pp) { return pp->epi == EK_CONV ? 3 : 2; }
__device__ __forceinline__ int fused_stage_units(int S) { return S == 3 ? kConvG : kMoeG; }
__device__ __forceinline__ int64_t fused_row(const PhaseDesc* pp, int src, int e, int j) {
    return pp->epi == EK_CONV ? (int64_t)j + (int64_t)src * pp->stride : (int64_t)e * pp->N + j;
}

// The stages of this CTA's run of a fused phase, in consumption order: first the S source rows
// of its units (G units a stage, never straddling two experts), then the same units' rows of
// the transposed second matrix (down, or out_proj) with the block scales they need (kMoeDU
// units a stage).  A masked expert's stages carry no bytes.
// A routed phase passes its routing barrier: the first stage is reserved in the ring (and all the
// bookkeeping done) before the wait for the routing, so the first expert copy leaves right after it.
__device__ __forceinline__ bool fused_produce(const PhaseDesc* pp, const DecRing& r, const DecRoute* route,
                                              ProdRing& pr, uint64_t pol, int* err, unsigned long long* sub,
                                              uint64_t* route_bar, uint32_t route_parity) {
    const int K = pp->K, N = pp->N, EO = pp->n_out;
    const int S = fused_sources(pp), G = fused_stage_units(S);
    const bool conv = pp->epi == EK_CONV;
    int u0, u1;
    moe_range(pp->top_k * N, u0, u1);
    const uint32_t qsz = qs_stride(G, K), dsz = d_stride(G, K), need = stage_bytes(S, G, K);
    const int64_t KS = K >> 5;
    for (int u = u0; u < u1; ++pr.i) {
        const int n = moe_stage_len(u, u1, N, G);
        const int s = u / N, j = u - s * N;
        int slot;
        uint8_t* sb;
        if (!pr.alloc(r, need, err, slot, sb)) return false;
        if (route_bar) {
            if (!slot_wait(route_bar, route_parity, err, kProducerBackoffNs)) return false;
            route_bar = nullptr;
            if (sub) sub[SUB_PROD_ROUTED] = globaltimer_ns();
        }
        const int e = ffn_expert(pp, route, s);
        const bool on = !ffn_skip(pp, route, s);
        const uint32_t qb = (uint32_t)n * K, db = round16((uint32_t)n * (K >> 4));
        mbar_arrive_expect_tx(&r.full[slot], on ? (uint32_t)S * (qb + db) : 0u);
        if (on) {
#pragma unroll
            for (int src = 0; src < 3; src++) {
                if (src >= S) break;
                const int64_t row = fused_row(pp, src, e, j);
                const int8_t* q = conv ? pp->qs[0] : pp->qs[src];
                const __half* d = conv ? pp->d[0] : pp->d[src];
                weight_g2s(sb + src * qsz, q + row * K, qb, &r.full[slot], pol);
                weight_g2s(sb + S * qsz + src * dsz, d + row * KS, db, &r.full[slot], pol);
            }
        }
        if (sub && u == u0) sub[SUB_PROD_ISSUE] = globaltimer_ns();
        u += n;
    }
    // a CTA without units still takes this phase of the routing barrier (phases are awaited in order)
    if (route_bar && !slot_wait(route_bar, route_parity, err, kProducerBackoffNs)) return false;
    const uint32_t dq = (uint32_t)kMoeDU * EO, need2 = (dq + 4u * EO + 127u) & ~127u;
    for (int u = u0; u < u1; ++pr.i) {
        const int n = moe_stage_len(u, u1, N, kMoeDU);
        const int s = u / N, j = u - s * N;
        const int e = ffn_expert(pp, route, s);
        const bool on = !ffn_skip(pp, route, s);
        int slot;
        uint8_t* sb;
        if (!pr.alloc(r, need2, err, slot, sb)) return false;
        const int b0 = j >> 5, nb = ((j + n - 1) >> 5) - b0 + 1;  // <= 2 scale rows
        const uint32_t qb = (uint32_t)n * EO, sbytes = (uint32_t)nb * EO * 2u;
        mbar_arrive_expect_tx(&r.full[slot], on ? qb + sbytes : 0u);
        if (on) {
            weight_g2s(sb, pp->dt_qs + ((int64_t)e * N + j) * EO, qb, &r.full[slot], pol);
            weight_g2s(sb + dq, pp->dt_d + ((int64_t)e * (N >> 5) + b0) * EO, sbytes, &r.full[slot], pol);
        }
        u += n;
    }
    return true;
}

// The producer's descriptors: phase ph in pdesc[ph & 1], copied by one bulk copy completing on
// pbar[ph & 1], the copy of phase ph + 1 issued once phase ph's has landed.
__device__ __forceinline__ void pdesc_fetch(const PhaseDesc* prog, int ph, PhaseDesc* pdesc, uint64_t* pbar) {
    // the buffer was last read by this thread's generic loads (phase ph - 2): order them before
    // the async-proxy write
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&pbar[ph & 1], (uint32_t)sizeof(PhaseDesc));
    bulk_g2s(&pdesc[ph & 1], prog + ph, (uint32_t)sizeof(PhaseDesc), &pbar[ph & 1]);
}

__device__ void dec_producer(const PhaseDesc* prog, int n_phases, DecRing r, DecRoute* route, PhaseDesc* pdesc,
                             uint64_t* pbar, unsigned long long* sub, int* err) {
    ProdRing pr;
    const uint64_t pol = l2_policy_evict_first();
    uint32_t routed = 0;  // MoE layers whose routing this CTA has seen
    int desc_landed = 0;  // descriptor copies waited for (one more may be in flight)
    pdesc_fetch(prog, 0, pdesc, pbar);
    for (int ph = 0; ph < n_phases; ph++) {
        if (!slot_wait(&pbar[ph & 1], (uint32_t)(ph >> 1) & 1u, err)) goto drain;
        desc_landed = ph + 1;
        if (ph + 1 < n_phases) pdesc_fetch(prog, ph + 1, pdesc, pbar);
        const PhaseDesc* pp = &pdesc[ph & 1];
        if (!streamed(pp->type)) continue;
        const bool ex = expert_map(pp->map);
        if (pp->r_qs && (pp->map == MK_EXPERT_PAIR || pp->type == PH_FUSED)) {  // a phase with a router
            // The router rows go first, as two stages of up to 16 rows (one per consumer set).
            const int K = pp->K, ne = pp->n_expert;
            for (int h = 0; h < 2; ++h, ++pr.i) {
                int slot;
                uint8_t* sb;
                if (!pr.alloc(r, stage_bytes(1, 16, K), err, slot, sb)) goto drain;
                const int rows = max(0, min(16, ne - 16 * h));
                const uint32_t qb = (uint32_t)rows * K, db = round16((uint32_t)rows * (K >> 4));
                mbar_arrive_expect_tx(&r.full[slot], rows ? qb + db : 0u);
                if (rows) {
                    bulk_g2s(sb, pp->r_qs + (int64_t)16 * h * K, qb, &r.full[slot]);
                    bulk_g2s(sb + qs_stride(16, K), pp->r_d + (int64_t)16 * h * (K >> 5), db, &r.full[slot]);
                }
            }
            if (kRoutePrefetchBytes > 0) {
                uint32_t budget = kRoutePrefetchBytes;
                for (int ph2 = ph + 1; ph2 < n_phases && budget > 0; ph2++) {
                    const PhaseDesc* p2 = prog + ph2;
                    if (p2->type == PH_FUSED || p2->type == PH_DOWN4 || p2->map == MK_EXPERT_PAIR) break;
                    if (p2->type == PH_GEMV) budget = prefetch_phase_l2(p2, budget);
                }
            }
            // Wait for this CTA's routing (a fused phase waits inside fused_produce, after reserving
            // its first stage).  (Pulling the rows of the next phase into L2 meanwhile, from the
            // moment the phase's input is there, was measured slower: 706 -> 732 us per step; the
            // copies compete with the expert rows and the next phase's own stream.)
            if (pp->type != PH_FUSED) {
                if (!slot_wait(&route->bar, routed & 1u, err, kProducerBackoffNs)) goto drain;
                if (sub) sub[(size_t)ph * kSubStamps + SUB_PROD_ROUTED] = globaltimer_ns();
            }
            ++routed;
        }
        const uint32_t i_first = pr.i;  // the phase's first weight stage (stamped once issued)
        if (pp->type == PH_FUSED) {
            const bool rt = pp->r_qs != nullptr;
            if (!fused_produce(pp, r, route, pr, pol, err, sub ? sub + (size_t)ph * kSubStamps : nullptr,
                               rt ? &route->bar : nullptr, (routed - 1u) & 1u))
                goto drain;
            continue;
        }
        {
            PhaseRegs R;
            load_phase(pp, R, ex ? route : nullptr);
            const int K = R.K, S = R.S, G = R.G;
            const uint32_t need = stage_bytes(S, G, K), qsz = qs_stride(G, K), dsz = d_stride(G, K);
            const int n_groups = (R.n_items + G - 1) / G;
            for (int g = blockIdx.x; g < n_groups; g += gridDim.x, ++pr.i) {
                int slot;
                uint8_t* sb;
                if (!pr.alloc(r, need, err, slot, sb)) goto drain;
                const int item0 = g * G;
                const int rows = min(G, R.n_items - item0);
                const int8_t* q[4];
                const __half* d[4];
                bool on[4] = {false, false, false, false};
                group_ptrs(R, item0, q, d, on);
                const uint32_t qb = (uint32_t)rows * K, db = round16((uint32_t)rows * (K >> 4));
                uint32_t tx = 0;
#pragma unroll
                for (int s = 0; s < 4; s++)
                    if (s < S && on[s]) tx += qb + db;
                mbar_arrive_expect_tx(&r.full[slot], tx);  // release: publishes r.off[slot] too
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    if (s >= S || !on[s]) continue;
                    weight_g2s(sb + s * qsz, q[s], qb, &r.full[slot], pol);
                    weight_g2s(sb + S * qsz + s * dsz, d[s], db, &r.full[slot], pol);
                }
                if (sub && pr.i == i_first) sub[(size_t)ph * kSubStamps + SUB_PROD_ISSUE] = globaltimer_ns();
            }
        }
    }
    return;
drain:
    // abort: let every copy already issued land before the CTA exits (bounded by the poll limit,
    // not cut short by the error word, which is set by now)
    for (uint32_t j = pr.tail; j < pr.i; ++j) mbar_wait(&r.full[j % kDecSlots], (j / kDecSlots) & 1u);
    if (desc_landed < n_phases)  // the descriptor copy in flight
        mbar_wait(&pbar[desc_landed & 1], (uint32_t)(desc_landed >> 1) & 1u);
}

// ---- consumer helpers --------------------------------------------------------------------

// Where a phase reads its input: tagged words, or an accumulated vector once its counter is
// complete; optionally also the counter of an accumulated residual the phase's epilogue reads,
// and a shared-memory copy of the raw (un-normalised) input.
struct StageIn {
    const tword* x;
    uint32_t tag;
    const float* xa;
    const unsigned* cnt;
    unsigned n;
    const unsigned* rcnt;
    unsigned rn;
    float* raw;
};

__device__ __forceinline__ StageIn stage_in(const PhaseDesc& p, uint32_t epoch, long long aoff) {
    StageIn in;
    in.x = p.x;
    in.tag = step_tag(epoch, p.x_ph);
    in.xa = p.xa ? p.xa + aoff : nullptr;
    in.cnt = p.xa ? p.xa_cnt + aoff : nullptr;
    in.n = (unsigned)p.xa_n;
    in.rcnt = p.ra ? p.ra_cnt + aoff : nullptr;
    in.rn = (unsigned)p.ra_n;
    in.raw = nullptr;
    return in;
}

// Digitise an input of runtime length K <= kMaxStageK (8 elements per consumer thread per
// pass, at most 4 passes held in registers), with an optional RMSNorm (tensor.js:103-114;
// sum of squares in double as the JS does).
__device__ void dec_stage_digits(const StageIn& in, const float* __restrict__ norm_w, float eps, int K, uint4* dig,
                                 float* xsc, double* red, int* err) {
    const int t = threadIdx.x;
    float xv[4][8];
    double ss = 0.0;
    // the norm weights do not depend on the input: request them before waiting for it (they are
    // read once per step, so they usually come from DRAM)
    float4 nw[4][2];
#pragma unroll
    for (int ps = 0; ps < 4; ps++) {
        const int e0 = 8 * t + ps * 8 * kConsumerThreads;
        nw[ps][0] = nw[ps][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (norm_w && e0 < K) {
            nw[ps][0] = ld_early_f4(norm_w + e0);
            nw[ps][1] = ld_early_f4(norm_w + e0 + 4);
        }
    }
    if (in.rcnt && t == 0) wait_cnt(in.rcnt, in.rn, err);  // the barrier after staging publishes it
    if (in.xa) {
        if (t == 0) {
            wait_cnt(in.cnt, in.n, err);
            sub_stamp(SUB_INPUT);
        }
        named_bar(1, kConsumerThreads);
#pragma unroll
        for (int ps = 0; ps < 4; ps++) {
            const int e0 = 8 * t + ps * 8 * kConsumerThreads;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (e0 < K) {
#pragma unroll
                for (int c = 0; c < kAccCopies; c++) {  // the copies of the accumulated vector
                    const float4 ca = __ldcg(reinterpret_cast<const float4*>(in.xa + (size_t)c * K + e0));
                    const float4 cb = __ldcg(reinterpret_cast<const float4*>(in.xa + (size_t)c * K + e0 + 4));
                    a.x += ca.x; a.y += ca.y; a.z += ca.z; a.w += ca.w;
                    b.x += cb.x; b.y += cb.y; b.z += cb.z; b.w += cb.w;
                }
            }
            xv[ps][0] = a.x; xv[ps][1] = a.y; xv[ps][2] = a.z; xv[ps][3] = a.w;
            xv[ps][4] = b.x; xv[ps][5] = b.y; xv[ps][6] = b.z; xv[ps][7] = b.w;
        }
    } else {
#pragma unroll
        for (int ps = 0; ps < 4; ps++) {
            const int e0 = 8 * t + ps * 8 * kConsumerThreads;
            if (e0 < K) {
                wait_tw8(in.x + e0, in.tag, err, xv[ps]);
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) xv[ps][e] = 0.f;
            }
        }
        sub_stamp(SUB_INPUT);
    }
    if (in.raw) {
#pragma unroll
        for (int ps = 0; ps < 4; ps++) {
            const int e0 = 8 * t + ps * 8 * kConsumerThreads;
            if (e0 < K) {
                reinterpret_cast<float4*>(in.raw + e0)[0] = make_float4(xv[ps][0], xv[ps][1], xv[ps][2], xv[ps][3]);
                reinterpret_cast<float4*>(in.raw + e0)[1] = make_float4(xv[ps][4], xv[ps][5], xv[ps][6], xv[ps][7]);
            }
        }
    }
    if (norm_w) {
#pragma unroll
        for (int ps = 0; ps < 4; ps++)
#pragma unroll
            for (int e = 0; e < 8; e++) ss += (double)xv[ps][e] * xv[ps][e];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((t & 31) == 0) red[t >> 5] = ss;  // stage_scale() sums the warps' parts after the barrier
        // the digits are of w.x: the common factor 1/rms scales the dot products instead, so
        // the digits need not wait for the CTA-wide sum
#pragma unroll
        for (int ps = 0; ps < 4; ps++) {
            const int e0 = 8 * t + ps * 8 * kConsumerThreads;
            if (e0 < K) {
                const float4 wa = nw[ps][0], wb = nw[ps][1];
                const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
                for (int e = 0; e < 8; e++) xv[ps][e] = wv[e] * xv[ps][e];
            }
        }
    }
#pragma unroll
    for (int ps = 0; ps < 4; ps++) {
        const int e0 = 8 * t + ps * 8 * kConsumerThreads;
        if (ps * 8 * kConsumerThreads < K) digitise8(xv[ps], e0, K, dig, xsc);
    }
}

// The RMSNorm factor 1/sqrt(mean(x^2) + eps) of the staged input (tensor.js:103-114, the sum in
// double), from the warps' partial sums; valid after the barrier that follows the staging.
// Without a fused norm the scale is 1.
__device__ __forceinline__ float stage_scale(const double* red, const float* norm_w, int K, float eps) {
    if (!norm_w) return 1.0f;
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kCW; w++) tot += red[w];
    return (float)(1.0 / sqrt(tot / (double)K + (double)eps));
}

// 24 dp4a of one 32-weight Q8_0 block (w0 | w1) against its three digit planes, combined in
// fp32: (i1 + i2/254 + i3/254^2).  |i| <= 32*127*127 < 2^22, so the conversions are exact.
__device__ __forceinline__ float block_dot(const uint4 w0, const uint4 w1, const uint4 (&g)[3][2]) {
    int a1 = __dp4a((int)w0.x, (int)g[0][0].x, 0);
    int a2 = __dp4a((int)w0.x, (int)g[1][0].x, 0);
    int a3 = __dp4a((int)w0.x, (int)g[2][0].x, 0);
    a1 = __dp4a((int)w0.y, (int)g[0][0].y, a1);
    a2 = __dp4a((int)w0.y, (int)g[1][0].y, a2);
    a3 = __dp4a((int)w0.y, (int)g[2][0].y, a3);
    a1 = __dp4a((int)w0.z, (int)g[0][0].z, a1);
    a2 = __dp4a((int)w0.z, (int)g[1][0].z, a2);
    a3 = __dp4a((int)w0.z, (int)g[2][0].z, a3);
    a1 = __dp4a((int)w0.w, (int)g[0][0].w, a1);
    a2 = __dp4a((int)w0.w, (int)g[1][0].w, a2);
    a3 = __dp4a((int)w0.w, (int)g[2][0].w, a3);
    a1 = __dp4a((int)w1.x, (int)g[0][1].x, a1);
    a2 = __dp4a((int)w1.x, (int)g[1][1].x, a2);
    a3 = __dp4a((int)w1.x, (int)g[2][1].x, a3);
    a1 = __dp4a((int)w1.y, (int)g[0][1].y, a1);
    a2 = __dp4a((int)w1.y, (int)g[1][1].y, a2);
    a3 = __dp4a((int)w1.y, (int)g[2][1].y, a3);
    a1 = __dp4a((int)w1.z, (int)g[0][1].z, a1);
    a2 = __dp4a((int)w1.z, (int)g[1][1].z, a2);
    a3 = __dp4a((int)w1.z, (int)g[2][1].z, a3);
    a1 = __dp4a((int)w1.w, (int)g[0][1].w, a1);
    a2 = __dp4a((int)w1.w, (int)g[1][1].w, a2);
    a3 = __dp4a((int)w1.w, (int)g[2][1].w, a3);
    return fmaf(i2f_small(a3), 1.0f / 64516.0f, fmaf(i2f_small(a2), 1.0f / 254.0f, i2f_small(a1)));
}

// Lane partials of NR rows (in a ring slot) against the staged input.  Lane l takes the
// 32-weight blocks l, l+32, ... of every row (one float combination per block); the digits of a
// block are read once for all rows.  Every row is computed (rows past the valid ones point at
// valid shared memory and their sums are discarded), so the compiler can interleave the NR x 3
// dp4a chains.  A block is two 16-byte halves 32 bytes apart from the next lane's: lanes with
// bit 2 set read their second half first, so each quarter-warp's 16-byte loads cover all 32
// banks once (no conflict); the digits are read in the same order, so the sums are unchanged.
template <int NR>
__device__ __forceinline__ void rows_dot(const int8_t* const (&q)[NR], const __half* const (&d)[NR],
                                         const uint4* dig, const float* xsc, int nch, int pstride, float (&acc)[NR]) {
    const int lane = threadIdx.x & 31;
    const int nb = nch >> 1;
    const int h0 = (lane >> 2) & 1, h1 = h0 ^ 1;  // the half read first, then the other
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = 0.f;
#pragma unroll 1
    for (int b = lane; b < nb; b += 32) {
        uint4 g[3][2];
#pragma unroll
        for (int pl = 0; pl < 3; pl++) {
            g[pl][0] = dig[pl * pstride + 2 * b + h0];
            g[pl][1] = dig[pl * pstride + 2 * b + h1];
        }
        const float sx = xsc[b];
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const uint4* wp = reinterpret_cast<const uint4*>(q[r] + 32 * b);
            const uint4 w0 = wp[h0], w1 = wp[h1];
            const float dw = __half2float(d[r][b]);
            acc[r] = fmaf(block_dot(w0, w1, g), dw * sx, acc[r]);
        }
    }
}

// Warp sums of NR (1, 2, 4 or 8) lane values by halving: a level exchanges half of the values a
// lane still holds.  Returns the sum of row (lane >> 2) for NR = 8, (lane >> 3) for NR = 4,
// (lane >> 4) for NR = 2, row 0 for NR = 1, in every lane of that row's group.
template <int NR>
__device__ __forceinline__ float warp_reduce_rows(const float (&v)[NR]) {
    const int lane = threadIdx.x & 31;
    float k;
    if (NR == 8) {
        const bool h16 = lane & 16;
        float k4[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            k4[j] = h16 ? v[(4 + j) % NR] : v[j];
            k4[j] += __shfl_xor_sync(0xffffffffu, h16 ? v[j] : v[(4 + j) % NR], 16);
        }
        const bool h8 = lane & 8;
        float k2[2];
#pragma unroll
        for (int j = 0; j < 2; j++) {
            k2[j] = h8 ? k4[2 + j] : k4[j];
            k2[j] += __shfl_xor_sync(0xffffffffu, h8 ? k4[j] : k4[2 + j], 8);
        }
        const bool h4 = lane & 4;
        k = h4 ? k2[1] : k2[0];
        k += __shfl_xor_sync(0xffffffffu, h4 ? k2[0] : k2[1], 4);
        k += __shfl_xor_sync(0xffffffffu, k, 2);
        k += __shfl_xor_sync(0xffffffffu, k, 1);
        return k;
    }
    if (NR == 4) {
        const bool hi = lane & 16;
        float k0 = hi ? v[2 % NR] : v[0];
        float k1 = hi ? v[3 % NR] : v[1 % NR];
        const float s0 = hi ? v[0] : v[2 % NR];
        const float s1 = hi ? v[1 % NR] : v[3 % NR];
        k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        const bool b3 = lane & 8;
        k = b3 ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
    } else if (NR == 2) {
        const bool hi = lane & 16;
        k = hi ? v[1 % NR] : v[0];
        k += __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[1 % NR], 16);
        k += __shfl_xor_sync(0xffffffffu, k, 8);
    } else {
        k = v[0];
        k += __shfl_xor_sync(0xffffffffu, k, 16);
        k += __shfl_xor_sync(0xffffffffu, k, 8);
    }
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

// butterfly sums of the first n (warp-uniform) of N lane values, interleaved
template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N], int n) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < N; j++)
            if (j < n) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g * (1.0f / (1.0f + expf(-g))) * u; }

// ---- the fused router (every CTA, at the start of the expert gate/up phase) -----------------
// lfm2-engine.js:417-447: logits = W_router . norm(h); p = sigmoid(logits); top-k on p + bias
// (stable: the lower expert id wins a tie); weights = p / (sum + 1e-6).
__device__ void dec_route(const PhaseDesc& p, const DecRing& r, uint32_t& i, const uint4* dig, const float* xsc,
                          float sc, int nch, float bias_v, DecRoute* route, int* err) {
    sub_stamp(SUB_ROUTE_START);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = p.K, ne = p.n_expert;
    const int set = warp / 4, w = warp % 4;
    // the expert mask word (n_expert <= 32) does not depend on the token: request it first
    const uint32_t mword = (warp == kRouteWarp && p.mask) ? ld_early_u32(p.mask) : 0u;
    // the router rows arrive as two ring stages of 16 rows; warp w of the set dots rows 4w..4w+3
    for (int h = 0; h < 2; h++) {
        const uint32_t ih = i + h;
        if ((int)(ih % kSets) != set) continue;
        const int slot = ih % kDecSlots;
        const bool ok = slot_wait(&r.full[slot], (ih / kDecSlots) & 1u, err);
        sub_stamp(SUB_ROUTE_STAGE);
        const uint8_t* sb = r.base + r.off[slot];
        const int row0 = 16 * h + 4 * w;
        const int n_rows = ok ? max(0, min(4, ne - row0)) : 0;
        const int8_t* q[4];
        const __half* d[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            q[j] = reinterpret_cast<const int8_t*>(sb) + (size_t)(4 * w + j) * K;
            d[j] = reinterpret_cast<const __half*>(sb + qs_stride(16, K)) + (4 * w + j) * (K >> 5);
        }
        float acc[4];
        rows_dot<4>(q, d, dig, xsc, nch, nch, acc);
        const float sum = warp_reduce_rows<4>(acc) * sc;
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
        const int j = lane >> 3;
        if ((lane & 7) == 0 && j < n_rows) {
            route->logit[row0 + j] = sum;
            route->prob[row0 + j] = 1.0f / (1.0f + expf(-sum));
        }
    }
    i += 2;
    named_bar(1, kConsumerThreads);
    sub_stamp(SUB_ROUTE_DOTS);
    if (warp == kRouteWarp) {  // not warp 0: it shares a sub-partition with the producer warp
        sub_stamp_lane0(SUB_TOPK_START);
        const bool live = lane < ne;
        const float prob = live ? route->prob[lane] : 0.f;
        const float sel = live ? prob + bias_v : -INFINITY;
        // rank of this expert in the stable descending order of the selection scores (a higher
        // score first; the lower id first on a tie): 32 independent comparisons, no dependent
        // reduction chain.  The top-k are the experts of rank 0..k-1 (lfm2-engine.js:434-442);
        // the expert of rank k < 4 writes itself into slot k (ne >= 4 for a routed phase).
        // every lane reads all 32 scores back as 8 broadcast 16-byte loads (a chain of 32 shuffles
        // measured ~0.6 us)
        route->sel[lane] = sel;
        __syncwarp();
        int before[8];
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 o = reinterpret_cast<const float4*>(route->sel)[c];
            const int j = 4 * c;
            before[c] = ((o.x > sel || (o.x == sel && j < lane)) ? 1 : 0) +
                        ((o.y > sel || (o.y == sel && j + 1 < lane)) ? 1 : 0) +
                        ((o.z > sel || (o.z == sel && j + 2 < lane)) ? 1 : 0) +
                        ((o.w > sel || (o.w == sel && j + 3 < lane)) ? 1 : 0);
        }
        const int rank = ((before[0] + before[1]) + (before[2] + before[3])) +
                         ((before[4] + before[5]) + (before[6] + before[7]));
        if (live && rank < 4) {
            route->top_i[rank] = lane;
            route->top_p[rank] = prob;
        }
        __syncwarp();
        sub_stamp_lane0(SUB_TOPK_RANKS);
        if (lane < 4) {
            double sum_w = 1e-6;
#pragma unroll
            for (int k = 0; k < 4; k++) sum_w += (double)route->top_p[k];  // selection order, as the JS sums
            const double inv = 1.0 / sum_w;
            const int ik = route->top_i[lane];
            const float wk = (float)((double)route->top_p[lane] * inv);
            route->id[lane] = ik;
            route->skip[lane] = (int)((mword >> (ik & 31)) & 1u);
            route->w[lane] = wk;
            if (blockIdx.x == 0) {
                p.ridx[lane] = ik;
                p.rw[lane] = wk;
                p.rec[lane] = (float)ik;
                p.rec[4 + lane] = wk;
            }
        }
        if (blockIdx.x == 0 && live) p.rec[8 + lane] = prob;
        __syncwarp();
        sub_stamp_lane0(SUB_TOPK_DONE);
        if (lane == 0) mbar_arrive(&route->bar);  // release: the producer may read id[]
    }
    named_bar(1, kConsumerThreads);
}

// ---- mode A: one shared input, S sources per item, G = 4 IPW items per stage ------------------
// The four warps of a set share each stage: warp w takes items w IPW .. w IPW + IPW - 1, i.e.
// NR = S IPW <= 4 rows (item-major, source-minor), so its row dots and reductions overlap.
template <int S, int IPW>
__device__ __forceinline__ void consume_a(const PhaseDesc& p, const PhaseRegs& R, const DecRing& r, uint32_t& i,
                                          const uint4* dig, const float* xsc, float sc, uint32_t tag_out,
                                          uint32_t tag_res, const float* ra, unsigned long long& best_k, int* err) {
    constexpr int NR = S * IPW;
    constexpr int NRP = NR == 3 ? 4 : (NR > 4 ? 8 : NR);  // rows padded for the halving reduction
    constexpr int SH = NRP == 8 ? 2 : (NRP == 4 ? 3 : (NRP == 2 ? 4 : 5));  // lane >> SH = row of the sum
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int set = warp / 4, w = warp % 4;
    const int K = R.K, nch = K >> 4;
    constexpr int G = 4 * IPW;
    const uint32_t qsz = qs_stride(G, K), dsz = d_stride(G, K);
    const int n_groups = (R.n_items + G - 1) / G;
    const int epi = p.epi;
    const int skip = (epi == EK_ARGMAX && p.suppress) ? *p.suppress : -1;
    tword* const y = p.y;
    // the lane that finishes item j of the warp (after the reduction it holds the item's first
    // source; the other sources come from the lanes of the next row groups)
    const int row = lane >> SH;
    const bool lead = (lane & ((1 << SH) - 1)) == 0 && row < NR && row % S == 0;
    const int my_j = row / S;
    bool first = true;
    for (int g = blockIdx.x; g < n_groups; g += gridDim.x, ++i) {
        if ((int)(i % kSets) != set) continue;
        const int slot = i % kDecSlots;
        // on a timeout leave the loop but keep every later barrier of the CTA (the next
        // phase wait sees the error word and all consumer warps return together)
        if (!slot_wait(&r.full[slot], (i / kDecSlots) & 1u, err)) break;
        if (first) {
            sub_stamp(SUB_FIRST);
            first = false;
        }
        const uint8_t* sb = r.base + r.off[slot];
        const bool gon = R.map != MK_EXPERT_PAIR || pick4(R.on, (g * G) / R.N);
        const int li0 = w * IPW;
        const int n_left = R.n_items - g * G - li0;  // items of this warp that exist
        const int n_have = n_left >= IPW ? IPW : (n_left > 0 ? n_left : 0);
        const int item = g * G + li0 + my_j;
        const bool mine = lead && my_j < n_have;
        float pre[5] = {0.f, 0.f, 0.f, 0.f, 0.f};  // epilogue operands, fetched before the dots
        if (mine) {
            if (epi == EK_RESID) {
                // an accumulated residual is complete: its counter was awaited while staging
                if (ra) {
#pragma unroll
                    for (int c = 0; c < kAccCopies; c++) pre[0] += __ldcg(ra + (size_t)c * R.n_items + item);
                } else {
                    pre[0] = wait_tw(p.res + item, tag_res, err);
                }
            } else if (epi == EK_CONV) {
                pre[0] = p.state[item];
                pre[1] = p.state[p.E + item];
                pre[2] = p.conv_w[item * 3];
                pre[3] = p.conv_w[item * 3 + 1];
                pre[4] = p.conv_w[item * 3 + 2];
            }
        }
        const int8_t* q[NRP];
        const __half* d[NRP];
#pragma unroll
        for (int j = 0; j < NRP; j++) {
            const int jj = j < NR ? j : 0;
            const int li = li0 + jj / S, s = jj % S;
            q[j] = reinterpret_cast<const int8_t*>(sb + s * qsz) + (size_t)li * K;
            d[j] = reinterpret_cast<const __half*>(sb + S * qsz + s * dsz) + li * (K >> 5);
        }
        float acc[NRP];
        rows_dot<NRP>(q, d, dig, xsc, nch, nch, acc);
        const float a0 = warp_reduce_rows<NRP>(acc) * sc;
        const float a1 = S > 1 ? __shfl_down_sync(0xffffffffu, a0, 1 << SH) : 0.f;
        const float a2 = S > 2 ? __shfl_down_sync(0xffffffffu, a0, 2 << SH) : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
        if (mine) {
            switch (epi) {
                case EK_STORE: st_tw(y + item, a0, tag_out); break;
                case EK_RESID: st_tw(y + item, pre[0] + a0, tag_out); break;
                // a masked expert's outputs are written as zeros (its down rows are skipped)
                case EK_SWIGLU: st_tw(y + item, gon ? silu_mul(a0, a1) : 0.f, tag_out); break;
                case EK_CONV: {  // lfm2-engine.js:294-321
                    const float bx = a0 * a2;
                    const float co = pre[2] * pre[0] + pre[3] * pre[1] + pre[4] * bx;
                    p.state[item] = pre[1];
                    p.state[p.E + item] = bx;
                    st_tw(y + item, a1 * co, tag_out);
                    break;
                }
                case EK_ARGMAX: {
                    p.logits[item] = a0;
                    if (item != skip) {
                        const unsigned long long k = argmax_key(a0, item);
                        if (k > best_k) best_k = k;
                    }
                    break;
                }
            }
        }
    }
}

// ---- mode B: MoE down + combine + residual (4 sources with their own inputs) -----------------
// Warp (set, src) holds the digits of expert input src; per stage it dots the kG rows of its
// source, the set combines them in expert-slot order (lfm2-engine.js:459-486).
__device__ __forceinline__ void consume_b(const PhaseDesc& p, const PhaseRegs& R, const DecRing& r, uint32_t& i,
                                          const uint4* dg, const float* xsc, const DecRoute* route,
                                          float (*part)[kG][4], int* set_ok, uint32_t tag_out, uint32_t tag_res,
                                          int* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int src = warp % 4, set = warp / 4;
    const int K = R.K, nch = K >> 4;
    tword* const y = p.y;
    float wk[4];
#pragma unroll
    for (int s = 0; s < 4; s++) wk[s] = route->w[s];
    const uint32_t qsz = qs_stride(kG, K), dsz = d_stride(kG, K);
    const int n_groups = (R.n_items + kG - 1) / kG;
    for (int g = blockIdx.x; g < n_groups; g += gridDim.x, ++i) {
        if ((int)(i % 2) != set) continue;
        const int slot = i % kDecSlots;
        const int rows = min(kG, R.n_items - g * kG);
        const bool mine = src == 0 && lane < rows;
        const float yold = mine ? wait_tw(p.res + g * kG + lane, tag_res, err) : 0.f;
        // one warp of the set waits; the set follows it through a named barrier, so a
        // timeout makes the same decision in all four warps
        if (src == 0 && lane == 0) set_ok[set] = slot_wait(&r.full[slot], (i / kDecSlots) & 1u, err) ? 1 : 0;
        named_bar(2 + set, 128);
        if (!set_ok[set]) break;
        const uint8_t* sb = r.base + r.off[slot];
        const int8_t* q[kG];
        const __half* d[kG];
#pragma unroll
        for (int j = 0; j < kG; j++) {
            q[j] = reinterpret_cast<const int8_t*>(sb + src * qsz) + (size_t)j * K;
            d[j] = reinterpret_cast<const __half*>(sb + 4 * qsz + src * dsz) + j * (K >> 5);
        }
        float acc[kG];
        rows_dot<kG>(q, d, dg, xsc, nch, 4 * nch, acc);
        const float sum = warp_reduce_rows<kG>(acc);
        if ((lane & 7) == 0) part[set][lane >> 3][src] = sum;
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[slot]);
        named_bar(2 + set, 128);
        if (mine) {
            float moe = 0.f;
#pragma unroll
            for (int s = 0; s < 4; s++)
                if (R.on[s]) moe += wk[s] * part[set][lane][s];
            st_tw(y + g * kG + lane, yold + moe, tag_out);
        }
        named_bar(2 + set, 128);
    }
}

// ---- fused MoE: router, expert gate/up + SwiGLU, down and combine in one phase -------------
// lfm2-engine.js:413-487 restated as a split over the hidden units of the routed experts: the
// CTA owning units [u0, u1) computes h_u = w_slot * silu(gate_u . x) * (up_u . x) for its units,
// then its partial out[r] = sum_u h_u * down[r][u] for all n_out rows from the transposed down
// rows, and adds it to the accumulated output with a bulk reduction.  One CTA also adds the
// residual rows it owns.  The sum is the JS combine (w_k-weighted expert outputs in slot order
// plus the residual), reassociated; its rounding differs by ~1e-7 relative.

// out-row partials of the units [k0, k1) of a down stage whose scale row is dsc (one 32-unit
// block): part[r] = sum_k h_k q_k[r], then acc[r] += part[r] * d[r]
__device__ __forceinline__ void moe_down_seg(const uint8_t* q, int EO, const float* h, int k0, int k1,
                                             const __half* dsc, float (&acc)[kMoeRows]) {
    float part[kMoeRows];
#pragma unroll
    for (int j = 0; j < kMoeRows; j++) part[j] = 0.f;
    for (int k = k0; k < k1; k++) {
        const float hv = h[k];
        const uint4 w = *reinterpret_cast<const uint4*>(q + (size_t)k * EO);
        const uint32_t ww[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
            for (int b = 0; b < 4; b++) {
                // byte b + 128 in the low mantissa bits of 2^23: exact int8 -> float in two ops
                const float f = __uint_as_float(__byte_perm(ww[c], 0x4B000000u, 0x7650u + b)) - 8388736.0f;
                part[4 * c + b] = fmaf(hv, f, part[4 * c + b]);
            }
    }
    const uint4 s0 = reinterpret_cast<const uint4*>(dsc)[0], s1 = reinterpret_cast<const uint4*>(dsc)[1];
    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&sw[j]));
        acc[2 * j] = fmaf(part[2 * j], dd.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(part[2 * j + 1], dd.y, acc[2 * j + 1]);
    }
}

// First part of a fused phase: the stages of the CTA's units [u0, u1); warp w of a stage's set
// dots units IPW w .. IPW w + IPW - 1 (their S rows interleaved) and the lane holding a unit's
// first sum writes the unit's value to hbuf: w_slot * silu(gate . x) * (up . x) for an FFN
// (tensor.js:168-180), or for a short-conv channel C * (k0 s0 + k1 s1 + k2 (B . x)) with the
// conv state shifted (lfm2-engine.js:294-321).  False after a failed wait.
template <int S, int IPW>
__device__ __forceinline__ bool fused_part1(const PhaseDesc& p, const DecRing& r, uint32_t& i, const uint4* dig,
                                            const float* xsc, float sc, const DecRoute* route, int u0, int u1,
                                            float* hbuf, int* err) {
    constexpr int G = 4 * IPW, NR = S * IPW;
    constexpr int NRP = NR == 3 ? 4 : (NR > 4 ? 8 : NR);  // rows padded for the halving reduction
    constexpr int SH = NRP == 8 ? 2 : (NRP == 4 ? 3 : (NRP == 2 ? 4 : 5));  // lane >> SH = row of the sum
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int set = warp / 4, w = warp % 4;
    const int K = p.K, nch = K >> 4, N = p.N;
    const uint32_t qsz = qs_stride(G, K), dsz = d_stride(G, K);
    const int row = lane >> SH;
    const bool lead = (lane & ((1 << SH) - 1)) == 0 && row < NR && row % S == 0;
    const int my_j = w * IPW + row / S;
    bool ok = true, first = true;
    for (int u = u0; u < u1; ++i) {
        const int n = moe_stage_len(u, u1, N, G);
        const int s = u / N;
        if ((int)(i % kSets) == set && ok) {
            const int slot = i % kDecSlots;
            const bool mine = lead && my_j < n;
            const int ch = u - s * N + my_j;  // the unit within its expert (a conv channel)
            float pre[5] = {0.f, 0.f, 0.f, 0.f, 0.f};  // conv state and taps, requested before the wait
            if (S == 3 && mine) {
                pre[0] = p.state[ch];
                pre[1] = p.state[p.E + ch];
                pre[2] = p.conv_w[ch * 3];
                pre[3] = p.conv_w[ch * 3 + 1];
                pre[4] = p.conv_w[ch * 3 + 2];
            }
            ok = slot_wait(&r.full[slot], (i / kDecSlots) & 1u, err);
            if (ok && first) {
                sub_stamp(SUB_FIRST);
                first = false;
            }
            if (ok) {
                const uint8_t* sb = r.base + r.off[slot];
                const int8_t* q[NRP];
                const __half* d[NRP];
#pragma unroll
                for (int j = 0; j < NRP; j++) {
                    const int jj = j < NR ? j : 0;
                    const int li = w * IPW + jj / S, src = jj % S;
                    q[j] = reinterpret_cast<const int8_t*>(sb + src * qsz) + (size_t)li * K;
                    d[j] = reinterpret_cast<const __half*>(sb + S * qsz + src * dsz) + li * (K >> 5);
                }
                float a[NRP];
                rows_dot<NRP>(q, d, dig, xsc, nch, nch, a);
                const float a0 = warp_reduce_rows<NRP>(a) * sc;
                const float a1 = __shfl_down_sync(0xffffffffu, a0, 1 << SH);
                const float a2 = S > 2 ? __shfl_down_sync(0xffffffffu, a0, 2 << SH) : 0.f;
                __syncwarp();
                if (lane == 0) mbar_arrive(&r.empty[slot]);
                if (mine) {
                    float h;
                    if (S == 3) {
                        const float bx = a0 * a2;
                        const float co = pre[2] * pre[0] + pre[3] * pre[1] + pre[4] * bx;
                        p.state[ch] = pre[1];
                        p.state[p.E + ch] = bx;
                        h = a1 * co;
                    } else {
                        h = ffn_skip(&p, route, s) ? 0.f : silu_mul(a0, a1) * (p.r_qs ? route->w[s] : 1.0f);
                    }
                    hbuf[u - u0 + my_j] = h;
                }
            }
        }
        u += n;
    }
    return ok;
}

// scratch: raw input [kMoeOut] (written by the staging), set-1 partials [kMoeOut], h [kMoeMaxUnits]
__device__ void moe_fused(const PhaseDesc& p, const DecRing& r, uint32_t& i, const uint4* dig, const float* xsc,
                          float sc, const DecRoute* route, float* scratch, float* acc_out, unsigned* cnt, int* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int set = warp / 4;
    const int N = p.N, EO = p.n_out;
    const float* raw = scratch;
    float* comb = scratch + kMoeOut;
    float* hbuf = comb + kMoeOut;
    int u0, u1;
    moe_range(p.top_k * N, u0, u1);
    const bool ok = fused_sources(&p) == 3
                        ? fused_part1<3, kConvG / 4>(p, r, i, dig, xsc, sc, route, u0, u1, hbuf, err)
                        : fused_part1<2, kMoeG / 4>(p, r, i, dig, xsc, sc, route, u0, u1, hbuf, err);
    named_bar(1, kConsumerThreads);  // h complete
    sub_stamp(SUB_PART1);
    // down: thread tp of the stage's set accumulates out rows 16 tp .. 16 tp + 15
    const int tp = threadIdx.x & 127;
    float acc[kMoeRows];
#pragma unroll
    for (int j = 0; j < kMoeRows; j++) acc[j] = 0.f;
    {
        bool live = ok;
        const uint32_t dq = (uint32_t)kMoeDU * EO;
        for (int u = u0; u < u1; ++i) {
            const int n = moe_stage_len(u, u1, N, kMoeDU);
            const int s = u / N, j0 = u - s * N;
            if ((int)(i % kSets) == set && live) {
                const int slot = i % kDecSlots;
                live = slot_wait(&r.full[slot], (i / kDecSlots) & 1u, err);
                if (live) {
                    if (!ffn_skip(&p, route, s)) {  // a masked expert's stage holds no bytes
                        const uint8_t* sb = r.base + r.off[slot];
                        const __half* dsc = reinterpret_cast<const __half*>(sb + dq) + tp * kMoeRows;
                        const int kb = min(n, 32 - (j0 & 31));  // units in the first scale block
                        moe_down_seg(sb + tp * 16, EO, hbuf + (u - u0), 0, kb, dsc, acc);
                        if (kb < n) moe_down_seg(sb + tp * 16, EO, hbuf + (u - u0), kb, n, dsc + EO, acc);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&r.empty[slot]);
                }
            }
            u += n;
        }
    }
    sub_stamp(SUB_PART2);
    // combine the two sets, add the owned residual rows, add the CTA's vector to the output with
    // one bulk reduction (at L2; 8x fewer requests than per-thread float4 atomics, which contend
    // on the same lines from every CTA), count this CTA
    if (set == 1) {
#pragma unroll
        for (int j = 0; j < kMoeRows; j += 4)
            *reinterpret_cast<float4*>(comb + tp * kMoeRows + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    }
    named_bar(1, kConsumerThreads);
    if (set == 0) {
        const bool owner = tp % (int)gridDim.x == (int)blockIdx.x;
#pragma unroll
        for (int j = 0; j < kMoeRows; j += 4) {
            const float4 c = *reinterpret_cast<const float4*>(comb + tp * kMoeRows + j);
            float4 v = make_float4(acc[j] + c.x, acc[j + 1] + c.y, acc[j + 2] + c.z, acc[j + 3] + c.w);
            if (owner) {
                const float4 x = *reinterpret_cast<const float4*>(raw + tp * kMoeRows + j);
                v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
            }
            *reinterpret_cast<float4*>(comb + tp * kMoeRows + j) = v;
        }
        fence_proxy_async_smem();  // the bulk reduction reads comb through the async proxy
    }
    named_bar(1, kConsumerThreads);
    if (threadIdx.x == 0) {
        bulk_add_f32_s2g(acc_out + (size_t)(blockIdx.x % kAccCopies) * EO, comb, (uint32_t)EO * 4u);  // returns once performed
        sub_stamp(SUB_REDUCED);
        red_release_add(cnt, 1u);
        sub_stamp(SUB_PUBLISHED);
    }
}

// ---- attention phase (8 consumer warps per (kv head, split) item) ------------------------

template <int HD>
__device__ void dec_norm_rope(float* v, const float* __restrict__ w, float eps, const float* __restrict__ cs) {
    const int lane = threadIdx.x & 31;
    double ss = 0.0;
    for (int i = lane; i < HD; i += 32) ss += (double)v[i] * v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = (float)(1.0 / sqrt(ss / (double)HD + (double)eps));
    __syncwarp();
    for (int i = lane; i < HD; i += 32) v[i] = (w[i] * v[i]) * inv;
    __syncwarp();
    constexpr int half = HD / 2;
    for (int i = lane; i < half; i += 32) {
        const float c = cs[2 * i], s = cs[2 * i + 1];
        const float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * c - x1 * s;
        v[i + half] = x0 * s + x1 * c;
    }
    __syncwarp();
}

// One (kv head, split) item: the G query heads of kv head `kvh` over positions [p0, p1).
// Tiles of 32 positions are staged in shared memory by all consumer threads (K rows padded so
// that lane-per-position reads do not conflict); warp g < G then scores query head g with one
// position per lane, updates its online softmax and accumulates V (lane owns HD/32 dims).
// Shared layout (floats): q [8][HD] | kv [2][HD] | K tile [32][HD+4] | V tile [32][HD] |
// q norm, k norm, RoPE row [3][HD].
template <int HD>
__device__ void dec_attention(const AttnArgs& a, const tword* qkv, uint32_t tag_in, tword* out, uint32_t tag_out,
                              float* scratch, int* err) {
    constexpr int PL = HD / 32;
    constexpr int T = 32;
    constexpr int KS = HD + 4;  // padded K row stride
    const int G = a.n_head / a.n_kv;
    float* q_s = scratch;          // [8][HD]
    float* kv_s = q_s + 8 * HD;    // [2][HD]
    float* k_t = kv_s + 2 * HD;    // [T][KS]
    float* v_t = k_t + T * KS;     // [T][HD]
    float* nrm_s = v_t + T * HD;   // [3][HD]: q norm, k norm, RoPE row
    __shared__ int is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = *a.pos;
    const int len = pos + 1;
    const float scale = (float)(1.0 / sqrt((double)HD));
    const float* cs = a.rope_cs + (size_t)pos * HD;
    const int n_split = dec_attn_splits(a);
    const int n_items = a.n_kv * n_split;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int kvh = item / n_split, split = item - kvh * n_split;
        int p0, p1;
        dec_attn_range(len, n_split, split, p0, p1);
        float* kc = a.k_cache + (size_t)kvh * a.max_ctx * HD;
        float* vc = a.v_cache + (size_t)kvh * a.max_ctx * HD;
        float* part_base = a.part + (size_t)kvh * G * a.n_split * (HD + 2);
        if (p0 < p1) {
            // norm weights and the RoPE row do not depend on this step's data: request them
            // before waiting for q/k/v, store them after (HD <= 128 < consumer threads)
            float qn = 0.f, kn = 0.f, cr = 0.f;
            if (threadIdx.x < HD) {
                qn = ld_early_f32(a.q_norm + threadIdx.x);
                kn = ld_early_f32(a.k_norm + threadIdx.x);
                cr = ld_early_f32(cs + threadIdx.x);
            }
            for (int i = threadIdx.x; i < G * HD; i += kConsumerThreads)
                q_s[i] = wait_tw(qkv + (size_t)kvh * G * HD + i, tag_in, err);
            sub_stamp(SUB_INPUT);
            const bool owns = p0 <= pos && pos < p1;
            if (owns)
                for (int d = threadIdx.x; d < HD; d += kConsumerThreads) {
                    kv_s[d] = wait_tw(qkv + (size_t)a.n_head * HD + (size_t)kvh * HD + d, tag_in, err);
                    kv_s[HD + d] = wait_tw(qkv + (size_t)(a.n_head + a.n_kv) * HD + (size_t)kvh * HD + d, tag_in, err);
                }
            if (threadIdx.x < HD) {
                nrm_s[threadIdx.x] = qn;
                nrm_s[HD + threadIdx.x] = kn;
                nrm_s[2 * HD + threadIdx.x] = cr;
            }
            named_bar(1, kConsumerThreads);
            for (int g = warp; g < G; g += kCW) dec_norm_rope<HD>(q_s + g * HD, nrm_s, a.eps, nrm_s + 2 * HD);
            if (owns && warp == kCW - 1) {
                dec_norm_rope<HD>(kv_s, nrm_s + HD, a.eps, nrm_s + 2 * HD);
                for (int d = lane; d < HD; d += 32) {
                    kc[(size_t)pos * HD + d] = kv_s[d];
                    vc[(size_t)pos * HD + d] = kv_s[HD + d];
                }
            }
            named_bar(1, kConsumerThreads);
            float m = -INFINITY, l = 0.f, acc[PL];
#pragma unroll
            for (int j = 0; j < PL; j++) acc[j] = 0.f;
            for (int t0 = p0; t0 < p1; t0 += T) {
                const int n = min(T, p1 - t0);
                // rows before `pos` were written by earlier steps; the row at `pos` is in kv_s
                for (int idx = threadIdx.x; idx < n * (HD / 4); idx += kConsumerThreads) {
                    const int row = idx / (HD / 4), c = (idx % (HD / 4)) * 4;
                    const int p = t0 + row;
                    float4 k4, v4;
                    if (owns && p == pos) {
                        k4 = *reinterpret_cast<const float4*>(kv_s + c);
                        v4 = *reinterpret_cast<const float4*>(kv_s + HD + c);
                    } else {
                        k4 = __ldg(reinterpret_cast<const float4*>(kc + (size_t)p * HD + c));
                        v4 = __ldg(reinterpret_cast<const float4*>(vc + (size_t)p * HD + c));
                    }
                    *reinterpret_cast<float4*>(k_t + row * KS + c) = k4;
                    *reinterpret_cast<float4*>(v_t + row * HD + c) = v4;
                }
                named_bar(1, kConsumerThreads);
                if (warp < G) {
                    const float* qg = q_s + warp * HD;
                    float s = -INFINITY;
                    if (lane < n) {
                        const float* kr = k_t + lane * KS;
                        float dot = 0.f;
#pragma unroll
                        for (int c = 0; c < HD; c += 4) {
                            const float4 q4 = *reinterpret_cast<const float4*>(qg + c);
                            const float4 k4 = *reinterpret_cast<const float4*>(kr + c);
                            dot = fmaf(q4.x, k4.x, dot);
                            dot = fmaf(q4.y, k4.y, dot);
                            dot = fmaf(q4.z, k4.z, dot);
                            dot = fmaf(q4.w, k4.w, dot);
                        }
                        s = dot * scale;
                    }
                    const float m_new = fmaxf(m, warp_max(s));
                    const float pl = lane < n ? expf(s - m_new) : 0.f;
                    const float cf = expf(m - m_new);
                    l = l * cf + warp_sum(pl);
#pragma unroll
                    for (int j = 0; j < PL; j++) acc[j] *= cf;
                    for (int jj = 0; jj < n; jj++) {
                        const float pj = __shfl_sync(0xffffffffu, pl, jj);
#pragma unroll
                        for (int j = 0; j < PL; j++) acc[j] = fmaf(pj, v_t[jj * HD + lane * PL + j], acc[j]);
                    }
                    m = m_new;
                }
                named_bar(1, kConsumerThreads);  // the next tile reuses the buffers
            }
            sub_stamp(SUB_PART1);
            if (warp < G) {
                float* pp = part_base + ((size_t)warp * a.n_split + split) * (HD + 2);
#pragma unroll
                for (int j = 0; j < PL; j++) pp[lane * PL + j] = acc[j];
                if (lane == 0) { pp[HD] = m; pp[HD + 1] = l; }
            }
        } else {
            for (int i = threadIdx.x; i < G * HD; i += kConsumerThreads) {
                const int g = i / HD, d = i - g * HD;
                float* pp = part_base + ((size_t)g * a.n_split + split) * (HD + 2);
                pp[d] = 0.f;
                if (d == 0) { pp[HD] = -INFINITY; pp[HD + 1] = 0.f; }
            }
        }
        named_bar(1, kConsumerThreads);
        if (threadIdx.x == 0) {
            // release: the CTA's partials (ordered before by the barrier); acquire: the other
            // splits' partials, which the barrier below orders before this CTA's merge loads
            is_last = atom_acq_rel_add(a.counter + kvh, 1u) == (unsigned)n_split - 1;
            sub_stamp(SUB_REDUCED);
        }
        named_bar(1, kConsumerThreads);
        if (is_last) {
            // merge the splits; all loads of a thread are issued before the first use
            for (int i = threadIdx.x; i < G * HD; i += kConsumerThreads) {
                const int g = i / HD, d = i - g * HD;
                const float* base = part_base + (size_t)g * a.n_split * (HD + 2);
                float ms[32];
#pragma unroll
                for (int s = 0; s < 32; s++) ms[s] = s < n_split ? __ldcg(base + s * (HD + 2) + HD) : -INFINITY;
                float M = -INFINITY;
#pragma unroll
                for (int s = 0; s < 32; s++) M = fmaxf(M, ms[s]);
                float L = 0.f, A = 0.f;
#pragma unroll
                for (int s0 = 0; s0 < 32; s0 += 8) {
                    if (s0 >= n_split) break;
                    float ls[8], as[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const bool live = s0 + j < n_split;
                        ls[j] = live ? __ldcg(base + (s0 + j) * (HD + 2) + HD + 1) : 0.f;
                        as[j] = live ? __ldcg(base + (s0 + j) * (HD + 2) + d) : 0.f;
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (ms[s0 + j] == -INFINITY) continue;
                        const float f = expf(ms[s0 + j] - M);
                        L += ls[j] * f;
                        A += as[j] * f;
                    }
                }
                st_tw(out + (size_t)(kvh * G + g) * HD + d, A / L, tag_out);
            }
            if (threadIdx.x == 0) a.counter[kvh] = 0u;
            sub_stamp(SUB_PUBLISHED);
        }
        named_bar(1, kConsumerThreads);
    }
}

// ---- the kernel ----------------------------------------------------------------------------

__global__ void __launch_bounds__(kDecThreads, 1)
    k_decode(const PhaseDesc* __restrict__ prog, int n_phases, DecodeCtl* ctl, int* err) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ double red[kCW];
    __shared__ unsigned long long keys[kCW];
    __shared__ float part[2][kG][4];
    __shared__ int set_ok[2];
    __shared__ DecRoute route;
    // phase descriptors in shared memory: the consumers' current one (double-buffered, the next
    // one loaded into registers during a phase) and the producer's (double-buffered bulk copies)
    __shared__ PhaseDesc s_desc[2];
    __shared__ PhaseDesc s_pdesc[2];
    __shared__ __align__(8) uint64_t pdesc_bar[2];
    DecRing r;
    r.base = smem;
    uint8_t* dig_base = smem + kDecRingBytes;
    r.full = reinterpret_cast<uint64_t*>(dig_base + kDecDigitBytes + kDecAttnBytes);
    r.empty = r.full + kDecSlots;
    r.off = reinterpret_cast<uint32_t*>(r.empty + kDecSlots);
    r.charge = r.off + kDecSlots;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // every CTA reads the epoch before any CTA can close the step (the closing CTA is the last
    // one to finish all phases)
    const uint32_t epoch = *reinterpret_cast<const volatile unsigned int*>(&ctl->epoch);
    unsigned long long* trace = ctl->trace ? ctl->trace + (size_t)blockIdx.x * (n_phases + 1) : nullptr;
    if (trace && threadIdx.x == 0) trace[0] = globaltimer_ns();
    unsigned long long* sub = ctl->sub ? ctl->sub + (size_t)blockIdx.x * n_phases * kSubStamps : nullptr;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kDecSlots; s++) {
            mbar_init(&r.full[s], 1);
            mbar_init(&r.empty[s], kG);
        }
        mbar_init(&route.bar, 1);
        mbar_init(&pdesc_bar[0], 1);
        mbar_init(&pdesc_bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (warp == kCW) {
        if (lane == 0) dec_producer(prog, n_phases, r, &route, s_pdesc, pdesc_bar, sub, err);
        return;
    }
    // descriptor words: consumer thread t < kDescWords copies word t of the next phase's descriptor
    constexpr int kDescWords = (int)(sizeof(PhaseDesc) / 4);
    static_assert(kDescWords <= kConsumerThreads, "one descriptor word per consumer thread");
    const uint32_t* progw = reinterpret_cast<const uint32_t*>(prog);
    uint32_t desc_word = threadIdx.x < kDescWords ? __ldg(progw + threadIdx.x) : 0u;
    // this step's half of the accumulated-vector arena; zero the other half (the previous step
    // used it, the next one will: kernel boundaries order the zeroing against both)
    long long aoff = 0;
    {
        float* arena = ctl->arena;
        const long long half = ctl->arena_half;
        const int par = (int)(epoch & 1u);
        aoff = par * half;
        if (arena && half > 0) {
            float* z = arena + (1 - par) * half;
            for (long long k = (long long)blockIdx.x * kConsumerThreads + threadIdx.x; k < half;
                 k += (long long)gridDim.x * kConsumerThreads)
                z[k] = 0.f;
        }
    }
    uint32_t i = 0;  // ring position, advanced exactly as the producer advances it
    for (int ph = 0; ph < n_phases; ph++) {
        // the previous phase is over for this CTA (also when it skipped that phase)
        if (trace && threadIdx.x == 0 && ph > 0) trace[ph] = globaltimer_ns();
        if (threadIdx.x == 0) s_sub = sub ? sub + (size_t)ph * kSubStamps : nullptr;
        // publish this phase's descriptor (loaded during the previous phase) and request the next
        // one; every warp has left phase ph - 2, the last reader of this buffer
        if (threadIdx.x < kDescWords) reinterpret_cast<uint32_t*>(&s_desc[ph & 1])[threadIdx.x] = desc_word;
        named_bar(1, kConsumerThreads);
        if (threadIdx.x < kDescWords && ph + 1 < n_phases)
            desc_word = __ldg(progw + (size_t)(ph + 1) * kDescWords + threadIdx.x);
        const PhaseDesc& p = s_desc[ph & 1];
        const uint32_t tag = step_tag(epoch, ph);
        if (p.type == PH_EMBED) {
            if (blockIdx.x != 0) continue;
            int tok = p.ctl[0];
            if (tok < 0 || tok >= p.n_vocab) tok = 0;
            const int8_t* q = p.emb_qs + (int64_t)tok * p.emb_K;
            const __half* d = p.emb_d + (int64_t)tok * (p.emb_K >> 5);
            for (int e = threadIdx.x; e < p.emb_K; e += kConsumerThreads)
                st_tw(p.y + e, (float)q[e] * __half2float(d[e >> 5]), tag);
        } else if (p.type == PH_ATTN) {
            if ((int)blockIdx.x >= p.attn.n_kv * dec_attn_splits(p.attn)) continue;
            const uint32_t tin = step_tag(epoch, p.a_qkv_ph);
            // the attention phase uses the digit buffer and the attention scratch as one region
            float* scratch = reinterpret_cast<float*>(dig_base);
            if (p.attn.hd == 64) dec_attention<64>(p.attn, p.a_qkv, tin, p.a_out, tag, scratch, err);
            else dec_attention<128>(p.attn, p.a_qkv, tin, p.a_out, tag, scratch, err);
        } else if (p.type == PH_FINISH) {
            continue;  // done by the CTA that closes the step
        } else if (p.type == PH_GEMV) {
            // a CTA without groups skips the phase; the router phase runs everywhere (every CTA
            // needs the routing of its own down rows)
            if (!p.r_qs && (int)blockIdx.x >= (p.n_items + p.G - 1) / p.G) continue;
            const int K = p.K, nch = K >> 4;
            // the short-conv state and taps of this CTA's items are read once per step: pull them
            // into L2 now, before the input wait (tiny; the epilogue then hits L2)
            if (p.epi == EK_CONV) {
                const int G = p.G, n_groups = (p.n_items + G - 1) / G;
                const int mine = (n_groups - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
                for (int j = threadIdx.x; j < mine * G; j += kConsumerThreads) {
                    const int item = ((int)blockIdx.x + (j / G) * (int)gridDim.x) * G + (j % G);
                    if (item < p.n_items) {
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.state + item));
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.state + p.E + item));
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(p.conv_w + 3 * item));
                    }
                }
            }
            // the router's expert bias is read once per step: request it before the input wait
            float bias_v = 0.f;
            if (p.r_qs && warp == kRouteWarp && lane < p.n_expert && p.bias) bias_v = ld_early_f32(p.bias + lane);
            uint4* dig = reinterpret_cast<uint4*>(dig_base);
            float* xsc = reinterpret_cast<float*>(dig + 3 * nch);
            dec_stage_digits(stage_in(p, epoch, aoff), p.norm_w, p.eps, K, dig, xsc, red, err);
            named_bar(1, kConsumerThreads);
            sub_stamp(SUB_STAGED);
            const float sc = stage_scale(red, p.norm_w, K, p.eps);
            if (p.r_qs) {
                dec_route(p, r, i, dig, xsc, sc, nch, bias_v, &route, err);
                sub_stamp(SUB_ROUTED);
            }
            const float* ra = p.ra ? p.ra + aoff : nullptr;
            PhaseRegs R;
            load_phase(&p, R, expert_map(p.map) ? &route : nullptr);
            unsigned long long best_k = 0ull;
            const int ipw = R.G / 4;
            const uint32_t tres = step_tag(epoch, p.res_ph);
            if (R.S == 1 && ipw == 8) consume_a<1, 8>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 1 && ipw == 4) consume_a<1, 4>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 1 && ipw == 2) consume_a<1, 2>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 1) consume_a<1, 1>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 2 && ipw == 4) consume_a<2, 4>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 2 && ipw == 2) consume_a<2, 2>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 2) consume_a<2, 1>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else if (R.S == 3 && ipw == 2) consume_a<3, 2>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            else consume_a<3, 1>(p, R, r, i, dig, xsc, sc, tag, tres, ra, best_k, err);
            sub_stamp(SUB_PART1);
            if (p.epi == EK_ARGMAX) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best_k, o);
                    best_k = ok > best_k ? ok : best_k;
                }
                if (lane == 0) keys[warp] = best_k;
                named_bar(1, kConsumerThreads);
                if (threadIdx.x == 0) {
                    unsigned long long m = 0ull;
                    for (int ww = 0; ww < kCW; ww++) m = keys[ww] > m ? keys[ww] : m;
                    if (m) atomicMax(p.best, m);
                }
            }
        } else if (p.type == PH_FUSED) {
            // every CTA routes and owns a run of hidden units (all count into the output)
            const int K = p.K, nch = K >> 4;
            float bias_v = 0.f;
            if (warp == kRouteWarp && lane < p.n_expert && p.bias) bias_v = ld_early_f32(p.bias + lane);
            uint4* dig = reinterpret_cast<uint4*>(dig_base);
            float* xsc = reinterpret_cast<float*>(dig + 3 * nch);
            float* scratch = reinterpret_cast<float*>(dig_base + kDecDigitBytes);
            StageIn in = stage_in(p, epoch, aoff);
            in.raw = scratch;
            dec_stage_digits(in, p.norm_w, p.eps, K, dig, xsc, red, err);
            named_bar(1, kConsumerThreads);
            sub_stamp(SUB_STAGED);
            const float sc = stage_scale(red, p.norm_w, K, p.eps);
            if (p.r_qs) {
                dec_route(p, r, i, dig, xsc, sc, nch, bias_v, &route, err);
                sub_stamp(SUB_ROUTED);
            }
            moe_fused(p, r, i, dig, xsc, sc, &route, scratch, p.acc + aoff, p.acc_cnt + aoff, err);
        } else if (p.type == PH_DOWN4) {
            if ((int)blockIdx.x >= (p.n_items + kG - 1) / kG) continue;
            PhaseRegs R;
            load_phase(&p, R, &route);
            const int K = R.K, nch = K >> 4;
            // the four expert inputs are one vector of 4K (blocks never straddle two of them)
            uint4* dig = reinterpret_cast<uint4*>(dig_base);
            float* xsc_all = reinterpret_cast<float*>(dig + 3 * 4 * nch);
            dec_stage_digits(stage_in(p, epoch, aoff), nullptr, 0.f, 4 * K, dig, xsc_all, red, err);
            named_bar(1, kConsumerThreads);
            const int src = warp % 4;
            const uint4* dg = dig + src * nch;
            const float* xsc = xsc_all + src * (K >> 5);
            consume_b(p, R, r, i, dg, xsc, &route, part, set_ok, tag, step_tag(epoch, p.res_ph), err);
        }
        // the CTA's warps leave the phase together (shared digits and scratch are reused)
        named_bar(1, kConsumerThreads);
    }
    if (trace && threadIdx.x == 0) trace[n_phases] = globaltimer_ns();
    // close the step: the last CTA to get here finishes the token and advances the epoch
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(&ctl->end_ticket, 1u);
        if (t == gridDim.x - 1) {
            __threadfence();
            const PhaseDesc& f = prog[n_phases - 1];
            if (f.type == PH_FINISH) {
                const int tok = argmax_key_index(__ldcg(f.best));
                const int pos = f.ctl[1] + 1;
                f.ctl[0] = tok;
                f.ctl[1] = pos;
                f.ctl[2] = ld_volatile(err);  // read back with the token by a host-driven step
                f.trace[pos] = tok;
            }
            ctl->best = 0ull;
            ctl->end_ticket = 0u;
            __threadfence();
            ctl->epoch = epoch + 1u;
        }
    }
}

int decode_stage_items(int S, int K, int n_div, int n_total) {
    // Large stages amortise the per-stage work of the producer and of the consumer warps (up to
    // kMaxRowsPerWarp rows each).  Measured on the LFM2-8B-A1B step, this wins even where it
    // leaves CTAs without a stage in a small phase (out_proj: 64 groups of 32 rows beat 256 of
    // 8).  G divides n_div (groups must not straddle a tensor or an expert).
    (void)n_total;
    const int per_item = S * (K + K / 16);
    int G = 4;
    while (S * (2 * G) / 4 <= kMaxRowsPerWarp && G * per_item < kStageTarget && (G * 2) * per_item <= kDecMaxStageBytes)
        G *= 2;
    while (G > 4 && n_div % G) G /= 2;
    return G;
}

bool decode_moe_fits(int K, int N, int n_out, int n_expert, int top_k, int S) {
    static_assert((size_t)(2 * kMoeOut + kMoeMaxUnits) * 4 <= (size_t)kDecAttnBytes, "fused MoE scratch");
    if (K < 64 || K % 64 || n_out != kMoeOut || K != n_out) return false;  // the residual is the input
    // routed (top-4 of 4..32 experts), or a dense FFN as one expert without a router
    const bool dense = n_expert == 1 && top_k == 1;
    if (N < 32 || N % 32 || (!dense && (top_k != 4 || n_expert < 4 || n_expert > kMaxRoutes))) return false;
    const int64_t quads = (int64_t)top_k * N / 4;
    if ((quads + num_sms() - 1) / num_sms() * 4 > kMoeMaxUnits) return false;
    if (S != 2 && S != 3) return false;
    const size_t G = S == 3 ? kConvG : kMoeG;
    const size_t gu = (size_t)S * (G * K + ((G * (K >> 4) + 15) & ~(size_t)15));
    const size_t dn = (size_t)kMoeDU * n_out + 4 * (size_t)n_out;
    if (gu > (size_t)kDecMaxStageBytes || dn > (size_t)kDecMaxStageBytes) return false;
    if ((size_t)16 * K + K > (size_t)kDecMaxStageBytes) return false;  // router stages
    return (size_t)3 * (K >> 4) * 16 + (size_t)(K >> 5) * 4 <= (size_t)kDecDigitBytes;
}

bool decode_phase_fits(const PhaseDesc& p) {
    if (p.type == PH_FUSED)
        return p.dt_qs && (p.r_qs || p.n_expert == 1) &&
               (p.epi != EK_CONV || (p.state && p.conv_w && p.stride == p.N && p.E == p.N)) &&
               decode_moe_fits(p.K, p.N, p.n_out, p.n_expert, p.top_k, p.epi == EK_CONV ? 3 : 2);
    if (p.type != PH_GEMV && p.type != PH_DOWN4) {
        if (p.type == PH_ATTN) {
            const int G = p.attn.n_head / p.attn.n_kv, hd = p.attn.hd;
            const size_t need = ((size_t)8 * hd + 2 * hd + (size_t)32 * (hd + 4) + (size_t)32 * hd + 3 * hd) * 4;
            return (hd == 64 || hd == 128) && G >= 1 && G <= kCW && p.attn.n_head % p.attn.n_kv == 0 &&
                   need <= (size_t)(kDecDigitBytes + kDecAttnBytes) && p.attn.n_split <= 32;
        }
        return true;
    }
    const int K = p.K, G = p.G;
    if (K < 64 || K % 64 != 0 || K > kMaxStageK || G < 4 || G % 4 != 0) return false;
    if (p.type == PH_GEMV && (G > 32 || p.S * G / 4 > kMaxRowsPerWarp)) return false;
    if (p.S < 1 || p.S > (p.type == PH_DOWN4 ? 4 : 3)) return false;
    if (p.type == PH_DOWN4 && (G != kG || p.top_k != 4)) return false;
    const size_t qs = (size_t)G * K, d = ((size_t)G * (K >> 4) + 15) & ~(size_t)15;
    if ((size_t)p.S * (qs + d) > (size_t)kDecMaxStageBytes) return false;
    const int KT = p.type == PH_DOWN4 ? 4 * K : K;  // staged input length
    if (KT > kMaxStageK) return false;
    if ((size_t)3 * (KT >> 4) * 16 + (size_t)(KT >> 5) * 4 > (size_t)kDecDigitBytes) return false;
    if (p.map == MK_CONCAT3 && (p.n0 % G || p.n1 % G)) return false;
    if ((p.map == MK_EXPERT_PAIR || p.map == MK_DOWN4) && p.N % G) return false;
    if (p.map == MK_STRIDE3 && p.stride % G) return false;
    if (p.map == MK_EXPERT_PAIR &&
        (!p.r_qs || p.top_k != 4 || p.n_expert < 4 || p.n_expert > kMaxRoutes ||
         (size_t)16 * K + K > (size_t)kDecMaxStageBytes))  // router stages: 16 rows each
        return false;
    return true;
}

void launch_decode_step(const PhaseDesc* prog, int n_phases, DecodeCtl* ctl, int* err, cudaStream_t s) {
    const size_t smem = (size_t)kDecRingBytes + kDecDigitBytes + kDecAttnBytes + 2 * kDecSlots * 8 + 2 * kDecSlots * 4;
    if (first_use_on_device(reinterpret_cast<const void*>(k_decode)))
        QQ_CUDA_TRY(cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    static int per_sm = -1;
    if (per_sm < 0) QQ_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode, kDecThreads, smem));
    QQ_CHECK(per_sm >= 1, -4, "persistent decode kernel does not fit on an SM");
    // every CTA waits on the others, so all must be resident: a cooperative launch guarantees it
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, k_decode, prog, n_phases, ctl, err));
}

}  // namespace qq3
