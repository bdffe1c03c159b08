// moe_api.cu -- the lk_* C ABI (include/loki_moe.h): context, scratch buffers and the launch sequence
// of one MoE layer: router -> (dispatch) -> gate/up + SwiGLU -> down -> combine, all on the caller's
// stream, no host synchronisation.
#include <cstdio>
#include <cstring>
#include <cstdarg>
#include <string>
#include <algorithm>
#include "../../include/loki_moe.h"
#include "../../include/loki_ep.h"
#include "moe_internal.h"

using namespace lk;

struct LkMoeCtx {
    LkMoeConfig cfg;
    int device = 0, nsm = 0;
    // scratch (device)
    float* logits = nullptr; float* probs = nullptr; int* sel = nullptr; float* w = nullptr;
    int* counts = nullptr; int* offsets = nullptr; int* perm = nullptr;
    int* slot_expert = nullptr; int* slot_tok = nullptr; int* slot_out = nullptr; float* slot_w = nullptr;
    int* nslots = nullptr; int max_slots = 0;
    int8_t* hq = nullptr; float* hd = nullptr; float* y = nullptr;
    int* err = nullptr; int* tile_count = nullptr;
    int8_t* xq = nullptr; int8_t* xqn = nullptr; float* xd = nullptr;   // token 0's q8 x from the router (T == 1)
    bool xq_ready = false;            // set while a one-token forward's expert stage runs, for x == xq_src
    const float* xq_src = nullptr;
    int sh_t0 = 0, sh_n = 0;          // shared-expert token range of the next expert stage (SlotParams semantics)
    // the shared expert in the real model's formats (W->sh_fmt == LK_FMT_Q5K) runs as its own launches
    // (shared_kq.cu); the routed slot tables then carry no shared slots (rs = 0).  shgu: its fp32 gate/up rows
    int rs = 0; float* shgu = nullptr; int* shpair = nullptr;
    // its dense path for calls of >= sh_gemm_min tokens (launch_shared_gemm, tcgen05), allocated on first use
    // outside a stream capture: dequantised weights (147 MB), x and h token tiles
    int sh_gemm_min = 16; uint8_t* shw16 = nullptr; uint8_t* shx16 = nullptr; uint8_t* shh16 = nullptr;
    // batch regimes (T >= mma_min_tokens): the q8 gate/up on GEMM_NT-token slots (bt: its hi/lo activation
    // tiles), the IQ2_XXS down on tcgen05 from gemm_min_tokens (ht: its B tiles)
    int* g_expert = nullptr; int* g_tok = nullptr; int* g_out = nullptr; float* g_w = nullptr; int* g_n = nullptr; int g_max = 0;
    __half* bt = nullptr; __half* ht = nullptr; int* g_cnt = nullptr; int gemm_min_tokens = 192;
    // the mma.sync downs (IQ2_XXS below gemm_min_tokens, K-quant always): MM_NT-token slots reading the fp16
    // q8 SwiGLU rows hb
    int* m_expert = nullptr; int* m_tok = nullptr; int* m_out = nullptr; float* m_w = nullptr; int* m_n = nullptr;
    int* m_cnt = nullptr; int m_max = 0; __half* hb = nullptr; int mma_min_tokens = 48;
    // defaults from a per-layer sweep (keep 8, uniform routing): single-token dp4a matvecs fastest up to ~32
    // tokens (T=32: 1.67 ms vs 2.03 mma, 2.23 tcgen05), mma.sync from 48 (T=64: 2.65 vs 3.24 / 2.96 ms,
    // T=128: 3.26 vs 3.56 tcgen05), tcgen05 from 192 (T=256: 3.84 vs 4.13 mma; T=512: 4.31 vs 6.26)
    float* ep_x = nullptr;            // lk_ep_experts: the received rows' activations, dequantised (on first use)
    const uint8_t* ep_rows = nullptr; // lk_ep_experts on the single-token path: the rows themselves (their q8 codes)
    float* ep_shared_out = nullptr;   // lk_ep_experts: where the combine copies the shared expert's rows
    float** ydst = nullptr;           // [max_slots] lk_ep_p2p_experts: each slot's output row (the direct return)
    bool ydst_on = false;             // set while lk_ep_p2p_experts' expert kernels run (with epw: their rows wait)
    EpWait epw{};
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    char msg[256] = {0};
};

static int set_err(LkMoeCtx* c, int code, const char* fmt, ...) {
    if (c) { va_list ap; va_start(ap, fmt); vsnprintf(c->msg, sizeof(c->msg), fmt, ap); va_end(ap); }
    return code;
}

#define LK_CU(call) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) \
    return set_err(c, LK_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); } while (0)

// the shared expert's dense path: its buffers on first use; false while a stream capture is active and they
// are missing, or an allocation failed (the caller then takes the per-token kernels)
static bool ensure_shared_gemm(LkMoeCtx* c, cudaStream_t st) {
    if (c->shh16) return true;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
    const size_t T = (size_t)(c->cfg.max_tokens + 127) / 128 * 128;    // >= sh_gemm_pad(n) for every n <= max_tokens
    if (!c->shw16 && cudaMalloc((void**)&c->shw16, SH_GEMM_W16_BYTES) != cudaSuccess) { c->shw16 = nullptr; return false; }
    if (!c->shx16 && cudaMalloc((void**)&c->shx16, T * HIDDEN * 4) != cudaSuccess) { c->shx16 = nullptr; return false; }
    if (cudaMalloc((void**)&c->shh16, T * MOE_INTER * 2) != cudaSuccess) { c->shh16 = nullptr; return false; }
    return true;
}

template <class T> static cudaError_t dalloc(T** p, size_t n) { return cudaMalloc((void**)p, (n ? n : 1) * sizeof(T)); }

// event record that also becomes a graph node under stream capture (a plain record only marks a
// capture dependency there)
static cudaError_t record_event(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) return e;
    return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal) : cudaEventRecord(ev, st);
}

// tokens per matvec slot below the GEMM threshold: one.  Measured per layer (keep 8): T=2 169 vs 187 us
// (NT=2), T=8 476 vs 978 us (NT=8), T=32 1658 vs 2664 us -- the single-token kernels' cheaper inner loop
// outweighs re-reading an expert's weights for each of its (few) tokens.
static int slot_nt(int) { return 1; }

extern "C" {

const char* lk_moe_strerror(int code) {
    switch (code) {
        case LK_OK: return "ok";
        case LK_ERR_ARG: return "bad argument";
        case LK_ERR_CUDA: return "CUDA error";
        case LK_ERR_UNSUPPORTED: return "unsupported configuration";
        case LK_ERR_CAPACITY: return "token count above context capacity";
        case LK_ERR_DEVICE: return "device-side error (bounded wait expired or bad slot)";
        default: return "unknown";
    }
}

const char* lk_moe_last_error(LkMoeCtx* c) { return c ? c->msg : "null context"; }

int lk_moe_create(const LkMoeConfig* cfg, int device, LkMoeCtx** out) {
    LkMoeCtx* c = nullptr;
    if (!cfg || !out) return LK_ERR_ARG;
    *out = nullptr;
    if (cfg->n_experts < 1 || cfg->n_experts > N_EXPERTS || cfg->topk < 1 || cfg->topk > MAX_TOPK || cfg->keep < 1 || cfg->keep > cfg->topk ||
        cfg->max_tokens < 1 || !(cfg->n_group == 1 || (cfg->n_group * 32 == cfg->n_experts && cfg->topk_group >= 1 &&
        cfg->topk_group <= cfg->n_group)))
        return LK_ERR_UNSUPPORTED;
    c = new LkMoeCtx();
    c->cfg = *cfg; c->device = device;
    int prev = 0; cudaGetDevice(&prev);
    LK_CU(cudaSetDevice(device));
    c->nsm = num_sms(device);
    const int T = cfg->max_tokens, NE = cfg->n_experts, KE = cfg->keep;
    const size_t rows = (size_t)T * KE + (cfg->with_shared ? T : 0);
    c->max_slots = 0;
    for (int nt = 1; nt <= MAX_NT; nt *= 2) c->max_slots = std::max(c->max_slots, max_slots_for(T, KE, NE, nt, cfg->with_shared));
    LK_CU(dalloc(&c->logits, (size_t)T * NE)); LK_CU(dalloc(&c->probs, (size_t)T * NE));
    LK_CU(dalloc(&c->sel, (size_t)T * KE)); LK_CU(dalloc(&c->w, (size_t)T * KE));
    LK_CU(dalloc(&c->counts, NE)); LK_CU(dalloc(&c->offsets, NE + 1)); LK_CU(dalloc(&c->perm, (size_t)T * KE));
    LK_CU(dalloc(&c->slot_expert, c->max_slots)); LK_CU(dalloc(&c->slot_tok, (size_t)c->max_slots * MAX_NT));
    LK_CU(dalloc(&c->slot_out, (size_t)c->max_slots * MAX_NT)); LK_CU(dalloc(&c->slot_w, (size_t)c->max_slots * MAX_NT));
    LK_CU(dalloc(&c->nslots, 1)); LK_CU(dalloc(&c->ydst, c->max_slots));
    LK_CU(dalloc(&c->hq, rows * MOE_INTER)); LK_CU(dalloc(&c->hd, rows * (MOE_INTER / 32)));
    LK_CU(dalloc(&c->y, rows * HIDDEN));
    LK_CU(dalloc(&c->err, 1));
    LK_CU(cudaMemset(c->err, 0, sizeof(int)));
    LK_CU(dalloc(&c->xq, HIDDEN)); LK_CU(dalloc(&c->xqn, HIDDEN)); LK_CU(dalloc(&c->xd, HIDDEN / 32));
    LK_CU(dalloc(&c->tile_count, T));
    LK_CU(cudaMemset(c->tile_count, 0, (size_t)T * sizeof(int)));
    c->g_max = max_slots_for(T, KE, NE, GEMM_NT, cfg->with_shared);
    LK_CU(dalloc(&c->g_expert, c->g_max)); LK_CU(dalloc(&c->g_tok, (size_t)c->g_max * GEMM_NT));
    LK_CU(dalloc(&c->g_out, (size_t)c->g_max * GEMM_NT)); LK_CU(dalloc(&c->g_w, (size_t)c->g_max * GEMM_NT)); LK_CU(dalloc(&c->g_n, 1));
    LK_CU(dalloc(&c->bt, gate_q8_tile_halfs(c->g_max))); LK_CU(dalloc(&c->ht, down_tile_halfs(c->g_max)));
    LK_CU(dalloc(&c->g_cnt, c->g_max));
    c->m_max = max_slots_for(T, KE, NE, MM_NT, cfg->with_shared);
    LK_CU(dalloc(&c->m_expert, c->m_max)); LK_CU(dalloc(&c->m_tok, (size_t)c->m_max * MM_NT));
    LK_CU(dalloc(&c->m_out, (size_t)c->m_max * MM_NT)); LK_CU(dalloc(&c->m_w, (size_t)c->m_max * MM_NT)); LK_CU(dalloc(&c->m_n, 1));
    LK_CU(dalloc(&c->m_cnt, c->m_max));
    LK_CU(dalloc(&c->hb, rows * MOE_INTER));
    if (cfg->with_shared) {
        LK_CU(dalloc(&c->shgu, (size_t)T * 2 * MOE_INTER));
        LK_CU(dalloc(&c->shpair, (size_t)T * (MOE_INTER / 32)));
        LK_CU(cudaMemset(c->shpair, 0, (size_t)T * (MOE_INTER / 32) * sizeof(int)));
    }
    LK_CU(cudaMemset(c->y, 0, rows * HIDDEN * sizeof(float)));
    LK_CU(cudaDeviceSynchronize());
    cudaSetDevice(prev);
    *out = c;
    return LK_OK;
}

void lk_moe_destroy(LkMoeCtx* c) {
    if (!c) return;
    void* ptrs[] = { c->logits, c->probs, c->sel, c->w, c->counts, c->offsets, c->perm, c->slot_expert, c->slot_tok,
                     c->slot_out, c->slot_w, c->nslots, c->hq, c->hd, c->y, c->err, c->tile_count, c->xq, c->xqn, c->xd,
                     c->g_expert, c->g_tok, c->g_out, c->g_w, c->g_n, c->bt, c->ht, c->g_cnt,
                     c->m_expert, c->m_tok, c->m_out, c->m_w, c->m_n, c->m_cnt, c->hb, c->ep_x, c->shgu, c->shpair,
                     c->ydst };
    for (void* p : ptrs) if (p) cudaFree(p);
    void* gp[] = { c->shw16, c->shx16, c->shh16 };
    for (void* p : gp) if (p) cudaFree(p);
    delete c;
}

static int check_weights(LkMoeCtx* c, const LkMoeWeights* W, bool need_router) {
    if (!W) return set_err(c, LK_ERR_ARG, "null weights");
    if (W->down_fmt != LK_FMT_IQ2 && W->down_fmt != LK_FMT_Q2K && W->down_fmt != LK_FMT_Q3K)
        return set_err(c, LK_ERR_UNSUPPORTED, "down format %d: IQ2_XXS (4), Q2_K (5) or Q3_K (6)", W->down_fmt);
    const void* mats[] = { W->gate, W->up, W->down };
    for (const void* m : mats) if (!m || ((uintptr_t)m & 15)) return set_err(c, LK_ERR_ARG, "expert arena null or not 16-byte aligned");
    if ((W->gate_stride & 15) || (W->up_stride & 15) || (W->down_stride & 15))
        return set_err(c, LK_ERR_ARG, "expert strides must be multiples of 16 bytes");
    if (c->cfg.with_shared) {
        const void* sm[] = { W->sh_gate, W->sh_up, W->sh_down };
        for (const void* m : sm) if (!m || ((uintptr_t)m & 15)) return set_err(c, LK_ERR_ARG, "shared expert null or not 16-byte aligned");
    }
    if (W->sh_fmt != 0 && W->sh_fmt != LK_FMT_IQ2 && W->sh_fmt != LK_FMT_Q5K)
        return set_err(c, LK_ERR_UNSUPPORTED, "shared-expert format %d: IQ2_XXS (4) or Q5_K/Q6_K (3)", W->sh_fmt);
    c->rs = c->cfg.with_shared && W->sh_fmt != LK_FMT_Q5K;
    if (need_router && (!W->router_w || !W->router_bias)) return set_err(c, LK_ERR_ARG, "router weights missing");
    return LK_OK;
}

static RouterParams router_params(LkMoeCtx* c, const LkMoeWeights* W, const float* x, int T, const float* logits_override,
                                  int* sel, float* w, bool decode_slots) {
    RouterParams p{};
    p.x = x; p.T = T; p.ld_x = HIDDEN; p.W = W->router_w; p.w_f16 = W->router_w_f16;
    p.logits_override = logits_override; p.bias = W->router_bias;
    p.logits = c->logits; p.probs = c->probs; p.sel = sel; p.w = w; p.tile_count = c->tile_count;
    p.n_experts = c->cfg.n_experts; p.topk = c->cfg.topk; p.keep = c->cfg.keep; p.renorm = c->cfg.renorm;
    p.n_group = c->cfg.n_group; p.topk_group = c->cfg.topk_group; p.scale = c->cfg.scale;
    if (decode_slots) {
        p.slot_expert = c->slot_expert; p.slot_tok = c->slot_tok; p.slot_out = c->slot_out; p.slot_w = c->slot_w;
        p.nslots = c->nslots; p.with_shared = c->rs;
    }
    return p;
}

int lk_moe_route(LkMoeCtx* c, const LkMoeWeights* W, const float* x, int T, const float* logits_override,
                 int* sel, float* w, float* probs, lk_stream_t stream) {
    if (!c || !x || T < 0) return set_err(c, LK_ERR_ARG, "null argument");
    if (T == 0) return LK_OK;
    if (T > c->cfg.max_tokens) return set_err(c, LK_ERR_CAPACITY, "T=%d > capacity %d", T, c->cfg.max_tokens);
    if (!W || !W->router_w || !W->router_bias) return set_err(c, LK_ERR_ARG, "router weights missing");
    if (c->cfg.n_experts != N_EXPERTS) return set_err(c, LK_ERR_UNSUPPORTED, "the router needs a 256-expert context");
    cudaStream_t st = (cudaStream_t)stream;
    RouterParams p = router_params(c, W, x, T, logits_override, sel ? sel : c->sel, w ? w : c->w, false);
    launch_router(p, st);
    if (probs) LK_CU(cudaMemcpyAsync(probs, c->probs, (size_t)T * c->cfg.n_experts * 4, cudaMemcpyDeviceToDevice, st));
    LK_CU(cudaGetLastError());
    return LK_OK;
}

int lk_moe_dispatch(LkMoeCtx* c, const int* sel, const float* w, int T, int keep, int* counts, int* offsets, int* perm,
                    lk_stream_t stream) {
    if (!c || !sel || !w || T < 0 || keep < 1 || keep > MAX_TOPK) return set_err(c, LK_ERR_ARG, "bad argument");
    if (T > c->cfg.max_tokens || keep > c->cfg.keep) return set_err(c, LK_ERR_CAPACITY, "T=%d keep=%d above capacity", T, keep);
    SlotParams s{};
    s.sel = sel; s.w = w; s.T = T; s.keep = keep; s.n_experts = c->cfg.n_experts; s.nt = slot_nt(T);
    s.with_shared = c->cfg.with_shared;
    s.counts = counts ? counts : c->counts; s.offsets = offsets ? offsets : c->offsets; s.perm = perm ? perm : c->perm;
    s.slot_expert = c->slot_expert; s.slot_tok = c->slot_tok; s.slot_out = c->slot_out; s.slot_w = c->slot_w;
    s.nslots = c->nslots; s.max_slots = c->max_slots; s.err = c->err; s.sh_t0 = c->sh_t0; s.sh_n = c->sh_n;
    launch_build_slots(s, (cudaStream_t)stream);
    LK_CU(cudaGetLastError());
    return LK_OK;
}

// experts for routing already in c->slot_* (built by the router for T == 1, or by the dispatch kernel)
// x rows are ld_x floats apart; sel (optional) marks absent entries (negative ids) that the combine skips
static int run_experts(LkMoeCtx* c, const LkMoeWeights* W, const float* x, int ld_x, const float* resid, int T, int keep,
                       const int* sel, float* h, float* moe, int nt, cudaStream_t st) {
    ExpertParams e{};
    e.gate = (const uint8_t*)W->gate; e.up = (const uint8_t*)W->up; e.down = (const uint8_t*)W->down;
    e.gate_stride = W->gate_stride; e.up_stride = W->up_stride; e.down_stride = W->down_stride;
    e.sh_gate = (const uint8_t*)W->sh_gate; e.sh_up = (const uint8_t*)W->sh_up; e.sh_down = (const uint8_t*)W->sh_down;
    e.x = x; e.ld_x = ld_x;
    e.slot_expert = c->slot_expert; e.slot_tok = c->slot_tok; e.slot_out = c->slot_out; e.slot_w = c->slot_w; e.nslots = c->nslots;
    e.hq = c->hq; e.hd = c->hd; e.y = c->y; e.err = c->err; e.down_fmt = W->down_fmt;
    if (c->xq_ready && x == c->xq_src) { e.xq = c->xq; e.xqn = c->xqn; e.xd = c->xd; }
    e.xrows = c->ep_rows;
    if (c->ydst_on) { e.ydst = c->ydst; e.epw = c->epw; }
    if (c->ev[0]) LK_CU(record_event(c->ev[0], st));
    launch_gate_up(e, nt, c->nsm, st);
    if (c->ev[1]) LK_CU(record_event(c->ev[1], st));
    launch_down(e, nt, c->nsm, st);
    if (c->ev[2]) LK_CU(record_event(c->ev[2], st));
    if (h || moe) {                   // a separate kernel: fusing it into the down kernel's tail measured slower
        CombineParams cp{};
        cp.y = c->y; cp.resid = resid; cp.T = T; cp.keep = keep; cp.with_shared = c->cfg.with_shared; cp.shared = nullptr;
        cp.h = h; cp.moe = moe; cp.ld_out = HIDDEN; cp.sel = sel; cp.sh_t0 = c->sh_t0; cp.sh_n = c->sh_n;
        cp.shared_out = c->ep_shared_out;
        launch_combine(cp, st);
    }
    if (c->ev[3]) LK_CU(record_event(c->ev[3], st));
    LK_CU(cudaGetLastError());
    return LK_OK;
}

// the batch regimes (T >= the mma threshold): the gate/up + SwiGLU phase on tcgen05 with the reference's q8
// numerics (gate_up_q8.cu) on slots of up to GEMM_NT tokens, then the down: IQ2_XXS from the GEMM threshold on
// tcgen05 (its B tiles written by the gate/up epilogue), below it on mma.sync (MM_NT-token slots reading the
// fp16 q8 rows hb); K-quant downs on kq_mma.cu's mma.sync kernel (MM_NT-token slots, hb); then the combine
static int run_batch_path(LkMoeCtx* c, const LkMoeWeights* W, const float* x, int ld_x, const float* resid, int T, const int* sel,
                          const float* w, int keep, float* h, float* moe, cudaStream_t st) {
    const bool tc_down = W->down_fmt == LK_FMT_IQ2 && T >= c->gemm_min_tokens;
    SlotParams s{};
    s.sel = sel; s.w = w; s.T = T; s.keep = keep; s.n_experts = c->cfg.n_experts; s.nt = GEMM_NT; s.with_shared = c->rs;
    s.counts = c->counts; s.offsets = c->offsets; s.perm = c->perm;
    s.slot_expert = c->g_expert; s.slot_tok = c->g_tok; s.slot_out = c->g_out; s.slot_w = c->g_w; s.nslots = c->g_n;
    s.max_slots = c->g_max; s.err = c->err; s.sh_t0 = c->sh_t0; s.sh_n = c->sh_n;
    launch_build_slots(s, st);
    GemmParams g{};
    g.gate = (const uint8_t*)W->gate; g.up = (const uint8_t*)W->up; g.down = (const uint8_t*)W->down;
    g.gate_stride = W->gate_stride; g.up_stride = W->up_stride; g.down_stride = W->down_stride;
    g.sh_gate = (const uint8_t*)W->sh_gate; g.sh_up = (const uint8_t*)W->sh_up; g.sh_down = (const uint8_t*)W->sh_down;
    g.x = x; g.ld_x = ld_x; g.T = T;
    g.slot_expert = c->g_expert; g.slot_tok = c->g_tok; g.slot_out = c->g_out; g.slot_w = c->g_w; g.nslots = c->g_n;
    g.max_slots = c->g_max; g.slot_cnt = c->g_cnt; g.bt = c->bt; g.ht = c->ht; g.y = c->y; g.err = c->err;
    g.hb = tc_down ? nullptr : c->hb;
    if (c->ev[0]) LK_CU(record_event(c->ev[0], st));
    launch_gate_up_q8(g, c->nsm, st);
    if (c->ev[1]) LK_CU(record_event(c->ev[1], st));
    if (tc_down) {
        launch_prefill_gemm_down(g, c->nsm, st);
    } else {
        SlotParams ms = s;
        ms.nt = MM_NT; ms.slot_expert = c->m_expert; ms.slot_tok = c->m_tok; ms.slot_out = c->m_out; ms.slot_w = c->m_w;
        ms.nslots = c->m_n; ms.max_slots = c->m_max;
        launch_build_slots(ms, st);
        MmaParams m{};
        m.down = (const uint8_t*)W->down; m.down_stride = W->down_stride; m.sh_down = (const uint8_t*)W->sh_down;
        m.slot_expert = c->m_expert; m.slot_tok = c->m_tok; m.slot_out = c->m_out; m.slot_w = c->m_w; m.nslots = c->m_n;
        m.max_slots = c->m_max; m.slot_cnt = c->m_cnt; m.hb = c->hb; m.y = c->y; m.err = c->err;
        if (W->down_fmt == LK_FMT_IQ2) {
            launch_slot_mma_down(m, c->nsm, st);      // its prep pass writes slot_cnt
        } else {
            m.slot_cnt = nullptr;                     // the K-quant down counts each slot's tokens itself
            launch_kq_mma_down(m, W->down_fmt, c->nsm, st);
        }
    }
    if (c->ev[2]) LK_CU(record_event(c->ev[2], st));
    if (h || moe) {
        CombineParams cp{};
        cp.y = c->y; cp.resid = resid; cp.T = T; cp.keep = keep; cp.with_shared = c->cfg.with_shared; cp.shared = nullptr;
        cp.h = h; cp.moe = moe; cp.ld_out = HIDDEN; cp.sel = sel; cp.sh_t0 = c->sh_t0; cp.sh_n = c->sh_n;
        cp.shared_out = c->ep_shared_out;
        launch_combine(cp, st);
    }
    if (c->ev[3]) LK_CU(record_event(c->ev[3], st));
    LK_CU(cudaGetLastError());
    return LK_OK;
}

// the expert stage for routing (sel, w) [T][keep], by token count: single-token dp4a matvecs (the slot
// tables of T == 1 may already have been written by the router: slots_ready), the register-fed mma.sync
// path, or the tcgen05 GEMMs.  K-quant (Q2_K / Q3_K) downs take the dp4a matvecs below the mma threshold
// (q8 SwiGLU output, the reference's numerics); above it their gate/up is the mma.sync or (from the GEMM
// threshold) tcgen05 IQ2_XXS phase writing fp16 SwiGLU rows, and their down kq_mma.cu's mma.sync kernel.
static int run_stage(LkMoeCtx* c, const LkMoeWeights* W, const float* x, int ld_x, const float* resid, int T, const int* sel,
                     const float* w, int keep, float* h, float* moe, bool slots_ready, cudaStream_t st) {
    const bool iq2_down = W->down_fmt == LK_FMT_IQ2;
    if (c->cfg.with_shared && !c->rs) {               // the real model's shared expert: its own launches first
        SharedKqParams sp{};
        sp.gate = (const uint8_t*)W->sh_gate; sp.up = (const uint8_t*)W->sh_up; sp.down = (const uint8_t*)W->sh_down;
        sp.x = x; sp.ld_x = ld_x;
        sp.n = c->sh_n < 0 ? 0 : (c->sh_n > 0 ? c->sh_n : T); sp.t0 = c->sh_n > 0 ? c->sh_t0 : 0; sp.row0 = T * keep;
        if (c->xq_ready && x == c->xq_src) { sp.xq = c->xq; sp.xd = c->xd; }
        sp.gu = c->shgu; sp.hq = c->hq; sp.hd = c->hd; sp.pair = c->shpair; sp.y = c->y; sp.err = c->err;
        if (sp.n >= c->sh_gemm_min && ensure_shared_gemm(c, st)) {
            SharedGemmParams gp{};
            gp.gate = sp.gate; gp.up = sp.up; gp.down = sp.down; gp.x = x; gp.ld_x = ld_x; gp.t0 = sp.t0; gp.n = sp.n; gp.row0 = sp.row0;
            gp.w16 = c->shw16; gp.x16 = c->shx16; gp.h16 = c->shh16; gp.y = c->y; gp.err = c->err;
            if (launch_shared_gemm(gp, st)) LK_CU(cudaGetLastError());
        } else {
            launch_shared_kq(sp, c->nsm, st);
        }
        if (keep == 0) {                              // shared expert only (lk_ep_shared)
            if (h || moe) {
                CombineParams cp{};
                cp.y = c->y; cp.resid = resid; cp.T = T; cp.keep = 0; cp.with_shared = 1; cp.shared = nullptr;
                cp.h = h; cp.moe = moe; cp.ld_out = HIDDEN; cp.sel = nullptr; cp.sh_t0 = c->sh_t0; cp.sh_n = c->sh_n;
                launch_combine(cp, st);
            }
            LK_CU(cudaGetLastError());
            return LK_OK;
        }
    }
    if (T >= c->mma_min_tokens) return run_batch_path(c, W, x, ld_x, resid, T, sel, w, keep, h, moe, st);
    if (!slots_ready) {
        SlotParams s{};
        s.sel = sel; s.w = w; s.T = T; s.keep = keep; s.n_experts = c->cfg.n_experts; s.nt = slot_nt(T);
        s.with_shared = c->rs;
        s.counts = c->counts; s.offsets = c->offsets; s.perm = c->perm;
        s.slot_expert = c->slot_expert; s.slot_tok = c->slot_tok; s.slot_out = c->slot_out; s.slot_w = c->slot_w;
        s.nslots = c->nslots; s.max_slots = c->max_slots; s.err = c->err; s.sh_t0 = c->sh_t0; s.sh_n = c->sh_n;
        launch_build_slots(s, st);
    }
    return run_experts(c, W, x, ld_x, resid, T, keep, sel, h, moe, slot_nt(T), st);
}

int lk_moe_set_gemm_threshold(LkMoeCtx* c, int min_tokens) {
    if (!c || min_tokens < 1) return LK_ERR_ARG;
    c->gemm_min_tokens = min_tokens;
    return LK_OK;
}

int lk_moe_set_shared_gemm_threshold(LkMoeCtx* c, int min_tokens) {
    if (!c || min_tokens < 1) return LK_ERR_ARG;
    c->sh_gemm_min = min_tokens;
    return LK_OK;
}

int lk_moe_set_mma_threshold(LkMoeCtx* c, int min_tokens) {
    if (!c || min_tokens < 1) return LK_ERR_ARG;
    c->mma_min_tokens = min_tokens;
    return LK_OK;
}

int lk_moe_experts(LkMoeCtx* c, const LkMoeWeights* W, const float* x, const float* resid, int T, const int* sel,
                   const float* w, int keep, float* h, float* moe, lk_stream_t stream) {
    if (!c || !x || !sel || !w || T < 0 || keep < 1) return set_err(c, LK_ERR_ARG, "bad argument");
    if (T == 0) return LK_OK;
    int rc = check_weights(c, W, false);
    if (rc) return rc;
    if (T > c->cfg.max_tokens || keep > c->cfg.keep) return set_err(c, LK_ERR_CAPACITY, "T=%d keep=%d above capacity", T, keep);
    return run_stage(c, W, x, HIDDEN, resid, T, sel, w, keep, h, moe, false, (cudaStream_t)stream);
}

int lk_moe_forward(LkMoeCtx* c, const LkMoeWeights* W, const float* x, const float* resid, int T,
                   const float* logits_override, float* h, float* moe, int* sel, float* w, lk_stream_t stream) {
    if (!c || !x || T < 0) return set_err(c, LK_ERR_ARG, "bad argument");
    if (T == 0) return LK_OK;
    int rc = check_weights(c, W, true);
    if (rc) return rc;
    if (T > c->cfg.max_tokens) return set_err(c, LK_ERR_CAPACITY, "T=%d > capacity %d", T, c->cfg.max_tokens);
    if (c->cfg.n_experts != N_EXPERTS) return set_err(c, LK_ERR_UNSUPPORTED, "the router needs a 256-expert context");
    cudaStream_t st = (cudaStream_t)stream;
    const int keep = c->cfg.keep;
    RouterParams p = router_params(c, W, x, T, logits_override, c->sel, c->w, T == 1);
    if (T == 1) { p.xq = c->xq; p.xqn = c->xqn; p.xd = c->xd; }
    launch_router(p, st);
    c->xq_ready = T == 1; c->xq_src = x;
    rc = run_stage(c, W, x, HIDDEN, resid, T, c->sel, c->w, keep, h, moe, T == 1, st);
    c->xq_ready = false; c->xq_src = nullptr;
    if (rc) return rc;
    if (sel) LK_CU(cudaMemcpyAsync(sel, c->sel, (size_t)T * keep * 4, cudaMemcpyDeviceToDevice, st));
    if (w) LK_CU(cudaMemcpyAsync(w, c->w, (size_t)T * keep * 4, cudaMemcpyDeviceToDevice, st));
    return LK_OK;
}

// ---- expert-parallel stages that run on a context (include/loki_ep.h)
int lk_ep_experts(LkMoeCtx* c, const LkMoeWeights* W, const void* recv_rows, int R, int keep, int shared_row0,
                  int shared_rows, float* out, float* shared_out, lk_stream_t stream) {
    if (!c || !W || R < 0 || keep < 1 || (R > 0 && (!recv_rows || !out)) || (shared_rows > 0 && !shared_out))
        return set_err(c, LK_ERR_ARG, "bad argument");
    if (shared_rows < 0 || shared_row0 < 0 || shared_row0 + shared_rows > R)
        return set_err(c, LK_ERR_ARG, "shared rows [%d, +%d) outside the %d received rows", shared_row0, shared_rows, R);
    if (shared_rows > 0 && !c->cfg.with_shared) return set_err(c, LK_ERR_ARG, "shared rows need a with_shared context");
    if (R > c->cfg.max_tokens || keep > c->cfg.keep) return set_err(c, LK_ERR_CAPACITY, "R=%d keep=%d above capacity", R, keep);
    if (R == 0) return LK_OK;
    if ((uintptr_t)recv_rows & 15) return set_err(c, LK_ERR_ARG, "rows must be 16-byte aligned");
    int rc = check_weights(c, W, false);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    // the single-token path with an IQ2_XXS (or no) shared expert reads the rows' q8 codes directly; every other
    // path reads fp32 activations, the rows dequantised to q * d (their q8 is again q and d)
    const bool direct = R < c->mma_min_tokens && (c->rs || !c->cfg.with_shared);
    if (!direct && !c->ep_x) {        // the rows' fp32 activations: allocated on first use, outside a capture
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
            return set_err(c, LK_ERR_ARG, "the first lk_ep_experts call of a batch on a context must run outside a stream capture");
        LK_CU(dalloc(&c->ep_x, (size_t)c->cfg.max_tokens * HIDDEN));
    }
    // out = the routed partial sums; the shared expert runs in the same launches on the rows
    // [shared_row0, +shared_rows), and the combine writes its outputs (entry rows R*keep + j) to shared_out
    c->sh_t0 = shared_row0; c->sh_n = shared_rows > 0 ? shared_rows : -1;
    if (direct) {                     // headers and single-token slot tables in one kernel
        SlotParams sp{};
        sp.slot_expert = c->slot_expert; sp.slot_tok = c->slot_tok; sp.slot_out = c->slot_out; sp.slot_w = c->slot_w;
        sp.nslots = c->nslots; sp.max_slots = c->max_slots; sp.err = c->err; sp.with_shared = c->rs;
        sp.sh_t0 = c->sh_t0; sp.sh_n = c->sh_n;
        launch_ep_slots(recv_rows, R, keep, c->cfg.n_experts, c->sel, c->w, sp, st);
    } else {
        launch_ep_unpack(recv_rows, R, keep, c->sel, c->w, c->ep_x, st);
    }
    const float* x = direct ? nullptr : c->ep_x;
    const int ld = HIDDEN;
    c->ep_rows = direct ? (const uint8_t*)recv_rows : nullptr;
    c->ep_shared_out = shared_rows > 0 ? shared_out : nullptr;   // the combine writes them (no copy node)
    rc = run_stage(c, W, x, ld, nullptr, R, c->sel, c->w, keep, nullptr, out, direct, st);
    c->sh_t0 = 0; c->sh_n = 0; c->ep_rows = nullptr; c->ep_shared_out = nullptr;
    return rc;
}

int lk_ep_p2p_route_dispatch(LkEpMailbox* mb, LkMoeCtx* c, const LkMoeWeights* W, const float* x, int T,
                             const float* logits_override, int* sel, float* w, int* row_map, int* err, lk_stream_t stream) {
    (void)err;                                        // the router's ids are in range by construction
    if (!mb || !c || !x || !sel || !w || !row_map || T < 0) return set_err(c, LK_ERR_ARG, "null argument");
    if (T != 1) return set_err(c, LK_ERR_UNSUPPORTED, "the router's send serves one token (T=%d)", T);
    if (!W || !W->router_w || !W->router_bias) return set_err(c, LK_ERR_ARG, "router weights missing");
    if (c->cfg.n_experts != N_EXPERTS) return set_err(c, LK_ERR_UNSUPPORTED, "the router needs a 256-expert context");
    RouterParams p = router_params(c, W, x, T, logits_override, sel, w, false);
    p.xq = c->xq; p.xqn = c->xqn; p.xd = c->xd;
    if (!p2p_send_params(mb, row_map, &p.send)) return set_err(c, LK_ERR_ARG, "mailbox not connected");
    launch_router(p, (cudaStream_t)stream);
    LK_CU(cudaGetLastError());
    return LK_OK;
}

int lk_ep_p2p_experts(LkEpMailbox* mb, LkMoeCtx* c, const LkMoeWeights* W, int keep, int T, float* shared_out, int* err,
                      lk_stream_t stream) {
    if (!mb || !c || !W || keep < 1 || T < 0 || (T > 0 && !shared_out)) return set_err(c, LK_ERR_ARG, "bad argument");
    const int R = p2p_rows_count(mb), cap = p2p_cap(mb), rank = p2p_rank(mb);
    if (T > cap) return set_err(c, LK_ERR_ARG, "T=%d above the mailbox capacity %d", T, cap);
    if (R > c->cfg.max_tokens || keep > c->cfg.keep) return set_err(c, LK_ERR_CAPACITY, "R=%d keep=%d above capacity", R, keep);
    if (T > 0 && !c->cfg.with_shared) return set_err(c, LK_ERR_ARG, "shared rows need a with_shared context");
    int rc = check_weights(c, W, false);
    if (rc) return rc;
    if (!(R < c->mma_min_tokens && (c->rs || !c->cfg.with_shared)) || !p2p_direct_ok(mb))
        return set_err(c, LK_ERR_UNSUPPORTED, "the fused exchange serves the single-token path (R=%d rows)", R);
    cudaStream_t st = (cudaStream_t)stream;
    c->sh_t0 = rank * cap; c->sh_n = T > 0 ? T : -1;
    SlotParams sp{};
    sp.slot_expert = c->slot_expert; sp.slot_tok = c->slot_tok; sp.slot_out = c->slot_out; sp.slot_w = c->slot_w;
    sp.nslots = c->nslots; sp.max_slots = c->max_slots; sp.err = c->err; sp.with_shared = c->rs;
    sp.sh_t0 = c->sh_t0; sp.sh_n = c->sh_n;
    const uint8_t* rows = nullptr;
    // the gate/up kernel itself waits for the rows and builds the slot tables, each slot with its destination row:
    // the down kernel stores the routed entries' rows straight into their home ranks' mailboxes and the shared
    // rows into shared_out (no combine or copy)
    rc = p2p_rows_wait(mb, keep, c->cfg.n_experts, c->sel, c->w, sp, err, c->ydst, T > 0 ? shared_out : nullptr, &c->epw, &rows);
    if (rc == LK_OK) {
        c->ep_rows = rows;
        c->ydst_on = true;
        rc = run_experts(c, W, nullptr, HIDDEN, nullptr, R, keep, c->sel, nullptr, nullptr, 1, st);
        // the return flags: published by lk_ep_p2p_combine_entries' first CTA, or here when no combine follows
        if (rc == LK_OK && T == 0) rc = p2p_ret_flags(mb, st);
    }
    c->sh_t0 = 0; c->sh_n = 0; c->ep_rows = nullptr; c->ydst_on = false;
    return rc ? set_err(c, rc, "fused peer exchange: launch failed") : LK_OK;
}

int lk_ep_shared(LkMoeCtx* c, const LkMoeWeights* W, const float* x, const float* resid, int T, float* h_partial,
                 lk_stream_t stream) {
    if (!c || !W || T < 0 || (T > 0 && (!x || !resid || !h_partial))) return set_err(c, LK_ERR_ARG, "bad argument");
    if (!c->cfg.with_shared || !W->sh_gate || !W->sh_up || !W->sh_down)
        return set_err(c, LK_ERR_ARG, "the shared expert needs with_shared = 1 and W->sh_*");
    if (((uintptr_t)W->sh_gate | (uintptr_t)W->sh_up | (uintptr_t)W->sh_down) & 15)
        return set_err(c, LK_ERR_ARG, "shared expert matrices must be 16-byte aligned");
    if (W->down_fmt != LK_FMT_IQ2 && W->down_fmt != LK_FMT_Q2K && W->down_fmt != LK_FMT_Q3K)
        return set_err(c, LK_ERR_UNSUPPORTED, "down format %d", W->down_fmt);
    if (W->sh_fmt != 0 && W->sh_fmt != LK_FMT_IQ2 && W->sh_fmt != LK_FMT_Q5K)
        return set_err(c, LK_ERR_UNSUPPORTED, "shared-expert format %d", W->sh_fmt);
    c->rs = W->sh_fmt != LK_FMT_Q5K;
    if (T > c->cfg.max_tokens) return set_err(c, LK_ERR_CAPACITY, "T=%d > capacity %d", T, c->cfg.max_tokens);
    if (T == 0) return LK_OK;
    // keep = 0: shared-expert slots only
    return run_stage(c, W, x, HIDDEN, resid, T, nullptr, nullptr, 0, h_partial, nullptr, false, (cudaStream_t)stream);
}

const float* lk_moe_slot_outputs(LkMoeCtx* c) { return c ? c->y : nullptr; }

int lk_moe_set_events(LkMoeCtx* c, void* const* events) {
    if (!c) return LK_ERR_ARG;
    for (int i = 0; i < 4; ++i) c->ev[i] = events ? (cudaEvent_t)events[i] : nullptr;
    return LK_OK;
}

int lk_moe_get_error(LkMoeCtx* c, lk_stream_t stream) {
    if (!c) return LK_ERR_ARG;
    LK_CU(cudaStreamSynchronize((cudaStream_t)stream));
    int e = 0;
    LK_CU(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) { cudaMemset(c->err, 0, sizeof(int)); return set_err(c, LK_ERR_DEVICE, "device error code %d", e); }
    return LK_OK;
}

int lk_gen_iq2(void* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K, int64_t stride,
               lk_stream_t stream) {
    if (!dst || rows < 1 || K < QK || (K % QK) || n_exp < 1) return LK_ERR_ARG;
    launch_gen_iq2((uint8_t*)dst, seed, layer, matrix, expert0, n_exp, rows, K, stride, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_gen_weights(int fmt, void* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K, int64_t stride,
                   lk_stream_t stream) {
    if (fmt != LK_FMT_IQ2 && fmt != LK_FMT_Q2K && fmt != LK_FMT_Q3K && fmt != LK_FMT_Q5K && fmt != LK_FMT_Q6K) return LK_ERR_UNSUPPORTED;
    if (!dst || rows < 1 || K < QK || (K % QK) || n_exp < 1) return LK_ERR_ARG;
    launch_gen_weights(fmt, (uint8_t*)dst, seed, layer, matrix, expert0, n_exp, rows, K, stride, (cudaStream_t)stream);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

}  // extern "C"
