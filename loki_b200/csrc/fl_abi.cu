// fl_abi.cu -- loki's fused-layer MoE entry points (include/loki_fused_moe.h) on the B200 kernels.
//
// Same call sequence and ownership rules as the reference (src/fused_layer.cu:528-620): one stream per
// context, host arrays copied before return, results in library-owned pinned mirrors, the blocking calls
// synchronise the stream.  The state fl_attn leaves for the MoE calls (ncur, ffn_inp, router outputs,
// shared-expert output; src/fused_layer.cu:506-525) is produced by the additive fl_moe_prepare.
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <vector>
#include <algorithm>
#include <functional>
#include "../../include/loki_fused_moe.h"
#include "../../include/loki_moe.h"
#include "moe_internal.h"
#include "moe_device.cuh"

using namespace lk;

namespace {
constexpr int NB = 8;                 // narrow pass rows (fl_moe's n <= 8)
constexpr int PREP_ROWS = 64;         // rows per fl_moe_prepare call (fl_attn's 8 groups of 8)
constexpr int WIDE_SLOTS = 72;        // slots per wide launch set (the reference's XH_SLOTS)
constexpr int NARROW_SLOTS = NB * MAX_TOPK;
constexpr int P8 = PREP_ROWS * MAX_TOPK;           // router outputs of a prepare launch
}

struct FLCtx {
    cudaStream_t st = nullptr; int dev = 0, nsm = 0;
    bool own_stream = true;           // false: the stream was given to lkfl_init_on_stream (an attention context's)
    // prepare / narrow state (device)
    float* ncur = nullptr; float* ffn_inp = nullptr; float* logits = nullptr; float* probs = nullptr;
    int* sel = nullptr; float* wts = nullptr; float* shared_y = nullptr; float* h = nullptr; float* moe = nullptr;
    int* ids = nullptr; float* w = nullptr; float* mo = nullptr;
    int *s_expert = nullptr, *s_tok = nullptr, *s_out = nullptr; float* s_w = nullptr; int* s_n = nullptr;
    int *counts = nullptr, *offsets = nullptr, *perm = nullptr;
    int8_t* hq = nullptr; float* hd = nullptr; float* y = nullptr;
    int* err = nullptr; int* rcount = nullptr; int* h_err = nullptr;   // device error word and its pinned mirror
    // paired buffers are allocated as one block each, so each pair crosses the bus in one 2-D copy:
    // [ncur | ffn_inp], [h | moe] (rows PREP_ROWS * HIDDEN apart), [ids | w | err] (NARROW_SLOTS apart),
    // [sel | wts] (P8 apart), and the same for their pinned host mirrors
    void* blk[4] = {}; void* hblk[4] = {};
    // the folded shared expert's rows of the last fl_moe_auto are still in y (rows n*KE..): copied into
    // shared_y only when a later call needs it (materialize_shared)
    int sh_in_y_n = 0, sh_in_y_ke = 0;
    // host mirrors (pinned)
    int* h_sel = nullptr; float* h_wts = nullptr; float* h_ncur = nullptr; float* h_fi = nullptr; float* h_h = nullptr;
    float* h_moe = nullptr; int* h_tab = nullptr; float* h_tabw = nullptr; float* h_in = nullptr;
    // device views of h_h / h_moe / h_tab / h_tabw / h_err (null where the page-locked block is not mapped): the
    // one-row fl_moe_auto graph's kernels store its host outputs there directly instead of copying them back
    float* hd_h = nullptr; float* hd_moe = nullptr; int* hd_tab = nullptr; float* hd_tabw = nullptr; int* hd_err = nullptr;
    // ... and of h_ncur / h_fi: a host-input prepare's first kernel reads the rows from there (no copy node)
    const float* hd_ncur = nullptr; const float* hd_fi = nullptr;
    // a host-input, non-wide fl_moe_prepare is deferred (its rows already in the mirrors): the next fl_moe_auto
    // that folds the shared expert runs it in its own graph, any other call first runs it alone (flush_prepare)
    bool prep_deferred = false; FLMoeW prep_w{};
    // wide pass
    int wmax = 0, wke = 0;
    float* ncur_all = nullptr; float* base_all = nullptr; float* out_all = nullptr;
    __half* whb = nullptr;            // the pass's SwiGLU outputs: fp16 of the q8 values, one row per (row, k)
    __half* wbt = nullptr;            // the q8 gate/up's activation tiles (gate_q8_tile_halfs(WIDE_SLOTS))
    // per batch parity: the mma.sync down's slots (MM_NT tokens; w_*) and the q8 gate/up's slots (GEMM_NT
    // tokens; g_*), device tables and their pinned host images (hw_tab: experts, tokens, outputs, count)
    int *w_expert[2] = {}, *w_tok[2] = {}, *w_out[2] = {}, *w_n[2] = {}, *w_cnt[2] = {}; float* w_w[2] = {};
    int *g_expert[2] = {}, *g_tok[2] = {}, *g_out[2] = {}, *g_n[2] = {}, *g_cnt[2] = {}; float* g_w[2] = {};
    int* hw_tab[2] = {}; float* hw_w[2] = {}; int* hg_tab[2] = {}; float* hg_w[2] = {};
    float* h_wh = nullptr; float* h_wmoe = nullptr;
    float* wfin = nullptr;            // [2][wmax][HIDDEN]: fl_wide_finish's h and moe, fl_wide_skip's mo and h
    cudaEvent_t wev[2] = {}, em0 = nullptr, em1 = nullptr, ep0 = nullptr, ep1 = nullptr;
    cudaEvent_t eh2d = nullptr;       // after the last copy out of the pinned row mirrors (h_ncur / h_fi)
    double ms_moe = 0, ms_prep = 0;
    // last narrow call (for fl_moe_outs)
    int last_n = 0, last_ke = 0; std::vector<int> last_ids; std::vector<float> last_w;
    int last_err = 0; int prep_n = 0;
    // the shared expert of the last fl_moe_prepare, not yet computed: fl_moe_auto folds it into its own
    // expert launches; fl_moe / fl_skip compute it first (ensure_shared)
    bool sh_pending = false; const void* sh_w[3] = {nullptr, nullptr, nullptr}; int sh_fmt = 0;
    float* sh_gu = nullptr;           // fp32 gate/up rows of the real model's shared expert (shared_kq.cu)
    int* sh_pair = nullptr;           // its gate/up pairing counters (zeroed)
    // CUDA graphs of repeated call shapes (fl_moe_prepare, fl_moe, fl_moe_auto): one replay instead of a
    // dozen launches and copies.  A shape is captured on its second occurrence (the first runs directly).
    struct GraphKey { int kind, a, b, c, d; const void* p[8]; };
    struct GraphEntry { GraphKey k; int seen; cudaGraphExec_t exec; };
    std::vector<GraphEntry> graphs; bool use_graphs = true;
};
constexpr size_t FL_MAX_GRAPHS = 1024;

void impl_fl_free(FLCtx* c);
static void flush_prepare_any(FLCtx* c);          // a deferred fl_moe_prepare runs now (defined with the prepare)

static int fl_fail(FLCtx* c, int code, const char* what, cudaError_t e = cudaSuccess) {
    std::fprintf(stderr, "[loki_moe] %s%s%s\n", what, e != cudaSuccess ? ": " : "", e != cudaSuccess ? cudaGetErrorString(e) : "");
    if (c && !c->last_err) c->last_err = code;
    return code;
}
#define FLCK(call) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) { fl_fail(c, LK_ERR_CUDA, #call, e_); return; } } while (0)
#define FLCKR(call, r) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) { fl_fail(c, LK_ERR_CUDA, #call, e_); return r; } } while (0)

template <class T> static cudaError_t dz(T** p, size_t n) {
    cudaError_t e = cudaMalloc((void**)p, (n ? n : 1) * sizeof(T));
    if (e == cudaSuccess) e = cudaMemset(*p, 0, (n ? n : 1) * sizeof(T));
    return e;
}
template <class T> static cudaError_t hz(T** p, size_t n) {
    cudaError_t e = cudaHostAlloc((void**)p, (n ? n : 1) * sizeof(T), cudaHostAllocDefault);
    if (e == cudaSuccess) std::memset(*p, 0, (n ? n : 1) * sizeof(T));
    return e;
}

// tokens per expert slot: one.  The single-token kernels' cheaper inner loop outruns the multi-token ones
// at every narrow size (the device API's sweep: T=2 169 vs 187 us per layer, T=8 476 vs 978 us)
static int nt_for(int) { return 1; }

// rows [0, n) of two row-major buffers `pitch` bytes apart, in one copy
static cudaError_t copy_pair(void* dst, const void* src, size_t pitch, size_t bytes, cudaMemcpyKind kind, cudaStream_t st) {
    return cudaMemcpy2DAsync(dst, pitch, src, pitch, bytes, 2, kind, st);
}

// the device error word rides with a blocking call's result copies: queue_err before the stream
// synchronisation, check_dev after it (no separate synchronous copy per call)
static void queue_err(FLCtx* c) {
    if (cudaMemcpyAsync(c->h_err, c->err, 4, cudaMemcpyDeviceToHost, c->st) != cudaSuccess) fl_fail(c, LK_ERR_CUDA, "error-word copy");
}
static void check_dev(FLCtx* c) {
    if (*c->h_err) {
        *c->h_err = 0;
        cudaMemsetAsync(c->err, 0, 4, c->st);
        fl_fail(c, LK_ERR_DEVICE, "device-side error recorded by a kernel");
    }
}

static bool down_fmt_ok(int f) { return f == FL_IQ2 || f == FL_Q2K || f == FL_Q3K; }

static ExpertParams expert_params(FLCtx* c, const void* gate, const void* up, const void* down, int64_t sg, int64_t sd,
                                  const float* x, int* se, int* stok, int* sout, float* sw, int* sn,
                                  int8_t* hq, float* hd, float* y) {
    ExpertParams e{};
    e.gate = (const uint8_t*)gate; e.up = (const uint8_t*)up; e.down = (const uint8_t*)down;
    e.gate_stride = sg; e.up_stride = sg; e.down_stride = sd;
    e.x = x; e.ld_x = HIDDEN; e.slot_expert = se; e.slot_tok = stok; e.slot_out = sout; e.slot_w = sw; e.nslots = sn;
    e.hq = hq; e.hd = hd; e.y = y; e.err = c->err;
    return e;
}


// ext: run on the caller's stream (not owned) instead of a stream of the context's own
FLCtx* impl_fl_init(int kvp, int sc_cap, cudaStream_t ext = nullptr) {
    (void)kvp; (void)sc_cap;          // attention-side sizes: not used by the MoE path
    FLCtx* c = new FLCtx();
    c->own_stream = ext == nullptr;
    if (ext) c->st = ext;
    cudaGetDevice(&c->dev);
    c->nsm = num_sms(c->dev);
    const size_t R = (size_t)PREP_ROWS * HIDDEN;
    // hq / y rows of a narrow launch (n*KE routed + n shared entries) or a prepare launch
    const size_t rows = (size_t)std::max(NARROW_SLOTS + NB, PREP_ROWS);
    const int ms = max_slots_for(PREP_ROWS, MAX_TOPK, N_EXPERTS, 1, 1);
    float *io = nullptr, *ho = nullptr, *h_io = nullptr, *h_ho = nullptr;
    int *iwe = nullptr, *sw = nullptr, *h_iwe = nullptr, *h_sw = nullptr;
    bool ok =
        (ext || cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) == cudaSuccess) &&
        dz(&io, 2 * R) == cudaSuccess && dz(&ho, 2 * R) == cudaSuccess && dz(&iwe, 3 * NARROW_SLOTS) == cudaSuccess &&
        dz(&sw, 2 * P8) == cudaSuccess && hz(&h_io, 2 * R) == cudaSuccess && hz(&h_ho, 2 * R) == cudaSuccess &&
        hz(&h_iwe, 3 * NARROW_SLOTS) == cudaSuccess && hz(&h_sw, 2 * P8) == cudaSuccess &&
        dz(&c->logits, PREP_ROWS * N_EXPERTS) == cudaSuccess &&
        dz(&c->probs, PREP_ROWS * N_EXPERTS) == cudaSuccess && dz(&c->shared_y, R) == cudaSuccess &&
        dz(&c->sh_gu, (size_t)PREP_ROWS * 2 * MOE_INTER) == cudaSuccess && dz(&c->sh_pair, (size_t)PREP_ROWS * (MOE_INTER / 32)) == cudaSuccess &&
        dz(&c->mo, R) == cudaSuccess &&
        dz(&c->s_expert, ms) == cudaSuccess && dz(&c->s_tok, (size_t)ms * MAX_NT) == cudaSuccess &&
        dz(&c->s_out, (size_t)ms * MAX_NT) == cudaSuccess && dz(&c->s_w, (size_t)ms * MAX_NT) == cudaSuccess && dz(&c->s_n, 1) == cudaSuccess &&
        dz(&c->counts, N_EXPERTS) == cudaSuccess && dz(&c->offsets, N_EXPERTS + 1) == cudaSuccess && dz(&c->perm, NB * MAX_TOPK) == cudaSuccess &&
        dz(&c->hq, rows * MOE_INTER) == cudaSuccess && dz(&c->hd, rows * (MOE_INTER / 32)) == cudaSuccess &&
        dz(&c->y, rows * HIDDEN) == cudaSuccess &&
        dz(&c->rcount, PREP_ROWS) == cudaSuccess && hz(&c->h_in, R) == cudaSuccess &&
        cudaEventCreate(&c->em0) == cudaSuccess && cudaEventCreate(&c->em1) == cudaSuccess &&
        cudaEventCreate(&c->ep0) == cudaSuccess && cudaEventCreate(&c->ep1) == cudaSuccess &&
        cudaEventCreateWithFlags(&c->eh2d, cudaEventDisableTiming) == cudaSuccess;
    c->blk[0] = io; c->blk[1] = ho; c->blk[2] = iwe; c->blk[3] = sw;
    c->hblk[0] = h_io; c->hblk[1] = h_ho; c->hblk[2] = h_iwe; c->hblk[3] = h_sw;
    if (!ok) { fl_fail(c, LK_ERR_CUDA, "fl_init: allocation failed", cudaGetLastError()); impl_fl_free(c); return nullptr; }
    c->ncur = io; c->ffn_inp = io + R; c->h = ho; c->moe = ho + R;
    c->ids = iwe; c->w = (float*)(iwe + NARROW_SLOTS); c->err = iwe + 2 * NARROW_SLOTS;
    c->sel = sw; c->wts = (float*)(sw + P8);
    c->h_ncur = h_io; c->h_fi = h_io + R; c->h_h = h_ho; c->h_moe = h_ho + R;
    c->h_tab = h_iwe; c->h_tabw = (float*)(h_iwe + NARROW_SLOTS); c->h_err = h_iwe + 2 * NARROW_SLOTS;
    c->h_sel = h_sw; c->h_wts = (float*)(h_sw + P8);
    float* dho = nullptr; int* diwe = nullptr; float* dio = nullptr;
    if (cudaHostGetDevicePointer((void**)&dho, h_ho, 0) == cudaSuccess && cudaHostGetDevicePointer((void**)&diwe, h_iwe, 0) == cudaSuccess &&
        cudaHostGetDevicePointer((void**)&dio, h_io, 0) == cudaSuccess && dho && diwe && dio) {
        c->hd_h = dho; c->hd_moe = dho + R;
        c->hd_tab = diwe; c->hd_tabw = (float*)(diwe + NARROW_SLOTS); c->hd_err = diwe + 2 * NARROW_SLOTS;
        c->hd_ncur = dio; c->hd_fi = dio + R;
    } else {
        cudaGetLastError();                       // not mapped: the copies stay
    }
    return c;
}

void impl_fl_free(FLCtx* c) {
    if (!c) return;
    if (c->st) cudaStreamSynchronize(c->st);
    void* d[] = { c->blk[0], c->blk[1], c->blk[2], c->blk[3], c->logits, c->probs, c->shared_y, c->sh_gu, c->sh_pair, c->mo,
                  c->s_expert, c->s_tok, c->s_out, c->s_w, c->s_n, c->counts, c->offsets, c->perm, c->hq, c->hd, c->y,
                  c->ncur_all, c->base_all, c->out_all, c->whb, c->wbt, c->rcount, c->wfin };
    for (void* p : d) if (p) cudaFree(p);
    for (int p = 0; p < 2; ++p) {
        void* dd[] = { c->w_expert[p], c->w_tok[p], c->w_out[p], c->w_n[p], c->w_cnt[p], c->w_w[p],
                       c->g_expert[p], c->g_tok[p], c->g_out[p], c->g_n[p], c->g_cnt[p], c->g_w[p] };
        for (void* q : dd) if (q) cudaFree(q);
        void* hh[] = { c->hw_tab[p], c->hw_w[p], c->hg_tab[p], c->hg_w[p] };
        for (void* q : hh) if (q) cudaFreeHost(q);
        if (c->wev[p]) cudaEventDestroy(c->wev[p]);
    }
    void* h[] = { c->hblk[0], c->hblk[1], c->hblk[2], c->hblk[3], c->h_in, c->h_wh, c->h_wmoe };
    for (void* p : h) if (p) cudaFreeHost(p);
    for (auto& g : c->graphs) if (g.exec) cudaGraphExecDestroy(g.exec);
    cudaEvent_t ev[] = { c->em0, c->em1, c->ep0, c->ep1, c->eh2d };
    for (cudaEvent_t e : ev) if (e) cudaEventDestroy(e);
    if (c->st && c->own_stream) cudaStreamDestroy(c->st);
    delete c;
}

int impl_fl_moe_error(FLCtx* c) { if (!c) return LK_ERR_ARG; const int e = c->last_err; c->last_err = 0; return e; }

void impl_fl_h2d(FLCtx* c, void* dst, const void* src, size_t bytes) {
    if (!c || !bytes) return;
    FLCK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, c->st));
}

void impl_fl_wait_event(FLCtx* c, fl_event_t ev) { flush_prepare_any(c); if (c) FLCK(cudaStreamWaitEvent(c->st, (cudaEvent_t)ev, 0)); }

double impl_fl_gpu_ms(FLCtx* c, int which) { return !c ? 0.0 : which == 1 ? c->ms_moe : c->ms_prep; }

// event record that is also a graph node while the stream is being captured
static cudaError_t rec(cudaEvent_t ev, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) return e;
    return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal) : cudaEventRecord(ev, st);
}

// run `enqueue` (stream work only, with fixed pointers for a given key) directly, or as a replay of the CUDA
// graph captured for that key: a key is captured on its second occurrence; if capturing fails the work runs
// directly and the key is not tried again
static void run_graph(FLCtx* c, const FLCtx::GraphKey& k, const std::function<void()>& enqueue) {
    if (!c->use_graphs) { enqueue(); return; }
    FLCtx::GraphEntry* g = nullptr;
    for (auto& e : c->graphs)
        if (!std::memcmp(&e.k, &k, sizeof(k))) { g = &e; break; }
    if (!g) {
        if (c->graphs.size() < FL_MAX_GRAPHS) c->graphs.push_back({k, 1, nullptr});
        enqueue();
        return;
    }
    if (g->exec) { FLCK(cudaGraphLaunch(g->exec, c->st)); return; }
    if (g->seen < 0) { enqueue(); return; }           // capture failed before
    cudaGraph_t graph = nullptr;
    bool ok = cudaStreamBeginCapture(c->st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
        enqueue();
        ok = cudaStreamEndCapture(c->st, &graph) == cudaSuccess && graph;
        if (ok) ok = cudaGraphInstantiate(&g->exec, graph, 0) == cudaSuccess;
        if (graph) cudaGraphDestroy(graph);
    }
    if (!ok) {
        cudaGetLastError();
        g->exec = nullptr; g->seen = -1;
        enqueue();
        return;
    }
    FLCK(cudaGraphLaunch(g->exec, c->st));
}

// shared-expert-only slot table for rows [0, n) (slots of nt tokens), written on the device
__global__ void k_shared_slots(int n, int nt, int* se, int* stok, int* sout, float* sw, int* sn) {
    const int ns = (n + nt - 1) / nt;
    for (int i = threadIdx.x; i < ns * nt; i += blockDim.x) {
        const int t = i < n ? i : -1;
        if (i % nt == 0) se[i / nt] = SHARED_SLOT;
        stok[i] = t; sout[i] = t; sw[i] = t >= 0 ? 1.0f : 0.0f;
    }
    if (threadIdx.x == 0) *sn = ns;
}
static void shared_slots(FLCtx* c, int n, int nt) {
    k_shared_slots<<<1, 64, 0, c->st>>>(n, nt, c->s_expert, c->s_tok, c->s_out, c->s_w, c->s_n);
}

// the shared expert of rows [0, n) of ncur into shared_y, as its own launches: IQ2_XXS (sh_fmt 0 / FL_IQ2)
// through the routed kernels with shared-only slots, the real model's Q5_K / Q6_K (FL_Q5K) through shared_kq.cu
static void enqueue_shared(FLCtx* c, const void* g, const void* u, const void* d, int n, int sh_fmt) {
    if (sh_fmt == FL_Q5K) {
        SharedKqParams sp{};
        sp.gate = (const uint8_t*)g; sp.up = (const uint8_t*)u; sp.down = (const uint8_t*)d;
        sp.x = c->ncur; sp.ld_x = HIDDEN; sp.t0 = 0; sp.n = n; sp.row0 = 0;
        sp.gu = c->sh_gu; sp.hq = c->hq; sp.hd = c->hd; sp.pair = c->sh_pair; sp.y = c->shared_y; sp.err = c->err;
        launch_shared_kq(sp, c->nsm, c->st);
        return;
    }
    const int nt = nt_for(n);
    shared_slots(c, n, nt);
    ExpertParams e = expert_params(c, nullptr, nullptr, nullptr, 0, 0, c->ncur, c->s_expert, c->s_tok, c->s_out, c->s_w, c->s_n,
                                   c->hq, c->hd, c->shared_y);
    e.sh_gate = (const uint8_t*)g; e.sh_up = (const uint8_t*)u; e.sh_down = (const uint8_t*)d;
    launch_gate_up(e, nt, c->nsm, c->st);
    launch_down(e, nt, c->nsm, c->st);
}
// shared_y as fl_moe_prepare leaves it, after an fl_moe_auto that folded the shared expert into its launches
static void materialize_shared(FLCtx* c) {
    if (!c->sh_in_y_n) return;
    FLCK(cudaMemcpyAsync(c->shared_y, c->y + (size_t)c->sh_in_y_n * c->sh_in_y_ke * HIDDEN, (size_t)c->sh_in_y_n * HIDDEN * 4,
                         cudaMemcpyDeviceToDevice, c->st));
    c->sh_in_y_n = 0;
}

static void ensure_shared(FLCtx* c) {
    if (!c->sh_pending) return;
    enqueue_shared(c, c->sh_w[0], c->sh_w[1], c->sh_w[2], c->prep_n, c->sh_fmt);
    c->sh_pending = false;
}

// a host-input prepare's rows: every thread reads one float4 of each from the page-locked mirrors (over PCIe,
// through their device view) and stores it to ncur / ffn_inp.  Programmatic dependent launch lets the router that
// follows load its weights meanwhile; the wait first keeps the previous call's kernels' reads of ncur / ffn_inp
// ordered before these stores.
__global__ void __launch_bounds__(256) k_fl_h2d_rows(const float4* __restrict__ a, const float4* __restrict__ b, float4* da,
                                                     float4* db, int n4) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * 256 + threadIdx.x;
    if (i < n4) { const float4 u = a[i], v = b[i]; da[i] = u; db[i] = v; }
}

// the prepare's launches: rows in (from the host mirrors or device pointers), router, the shared expert for a wide
// pass; events: record ep0 / ep1 around them (the fetch accounts that time).  eh2d follows the router, so that
// no event node separates the row-reading kernel from the router (programmatic dependent launch)
static void enqueue_prepare(FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow, bool events) {
    cudaStream_t st = c->st;
    const size_t bytes = (size_t)N * HIDDEN * 4;
    if (events) FLCK(rec(c->ep0, st));
    if (host) {
        if (c->hd_ncur) {
            const int n4 = N * (HIDDEN / 4);
            FLCK(launch_pdl_n(k_fl_h2d_rows, dim3((n4 + 255) / 256), dim3(256), 0, st, (const float4*)c->hd_ncur, (const float4*)c->hd_fi,
                              (float4*)c->ncur, (float4*)c->ffn_inp, n4));
        } else {
            FLCK(copy_pair(c->ncur, c->h_ncur, (size_t)PREP_ROWS * HIDDEN * 4, bytes, cudaMemcpyHostToDevice, st));
        }
    } else {
        FLCK(cudaMemcpyAsync(c->ncur, ncur, bytes, cudaMemcpyDeviceToDevice, st));
        FLCK(cudaMemcpyAsync(c->ffn_inp, ffn_inp, bytes, cudaMemcpyDeviceToDevice, st));
    }
    // router: full top-8 (the engine applies its keep-KE pass on the fetched rows)
    RouterParams rp{};
    rp.x = c->ncur; rp.T = N; rp.ld_x = HIDDEN; rp.W = W->gate_inp; rp.w_f16 = W->gate_f16; rp.bias = W->probs_b;
    rp.logits = c->logits; rp.probs = c->probs; rp.sel = c->sel; rp.w = c->wts; rp.tile_count = c->rcount;
    rp.n_experts = N_EXPERTS; rp.topk = MAX_TOPK; rp.keep = MAX_TOPK; rp.renorm = 0; rp.n_group = 1; rp.topk_group = 1; rp.scale = 2.5f;
    launch_router(rp, st);
    if (host) FLCK(rec(c->eh2d, st));             // the mirrors have been read
    // shared expert on all rows: now for a wide pass (its base rows need it), else when first needed
    if (W->sh_gate && W->sh_up && W->sh_down && wrow >= 0) {
        enqueue_shared(c, W->sh_gate, W->sh_up, W->sh_down, N, c->sh_fmt);
    } else if (!(W->sh_gate && W->sh_up && W->sh_down)) {
        FLCK(cudaMemsetAsync(c->shared_y, 0, bytes, st));
    }
    if (wrow >= 0) {                  // wide pass: this group's ncur and base = ffn_inp + shared
        FLCK(cudaMemcpyAsync(c->ncur_all + (size_t)wrow * HIDDEN, c->ncur, bytes, cudaMemcpyDeviceToDevice, st));
        CombineParams cp{};
        cp.y = nullptr; cp.resid = c->ffn_inp; cp.T = N; cp.keep = 0; cp.with_shared = 0; cp.shared = c->shared_y;
        cp.h = c->base_all + (size_t)wrow * HIDDEN; cp.moe = nullptr; cp.ld_out = HIDDEN;
        launch_combine(cp, st);
    }
    if (events) FLCK(rec(c->ep1, st));
}

static FLCtx::GraphKey prepare_key(const FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow) {
    FLCtx::GraphKey key;
    std::memset(&key, 0, sizeof(key));            // padding included: keys compare with memcmp
    key.kind = 1; key.a = N; key.b = host; key.c = wrow; key.d = W->gate_f16 | (c->sh_fmt << 4);
    const void* kp[8] = { W->gate_inp, W->probs_b, W->sh_gate, W->sh_up, W->sh_down, host ? nullptr : ncur, host ? nullptr : ffn_inp, nullptr };
    std::memcpy(key.p, kp, sizeof(kp));
    return key;
}

// a deferred prepare runs now, alone (every entry point but fl_moe_auto calls this first)
static void flush_prepare(FLCtx* c) {
    if (!c || !c->prep_deferred) return;
    c->prep_deferred = false;
    const FLMoeW W = c->prep_w;
    const int N = c->prep_n;
    run_graph(c, prepare_key(c, &W, nullptr, nullptr, N, 1, -1), [&]() { enqueue_prepare(c, &W, nullptr, nullptr, N, 1, -1, true); });
    FLCK(cudaGetLastError());
}

static void flush_prepare_any(FLCtx* c) { flush_prepare(c); }

void impl_fl_moe_prepare(FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow) {
    flush_prepare(c);                             // an earlier deferred prepare first: its rows are in the mirrors
    if (!c || !W || !ncur || !ffn_inp || N < 1 || N > PREP_ROWS) { fl_fail(c, LK_ERR_ARG, "fl_moe_prepare: bad argument"); return; }
    if (wrow >= 0 && (!c->ncur_all || wrow + N > c->wmax)) { fl_fail(c, LK_ERR_ARG, "fl_moe_prepare: wide rows outside fl_wide_init capacity"); return; }
    if (W->sh_fmt != 0 && W->sh_fmt != FL_IQ2 && W->sh_fmt != FL_Q5K) { fl_fail(c, LK_ERR_UNSUPPORTED, "fl_moe_prepare: shared-expert format must be FL_IQ2 or FL_Q5K"); return; }
    const size_t bytes = (size_t)N * HIDDEN * 4;
    if (host) {                                   // the mirrors may still feed the previous call's queued copy
        FLCK(cudaEventSynchronize(c->eh2d));
        std::memcpy(c->h_ncur, ncur, bytes); std::memcpy(c->h_fi, ffn_inp, bytes);
    }
    c->prep_n = N;
    c->sh_pending = W->sh_gate && W->sh_up && W->sh_down && wrow < 0;
    c->sh_in_y_n = 0;                             // this prepare's shared expert supersedes the last one
    c->sh_w[0] = W->sh_gate; c->sh_w[1] = W->sh_up; c->sh_w[2] = W->sh_down; c->sh_fmt = W->sh_fmt == FL_Q5K ? FL_Q5K : 0;
    if (host && wrow < 0 && c->use_graphs) {      // the rows are in the mirrors: launch with the next call
        c->prep_deferred = true; c->prep_w = *W;
        return;
    }
    run_graph(c, prepare_key(c, W, ncur, ffn_inp, N, host, wrow), [&]() { enqueue_prepare(c, W, ncur, ffn_inp, N, host, wrow, true); });
    FLCK(cudaGetLastError());
}

void impl_fl_fetch(FLCtx* c, int n, int what, FLOut* out) {
    flush_prepare_any(c);
    if (!c || !out) return;
    std::memset(out, 0, sizeof(FLOut));
    n = std::min(n, c->prep_n > 0 ? c->prep_n : n);
    cudaStream_t st = c->st;
    if (what & 1) {
        FLCK(copy_pair(c->h_sel, c->sel, (size_t)P8 * 4, (size_t)n * MAX_TOPK * 4, cudaMemcpyDeviceToHost, st));
        FLCK(copy_pair(c->h_ncur, c->ncur, (size_t)PREP_ROWS * HIDDEN * 4, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
        out->sel = c->h_sel; out->wts = c->h_wts; out->ncur = c->h_ncur; out->fi = c->h_fi;
    }
    if (what & 32) { FLCK(cudaMemcpyAsync(c->h_h, c->h, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st)); out->h = c->h_h; }
    queue_err(c);
    FLCK(cudaStreamSynchronize(st));
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, c->ep0, c->ep1) == cudaSuccess) c->ms_prep += ms;
    check_dev(c);
}

// the narrow pass from routing already on the device (c->ids, c->w [n][KE]): slots, experts, combine, and the
// result copies into the pinned mirrors (h, moe; with ids_back also the routing), then the stream sync
// host_direct (fl_moe, and the one-row fl_moe_auto whose keep kernel stores ids / w into the host mirror): the
// combine stores h, moe and the error word straight into the page-locked mirrors, so no copy node ends the graph
static void enqueue_narrow(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int KE, int n, bool ids_back,
                           bool fold_shared = false, bool slots_ready = false, bool host_direct = false) {
    cudaStream_t st = c->st;
    const int nt = nt_for(n);
    if (!slots_ready) {                           // slot tables from the device routing (k_fl_keep1 writes them for n == 1)
        SlotParams sp{};
        sp.sel = c->ids; sp.w = c->w; sp.T = n; sp.keep = KE; sp.n_experts = N_EXPERTS; sp.nt = nt; sp.with_shared = fold_shared ? 1 : 0;
        sp.counts = c->counts; sp.offsets = c->offsets; sp.perm = c->perm;
        sp.slot_expert = c->s_expert; sp.slot_tok = c->s_tok; sp.slot_out = c->s_out; sp.slot_w = c->s_w; sp.nslots = c->s_n;
        sp.max_slots = max_slots_for(PREP_ROWS, MAX_TOPK, N_EXPERTS, 1, 1); sp.err = c->err;
        launch_build_slots(sp, st);
    }
    const int64_t sg = (int64_t)EXPERT_GU_BYTES, sd = (int64_t)down_matrix_bytes(down_fmt);
    ExpertParams e = expert_params(c, gate, up, down, sg, sd, c->ncur, c->s_expert, c->s_tok, c->s_out, c->s_w, c->s_n, c->hq, c->hd, c->y);
    e.down_fmt = down_fmt;
    if (fold_shared) {                            // the shared expert as n more slots of the same launches
        e.sh_gate = (const uint8_t*)c->sh_w[0]; e.sh_up = (const uint8_t*)c->sh_w[1]; e.sh_down = (const uint8_t*)c->sh_w[2];
    }
    launch_gate_up(e, nt, c->nsm, st);
    launch_down(e, nt, c->nsm, st);
    CombineParams cp{};                           // h = ffn_inp + shared + routed
    cp.y = c->y; cp.resid = c->ffn_inp; cp.T = n; cp.keep = KE; cp.with_shared = fold_shared ? 1 : 0;
    cp.shared = fold_shared ? nullptr : c->shared_y;
    cp.h = c->h; cp.moe = c->moe; cp.ld_out = HIDDEN;
    if (host_direct) { cp.h2 = c->hd_h; cp.moe2 = c->hd_moe; cp.err = c->err; cp.err2 = c->hd_err; }
    launch_combine(cp, st);
    // the folded shared rows stay in y until a later call needs shared_y (materialize_shared)
    if (!host_direct) {
        FLCK(copy_pair(c->h_h, c->h, (size_t)PREP_ROWS * HIDDEN * 4, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
        if (ids_back)                             // ids, w and the error word: three rows of one block
            FLCK(cudaMemcpy2DAsync(c->h_tab, (size_t)NARROW_SLOTS * 4, c->ids, (size_t)NARROW_SLOTS * 4, (size_t)n * KE * 4, 3,
                                   cudaMemcpyDeviceToHost, st));
    }
    FLCK(rec(c->em1, st));
    if (!ids_back && !host_direct) queue_err(c);
}

// after the enqueued narrow pass: wait for it, account its time, read the error word and the routing back
static void finish_narrow(FLCtx* c, int KE, int n, bool ids_back, FLOut* out) {
    FLCK(cudaStreamSynchronize(c->st));
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, c->em0, c->em1) == cudaSuccess) c->ms_moe += ms;
    check_dev(c);
    if (ids_back) { c->last_ids.assign(c->h_tab, c->h_tab + n * KE); c->last_w.assign(c->h_tabw, c->h_tabw + n * KE); }
    c->last_n = n; c->last_ke = KE;
    out->h = c->h_h; out->moe = c->h_moe;
}

void impl_fl_moe(FLCtx* c, const void* gate, const void* up, const void* down, int nexp, int down_fmt, const int* ids, const float* w,
            int KE, int n, FLOut* out) {
    flush_prepare_any(c);
    if (!c || !out) return;
    std::memset(out, 0, sizeof(FLOut));
    if (!down_fmt_ok(down_fmt)) { fl_fail(c, LK_ERR_UNSUPPORTED, "fl_moe: down format must be FL_IQ2, FL_Q2K or FL_Q3K"); return; }
    if (n < 1 || n > NB || KE < 1 || KE > MAX_TOPK || nexp < 1 || nexp > N_EXPERTS || !ids || !w) { fl_fail(c, LK_ERR_ARG, "fl_moe: bad argument"); return; }
    if ((((uintptr_t)gate | (uintptr_t)up | (uintptr_t)down) & 15)) { fl_fail(c, LK_ERR_ARG, "fl_moe: arena not 16-byte aligned"); return; }
    for (int i = 0; i < n * KE; ++i) if (ids[i] < 0 || ids[i] >= nexp) { fl_fail(c, LK_ERR_ARG, "fl_moe: slot id out of range"); return; }
    cudaStream_t st = c->st;
    int* hi = c->h_tab; float* hw = c->h_tabw;
    std::memcpy(hi, ids, (size_t)n * KE * 4); std::memcpy(hw, w, (size_t)n * KE * 4);
    c->last_ids.assign(ids, ids + n * KE); c->last_w.assign(w, w + n * KE);
    materialize_shared(c);
    const bool pend = c->sh_pending;              // the prepare's shared expert, in this call's launches
    const int pn = c->prep_n;
    // as in fl_moe_auto: an IQ2_XXS shared expert over all prepared rows joins the routed launches
    const bool fold = pend && c->sh_fmt == 0 && down_fmt == FL_IQ2 && n == pn;
    c->sh_pending = false;
    FLCtx::GraphKey key;
    std::memset(&key, 0, sizeof(key));            // padding included: keys compare with memcmp
    key.kind = 2; key.a = n; key.b = KE; key.c = down_fmt; key.d = pend ? pn | (c->sh_fmt << 16) | (fold ? 1 << 24 : 0) : 0;
    key.p[0] = gate; key.p[1] = up; key.p[2] = down;
    if (pend) { key.p[3] = c->sh_w[0]; key.p[4] = c->sh_w[1]; key.p[5] = c->sh_w[2]; }
    run_graph(c, key, [&]() {
        if (pend && !fold) enqueue_shared(c, c->sh_w[0], c->sh_w[1], c->sh_w[2], pn, c->sh_fmt);
        FLCK(rec(c->em0, st));
        FLCK(copy_pair(c->ids, hi, (size_t)NARROW_SLOTS * 4, (size_t)n * KE * 4, cudaMemcpyHostToDevice, st));   // ids, w
        enqueue_narrow(c, gate, up, down, down_fmt, KE, n, false, fold, false, c->hd_h != nullptr);
    });
    if (fold) { c->sh_in_y_n = n; c->sh_in_y_ke = KE; }
    finish_narrow(c, KE, n, false, out);
}


// the engine's keep-KE pass (src/server_core_fused.cpp:793-813, without --share-experts) on the device: row i
// of the router output (sel8 / w8 [n][8], top-8 by score) -> its KE highest-weight experts (equal weights in
// position order) and, with renorm, their weights scaled to sum to 2.5, in the host pass's float order
__device__ __forceinline__ void keep_row(const int* sel8, const float* w8, int i, int KE, int renorm, int* ids, float* w) {
    float wv[8]; int sv[8], rank[8];
    #pragma unroll
    for (int k = 0; k < 8; ++k) { wv[k] = w8[i * 8 + k]; sv[k] = sel8[i * 8 + k]; }
    if (KE >= 8) {                                // the engine compacts only for KE < 8
        #pragma unroll
        for (int k = 0; k < 8; ++k) { ids[i * 8 + k] = sv[k]; w[i * 8 + k] = wv[k]; }
        return;
    }
    #pragma unroll
    for (int k = 0; k < 8; ++k) {
        int r = 0;
        #pragma unroll
        for (int j = 0; j < 8; ++j) r += (wv[j] > wv[k]) || (wv[j] == wv[k] && j < k);
        rank[k] = r;
    }
    float kw[8]; int ks[8];
    #pragma unroll
    for (int r = 0; r < 8; ++r) {
        kw[r] = 0.0f; ks[r] = 0;
        #pragma unroll
        for (int k = 0; k < 8; ++k) if (rank[k] == r) { kw[r] = wv[k]; ks[r] = sv[k]; }
    }
    float sw = 0.0f;
    #pragma unroll
    for (int r = 0; r < 8; ++r) if (r < KE) sw += kw[r];
    const float f = (renorm && sw > 1e-6f) ? 2.5f / sw : 1.0f;
    #pragma unroll
    for (int r = 0; r < 8; ++r) if (r < KE) { ids[i * KE + r] = ks[r]; w[i * KE + r] = renorm && sw > 1e-6f ? kw[r] * f : kw[r]; }
}

__global__ void k_fl_keep(const int* sel8, const float* w8, int n, int KE, int renorm, int* ids, float* w) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) keep_row(sel8, w8, i, KE, renorm, ids, w);
}

// one row (the decode case): the keep pass and the expert stage's single-token slot tables -- the KE kept
// experts in rank order, then the folded shared expert -- so no dispatch kernel runs
struct Keep1Params {
    const int* sel8; const float* w8; int KE, renorm, fold;
    int* ids; float* w; int* se; int* stok; int* sout; float* sw; int* sn;
    int* ids2; float* w2;                         // optional: a second copy of ids / w (the page-locked host mirror)
};
__global__ void k_fl_keep1(Keep1Params p) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    keep_row(p.sel8, p.w8, 0, p.KE, p.renorm, p.ids, p.w);
    for (int k = 0; k < p.KE; ++k) { p.se[k] = p.ids[k]; p.stok[k] = 0; p.sout[k] = k; p.sw[k] = p.w[k]; }
    if (p.ids2) for (int k = 0; k < p.KE; ++k) { p.ids2[k] = p.ids[k]; p.w2[k] = p.w[k]; }
    if (p.fold) { p.se[p.KE] = SHARED_SLOT; p.stok[p.KE] = 0; p.sout[p.KE] = p.KE; p.sw[p.KE] = 1.0f; }
    *p.sn = p.KE + (p.fold ? 1 : 0);
}


void impl_fl_moe_auto(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int KE, int renorm, int n, FLOut* out) {
    if (!c || !out) return;
    std::memset(out, 0, sizeof(FLOut));
    if (!down_fmt_ok(down_fmt)) { fl_fail(c, LK_ERR_UNSUPPORTED, "fl_moe_auto: down format must be FL_IQ2, FL_Q2K or FL_Q3K"); return; }
    if (n < 1 || n > NB || n > c->prep_n || KE < 1 || KE > MAX_TOPK) { fl_fail(c, LK_ERR_ARG, "fl_moe_auto: bad argument (n <= 8 rows of the last fl_moe_prepare)"); return; }
    if ((((uintptr_t)gate | (uintptr_t)up | (uintptr_t)down) & 15)) { fl_fail(c, LK_ERR_ARG, "fl_moe_auto: arena not 16-byte aligned"); return; }
    cudaStream_t st = c->st;
    // the pending shared expert (IQ2_XXS) joins the routed launches when the downs are IQ2_XXS too; with a
    // K-quant down format, or in the real model's Q5_K / Q6_K formats, it runs on its own first
    const bool fold = c->sh_pending && c->sh_fmt == 0 && down_fmt == FL_IQ2 && n == c->prep_n;
    // a deferred prepare joins this call's graph when the shared expert folds in (nothing else needs its rows
    // before the experts); otherwise it runs alone first.  In the joined graph em0 precedes the prepare, so
    // fl_gpu_ms(1) then counts the prepare too, and no event node separates its router from the keep kernel.
    const bool merge = c->prep_deferred && fold;
    if (!merge) flush_prepare(c);
    materialize_shared(c);
    if (!fold) ensure_shared(c);
    c->sh_pending = false;
    const FLMoeW pw = c->prep_w;
    c->prep_deferred = false;
    FLCtx::GraphKey key;
    std::memset(&key, 0, sizeof(key));            // padding included: keys compare with memcmp
    key.kind = merge ? 4 : 3; key.a = n; key.b = KE; key.c = down_fmt; key.d = renorm | (fold ? 2 : 0);
    key.p[0] = gate; key.p[1] = up; key.p[2] = down;
    if (fold) { key.p[3] = c->sh_w[0]; key.p[4] = c->sh_w[1]; key.p[5] = c->sh_w[2]; }
    if (merge) { key.p[6] = pw.gate_inp; key.p[7] = pw.probs_b; key.d |= (pw.gate_f16 << 4) | (c->prep_n << 8); }
    run_graph(c, key, [&]() {
        FLCK(rec(c->em0, st));
        if (merge) enqueue_prepare(c, &pw, nullptr, nullptr, c->prep_n, 1, -1, false);
        const bool direct = n == 1 && c->hd_h;
        if (n == 1) {
            const Keep1Params kp{ c->sel, c->wts, KE, renorm, fold ? 1 : 0, c->ids, c->w, c->s_expert, c->s_tok, c->s_out, c->s_w, c->s_n,
                                  direct ? c->hd_tab : nullptr, direct ? c->hd_tabw : nullptr };
            FLCK(launch_pdl(k_fl_keep1, dim3(1), dim3(32), 0, st, kp));
        } else {
            k_fl_keep<<<1, 64, 0, st>>>(c->sel, c->wts, n, KE, renorm, c->ids, c->w);
        }
        enqueue_narrow(c, gate, up, down, down_fmt, KE, n, true, fold, n == 1, direct);
    });
    if (fold) { c->sh_in_y_n = n; c->sh_in_y_ke = KE; }
    finish_narrow(c, KE, n, true, out);
}

void impl_fl_use_graphs(FLCtx* c, int enable) { flush_prepare_any(c); if (c) c->use_graphs = enable != 0; }

void impl_fl_skip(FLCtx* c, const float* mo, int n, FLOut* out) {
    flush_prepare_any(c);
    if (!c || !out || !mo || n < 1 || n > PREP_ROWS) return;
    std::memset(out, 0, sizeof(FLOut));
    cudaStream_t st = c->st;
    materialize_shared(c);
    ensure_shared(c);
    std::memcpy(c->h_in, mo, (size_t)n * HIDDEN * 4);
    FLCK(cudaMemcpyAsync(c->mo, c->h_in, (size_t)n * HIDDEN * 4, cudaMemcpyHostToDevice, st));
    CombineParams cp{};
    cp.y = c->mo; cp.resid = c->ffn_inp; cp.T = n; cp.keep = 1; cp.with_shared = 0; cp.shared = c->shared_y;
    cp.h = c->h; cp.moe = nullptr; cp.ld_out = HIDDEN;
    launch_combine(cp, st);
    FLCK(cudaMemcpyAsync(c->h_h, c->h, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
    FLCK(cudaStreamSynchronize(st));
    out->h = c->h_h;
}

void impl_fl_moe_outs(FLCtx* c, int b, const int* ids, const float* w, int KE, float* out) {
    flush_prepare_any(c);
    if (!c || !ids || !w || !out || b < 0 || b >= c->last_n || KE != c->last_ke) { fl_fail(c, LK_ERR_ARG, "fl_moe_outs: no matching narrow pass"); return; }
    std::vector<float> rows((size_t)KE * HIDDEN);
    FLCK(cudaStreamSynchronize(c->st));
    FLCK(cudaMemcpy(rows.data(), c->y + (size_t)b * KE * HIDDEN, rows.size() * 4, cudaMemcpyDeviceToHost));
    for (int k = 0; k < KE; ++k) {
        int src = -1;
        for (int j = 0; j < KE; ++j) if (c->last_ids[b * KE + j] == ids[k]) { src = j; break; }
        const float lw = src >= 0 ? c->last_w[b * KE + src] : 0.f;
        for (int e = 0; e < HIDDEN; ++e)
            out[(size_t)k * HIDDEN + e] = (src >= 0 && lw != 0.f) ? rows[(size_t)src * HIDDEN + e] / lw * w[k] : 0.f;
    }
}

int impl_fl_wide_init(FLCtx* c, int wmax, int KE) {
    flush_prepare_any(c);
    if (!c || wmax < 1 || KE < 1 || KE > MAX_TOPK) return 0;
    c->wmax = wmax; c->wke = KE;
    const size_t R = (size_t)wmax * HIDDEN;
    const size_t ent = (size_t)wmax * KE;
    if (dz(&c->ncur_all, R) || dz(&c->base_all, R) || dz(&c->out_all, ent * HIDDEN) || dz(&c->wbt, gate_q8_tile_halfs(WIDE_SLOTS)) ||
        dz(&c->whb, ent * MOE_INTER) || dz(&c->wfin, 2 * R) || hz(&c->h_wh, R) || hz(&c->h_wmoe, R)) { fl_fail(c, LK_ERR_CUDA, "fl_wide_init: allocation failed"); return 0; }
    for (int p = 0; p < 2; ++p) {
        // room for WIDE_SLOTS slots of MM_NT tokens (the down's layout) and of GEMM_NT tokens (the gate/up's):
        // merging the engine's slots never makes more slots than it passed
        const int e = WIDE_SLOTS * MM_NT, eg = WIDE_SLOTS * GEMM_NT;
        if (dz(&c->w_expert[p], WIDE_SLOTS) || dz(&c->w_tok[p], e) || dz(&c->w_out[p], e) || dz(&c->w_w[p], e) ||
            dz(&c->w_n[p], 1) || dz(&c->w_cnt[p], WIDE_SLOTS) || hz(&c->hw_tab[p], WIDE_SLOTS + 2 * e + 1) ||
            dz(&c->g_expert[p], WIDE_SLOTS) || dz(&c->g_tok[p], eg) || dz(&c->g_out[p], eg) || dz(&c->g_w[p], eg) ||
            dz(&c->g_n[p], 1) || dz(&c->g_cnt[p], WIDE_SLOTS) || hz(&c->hg_tab[p], WIDE_SLOTS + 2 * eg + 1) ||
            hz(&c->hw_w[p], e) || hz(&c->hg_w[p], eg) || cudaEventCreateWithFlags(&c->wev[p], cudaEventDisableTiming)) {
            fl_fail(c, LK_ERR_CUDA, "fl_wide_init: allocation failed"); return 0;
        }
    }
    return 1;
}

void impl_fl_wide_moe(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int nexp, const int* midx, const int* rows,
                 const int* kidx, const float* wk, int nslots, int KE, int par) {
    flush_prepare_any(c);
    if (!c || !c->ncur_all) { fl_fail(c, LK_ERR_ARG, "fl_wide_moe: fl_wide_init first"); return; }
    if (!down_fmt_ok(down_fmt)) { fl_fail(c, LK_ERR_UNSUPPORTED, "fl_wide_moe: down format must be FL_IQ2, FL_Q2K or FL_Q3K"); return; }
    if (KE != c->wke || nslots < 0 || nexp < 1) { fl_fail(c, LK_ERR_ARG, "fl_wide_moe: bad argument"); return; }
    if ((((uintptr_t)gate | (uintptr_t)up | (uintptr_t)down) & 15)) { fl_fail(c, LK_ERR_ARG, "fl_wide_moe: arena not 16-byte aligned"); return; }
    par &= 1;
    cudaStream_t st = c->st;
    materialize_shared(c);
    const int64_t sg = (int64_t)EXPERT_GU_BYTES, sd = (int64_t)down_matrix_bytes(down_fmt);
    // The engine's slots (<= NB (row, k) pairs of one expert each), consecutive same-expert slots merged:
    // into slots of up to GEMM_NT tokens for the q8 gate/up (gate_up_q8.cu: tcgen05, the reference's numerics,
    // h re-quantised to q8), and into slots of up to MM_NT tokens for the mma.sync down (IQ2_XXS slot_mma.cu or
    // K-quant kq_mma.cu) that reads the q8 SwiGLU rows.
    for (int s0 = 0; s0 < nslots; s0 += WIDE_SLOTS) {
        const int ns = std::min(WIDE_SLOTS, nslots - s0);
        if (s0 > 0) FLCK(cudaStreamSynchronize(st));          // the tables of this parity are reused
        int* he = c->hw_tab[par]; int* ht = he + WIDE_SLOTS; int* ho = ht + WIDE_SLOTS * MM_NT; float* hw = c->hw_w[par];
        int* ge = c->hg_tab[par]; int* gt = ge + WIDE_SLOTS; int* go = gt + WIDE_SLOTS * GEMM_NT; float* gw = c->hg_w[par];
        int nout = 0, fill = 0, cur = -1, gout = 0, gfill = 0, gcur = -1;
        for (int s = 0; s < ns; ++s) {
            const int m = midx[s0 + s];
            if (m < 0 || m >= nexp) { fl_fail(c, LK_ERR_ARG, "fl_wide_moe: slot expert out of range"); return; }
            int live = 0;
            for (int i = 0; i < NB; ++i) {
                const int r = rows[(size_t)(s0 + s) * NB + i], k = kidx[(size_t)(s0 + s) * NB + i];
                live += (r >= 0 && r < c->wmax && k >= 0 && k < KE) ? 1 : 0;
            }
            if (live == 0) continue;
            if (m != cur || fill + live > MM_NT) {             // a new down slot
                he[nout] = m; cur = m; fill = 0;
                for (int i = 0; i < MM_NT; ++i) { ht[nout * MM_NT + i] = -1; ho[nout * MM_NT + i] = -1; hw[nout * MM_NT + i] = 0.f; }
                ++nout;
            }
            if (m != gcur || gfill + live > GEMM_NT) {         // a new gate/up slot
                ge[gout] = m; gcur = m; gfill = 0;
                for (int i = 0; i < GEMM_NT; ++i) { gt[gout * GEMM_NT + i] = -1; go[gout * GEMM_NT + i] = -1; gw[gout * GEMM_NT + i] = 0.f; }
                ++gout;
            }
            for (int i = 0; i < NB; ++i) {
                const int r = rows[(size_t)(s0 + s) * NB + i], k = kidx[(size_t)(s0 + s) * NB + i];
                if (!(r >= 0 && r < c->wmax && k >= 0 && k < KE)) continue;
                const int q = (nout - 1) * MM_NT + fill++, qg = (gout - 1) * GEMM_NT + gfill++;
                ht[q] = r; ho[q] = r * KE + k; hw[q] = wk[(size_t)(s0 + s) * NB + i];
                gt[qg] = r; go[qg] = r * KE + k; gw[qg] = hw[q];
            }
        }
        if (nout == 0) continue;
        ho[nout * MM_NT] = nout;
        go[gout * GEMM_NT] = gout;
        FLCK(cudaMemcpyAsync(c->w_expert[par], he, (size_t)nout * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->w_tok[par], ht, (size_t)nout * MM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->w_out[par], ho, (size_t)nout * MM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->w_w[par], hw, (size_t)nout * MM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->w_n[par], ho + nout * MM_NT, 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->g_expert[par], ge, (size_t)gout * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->g_tok[par], gt, (size_t)gout * GEMM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->g_out[par], go, (size_t)gout * GEMM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->g_w[par], gw, (size_t)gout * GEMM_NT * 4, cudaMemcpyHostToDevice, st));
        FLCK(cudaMemcpyAsync(c->g_n[par], go + gout * GEMM_NT, 4, cudaMemcpyHostToDevice, st));
        GemmParams g{};
        g.gate = (const uint8_t*)gate; g.up = (const uint8_t*)up; g.gate_stride = sg; g.up_stride = sg;
        g.x = c->ncur_all; g.ld_x = HIDDEN;
        g.slot_expert = c->g_expert[par]; g.slot_tok = c->g_tok[par]; g.slot_out = c->g_out[par]; g.slot_w = c->g_w[par];
        g.nslots = c->g_n[par]; g.max_slots = gout; g.slot_cnt = c->g_cnt[par]; g.bt = c->wbt; g.hb = c->whb; g.err = c->err;
        launch_gate_up_q8(g, c->nsm, st);
        MmaParams m{};
        m.down = (const uint8_t*)down; m.down_stride = sd;
        m.slot_expert = c->w_expert[par]; m.slot_tok = c->w_tok[par]; m.slot_out = c->w_out[par]; m.slot_w = c->w_w[par];
        m.nslots = c->w_n[par]; m.max_slots = WIDE_SLOTS; m.slot_cnt = c->w_cnt[par];
        m.hb = c->whb; m.y = c->out_all; m.err = c->err;
        if (down_fmt == FL_IQ2) {
            launch_slot_mma_down(m, c->nsm, st);      // its prep pass writes slot_cnt
        } else {
            m.slot_cnt = nullptr;                     // the K-quant down counts each slot's tokens itself
            launch_kq_mma_down(m, down_fmt, c->nsm, st);
        }
    }
    FLCK(cudaGetLastError());
}

void impl_fl_wide_mark(FLCtx* c, int par) { flush_prepare_any(c); if (c && c->wev[par & 1]) FLCK(cudaEventRecord(c->wev[par & 1], c->st)); }
void impl_fl_wide_wait(FLCtx* c, int par) { flush_prepare_any(c); if (c && c->wev[par & 1]) FLCK(cudaEventSynchronize(c->wev[par & 1])); }

void impl_fl_wide_finish(FLCtx* c, int n, int KE, FLOut* out) {
    flush_prepare_any(c);
    if (!c || !out) return;
    std::memset(out, 0, sizeof(FLOut));
    if (!c->ncur_all || n < 1 || n > c->wmax || KE != c->wke) { fl_fail(c, LK_ERR_ARG, "fl_wide_finish: bad argument"); return; }
    cudaStream_t st = c->st;
    // h and moe of the pass into the finish buffer (allocated by fl_wide_init), then into the pinned mirrors
    CombineParams cp{};
    cp.y = c->out_all; cp.resid = c->base_all; cp.T = n; cp.keep = KE; cp.with_shared = 0; cp.shared = nullptr;
    cp.ld_out = HIDDEN;
    float* hbuf = c->wfin;
    cp.h = hbuf; cp.moe = hbuf + (size_t)n * HIDDEN;
    launch_combine(cp, st);
    FLCK(cudaMemcpyAsync(c->h_wh, hbuf, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
    FLCK(cudaMemcpyAsync(c->h_wmoe, hbuf + (size_t)n * HIDDEN, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
    queue_err(c);
    FLCK(cudaStreamSynchronize(st));
    check_dev(c);
    out->h = c->h_wh; out->moe = c->h_wmoe;
}

void impl_fl_wide_skip(FLCtx* c, const float* mo, int n, FLOut* out) {
    flush_prepare_any(c);
    if (!c || !out || !mo || !c->ncur_all || n < 1 || n > c->wmax) return;
    std::memset(out, 0, sizeof(FLOut));
    cudaStream_t st = c->st;
    float* dmo = c->wfin;
    FLCK(cudaMemcpyAsync(dmo, mo, (size_t)n * HIDDEN * 4, cudaMemcpyHostToDevice, st));
    CombineParams cp{};
    cp.y = dmo; cp.resid = c->base_all; cp.T = n; cp.keep = 1; cp.with_shared = 0; cp.shared = nullptr;
    cp.h = dmo + (size_t)n * HIDDEN; cp.moe = nullptr; cp.ld_out = HIDDEN;
    launch_combine(cp, st);
    FLCK(cudaMemcpyAsync(c->h_wh, dmo + (size_t)n * HIDDEN, (size_t)n * HIDDEN * 4, cudaMemcpyDeviceToHost, st));
    FLCK(cudaStreamSynchronize(st));
    out->h = c->h_wh;
}

void impl_fl_wide_outs(FLCtx* c, int row, int KE, float* out) {
    flush_prepare_any(c);
    if (!c || !out || !c->out_all || row < 0 || row >= c->wmax || KE != c->wke) { fl_fail(c, LK_ERR_ARG, "fl_wide_outs: bad argument"); return; }
    FLCK(cudaStreamSynchronize(c->st));
    FLCK(cudaMemcpy(out, c->out_all + (size_t)row * KE * HIDDEN, (size_t)KE * HIDDEN * 4, cudaMemcpyDeviceToHost));
}

// ---- the attention context's MoE inputs, taken over (lkfl_moe_adopt)
// shared_y[i] = sum over the n_parts partial sums parts[k][i] ([k][part_rows][HIDDEN])
__global__ void k_sum_parts(const float* __restrict__ parts, int n_parts, size_t part_rows, int n, float* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)n * HIDDEN) return;
    float v = 0.0f;
    for (int k = 0; k < n_parts; ++k) v += parts[(size_t)k * part_rows * HIDDEN + i];
    out[i] = v;
}

void impl_fl_moe_adopt(FLCtx* c, const float* ncur, const float* ffn_inp, const float* shared_parts, int n_parts, size_t part_rows,
                       const int* sel, const float* wts, int N, int wrow) {
    flush_prepare_any(c);
    if (!c || !ncur || !ffn_inp || !sel || !wts || N < 1 || N > PREP_ROWS || n_parts < 0 || (n_parts > 0 && !shared_parts)) {
        fl_fail(c, LK_ERR_ARG, "lkfl_moe_adopt: bad argument"); return;
    }
    if (wrow >= 0 && (!c->ncur_all || wrow + N > c->wmax)) { fl_fail(c, LK_ERR_ARG, "lkfl_moe_adopt: wide rows outside fl_wide_init capacity"); return; }
    cudaStream_t st = c->st;
    const size_t bytes = (size_t)N * HIDDEN * 4;
    c->prep_n = N; c->sh_pending = false; c->sh_in_y_n = 0;
    FLCK(cudaMemcpyAsync(c->ncur, ncur, bytes, cudaMemcpyDeviceToDevice, st));
    FLCK(cudaMemcpyAsync(c->ffn_inp, ffn_inp, bytes, cudaMemcpyDeviceToDevice, st));
    FLCK(cudaMemcpyAsync(c->sel, sel, (size_t)N * MAX_TOPK * 4, cudaMemcpyDeviceToDevice, st));
    FLCK(cudaMemcpyAsync(c->wts, wts, (size_t)N * MAX_TOPK * 4, cudaMemcpyDeviceToDevice, st));
    if (n_parts > 0) k_sum_parts<<<(unsigned)(((size_t)N * HIDDEN + 255) / 256), 256, 0, st>>>(shared_parts, n_parts, part_rows, N, c->shared_y);
    else FLCK(cudaMemsetAsync(c->shared_y, 0, bytes, st));
    if (wrow >= 0) {                  // wide pass: this group's ncur and base = ffn_inp + shared
        FLCK(cudaMemcpyAsync(c->ncur_all + (size_t)wrow * HIDDEN, c->ncur, bytes, cudaMemcpyDeviceToDevice, st));
        CombineParams cp{};
        cp.y = nullptr; cp.resid = c->ffn_inp; cp.T = N; cp.keep = 0; cp.with_shared = 0; cp.shared = c->shared_y;
        cp.h = c->base_all + (size_t)wrow * HIDDEN; cp.moe = nullptr; cp.ld_out = HIDDEN;
        launch_combine(cp, st);
    }
    FLCK(cudaGetLastError());
}

// ---- the exported entry points: each under its fused_layer.h name (fl_*) and under lkfl_*, the names a
// bridge library calls when it re-exports fl_* itself (fl_bridge.cu).  The implementations above are internal
// to this library, so a process that loads both libraries never routes this library's own calls into the
// bridge's fl_* symbols.
#define LKFL_EXPORT(ret, name, params, args) \
    LK_API ret fl_##name params { return impl_fl_##name args; } \
    LK_API ret lkfl_##name params { return impl_fl_##name args; }

extern "C" {
LKFL_EXPORT(FLCtx*, init, (int kvp, int sc_cap), (kvp, sc_cap))
LKFL_EXPORT(void, free, (FLCtx* c), (c))
LKFL_EXPORT(int, moe_error, (FLCtx* c), (c))
LKFL_EXPORT(void, h2d, (FLCtx* c, void* dst, const void* src, size_t bytes), (c, dst, src, bytes))
LKFL_EXPORT(void, wait_event, (FLCtx* c, fl_event_t ev), (c, ev))
LKFL_EXPORT(double, gpu_ms, (FLCtx* c, int which), (c, which))
LKFL_EXPORT(void, moe_prepare, (FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow),
            (c, W, ncur, ffn_inp, N, host, wrow))
LKFL_EXPORT(void, fetch, (FLCtx* c, int n, int what, FLOut* out), (c, n, what, out))
LKFL_EXPORT(void, moe, (FLCtx* c, const void* gate, const void* up, const void* down, int nexp, int down_fmt, const int* ids,
                        const float* w, int KE, int n, FLOut* out), (c, gate, up, down, nexp, down_fmt, ids, w, KE, n, out))
LKFL_EXPORT(void, moe_auto, (FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int KE, int renorm, int n,
                             FLOut* out), (c, gate, up, down, down_fmt, KE, renorm, n, out))
LKFL_EXPORT(void, use_graphs, (FLCtx* c, int enable), (c, enable))
LKFL_EXPORT(void, skip, (FLCtx* c, const float* mo, int n, FLOut* out), (c, mo, n, out))
LKFL_EXPORT(void, moe_outs, (FLCtx* c, int b, const int* ids, const float* w, int KE, float* out), (c, b, ids, w, KE, out))
LKFL_EXPORT(int, wide_init, (FLCtx* c, int wmax, int KE), (c, wmax, KE))
LKFL_EXPORT(void, wide_moe, (FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int nexp, const int* midx,
                             const int* rows, const int* kidx, const float* wk, int nslots, int KE, int par),
            (c, gate, up, down, down_fmt, nexp, midx, rows, kidx, wk, nslots, KE, par))
LKFL_EXPORT(void, wide_mark, (FLCtx* c, int par), (c, par))
LKFL_EXPORT(void, wide_wait, (FLCtx* c, int par), (c, par))
LKFL_EXPORT(void, wide_finish, (FLCtx* c, int n, int KE, FLOut* out), (c, n, KE, out))
LKFL_EXPORT(void, wide_skip, (FLCtx* c, const float* mo, int n, FLOut* out), (c, mo, n, out))
LKFL_EXPORT(void, wide_outs, (FLCtx* c, int row, int KE, float* out), (c, row, KE, out))

LK_API FLCtx* lkfl_init_on_stream(void* stream) { return impl_fl_init(0, 0, (cudaStream_t)stream); }
LK_API void lkfl_moe_adopt(FLCtx* c, const float* ncur, const float* ffn_inp, const float* shared_parts, int n_parts, size_t part_rows,
                           const int* sel, const float* wts, int N, int wrow) {
    impl_fl_moe_adopt(c, ncur, ffn_inp, shared_parts, n_parts, part_rows, sel, wts, N, wrow);
}
LK_API const float* lkfl_device_h(FLCtx* c) { return c ? c->h : nullptr; }
}  // extern "C"
