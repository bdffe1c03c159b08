// noalloc.cu -- lk_moe_experts_noalloc: the expert stage (dispatch -> gate/up + SwiGLU -> down -> combine)
// for callers that cannot allocate device memory.
//
// Who needs it: an engine that has already handed all free HBM to its resident expert shards and KV cache
// (any further cudaMalloc fails or forces an eviction), and callers on a latency-critical path that cannot
// accept cudaMalloc's implicit device-wide synchronisation.  lk_moe_create allocates its scratch with
// cudaMalloc; this entry point instead uses one file-scope device array, sized for at most
// LK_NOALLOC_MAX_TOKENS tokens, that every GPU which loads the library holds until the process exits.
//
// Rules of use (also in include/loki_moe.h):
//   * the caller passes every input and output; nothing is allocated or freed by any call;
//   * the array's device address is looked up once per device (cudaGetSymbolAddress) by the first call
//     on that device, with that device current -- make that first call before any stream capture;
//   * all calls share the one array and it keeps the last call's contents: calls that overlap on the GPU
//     (two streams, or two host threads) race on it and must be serialised by the caller;
//   * the kernel error word inside the array is cleared at the start of every call; everything else the
//     kernels read is written earlier in the same call (y rows of absent entries -- negative ids -- are
//     left stale, and the combine skips exactly those entries).
#include <cstdio>
#include <mutex>
#include "../../include/loki_moe.h"
#include "moe_internal.h"

using namespace lk;

namespace {

constexpr int NA_TOKENS = LK_NOALLOC_MAX_TOKENS;                  // 8
constexpr int NA_ROWS = NA_TOKENS * MAX_TOPK + NA_TOKENS;         // routed entries + shared rows = 72
// with single-token slots (slot width 1) every routed entry and every shared row is one slot, so a call uses
// at most T*keep + T = 72 slots; 8 more are headroom
constexpr int NA_SLOTS = NA_TOKENS * MAX_TOPK + NA_TOKENS + 8;
static_assert(NA_SLOTS >= NA_TOKENS * MAX_TOPK + NA_TOKENS, "one slot per routed entry and per shared row");
constexpr size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
constexpr size_t OFF_ERR = 0;
constexpr size_t OFF_NSLOTS = OFF_ERR + 256;
constexpr size_t OFF_SEXP = OFF_NSLOTS + 256;
constexpr size_t OFF_STOK = OFF_SEXP + al256(NA_SLOTS * 4);
constexpr size_t OFF_SOUT = OFF_STOK + al256((size_t)NA_SLOTS * MAX_NT * 4);
constexpr size_t OFF_SW = OFF_SOUT + al256((size_t)NA_SLOTS * MAX_NT * 4);
constexpr size_t OFF_COUNTS = OFF_SW + al256((size_t)NA_SLOTS * MAX_NT * 4);
constexpr size_t OFF_OFFSETS = OFF_COUNTS + al256(N_EXPERTS * 4);
constexpr size_t OFF_PERM = OFF_OFFSETS + al256((N_EXPERTS + 1) * 4);
constexpr size_t OFF_HQ = OFF_PERM + al256(NA_TOKENS * MAX_TOPK * 4);
constexpr size_t OFF_HD = OFF_HQ + al256((size_t)NA_ROWS * MOE_INTER);
constexpr size_t OFF_Y = OFF_HD + al256((size_t)NA_ROWS * (MOE_INTER / 32) * 4);
constexpr size_t NA_BYTES = OFF_Y + al256((size_t)NA_ROWS * HIDDEN * 4);   // 2241536 bytes
static_assert(NA_BYTES == LK_NOALLOC_SCRATCH_BYTES, "keep the documented scratch size in step with the layout");

// the scratch itself: one per device, zero-initialised at module load
static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

constexpr int NA_MAX_DEVICES = 64;
std::mutex g_mu;
unsigned char* g_addr[NA_MAX_DEVICES] = {};
int g_nsm[NA_MAX_DEVICES] = {};

int slot_nt_na(int) { return 1; }             // as the context path: single-token slots

// device address of the scratch on the current device (looked up once per device)
int scratch_for_current_device(unsigned char** out, int* nsm) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES) return LK_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            std::fprintf(stderr, "lk_moe_experts_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev, cudaGetErrorString(e));
            return LK_ERR_CUDA;
        }
        g_addr[dev] = (unsigned char*)p;
        g_nsm[dev] = num_sms(dev);
    }
    *out = g_addr[dev];
    *nsm = g_nsm[dev];
    return LK_OK;
}

}  // namespace

extern "C" int lk_moe_experts_noalloc(const LkMoeWeights* W, const float* x, const float* resid, int T, const int* sel,
                                      const float* w, int keep, int with_shared, float* h, float* moe, int* status,
                                      lk_stream_t stream) {
    if (!W || !x || !sel || !w || (h && !resid) || T < 0 || keep < 1) return LK_ERR_ARG;
    if (T > NA_TOKENS || keep > MAX_TOPK) {
        std::fprintf(stderr, "lk_moe_experts_noalloc: T=%d keep=%d outside the static scratch limits (T <= %d, keep <= %d)\n",
                     T, keep, NA_TOKENS, MAX_TOPK);
        return LK_ERR_CAPACITY;
    }
    if (T == 0) return LK_OK;                         // as lk_moe_experts: nothing to do, status untouched
    if (W->down_fmt != LK_FMT_IQ2) return LK_ERR_UNSUPPORTED;
    if (with_shared && W->sh_fmt != 0 && W->sh_fmt != LK_FMT_IQ2) return LK_ERR_UNSUPPORTED;   // IQ2_XXS shared expert only
    const void* mats[] = { W->gate, W->up, W->down };
    for (const void* m : mats) if (!m || ((uintptr_t)m & 15)) return LK_ERR_ARG;
    if ((W->gate_stride & 15) || (W->up_stride & 15) || (W->down_stride & 15)) return LK_ERR_ARG;
    if (with_shared) {
        const void* sm[] = { W->sh_gate, W->sh_up, W->sh_down };
        for (const void* m : sm) if (!m || ((uintptr_t)m & 15)) return LK_ERR_ARG;
    }
    unsigned char* base = nullptr; int nsm = 0;
    int rc = scratch_for_current_device(&base, &nsm);
    if (rc != LK_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    int* err = (int*)(base + OFF_ERR);
    if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return LK_ERR_CUDA;

    const int nt = slot_nt_na(T);
    SlotParams sp{};
    sp.sel = sel; sp.w = w; sp.T = T; sp.keep = keep; sp.n_experts = N_EXPERTS; sp.nt = nt; sp.with_shared = with_shared ? 1 : 0;
    sp.counts = (int*)(base + OFF_COUNTS); sp.offsets = (int*)(base + OFF_OFFSETS); sp.perm = (int*)(base + OFF_PERM);
    sp.slot_expert = (int*)(base + OFF_SEXP); sp.slot_tok = (int*)(base + OFF_STOK); sp.slot_out = (int*)(base + OFF_SOUT);
    sp.slot_w = (float*)(base + OFF_SW); sp.nslots = (int*)(base + OFF_NSLOTS); sp.max_slots = NA_SLOTS; sp.err = err;
    launch_build_slots(sp, st);

    ExpertParams e{};
    e.gate = (const uint8_t*)W->gate; e.up = (const uint8_t*)W->up; e.down = (const uint8_t*)W->down;
    e.gate_stride = W->gate_stride; e.up_stride = W->up_stride; e.down_stride = W->down_stride;
    e.sh_gate = (const uint8_t*)W->sh_gate; e.sh_up = (const uint8_t*)W->sh_up; e.sh_down = (const uint8_t*)W->sh_down;
    e.x = x; e.ld_x = HIDDEN;
    e.slot_expert = sp.slot_expert; e.slot_tok = sp.slot_tok; e.slot_out = sp.slot_out; e.slot_w = sp.slot_w; e.nslots = sp.nslots;
    e.hq = (int8_t*)(base + OFF_HQ); e.hd = (float*)(base + OFF_HD); e.y = (float*)(base + OFF_Y); e.err = err;
    launch_gate_up(e, nt, nsm, st);
    launch_down(e, nt, nsm, st);
    if (h || moe) {
        CombineParams cp{};
        cp.y = e.y; cp.resid = resid; cp.T = T; cp.keep = keep; cp.with_shared = with_shared ? 1 : 0; cp.shared = nullptr;
        cp.h = h; cp.moe = moe; cp.ld_out = HIDDEN;
        cp.sel = sel;                                 // absent entries (negative ids) own no y row: not summed
        launch_combine(cp, st);
    }
    if (status && cudaMemcpyAsync(status, err, sizeof(int), cudaMemcpyDeviceToDevice, st) != cudaSuccess) return LK_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}
