// dispatch.cu -- token -> expert dispatch on the device (replaces the engine's host pass that builds
// per-expert (row, k) lists, src/server_core_fused.cpp:937, and the slot tables of fl_wide_moe,
// src/server_core_fused.cpp:945).
//
// One CTA builds, from sel[T][keep]:
//   counts[e], offsets[e] (exclusive scan) and perm[]: the flat entries t*keep+k grouped by expert,
//   stable by (t, k) -- a counting sort whose in-chunk ranks come from warp match masks;
//   the work-slot table of the grouped matvecs: expert e's list cut into slots of `nt` entries
//   (slot_tok = token, slot_out = entry row of the hq/y buffers, slot_w = routing weight; -1/0 pads),
//   experts in ascending order, then the shared-expert slots (tokens sh_t0.. of SlotParams, entry rows
//   T*keep + j, weight 1).
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

constexpr int DS_THREADS = 1024;

int max_slots_for(int T, int keep, int n_experts, int nt, int with_shared) {
    const int entries = T * keep;
    const int routed = (entries + nt - 1) / nt + (entries < n_experts ? entries : n_experts);
    return routed + (with_shared ? (T + nt - 1) / nt : 0);
}

__global__ void __launch_bounds__(DS_THREADS) k_build_slots(SlotParams p) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    __shared__ int cnt[N_EXPERTS], off[N_EXPERTS + 1], soff[N_EXPERTS + 1], run[N_EXPERTS];
    __shared__ unsigned short wcnt[DS_THREADS / 32][N_EXPERTS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int NE = p.n_experts, nt = p.nt, entries = p.T * p.keep;
    for (int i = tid; i < NE; i += DS_THREADS) { cnt[i] = 0; run[i] = 0; }
    for (int i = tid; i < (DS_THREADS / 32) * N_EXPERTS; i += DS_THREADS) (&wcnt[0][0])[i] = 0;
    __syncthreads();
    // negative ids mark absent entries (an expert-parallel row's experts that live on another rank) and are
    // skipped; ids >= n_experts are reported through the error word and dropped from every table
    for (int i = tid; i < entries; i += DS_THREADS) {
        const int e = p.sel[i];
        if (e >= 0 && e < NE) atomicAdd(&cnt[e], 1);
        else if (e >= NE && p.err) atomicCAS(p.err, 0, DEV_ERR_BAD_SLOT);
    }
    __syncthreads();
    if (tid == 0) {
        int a = 0, s = 0;
        for (int e = 0; e < NE; ++e) { off[e] = a; soff[e] = s; a += cnt[e]; s += (cnt[e] + nt - 1) / nt; }
        off[NE] = a; soff[NE] = s;
    }
    __syncthreads();
    // stable ranks, one chunk of DS_THREADS entries at a time
    for (int c0 = 0; c0 < entries; c0 += DS_THREADS) {
        const int i = c0 + tid;
        const int ev = i < entries ? p.sel[i] : -1;
        const bool live = ev >= 0 && ev < NE;
        const int e = live ? ev : -1 - lane;         // distinct negative keys for dead lanes
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank_w = __popc(peers & ((1u << lane) - 1u));
        if (live && rank_w == 0) wcnt[warp][e] = (unsigned short)__popc(peers);
        __syncthreads();
        if (live) {                                   // rank r of the entry in expert e's stable list
            int before = 0;
            for (int w = 0; w < warp; ++w) before += wcnt[w][e];
            const int r = run[e] + before + rank_w;
            p.perm[off[e] + r] = i;
            const int s = soff[e] + r / nt, m = r % nt;   // its slot and position: written here, in parallel
            if (s < p.max_slots) { p.slot_tok[s * nt + m] = i / p.keep; p.slot_out[s * nt + m] = i; p.slot_w[s * nt + m] = p.w[i]; }
        }
        __syncthreads();
        for (int x = tid; x < NE; x += DS_THREADS) {
            int s = 0;
            for (int w = 0; w < DS_THREADS / 32; ++w) { s += wcnt[w][x]; wcnt[w][x] = 0; }
            run[x] += s;
        }
        __syncthreads();
    }
    // slot tables: the entries were placed by the rank pass; here each slot's expert and the pads that
    // fill the last slot of every expert (positions cnt % nt .. nt-1), over (expert, position) pairs
    for (int e = tid; e < NE; e += DS_THREADS) {
        p.counts[e] = cnt[e];
        p.offsets[e] = off[e];
        for (int s = soff[e]; s < soff[e + 1] && s < p.max_slots; ++s) p.slot_expert[s] = e;
    }
    for (int x = tid; x < NE * nt; x += DS_THREADS) {
        const int e = x / nt, m = x % nt;
        if (cnt[e] % nt == 0 || m < cnt[e] % nt) continue;
        const int s = soff[e + 1] - 1;
        if (s >= p.max_slots) continue;
        p.slot_tok[s * nt + m] = -1; p.slot_out[s * nt + m] = -1; p.slot_w[s * nt + m] = 0.0f;
    }
    const int nrs = soff[NE];
    const int nsh = !p.with_shared || p.sh_n < 0 ? 0 : (p.sh_n > 0 ? p.sh_n : p.T);
    const int nss = (nsh + nt - 1) / nt;
    for (int j = tid; j < nss; j += DS_THREADS) {
        const int s = nrs + j;
        if (s >= p.max_slots) continue;
        p.slot_expert[s] = SHARED_SLOT;
        for (int m = 0; m < nt; ++m) {
            const int t = j * nt + m;
            p.slot_tok[s * nt + m] = t < nsh ? p.sh_t0 + t : -1;
            p.slot_out[s * nt + m] = t < nsh ? entries + t : -1;
            p.slot_w[s * nt + m] = t < nsh ? 1.0f : 0.0f;
        }
    }
    if (tid == 0) { p.offsets[NE] = off[NE]; *p.nslots = min(nrs + nss, p.max_slots); }
}

void launch_build_slots(const SlotParams& p, cudaStream_t st) {
    launch_pdl(k_build_slots, dim3(1), dim3(DS_THREADS), 0, st, p);
}

}  // namespace lk
