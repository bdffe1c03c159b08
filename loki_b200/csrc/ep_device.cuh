// ep_device.cuh -- device pieces shared by the expert-parallel kernels (ep.cu, ep_p2p.cu): the row header of
// include/loki_ep.h and the single-token slot tables built straight from received rows.
#pragma once
#include "../../include/loki_ep.h"
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

struct EpRowHdr { int sel[8]; float w[8]; };
static_assert(sizeof(EpRowHdr) == LK_EP_ROW_HDR_BYTES, "header size");

constexpr int EPS_THREADS = 256;

// the direct return's destinations: entry (row i / keep, k = i % keep) of received row (source s = row / cap,
// r = row % cap) goes to ret[s] + ((self * cap + r) * MAX_TOPK + k) * HIDDEN -- its row in the home rank's
// mailbox -- and shared slot j to shared_out + j * HIDDEN; ydst [max_slots] receives the row pointers
struct EpYDst {
    float* ret[LK_EP_MAX_RANKS];
    int self, cap;
    float* shared_out;
    float** ydst;
};

// rows -> sel/w [R][keep] and the single-token slot tables of sp: one slot per live entry in (row, k) order,
// then the shared expert's slots of rows [sh_t0, +sh_n) (sh_n < 0: none); ids outside [0, n_experts) are
// reported (DEV_ERR_BAD_SLOT) and dropped.  Every slot writes its own output row, so the order of the slots
// changes no result.  Called by all EPS_THREADS threads of one CTA.
__device__ __forceinline__ void ep_slots_dev(const uint8_t* __restrict__ recv, int R, int keep, int n_experts, int* sel,
                                             float* w, const SlotParams& sp, const EpYDst* yd = nullptr) {
    __shared__ int wsum[EPS_THREADS / 32];
    __shared__ int base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int entries = R * keep;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int c0 = 0; c0 < entries; c0 += EPS_THREADS) {
        const int i = c0 + tid;
        int e = -1; float wv = 0.0f;
        if (i < entries) {
            const EpRowHdr* h = (const EpRowHdr*)(recv + (size_t)(i / keep) * LK_EP_ROW_BYTES);
            e = h->sel[i % keep]; wv = h->w[i % keep];
            sel[i] = e; w[i] = wv;
            if (e >= n_experts && sp.err) atomicCAS(sp.err, 0, DEV_ERR_BAD_SLOT);
        }
        const bool live = i < entries && e >= 0 && e < n_experts;
        const unsigned b = __ballot_sync(0xffffffffu, live);
        if (lane == 0) wsum[warp] = __popc(b);
        __syncthreads();
        int before = base;
        for (int k = 0; k < warp; ++k) before += wsum[k];
        const int s = before + __popc(b & ((1u << lane) - 1u));
        if (live && s < sp.max_slots) {
            sp.slot_expert[s] = e; sp.slot_tok[s] = i / keep; sp.slot_out[s] = i; sp.slot_w[s] = wv;
            if (yd) {
                const int row = i / keep, src = row / yd->cap, r = row % yd->cap;
                yd->ydst[s] = yd->ret[src] + ((size_t)(yd->self * yd->cap + r) * MAX_TOPK + i % keep) * HIDDEN;
            }
        }
        __syncthreads();
        if (tid == 0) { int t = base; for (int k = 0; k < EPS_THREADS / 32; ++k) t += wsum[k]; base = t; }
        __syncthreads();
    }
    const int nrs = base;
    const int nsh = !sp.with_shared || sp.sh_n < 0 ? 0 : (sp.sh_n > 0 ? sp.sh_n : R);
    for (int j = tid; j < nsh; j += EPS_THREADS) {
        const int s = nrs + j;
        if (s >= sp.max_slots) continue;
        sp.slot_expert[s] = SHARED_SLOT; sp.slot_tok[s] = sp.sh_t0 + j; sp.slot_out[s] = entries + j; sp.slot_w[s] = 1.0f;
        if (yd) yd->ydst[s] = yd->shared_out + (size_t)j * HIDDEN;
    }
    if (tid == 0) *sp.nslots = min(nrs + nsh, sp.max_slots);
}

}  // namespace lk
