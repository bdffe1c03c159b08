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

// ---- the peer-exchange mailbox (ep_p2p.cu): [flags: 2 x LK_EP_MAX_RANKS u32, epoch u32, pad to P2P_HDR]
// [rows: n_ranks x cap x LK_EP_ROW_BYTES] [rets: n_ranks x cap x 7168 fp32] [entry rets (direct return), when
// n_ranks x cap <= P2P_DIRECT_ROWS: n_ranks x cap x 8 x 7168 fp32]
constexpr int P2P_HDR = 256;
constexpr int P2P_DIRECT_ROWS = 64;             // mailboxes of at most this many rows carry the entry rets

struct P2PPeers {
    uint8_t* mb[LK_EP_MAX_RANKS];     // every rank's mailbox base, as mapped in this process
};

__device__ __forceinline__ uint32_t* mb_flags(uint8_t* mb, int which) { return (uint32_t*)mb + which * LK_EP_MAX_RANKS; }
__device__ __forceinline__ uint32_t* mb_epoch(uint8_t* mb) { return (uint32_t*)mb + 2 * LK_EP_MAX_RANKS; }
__device__ __forceinline__ uint8_t* mb_rows(uint8_t* mb) { return mb + P2P_HDR; }
__device__ __forceinline__ float* mb_rets(uint8_t* mb, int n_ranks, int cap) {
    return (float*)(mb + P2P_HDR + (size_t)n_ranks * cap * LK_EP_ROW_BYTES);
}
__host__ __device__ __forceinline__ float* mb_erets(uint8_t* mb, int n_ranks, int cap) {
    return (float*)(mb + P2P_HDR + (size_t)n_ranks * cap * LK_EP_ROW_BYTES) + (size_t)n_ranks * cap * HIDDEN;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v; asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory"); return v;
}

// the router's send for one token (EpSendParams, moe_internal.h), by all threads of the router's last CTA after
// its top-k (sel, w: the token's [keep] entries; xq, xd: its q8 codes and scales): for every rank d the token's
// row in d's mailbox block `self` -- row 0, when the token has an entry on d or d is this rank (its shared
// expert), with the header of d's entries (local ids) and the codes, else an empty header; rows 1 .. cap-1
// empty -- and row_map[d] (d * cap or -1); then each rank's rows flag gets this layer's epoch + 1 (as
// k_p2p_send)
__device__ __forceinline__ void ep_send_token(const EpSendParams& sp, const int* sel, const float* w, int keep,
                                              const int8_t* xq, const float* xd) {
    const int tid = threadIdx.x;
    const int epr = N_EXPERTS / sp.n_ranks;
    int es[MAX_TOPK];
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) es[k] = k < keep ? sel[k] : -1;
    const uint32_t epoch = *mb_epoch(sp.mb[sp.self]) + 1u;
    for (int d = 0; d < sp.n_ranks; ++d) {
        bool has = d == sp.self;
        #pragma unroll
        for (int k = 0; k < MAX_TOPK; ++k) has = has || (es[k] >= d * epr && es[k] < (d + 1) * epr);
        uint8_t* block = mb_rows(sp.mb[d]) + (size_t)sp.self * sp.cap * LK_EP_ROW_BYTES;
        if (tid == 0) sp.row_map[d] = has ? d * sp.cap : -1;
        if (has) {
            if (tid < 16) {
                const int k = tid & 7, e = es[k];
                const bool mine = e >= d * epr && e < (d + 1) * epr;
                if (tid < 8) ((int*)block)[tid] = mine ? e - d * epr : -1;
                else ((float*)block)[tid] = mine ? w[k] : 0.f;
            }
            if (tid < HIDDEN / 32) {
                const uint4* src = (const uint4*)(xq + tid * 32);
                uint4* dst = (uint4*)(block + LK_EP_ROW_Q_OFF + tid * 32);
                dst[0] = src[0]; dst[1] = src[1];
                ((float*)(block + LK_EP_ROW_D_OFF))[tid] = xd[tid];
            }
        }
        for (int rr = has ? 1 : 0; rr < sp.cap; ++rr)
            if (tid < 16) ((int*)(block + (size_t)rr * LK_EP_ROW_BYTES))[tid] = tid < 8 ? -1 : 0;
    }
    __syncthreads();
    if (tid < sp.n_ranks) {
        __threadfence_system();
        st_release_sys(mb_flags(sp.mb[tid], 0) + sp.self, epoch);
    }
}

static_assert(LK_EP_MAX_RANKS == 8, "EpYDst / EpSendParams hold 8 ranks");

// rows -> sel/w [R][keep] and the single-token slot tables of sp: one slot per live entry in (row, k) order,
// then the shared expert's slots of rows [sh_t0, +sh_n) (sh_n < 0: none); ids outside [0, n_experts) are
// reported (DEV_ERR_BAD_SLOT) and dropped.  Every slot writes its own output row, so the order of the slots
// changes no result.  Called by all EPS_THREADS threads of one CTA.
// NT: the CTA's thread count (every thread calls; the function synchronises the CTA).
template <int NT = EPS_THREADS>
__device__ __forceinline__ void ep_slots_dev(const uint8_t* __restrict__ recv, int R, int keep, int n_experts, int* sel,
                                             float* w, const SlotParams& sp, const EpYDst* yd = nullptr) {
    static_assert(NT % 32 == 0, "whole warps");
    __shared__ int wsum[NT / 32];
    __shared__ int base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int entries = R * keep;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int c0 = 0; c0 < entries; c0 += NT) {
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
        if (tid == 0) { int t = base; for (int k = 0; k < NT / 32; ++k) t += wsum[k]; base = t; }
        __syncthreads();
    }
    const int nrs = base;
    const int nsh = !sp.with_shared || sp.sh_n < 0 ? 0 : (sp.sh_n > 0 ? sp.sh_n : R);
    for (int j = tid; j < nsh; j += NT) {
        const int s = nrs + j;
        if (s >= sp.max_slots) continue;
        sp.slot_expert[s] = SHARED_SLOT; sp.slot_tok[s] = sp.sh_t0 + j; sp.slot_out[s] = entries + j; sp.slot_w[s] = 1.0f;
        if (yd) yd->ydst[s] = yd->shared_out + (size_t)j * HIDDEN;
    }
    if (tid == 0) *sp.nslots = min(nrs + nsh, sp.max_slots);
}

// the expert-parallel rows wait fused into a single-token expert kernel (EpWait, moe_internal.h), by all NT threads
// of each CTA after its griddepcontrol.wait: threads s < n_ranks wait (bounded) until source s's rows flag reaches
// this layer's epoch + 1 (the epoch itself advances later, in the return flags kernel, once every CTA has read
// it); then every CTA builds the same slot tables (and destination rows) from the received rows
template <int NT>
__device__ __forceinline__ void ep_rows_wait_slots(const EpWait& ew) {
    const int tid = threadIdx.x;
    if (tid < ew.n_ranks) {
        const uint32_t want = *mb_epoch(ew.mb) + 1u;
        const uint32_t* f = mb_flags(ew.mb, 0) + tid;
        if ((int)(ld_acquire_sys(f) - want) < 0) {
            const unsigned long long t0 = globaltimer_ns();
            while ((int)(ld_acquire_sys(f) - want) < 0) {
                if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (ew.err) atomicCAS(ew.err, 0, DEV_ERR_TIMEOUT_FULL); break; }
            }
        }
    }
    __syncthreads();
    ep_slots_dev<NT>(mb_rows(ew.mb), ew.n_ranks * ew.cap, ew.keep, ew.n_experts, ew.sel, ew.w, ew.sp,
                     ew.yd.ydst ? &ew.yd : nullptr);
    __syncthreads();
}

}  // namespace lk
