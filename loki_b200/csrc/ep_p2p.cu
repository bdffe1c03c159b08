// ep_p2p.cu -- the expert-parallel decode exchange over NVLink peer memory (include/loki_ep.h).
//
// For small per-layer messages (decode: a few 8 KB rows per rank pair) a collective library's launch and
// protocol latency dominates.  Here every rank owns a mailbox in its HBM -- rows received from each
// source rank, partial sums returned by each owner rank, and two flag arrays -- exported with CUDA IPC and
// mapped by every peer.  Senders store straight into the destination's mailbox over NVLink, then publish
// a flag (fence + release store, system scope); receivers poll their local flags (acquire loads, system
// scope) with a bounded wait before reading.  Flags carry a per-rank epoch E: a layer's sends publish E + 1,
// the rows wait (one CTA) waits for E + 1 and then advances the epoch, and the returns publish, and the
// combine waits for, the advanced value; so the same kernels replay correctly inside a captured CUDA graph.
// No rank can run a layer ahead: each layer ends with a wait for every owner's return.
//
// Layout of one mailbox (bytes): [flags: 2 x LK_EP_MAX_RANKS u32, epoch u32, pad to 256]
//   [rows: n_ranks x cap x LK_EP_ROW_BYTES] [rets: n_ranks x cap x 7168 fp32]
//   [entry rets, when n_ranks x cap <= P2P_DIRECT_ROWS: n_ranks x cap x 8 x 7168 fp32]
// Row (s, r) is source rank s's r-th row for this rank; ret (d, r) is owner d's partial sum for this rank's
// r-th row sent to d -- the same indices as the fixed-capacity send buffer, so row_map indexes rets.
// Entry ret ((d, r), k) is owner d's weighted expert output for entry k of that row: the direct return of
// lk_ep_p2p_experts, where the down kernel stores each entry's row straight into the home mailbox and the
// home combine sums the entries in k order (the single-GPU combine's order).
#include <cstring>
#include "ep_device.cuh"

namespace lk {

constexpr int P2P_THREADS = 256;

// one CTA per destination rank d: this rank's rows for d (tokens with an entry on d, and every token to
// itself) into d's mailbox block `self`, unused rows with empty headers, then the dispatch flag
// (and row_map[t][d]: block d's row of token t, d * cap + r, or -1 -- the fixed-capacity pack's map)
__global__ void __launch_bounds__(P2P_THREADS) k_p2p_send(const int* __restrict__ sel, const float* __restrict__ w,
                                                           const float* __restrict__ x, int T, int keep, int n_ranks,
                                                           int self, int cap, P2PPeers peers, int* row_map, int* err) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int d = blockIdx.x, tid = threadIdx.x;
    const int epr = N_EXPERTS / n_ranks;
    const uint32_t epoch = *mb_epoch(peers.mb[self]) + 1u;
    uint8_t* block = mb_rows(peers.mb[d]) + (size_t)self * cap * LK_EP_ROW_BYTES;
    int r = 0;
    for (int t = 0; t < T; ++t) {
        bool has = d == self;
        for (int k = 0; k < keep; ++k) {
            const int e = sel[t * keep + k];
            has = has || (e >= d * epr && e < (d + 1) * epr);
            if ((e < 0 || e >= N_EXPERTS) && tid == 0 && d == 0 && err) atomicCAS(err, 0, DEV_ERR_BAD_SLOT);
        }
        if (tid == 0) row_map[(size_t)t * n_ranks + d] = has ? d * cap + r : -1;
        if (!has) continue;                            // uniform across the CTA
        uint8_t* row = block + (size_t)r * LK_EP_ROW_BYTES;
        if (tid < 16) {
            const int k = tid & 7;
            const int e = k < keep ? sel[t * keep + k] : -1;
            const bool mine = e >= d * epr && e < (d + 1) * epr;
            if (tid < 8) ((int*)row)[tid] = mine ? e - d * epr : -1;
            else ((float*)row)[tid] = mine ? w[t * keep + k] : 0.f;
        }
        ep_row_q8(x + (size_t)t * HIDDEN, (int8_t*)(row + LK_EP_ROW_Q_OFF), (float*)(row + LK_EP_ROW_D_OFF), tid);
        ++r;
    }
    for (int rr = r; rr < cap; ++rr)
        if (tid < 16) ((int*)(block + (size_t)rr * LK_EP_ROW_BYTES))[tid] = tid < 8 ? -1 : 0;
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        st_release_sys(mb_flags(peers.mb[d], 0) + self, epoch);
    }
}

// one CTA per source rank s: this rank's partial sums for s's rows into s's mailbox block `self`
__global__ void __launch_bounds__(P2P_THREADS) k_p2p_return(const float* __restrict__ partial, int n_ranks, int self,
                                                             int cap, P2PPeers peers) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int s = blockIdx.x, tid = threadIdx.x;
    const uint32_t epoch = *mb_epoch(peers.mb[self]);            // advanced by this layer's rows wait
    const float4* src = (const float4*)(partial + (size_t)s * cap * HIDDEN);
    float4* dst = (float4*)(mb_rets(peers.mb[s], n_ranks, cap) + (size_t)self * cap * HIDDEN);
    for (int i = tid; i < cap * HIDDEN / 4; i += P2P_THREADS) dst[i] = src[i];
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        st_release_sys(mb_flags(peers.mb[s], 1) + self, epoch);
    }
}

// the rows wait: lane s waits (bounded) until source s's rows flag reaches this layer's epoch + 1, then the
// epoch advances to it (one CTA: every lane has read the old value before lane 0 writes)
__global__ void k_p2p_wait(uint8_t* mb, int which, int n_ranks, int advance, int* err) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int s = threadIdx.x;
    const uint32_t want = *mb_epoch(mb) + 1u;
    bool ok = true;
    if (s < n_ranks) {
        const uint32_t* f = mb_flags(mb, which) + s;
        if ((int)(ld_acquire_sys(f) - want) < 0) {
            const unsigned long long t0 = globaltimer_ns();
            while ((int)(ld_acquire_sys(f) - want) < 0) {
                if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { ok = false; break; }
            }
        }
        if (!ok && err) atomicCAS(err, 0, which ? DEV_ERR_TIMEOUT_EMPTY : DEV_ERR_TIMEOUT_FULL);
    }
    __syncwarp();
    if (advance && s == 0) *mb_epoch(mb) = want;
}

// the home combine fused with the returns wait: in every CTA, threads s < n_ranks wait (bounded) for owner s's
// return flag to reach this layer's (already advanced) epoch; then h = resid + shared + sum over ranks (rank
// order) and moe = that sum, as k_ep_combine
__global__ void k_p2p_combine(const uint8_t* mb, int n_ranks, int cap, const int* __restrict__ row_map, int T,
                              const float* __restrict__ hpart, const float* __restrict__ shared, float* h, float* moe,
                              int* err) {
    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x;
    if (tid < n_ranks) {
        const uint32_t want = *mb_epoch((uint8_t*)mb);
        const uint32_t* f = mb_flags((uint8_t*)mb, 1) + tid;
        if ((int)(ld_acquire_sys(f) - want) < 0) {
            const unsigned long long t0 = globaltimer_ns();
            while ((int)(ld_acquire_sys(f) - want) < 0) {
                if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_EMPTY); break; }
            }
        }
    }
    __syncthreads();
    const float* ret = mb_rets((uint8_t*)mb, n_ranks, cap);
    const int i = blockIdx.x * blockDim.x + tid;                     // float4 index over T x HIDDEN
    if (i >= T * (HIDDEN / 4)) return;
    const int t = i / (HIDDEN / 4), c = i % (HIDDEN / 4);
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int d = 0; d < n_ranks; ++d) {
        const int row = row_map[(size_t)t * n_ranks + d];
        if (row < 0) continue;
        const float4 v = ((const float4*)(ret + (size_t)row * HIDDEN))[c];
        r.x += v.x; r.y += v.y; r.z += v.z; r.w += v.w;
    }
    if (moe) ((float4*)(moe + (size_t)t * HIDDEN))[c] = r;
    if (h && hpart) {
        float4 b = ((const float4*)(hpart + (size_t)t * HIDDEN))[c];
        if (shared) {
            const float4 v = ((const float4*)(shared + (size_t)t * HIDDEN))[c];
            b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
        }
        ((float4*)(h + (size_t)t * HIDDEN))[c] = make_float4(b.x + r.x, b.y + r.y, b.z + r.z, b.w + r.w);
    }
}

// the direct return's flags for a rank with no tokens of its own (no entry combine follows; otherwise the combine's
// first CTA publishes them), one thread per home rank s: the down kernel that stored the entry rows has completed
// (griddepcontrol.wait: its stores are performed and visible), so a system-scope release of this layer's epoch + 1
// into s's return flag `self` publishes them; then the local epoch advances (every lane has read it first).  The
// single-token gate/up's rows wait read the epoch unadvanced.  (The same release raised by the down kernel's last
// CTA, after a system-scope fence in every CTA, measured ~2.5 us slower per layer.)
__global__ void k_p2p_ret_flags(int n_ranks, int self, P2PPeers peers) {
    pdl_trigger();
    pdl_wait();
    const int s = threadIdx.x;
    const uint32_t epoch = *mb_epoch(peers.mb[self]) + 1u;
    __syncwarp();
    if (s < n_ranks) {
        __threadfence_system();
        st_release_sys(mb_flags(peers.mb[s], 1) + self, epoch);
    }
    __syncwarp();
    if (s == 0) *mb_epoch(peers.mb[self]) = epoch;
}

// the home combine of the direct return (one token per CTA of 64 threads, 28 CTAs per token).  CTA 0 first
// publishes this rank's own return flags (the owner side of the layer: its down kernel has completed) and advances
// the epoch.  Then, in every CTA, threads s < n_ranks poll owner s's flag (bounded) while warp 1 resolves the CTA's
// token's entries -- the owner d of sel[t][k] stored its row at entry ret (row_map[t][d], k) -- and every thread
// loads its resid and shared values; after the wait, moe = the entries summed in k order and h = resid + shared +
// moe (the single-GPU order).  Every rank publishes before it waits, so no rank waits on one that has not.
constexpr int P2PC_THREADS = 64;
__global__ void __launch_bounds__(P2PC_THREADS) k_p2p_combine_k(const uint8_t* mb, int n_ranks, int cap, const int* __restrict__ sel,
                                                                int keep, const int* __restrict__ row_map, int T,
                                                                const float* __restrict__ hpart, const float* __restrict__ shared,
                                                                float* h, float* moe, int self, P2PPeers peers, int* err) {
    __shared__ int eoff[MAX_TOPK];
    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x;
    const int i = blockIdx.x * P2PC_THREADS + tid;                   // float4 index over T x HIDDEN
    const int t = (blockIdx.x * P2PC_THREADS) / (HIDDEN / 4), c = i % (HIDDEN / 4);   // HIDDEN / 4 = 28 CTAs
    // this layer's value: the rows flag this rank's own send published to itself (no peer writes that word)
    const uint32_t want = *(const volatile uint32_t*)(mb_flags((uint8_t*)mb, 0) + self);
    if (blockIdx.x == 0 && tid < n_ranks) {          // this rank's return flags: its down kernel (an earlier
        __threadfence_system();                      // launch) has stored every entry row it owns
        st_release_sys(mb_flags(peers.mb[tid], 1) + self, want);
        if (tid == 0) *mb_epoch((uint8_t*)mb) = want;   // the layer's epoch advance (the gate/up waits read it)
    }
    if (tid < n_ranks) {
        const uint32_t* f = mb_flags((uint8_t*)mb, 1) + tid;
        if ((int)(ld_acquire_sys(f) - want) < 0) {
            const unsigned long long t0 = globaltimer_ns();
            while ((int)(ld_acquire_sys(f) - want) < 0) {
                if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (err) atomicCAS(err, 0, DEV_ERR_TIMEOUT_EMPTY); break; }
            }
        }
    } else if (tid >= 32 && tid < 32 + MAX_TOPK) {
        const int k = tid - 32;
        const int e = k < keep ? sel[t * keep + k] : -1;
        const int row = e >= 0 && e < N_EXPERTS ? row_map[(size_t)t * n_ranks + e / (N_EXPERTS / n_ranks)] : -1;
        eoff[k] = row;
    }
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 b0 = h && hpart ? ((const float4*)(hpart + (size_t)t * HIDDEN))[c] : zero;
    const float4 b1 = h && hpart && shared ? ((const float4*)(shared + (size_t)t * HIDDEN))[c] : zero;
    __syncthreads();
    const float* eret = mb_erets((uint8_t*)mb, n_ranks, cap);
    float4 v[MAX_TOPK];
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k)                                // every load before any sum
        v[k] = eoff[k] >= 0 ? ((const float4*)(eret + ((size_t)eoff[k] * MAX_TOPK + k) * HIDDEN))[c] : zero;
    float4 r = zero;
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k)
        if (eoff[k] >= 0) { r.x += v[k].x; r.y += v[k].y; r.z += v[k].z; r.w += v[k].w; }
    if (moe) ((float4*)(moe + (size_t)t * HIDDEN))[c] = r;
    if (h && hpart) {
        float4 b = b0;
        if (shared) { b.x += b1.x; b.y += b1.y; b.z += b1.z; b.w += b1.w; }
        ((float4*)(h + (size_t)t * HIDDEN))[c] = make_float4(b.x + r.x, b.y + r.y, b.z + r.z, b.w + r.w);
    }
}

}  // namespace lk

using namespace lk;

struct LkEpMailbox {
    int n_ranks = 0, rank = 0, cap = 0, device = 0;
    size_t bytes = 0;
    uint8_t* local = nullptr;
    P2PPeers peers{};
    bool opened[LK_EP_MAX_RANKS] = {};
};

static bool has_erets(int n_ranks, int cap) { return n_ranks * cap <= P2P_DIRECT_ROWS; }
static size_t mailbox_bytes(int n_ranks, int cap) {
    const size_t rows = (size_t)n_ranks * cap;
    return (size_t)P2P_HDR + rows * LK_EP_ROW_BYTES + rows * HIDDEN * sizeof(float) +
           (has_erets(n_ranks, cap) ? rows * MAX_TOPK * HIDDEN * sizeof(float) : 0);
}

extern "C" {

int lk_ep_mailbox_create(int n_ranks, int rank, int cap, int device, LkEpMailbox** out, void* ipc_handle_out) {
    if (!out || !ipc_handle_out || n_ranks < 1 || n_ranks > LK_EP_MAX_RANKS || rank < 0 || rank >= n_ranks || cap < 1 ||
        cap > 64)
        return LK_ERR_ARG;
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) return LK_ERR_CUDA;
    LkEpMailbox* m = new LkEpMailbox();
    m->n_ranks = n_ranks; m->rank = rank; m->cap = cap; m->device = device;
    m->bytes = mailbox_bytes(n_ranks, cap);
    if (cudaMalloc((void**)&m->local, m->bytes) != cudaSuccess || cudaMemset(m->local, 0, m->bytes) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        if (m->local) cudaFree(m->local);
        delete m;
        return LK_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, m->local) != cudaSuccess) { cudaFree(m->local); delete m; return LK_ERR_CUDA; }
    memcpy(ipc_handle_out, &h, sizeof(h));
    m->peers.mb[rank] = m->local;
    *out = m;
    return LK_OK;
}

int lk_ep_mailbox_connect(LkEpMailbox* m, const void* handles) {
    if (!m || !handles) return LK_ERR_ARG;
    if (cudaSetDevice(m->device) != cudaSuccess) return LK_ERR_CUDA;
    for (int r = 0; r < m->n_ranks; ++r) {
        if (r == m->rank || m->opened[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + (size_t)r * LK_EP_IPC_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return LK_ERR_CUDA;
        m->peers.mb[r] = (uint8_t*)p;
        m->opened[r] = true;
    }
    return LK_OK;
}

void lk_ep_mailbox_destroy(LkEpMailbox* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < m->n_ranks; ++r)
        if (m->opened[r]) cudaIpcCloseMemHandle(m->peers.mb[r]);
    if (m->local) cudaFree(m->local);
    delete m;
}

int lk_ep_p2p_dispatch(LkEpMailbox* m, const int* sel, const float* w, const float* x, int T, int keep, int* row_map,
                       int* err, lk_stream_t stream) {
    if (!m || T < 1 || T > m->cap || keep < 1 || keep > MAX_TOPK || !sel || !w || !x || !row_map) return LK_ERR_ARG;
    for (int r = 0; r < m->n_ranks; ++r) if (!m->peers.mb[r]) return LK_ERR_ARG;   // not connected
    cudaStream_t st = (cudaStream_t)stream;
    // the send kernel also writes row_map (the fixed-capacity pack's map) and checks the ids
    launch_pdl_n(k_p2p_send, dim3(m->n_ranks), dim3(P2P_THREADS), 0, st, sel, w, x, T, keep, m->n_ranks, m->rank, m->cap, m->peers,
                 row_map, err);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_ep_p2p_rows(LkEpMailbox* m, const void** rows, int* err, lk_stream_t stream) {
    if (!m || !rows) return LK_ERR_ARG;
    launch_pdl_n(k_p2p_wait, dim3(1), dim3(32), 0, (cudaStream_t)stream, m->local, 0, m->n_ranks, 1, err);
    *rows = m->local + P2P_HDR;
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_ep_p2p_return(LkEpMailbox* m, const float* partial, lk_stream_t stream) {
    if (!m || !partial) return LK_ERR_ARG;
    launch_pdl_n(k_p2p_return, dim3(m->n_ranks), dim3(P2P_THREADS), 0, (cudaStream_t)stream, partial, m->n_ranks, m->rank, m->cap, m->peers);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_ep_p2p_combine(LkEpMailbox* m, const int* row_map, int T, const float* resid, const float* shared, float* h,
                      float* moe, int* err, lk_stream_t stream) {
    if (!m || T < 1 || T > m->cap || !row_map) return LK_ERR_ARG;
    const int n = T * (HIDDEN / 4);
    launch_pdl_n(k_p2p_combine, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t)stream, (const uint8_t*)m->local, m->n_ranks,
                 m->cap, row_map, T, resid, shared, h, moe, err);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_ep_p2p_combine_entries(LkEpMailbox* m, const int* sel, int keep, const int* row_map, int T, const float* resid,
                              const float* shared, float* h, float* moe, int* err, lk_stream_t stream) {
    if (!m || T < 1 || T > m->cap || !sel || keep < 1 || keep > MAX_TOPK || !row_map) return LK_ERR_ARG;
    for (int r = 0; r < m->n_ranks; ++r) if (!m->peers.mb[r]) return LK_ERR_ARG;   // not connected
    if (!has_erets(m->n_ranks, m->cap)) return LK_ERR_UNSUPPORTED;
    static_assert((HIDDEN / 4) % P2PC_THREADS == 0, "a combine CTA covers one token");
    launch_pdl_n(k_p2p_combine_k, dim3(T * (HIDDEN / 4) / P2PC_THREADS), dim3(P2PC_THREADS), 0, (cudaStream_t)stream, (const uint8_t*)m->local,
                 m->n_ranks, m->cap, sel, keep, row_map, T, resid, shared, h, moe, m->rank, m->peers, err);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

}  // extern "C"

namespace lk {

int p2p_rows_count(const LkEpMailbox* m) { return m->n_ranks * m->cap; }
int p2p_rank(const LkEpMailbox* m) { return m->rank; }
int p2p_cap(const LkEpMailbox* m) { return m->cap; }

bool p2p_direct_ok(const LkEpMailbox* m) { return has_erets(m->n_ranks, m->cap); }

int p2p_rows_wait(LkEpMailbox* m, int keep, int n_experts, int* sel, float* w, const SlotParams& sp, int* err,
                  float** ydst, float* shared_out, EpWait* out, const uint8_t** rows) {
    for (int r = 0; r < m->n_ranks; ++r) if (!m->peers.mb[r]) return LK_ERR_ARG;   // not connected
    EpWait ew{};
    ew.mb = m->local; ew.n_ranks = m->n_ranks; ew.cap = m->cap; ew.keep = keep; ew.n_experts = n_experts;
    ew.sel = sel; ew.w = w; ew.sp = sp; ew.err = err;
    if (ydst) {
        if (!has_erets(m->n_ranks, m->cap)) return LK_ERR_UNSUPPORTED;
        for (int r = 0; r < m->n_ranks; ++r) ew.yd.ret[r] = mb_erets(m->peers.mb[r], m->n_ranks, m->cap);
        ew.yd.self = m->rank; ew.yd.cap = m->cap; ew.yd.shared_out = shared_out; ew.yd.ydst = ydst;
    }
    *out = ew;
    *rows = m->local + P2P_HDR;
    return LK_OK;
}

bool p2p_send_params(const LkEpMailbox* m, int* row_map, EpSendParams* out) {
    *out = EpSendParams{};
    for (int r = 0; r < m->n_ranks; ++r) {
        if (!m->peers.mb[r]) return false;
        out->mb[r] = m->peers.mb[r];
    }
    out->n_ranks = m->n_ranks; out->self = m->rank; out->cap = m->cap; out->row_map = row_map;
    return true;
}

int p2p_ret_flags(LkEpMailbox* m, cudaStream_t st) {
    launch_pdl_n(k_p2p_ret_flags, dim3(1), dim3(32), 0, st, m->n_ranks, m->rank, m->peers);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

}  // namespace lk
