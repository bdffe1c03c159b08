// ep.cu -- expert-parallel row exchange kernels (include/loki_ep.h): pack rows for their owner ranks,
// unpack the received row headers, and the home-side combine of the returned partial sums.
//
// No counterpart in the reference (one GPU, experts streamed from NVMe by src/moe_stream_buffer.h).  The
// arithmetic the rows feed is the single-GPU expert stage; only the order of the final sum differs: the
// home rank adds the per-rank partial sums (each summed in entry order on its rank) in rank order.
#include "ep_device.cuh"

namespace lk {

constexpr int EP_PLAN_THREADS = 1024;
static_assert(LK_EP_ROW_BYTES % 16 == 0 && LK_EP_ROW_Q_OFF % 16 == 0 && LK_EP_ROW_D_OFF % 16 == 0,
              "rows and their parts must keep 16-byte alignment");


// one CTA: per destination rank the stable (token-ascending) row index of every token that has an entry
// there, the per-rank counts, block offsets (fixed capacity or compact) and the headers of unused rows
__global__ void __launch_bounds__(EP_PLAN_THREADS) k_ep_plan(const int* __restrict__ sel, int T, int keep, int n_ranks,
                                                              int self_rank, int cap, int* counts, int* row_map, uint8_t* send,
                                                              int* err) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    __shared__ int wc[LK_EP_MAX_RANKS][32], pre[LK_EP_MAX_RANKS][32], base[LK_EP_MAX_RANKS], off[LK_EP_MAX_RANKS + 1];
    __shared__ int cnt[LK_EP_MAX_RANKS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int epr = N_EXPERTS / n_ranks;
    if (tid < LK_EP_MAX_RANKS) base[tid] = 0;
    __syncthreads();
    for (int c0 = 0; c0 < T; c0 += EP_PLAN_THREADS) {
        const int t = c0 + tid;
        unsigned mask = 0;
        if (t < T) {
            if (self_rank >= 0) mask |= 1u << self_rank;     // every token's row to its own rank (shared expert)
            for (int k = 0; k < keep; ++k) {
                const int e = sel[t * keep + k];
                if (e >= 0 && e < N_EXPERTS) mask |= 1u << (e / epr);
                else if (err) atomicCAS(err, 0, DEV_ERR_BAD_SLOT);
            }
        }
        int in_warp[LK_EP_MAX_RANKS];
        #pragma unroll
        for (int d = 0; d < LK_EP_MAX_RANKS; ++d) {
            const unsigned b = __ballot_sync(0xffffffffu, d < n_ranks && ((mask >> d) & 1u));
            in_warp[d] = __popc(b & ((1u << lane) - 1u));
            if (lane == 0) wc[d][warp] = __popc(b);
        }
        __syncthreads();
        if (tid < LK_EP_MAX_RANKS * 32) {
            const int d = tid >> 5, w = tid & 31;
            int s = 0;
            for (int i = 0; i < w; ++i) s += wc[d][i];
            pre[d][w] = s;
        }
        __syncthreads();
        if (t < T) {
            for (int d = 0; d < n_ranks; ++d)
                row_map[(size_t)t * n_ranks + d] = ((mask >> d) & 1u) ? base[d] + pre[d][warp] + in_warp[d] : -1;
        }
        __syncthreads();
        if (tid < LK_EP_MAX_RANKS) base[tid] += pre[tid][31] + wc[tid][31];
        __syncthreads();
    }
    if (tid == 0) {
        off[0] = 0;
        for (int d = 0; d < n_ranks; ++d) {
            int n = base[d];
            if (cap > 0 && n > cap) { if (err) atomicCAS(err, 0, DEV_ERR_BAD_SLOT); n = cap; }
            counts[d] = n; cnt[d] = n;
            off[d + 1] = off[d] + (cap > 0 ? cap : n);
        }
    }
    __syncthreads();
    for (int t = tid; t < T; t += EP_PLAN_THREADS) {           // same tokens as above: own writes are visible
        for (int d = 0; d < n_ranks; ++d) {
            int* m = row_map + (size_t)t * n_ranks + d;
            const int v = *m;
            if (v >= 0) *m = (cap > 0 && v >= cap) ? -1 : off[d] + v;
        }
    }
    if (cap > 0 && send) {                                     // unused rows of fixed-capacity blocks: no entries
        for (int d = 0; d < n_ranks; ++d) {
            for (int r = cnt[d] + (tid >> 4); r < cap; r += EP_PLAN_THREADS / 16) {
                int* h = (int*)(send + (size_t)(off[d] + r) * LK_EP_ROW_BYTES);
                h[tid & 15] = (tid & 15) < 8 ? -1 : 0;
            }
        }
    }
}

// one CTA per token: header and activations of each of its rows (x read once, written to every row)
__global__ void __launch_bounds__(256) k_ep_copy(const int* __restrict__ sel, const float* __restrict__ w,
                                                  const float* __restrict__ x, int keep, int n_ranks,
                                                  const int* __restrict__ row_map, uint8_t* send) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int t = blockIdx.x, tid = threadIdx.x;
    const int epr = N_EXPERTS / n_ranks;
    int rows[LK_EP_MAX_RANKS];
    #pragma unroll
    for (int d = 0; d < LK_EP_MAX_RANKS; ++d) rows[d] = d < n_ranks ? row_map[(size_t)t * n_ranks + d] : -1;
    if (tid < 16 * LK_EP_MAX_RANKS) {
        const int d = tid >> 4, j = tid & 15, k = j & 7;
        if (rows[d] >= 0) {
            int* h = (int*)(send + (size_t)rows[d] * LK_EP_ROW_BYTES);
            const int e = k < keep ? sel[t * keep + k] : -1;
            const bool mine = e >= d * epr && e < (d + 1) * epr;
            if (j < 8) h[j] = mine ? e - d * epr : -1;
            else ((float*)h)[j] = mine ? w[t * keep + k] : 0.f;
        }
    }
    // the q8 of x, computed once and written to every row of the token
    __shared__ __align__(16) int8_t q[HIDDEN];
    __shared__ float dq[HIDDEN / 32];
    ep_row_q8(x + (size_t)t * HIDDEN, q, dq, tid);
    __syncthreads();
    for (int i = tid; i < (HIDDEN + HIDDEN / 8) / 16; i += 256) {     // codes then scales, 16 bytes at a time
        const uint4 v = i < HIDDEN / 16 ? ((const uint4*)q)[i] : ((const uint4*)dq)[i - HIDDEN / 16];
        #pragma unroll
        for (int d = 0; d < LK_EP_MAX_RANKS; ++d)
            if (rows[d] >= 0) ((uint4*)(send + (size_t)rows[d] * LK_EP_ROW_BYTES + LK_EP_ROW_Q_OFF))[i] = v;
    }
}

// received rows -> fp32 activations [R][HIDDEN] (q * d; the expert kernels' q8 of these values gives back q)
__global__ void k_ep_dequant(const uint8_t* __restrict__ recv, int R, float* __restrict__ x) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // over R x HIDDEN / 4
    if (i >= (size_t)R * (HIDDEN / 4)) return;
    const int r = (int)(i / (HIDDEN / 4)), c = (int)(i % (HIDDEN / 4));
    const uint8_t* row = recv + (size_t)r * LK_EP_ROW_BYTES;
    const uint32_t qw = ((const uint32_t*)(row + LK_EP_ROW_Q_OFF))[c];
    const float d = ((const float*)(row + LK_EP_ROW_D_OFF))[(4 * c) / 32];
    ((float4*)(x + (size_t)r * HIDDEN))[c] = make_float4((float)(int8_t)qw * d, (float)(int8_t)(qw >> 8) * d,
                                                         (float)(int8_t)(qw >> 16) * d, (float)(int8_t)(qw >> 24) * d);
}

__global__ void k_ep_unpack(const uint8_t* __restrict__ recv, int R, int keep, int* sel, float* w) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R * keep) return;
    const int r = i / keep, k = i % keep;
    const EpRowHdr* h = (const EpRowHdr*)(recv + (size_t)r * LK_EP_ROW_BYTES);
    sel[i] = h->sel[k];
    w[i] = h->w[k];
}

__global__ void k_ep_combine(const float* __restrict__ ret, const int* __restrict__ row_map, int T, int n_ranks,
                             const float* __restrict__ hpart, const float* __restrict__ shared, float* h, float* moe) {
    pdl_trigger();                                // the next kernel may be scheduled; it waits for this grid
    pdl_wait();                                   // the predecessor grid has completed
    const int i = blockIdx.x * blockDim.x + threadIdx.x;       // float4 index over T x HIDDEN
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

int ep_plan(const int* sel, int T, int keep, int n_ranks, int self_rank, int cap, int* counts, int* row_map, uint8_t* send,
            int* err, cudaStream_t st) {
    launch_pdl_n(k_ep_plan, dim3(1), dim3(EP_PLAN_THREADS), 0, st, sel, T, keep, n_ranks, self_rank, cap, counts, row_map, send, err);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

// received rows -> sel/w [R][keep] and, for single-token slots, the slot tables directly (the general slot
// builder is a histogram over 256 experts with many barriers, ~20 us for a handful of rows)
__global__ void __launch_bounds__(EPS_THREADS) k_ep_slots(const uint8_t* __restrict__ recv, int R, int keep, int n_experts,
                                                          int* sel, float* w, SlotParams sp) {
    pdl_trigger();
    pdl_wait();
    ep_slots_dev(recv, R, keep, n_experts, sel, w, sp);
}

void launch_ep_slots(const void* recv, int R, int keep, int n_experts, int* sel, float* w, const SlotParams& sp, cudaStream_t st) {
    launch_pdl_n(k_ep_slots, dim3(1), dim3(EPS_THREADS), 0, st, (const uint8_t*)recv, R, keep, n_experts, sel, w, sp);
}

void launch_ep_unpack(const void* recv, int R, int keep, int* sel, float* w, float* x, cudaStream_t st) {
    const int n = R * keep;
    launch_pdl_n(k_ep_unpack, dim3((n + 255) / 256), dim3(256), 0, st, (const uint8_t*)recv, R, keep, sel, w);
    const size_t nx = (size_t)R * (HIDDEN / 4);
    if (x && R > 0) launch_pdl_n(k_ep_dequant, dim3((unsigned)((nx + 255) / 256)), dim3(256), 0, st, (const uint8_t*)recv, R, x);
}

}  // namespace lk

using namespace lk;

extern "C" {

int lk_ep_pack(const int* sel, const float* w, const float* x, int T, int keep, int n_ranks, int self_rank, int cap,
               void* send_rows, int* send_counts, int* row_map, int* err, lk_stream_t stream) {
    if (T < 0 || keep < 1 || keep > MAX_TOPK || n_ranks < 1 || n_ranks > LK_EP_MAX_RANKS || (N_EXPERTS % n_ranks) ||
        self_rank < -1 || self_rank >= n_ranks ||
        cap < 0 || (cap > 0 && cap < T) || !send_counts || (T > 0 && (!sel || !w || !x || !send_rows || !row_map)))
        return LK_ERR_ARG;
    if (((uintptr_t)send_rows & 15) || ((uintptr_t)x & 15)) return LK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    if (ep_plan(sel, T, keep, n_ranks, self_rank, cap, send_counts, row_map, (uint8_t*)send_rows, err, st)) return LK_ERR_CUDA;
    if (T > 0) launch_pdl_n(k_ep_copy, dim3(T), dim3(256), 0, st, sel, w, x, keep, n_ranks, (const int*)row_map, (uint8_t*)send_rows);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

int lk_ep_combine(const float* ret, const int* row_map, int T, int n_ranks, const float* h_partial, const float* shared,
                  float* h, float* moe, lk_stream_t stream) {
    if (T < 0 || n_ranks < 1 || n_ranks > LK_EP_MAX_RANKS || (T > 0 && (!row_map || (!ret && n_ranks > 0))))
        return LK_ERR_ARG;
    if (T == 0) return LK_OK;
    const int n = T * (HIDDEN / 4);
    launch_pdl_n(k_ep_combine, dim3((n + 255) / 256), dim3(256), 0, (cudaStream_t)stream, ret, row_map, T, n_ranks, h_partial, shared, h, moe);
    return cudaGetLastError() == cudaSuccess ? LK_OK : LK_ERR_CUDA;
}

}  // extern "C"
