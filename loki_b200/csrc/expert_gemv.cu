// expert_gemv.cu -- grouped IQ2_XXS matvecs on q8 activations (the decode / narrow regime).
//
// Replaces tc_matvec<F_IQ2> + swiglu_q8 + the IQ2 down (reference src/fused_layer.cu:178-202, 334-341,
// launched at :605-608 and :548-550).  Work is a list of slots (expert, up to NT tokens); a persistent
// CTA walks (slot, row tile) tiles.  Per CTA:
//   * one producer warp streams whole weight-row chunks (contiguous in the IQ2_XXS matrix) into a
//     shared-memory ring with cp.async.bulk (1-D TMA) and mbarrier transaction counts;
//   * each consumer thread owns one 32-weight group (column block) of K and keeps that group's q8
//     activations of the slot's tokens in registers, so activations are read once per tile;
//   * per row it decodes its group with lane-private shared-memory tables (grid magnitudes by 64-bit
//     loads, sign selectors applied with one byte-permute per 4 weights) and dp4a's against the q8
//     activations: exact int32 group sums, scaled by d * (2*scale+1) * dx (the 0.125 is applied after
//     the reduction, exactly);
//   * 32 (row, token) partials per thread are summed across the row's threads by a warp
//     transpose-reduction and a fixed-order cross-warp sum (deterministic, no atomics).
// gate/up: 224 consumers (= 7168/32 groups), tile = 32 h rows = 32 gate + 32 up rows (8 chunks of 8
//   rows); the tile's SwiGLU and its q8 re-quantisation (per 32 rows, one tile) are fused in.
// down: 256 consumers = 4 row streams x 64 groups (K = 2048), tile = 128 rows (4 chunks of 32 rows);
//   output y[entry][row] = w * (W_down h)[row].
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

// ------------------------------------------------------------------ gate / up
constexpr int GU_CONS = HIDDEN / 32;                 // 224 consumer threads (7 warps)
constexpr int GU_CWARPS = GU_CONS / 32;
constexpr int GU_THREADS = GU_CONS + 32;             // + producer warp
constexpr int GU_ROWB = (HIDDEN / QK) * BLK_IQ2;     // 1848 bytes per row
constexpr int GU_CH_ROWS = 8;
constexpr int GU_CH_BYTES = GU_CH_ROWS * GU_ROWB;    // 14784
constexpr int GU_NST = 6;
constexpr int GU_TILE = 32;                          // h rows per tile
constexpr int GU_TILES_PER_SLOT = MOE_INTER / GU_TILE;   // 64
constexpr int GU_CHUNKS = 2 * GU_TILE / GU_CH_ROWS;       // 8 per tile (4 gate, 4 up)

constexpr int GU_OFF_GRID = 0;
constexpr int GU_OFF_SIGN = GU_OFF_GRID + GRID_TAB_BYTES;
constexpr int GU_OFF_RING = GU_OFF_SIGN + SIGN_TAB_BYTES;
constexpr int GU_OFF_RED = GU_OFF_RING + GU_NST * GU_CH_BYTES;
constexpr int GU_OFF_GS = GU_OFF_RED + 2 * GU_CWARPS * 32 * 4;
constexpr int GU_OFF_US = GU_OFF_GS + GU_TILE * MAX_NT * 4;
constexpr int GU_OFF_BAR = GU_OFF_US + GU_TILE * MAX_NT * 4;
constexpr int GU_OFF_ABORT = GU_OFF_BAR + 2 * GU_NST * 8;
constexpr int GU_SMEM = GU_OFF_ABORT + 16;

__device__ __forceinline__ const uint8_t* slot_matrix(const ExpertParams& p, int e, int which) {
    // which: 0 gate, 1 up, 2 down
    if (e == SHARED_SLOT) return which == 0 ? p.sh_gate : which == 1 ? p.sh_up : p.sh_down;
    return which == 0 ? p.gate + (size_t)e * p.gate_stride
         : which == 1 ? p.up + (size_t)e * p.up_stride : p.down + (size_t)e * p.down_stride;
}

template <int NT>
__global__ void __launch_bounds__(GU_THREADS, 1) k_gate_up(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint2* gtab = (uint2*)(smem + GU_OFF_GRID);
    uint32_t* stab = (uint32_t*)(smem + GU_OFF_SIGN);
    uint8_t* ring = smem + GU_OFF_RING;
    float* red = (float*)(smem + GU_OFF_RED);
    float* gs = (float*)(smem + GU_OFF_GS);
    float* us = (float*)(smem + GU_OFF_US);
    uint64_t* full = (uint64_t*)(smem + GU_OFF_BAR);
    uint64_t* empty = full + GU_NST;
    volatile int* abort_flag = (volatile int*)(smem + GU_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int ntiles = nslots * GU_TILES_PER_SLOT;
    if ((int)blockIdx.x >= ntiles) return;

    init_iq2_tables(gtab, stab, tid, GU_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < GU_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], GU_CWARPS); }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GU_CWARPS) {                          // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0; bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const int e = p.slot_expert[s];
                const uint8_t* g = slot_matrix(p, e, 0);
                const uint8_t* u = slot_matrix(p, e, 1);
                for (int c = 0; c < GU_CHUNKS; ++c, ++it) {
                    const int st = it % GU_NST;
                    if (!mbar_wait(&empty[st], ((it / GU_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { ok = false; break; }
                    const uint8_t* src = (c < 4 ? g : u) + (size_t)(rt * GU_TILE + (c & 3) * GU_CH_ROWS) * GU_ROWB;
                    mbar_arrive_expect_tx(&full[st], GU_CH_BYTES);
                    bulk_g2s(ring + st * GU_CH_BYTES, src, GU_CH_BYTES, &full[st]);
                }
            }
            // drain: every issued copy must land before the CTA may exit
            const uint32_t first = it > GU_NST ? it - GU_NST : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % GU_NST], (j / GU_NST) & 1, p.err, DEV_ERR_TIMEOUT_DRAIN);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int g = tid;                                // K group owned by this thread
    const int goff = 2 + BLK_IQ2 * (g >> 3) + 8 * (g & 7);
    const int boff = BLK_IQ2 * (g >> 3);
    const uint2* gt = gtab + lane;
    const uint32_t* stl = stab + lane;
    constexpr int RB = 32 / NT;                       // rows per reduction batch
    constexpr int NB = 2 * GU_TILE / RB;              // batches per tile
    uint32_t it = 0; int rbuf = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int s = tile % nslots, rt = tile / nslots;
        // this slot's tokens: q8 of this thread's 32-wide group, in registers
        uint32_t xr[NT][8]; float dx[NT];
        #pragma unroll
        for (int m = 0; m < NT; ++m) {
            const int tok = p.slot_tok[s * NT + m];
            float xv[32];
            if (tok >= 0) {
                const float4* src = (const float4*)(p.x + (size_t)tok * p.ld_x + g * 32);
                #pragma unroll
                for (int j = 0; j < 8; ++j) { const float4 v = src[j]; xv[4*j] = v.x; xv[4*j+1] = v.y; xv[4*j+2] = v.z; xv[4*j+3] = v.w; }
            } else {
                #pragma unroll
                for (int j = 0; j < 32; ++j) xv[j] = 0.0f;
            }
            int8_t q[32];
            dx[m] = quant_q8_group(xv, q);
            #pragma unroll
            for (int j = 0; j < 8; ++j)
                xr[m][j] = (uint32_t)(uint8_t)q[4*j] | ((uint32_t)(uint8_t)q[4*j+1] << 8) |
                           ((uint32_t)(uint8_t)q[4*j+2] << 16) | ((uint32_t)(uint8_t)q[4*j+3] << 24);
        }
        bool aborted = false;
        for (int b = 0; b < NB; ++b) {
            float v[32];
            #pragma unroll
            for (int rr = 0; rr < RB; ++rr) {
                const int trow = b * RB + rr;          // 0..63 within the tile (gate rows, then up rows)
                const int rc = trow % GU_CH_ROWS;
                if (rc == 0) { if (!mbar_wait(&full[it % GU_NST], (it / GU_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1; }
                const uint8_t* row = ring + (it % GU_NST) * GU_CH_BYTES + rc * GU_ROWB;
                uint32_t aux0, aux1;
                load_group_smem(row, goff, aux0, aux1);
                const float f = load_d_smem(row, boff) * (float)(2 * (int)(aux1 >> 28) + 1);
                #pragma unroll
                for (int m = 0; m < NT; ++m) {
                    const int isum = iq2_group_dot(aux0, aux1, xr[m], gt, stl);
                    v[rr * NT + m] = (float)isum * (f * dx[m]);
                }
                if (rc == GU_CH_ROWS - 1) { __syncwarp(); if (lane == 0) mbar_arrive(&empty[it % GU_NST]); ++it; }
            }
            const float tot = warp_transpose_reduce32(v, lane);
            float* rb_ = red + rbuf * GU_CWARPS * 32;
            rb_[warp * 32 + lane] = tot;
            named_bar_sync(1, GU_CONS);
            if (*abort_flag) { aborted = true; break; }   // every consumer warp sees the same flag here
            if (warp == 0) {
                float a = rb_[lane];
                #pragma unroll
                for (int w = 1; w < GU_CWARPS; ++w) a += rb_[w * 32 + lane];
                const int rr = lane / NT, m = lane % NT;
                const int trow = b * RB + rr;
                if (trow < GU_TILE) gs[trow * MAX_NT + m] = a * 0.125f;
                else us[(trow - GU_TILE) * MAX_NT + m] = a * 0.125f;
            }
            rbuf ^= 1;
        }
        if (aborted) break;
        named_bar_sync(1, GU_CONS);
        // SwiGLU + q8 per 32 rows (this tile), one warp per token
        for (int m = warp; m < NT; m += GU_CWARPS) {
            const int out = p.slot_out[s * NT + m];
            const float hv = lk_swiglu(gs[lane * MAX_NT + m], us[lane * MAX_NT + m]);
            float amax = fabsf(hv);
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
            if (out >= 0) {
                p.hq[(size_t)out * MOE_INTER + rt * GU_TILE + lane] = (int8_t)(int)rintf(hv * id);
                if (lane == 0) p.hd[(size_t)out * (MOE_INTER / 32) + rt] = d;
            }
        }
    }
}

// ------------------------------------------------------------------ down
constexpr int DN_GROUPS = MOE_INTER / 32;            // 64 groups per row
constexpr int DN_STREAMS = 4;
constexpr int DN_CONS = DN_GROUPS * DN_STREAMS;      // 256 consumers (8 warps)
constexpr int DN_CWARPS = DN_CONS / 32;
constexpr int DN_THREADS = DN_CONS + 32;
constexpr int DN_ROWB = (MOE_INTER / QK) * BLK_IQ2;  // 528
constexpr int DN_CH_ROWS = 32;
constexpr int DN_CH_BYTES = DN_CH_ROWS * DN_ROWB;    // 16896
constexpr int DN_NST = 5;
constexpr int DN_TILE = 128;
constexpr int DN_CHUNKS = DN_TILE / DN_CH_ROWS;      // 4
constexpr int DN_TILES_PER_SLOT = HIDDEN / DN_TILE;  // 56
constexpr int DN_SROWS = DN_CH_ROWS / DN_STREAMS;    // 8 rows of each chunk per stream

constexpr int DN_OFF_GRID = 0;
constexpr int DN_OFF_SIGN = DN_OFF_GRID + GRID_TAB_BYTES;
constexpr int DN_OFF_RING = DN_OFF_SIGN + SIGN_TAB_BYTES;
constexpr int DN_OFF_RED = DN_OFF_RING + DN_NST * DN_CH_BYTES;
constexpr int DN_OFF_BAR = DN_OFF_RED + 2 * DN_CWARPS * 32 * 4;
constexpr int DN_OFF_ABORT = DN_OFF_BAR + 2 * DN_NST * 8;
constexpr int DN_SMEM = DN_OFF_ABORT + 16;

template <int NT>
__global__ void __launch_bounds__(DN_THREADS, 1) k_down(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint2* gtab = (uint2*)(smem + DN_OFF_GRID);
    uint32_t* stab = (uint32_t*)(smem + DN_OFF_SIGN);
    uint8_t* ring = smem + DN_OFF_RING;
    float* red = (float*)(smem + DN_OFF_RED);
    uint64_t* full = (uint64_t*)(smem + DN_OFF_BAR);
    uint64_t* empty = full + DN_NST;
    volatile int* abort_flag = (volatile int*)(smem + DN_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int ntiles = nslots * DN_TILES_PER_SLOT;
    if ((int)blockIdx.x >= ntiles) return;

    init_iq2_tables(gtab, stab, tid, DN_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < DN_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], DN_CWARPS); }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == DN_CWARPS) {                          // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0; bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const uint8_t* dw = slot_matrix(p, p.slot_expert[s], 2);
                for (int c = 0; c < DN_CHUNKS; ++c, ++it) {
                    const int st = it % DN_NST;
                    if (!mbar_wait(&empty[st], ((it / DN_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { ok = false; break; }
                    const uint8_t* src = dw + (size_t)(rt * DN_TILE + c * DN_CH_ROWS) * DN_ROWB;
                    mbar_arrive_expect_tx(&full[st], DN_CH_BYTES);
                    bulk_g2s(ring + st * DN_CH_BYTES, src, DN_CH_BYTES, &full[st]);
                }
            }
            const uint32_t first = it > DN_NST ? it - DN_NST : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % DN_NST], (j / DN_NST) & 1, p.err, DEV_ERR_TIMEOUT_DRAIN);
        }
        return;
    }

    const int strm = tid / DN_GROUPS, g = tid % DN_GROUPS;
    const int goff = 2 + BLK_IQ2 * (g >> 3) + 8 * (g & 7);
    const int boff = BLK_IQ2 * (g >> 3);
    const uint2* gt = gtab + lane;
    const uint32_t* stl = stab + lane;
    constexpr int RB = 32 / NT;                       // rows per reduction batch (per stream)
    constexpr int ROWS_PER_STREAM = DN_TILE / DN_STREAMS;   // 32
    constexpr int NB = ROWS_PER_STREAM / RB;
    uint32_t it = 0; int rbuf = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int s = tile % nslots, rt = tile / nslots;
        uint32_t xr[NT][8]; float dx[NT]; float wm[NT]; int outm[NT];
        #pragma unroll
        for (int m = 0; m < NT; ++m) {
            const int out = p.slot_out[s * NT + m];
            outm[m] = out; wm[m] = p.slot_w[s * NT + m];
            if (out >= 0) {
                const uint4* src = (const uint4*)(p.hq + (size_t)out * MOE_INTER + g * 32);
                const uint4 a = src[0], c = src[1];
                xr[m][0] = a.x; xr[m][1] = a.y; xr[m][2] = a.z; xr[m][3] = a.w;
                xr[m][4] = c.x; xr[m][5] = c.y; xr[m][6] = c.z; xr[m][7] = c.w;
                dx[m] = p.hd[(size_t)out * (MOE_INTER / 32) + g];
            } else {
                #pragma unroll
                for (int j = 0; j < 8; ++j) xr[m][j] = 0u;
                dx[m] = 0.0f;
            }
        }
        bool aborted = false;
        for (int b = 0; b < NB; ++b) {
            float v[32];
            #pragma unroll
            for (int rr = 0; rr < RB; ++rr) {
                const int srow = b * RB + rr;         // 0..31 within this stream's share of the tile
                const int ri = srow % DN_SROWS;
                if (ri == 0) { if (!mbar_wait(&full[it % DN_NST], (it / DN_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1; }
                const uint8_t* row = ring + (it % DN_NST) * DN_CH_BYTES + (strm * DN_SROWS + ri) * DN_ROWB;
                uint32_t aux0, aux1;
                load_group_smem(row, goff, aux0, aux1);
                const float f = load_d_smem(row, boff) * (float)(2 * (int)(aux1 >> 28) + 1);
                #pragma unroll
                for (int m = 0; m < NT; ++m) {
                    const int isum = iq2_group_dot(aux0, aux1, xr[m], gt, stl);
                    v[rr * NT + m] = (float)isum * (f * dx[m]);
                }
                if (ri == DN_SROWS - 1) { __syncwarp(); if (lane == 0) mbar_arrive(&empty[it % DN_NST]); ++it; }
            }
            const float tot = warp_transpose_reduce32(v, lane);
            float* rb_ = red + rbuf * DN_CWARPS * 32;
            rb_[warp * 32 + lane] = tot;
            named_bar_sync(1, DN_CONS);
            if (*abort_flag) { aborted = true; break; }
            if ((warp & 1) == 0) {                    // first warp of each stream: combine its 2 warps
                const float a = rb_[warp * 32 + lane] + rb_[(warp + 1) * 32 + lane];
                const int rr = lane / NT, m = lane % NT;
                const int srow = b * RB + rr;
                const int row = rt * DN_TILE + (srow / DN_SROWS) * DN_CH_ROWS + strm * DN_SROWS + (srow % DN_SROWS);
                float wv = 0.0f; int ov = -1;
                #pragma unroll
                for (int k = 0; k < NT; ++k) if (k == m) { wv = wm[k]; ov = outm[k]; }
                if (ov >= 0) p.y[(size_t)ov * HIDDEN + row] = wv * (a * 0.125f);
            }
            rbuf ^= 1;
        }
        if (aborted) break;
    }
}

// ------------------------------------------------------------------ launchers
template <int NT> static void gu_launch(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_gate_up<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GU_SMEM); attr = true; }
    k_gate_up<NT><<<grid, GU_THREADS, GU_SMEM, st>>>(p);
}
template <int NT> static void dn_launch(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_down<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DN_SMEM); attr = true; }
    k_down<NT><<<grid, DN_THREADS, DN_SMEM, st>>>(p);
}

void launch_gate_up(const ExpertParams& p, int nt, int grid, cudaStream_t st) {
    switch (nt) {
        case 1: gu_launch<1>(p, grid, st); break;
        case 2: gu_launch<2>(p, grid, st); break;
        case 4: gu_launch<4>(p, grid, st); break;
        default: gu_launch<8>(p, grid, st); break;
    }
}
void launch_down(const ExpertParams& p, int nt, int grid, cudaStream_t st) {
    switch (nt) {
        case 1: dn_launch<1>(p, grid, st); break;
        case 2: dn_launch<2>(p, grid, st); break;
        case 4: dn_launch<4>(p, grid, st); break;
        default: dn_launch<8>(p, grid, st); break;
    }
}

// ------------------------------------------------------------------ combine
__global__ void k_combine(CombineParams p) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;       // float4 index over T x HIDDEN
    const int per = HIDDEN / 4;
    if (i >= p.T * per) return;
    const int t = i / per, c = i % per;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < p.keep; ++k) {
        const float4 v = ((const float4*)(p.y + ((size_t)t * p.keep + k) * HIDDEN))[c];
        r.x += v.x; r.y += v.y; r.z += v.z; r.w += v.w;
    }
    if (p.moe) ((float4*)(p.moe + (size_t)t * p.ld_out))[c] = r;
    float4 h = ((const float4*)(p.resid + (size_t)t * p.ld_out))[c];
    if (p.with_shared) {
        const float4 v = ((const float4*)(p.y + ((size_t)p.T * p.keep + t) * HIDDEN))[c];
        h.x += v.x; h.y += v.y; h.z += v.z; h.w += v.w;
    }
    if (p.shared) {
        const float4 v = ((const float4*)(p.shared + (size_t)t * HIDDEN))[c];
        h.x += v.x; h.y += v.y; h.z += v.z; h.w += v.w;
    }
    h.x += r.x; h.y += r.y; h.z += r.z; h.w += r.w;
    if (p.h) ((float4*)(p.h + (size_t)t * p.ld_out))[c] = h;
}

void launch_combine(const CombineParams& p, cudaStream_t st) {
    const int n = p.T * (HIDDEN / 4);
    k_combine<<<(n + 255) / 256, 256, 0, st>>>(p);
}

// ------------------------------------------------------------------ seeded weight generation
// one CTA = 64 consecutive blocks of one expert matrix, staged in shared memory, written as 16-byte words
__global__ void __launch_bounds__(64) k_gen_iq2(uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0,
                                                int rows, int K, int64_t stride) {
    __shared__ __align__(16) uint8_t buf[64 * BLK_IQ2];
    const int e = expert0 + blockIdx.y;
    const uint64_t key = iq2_gen_key(seed, (uint32_t)layer, (uint32_t)matrix, (uint32_t)e);
    const int64_t nblk = (int64_t)rows * (K / QK);
    const int64_t b0 = (int64_t)blockIdx.x * 64;
    const int64_t b = b0 + threadIdx.x;
    if (b < nblk) iq2_gen_block(key, (uint64_t)b, buf + threadIdx.x * BLK_IQ2);
    __syncthreads();
    uint8_t* out = dst + (size_t)blockIdx.y * stride + (size_t)b0 * BLK_IQ2;
    const int nb = (int)(nblk - b0 < 64 ? nblk - b0 : 64);
    const int bytes = nb * BLK_IQ2;
    if (((uintptr_t)out & 15) == 0 && (bytes & 15) == 0) {
        for (int i = threadIdx.x; i < bytes / 16; i += 64) ((uint4*)out)[i] = ((const uint4*)buf)[i];
    } else {
        for (int i = threadIdx.x; i < bytes; i += 64) out[i] = buf[i];
    }
}

void launch_gen_iq2(uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                    int64_t stride, cudaStream_t st) {
    const int64_t nblk = (int64_t)rows * (K / QK);
    dim3 grid((unsigned)((nblk + 63) / 64), (unsigned)n_exp);
    k_gen_iq2<<<grid, 64, 0, st>>>(dst, seed, layer, matrix, expert0, rows, K, stride);
}

int num_sms(int device) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n;
}

}  // namespace lk
