// expert_gemv.cu -- grouped IQ2_XXS matvecs on q8 activations (the decode / narrow regime).
//
// Replaces tc_matvec<F_IQ2> + swiglu_q8 + the IQ2 down (reference src/fused_layer.cu:178-202, 334-341,
// launched at :605-608 and :548-550).  Work is a list of slots (expert, up to NT tokens); a persistent
// CTA per SM walks (slot, row tile) tiles.  Per CTA:
//   * one producer thread streams whole weight-row chunks (contiguous in the IQ2_XXS matrix) into a
//     shared-memory ring with cp.async.bulk (1-D TMA) and mbarrier transaction counts;
//   * consumer threads each own one 32-weight group (column block) of K and keep that group's q8
//     activations of the slot's tokens in registers; several consumer streams work on different chunks;
//   * per row a thread decodes its group with the 64 KB lane-private selector table (moe_device.cuh:
//     two conflict-free 32-bit lookups and two byte-permutes per 8 weights) and dp4a's the signed int8
//     weights against the activations: exact int32 group sums, scaled by d * (2*scale+1) * dx (the
//     format's 0.125 is applied after the reduction, exactly);
//   * 8 (row, token) partials per thread are summed over the warp (warp_reduce8) and across the row's
//     warps in a fixed order: deterministic, no atomics.
// gate/up: 2 streams x 224 consumers (7168/32 groups), tile = 32 h rows = 32 gate + 32 up rows (8 chunks
//   of 8 rows, even chunks to stream 0, odd to stream 1); SwiGLU and its q8 re-quantisation (per 32 rows
//   = one tile) are fused in.
// down: 8 streams x 64 consumers (2048/32 groups), tile = 64 rows (8 chunks of 8 rows, one per stream);
//   output y[entry][row] = w * (W_down h)[row].
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

__device__ __forceinline__ const uint8_t* slot_matrix(const ExpertParams& p, int e, int which) {
    // which: 0 gate, 1 up, 2 down
    if (e == SHARED_SLOT) return which == 0 ? p.sh_gate : which == 1 ? p.sh_up : p.sh_down;
    return which == 0 ? p.gate + (size_t)e * p.gate_stride
         : which == 1 ? p.up + (size_t)e * p.up_stride : p.down + (size_t)e * p.down_stride;
}

// q8 of this thread's 32-wide group of token `tok`'s activation row (zeros for a pad member)
__device__ __forceinline__ float load_q8_group(const float* x, int ld, int tok, int g, uint32_t (&xr)[8]) {
    float xv[32];
    if (tok >= 0) {
        const float4* src = (const float4*)(x + (size_t)tok * ld + g * 32);
        #pragma unroll
        for (int j = 0; j < 8; ++j) { const float4 v = src[j]; xv[4*j] = v.x; xv[4*j+1] = v.y; xv[4*j+2] = v.z; xv[4*j+3] = v.w; }
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) xv[j] = 0.0f;
    }
    int8_t q[32];
    const float d = quant_q8_group(xv, q);
    #pragma unroll
    for (int j = 0; j < 8; ++j)
        xr[j] = (uint32_t)(uint8_t)q[4*j] | ((uint32_t)(uint8_t)q[4*j+1] << 8) |
                ((uint32_t)(uint8_t)q[4*j+2] << 16) | ((uint32_t)(uint8_t)q[4*j+3] << 24);
    return d;
}

// one row of a staged chunk: this thread's group -> NT partials v[m]
template <int NT>
__device__ __forceinline__ void row_partials(const uint8_t* row, int goff, int boff, const uint32_t (&xr)[NT][8],
                                             const float (&dx)[NT], const unsigned char* tab, uint32_t lane4,
                                             float* v) {
    uint32_t aux0, aux1;
    load_group_smem(row, goff, aux0, aux1);
    const float d = load_d_smem(row, boff);
    int acc[NT];
    #pragma unroll
    for (int m = 0; m < NT; ++m) acc[m] = 0;
    iq2_dot_sel<NT>(aux0, aux1, xr, acc, tab, lane4);
    const int mult = (int)((aux1 >> 27) & 0x1Eu) + 1;          // 2*scale + 1
    #pragma unroll
    for (int m = 0; m < NT; ++m) v[m] = (float)(acc[m] * mult) * (d * dx[m]);
}

// ------------------------------------------------------------------ gate / up
constexpr int GU_KG = HIDDEN / 32;                   // 224 groups = consumers per stream
constexpr int GU_NS = 2;
constexpr int GU_SW = GU_KG / 32;                    // 7 warps per stream
constexpr int GU_CONS = GU_KG * GU_NS;               // 448
constexpr int GU_THREADS = GU_CONS + 32;             // + producer warp
constexpr int GU_ROWB = (HIDDEN / QK) * BLK_IQ2;     // 1848 bytes per row
constexpr int GU_CH_ROWS = 8;
constexpr int GU_CH_BYTES = GU_CH_ROWS * GU_ROWB;    // 14784
constexpr int GU_TILE = 32;                          // h rows per tile
constexpr int GU_CHUNKS = 2 * GU_TILE / GU_CH_ROWS;  // 8 per tile (0-3 gate, 4-7 up)
constexpr int GU_NST = GU_CHUNKS;                    // one tile in flight: chunk c always uses stage c
constexpr int GU_TILES_PER_SLOT = MOE_INTER / GU_TILE;   // 64

constexpr int GU_OFF_TAB = 0;
constexpr int GU_OFF_RING = GU_OFF_TAB + SEL_TAB_BYTES;
constexpr int GU_OFF_RED = GU_OFF_RING + GU_NST * GU_CH_BYTES;
constexpr int GU_OFF_GS = GU_OFF_RED + GU_NS * 2 * GU_SW * 32 * 4;
constexpr int GU_OFF_US = GU_OFF_GS + 2 * GU_TILE * MAX_NT * 4;
constexpr int GU_OFF_BAR = GU_OFF_US + 2 * GU_TILE * MAX_NT * 4;
constexpr int GU_OFF_ABORT = GU_OFF_BAR + 2 * GU_NST * 8;
constexpr int GU_SMEM = GU_OFF_ABORT + 16;

template <int NT>
__global__ void __launch_bounds__(GU_THREADS, 1) k_gate_up(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const unsigned char* tab = smem + GU_OFF_TAB;
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

    init_sel_table((uint32_t*)(smem + GU_OFF_TAB), tid, GU_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < GU_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], GU_SW); }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == GU_CONS / 32) {                       // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0;                          // copies issued; copy j uses stage j % 8 in phase j / 8
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const int e = p.slot_expert[s];
                const uint8_t* g = slot_matrix(p, e, 0);
                const uint8_t* u = slot_matrix(p, e, 1);
                for (int c = 0; c < GU_CHUNKS; ++c, ++it) {
                    if (*abort_flag || !mbar_wait(&empty[c], ((it / GU_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    const uint8_t* src = (c < 4 ? g : u) + (size_t)(rt * GU_TILE + (c & 3) * GU_CH_ROWS) * GU_ROWB;
                    mbar_arrive_expect_tx(&full[c], GU_CH_BYTES);
                    bulk_g2s(ring + c * GU_CH_BYTES, src, GU_CH_BYTES, &full[c]);
                }
            }
        drain:
            {   // every issued copy must land before the CTA may exit
                const uint32_t first = it > GU_NST ? it - GU_NST : 0;
                for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % GU_NST], (j / GU_NST) & 1, nullptr, 0);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int strm = tid / GU_KG, g = tid % GU_KG, sw = g >> 5;
    const int goff = 2 + BLK_IQ2 * (g >> 3) + 8 * (g & 7);
    const int boff = BLK_IQ2 * (g >> 3);
    const uint32_t lane4 = (uint32_t)lane << 2;
    constexpr int RB = 8 / NT;                        // rows per reduction batch (8 values)
    uint32_t xr[NT][8]; float dx[NT]; int xtok[NT];
    #pragma unroll
    for (int m = 0; m < NT; ++m) xtok[m] = -2;
    uint32_t ti = 0; int ebuf = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++ti) {
        const int s = tile % nslots, rt = tile / nslots;
        #pragma unroll
        for (int m = 0; m < NT; ++m) {
            const int tok = p.slot_tok[s * NT + m];
            if (tok != xtok[m]) { dx[m] = load_q8_group(p.x, p.ld_x, tok, g, xr[m]); xtok[m] = tok; }
        }
        const int tb = ti & 1;
        for (int e = 0; e < NT; ++e) {                // NT exchanges of 4 batches per stream and tile
            float kept = 0.0f;
            #pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const int b = e * 4 + bb;
                const int r0 = b * RB;                // first row of the batch within this stream's 32 rows
                const int ci = r0 >> 3, r8 = r0 & 7;
                const int c = strm + GU_NS * ci;      // chunk (= stage) index in the tile
                if (r8 == 0 && !*abort_flag && !mbar_wait(&full[c], ti & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1;
                const uint8_t* base = ring + c * GU_CH_BYTES + r8 * GU_ROWB;
                float v[8];
                #pragma unroll
                for (int rr = 0; rr < RB; ++rr) row_partials<NT>(base + rr * GU_ROWB, goff, boff, xr, dx, tab, lane4, v + rr * NT);
                if (r8 + RB == GU_CH_ROWS) { __syncwarp(); if (lane == 0) mbar_arrive(&empty[c]); }
                const float r = warp_reduce8(v, lane);
                if ((lane & 3) == bb) kept = r;
            }
            float* rb = red + ((strm * 2 + ebuf) * GU_SW) * 32;
            rb[sw * 32 + lane] = kept;
            named_bar_sync(1 + strm, GU_KG);
            if (sw == 0) {
                float a = rb[lane];
                #pragma unroll
                for (int w = 1; w < GU_SW; ++w) a += rb[w * 32 + lane];
                const int b = e * 4 + (lane & 3), vi = lane >> 2;
                const int row_s = b * RB + vi / NT, m = vi % NT;
                const int c = strm + GU_NS * (row_s >> 3);
                const int hrow = (c & 3) * GU_CH_ROWS + (row_s & 7);
                float* dst = c < 4 ? gs : us;
                dst[(tb * GU_TILE + hrow) * MAX_NT + m] = a * 0.125f;
            }
            ebuf ^= 1;
        }
        named_bar_sync(1 + GU_NS, GU_CONS);
        if (*abort_flag) break;                       // every consumer warp sees the same flag here
        // SwiGLU + q8 per 32 rows (this tile), one warp per token
        for (int m = warp; m < NT; m += GU_CONS / 32) {
            const int out = p.slot_out[s * NT + m];
            const float hv = lk_swiglu(gs[(tb * GU_TILE + lane) * MAX_NT + m], us[(tb * GU_TILE + lane) * MAX_NT + m]);
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
constexpr int DN_KG = MOE_INTER / 32;                // 64 groups per row = consumers per stream
constexpr int DN_NS = 8;
constexpr int DN_CONS = DN_KG * DN_NS;               // 512
constexpr int DN_THREADS = DN_CONS + 32;
constexpr int DN_ROWB = (MOE_INTER / QK) * BLK_IQ2;  // 528
constexpr int DN_CH_ROWS = 8;
constexpr int DN_CH_BYTES = DN_CH_ROWS * DN_ROWB;    // 4224
constexpr int DN_TILE = DN_CH_ROWS * DN_NS;          // 64 rows: chunk c -> stream c
constexpr int DN_DEPTH = 3;                          // tiles in flight
constexpr int DN_NST = DN_NS * DN_DEPTH;
constexpr int DN_TILES_PER_SLOT = HIDDEN / DN_TILE;  // 112

constexpr int DN_OFF_TAB = 0;
constexpr int DN_OFF_RING = DN_OFF_TAB + SEL_TAB_BYTES;
constexpr int DN_OFF_RED = DN_OFF_RING + DN_NST * DN_CH_BYTES;
constexpr int DN_OFF_BAR = DN_OFF_RED + DN_NS * 2 * 2 * 8 * 4;
constexpr int DN_OFF_ABORT = DN_OFF_BAR + 2 * DN_NST * 8;
constexpr int DN_SMEM = DN_OFF_ABORT + 16;

template <int NT>
__global__ void __launch_bounds__(DN_THREADS, 1) k_down(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const unsigned char* tab = smem + DN_OFF_TAB;
    uint8_t* ring = smem + DN_OFF_RING;
    float* red = (float*)(smem + DN_OFF_RED);
    uint64_t* full = (uint64_t*)(smem + DN_OFF_BAR);
    uint64_t* empty = full + DN_NST;
    volatile int* abort_flag = (volatile int*)(smem + DN_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int ntiles = nslots * DN_TILES_PER_SLOT;
    if ((int)blockIdx.x >= ntiles) return;

    init_sel_table((uint32_t*)(smem + DN_OFF_TAB), tid, DN_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < DN_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 2); }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == DN_CONS / 32) {                       // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0;
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const uint8_t* dw = slot_matrix(p, p.slot_expert[s], 2);
                for (int c = 0; c < DN_NS; ++c, ++it) {
                    const int st = it % DN_NST;
                    if (*abort_flag || !mbar_wait(&empty[st], ((it / DN_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    const uint8_t* src = dw + (size_t)(rt * DN_TILE + c * DN_CH_ROWS) * DN_ROWB;
                    mbar_arrive_expect_tx(&full[st], DN_CH_BYTES);
                    bulk_g2s(ring + st * DN_CH_BYTES, src, DN_CH_BYTES, &full[st]);
                }
            }
        drain:
            {
                const uint32_t first = it > DN_NST ? it - DN_NST : 0;
                for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % DN_NST], (j / DN_NST) & 1, nullptr, 0);
            }
        }
        return;
    }

    const int strm = tid / DN_KG, g = tid % DN_KG, hw = (tid >> 5) & 1;
    const int goff = 2 + BLK_IQ2 * (g >> 3) + 8 * (g & 7);
    const int boff = BLK_IQ2 * (g >> 3);
    const uint32_t lane4 = (uint32_t)lane << 2;
    constexpr int RB = 8 / NT;
    int ebuf = 0; uint32_t ti = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++ti) {
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
        const uint32_t it = ti * DN_NS + strm;
        const int st = it % DN_NST;
        if (!*abort_flag && !mbar_wait(&full[st], (it / DN_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1;
        const uint8_t* base = ring + st * DN_CH_BYTES;
        bool aborted = false;
        for (int b = 0; b < NT; ++b) {                // NT batches of RB rows (8 values each)
            float v[8];
            #pragma unroll
            for (int rr = 0; rr < RB; ++rr) row_partials<NT>(base + (b * RB + rr) * DN_ROWB, goff, boff, xr, dx, tab, lane4, v + rr * NT);
            if (b == NT - 1) { __syncwarp(); if (lane == 0) mbar_arrive(&empty[st]); }
            const float r = warp_reduce8(v, lane);
            float* rb = red + ((strm * 2 + ebuf) * 2) * 8;
            if ((lane & 3) == 0) rb[hw * 8 + (lane >> 2)] = r;
            named_bar_sync(1 + strm, DN_KG);
            if (*abort_flag) { aborted = true; break; }  // both warps of the stream see the same flag
            if (hw == 0 && lane < 8) {
                const float a = rb[lane] + rb[8 + lane];
                const int rr = lane / NT, m = lane % NT;
                const int row = rt * DN_TILE + strm * DN_CH_ROWS + b * RB + rr;
                float wv = 0.0f; int ov = -1;
                #pragma unroll
                for (int k = 0; k < NT; ++k) if (k == m) { wv = wm[k]; ov = outm[k]; }
                if (ov >= 0) p.y[(size_t)ov * HIDDEN + row] = wv * (a * 0.125f);
            }
            ebuf ^= 1;
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

void launch_gate_up1(const ExpertParams& p, int grid, cudaStream_t st);   // expert_gemv1.cu (one token)
void launch_down1(const ExpertParams& p, int grid, cudaStream_t st);

void launch_gate_up(const ExpertParams& p, int nt, int grid, cudaStream_t st) {
    switch (nt) {
        case 1: launch_gate_up1(p, grid, st); break;
        case 2: gu_launch<2>(p, grid, st); break;
        case 4: gu_launch<4>(p, grid, st); break;
        default: gu_launch<8>(p, grid, st); break;
    }
}
void launch_down(const ExpertParams& p, int nt, int grid, cudaStream_t st) {
    if (p.down_fmt == FMT_Q2K || p.down_fmt == FMT_Q3K) { launch_down1_kq(p, grid, st); return; }   // single-token slots only
    switch (nt) {
        case 1: launch_down1(p, grid, st); break;
        case 2: dn_launch<2>(p, grid, st); break;
        case 4: dn_launch<4>(p, grid, st); break;
        default: dn_launch<8>(p, grid, st); break;
    }
}

}  // namespace lk
