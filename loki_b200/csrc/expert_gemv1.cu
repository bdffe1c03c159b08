// expert_gemv1.cu -- the single-token (decode, NT = 1) grouped IQ2_XXS matvecs.
//
// Same contract as expert_gemv.cu's kernels for NT = 1 (slot tables in, hq/hd and y out).  Both kernels
// stream weight rows into a shared-memory ring with cp.async.bulk from one producer thread.
//   gate/up (k_gate_up1): one 32-weight K group per consumer thread, 4 streams of 224 threads, decode
//     with the signs applied to the activations (moe_device.cuh, iq2_dot_xs); SwiGLU and the q8 of h are
//     fused in;
//   down (k_down1): a warp computes whole row dot products -- lane l owns the K groups l and l + 32 --
//     over units of 32 rows (one 16 896-byte copy each), 4 warps per unit, each warp 8 rows: 8 row
//     sums by one warp_reduce8, y = w * 0.125 * sum.  Decode: the selector table (iq2_dot1), which
//     measured faster here than the sign-on-activation core.
#include "../../include/loki_ep.h"
#include "moe_internal.h"
#include "moe_device.cuh"
#include "ep_device.cuh"

namespace lk {

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v; asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a)); return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v; asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a)); return v;
}

// group starting sh/8 bytes past the 4-byte-aligned shared address b: aux0, aux1 via three aligned words
__device__ __forceinline__ void lds_group(uint32_t b, uint32_t sh, uint32_t& aux0, uint32_t& aux1) {
    const uint32_t w0 = lds_u32(b), w1 = lds_u32(b + 4), w2 = lds_u32(b + 8);
    aux0 = __funnelshift_r(w0, w1, sh);
    aux1 = __funnelshift_r(w1, w2, sh);
}

// selector-table dot with the table at shared address tab_s (row i at tab_s + 256 i)
__device__ __forceinline__ int iq2_dot1(uint32_t aux0, uint32_t aux1, const uint32_t (&x)[8], uint32_t tab_s, uint32_t lane4) {
    const uint32_t a1s = aux1 >> 13;
    const uint32_t so = tab_s + (128u | lane4);
    const uint32_t gb = tab_s + lane4;
    const uint32_t sa[4] = { ((aux1 << 8) & 0x7F00u) + so, ((aux1 << 1) & 0x7F00u) + so,
                             ((a1s << 7) & 0x7F00u) + so, (a1s & 0x7F00u) + so };
    int acc = 0;
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint32_t ga = gb + __byte_perm(aux0, 0u, 0x4404u | (uint32_t)(l << 4));   // + idx << 8
        const uint32_t sel = lds_u32(ga) | lds_u32(sa[l]);
        acc = __dp4a((int)__byte_perm(IQ2_POS, IQ2_NEG, sel), (int)x[2 * l], acc);
        acc = __dp4a((int)__byte_perm(IQ2_POS, IQ2_NEG, sel >> 16), (int)x[2 * l + 1], acc);
    }
    return acc;
}

// q8 of the 32-wide group g of an fp32 row (global)
__device__ __forceinline__ float q8_group_global(const float* row, int g, uint32_t (&xr)[8]) {
    float xv[32];
    const float4* src = (const float4*)(row + g * 32);
    #pragma unroll
    for (int j = 0; j < 8; ++j) { const float4 v = src[j]; xv[4*j] = v.x; xv[4*j+1] = v.y; xv[4*j+2] = v.z; xv[4*j+3] = v.w; }
    int8_t q[32];
    const float d = quant_q8_group(xv, q);
    #pragma unroll
    for (int j = 0; j < 8; ++j)
        xr[j] = (uint32_t)(uint8_t)q[4*j] | ((uint32_t)(uint8_t)q[4*j+1] << 8) |
                ((uint32_t)(uint8_t)q[4*j+2] << 16) | ((uint32_t)(uint8_t)q[4*j+3] << 24);
    return d;
}

__device__ __forceinline__ const uint8_t* slot_matrix1(const ExpertParams& p, int e, int which) {
    if (e == SHARED_SLOT) return which == 0 ? p.sh_gate : which == 1 ? p.sh_up : p.sh_down;
    return which == 0 ? p.gate + (size_t)e * p.gate_stride
         : which == 1 ? p.up + (size_t)e * p.up_stride : p.down + (size_t)e * p.down_stride;
}

// ------------------------------------------------------------------ gate / up, one token per slot
// 4 consumer streams x 224 threads (one 32-weight K group each) + a producer warp.  A tile is 32 h rows
// = 8 chunks of 8 rows (chunks 0-3 gate, 4-7 up), each chunk one 14 784-byte bulk copy into stage c.
// Stream k takes chunk k (gate rows 8k..8k+7) and then chunk k + 4 (the same up rows).  Per chunk a
// warp sums its 8 row partials with warp_reduce8.  At the end of the tile every consumer leaves one
// value in a double-buffered shared array, and after one barrier warp 0 adds the 7 warps of each row
// (fixed order), applies SwiGLU and quantises the tile's 32 h values to q8.
// A CTA walks a contiguous range of (slot, row tile) pairs, so the activations are re-quantised only
// when the slot's token changes.
constexpr int G1_NS = 4;
constexpr int G1_KG = HIDDEN / 32;                   // 224 consumers per stream
constexpr int G1_SW = G1_KG / 32;                    // 7 warps per stream
constexpr int G1_CONS = G1_NS * G1_KG;               // 896
constexpr int G1_THREADS = G1_CONS + 32;             // + producer warp
constexpr int G1_ROWB = (HIDDEN / QK) * BLK_IQ2;     // 1848
constexpr int G1_CROWS = 8;
constexpr int G1_CBYTES = G1_CROWS * G1_ROWB;        // 14784
constexpr int G1_TILE = 32;                          // h rows per tile
constexpr int G1_CPT = 2 * G1_TILE / G1_CROWS;       // 8 chunks per tile; chunk c always uses stage c
constexpr int G1_TILES_PER_SLOT = MOE_INTER / G1_TILE;   // 64
static_assert(G1_CPT == 2 * G1_NS, "each stream takes one gate and one up chunk per tile");

constexpr int G1_OFF_TAB = 0;
constexpr int G1_OFF_RING = G1_OFF_TAB + XS_TAB_BYTES;
constexpr int G1_OFF_RED = G1_OFF_RING + G1_CPT * G1_CBYTES;
constexpr int G1_OFF_BAR = G1_OFF_RED + 2 * G1_NS * G1_SW * 32 * 4;
constexpr int G1_OFF_ABORT = G1_OFF_BAR + 2 * G1_CPT * 8;
constexpr int G1_SMEM = G1_OFF_ABORT + 16;
static_assert(G1_SMEM <= 232448, "gate/up shared-memory layout exceeds the 227 KB a CTA can have");

__global__ void __launch_bounds__(G1_THREADS, 1) k_gate_up1(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const unsigned char* tab = smem + G1_OFF_TAB;
    uint8_t* ring = smem + G1_OFF_RING;
    float* red = (float*)(smem + G1_OFF_RED);
    uint64_t* full = (uint64_t*)(smem + G1_OFF_BAR);
    uint64_t* empty = full + G1_CPT;
    volatile int* abort_flag = (volatile int*)(smem + G1_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // shared-memory setup overlaps the previous kernel; everything it produced is read after pdl_wait
    init_xs_table(smem + G1_OFF_TAB, tid, G1_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int c = 0; c < G1_CPT; ++c) { mbar_init(&full[c], 1); mbar_init(&empty[c], G1_SW); }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    if (p.epw.mb) ep_rows_wait_slots<G1_THREADS>(p.epw);   // expert-parallel: the rows wait + slot tables, per CTA
    const int nslots = *p.nslots;
    const int ntiles = nslots * G1_TILES_PER_SLOT;
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x);
    const int t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    if (t0 >= t1) return;

    if (warp == G1_CONS / 32) {                       // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0;                          // copies issued; copy it uses stage it % 8, phase it / 8
            for (int tile = t0; tile < t1; ++tile) {
                const int s = tile / G1_TILES_PER_SLOT, rt = tile % G1_TILES_PER_SLOT;
                const int e = p.slot_expert[s];
                const uint8_t* g = slot_matrix1(p, e, 0);
                const uint8_t* u = slot_matrix1(p, e, 1);
                for (int c = 0; c < G1_CPT; ++c, ++it) {
                    if (*abort_flag || !mbar_wait(&empty[c], ((it / G1_CPT) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    const uint8_t* src = (c < G1_NS ? g : u) + (size_t)(rt * G1_TILE + (c % G1_NS) * G1_CROWS) * G1_ROWB;
                    mbar_arrive_expect_tx(&full[c], G1_CBYTES);
                    bulk_g2s(ring + c * G1_CBYTES, src, G1_CBYTES, &full[c]);
                }
            }
        drain:
            {   // every issued copy must land before the CTA may exit
                const uint32_t first = it > G1_CPT ? it - G1_CPT : 0;
                for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % G1_CPT], (j / G1_CPT) & 1, nullptr, 0);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int strm = tid / G1_KG, g = tid % G1_KG, sw = g >> 5;
    const int goff = 2 + BLK_IQ2 * (g >> 3) + 8 * (g & 7);
    const int boff = BLK_IQ2 * (g >> 3);
    const uint32_t lane4 = (uint32_t)lane << 2, lane8 = (uint32_t)lane << 3;
    uint32_t xr[8], nx[8];
    float dx = 0.0f;
    int xtok = -2;
    bool aborted = false;
    uint32_t ti = 0;
    for (int tile = t0; tile < t1; ++tile, ++ti) {
        const int s = tile / G1_TILES_PER_SLOT, rt = tile % G1_TILES_PER_SLOT;
        const int tok = p.slot_tok[s];
        if (tok != xtok) {
            if (tok == 0 && p.xq) {                  // quantised by the router (one-token forward)
                const uint4 a0 = ((const uint4*)(p.xq + g * 32))[0], a1 = ((const uint4*)(p.xq + g * 32))[1];
                const uint4 b0 = ((const uint4*)(p.xqn + g * 32))[0], b1 = ((const uint4*)(p.xqn + g * 32))[1];
                xr[0] = a0.x; xr[1] = a0.y; xr[2] = a0.z; xr[3] = a0.w; xr[4] = a1.x; xr[5] = a1.y; xr[6] = a1.z; xr[7] = a1.w;
                nx[0] = b0.x; nx[1] = b0.y; nx[2] = b0.z; nx[3] = b0.w; nx[4] = b1.x; nx[5] = b1.y; nx[6] = b1.z; nx[7] = b1.w;
                dx = p.xd[g];
            } else {
                if (tok >= 0 && p.xrows) {           // an expert-parallel row: its q8 codes and scale as sent
                    const uint8_t* row = p.xrows + (size_t)tok * LK_EP_ROW_BYTES;
                    const uint4 a0 = ((const uint4*)(row + LK_EP_ROW_Q_OFF + g * 32))[0];
                    const uint4 a1 = ((const uint4*)(row + LK_EP_ROW_Q_OFF + g * 32))[1];
                    xr[0] = a0.x; xr[1] = a0.y; xr[2] = a0.z; xr[3] = a0.w; xr[4] = a1.x; xr[5] = a1.y; xr[6] = a1.z; xr[7] = a1.w;
                    dx = ((const float*)(row + LK_EP_ROW_D_OFF))[g];
                } else if (tok >= 0) dx = q8_group_global(p.x + (size_t)tok * p.ld_x, g, xr);
                else { dx = 0.0f; for (int j = 0; j < 8; ++j) xr[j] = 0u; }
                #pragma unroll
                for (int j = 0; j < 8; ++j) nx[j] = neg_i8x4(xr[j]);
            }
            xtok = tok;
        }
        float kept = 0.0f;
        #pragma unroll
        for (int bb = 0; bb < 2; ++bb) {
            const int c = strm + G1_NS * bb;
            if (!aborted && !mbar_wait(&full[c], ti & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { aborted = true; *abort_flag = 1; }
            const uint8_t* base = ring + c * G1_CBYTES;
            float v[8];
            #pragma unroll
            for (int rr = 0; rr < G1_CROWS; ++rr) {
                const uint8_t* row = base + rr * G1_ROWB;
                uint32_t aux0, aux1;
                load_group_smem(row, goff, aux0, aux1);
                const float d = load_d_smem(row, boff);
                const int acc = iq2_dot_xs(aux0, aux1, xr, nx, tab, lane4, lane8);
                const int mult = (int)((aux1 >> 27) & 0x1Eu) + 1;          // 2*scale + 1
                v[rr] = (float)(acc * mult) * (d * dx);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[c]);
            const float r = warp_reduce8(v, lane);    // lane l: row l >> 2 of the chunk
            if ((lane & 3) == bb) kept = r;
        }
        float* rb = red + (ti & 1) * (G1_NS * G1_SW * 32);
        rb[(strm * G1_SW + sw) * 32 + lane] = kept;
        if (named_bar_or(1, G1_CONS, aborted)) break;   // uniform: every consumer leaves here together
        if (warp == 0) {                              // h row `lane` of the tile: stream lane/8, chunk row lane%8
            const float* q = rb + (lane >> 3) * G1_SW * 32 + (lane & 7) * 4;
            float ga = q[0], ua = q[1];
            #pragma unroll
            for (int w = 1; w < G1_SW; ++w) { ga += q[w * 32]; ua += q[w * 32 + 1]; }
            const float hv = lk_swiglu(ga * 0.125f, ua * 0.125f);
            float amax = fabsf(hv);
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
            const int out = p.slot_out[s];
            if (out >= 0) {
                p.hq[(size_t)out * MOE_INTER + rt * G1_TILE + lane] = (int8_t)(int)rintf(hv * id);
                if (lane == 0) p.hd[(size_t)out * (MOE_INTER / 32) + rt] = d;
            }
        }
    }
}

// ------------------------------------------------------------------ down, one token
constexpr int D1_WARPS = 16;
constexpr int D1_THREADS = (D1_WARPS + 1) * 32;
constexpr int D1_ROWB = (MOE_INTER / QK) * BLK_IQ2;  // 528
constexpr int D1_UROWS = 8;                          // rows per warp
constexpr int D1_CROWS = 32;                         // rows per unit = one bulk copy (16 896 B: copies under
constexpr int D1_CBYTES = D1_CROWS * D1_ROWB;        //   ~8 KB cannot stream HBM at full rate)
constexpr int D1_GROUPS = D1_WARPS / (D1_CROWS / D1_UROWS);   // 4 groups of 4 warps, one unit each at a time
constexpr int D1_NST = 2 * D1_GROUPS;                // group g always uses stages g and g + 4
constexpr int D1_UNITS_PER_SLOT = HIDDEN / D1_CROWS; // 224

constexpr int D1_OFF_TAB = 0;
constexpr int D1_OFF_RING = D1_OFF_TAB + SEL_TAB_BYTES;
constexpr int D1_OFF_BAR = D1_OFF_RING + D1_NST * D1_CBYTES;
constexpr int D1_OFF_ABORT = D1_OFF_BAR + 2 * D1_NST * 8;
constexpr int D1_SMEM = D1_OFF_ABORT + 16;

// A CTA takes a contiguous range of units (32 output rows of one slot): 9 slots x 224 units over 148 CTAs
// is 13 or 14 units each.  Local unit j goes to stage j % 8 and to warp group j % 4.
__global__ void __launch_bounds__(D1_THREADS, 1) k_down1(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem + D1_OFF_RING;
    uint64_t* full = (uint64_t*)(smem + D1_OFF_BAR);
    uint64_t* empty = full + D1_NST;
    volatile int* abort_flag = (volatile int*)(smem + D1_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    init_sel_table((uint32_t*)(smem + D1_OFF_TAB), tid, D1_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < D1_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], D1_CROWS / D1_UROWS); }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const int nslots = *p.nslots;
    const int nunits = nslots * D1_UNITS_PER_SLOT;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x);
    const int nu = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x) - u0;
    if (nu <= 0) return;
    if (warp == D1_WARPS) {                           // ---------------- producer
        if (lane == 0) {
            int j = 0;
            for (; j < nu; ++j) {
                const int u = u0 + j, s = u / D1_UNITS_PER_SLOT, cu = u % D1_UNITS_PER_SLOT;
                const int st = j % D1_NST;
                if (*abort_flag || !mbar_wait(&empty[st], ((j / D1_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                const uint8_t* dw = slot_matrix1(p, p.slot_expert[s], 2);
                mbar_arrive_expect_tx(&full[st], D1_CBYTES);
                bulk_g2s(ring + st * D1_CBYTES, dw + (size_t)cu * D1_CBYTES, D1_CBYTES, &full[st]);
            }
            {   // every issued copy must land before the CTA may exit
                const int first = j > D1_NST ? j - D1_NST : 0;
                for (int i = first; i < j; ++i) mbar_wait(&full[i % D1_NST], (i / D1_NST) & 1, nullptr, 0);
            }
        }
        return;
    }

    const uint32_t tab_s = smem_u32(smem + D1_OFF_TAB);
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t lane4 = (uint32_t)lane << 2;
    const uint32_t goff0 = 2u + BLK_IQ2 * (lane >> 3) + 8u * (lane & 7);   // groups lane, lane + 32 (+264)
    const uint32_t gal = goff0 & ~3u, gsh = (goff0 & 3u) * 8u;
    const uint32_t boff0 = BLK_IQ2 * (lane >> 3);
    const int grp = warp / (D1_CROWS / D1_UROWS), sub = warp % (D1_CROWS / D1_UROWS);
    uint32_t xr[2][8]; float dx[2] = {0.0f, 0.0f};
    int xslot = -1, out = -1;
    float wv = 0.0f;
    float* yrow = nullptr;
    for (int j = grp; j < nu; j += D1_GROUPS) {
        const int u = u0 + j, s = u / D1_UNITS_PER_SLOT, cu = u % D1_UNITS_PER_SLOT;
        if (s != xslot) {                             // this slot's h (q8) as the activations
            xslot = s; out = p.slot_out[s]; wv = p.slot_w[s];
            yrow = out < 0 ? nullptr : (p.ydst ? p.ydst[s] : p.y + (size_t)out * HIDDEN);
            #pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int g = lane + 32 * q;
                if (out >= 0) {
                    const uint4* src = (const uint4*)(p.hq + (size_t)out * MOE_INTER + g * 32);
                    const uint4 a = src[0], c = src[1];
                    xr[q][0] = a.x; xr[q][1] = a.y; xr[q][2] = a.z; xr[q][3] = a.w;
                    xr[q][4] = c.x; xr[q][5] = c.y; xr[q][6] = c.z; xr[q][7] = c.w;
                    dx[q] = p.hd[(size_t)out * (MOE_INTER / 32) + g];
                } else {
                    #pragma unroll
                    for (int w = 0; w < 8; ++w) xr[q][w] = 0u;
                    dx[q] = 0.0f;
                }
            }
        }
        const int st = j % D1_NST;
        if (!mbar_wait(&full[st], (j / D1_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { *abort_flag = 1; break; }
        const uint32_t ub = ring_s + st * D1_CBYTES + sub * D1_UROWS * D1_ROWB;
        const uint32_t ubg = ub + gal, ubd = ub + boff0;
        float v[8];
        #pragma unroll
        for (int r = 0; r < D1_UROWS; ++r) {
            float a = 0.0f;
            #pragma unroll
            for (int q = 0; q < 2; ++q) {
                uint32_t aux0, aux1;
                lds_group(ubg + r * D1_ROWB + 264u * q, gsh, aux0, aux1);
                const float d = __half2float(__ushort_as_half(lds_u16(ubd + r * D1_ROWB + 264u * q)));
                const int isum = iq2_dot1(aux0, aux1, xr[q], tab_s, lane4);
                a = fmaf((float)(isum * ((int)((aux1 >> 27) & 0x1Eu) + 1)), d * dx[q], a);
            }
            v[r] = a;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        const float sum = warp_reduce8(v, lane);   // lane l: row (l >> 2), 4 replicas
        const int row0 = cu * D1_CROWS + sub * D1_UROWS;
        if ((lane & 3) == 0 && yrow) yrow[row0 + (lane >> 2)] = wv * (sum * 0.125f);
        if (*abort_flag) break;
    }
}

void launch_gate_up1(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_gate_up1, cudaFuncAttributeMaxDynamicSharedMemorySize, G1_SMEM); attr = true; }
    launch_pdl(k_gate_up1, dim3(grid), dim3(G1_THREADS), G1_SMEM, st, p);
}
void launch_down1(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_down1, cudaFuncAttributeMaxDynamicSharedMemorySize, D1_SMEM); attr = true; }
    launch_pdl(k_down1, dim3(grid), dim3(D1_THREADS), D1_SMEM, st, p);
}

}  // namespace lk
