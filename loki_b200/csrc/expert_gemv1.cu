// expert_gemv1.cu -- the single-token (decode, NT = 1) grouped IQ2_XXS matvecs, one warp per row.
//
// Same contract as expert_gemv.cu's kernels for NT = 1 (slot tables in, hq/hd and y out), organised for one token: a warp computes whole row dot products -- lane l owns the K groups
// l, l+32, ... and holds their q8 activations in registers -- so rows need no cross-warp reduction and
// no named barriers.  A producer thread streams small row units into a deep shared-memory ring with
// cp.async.bulk; each unit is consumed by one warp.
//   gate/up unit = 2 h rows (2 gate rows + 2 up rows, two 3 696-byte copies); the warp writes
//     h = silu(g)*u for its 2 rows into a per-tile shared buffer, and the last of the 16 units of a
//     32-row tile (a shared-memory count) quantises the tile to q8 (hq, hd);
//   down: copies of 32 rows (16 896 bytes), 4 per 128-row tile; warp w takes 8 rows of copy w/4: 8 row sums
//     by one warp_reduce8, y = w * 0.125 * sum.
// The IQ2 decode is moe_device.cuh's selector-table path (iq2_dot_sel), table at shared offset 0.
#include "moe_internal.h"
#include "moe_device.cuh"

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

// ------------------------------------------------------------------ gate / up, one token
constexpr int G1_WARPS = 16;
constexpr int G1_THREADS = (G1_WARPS + 1) * 32;
constexpr int G1_ROWB = (HIDDEN / QK) * BLK_IQ2;     // 1848
constexpr int G1_UROWS = 2;                          // h rows per unit
constexpr int G1_UBYTES = 2 * G1_UROWS * G1_ROWB;    // 7392: gate rows then up rows
constexpr int G1_NST = 20;
constexpr int G1_TILE = 32;                          // h rows per q8 tile
constexpr int G1_UPT = G1_TILE / G1_UROWS;           // 16 units per tile
constexpr int G1_TILES_PER_SLOT = MOE_INTER / G1_TILE;
constexpr int G1_GPL = HIDDEN / 32 / 32;             // 7 groups per lane
constexpr int G1_NBUF = 4;                           // tiles in flight per CTA (<= NST/UPT + 2)

constexpr int G1_OFF_TAB = 0;
constexpr int G1_OFF_RING = G1_OFF_TAB + SEL_TAB_BYTES;
constexpr int G1_OFF_H = G1_OFF_RING + G1_NST * G1_UBYTES;
constexpr int G1_OFF_CNT = G1_OFF_H + G1_NBUF * G1_TILE * 4;
constexpr int G1_OFF_BAR = G1_OFF_CNT + G1_NBUF * 4;
constexpr int G1_OFF_ABORT = G1_OFF_BAR + 2 * G1_NST * 8;
constexpr int G1_SMEM = G1_OFF_ABORT + 16;

__global__ void __launch_bounds__(G1_THREADS, 1) k_gate_up1(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem + G1_OFF_RING;
    float* hbuf = (float*)(smem + G1_OFF_H);
    int* hcnt = (int*)(smem + G1_OFF_CNT);
    uint64_t* full = (uint64_t*)(smem + G1_OFF_BAR);
    uint64_t* empty = full + G1_NST;
    volatile int* abort_flag = (volatile int*)(smem + G1_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int ntiles = nslots * G1_TILES_PER_SLOT;
    if ((int)blockIdx.x >= ntiles) return;
    init_sel_table((uint32_t*)(smem + G1_OFF_TAB), tid, G1_THREADS);
    if (tid < G1_NBUF) hcnt[tid] = 0;
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < G1_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        fence_mbar_init();
    }
    __syncthreads();
    // unit sequence of this CTA: tiles blockIdx.x + k*gridDim.x, each as 16 units; unit j -> stage j % NST,
    // consumed by warp j % G1_WARPS
    if (warp == G1_WARPS) {                           // ---------------- producer
        if (lane == 0) {
            uint32_t j = 0;
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const int e = p.slot_expert[s];
                const uint8_t* g = slot_matrix1(p, e, 0);
                const uint8_t* u = slot_matrix1(p, e, 1);
                for (int k = 0; k < G1_UPT; ++k, ++j) {
                    const int st = j % G1_NST;
                    if (*abort_flag || !mbar_wait(&empty[st], ((j / G1_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    const size_t roff = (size_t)(rt * G1_TILE + k * G1_UROWS) * G1_ROWB;
                    mbar_arrive_expect_tx(&full[st], G1_UBYTES);
                    bulk_g2s(ring + st * G1_UBYTES, g + roff, G1_UBYTES / 2, &full[st]);
                    bulk_g2s(ring + st * G1_UBYTES + G1_UBYTES / 2, u + roff, G1_UBYTES / 2, &full[st]);
                }
            }
        drain:
            {
                const uint32_t first = j > G1_NST ? j - G1_NST : 0;
                for (uint32_t i = first; i < j; ++i) mbar_wait(&full[i % G1_NST], (i / G1_NST) & 1, nullptr, 0);
            }
        }
        return;
    }

    const uint32_t tab_s = smem_u32(smem + G1_OFF_TAB);
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t lane4 = (uint32_t)lane << 2;
    const uint32_t goff0 = 2u + BLK_IQ2 * (lane >> 3) + 8u * (lane & 7);   // group `lane`; +264 per 32 groups
    const uint32_t gal = goff0 & ~3u, gsh = (goff0 & 3u) * 8u;
    const uint32_t boff0 = BLK_IQ2 * (lane >> 3);
    uint32_t xr[G1_GPL][8]; float dx[G1_GPL]; int xtok = -2;
    uint32_t j = 0; int tseq = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tseq) {
        const int s = tile % nslots, rt = tile / nslots;
        const int tok = p.slot_tok[s];
        if (tok != xtok) {
            #pragma unroll
            for (int q = 0; q < G1_GPL; ++q) {
                if (tok >= 0) dx[q] = q8_group_global(p.x + (size_t)tok * p.ld_x, lane + 32 * q, xr[q]);
                else { dx[q] = 0.0f; for (int w = 0; w < 8; ++w) xr[q][w] = 0u; }
            }
            xtok = tok;
        }
        const int hb = tseq % G1_NBUF;
        for (int k = warp; k < G1_UPT; k += G1_WARPS) {   // this warp's units of the tile
            const uint32_t ju = j + (uint32_t)k;
            const int st = ju % G1_NST;
            if (!*abort_flag && !mbar_wait(&full[st], (ju / G1_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1;
            const uint32_t ub = ring_s + st * G1_UBYTES;
            const uint32_t ubg = ub + gal, ubd = ub + boff0;
            float v[4];                               // g(row0), g(row1), u(row0), u(row1)
            #pragma unroll
            for (int r = 0; r < 4; ++r) {
                float a = 0.0f;
                #pragma unroll
                for (int q = 0; q < G1_GPL; ++q) {
                    uint32_t aux0, aux1;
                    lds_group(ubg + r * G1_ROWB + 264u * q, gsh, aux0, aux1);
                    const float d = __half2float(__ushort_as_half(lds_u16(ubd + r * G1_ROWB + 264u * q)));
                    const int isum = iq2_dot1(aux0, aux1, xr[q], tab_s, lane4);
                    a = fmaf((float)(isum * ((int)((aux1 >> 27) & 0x1Eu) + 1)), d * dx[q], a);
                }
                v[r] = a;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            // 4 values over the warp: halving over 16, 8, then butterflies 4, 2, 1 -> lane l holds v[(l >> 3) & 3]
            #pragma unroll
            for (int o = 16, h = 2; o >= 8; o >>= 1, h >>= 1) {
                const bool up = (lane & o) != 0;
                #pragma unroll
                for (int i = 0; i < h; ++i) {
                    const float send = up ? v[i] : v[i + h];
                    const float keep = up ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            float r0 = v[0];
            r0 += __shfl_xor_sync(0xffffffffu, r0, 4);
            r0 += __shfl_xor_sync(0xffffffffu, r0, 2);
            r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
            // lanes 0-7: g row0, 8-15: g row1, 16-23: u row0, 24-31: u row1
            const float uo = __shfl_xor_sync(0xffffffffu, r0, 16);
            if (lane == 0 || lane == 8) {
                const int hr = k * G1_UROWS + (lane >> 3);
                hbuf[hb * G1_TILE + hr] = lk_swiglu(r0 * 0.125f, uo * 0.125f);
            }
            __syncwarp();
            int last = 0;
            if (lane == 0) { __threadfence_block(); last = atomicAdd(&hcnt[hb], 1) == G1_UPT - 1; }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {                               // all 32 h rows of the tile are in hbuf: q8 them
                __threadfence_block();
                const float hv = ((volatile float*)hbuf)[hb * G1_TILE + lane];
                float amax = fabsf(hv);
                #pragma unroll
                for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
                const int out = p.slot_out[s];
                if (out >= 0) {
                    p.hq[(size_t)out * MOE_INTER + rt * G1_TILE + lane] = (int8_t)(int)rintf(hv * id);
                    if (lane == 0) p.hd[(size_t)out * (MOE_INTER / 32) + rt] = d;
                }
                if (lane == 0) hcnt[hb] = 0;
            }
        }
        j += G1_UPT;
        if (*abort_flag) break;
    }
}

// ------------------------------------------------------------------ down, one token
constexpr int D1_WARPS = 16;
constexpr int D1_THREADS = (D1_WARPS + 1) * 32;
constexpr int D1_ROWB = (MOE_INTER / QK) * BLK_IQ2;  // 528
constexpr int D1_UROWS = 8;                          // rows per warp unit
constexpr int D1_CROWS = 32;                         // rows per bulk copy (16 896 B: copies under ~8 KB
constexpr int D1_CBYTES = D1_CROWS * D1_ROWB;        //   cannot stream HBM at full rate)
constexpr int D1_TILE = 128;                         // rows per (slot, tile): 4 copies, 16 warp units
constexpr int D1_CPT = D1_TILE / D1_CROWS;
constexpr int D1_NST = 2 * D1_CPT;                   // two tiles: warp w always uses stages w/4 and w/4 + 4
constexpr int D1_TILES_PER_SLOT = HIDDEN / D1_TILE;  // 56

constexpr int D1_OFF_TAB = 0;
constexpr int D1_OFF_RING = D1_OFF_TAB + SEL_TAB_BYTES;
constexpr int D1_OFF_BAR = D1_OFF_RING + D1_NST * D1_CBYTES;
constexpr int D1_OFF_ABORT = D1_OFF_BAR + 2 * D1_NST * 8;
constexpr int D1_SMEM = D1_OFF_ABORT + 16;

__global__ void __launch_bounds__(D1_THREADS, 1) k_down1(ExpertParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem + D1_OFF_RING;
    uint64_t* full = (uint64_t*)(smem + D1_OFF_BAR);
    uint64_t* empty = full + D1_NST;
    volatile int* abort_flag = (volatile int*)(smem + D1_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int ntiles = nslots * D1_TILES_PER_SLOT;
    if ((int)blockIdx.x >= ntiles) return;
    init_sel_table((uint32_t*)(smem + D1_OFF_TAB), tid, D1_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < D1_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], D1_CROWS / D1_UROWS); }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == D1_WARPS) {                           // ---------------- producer
        if (lane == 0) {
            uint32_t j = 0;
            for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
                const int s = tile % nslots, rt = tile / nslots;
                const uint8_t* dw = slot_matrix1(p, p.slot_expert[s], 2);
                for (int k = 0; k < D1_CPT; ++k, ++j) {
                    const int st = j % D1_NST;
                    if (*abort_flag || !mbar_wait(&empty[st], ((j / D1_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    mbar_arrive_expect_tx(&full[st], D1_CBYTES);
                    bulk_g2s(ring + st * D1_CBYTES, dw + (size_t)(rt * D1_TILE + k * D1_CROWS) * D1_ROWB, D1_CBYTES, &full[st]);
                }
            }
        drain:
            {
                const uint32_t first = j > D1_NST ? j - D1_NST : 0;
                for (uint32_t i = first; i < j; ++i) mbar_wait(&full[i % D1_NST], (i / D1_NST) & 1, nullptr, 0);
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
    uint32_t j = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int s = tile % nslots, rt = tile / nslots;
        const int out = p.slot_out[s];
        const float wv = p.slot_w[s];
        uint32_t xr[2][8]; float dx[2];
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
        {
            const int k = warp;                       // warp unit: rows 8k..8k+7 of the tile, copy k / 4
            const uint32_t ju = j + (uint32_t)(k / (D1_CROWS / D1_UROWS));
            const int st = ju % D1_NST;
            if (!*abort_flag && !mbar_wait(&full[st], (ju / D1_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1;
            const uint32_t ub = ring_s + st * D1_CBYTES + (k % (D1_CROWS / D1_UROWS)) * D1_UROWS * D1_ROWB;
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
            const int row0 = rt * D1_TILE + k * D1_UROWS;
            if ((lane & 3) == 0 && out >= 0) p.y[(size_t)out * HIDDEN + row0 + (lane >> 2)] = wv * (sum * 0.125f);
        }
        j += D1_CPT;
        if (*abort_flag) break;
    }
}

void launch_gate_up1(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_gate_up1, cudaFuncAttributeMaxDynamicSharedMemorySize, G1_SMEM); attr = true; }
    k_gate_up1<<<grid, G1_THREADS, G1_SMEM, st>>>(p);
}
void launch_down1(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_down1, cudaFuncAttributeMaxDynamicSharedMemorySize, D1_SMEM); attr = true; }
    k_down1<<<grid, D1_THREADS, D1_SMEM, st>>>(p);
}

}  // namespace lk
