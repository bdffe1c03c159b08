// slot_mma.cu -- the IQ2_XXS down projection of the mid-size regime (the mma threshold <= T < the GEMM threshold)
// with the weights dequantised straight into mma.sync A fragments in registers.  Its input is the fp16 of the
// q8-re-quantised SwiGLU output that gate_up_q8.cu wrote as rows hb[entry][MOE_INTER].
//
// Why not tcgen05 here: with 2..16 tokens per expert slot the weights-on-M GEMM (prefill_gemm.cu) is bound by MMA
// instructions, not by bytes.  Here each decoded weight goes from the byte-permute straight into an
// mma.sync.m16n8k16 fragment and is reused for every 8-token N tile of the slot (slots of up to MM_NT tokens).
//
// K permutation: mma's A fragment gives lane (g = lane/4, c = lane%4) the K positions {2c, 2c+1, 2c+8,
// 2c+9} of each 16-deep step.  Within each 32-deep IQ2 group the kernel maps fragment position
// p = 16*ks + 8*h + 2*c + e to weight k = 8*c + 4*ks + 2*h + e, so lane c's eight positions over the two
// steps are exactly the 8 weights of the group's grid entry c -- one table lookup pair, four byte-permutes,
// four hfma2 -- and the B fragments of token n are the 16 contiguous activations h[n][32j + 8c .. +8], one
// 16-byte load (the dot product is unchanged by permuting K on both sides).
//
// Per work item (slot, block of 256 output rows): each of 8 warps owns 32 rows (two m16 tiles).  A copy warp
// stages each weight row's next IQ2 superblock (80-byte 16-aligned window, 16-byte cp.async, coalesced) into a
// 3-stage raw ring; the decode tables are 16-lane private (64-bit lookups are served per half-warp, so lanes l
// and l+16 share a copy without bank conflicts).  The B rows are L2-resident.
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

constexpr int MM_WARPS = 8;
constexpr int MM_COPY_WARP = MM_WARPS;
constexpr int MM_THREADS = (MM_WARPS + 1) * 32;
constexpr int MM_RAW_ROWB = 80;
constexpr int MM_RAW_ROWS = 256;
constexpr int MM_RAW_STAGE = MM_RAW_ROWS * MM_RAW_ROWB;    // 20 KB
constexpr int MM_RAW_NST = 3;
constexpr int MM_GTAB = 256 * 16 * 8;                      // 32 KB grid pair selectors, 16 lane copies
constexpr int MM_STAB = 128 * 16 * 8;                      // 16 KB sign pair selectors
constexpr int MM_OFF_GTAB = 0;
constexpr int MM_OFF_STAB = MM_OFF_GTAB + MM_GTAB;
constexpr int MM_OFF_RAW = MM_OFF_STAB + MM_STAB;
constexpr int MM_OFF_BAR = MM_OFF_RAW + MM_RAW_NST * MM_RAW_STAGE + 64;   // + slack for the last row's over-read
constexpr int MM_OFF_ROWP = MM_OFF_BAR + 2 * MM_RAW_NST * 8;
constexpr int MM_OFF_MISC = MM_OFF_ROWP + MM_RAW_ROWS * 8;
constexpr int MM_SMEM = MM_OFF_MISC + 16;                   // ~110 KB: two CTAs per SM
constexpr uint32_t F16_LO = 0x642B1908u;                    // fp16(1024 + v) bytes, v in {8, 25, 43}: lows, 0x64
constexpr uint32_t F16_HI = 0x63AACEF0u;                    //   ... and for -v: lows, 0x63

__device__ __forceinline__ uint32_t mm_pair_codes(uint64_t g, int a) {
    const uint32_t ma = (uint32_t)(g >> (8 * a)) & 0xFFu, mb = (uint32_t)(g >> (8 * a + 8)) & 0xFFu;
    const uint32_t ca = ma == 0x08u ? 0u : (ma == 0x19u ? 1u : 2u), cb = mb == 0x08u ? 0u : (mb == 0x19u ? 1u : 2u);
    return ca | (3u << 4) | (cb << 8) | (3u << 12);
}
__device__ __forceinline__ uint32_t mm_pair_signs(uint32_t k, int a) {
    const uint32_t sa = (k >> a) & 1u, sb = (k >> (a + 1)) & 1u;
    return (sa * 0x44u) | ((sb * 0x44u) << 8);
}
// entry i of lane copy l at (i * 16 + l) * 8 bytes
__device__ __forceinline__ void mm_init_tables(uint2* gt, uint2* st, int tid, int nthr) {
    for (int t = tid; t < (256 + 128) * 16; t += nthr) {
        const int e = t >> 4, l = t & 15;
        uint2 v;
        if (e < 256) {
            const uint64_t g = c_iq2_grid[e];
            v = make_uint2(mm_pair_codes(g, 0) | (mm_pair_codes(g, 2) << 16), mm_pair_codes(g, 4) | (mm_pair_codes(g, 6) << 16));
            gt[e * 16 + l] = v;
        } else {
            const uint32_t k = iq2_ksigns((uint32_t)(e - 256));
            v = make_uint2(mm_pair_signs(k, 0) | (mm_pair_signs(k, 2) << 16), mm_pair_signs(k, 4) | (mm_pair_signs(k, 6) << 16));
            st[(e - 256) * 16 + l] = v;
        }
    }
}

__device__ __forceinline__ uint32_t mm_hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
// (not volatile: a pure register operation the compiler may interleave with the next decode)
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mm_cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void mm_cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// global down row of weight row r (0..255) of item (expert e, row block rb): rows rb*256 + r
__device__ __forceinline__ const uint8_t* mm_row(const MmaParams& p, int e, int rb, int r) {
    const uint8_t* wm = e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride;
    return wm + (size_t)(rb * 256 + r) * ((MOE_INTER / QK) * BLK_IQ2);
}

// the two A fragments (k steps 0, 1) of one row's grid entry c of a group, i.e. weights 8c..8c+7 in the
// permuted order: lo[ks] = weights (8c+4ks, +1), hi[ks] = weights (8c+4ks+2, +3)
// (plain shared loads: ordered after the barrier waits by their "memory" clobbers, free among themselves)
__device__ __forceinline__ void mm_decode_entry(uint32_t aux0, uint32_t aux1, uint32_t s2, uint32_t c2, int c,
                                                const uint2* gtl, const uint2* stl, uint32_t (&lo)[2], uint32_t (&hi)[2]) {
    const uint32_t gi = (aux0 >> (8 * c)) & 0xFFu, si = (aux1 >> (7 * c)) & 0x7Fu;
    const uint2 gv = gtl[gi * 16], sv = stl[si * 16];
    const uint32_t x = gv.x | sv.x, y = gv.y | sv.y;
    lo[0] = mm_hfma2(__byte_perm(F16_LO, F16_HI, x), s2, c2);
    hi[0] = mm_hfma2(__byte_perm(F16_LO, F16_HI, x >> 16), s2, c2);
    lo[1] = mm_hfma2(__byte_perm(F16_LO, F16_HI, y), s2, c2);
    hi[1] = mm_hfma2(__byte_perm(F16_LO, F16_HI, y >> 16), s2, c2);
}
// s2 = fp16x2 of d*(2*scale+1)/8, c2 = fp16x2 of -1024 * that (exact: a power-of-two multiple)
__device__ __forceinline__ void mm_scale(float d, uint32_t aux1, uint32_t& s2, uint32_t& c2) {
    const __half hs = __float2half_rn(d * (float)(2u * (aux1 >> 28) + 1u) * 0.125f);
    s2 = (uint32_t)__half_as_ushort(hs) * 0x10001u;
    c2 = (uint32_t)__half_as_ushort(__hmul(hs, __float2half_rn(-1024.0f))) * 0x10001u;
}

__global__ void __launch_bounds__(MM_THREADS, 2) k_slot_mma_down(MmaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* raw = smem + MM_OFF_RAW;
    uint64_t* rawfull = (uint64_t*)(smem + MM_OFF_BAR);
    uint64_t* rawempty = rawfull + MM_RAW_NST;
    uintptr_t* rowp = (uintptr_t*)(smem + MM_OFF_ROWP);
    volatile int* abort_flag = (volatile int*)(smem + MM_OFF_MISC);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    constexpr int BLOCKS = HIDDEN / 256;                                  // row blocks per slot: 28
    constexpr int K = MOE_INTER;
    constexpr int NSB = K / QK;
    const int nitems = nslots * BLOCKS;
    if ((int)blockIdx.x >= nitems) return;

    mm_init_tables((uint2*)(smem + MM_OFF_GTAB), (uint2*)(smem + MM_OFF_STAB), tid, MM_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < MM_RAW_NST; ++s) { mbar_init(&rawfull[s], 32); mbar_init(&rawempty[s], MM_WARPS); }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == MM_COPY_WARP) {
        // ---------------------------------------------------------------- raw superblock copies
        uint32_t rit = 0;
        const int rsub = lane / 5, chunk = lane - 5 * (lane / 5);
        for (int item = blockIdx.x; item < nitems && !*abort_flag; item += gridDim.x) {
            const int s = item % nslots, rb = item / nslots;
            const int e = p.slot_expert[s];
            __syncwarp();
            for (int r = lane; r < MM_RAW_ROWS; r += 32) rowp[r] = (uintptr_t)mm_row(p, e, rb, r);
            __syncwarp();
            for (int sb = 0; sb < NSB; ++sb, ++rit) {
                const int rs = rit % MM_RAW_NST;
                if (!mbar_wait(&rawempty[rs], ((rit / MM_RAW_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                uint8_t* dst = raw + rs * MM_RAW_STAGE;
                const size_t sboff = (size_t)sb * BLK_IQ2;
                if (lane < 30) {                      // lane -> (row rsub of 6, 16-byte chunk of 5)
                    #pragma unroll 4
                    for (int r = rsub; r < MM_RAW_ROWS; r += 6) {
                        const uintptr_t a = (rowp[r] + sboff) & ~(uintptr_t)15;
                        mm_cp_async16(dst + r * MM_RAW_ROWB + chunk * 16, (const void*)(a + 16 * chunk));
                    }
                }
                mm_cp_async_arrive(&rawfull[rs]);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        return;
    }

    // -------------------------------------------------------------------- compute warps
    const int g = lane >> 2, c = lane & 3;
    const uint2* gtl = (const uint2*)(smem + MM_OFF_GTAB) + (lane & 15);
    const uint2* stl = (const uint2*)(smem + MM_OFF_STAB) + (lane & 15);
    // raw rows of this thread: tile t, half h (rows g, g+8)
    int rr[2][2];
    #pragma unroll
    for (int t = 0; t < 2; ++t)
        #pragma unroll
        for (int h = 0; h < 2; ++h)
            rr[t][h] = 32 * warp + 16 * t + g + 8 * h;
    uint32_t rit = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int s = item % nslots, rb = item / nslots;
        const int e = p.slot_expert[s];
        const int cnt = p.slot_cnt[s];
        const int n8 = (cnt + 7) >> 3;
        // B rows of this thread's token in each N tile (token n = 8*nt + g): element offsets, -1 = none
        const __half* bbase = p.hb;
        int boff[MM_NT / 8];
        #pragma unroll
        for (int nt = 0; nt < MM_NT / 8; ++nt) {
            const int n = 8 * nt + g;
            const int src = n < cnt ? p.slot_out[s * MM_NT + n] : -1;
            boff[nt] = src >= 0 ? src * K + 8 * c : -1;
        }
        uint32_t wlo[2][2];                            // low bits of the global rows: the superblock's offset in its window
        #pragma unroll
        for (int t = 0; t < 2; ++t)
            #pragma unroll
            for (int h = 0; h < 2; ++h) wlo[t][h] = (uint32_t)(uintptr_t)mm_row(p, e, rb, rr[t][h]);
        float acc[2][MM_NT / 8][4];
        #pragma unroll
        for (int t = 0; t < 2; ++t)
            #pragma unroll
            for (int nt = 0; nt < MM_NT / 8; ++nt)
                #pragma unroll
                for (int i = 0; i < 4; ++i) acc[t][nt][i] = 0.0f;
        // activations of group j + 1 are loaded while group j is decoded
        uint4 bnext[MM_NT / 8];
        #pragma unroll
        for (int nt = 0; nt < MM_NT / 8; ++nt) bnext[nt] = (nt < n8 && boff[nt] >= 0) ? __ldg((const uint4*)(bbase + boff[nt])) : make_uint4(0u, 0u, 0u, 0u);
        for (int sb = 0; sb < NSB; ++sb, ++rit) {
            const int rs = rit % MM_RAW_NST;
            if (!*abort_flag && !mbar_wait(&rawfull[rs], (rit / MM_RAW_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) *abort_flag = 1;
            uint32_t roff[2][2]; float dv[2][2];          // byte offsets of this superblock in the raw stage
            const uint8_t* stage = raw + rs * MM_RAW_STAGE;
            #pragma unroll
            for (int t = 0; t < 2; ++t)
                #pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t delta = (wlo[t][h] + (uint32_t)sb * BLK_IQ2) & 15u;
                    roff[t][h] = rr[t][h] * MM_RAW_ROWB + delta;
                    dv[t][h] = __half2float(*(const __half*)(stage + roff[t][h]));
                }
            #pragma unroll 1
            for (int j = 0; j < 8; ++j) {
                uint4 bv[MM_NT / 8];
                #pragma unroll
                for (int nt = 0; nt < MM_NT / 8; ++nt) bv[nt] = bnext[nt];
                const int kn = (sb * 8 + j + 1) * 32;            // next group's first activation
                if (kn < K) {
                    #pragma unroll
                    for (int nt = 0; nt < MM_NT / 8; ++nt)
                        bnext[nt] = (nt < n8 && boff[nt] >= 0) ? __ldg((const uint4*)(bbase + boff[nt] + kn)) : make_uint4(0u, 0u, 0u, 0u);
                }
                #pragma unroll
                for (int t = 0; t < 2; ++t) {
                    uint32_t lo[2][2], hi[2][2];                 // [half][ks]
                    #pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t o = roff[t][h] + 2u + 8u * (uint32_t)j;
                        const uint32_t* wp = (const uint32_t*)(stage + (o & ~3u));
                        const uint32_t sh = (o & 3u) * 8u;
                        const uint32_t w0 = wp[0], w1 = wp[1], w2 = wp[2];
                        const uint32_t aux0 = __funnelshift_r(w0, w1, sh), aux1 = __funnelshift_r(w1, w2, sh);
                        uint32_t s2, c2;
                        mm_scale(dv[t][h], aux1, s2, c2);
                        mm_decode_entry(aux0, aux1, s2, c2, c, gtl, stl, lo[h], hi[h]);
                    }
                    #pragma unroll
                    for (int nt = 0; nt < MM_NT / 8; ++nt) {
                        if (nt < n8) {
                            mma16816(acc[t][nt], lo[0][0], lo[1][0], hi[0][0], hi[1][0], bv[nt].x, bv[nt].y);
                            mma16816(acc[t][nt], lo[0][1], lo[1][1], hi[0][1], hi[1][1], bv[nt].z, bv[nt].w);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rawempty[rs]);
            if (*abort_flag) break;
        }
        if (*abort_flag) break;
        // ------------------------------------------------ epilogue: C fragment (row g / g+8, tokens 2c, 2c+1)
        #pragma unroll
        for (int nt = 0; nt < MM_NT / 8; ++nt) {
            if (nt >= n8) break;
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int n = 8 * nt + 2 * c + (i & 1);
                if (n >= cnt) continue;
                const int out = p.slot_out[s * MM_NT + n];
                if (out < 0) continue;
                const float w = p.slot_w[s * MM_NT + n];
                const int row = rb * 256 + 32 * warp + g + 8 * (i >> 1);
                p.y[(size_t)out * HIDDEN + row] = w * acc[0][nt][i];
                p.y[(size_t)out * HIDDEN + row + 16] = w * acc[1][nt][i];
            }
        }
    }
}

// each slot's token count (pads are at the end of the slot)
__global__ void k_mma_counts(MmaParams p) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= *p.nslots) return;
    int cnt = 0;
    while (cnt < MM_NT && p.slot_tok[i * MM_NT + cnt] >= 0) ++cnt;
    p.slot_cnt[i] = cnt;
}

void launch_slot_mma_down(const MmaParams& p, int nsm, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_slot_mma_down, cudaFuncAttributeMaxDynamicSharedMemorySize, MM_SMEM); attr = true; }
    k_mma_counts<<<(p.max_slots + 255) / 256, 256, 0, st>>>(p);
    k_slot_mma_down<<<2 * nsm, MM_THREADS, MM_SMEM, st>>>(p);
}

}  // namespace lk
