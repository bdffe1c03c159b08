// iq2_tc.cuh -- IQ2_XXS decode into fp16 tensor-core operands and the staging helpers shared by the
// tcgen05 GEMMs (prefill_gemm.cu, gate_up_q8.cu).
//
// Decode trick: for a weight v in {+-8, +-25, +-43}, fp16(1024 + v) has a low byte in {08, 19, 2B, F0, CE, AA}
// and a high byte in {64, 63} -- eight bytes -- so one byte-permute over the constant pair
// (0x642B1908, 0x63AACEF0) yields two fp16 values 1024+v; the selectors are the OR of a per-grid-entry table
// (codes) and a per-sign-index table (signs), both 64-bit and lane-private in shared memory.  One hfma2
// (x*s - 1024*s) then gives v*s for any fp16 scale s whose 1024*s is exact.
#pragma once
#include <stdint.h>
#include <cuda_fp16.h>
#include "moe_device.cuh"

namespace lk {

constexpr uint32_t F16_PAIR_LO = 0x642B1908u;            // bytes 08 19 2B 64
constexpr uint32_t F16_PAIR_HI = 0x63AACEF0u;            // bytes F0 CE AA 63
constexpr int IQ2TC_GTAB = 256 * 32 * 8;                 // 64 KB grid pair selectors (32 lane copies)
constexpr int IQ2TC_STAB = 128 * 32 * 8;                 // 32 KB sign pair selectors
// the same tables with 16 lane copies: a warp's 64-bit loads are served per half-warp, so lanes l and l + 16
// share copy l & 15 without a bank conflict
constexpr int IQ2TC_GTAB16 = 256 * 16 * 8;               // 32 KB
constexpr int IQ2TC_STAB16 = 128 * 16 * 8;               // 16 KB

__device__ __forceinline__ uint32_t pair_codes(uint64_t g, int a) {   // elements a, a+1 of grid entry g
    const uint32_t ma = (uint32_t)(g >> (8 * a)) & 0xFFu, mb = (uint32_t)(g >> (8 * a + 8)) & 0xFFu;
    const uint32_t ca = ma == 0x08u ? 0u : (ma == 0x19u ? 1u : 2u), cb = mb == 0x08u ? 0u : (mb == 0x19u ? 1u : 2u);
    return ca | (3u << 4) | (cb << 8) | (3u << 12);
}
__device__ __forceinline__ uint32_t pair_signs(uint32_t k, int a) {  // sign bits a, a+1 of ksigns value k
    const uint32_t sa = (k >> a) & 1u, sb = (k >> (a + 1)) & 1u;
    return (sa * 0x44u) | ((sb * 0x44u) << 8);
}
// grid pair selectors (gt, 256 entries) and sign pair selectors (st, 128 entries), lane-private: entry i of
// lane l at (i * 32 + l) * 8 bytes
__device__ __forceinline__ void init_pair_tables(uint2* gt, uint2* st, int tid, int nthr) {
    for (int t = tid; t < 256 + 128; t += nthr) {
        uint2 v;
        if (t < 256) {
            const uint64_t g = c_iq2_grid[t];
            v = make_uint2(pair_codes(g, 0) | (pair_codes(g, 2) << 16), pair_codes(g, 4) | (pair_codes(g, 6) << 16));
        } else {
            const uint32_t k = iq2_ksigns((uint32_t)(t - 256));
            v = make_uint2(pair_signs(k, 0) | (pair_signs(k, 2) << 16), pair_signs(k, 4) | (pair_signs(k, 6) << 16));
        }
        uint4* row = (uint4*)(t < 256 ? gt + t * 32 : st + (t - 256) * 32);
        const uint4 q = make_uint4(v.x, v.y, v.x, v.y);
        #pragma unroll
        for (int k = 0; k < 16; ++k) row[(k + t) & 15] = q;
    }
}

// 16-copy layout: entry i of copy l at (i * 16 + l) * 8 bytes
__device__ __forceinline__ void init_pair_tables16(uint2* gt, uint2* st, int tid, int nthr) {
    for (int t = tid; t < (256 + 128) * 16; t += nthr) {
        const int e = t >> 4, l = t & 15;
        if (e < 256) {
            const uint64_t g = c_iq2_grid[e];
            gt[e * 16 + l] = make_uint2(pair_codes(g, 0) | (pair_codes(g, 2) << 16), pair_codes(g, 4) | (pair_codes(g, 6) << 16));
        } else {
            const uint32_t k = iq2_ksigns((uint32_t)(e - 256));
            st[(e - 256) * 16 + l] = make_uint2(pair_signs(k, 0) | (pair_signs(k, 2) << 16), pair_signs(k, 4) | (pair_signs(k, 6) << 16));
        }
    }
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}

// decode one IQ2_XXS group (32 weights) into 16 fp16x2 words in K order (word j = elements 2j, 2j+1), each
// weight times the fp16 scale whose broadcast pair is s2 (c2 = the pair of -1024 * that scale, exact);
// COPIES = the lane copies of the tables (32 or 16), gtl/stl already offset to this lane's copy
template <int COPIES = 32>
__device__ __forceinline__ void decode_group_f16_s(uint32_t aux0, uint32_t aux1, uint32_t s2, uint32_t c2,
                                                   const uint2* gtl, const uint2* stl, uint32_t (&o)[16]) {
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint2 g = gtl[((aux0 >> (8 * l)) & 0xFFu) * COPIES];
        const uint2 sg = stl[((aux1 >> (7 * l)) & 0x7Fu) * COPIES];
        const uint32_t sx = g.x | sg.x, sy = g.y | sg.y;
        o[4 * l + 0] = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sx), s2, c2);
        o[4 * l + 1] = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sx >> 16), s2, c2);
        o[4 * l + 2] = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sy), s2, c2);
        o[4 * l + 3] = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sy >> 16), s2, c2);
    }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
// arrive on `bar` once every cp.async this thread issued so far has landed (counts as one of its arrivals)
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// registers -> tensor memory: 32 lanes x 16 consecutive 32-bit columns (thread i -> lane base + i)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                    "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// byte offset of element (n, k) in a B K-block tile of n16 rows (K-major core matrices, LBO = n16/8*128)
__device__ __forceinline__ uint32_t btile_off(int n, int k, int n16) {
    return (uint32_t)((k >> 3) * (n16 >> 3) * 128 + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
}
__device__ __forceinline__ int round16(int c) { return c <= 16 ? 16 : (c + 15) & ~15; }   // MMA N: 16, 32, ...

}  // namespace lk
