// moe_device.cuh -- sm_100a device building blocks shared by the MoE kernels:
//   * mbarrier + cp.async.bulk (1-D TMA) staging with bounded waits (every wait gives up after a
//     %globaltimer deadline, records an error code and lets the kernel return),
//   * the IQ2_XXS decode tables in shared memory, laid out lane-private (entry i of lane l at word
//     i*32 + l) so that the data-dependent lookups of a warp never conflict on a bank,
//   * the warp transpose-reduction used by the grouped matvecs.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "moe_format.h"

namespace lk {

// error codes written to the context's device error word (first writer wins)
enum { DEV_OK = 0, DEV_ERR_TIMEOUT_FULL = 1, DEV_ERR_TIMEOUT_EMPTY = 2, DEV_ERR_BAD_SLOT = 3, DEV_ERR_TIMEOUT_DRAIN = 4 };

// a staging wait that has not completed after this long means the pipeline is broken (a kernel step
// normally takes microseconds); the waiter records an error and the kernel unwinds.
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// wait for the phase of `parity` to complete; false (after recording `code`) once the deadline passes
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (err) atomicCAS(err, 0, code); return false; }
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (src/dst 16-byte aligned, bytes % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// hint: fetch [src, src+bytes) into L2 (bytes % 16 == 0, src 16-byte aligned)
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ---- IQ2_XXS tables in shared memory (lane-private layouts)
//  grid:  uint2 gt[256][32]  (64 KB): entry i, lane l = the 8 magnitudes of grid[i] (x: elements 0-3, y: 4-7)
//  signs: uint32 st[128][32] (16 KB): byte-permute selectors that pick, per element, the magnitude (nibble j)
//         or its negation (nibble 4+j) for the 8 sign bits ksigns(i): low 16 bits elements 0-3, high 16 bits 4-7
constexpr int GRID_TAB_BYTES = 256 * 32 * 8;
constexpr int SIGN_TAB_BYTES = 128 * 32 * 4;

static __constant__ uint64_t c_iq2_grid[256] = {
#include "iq2_grid.inc"
};

__device__ __forceinline__ uint32_t sign_selectors(uint32_t si) {
    const uint32_t s = iq2_ksigns(si);
    uint32_t lo = 0, hi = 0;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        lo |= (uint32_t)(j + 4 * ((s >> j) & 1u)) << (4 * j);
        hi |= (uint32_t)(j + 4 * ((s >> (4 + j)) & 1u)) << (4 * j);
    }
    return lo | (hi << 16);
}

__device__ __forceinline__ void init_iq2_tables(uint2* gt, uint32_t* st, int tid, int nthr) {
    for (int i = tid; i < 256 * 32; i += nthr) {
        const uint64_t v = c_iq2_grid[i >> 5];
        gt[i] = make_uint2((uint32_t)v, (uint32_t)(v >> 32));
    }
    for (int i = tid; i < 128 * 32; i += nthr) st[i] = sign_selectors((uint32_t)(i >> 5));
}

// signed int8 x4 of one half sub-group: magnitudes m (bytes 8/25/43) with per-byte negation chosen by sel
__device__ __forceinline__ uint32_t apply_signs(uint32_t m, uint32_t sel) {
    return __byte_perm(m, 0x01010100u - m, sel);   // 0x01010100 - m = bytewise -m (all m bytes are >= 8)
}

// integer dot of one IQ2_XXS group (aux0 = 4 grid indices, aux1 = 4 sign indices | scale<<28) with the
// 32 q8 activations x[0..8) (4 bytes per word); gt/st point at this lane's column of the tables
__device__ __forceinline__ int iq2_group_dot(uint32_t aux0, uint32_t aux1, const uint32_t* x,
                                             const uint2* gt, const uint32_t* st) {
    int acc = 0;
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint2 m = gt[((aux0 >> (8 * l)) & 0xFFu) * 32];
        const uint32_t sel = st[((aux1 >> (7 * l)) & 0x7Fu) * 32];
        acc = __dp4a((int)apply_signs(m.x, sel), (int)x[2 * l], acc);
        acc = __dp4a((int)apply_signs(m.y, sel >> 16), (int)x[2 * l + 1], acc);
    }
    return acc;
}

// the 8 bytes of IQ2 group `g` of a row staged in shared memory (row start 4-byte aligned): the group
// starts at 2 + 66*(g/8) + 8*(g%8), i.e. 2-byte aligned; read 3 aligned words and funnel-shift
__device__ __forceinline__ void load_group_smem(const uint8_t* row, int goff, uint32_t& aux0, uint32_t& aux1) {
    const uint32_t* w = (const uint32_t*)(row + (goff & ~3));
    const uint32_t sh = (uint32_t)(goff & 3) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
    aux0 = __funnelshift_r(w0, w1, sh);
    aux1 = __funnelshift_r(w1, w2, sh);
}
__device__ __forceinline__ float load_d_smem(const uint8_t* row, int boff) {
    return __half2float(*(const __half*)(row + boff));
}

// warp transpose-reduction of 32 values per lane: on return v[0] of lane l = sum over the warp's lanes
// of their v[l] (fixed order: butterfly halves 16, 8, 4, 2, 1)
__device__ __forceinline__ float warp_transpose_reduce32(float (&v)[32], int lane) {
    #pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const bool up = (lane & o) != 0;
        #pragma unroll
        for (int i = 0; i < o; ++i) {
            const float send = up ? v[i] : v[i + o];
            const float keep = up ? v[i + o] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    return v[0];
}

}  // namespace lk
