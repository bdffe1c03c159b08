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
// try_wait with a suspend-time hint: the warp sleeps until the phase completes or about `ns` pass,
// instead of re-issuing the test (a spinning warp takes issue slots from the compute warps of its SMSP)
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(ns) : "memory");
    return ok != 0;
}
constexpr uint32_t WAIT_SLEEP_NS = 20000;
// wait for the phase of `parity` to complete; false (after recording `code`) once the deadline passes
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, WAIT_SLEEP_NS)) return true;
        if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (err) atomicCAS(err, 0, code); return false; }
    }
}

// the same wait for roles whose waits are long (a warp that waits hundreds of cycles for another role):
// between tests the warp sleeps (__nanosleep, doubling from ns0 to 256 ns) instead of re-issuing, so the
// compute warps of its SM sub-partition keep the issue slots
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* err, int code, uint32_t ns0 = 32) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    uint32_t ns = ns0;
    while (true) {
        __nanosleep(ns);
        if (mbar_try_wait(bar, parity)) return true;
        ns = ns < 256u ? 2u * ns : 256u;
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
// programmatic dependent launch: let the next kernel in the stream be scheduled (its CTAs still wait in
// pdl_wait for this grid to complete), and wait for the previous kernel's completion and memory
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// named barrier that also ORs a predicate over the participating threads: every thread gets the same
// answer, so decisions taken on it (an abort) are uniform
__device__ __forceinline__ bool named_bar_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(nthreads) : "memory");
    return r != 0;
}

// ---- IQ2_XXS decode table in shared memory: 64 KB, lane-private, one 256-byte row per index i:
//   bytes [0, 128):   grid selector of grid entry i for lanes 0..31 (4 bytes each)
//   bytes [128, 256): sign selector of sign index i (i < 128) for lanes 0..31
//   grid selector: nibble j (bits 4j..4j+3, j < 4) = code of element j (0, 1, 2 for magnitude 8, 25, 43);
//                  bits 16 + 4j the same for element 4 + j.
//   sign selector: bit 2 of the same nibbles = sign bit of that element (ksigns(i), bit 7 = parity).
//   (grid | sign) is then a byte-permute selector over the constant pair (POS, NEG): nibble c + 4s picks
//   magnitude c with sign s, so one prmt yields 4 signed int8 weights.  Lane-private rows make every
//   data-dependent lookup of a warp hit 32 distinct banks; the lane offset rides in the same prmt that
//   extracts the grid index (address = idx << 8 | lane << 2).
constexpr int SEL_TAB_BYTES = 256 * 256;
constexpr uint32_t IQ2_POS = 0x002B1908u;   // bytes: 8, 25, 43, 0
constexpr uint32_t IQ2_NEG = 0x00D5E7F8u;   // bytes: -8, -25, -43, 0

static __constant__ uint64_t c_iq2_grid[256] = {
#include "iq2_grid.inc"
};

__device__ __forceinline__ uint32_t grid_selector(uint64_t g) {
    uint32_t s = 0;
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t m = (uint32_t)(g >> (8 * j)) & 0xFFu;
        const uint32_t code = m == 0x08u ? 0u : (m == 0x19u ? 1u : 2u);
        s |= code << ((j < 4 ? 0 : 16) + 4 * (j & 3));
    }
    return s;
}
__device__ __forceinline__ uint32_t sign_selector(uint32_t si) {
    const uint32_t k = iq2_ksigns(si);
    uint32_t s = 0;
    #pragma unroll
    for (int j = 0; j < 8; ++j) s |= ((k >> j) & 1u) << ((j < 4 ? 0 : 16) + 4 * (j & 3) + 2);
    return s;
}
// each selector is computed once (thread t: grid entry t, or sign index t - 256) and written to its 32
// lane copies with 16-byte stores; a thread starts at chunk t % 8 so the 8 lanes of a store wavefront hit
// distinct banks
__device__ __forceinline__ void init_sel_table(uint32_t* tab, int tid, int nthr) {
    for (int t = tid; t < 256 + 128; t += nthr) {
        const uint32_t v = t < 256 ? grid_selector(c_iq2_grid[t]) : sign_selector((uint32_t)(t - 256));
        uint4* row = (uint4*)(tab + (t < 256 ? t * 64 : (t - 256) * 64 + 32));
        const uint4 q = make_uint4(v, v, v, v);
        #pragma unroll
        for (int k = 0; k < 8; ++k) row[(k + t) & 7] = q;
    }
}

// integer dots of one IQ2_XXS group (aux0 = 4 grid indices, aux1 = 4 sign indices | scale << 28) with
// the 32 q8 activations of NT tokens (x[t][0..8), 4 int8 per word); tab = the shared table,
// lane4 = lane << 2.  acc[t] receives the exact int32 sums.
template <int NT>
__device__ __forceinline__ void iq2_dot_sel(uint32_t aux0, uint32_t aux1, const uint32_t (&x)[NT][8], int (&acc)[NT],
                                            const unsigned char* tab, uint32_t lane4) {
    const uint32_t a1s = aux1 >> 13;
    const uint32_t so = 128u | lane4;
    const uint32_t sa[4] = { ((aux1 << 8) & 0x7F00u) | so, ((aux1 << 1) & 0x7F00u) | so,
                             ((a1s << 7) & 0x7F00u) | so, (a1s & 0x7F00u) | so };
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint32_t ga = __byte_perm(aux0, lane4, 0x6504u | (uint32_t)(l << 4));
        const uint32_t sel = *(const uint32_t*)(tab + ga) | *(const uint32_t*)(tab + sa[l]);
        const uint32_t vlo = __byte_perm(IQ2_POS, IQ2_NEG, sel);
        const uint32_t vhi = __byte_perm(IQ2_POS, IQ2_NEG, sel >> 16);
        #pragma unroll
        for (int t = 0; t < NT; ++t) {
            acc[t] = __dp4a((int)vlo, (int)x[t][2 * l], acc[t]);
            acc[t] = __dp4a((int)vhi, (int)x[t][2 * l + 1], acc[t]);
        }
    }
}

// ---- IQ2_XXS decode with the signs applied to the activations (one token per thread): 80 KB,
// lane-private rows again.
//   [0, 64 KB):      grid magnitudes: entry i at i*256 + lane*8 = the 8 magnitude bytes of grid entry i
//   [64 KB, 80 KB):  sign selectors: entry s (7-bit sign index) at 64 KB + s*128 + lane*4; nibble j (bits
//                    4j..4j+3) = j + 4*sign_j, nibble 4 + j (bits 16 + 4j) = j + 4*sign_{4+j}
// A thread keeps its activations x (int8, 4 per word) and their negations nx.  Per 8 weights:
// prmt(x, nx, selector) gives the signed activations, and dp4a multiplies them by the unsigned magnitudes.
// Compared with the selector table: no OR of two lookups, and the sign index needs only mask (and shift)
// at stride 128.
constexpr int XS_TAB_BYTES = 80 * 1024;
constexpr int XS_SGN_OFF = 64 * 1024;

__device__ __forceinline__ uint32_t xs_sign_selector(uint32_t si) {
    const uint32_t k = iq2_ksigns(si);
    uint32_t s = 0;
    #pragma unroll
    for (int j = 0; j < 8; ++j) s |= ((uint32_t)(j & 3) + 4u * ((k >> j) & 1u)) << ((j < 4 ? 0 : 16) + 4 * (j & 3));
    return s;
}
__device__ __forceinline__ void init_xs_table(uint8_t* tab, int tid, int nthr) {
    for (int i = tid; i < 256 * 4; i += nthr) {           // 4 lanes' copies (32 B) per store pair
        const int e = i >> 2, l0 = (i & 3) * 8;
        const uint64_t g = c_iq2_grid[e];
        uint4* row = (uint4*)(tab + e * 256 + l0 * 8);
        const uint4 q = make_uint4((uint32_t)g, (uint32_t)(g >> 32), (uint32_t)g, (uint32_t)(g >> 32));
        #pragma unroll
        for (int k = 0; k < 4; ++k) row[k] = q;
    }
    for (int i = tid; i < 128 * 2; i += nthr) {
        const int s = i >> 1, l0 = (i & 1) * 16;
        const uint32_t v = xs_sign_selector((uint32_t)s);
        uint4* row = (uint4*)(tab + XS_SGN_OFF + s * 128 + l0 * 4);
        const uint4 q = make_uint4(v, v, v, v);
        #pragma unroll
        for (int k = 0; k < 4; ++k) row[k] = q;
    }
}
// bytewise negation of 4 int8 values in [-127, 127] (q8 never holds -128)
__device__ __forceinline__ uint32_t neg_i8x4(uint32_t v) {
    uint32_t r = 0;
    #pragma unroll
    for (int j = 0; j < 4; ++j) r |= (uint32_t)(uint8_t)(-(int8_t)(v >> (8 * j))) << (8 * j);
    return r;
}
// exact int32 dot of one IQ2_XXS group (aux0, aux1) with 32 q8 activations x (nx = their negations);
// tab = the xs table, lane4 / lane8 = lane << 2 / lane << 3
__device__ __forceinline__ int iq2_dot_xs(uint32_t aux0, uint32_t aux1, const uint32_t (&x)[8], const uint32_t (&nx)[8],
                                          const unsigned char* tab, uint32_t lane4, uint32_t lane8) {
    int acc = 0;
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint32_t ga = __byte_perm(aux0, lane8, 0x5504u | (uint32_t)(l << 4));   // idx << 8 | lane << 3
        const uint2 g = *(const uint2*)(tab + ga);
        const uint32_t sa = (l == 0 ? (aux1 << 7) : l == 1 ? aux1 : l == 2 ? (aux1 >> 7) : (aux1 >> 14)) & 0x3F80u;
        const uint32_t s = *(const uint32_t*)(tab + XS_SGN_OFF + (sa | lane4));
        acc = __dp4a((int)g.x, (int)__byte_perm(x[2 * l], nx[2 * l], s), acc);
        acc = __dp4a((int)g.y, (int)__byte_perm(x[2 * l + 1], nx[2 * l + 1], s >> 16), acc);
    }
    return acc;
}

// an expert-parallel row's activations (include/loki_ep.h): the q8 per 32 of the fp32 row x (quant_q8_group,
// bit for bit) as int8 codes at q and fp32 scales at d; threads tid < 224 of the block each take one group
__device__ __forceinline__ void ep_row_q8(const float* __restrict__ x, int8_t* q, float* d, int tid) {
    if (tid >= HIDDEN / 32) return;
    float v[32];
    const float4* src = (const float4*)(x + tid * 32);
    #pragma unroll
    for (int j = 0; j < 8; ++j) { const float4 a = src[j]; v[4*j] = a.x; v[4*j+1] = a.y; v[4*j+2] = a.z; v[4*j+3] = a.w; }
    int8_t qv[32];
    d[tid] = quant_q8_group(v, qv);
    uint4 w[2];
    memcpy(w, qv, 32);
    ((uint4*)(q + tid * 32))[0] = w[0];
    ((uint4*)(q + tid * 32))[1] = w[1];
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

// warp reduction of 8 values per lane: on return every lane holds the warp-wide sum of v[i] for
// i = 4*bit4 + 2*bit3 + bit2 of its lane id (the 4 lanes sharing bits 4..2 hold the same value).
// Fixed order: halving exchanges over lane offsets 16, 8, 4, then butterflies over 2 and 1.
__device__ __forceinline__ float warp_reduce8(float (&v)[8], int lane) {
    #pragma unroll
    for (int o = 16, h = 4; o >= 4; o >>= 1, h >>= 1) {
        const bool up = (lane & o) != 0;
        #pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = up ? v[i] : v[i + h];
            const float keep = up ? v[i + h] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float r = v[0];
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    return r;
}

// warp reduction of 4 values per lane: every lane ends with the warp-wide sum of v[2*bit4 + bit3] of its
// lane id (8 lanes share each).  Fixed order: halving exchanges over offsets 16 and 8, butterflies 4, 2, 1.
__device__ __forceinline__ float warp_reduce4(float (&v)[4], int lane) {
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
    float r = v[0];
    r += __shfl_xor_sync(0xffffffffu, r, 4);
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    return r;
}

}  // namespace lk
