// tcgen05.cuh -- thin wrappers over the sm_100a 5th-generation tensor-core instructions (inline PTX):
// tensor-memory allocation, the UMMA shared-memory / instruction descriptors, tcgen05.mma (kind::f16,
// A and B from shared memory, fp32 accumulator in tensor memory), commit to an mbarrier, and the
// 32-lane x 32-bit tensor-memory loads the epilogues use.
#pragma once
#include <stdint.h>
#include "moe_device.cuh"

namespace lk {

// ---- tensor memory allocation (one full warp executes these)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- UMMA shared-memory descriptor, K-major, no swizzle (canonical "interleaved" layout):
//   8 x 16-byte core matrices; element (r, k) of an fp16 tile lives at
//   start + (k/8)*LBO + (r/8)*SBO + (r%8)*16 + (k%8)*2.
//   bits 0-13 start >> 4, 16-29 LBO >> 4, 32-45 SBO >> 4, 46-47 version 1 (sm_100), 61-63 layout 0.
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// ---- instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 accumulate, M x N
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4)                              // accumulator format: f32
         | (0u << 7) | (0u << 10)                 // A, B format: f16
         | ((uint32_t)(N >> 3) << 17)             // N / 8
         | ((uint32_t)(M >> 4) << 24);            // M / 16
}

// D[tmem] (+)= A[smem] x B[smem]^T, one 16-deep K step, issued by a single thread
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// arrive once on the mbarrier when every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// ---- warp-level issue: the whole (converged) warp executes these with identical operands and elect.sync
// lets one lane issue.  Measured on B200: a lone thread issuing with operands in ordinary registers pays
// ~110-200 cycles per tcgen05.mma whatever the shape, while warp-uniform issue runs at the tensor pipe's
// rate (M=128: 39 cycles at N=16, 64 at N=128, 128 at N=256 for kind::f16).
// D[tmem] (+)= A[tmem] x B[smem]^T, one 16-deep K step
__device__ __forceinline__ void umma_f16_ta_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
                 :: "r"(smem_u32(bar)) : "memory");
}

// ---- tensor memory -> registers: 32 lanes x 16 consecutive 32-bit columns (thread i <- lane base+i)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    #pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace lk
