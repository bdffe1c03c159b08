// prefill_gemm.cu -- the prefill / batch regime: grouped expert GEMMs on the 5th-generation tensor cores.
//
// Replaces the wide pass's tc_matvec<F_IQ2> (mma.sync int8, 8 rows per slot; reference
// src/fused_layer.cu:540-553) for slots of up to 64 tokens per expert.  Per work item (slot, row tile):
//   D[128 weight rows x N tokens] = A[128 x K] . B[N x K]^T   with tcgen05.mma.cta_group::1.kind::f16,
//   fp32 accumulators in tensor memory (two tiles per item: gate+up rows, or two 128-row halves of down),
//   N = the slot's token count rounded up to 16.
// A (weights): IQ2_XXS decoded by 16 warps straight into fp16 in shared memory (UMMA canonical K-major,
//   no swizzle).  Decode trick: for a weight v in {+-8, +-25, +-43}, fp16(1024 + v) has a low byte in
//   {08, 19, 2B, F0, CE, AA} and a high byte in {64, 63} -- eight bytes -- so one byte-permute over the
//   constant pair (0x642B1908, 0x63AACEF0) yields two fp16 values 1024+v; the selectors are the OR of a
//   per-grid-entry table (codes) and a per-sign-index table (signs), both 64-bit and lane-private.  One
//   hfma2 (x*s - 1024*s, 1024*s exact) gives v*s, s = fp16(d*(2*scale+1)/8).
// B (activations): fp16 of the q8-dequantised values (k_x_q8_f16), gathered per slot token.
// Pipeline: decode warps fill a 2-stage ring and arrive on full[]; one thread issues 4 K=16 MMAs per
//   tile per stage and commits to empty[]; after the last stage a commit to accfull[] releases the
//   epilogue (tcgen05.ld of the accumulators), which frees the double-buffered accumulator via accempty[].
// Epilogues: gate/up -> h = silu(g)*u stored as fp16, the down GEMM's B (unlike the matvec path it is not
//   re-quantised to q8: with 16-bit operands that step would turn their rounding into q8 boundary flips);
//   down -> y[entry][row] = w * D (fp32), summed by the combine kernel.
#include "moe_internal.h"
#include "moe_device.cuh"
#include "tcgen05.cuh"

namespace lk {

constexpr int PG_M = 128;                    // weight rows per accumulator tile
constexpr int PG_NMAX = GEMM_NT;             // tokens per slot (64)
constexpr int PG_KB = 64;                    // K per pipeline stage
constexpr int PG_NST = 2;
constexpr int PG_PF = 4;                     // K blocks of global loads in flight per decode thread
constexpr int PG_DWARPS = 16;                // decode / B-load / epilogue warps
constexpr int PG_THREADS = (PG_DWARPS + 1) * 32;
constexpr int PG_A_BYTES = PG_M * PG_KB * 2;             // 16 KB
constexpr int PG_B_BYTES = PG_NMAX * PG_KB * 2;          // 8 KB
constexpr int PG_STAGE = 2 * PG_A_BYTES + PG_B_BYTES;    // 40 KB
constexpr int PG_A_LBO = (PG_M / 8) * 128;               // K-direction core-matrix stride in A
constexpr int PG_B_LBO = (PG_NMAX / 8) * 128;            // ... in B
constexpr int PG_GTAB = 256 * 32 * 8;                    // 64 KB grid pair selectors
constexpr int PG_STAB = 128 * 32 * 8;                    // 32 KB sign pair selectors
constexpr int PG_OFF_GTAB = 0;
constexpr int PG_OFF_STAB = PG_OFF_GTAB + PG_GTAB;
constexpr int PG_OFF_RING = PG_OFF_STAB + PG_STAB;
constexpr int PG_OFF_BAR = PG_OFF_RING + PG_NST * PG_STAGE;
constexpr int PG_NBAR = 2 * PG_NST + 2 + 2 + 1;          // full, empty, accfull, accempty, drain
constexpr int PG_OFF_MISC = PG_OFF_BAR + PG_NBAR * 8;
constexpr int PG_SMEM_USED = PG_OFF_MISC + 32;
// the whole 227 KB is reserved so that every operand read the descriptors can express stays inside this
// CTA's allocation
constexpr int PG_SMEM = 232448;
static_assert(PG_SMEM_USED <= PG_SMEM, "shared memory layout exceeds the allocation");
constexpr uint32_t PG_TMEM_COLS = 256;                   // 2 buffers x (2 tiles x 64 columns)
constexpr uint32_t F16_PAIR_LO = 0x642B1908u;            // bytes 08 19 2B 64
constexpr uint32_t F16_PAIR_HI = 0x63AACEF0u;            // bytes F0 CE AA 63

__device__ __forceinline__ uint32_t pair_codes(uint64_t g, int a) {   // elements a, a+1 of grid entry g
    const uint32_t ma = (uint32_t)(g >> (8 * a)) & 0xFFu, mb = (uint32_t)(g >> (8 * a + 8)) & 0xFFu;
    const uint32_t ca = ma == 0x08u ? 0u : (ma == 0x19u ? 1u : 2u), cb = mb == 0x08u ? 0u : (mb == 0x19u ? 1u : 2u);
    return ca | (3u << 4) | (cb << 8) | (3u << 12);
}
__device__ __forceinline__ uint32_t pair_signs(uint32_t k, int a) {  // sign bits a, a+1 of ksigns value k
    const uint32_t sa = (k >> a) & 1u, sb = (k >> (a + 1)) & 1u;
    return (sa * 0x44u) | ((sb * 0x44u) << 8);
}
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

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
    uint32_t d; asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
}

// decode one IQ2_XXS group (32 weights) of a row into 4 x 16-byte fp16 core-matrix rows of an A tile
__device__ __forceinline__ void decode_group_f16(uint32_t aux0, uint32_t aux1, float d, const uint2* gtl, const uint2* stl,
                                                 uint8_t* dst, int k8_stride) {
    // (1024 + v) * s - 1024 * s = v * s with s = fp16(d * (2*scale+1) / 8); 1024 * s is exact (power of two)
    const __half hs = __float2half_rn(d * (float)(2u * (aux1 >> 28) + 1u) * 0.125f);
    const uint32_t s2 = (uint32_t)__half_as_ushort(hs) * 0x10001u;
    const uint32_t c2 = (uint32_t)__half_as_ushort(__hmul(hs, __float2half_rn(-1024.0f))) * 0x10001u;
    #pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint2 g = gtl[((aux0 >> (8 * l)) & 0xFFu) * 32];
        const uint2 sg = stl[((aux1 >> (7 * l)) & 0x7Fu) * 32];
        const uint32_t sx = g.x | sg.x, sy = g.y | sg.y;
        uint4 out;
        out.x = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sx), s2, c2);
        out.y = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sx >> 16), s2, c2);
        out.z = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sy), s2, c2);
        out.w = hfma2_u32(__byte_perm(F16_PAIR_LO, F16_PAIR_HI, sy >> 16), s2, c2);
        *(uint4*)(dst + l * k8_stride) = out;
    }
}

// the IQ2 bytes of group `gi` (0..7) of superblock `sb` of a row in global memory
__device__ __forceinline__ void load_group_global(const uint8_t* row, int sb, int gi, uint32_t& aux0, uint32_t& aux1, float& d) {
    const uint32_t off = (uint32_t)sb * BLK_IQ2 + 2u + 8u * (uint32_t)gi;
    const uint32_t* w = (const uint32_t*)(row + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    const uint32_t w0 = __ldg(w), w1 = __ldg(w + 1), w2 = __ldg(w + 2);
    aux0 = __funnelshift_r(w0, w1, sh);
    aux1 = __funnelshift_r(w1, w2, sh);
    d = __half2float(__ushort_as_half(__ldg((const unsigned short*)(row + (size_t)sb * BLK_IQ2))));
}

template <bool DOWN>
__global__ void __launch_bounds__(PG_THREADS, 1) k_prefill_gemm(GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint2* gtab = (const uint2*)(smem + PG_OFF_GTAB);
    const uint2* stab = (const uint2*)(smem + PG_OFF_STAB);
    uint8_t* ring = smem + PG_OFF_RING;
    uint64_t* bars = (uint64_t*)(smem + PG_OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + PG_NST;
    uint64_t* accfull = bars + 2 * PG_NST;
    uint64_t* accempty = accfull + 2;
    uint64_t* drain = accempty + 2;
    uint32_t* tmem_slot = (uint32_t*)(smem + PG_OFF_MISC);
    volatile int* abort_flag = (volatile int*)(smem + PG_OFF_MISC + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    constexpr int TILES = DOWN ? HIDDEN / (2 * PG_M) : MOE_INTER / PG_M;   // 28 down pairs, 16 gate/up tiles
    const int nitems = nslots * TILES;
    if ((int)blockIdx.x >= nitems) return;
    constexpr int K = DOWN ? MOE_INTER : HIDDEN;
    constexpr int NKB = K / PG_KB;
    const size_t rowbytes = (size_t)(K / QK) * BLK_IQ2;

    init_pair_tables((uint2*)(smem + PG_OFF_GTAB), (uint2*)(smem + PG_OFF_STAB), tid, PG_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < PG_NST; ++s) { mbar_init(&full[s], PG_DWARPS); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&accfull[b], 1); mbar_init(&accempty[b], PG_DWARPS); }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == PG_DWARPS) { tmem_alloc(tmem_slot, PG_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t ring_s = smem_u32(ring);

    if (warp == PG_DWARPS) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0; int issued = 0;
            for (int i = 0, item = blockIdx.x; item < nitems && !*abort_flag; ++i, item += gridDim.x) {
                const int s = item % nslots;
                int cnt = 0;
                while (cnt < PG_NMAX && p.slot_tok[s * PG_NMAX + cnt] >= 0) ++cnt;
                const int N = cnt <= 16 ? 16 : (cnt <= 32 ? 32 : (cnt <= 48 ? 48 : 64));
                const uint32_t idesc = idesc_f16_f32(PG_M, N);
                const int buf = i & 1;
                if (i >= 2 && !mbar_wait(&accempty[buf], ((i >> 1) - 1) & 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d0 = tmem + (uint32_t)(buf * 2 * PG_NMAX), d1 = d0 + PG_NMAX;
                for (int kb = 0; kb < NKB; ++kb, ++it) {
                    const int st = it % PG_NST;
                    if (!mbar_wait(&full[st], (it / PG_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { *abort_flag = 1; break; }
                    tc_fence_after();
                    const uint32_t a0 = ring_s + st * PG_STAGE, a1 = a0 + PG_A_BYTES, b = a1 + PG_A_BYTES;
                    #pragma unroll
                    for (int ks = 0; ks < PG_KB / 16; ++ks) {
                        const uint64_t bd = umma_desc(b + ks * 2 * PG_B_LBO, PG_B_LBO, 128);
                        umma_f16(d0, umma_desc(a0 + ks * 2 * PG_A_LBO, PG_A_LBO, 128), bd, idesc, (kb | ks) != 0);
                        umma_f16(d1, umma_desc(a1 + ks * 2 * PG_A_LBO, PG_A_LBO, 128), bd, idesc, (kb | ks) != 0);
                    }
                    umma_commit(&empty[st]);
                    issued = 1;
                }
                if (*abort_flag) break;
                umma_commit(&accfull[buf]);
            }
            if (issued) {                             // every issued MMA has completed before teardown
                umma_commit(drain);
                mbar_wait(drain, 0, nullptr, 0);
            }
        }
    } else {
        // ---------------------------------------------------------------- decode / B load / epilogue warps
        const int mat = tid >> 8, row = (tid >> 1) & (PG_M - 1), grp = tid & 1;   // A unit: lane pairs share a row (L1 lines)
        const uint2* gtl = gtab + lane;
        const uint2* stl = stab + lane;
        const int bn = tid >> 3, bk8 = tid & 7;                                       // B chunk: 8 lanes read one token's 128 B
        uint32_t it = 0;
        for (int i = 0, item = blockIdx.x; item < nitems; ++i, item += gridDim.x) {
            const int s = item % nslots, rt = item / nslots;
            const int e = p.slot_expert[s];
            const uint8_t* wm;
            int grow;                                                                  // global weight row of this thread
            if (DOWN) {
                wm = e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride;
                grow = rt * 2 * PG_M + mat * PG_M + row;
            } else {
                wm = e == SHARED_SLOT ? (mat ? p.sh_up : p.sh_gate) : (mat ? p.up + (size_t)e * p.up_stride : p.gate + (size_t)e * p.gate_stride);
                grow = rt * PG_M + row;
            }
            const uint8_t* wrow = wm + (size_t)grow * rowbytes;
            const int btok = p.slot_tok[s * PG_NMAX + bn];
            const int bsrc = DOWN ? p.slot_out[s * PG_NMAX + bn] : btok;            // B row: h entry (down) / token (gate/up)
            const __half* bbase = DOWN ? p.hb : p.xh;
            // register prefetch ring: the global loads of K block kb + PG_PF are issued while kb is decoded
            uint32_t pw[PG_PF][3]; unsigned short pd[PG_PF]; uint4 pb[PG_PF];
            auto issue = [&](int kb, int j) {
                const int sb = kb >> 2, gi = (kb & 3) * 2 + grp;
                const uint32_t off = (uint32_t)sb * BLK_IQ2 + 2u + 8u * (uint32_t)gi;
                const uint32_t* w = (const uint32_t*)(wrow + (off & ~3u));
                pw[j][0] = __ldg(w); pw[j][1] = __ldg(w + 1); pw[j][2] = __ldg(w + 2);
                pd[j] = __ldg((const unsigned short*)(wrow + (size_t)sb * BLK_IQ2));
                pb[j] = bsrc >= 0 ? __ldg((const uint4*)(bbase + (size_t)bsrc * K + kb * PG_KB + bk8 * 8)) : make_uint4(0u, 0u, 0u, 0u);
            };
            #pragma unroll
            for (int j = 0; j < PG_PF; ++j) issue(j, j);
            for (int kb0 = 0; kb0 < NKB; kb0 += PG_PF) {
                #pragma unroll
                for (int j = 0; j < PG_PF; ++j, ++it) {
                    const int kb = kb0 + j;
                    const int st = it % PG_NST;
                    if (!*abort_flag && !mbar_wait(&empty[st], ((it / PG_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) *abort_flag = 1;
                    uint8_t* a = ring + st * PG_STAGE + mat * PG_A_BYTES;
                    uint8_t* b = ring + st * PG_STAGE + 2 * PG_A_BYTES;
                    // A: group grp of this K block (2 groups per 64 columns) -> k8 blocks 4*grp .. 4*grp+3, row `row`
                    const int gi = (kb & 3) * 2 + grp;
                    const uint32_t sh = ((((uint32_t)(kb >> 2) * BLK_IQ2 + 2u + 8u * (uint32_t)gi)) & 3u) * 8u;
                    const uint32_t aux0 = __funnelshift_r(pw[j][0], pw[j][1], sh), aux1 = __funnelshift_r(pw[j][1], pw[j][2], sh);
                    const float d = __half2float(__ushort_as_half(pd[j]));
                    const uint4 bv = pb[j];
                    if (kb + PG_PF < NKB) issue(kb + PG_PF, j);
                    decode_group_f16(aux0, aux1, d, gtl, stl, a + (4 * grp) * PG_A_LBO + (row >> 3) * 128 + (row & 7) * 16, PG_A_LBO);
                    // B: token bn, k8 block bk8 (16 bytes)
                    *(uint4*)(b + bk8 * PG_B_LBO + (bn >> 3) * 128 + (bn & 7) * 16) = bv;
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[st]);
                }
                if (*abort_flag) break;
            }
            if (*abort_flag) break;
            // ------------------------------------------------ epilogue of item i
            const int buf = i & 1;
            if (!mbar_wait(&accfull[buf], (i >> 1) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { *abort_flag = 1; break; }
            tc_fence_after();
            const int q = warp & 3, cc = warp >> 2;                // lanes 32q.., tokens 16cc..
            int cnt = 0;
            while (cnt < PG_NMAX && p.slot_tok[s * PG_NMAX + cnt] >= 0) ++cnt;
            if (cc * 16 < cnt) {
                const uint32_t t0 = tmem + (uint32_t)(buf * 2 * PG_NMAX + cc * 16) + ((uint32_t)(32 * q) << 16);
                float v0[16], v1[16];
                tmem_ld16(t0, v0);
                tmem_ld16(t0 + PG_NMAX, v1);
                #pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = cc * 16 + j;
                    const int out = n < cnt ? p.slot_out[s * PG_NMAX + n] : -1;
                    if (DOWN) {
                        if (out >= 0) {
                            const float w = p.slot_w[s * PG_NMAX + n];
                            const int r0 = rt * 2 * PG_M + 32 * q + lane;
                            p.y[(size_t)out * HIDDEN + r0] = w * v0[j];
                            p.y[(size_t)out * HIDDEN + r0 + PG_M] = w * v1[j];
                        }
                    } else if (out >= 0) {                // h = silu(g)*u enters the down GEMM at fp16
                        p.hb[(size_t)out * MOE_INTER + rt * PG_M + 32 * q + lane] = __float2half_rn(lk_swiglu(v0[j], v1[j]));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PG_DWARPS) { tc_fence_after(); tmem_dealloc(tmem, PG_TMEM_COLS); }
}

// x (fp32 [T][HIDDEN]) -> fp16 of its q8-per-32 dequantisation, the B operand of the gate/up GEMM
__global__ void k_x_q8_f16(const float* __restrict__ x, int ld, int T, __half* __restrict__ xh) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;             // one 32-group per thread
    if (i >= T * (HIDDEN / 32)) return;
    const int t = i / (HIDDEN / 32), g = i % (HIDDEN / 32);
    float v[32];
    const float4* src = (const float4*)(x + (size_t)t * ld + g * 32);
    #pragma unroll
    for (int j = 0; j < 8; ++j) { const float4 a = src[j]; v[4*j] = a.x; v[4*j+1] = a.y; v[4*j+2] = a.z; v[4*j+3] = a.w; }
    int8_t q[32];
    const float d = quant_q8_group(v, q);
    __half2* dst = (__half2*)(xh + (size_t)t * HIDDEN + g * 32);
    #pragma unroll
    for (int j = 0; j < 16; ++j) dst[j] = __halves2half2(__float2half_rn((float)q[2*j] * d), __float2half_rn((float)q[2*j+1] * d));
}

template <bool DOWN> static void pg_launch(const GemmParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_prefill_gemm<DOWN>, cudaFuncAttributeMaxDynamicSharedMemorySize, PG_SMEM); attr = true; }
    k_prefill_gemm<DOWN><<<grid, PG_THREADS, PG_SMEM, st>>>(p);
}

void launch_prefill_gemm(const GemmParams& p, int grid, cudaStream_t st) {
    k_x_q8_f16<<<(p.T * (HIDDEN / 32) + 255) / 256, 256, 0, st>>>(p.x, p.ld_x, p.T, p.xh);
    pg_launch<false>(p, grid, st);
    pg_launch<true>(p, grid, st);
}

}  // namespace lk
