// prefill_gemm.cu -- the IQ2_XXS down projection of the tensor-core regime (T >= the GEMM threshold) on the
// 5th-generation tensor cores.  The gate/up + SwiGLU phase before it is gate_up_q8.cu, whose epilogue writes this
// kernel's B tiles: fp16 of the q8-re-quantised h (the reference's swiglu_q8, src/fused_layer.cu:334-341).
//
// Replaces the wide pass's tc_matvec down (mma.sync int8; reference src/fused_layer.cu:540-553) for slots of up to
// 128 tokens per expert.  Per work item (slot, pair of 128-row tiles of the 7168 output rows):
//   D[128 weight rows x N tokens] = A[128 x 2048] . B[N x 2048]^T   with tcgen05.mma.cta_group::1.kind::f16,
//   fp32 accumulators in tensor memory (two tiles per item), N = the slot's token count rounded up to 16 (up to
//   128).  The two tiles' MMAs alternate, so two accumulators are in flight.  The down is linear in its inputs,
//   so A = fp16(v * s), s = fp16(d*(2*scale+1)/8), rounds each weight once (~2.4e-4) and that error passes to
//   the output unamplified.
//
// A (weights) never touches shared memory as fp16: the IQ2_XXS groups are decoded in registers (iq2_tc.cuh) and
// written to tensor memory with tcgen05.st (thread = weight row = TMEM lane, 32 weights = 16 columns), and the MMA
// reads A from tensor memory.  B arrives as pre-tiled K-blocks (UMMA K-major core-matrix layout, N rows, LBO =
// N/8 * 128 bytes), one bulk copy (1-D TMA) per K-block.
//
// Warp roles (608 threads, one CTA per SM, persistent over (slot, tile) items); one pipeline stage is a
// 128-deep K-block (4 IQ2 groups), two stages in flight:
//   warps 0-15  decode: warp w = TMEM lane quarter w&3, tile (w>>2)&1, groups 2(w>>3), 2(w>>3)+1 of each
//               K-block (two independent decode chains per thread); then the epilogue
//   warp 16     MMA issuer (the whole warp on warp-uniform operands, elect.sync issues): 16 MMAs per K-block,
//               commit to empty[], accfull per item
//   warp 17     B K-block tiles into the B ring (1-D TMA bulk copies), one thread
//   warp 18     raw superblocks: each weight row's next IQ2 superblock, as the 80-byte 16-aligned window around
//               it, into a 3-stage raw ring (16-byte cp.async, 6 rows per instruction, coalesced), up to three
//               superblocks ahead of the decode warps whatever the B stages do
// Barriers: rawfull/rawempty (raw ring), full/empty (A stage in TMEM + B stage in shared memory),
// accfull/accempty (the accumulators; the decode warps run the epilogue, so a second accumulator buffer
// would not let the MMA run ahead).  Every wait is bounded (moe_device.cuh); the waits of every role back
// off with __nanosleep so a waiting warp leaves the issue slots to the decode warps.
#include "moe_internal.h"
#include "moe_device.cuh"
#include "tcgen05.cuh"
#include "iq2_tc.cuh"

namespace lk {

constexpr int PG_M = 128;                    // weight rows per accumulator tile
constexpr int PG_NMAX = GEMM_NT;             // tokens per slot (128)
constexpr int PG_KB = 128;                   // K per pipeline stage: 4 IQ2 groups, half a superblock
constexpr int PG_NST = 2;                    // A (TMEM) / B (smem) stages
constexpr int PG_DWARPS = 16;
constexpr int PG_MMA_WARP = PG_DWARPS;
constexpr int PG_COPY_WARP = PG_DWARPS + 1;  // B tiles
constexpr int PG_RAW_WARP = PG_DWARPS + 2;   // raw superblocks
constexpr int PG_THREADS = (PG_DWARPS + 3) * 32;
constexpr int PG_B_TILE = PG_NMAX * PG_KB * 2;           // 32 KB: one K-block of B at N = 128
constexpr int PG_RAW_ROWB = 80;                          // one superblock (66 B) in its 16-aligned 80-byte window
constexpr int PG_RAW_STAGE = 2 * PG_M * PG_RAW_ROWB;     // 256 weight rows: 20 KB
constexpr int PG_RAW_NST = 3;
constexpr int PG_GTAB = IQ2TC_GTAB;                      // 64 KB grid pair selectors
constexpr int PG_STAB = IQ2TC_STAB;                      // 32 KB sign pair selectors
constexpr int PG_OFF_GTAB = 0;
constexpr int PG_OFF_STAB = PG_OFF_GTAB + PG_GTAB;
constexpr int PG_OFF_B = PG_OFF_STAB + PG_STAB;
constexpr int PG_OFF_RAW = PG_OFF_B + PG_NST * PG_B_TILE;
constexpr int PG_OFF_BAR = PG_OFF_RAW + PG_RAW_NST * PG_RAW_STAGE + 64;   // + slack for the last row's over-read
constexpr int PG_NBAR = 2 * PG_NST + 2 + 2 + 1 + 2 * PG_RAW_NST;
constexpr int PG_OFF_ROWP = PG_OFF_BAR + PG_NBAR * 8;          // raw copy warp: the current item's 256 row addresses
constexpr int PG_OFF_MISC = PG_OFF_ROWP + 2 * PG_M * 8;
constexpr int PG_SMEM_USED = PG_OFF_MISC + 32;
// the whole 227 KB is reserved: one CTA per SM (it allocates all 512 tensor-memory columns), and every
// operand read the descriptors can express stays inside this CTA's allocation
constexpr int PG_SMEM = 232448;
static_assert(PG_SMEM_USED <= PG_SMEM, "shared memory layout exceeds the allocation");
constexpr uint32_t PG_TMEM_COLS = 512;
constexpr uint32_t PG_ACC_COLS = 2 * PG_NMAX;             // 256: 2 tiles x 128 fp32 columns
constexpr uint32_t PG_A_COLS = 2 * (PG_KB / 2);          // 128 per stage: 2 tiles x 64 columns (128 fp16)
static_assert(PG_ACC_COLS + PG_NST * PG_A_COLS <= PG_TMEM_COLS, "tensor memory layout");
// decode one IQ2_XXS group into fp16 v*s, s = fp16(d*(2*scale+1)/8) (iq2_tc.cuh)
__device__ __forceinline__ void decode_group_f16(uint32_t aux0, uint32_t aux1, float d, const uint2* gtl, const uint2* stl,
                                                 uint32_t (&o)[16]) {
    const __half hs = __float2half_rn(d * (float)(2u * (aux1 >> 28) + 1u) * 0.125f);
    const uint32_t s2 = (uint32_t)__half_as_ushort(hs) * 0x10001u;
    const uint32_t c2 = (uint32_t)__half_as_ushort(__hmul(hs, __float2half_rn(-1024.0f))) * 0x10001u;
    decode_group_f16_s(aux0, aux1, s2, c2, gtl, stl, o);
}

// D[tmem] (+)= A[tmem] x B[smem]^T, one 16-deep K step, issued by a single thread
__device__ __forceinline__ void umma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// global down row of weight row r (0..255) of work item (slot expert e, tile pair rt): rows rt*256 + r
__device__ __forceinline__ const uint8_t* item_row(const GemmParams& p, int e, int rt, int r, size_t rowbytes) {
    const uint8_t* wm = e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride;
    return wm + (size_t)(rt * 2 * PG_M + r) * rowbytes;
}

__global__ void __launch_bounds__(PG_THREADS, 1) k_prefill_down(GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint2* gtab = (const uint2*)(smem + PG_OFF_GTAB);
    const uint2* stab = (const uint2*)(smem + PG_OFF_STAB);
    uint8_t* bring = smem + PG_OFF_B;
    uint8_t* raw = smem + PG_OFF_RAW;
    uint64_t* bars = (uint64_t*)(smem + PG_OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + PG_NST;
    uint64_t* accfull = bars + 2 * PG_NST;
    uint64_t* accempty = accfull + 2;
    uint64_t* drain = accempty + 2;
    uint64_t* rawfull = drain + 1;
    uint64_t* rawempty = rawfull + PG_RAW_NST;
    uintptr_t* rowp = (uintptr_t*)(smem + PG_OFF_ROWP);
    uint32_t* tmem_slot = (uint32_t*)(smem + PG_OFF_MISC);
    volatile int* abort_flag = (volatile int*)(smem + PG_OFF_MISC + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    constexpr int TILES = HIDDEN / (2 * PG_M);                            // 28 pairs of 128-row tiles
    const int nitems = nslots * TILES;
    if ((int)blockIdx.x >= nitems) return;
    constexpr int K = MOE_INTER;
    constexpr int NKB = K / PG_KB;
    const size_t rowbytes = (size_t)(K / QK) * BLK_IQ2;
    const __half* btiles = p.ht;

    init_pair_tables((uint2*)(smem + PG_OFF_GTAB), (uint2*)(smem + PG_OFF_STAB), tid, PG_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        // full: 16 decode-warp arrivals + the copy warp's expect_tx arrival (B bytes)
        for (int s = 0; s < PG_NST; ++s) { mbar_init(&full[s], PG_DWARPS + 1); mbar_init(&empty[s], 1); }
        mbar_init(accfull, 1); mbar_init(accempty, PG_DWARPS);
        mbar_init(drain, 1);
        for (int s = 0; s < PG_RAW_NST; ++s) { mbar_init(&rawfull[s], 32); mbar_init(&rawempty[s], PG_DWARPS); }
        fence_mbar_init();
    }
    if (warp == PG_MMA_WARP) { tmem_alloc(tmem_slot, PG_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == PG_RAW_WARP) {
        // ---------------------------------------------------------------- raw superblocks (2 stages of K each)
        // runs up to PG_RAW_NST superblocks ahead of the decode warps, independently of the B stages
        uint32_t rit = 0;
        for (int item = blockIdx.x; item < nitems && !*abort_flag; item += gridDim.x) {
            const int s = item % nslots, rt = item / nslots;
            const int e = p.slot_expert[s];
            __syncwarp();
            for (int r = lane; r < 2 * PG_M; r += 32) rowp[r] = (uintptr_t)item_row(p, e, rt, r, rowbytes);
            __syncwarp();
            for (int sb = 0; sb < K / QK; ++sb, ++rit) {
                const int rs = rit % PG_RAW_NST;
                if (!mbar_wait_backoff(&rawempty[rs], ((rit / PG_RAW_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                uint8_t* dst = raw + rs * PG_RAW_STAGE;
                const size_t sboff = (size_t)sb * BLK_IQ2;
                if (lane < 30) {                      // lane -> (row rsub of 6, 16-byte chunk of 5)
                    const int rsub = lane / 5, chunk = lane - 5 * rsub;
                    #pragma unroll 4
                    for (int r = rsub; r < 2 * PG_M; r += 6) {
                        const uintptr_t a = (rowp[r] + sboff) & ~(uintptr_t)15;
                        cp_async16(dst + r * PG_RAW_ROWB + chunk * 16, (const void*)(a + 16 * chunk));
                    }
                }
                cp_async_mbar_arrive(&rawfull[rs]);
            }
        }
        cp_async_wait_all();
    } else if (warp == PG_COPY_WARP) {
        // ---------------------------------------------------------------- B tiles (one bulk copy per K-block)
        uint32_t it = 0;
        if (lane == 0) {
            for (int item = blockIdx.x; item < nitems && !*abort_flag; item += gridDim.x) {
                const int s = item % nslots;
                const int n16 = round16(p.slot_cnt[s]);
                for (int kb = 0; kb < NKB; ++kb, ++it) {
                    const int st = it % PG_NST;
                    if (!mbar_wait_backoff(&empty[st], ((it / PG_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                    const uint32_t bytes = (uint32_t)n16 * PG_KB * 2;
                    mbar_arrive_expect_tx(&full[st], bytes);
                    bulk_g2s(bring + st * PG_B_TILE, btiles + ((size_t)s * NKB + kb) * (PG_B_TILE / 2), bytes, &full[st]);
                }
            }
            // every bulk copy issued must land before the CTA may exit
            const uint32_t first = it > PG_NST ? it - PG_NST : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait_backoff(&full[j % PG_NST], (j / PG_NST) & 1, nullptr, 0);
        }
    } else if (warp == PG_MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer (the whole warp, elect.sync)
        // every lane runs the loop on the same values (broadcast from lane 0 where they come from memory), so
        // the operands are warp-uniform; each decision after a bounded wait is taken by the whole warp
        uint32_t it = 0; int issued = 0;
        const uint32_t bring_s = smem_u32(bring);
        for (int i = 0, item = blockIdx.x; item < nitems; ++i, item += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            const int s = item % nslots;
            const int N = __shfl_sync(0xffffffffu, round16(p.slot_cnt[s]), 0);
            const uint32_t idesc = idesc_f16_f32(PG_M, N);
            const uint32_t lbo = (uint32_t)(N >> 3) * 128;
            if (i >= 1 && !__all_sync(0xffffffffu, mbar_wait_backoff(accempty, (i - 1) & 1, p.err, DEV_ERR_TIMEOUT_EMPTY))) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d0 = tmem, d1 = d0 + PG_NMAX;
            const uint64_t bstep = (uint64_t)((2 * lbo) >> 4);             // one K=16 step along the B tile
            bool ok = true;
            for (int kb = 0; kb < NKB; ++kb, ++it) {
                const int st = it % PG_NST;
                if (!__all_sync(0xffffffffu, mbar_wait_backoff(&full[st], (it / PG_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL))) { ok = false; break; }
                tc_fence_after();
                const uint64_t b0 = umma_desc(bring_s + st * PG_B_TILE, lbo, 128);
                const uint32_t a0 = tmem + PG_ACC_COLS + st * PG_A_COLS, a1 = a0 + PG_A_COLS / 2;
                #pragma unroll
                for (int ks = 0; ks < PG_KB / 16; ++ks) {
                    const uint64_t bd = b0 + (uint64_t)ks * bstep;
                    umma_f16_ta_warp(d0, a0 + ks * 8, bd, idesc, (kb | ks) != 0);
                    umma_f16_ta_warp(d1, a1 + ks * 8, bd, idesc, (kb | ks) != 0);
                }
                umma_commit_warp(&empty[st]);
                issued = 1;
            }
            if (!ok) { if (lane == 0) *abort_flag = 1; break; }
            umma_commit_warp(accfull);
        }
        if (issued) {                                 // every issued MMA has completed before teardown
            umma_commit_warp(drain);
            mbar_wait_backoff(drain, 0, nullptr, 0);
        }
    } else {
        // ---------------------------------------------------------------- decode warps, then epilogue
        // warp w: TMEM lane quarter q = w & 3 (its rows), tile mat, groups 2gp, 2gp + 1 of every K-block
        const int q = warp & 3, mat = (warp >> 2) & 1, gp = warp >> 3;
        const int row = 32 * q + lane;                                      // weight row in tile `mat` = TMEM lane
        const uint2* gtl = gtab + lane;
        const uint2* stl = stab + lane;
        const uint8_t* rrow0 = raw + (mat * PG_M + row) * PG_RAW_ROWB;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t it = 0, rit = 0;
        for (int i = 0, item = blockIdx.x; item < nitems; ++i, item += gridDim.x) {
            const int s = item % nslots, rt = item / nslots;
            const int e = p.slot_expert[s];
            const uintptr_t wrow = (uintptr_t)item_row(p, e, rt, mat * PG_M + row, rowbytes);   // global row
            for (int kb = 0; kb < NKB; ++kb, ++it) {
                const int st = it % PG_NST, rs = rit % PG_RAW_NST;
                if ((kb & 1) == 0 && !*abort_flag && !mbar_wait_backoff(&rawfull[rs], (rit / PG_RAW_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL))
                    *abort_flag = 1;
                // the superblock sits `delta` (0..14) bytes into its staged 16-aligned window
                const uint8_t* rrow = rrow0 + rs * PG_RAW_STAGE;
                const int delta = (int)((wrow + (uintptr_t)(kb >> 1) * BLK_IQ2) & 15u);
                const int g0 = (kb & 1) * 4 + 2 * gp;                      // first of this thread's groups in the superblock
                uint32_t aux0a, aux1a, aux0b, aux1b;
                load_group_smem(rrow, delta + 2 + 8 * g0, aux0a, aux1a);
                load_group_smem(rrow, delta + 10 + 8 * g0, aux0b, aux1b);
                const float d = __half2float(*(const __half*)(rrow + delta));
                uint32_t oa[16], ob[16];
                decode_group_f16(aux0a, aux1a, d, gtl, stl, oa);
                decode_group_f16(aux0b, aux1b, d, gtl, stl, ob);
                if (!*abort_flag && !mbar_wait_backoff(&empty[st], ((it / PG_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) *abort_flag = 1;
                tc_fence_after();
                const uint32_t ta = tmem + lane_base + PG_ACC_COLS + st * PG_A_COLS + mat * (PG_A_COLS / 2) + gp * 32;
                tmem_st16(ta, oa);
                tmem_st16(ta + 16, ob);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full[st]);
                    if (kb & 1) mbar_arrive(&rawempty[rs]);
                }
                if (kb & 1) ++rit;
                if (*abort_flag) break;
            }
            if (*abort_flag) break;
            // ------------------------------------------------ epilogue of item i
            if (!mbar_wait_backoff(accfull, i & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { *abort_flag = 1; break; }
            tc_fence_after();
            const int cnt = p.slot_cnt[s];
            for (int cc = warp >> 2; cc * 16 < cnt; cc += 4) {              // tokens 16cc..16cc+15
                const uint32_t t0 = tmem + (uint32_t)(cc * 16) + lane_base;
                float v0[16], v1[16];
                tmem_ld16(t0, v0);
                tmem_ld16(t0 + PG_NMAX, v1);
                #pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = cc * 16 + j;
                    if (n < cnt) {
                        const int out = p.slot_out[s * PG_NMAX + n];
                        const float w = p.slot_w[s * PG_NMAX + n];
                        const int r0 = rt * 2 * PG_M + row;
                        p.y[(size_t)out * HIDDEN + r0] = w * v0[j];
                        p.y[(size_t)out * HIDDEN + r0 + PG_M] = w * v1[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accempty);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PG_MMA_WARP) { tc_fence_after(); tmem_dealloc(tmem, PG_TMEM_COLS); }
}

void launch_prefill_gemm_down(const GemmParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_prefill_down, cudaFuncAttributeMaxDynamicSharedMemorySize, PG_SMEM); attr = true; }
    k_prefill_down<<<grid, PG_THREADS, PG_SMEM, st>>>(p);
}

size_t down_tile_halfs(int max_slots) { return (size_t)max_slots * (MOE_INTER / PG_KB) * (PG_B_TILE / 2); }

}  // namespace lk
