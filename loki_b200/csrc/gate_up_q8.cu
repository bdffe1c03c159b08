// gate_up_q8.cu -- the gate/up + SwiGLU phase of the batch regimes (T >= the mma threshold) on the 5th-generation
// tensor cores, with the reference's numerics: products as exact as its int8 group sums, then h re-quantised
// to q8 per 32 (reference src/fused_layer.cu:334-341 swiglu_q8, as the wide pass uses it at :540-553).
//
// Why the products must be exact: the reference forms each 32-weight group sum in int32 (q8 x against the
// IQ2 grid values) and scales it in float, then quantises h = silu(g)*u to q8.  A product that differs from
// it by fp16 operand rounding (~2.4e-4 per element, the plain fp16 GEMM's error) moves h across q8 rounding
// boundaries, and those flips alone cost ~2-3e-3 relative L2 in the layer output.  Here:
//   * A (weights) = v * (2*scale + 1), an integer of at most 43*31 = 1333: exact in fp16.  The decode is the
//     byte-permute + hfma2 of iq2_tc.cuh with s = 2*scale + 1 (1024*s exact, the fma result an exact
//     integer).  The superblock's d/8 is applied outside the MMA, per superblock (below).
//   * B (activations) = the q8-dequantised x, q*dx in fp32, as two fp16 rows: hi = fp16(q*dx) and
//     lo = fp16(q*dx - hi).  hi + lo carries ~22 bits; products with the 11-bit A are exact in the fp32
//     accumulator.  The two rows sit side by side along N, so one MMA of N' = 2N covers both.
//   * Per superblock (256 weights, 2 K-blocks) the MMA accumulates P = sum A*B into a fresh TMEM buffer (two
//     buffers alternate); epilogue warps fold R += (d/8) * (P_hi + P_lo) into a running sum R in TMEM.
//     (hi + lo of one accumulator are summed in fp32 first, then the accumulators, then scaled: fp32 rounding
//     at the level of the reference's own float reassociation.)
//   * After the last superblock, R is g (rows 0-63 of the tile) or u (rows 64-127); the epilogue forms
//     h = silu(g)*u, quantises it per 32 (d = amax/127, round half even: quant_q8_group bit for bit) and
//     writes fp16(q*d) -- exactly representable up to fp16 rounding of the product -- as the down's input:
//     the down GEMM's B tiles (p.ht) or fp16 rows (p.hb) for the K-quant downs.
//
// Work item = (slot s, h tile rt of 64 rows, token half nh): M = 128 weight rows (64 gate rows + the same 64
// up rows), N = up to 64 tokens (a slot of up to GEMM_NT = 128 tokens is two halves; the second is skipped
// when the slot holds <= 64).  TMEM (512 columns): three A stages of 64 columns at 0, 64 and 192, R [128,192),
// P buffers [256,384) and [384,512).  The decode tables have 16 lane copies (48 KB).
//   A dependent tcgen05.mma (one accumulator, K = 16) measured ~260 cycles whatever N is up to 128, while one of
//   M=128, N'=32 is ~16 cycles of tensor work.  So a superblock's K steps go round-robin to nacc = 128 / N'
//   independent accumulators inside its P buffer (4 at N' = 32, 2 at N' = 64, 1 above), which the fold sums.
//
// Warp roles (736 threads, one CTA per SM, persistent over items):
//   warps 0-15  decode: warp w = TMEM lane quarter w&3 (rows 32*(w&3)..), group w>>2 of each K-block; writes
//               its 32 fp16 A values per K-block to tensor memory with tcgen05.st
//   warp 16     MMA issuer (whole warp, warp-uniform operands, elect.sync issues), 8 MMAs per K-block; at a
//               superblock's first K-block it waits for its P buffer to be drained, at its last it commits
//   warp 17     B K-block tiles (hi and lo rows of the item's token half) by 1-D TMA bulk copies
//   warp 18     raw superblocks: each weight row's next IQ2 superblock (80-byte 16-aligned window, 16-byte
//               cp.async, coalesced) into a 4-stage raw ring
//   warps 19-22 epilogue: warp w = lane quarter w&3; per superblock the P -> R fold, per item SwiGLU + q8
// Every wait is bounded (moe_device.cuh); a timed-out wait records an error code and the CTA unwinds.
#include "moe_internal.h"
#include "moe_device.cuh"
#include "tcgen05.cuh"
#include "iq2_tc.cuh"

namespace lk {

namespace {

constexpr int GQ_M = 128;                       // weight rows per item: 64 gate + 64 up
constexpr int GQ_H = 64;                        // h rows per item
constexpr int GQ_TILES = MOE_INTER / GQ_H;      // 32
constexpr int GQ_NH = 64;                       // tokens per item (half of a GEMM_NT slot)
constexpr int GQ_KB = 128;                      // K per stage
constexpr int GQ_NKB = HIDDEN / GQ_KB;          // 56
constexpr int GQ_NSB = HIDDEN / QK;             // 28 superblocks per row
constexpr int GQ_NST = 3;                       // A (TMEM) / B (smem) stages
constexpr int GQ_DWARPS = 16;
constexpr int GQ_MMA_WARP = GQ_DWARPS, GQ_COPY_WARP = GQ_DWARPS + 1, GQ_RAW_WARP = GQ_DWARPS + 2;
constexpr int GQ_EPI_WARP0 = GQ_DWARPS + 3, GQ_EWARPS = 4;
constexpr int GQ_THREADS = (GQ_EPI_WARP0 + GQ_EWARPS) * 32;     // 736
constexpr int GQ_B_HALF = 2 * GQ_NH * GQ_KB * 2;                // 32 KB: hi + lo rows of one half, N = 64
constexpr int GQ_RAW_ROWB = 80;
constexpr int GQ_RAW_STAGE = GQ_M * GQ_RAW_ROWB;                // 10 KB
constexpr int GQ_RAW_NST = 4;
constexpr int GQ_XS = GQ_NH + 1;                                // exchange row stride (floats)
constexpr int GQ_OFF_GTAB = 0;
constexpr int GQ_OFF_STAB = GQ_OFF_GTAB + IQ2TC_GTAB16;
constexpr int GQ_OFF_B = GQ_OFF_STAB + IQ2TC_STAB16;
constexpr int GQ_OFF_RAW = GQ_OFF_B + GQ_NST * GQ_B_HALF;
constexpr int GQ_OFF_X = GQ_OFF_RAW + GQ_RAW_NST * GQ_RAW_STAGE + 64;   // + slack for the last row's over-read
constexpr int GQ_OFF_BAR = GQ_OFF_X + GQ_H * GQ_XS * 4;
constexpr int GQ_NBAR = 2 * GQ_NST + 4 + 1 + 2 * GQ_RAW_NST;
constexpr int GQ_OFF_ROWP = GQ_OFF_BAR + GQ_NBAR * 8;
constexpr int GQ_OFF_MISC = GQ_OFF_ROWP + GQ_M * 8;
constexpr int GQ_SMEM_USED = GQ_OFF_MISC + 32;
constexpr int GQ_SMEM = 232448;                                 // all of it: one CTA per SM (all 512 TMEM columns)
static_assert(GQ_SMEM_USED <= GQ_SMEM, "shared memory layout exceeds the allocation");
static_assert(GQ_OFF_B % 1024 == 0 && GQ_B_HALF % 1024 == 0, "B stages 16-byte (bulk copy) aligned");
constexpr uint32_t GQ_TMEM_COLS = 512;
constexpr uint32_t GQ_A_COLS = GQ_KB / 2;       // 64 per stage: 128 fp16 K values
constexpr uint32_t GQ_R_COL = 128, GQ_P_COL = 256, GQ_P_COLS = 128;
// A stages at columns 0, 64 and 192 (R sits at 128 .. 192)
__device__ __forceinline__ uint32_t gq_a_col(int st) { return st < 2 ? (uint32_t)st * GQ_A_COLS : 192u; }
static_assert(2 * GQ_A_COLS <= GQ_R_COL && GQ_R_COL + GQ_NH <= 192 && 192 + GQ_A_COLS <= GQ_P_COL &&
              GQ_P_COL + 2 * GQ_P_COLS <= GQ_TMEM_COLS, "tensor memory layout");
constexpr int GQ_EPI_BAR = 1;                   // named barrier of the 4 epilogue warps

// tensor memory -> registers without the wait (tcgen05.wait::ld before the values are used)
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// independent accumulators per P buffer for N' = 2 * round16(tokens) columns each (a power of two, <= 4)
__device__ __forceinline__ int gq_nacc(int n2) { return n2 <= 32 ? 4 : (n2 <= 64 ? 2 : 1); }

// the 8 MMAs of one K-block with N' = N2 known at compile time, as one asm block: one elect.sync, the
// instruction descriptor and the A / B / accumulator steps as immediates, the descriptor's high word shared
// (the MMA warp shares its sub-partition with busy decode warps, so its issue slots are scarce)
template <int N2>
__device__ __forceinline__ void gq_issue_kblock(uint32_t d, uint32_t a0, uint32_t bring_st, int kb) {
    constexpr int nacc = N2 <= 32 ? 4 : (N2 <= 64 ? 2 : 1);
    constexpr uint32_t idesc = idesc_f16_f32(GQ_M, N2);
    constexpr uint32_t lbo = (uint32_t)(N2 >> 3) * 128;
    constexpr uint32_t bstep = (2 * lbo) >> 4;                          // one K=16 step along the B tile
    const uint64_t b0 = umma_desc(bring_st, lbo, 128);
    const uint32_t blo = (uint32_t)b0, bhi = (uint32_t)(b0 >> 32);
    // K step ks: A columns a0 + 8 ks, B start + ks * bstep, accumulator ks % nacc; the first nacc steps
    // accumulate only in the superblock's second K-block
    asm volatile("{\n\t.reg .pred e, q0, q1, q2, q3, q4, q5, q6, q7;\n\t.reg .b32 aa, bl, dd;\n\t.reg .b64 bd;\n\t"
        "setp.ne.b32 q0, %5, 0;\n\t"
        "setp.ne.b32 q1, %5, %30;\n\t" "setp.ne.b32 q2, %5, %31;\n\t" "setp.ne.b32 q3, %5, %32;\n\t"
        "setp.ne.b32 q4, %5, %33;\n\t" "setp.ne.b32 q5, %5, %34;\n\t" "setp.ne.b32 q6, %5, %35;\n\t" "setp.ne.b32 q7, %5, %36;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "add.u32 aa, %1, %6;\n\t" "add.u32 bl, %2, %14;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %22;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q0;\n\t"
        "add.u32 aa, %1, %7;\n\t" "add.u32 bl, %2, %15;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %23;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q1;\n\t"
        "add.u32 aa, %1, %8;\n\t" "add.u32 bl, %2, %16;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %24;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q2;\n\t"
        "add.u32 aa, %1, %9;\n\t" "add.u32 bl, %2, %17;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %25;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q3;\n\t"
        "add.u32 aa, %1, %10;\n\t" "add.u32 bl, %2, %18;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %26;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q4;\n\t"
        "add.u32 aa, %1, %11;\n\t" "add.u32 bl, %2, %19;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %27;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q5;\n\t"
        "add.u32 aa, %1, %12;\n\t" "add.u32 bl, %2, %20;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %28;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q6;\n\t"
        "add.u32 aa, %1, %13;\n\t" "add.u32 bl, %2, %21;\n\t" "mov.b64 bd, {bl, %3};\n\t" "add.u32 dd, %0, %29;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [dd], [aa], bd, %4, q7;\n\t"
        "}"
        :: "r"(d), "r"(a0), "r"(blo), "r"(bhi), "n"(idesc), "r"((uint32_t)(kb & 1)),
           "n"(0), "n"(8), "n"(16), "n"(24), "n"(32), "n"(40), "n"(48), "n"(56),
           "n"(0), "n"(bstep), "n"(2 * bstep), "n"(3 * bstep), "n"(4 * bstep), "n"(5 * bstep), "n"(6 * bstep), "n"(7 * bstep),
           "n"(0), "n"((1 % nacc) * N2), "n"((2 % nacc) * N2), "n"((3 % nacc) * N2), "n"((4 % nacc) * N2),
           "n"((5 % nacc) * N2), "n"((6 % nacc) * N2), "n"((7 % nacc) * N2),
           "n"(1 < nacc ? 0 : 7), "n"(2 < nacc ? 0 : 7), "n"(3 < nacc ? 0 : 7), "n"(4 < nacc ? 0 : 7),
           "n"(5 < nacc ? 0 : 7), "n"(6 < nacc ? 0 : 7), "n"(7 < nacc ? 0 : 7)
        : "memory");
}

__device__ __forceinline__ void tmem_st16f(uint32_t taddr, const float (&v)[16]) {
    uint32_t r[16];
    #pragma unroll
    for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(v[i]);
    tmem_st16(taddr, r);
}

// global weight row r (0..127) of item (expert e, h tile rt): rows 0-63 gate rows rt*64.., 64-127 the up rows
__device__ __forceinline__ const uint8_t* gq_row(const GemmParams& p, int e, int rt, int r) {
    const int mat = r >> 6, row = rt * GQ_H + (r & (GQ_H - 1));
    const uint8_t* wm = e == SHARED_SLOT ? (mat ? p.sh_up : p.sh_gate)
                                         : (mat ? p.up + (size_t)e * p.up_stride : p.gate + (size_t)e * p.gate_stride);
    return wm + (size_t)row * ((HIDDEN / QK) * BLK_IQ2);
}

// item -> (slot, h tile, token half); false when the half holds no token.  Slot-major: the CTAs working at one
// time share a few slots, so each slot's activation tiles come from DRAM once and then from L2 for all of its
// h tiles (h-tile-major order re-read them from DRAM per tile: 4.3x the algorithmic bytes at T=512), and a
// hot expert's consecutive slots re-read its rows from L2
__device__ __forceinline__ bool gq_item(const GemmParams& p, int item, int nslots, int& s, int& rt, int& nh, int& cnt_h) {
    (void)nslots;
    s = item / (2 * GQ_TILES);
    const int rest = item - s * (2 * GQ_TILES);
    nh = rest / GQ_TILES; rt = rest - nh * GQ_TILES;
    cnt_h = p.slot_cnt[s] - GQ_NH * nh;
    cnt_h = cnt_h > GQ_NH ? GQ_NH : cnt_h;
    return cnt_h > 0;
}

}  // namespace

__global__ void __launch_bounds__(GQ_THREADS, 1) k_gate_up_q8(GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint2* gtab = (const uint2*)(smem + GQ_OFF_GTAB);
    const uint2* stab = (const uint2*)(smem + GQ_OFF_STAB);
    uint8_t* bring = smem + GQ_OFF_B;
    uint8_t* raw = smem + GQ_OFF_RAW;
    float* xchg = (float*)(smem + GQ_OFF_X);
    uint64_t* bars = (uint64_t*)(smem + GQ_OFF_BAR);
    uint64_t* full = bars;
    uint64_t* empty = bars + GQ_NST;
    uint64_t* pfull = bars + 2 * GQ_NST;
    uint64_t* pempty = pfull + 2;
    uint64_t* drain = pempty + 2;
    uint64_t* rawfull = drain + 1;
    uint64_t* rawempty = rawfull + GQ_RAW_NST;
    uintptr_t* rowp = (uintptr_t*)(smem + GQ_OFF_ROWP);
    uint32_t* tmem_slot = (uint32_t*)(smem + GQ_OFF_MISC);
    volatile int* abort_flag = (volatile int*)(smem + GQ_OFF_MISC + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nslots = *p.nslots;
    const int nitems = nslots * GQ_TILES * 2;
    if ((int)blockIdx.x >= nitems) return;

    init_pair_tables16((uint2*)(smem + GQ_OFF_GTAB), (uint2*)(smem + GQ_OFF_STAB), tid, GQ_THREADS);
    if (tid == 0) {
        *abort_flag = 0;
        // full: 16 decode-warp arrivals + the copy warp's expect_tx arrival (B bytes)
        for (int s = 0; s < GQ_NST; ++s) { mbar_init(&full[s], GQ_DWARPS + 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&pfull[b], 1); mbar_init(&pempty[b], GQ_EWARPS); }
        mbar_init(drain, 1);
        for (int s = 0; s < GQ_RAW_NST; ++s) { mbar_init(&rawfull[s], 32); mbar_init(&rawempty[s], GQ_DWARPS); }
        fence_mbar_init();
    }
    if (warp == GQ_MMA_WARP) { tmem_alloc(tmem_slot, GQ_TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == GQ_RAW_WARP) {
        // ---------------------------------------------------------------- raw superblocks
        uint32_t rit = 0;
        const int rsub = lane / 5, chunk = lane - 5 * (lane / 5);
        for (int item = blockIdx.x; item < nitems && !*abort_flag; item += gridDim.x) {
            int s, rt, nh, cnt_h;
            if (!gq_item(p, item, nslots, s, rt, nh, cnt_h)) continue;
            const int e = p.slot_expert[s];
            __syncwarp();
            for (int r = lane; r < GQ_M; r += 32) rowp[r] = (uintptr_t)gq_row(p, e, rt, r);
            __syncwarp();
            for (int sb = 0; sb < GQ_NSB; ++sb, ++rit) {
                const int rs = rit % GQ_RAW_NST;
                if (!mbar_wait_backoff(&rawempty[rs], ((rit / GQ_RAW_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                uint8_t* dst = raw + rs * GQ_RAW_STAGE;
                const size_t sboff = (size_t)sb * BLK_IQ2;
                if (lane < 30) {                      // lane -> (row rsub of 6, 16-byte chunk of 5)
                    #pragma unroll 4
                    for (int r = rsub; r < GQ_M; r += 6) {
                        const uintptr_t a = (rowp[r] + sboff) & ~(uintptr_t)15;
                        cp_async16(dst + r * GQ_RAW_ROWB + chunk * 16, (const void*)(a + 16 * chunk));
                    }
                }
                cp_async_mbar_arrive(&rawfull[rs]);
            }
        }
        cp_async_wait_all();
    } else if (warp == GQ_COPY_WARP) {
        // ---------------------------------------------------------------- B tiles (one bulk copy per K-block)
        uint32_t it = 0;
        if (lane == 0) {
            for (int item = blockIdx.x; item < nitems && !*abort_flag; item += gridDim.x) {
                int s, rt, nh, cnt_h;
                if (!gq_item(p, item, nslots, s, rt, nh, cnt_h)) continue;
                const uint32_t bytes = (uint32_t)(2 * round16(cnt_h)) * GQ_KB * 2;
                for (int kb = 0; kb < GQ_NKB; ++kb, ++it) {
                    const int st = it % GQ_NST;
                    if (!mbar_wait(&empty[st], ((it / GQ_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                    mbar_arrive_expect_tx(&full[st], bytes);
                    bulk_g2s(bring + st * GQ_B_HALF, p.bt + (((size_t)s * GQ_NKB + kb) * 2 + nh) * (GQ_B_HALF / 2), bytes, &full[st]);
                }
                if (*abort_flag) break;
            }
            // every bulk copy issued must land before the CTA may exit
            const uint32_t first = it > GQ_NST ? it - GQ_NST : 0;
            for (uint32_t j = first; j < it; ++j) mbar_wait_backoff(&full[j % GQ_NST], (j / GQ_NST) & 1, nullptr, 0);
        }
    } else if (warp == GQ_MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer (the whole warp, elect.sync)
        uint32_t it = 0, psb = 0; int issued = 0;
        const uint32_t bring_s = smem_u32(bring);
        bool ok = true;
        for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            int s, rt, nh, cnt_h;
            if (!gq_item(p, item, nslots, s, rt, nh, cnt_h)) continue;
            const int N2 = __shfl_sync(0xffffffffu, 2 * round16(cnt_h), 0);       // hi rows then lo rows
            for (int kb = 0; kb < GQ_NKB; ++kb, ++it) {
                const int st = it % GQ_NST;
                const uint32_t b = psb & 1;
                if ((kb & 1) == 0 &&
                    !__all_sync(0xffffffffu, mbar_wait(&pempty[b], ((psb >> 1) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY))) { ok = false; break; }
                if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (it / GQ_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL))) { ok = false; break; }
                tc_fence_after();
                const uint32_t a0 = tmem + gq_a_col(st);
                const uint32_t d = tmem + GQ_P_COL + b * GQ_P_COLS;
                const uint32_t bst = bring_s + st * GQ_B_HALF;
                switch (N2) {
                    case 32: gq_issue_kblock<32>(d, a0, bst, kb); break;
                    case 64: gq_issue_kblock<64>(d, a0, bst, kb); break;
                    case 96: gq_issue_kblock<96>(d, a0, bst, kb); break;
                    default: gq_issue_kblock<128>(d, a0, bst, kb); break;
                }
                umma_commit_warp(&empty[st]);
                issued = 1;
                if (kb & 1) { umma_commit_warp(&pfull[b]); ++psb; }
            }
        }
        if (!ok && lane == 0) *abort_flag = 1;
        if (issued) {                                 // every issued MMA has completed before teardown
            umma_commit_warp(drain);
            mbar_wait_backoff(drain, 0, nullptr, 0);
        }
    } else if (warp < GQ_DWARPS) {
        // ---------------------------------------------------------------- decode warps
        const int q = warp & 3, gsel = warp >> 2;
        const int row = 32 * q + lane;                                      // weight row of the item = TMEM lane
        const uint2* gtl = gtab + (lane & 15);
        const uint2* stl = stab + (lane & 15);
        const uint8_t* rrow0 = raw + row * GQ_RAW_ROWB;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t it = 0, rit = 0;
        for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
            int s, rt, nh, cnt_h;
            if (!gq_item(p, item, nslots, s, rt, nh, cnt_h)) continue;
            const int e = p.slot_expert[s];
            const uint32_t wlo = (uint32_t)(uintptr_t)gq_row(p, e, rt, row);
            for (int kb = 0; kb < GQ_NKB; ++kb, ++it) {
                const int st = it % GQ_NST, rs = rit % GQ_RAW_NST;
                if ((kb & 1) == 0 && !*abort_flag && !mbar_wait(&rawfull[rs], (rit / GQ_RAW_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL))
                    *abort_flag = 1;
                const uint8_t* rrow = rrow0 + rs * GQ_RAW_STAGE;
                const int delta = (int)((wlo + (uint32_t)(kb >> 1) * BLK_IQ2) & 15u);   // superblock offset in its window
                const int g0 = (kb & 1) * 4 + gsel;                         // this thread's group in the superblock
                uint32_t aux0, aux1;
                load_group_smem(rrow, delta + 2 + 8 * g0, aux0, aux1);
                // A = v * (2*scale + 1): integers <= 1333, exact in fp16; d/8 is applied per superblock
                const uint32_t sc = 2u * (aux1 >> 28) + 1u;
                const uint32_t s2 = (uint32_t)__half_as_ushort(__uint2half_rn(sc)) * 0x10001u;
                const uint32_t c2 = (uint32_t)__half_as_ushort(__uint2half_rn(1024u * sc)) * 0x10001u ^ 0x80008000u;
                uint32_t o[16];
                decode_group_f16_s<16>(aux0, aux1, s2, c2, gtl, stl, o);
                if (!*abort_flag && !mbar_wait(&empty[st], ((it / GQ_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) *abort_flag = 1;
                tc_fence_after();
                tmem_st16(tmem + lane_base + gq_a_col(st) + gsel * 16, o);
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
        }
    } else {
        // ---------------------------------------------------------------- epilogue warps
        const int q = warp & 3;                                             // TMEM lane quarter of this warp
        const int row = 32 * q + lane, mat = q >> 1, j = 32 * (q & 1) + lane;   // j: h row in the tile
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t tR = tmem + lane_base + GQ_R_COL;
        uint32_t psb = 0;
        bool bad = false;
        for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
            int s, rt, nh, cnt_h;
            if (!gq_item(p, item, nslots, s, rt, nh, cnt_h)) continue;
            const int e = p.slot_expert[s];
            const int n16 = round16(cnt_h);
            const __half* dptr = (const __half*)gq_row(p, e, rt, row);      // the superblock scales d of this row
            float dnext = __half2float(dptr[0]);
            for (int sb = 0; sb < GQ_NSB; ++sb, ++psb) {
                const float dw = dnext * 0.125f;                            // d * (0.5 + scale) * 0.25 = d/8 * A's factor
                if (sb + 1 < GQ_NSB) dnext = __half2float(dptr[(size_t)(sb + 1) * (BLK_IQ2 / 2)]);
                const uint32_t b = psb & 1;
                if (!bad && (*abort_flag || !mbar_wait(&pfull[b], (psb >> 1) & 1, p.err, DEV_ERR_TIMEOUT_FULL))) bad = true;
                if (!bad) {
                    tc_fence_after();
                    const uint32_t tP = tmem + lane_base + GQ_P_COL + b * GQ_P_COLS;
                    const int n2 = 2 * n16, nacc = gq_nacc(n2);
                    for (int c0 = 0; c0 < n16; c0 += 16) {
                        float sum[16], r[16];
                        #pragma unroll
                        for (int i = 0; i < 16; ++i) sum[i] = 0.0f;
                        for (int j = 0; j < nacc; ++j) {           // P = sum over the accumulators of hi + lo
                            uint32_t hi[16], lo[16];
                            tmem_ld16_nowait(tP + j * n2 + c0, hi);
                            tmem_ld16_nowait(tP + j * n2 + n16 + c0, lo);
                            tmem_ld_wait();
                            #pragma unroll
                            for (int i = 0; i < 16; ++i) sum[i] += __uint_as_float(hi[i]) + __uint_as_float(lo[i]);
                        }
                        if (sb == 0) {
                            #pragma unroll
                            for (int i = 0; i < 16; ++i) r[i] = dw * sum[i];
                        } else {
                            tmem_ld16(tR + c0, r);
                            #pragma unroll
                            for (int i = 0; i < 16; ++i) r[i] = fmaf(dw, sum[i], r[i]);
                        }
                        if (sb + 1 < GQ_NSB || mat == 0) {
                            tmem_st16f(tR + c0, r);                         // running sum (g kept here at the end)
                        } else {                                            // final u -> the exchange for SwiGLU
                            #pragma unroll
                            for (int i = 0; i < 16; ++i) xchg[j * GQ_XS + c0 + i] = r[i];
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                }
                __syncwarp();
                if (lane == 0 && !bad) mbar_arrive(&pempty[b]);
            }
            // ------------------------------------------------ item epilogue: h = silu(g)*u, q8 per 32, fp16(q*d) out
            if (named_bar_or(GQ_EPI_BAR, GQ_EWARPS * 32, bad)) break;
            if (mat == 0) {
                const int hj = rt * GQ_H + j;                                  // h row of this lane
                const int n16s = round16(p.slot_cnt[s]);                      // the down's N for the whole slot
                for (int c0 = 0; c0 < n16; c0 += 16) {
                    float g[16];
                    tc_fence_after();
                    tmem_ld16(tR + c0, g);
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int n = c0 + i;
                        if (n >= cnt_h) break;                                 // warp-uniform
                        const float h = lk_swiglu(g[i], xchg[j * GQ_XS + n]);
                        float amax = fabsf(h);
                        #pragma unroll
                        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                        const float dq = amax / 127.0f, id = dq > 0.0f ? 1.0f / dq : 0.0f;
                        const __half hv = __float2half_rn((float)__float2int_rn(h * id) * dq);
                        const int ng = GQ_NH * nh + n;                         // token position in the slot
                        if (p.hb) {
                            const int out = p.slot_out[s * GEMM_NT + ng];
                            if (out >= 0) p.hb[(size_t)out * MOE_INTER + hj] = hv;
                        } else {
                            uint8_t* tile = (uint8_t*)(p.ht + ((size_t)s * (MOE_INTER / GQ_KB) + hj / GQ_KB) * (GEMM_NT * GQ_KB));
                            *(__half*)(tile + btile_off(ng, hj % GQ_KB, n16s)) = hv;
                        }
                    }
                }
            }
            if (named_bar_or(GQ_EPI_BAR, GQ_EWARPS * 32, bad)) break;       // the exchange is free again
        }
        if (bad) *abort_flag = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == GQ_MMA_WARP) { tc_fence_after(); tmem_dealloc(tmem, GQ_TMEM_COLS); }
}

// gate/up B tiles with the q8 numerics: for slot s, K-block kb and token half nh, the q8-dequantised x of the
// half's tokens (q * dx in fp32, quant_q8_group) as hi rows fp16(v) then lo rows fp16(v - hi), in the UMMA
// K-major core-matrix layout of 2 * round16(half count) rows (pad rows zero); also the slot's token count
constexpr int GQ_BT_THREADS = GEMM_NT * (GQ_KB / 32);   // one thread per (token row, 32-group of the K-block)
__global__ void __launch_bounds__(GQ_BT_THREADS) k_gate_b_tiles_q8(GemmParams p) {
    const int s = blockIdx.x, kb = blockIdx.y, tid = threadIdx.x;
    if (s >= *p.nslots) return;
    const int n = tid / (GQ_KB / 32), g = tid % (GQ_KB / 32);     // token row, 32-group within the K-block
    const int tok = p.slot_tok[s * GEMM_NT + n];
    const int cnt = __syncthreads_count(tok >= 0) / (GQ_KB / 32);   // pads are at the end of the slot
    if (kb == 0 && tid == 0) p.slot_cnt[s] = cnt;
    const int nh = n / GQ_NH, nl = n % GQ_NH;
    int cnt_h = cnt - GQ_NH * nh;
    cnt_h = cnt_h > GQ_NH ? GQ_NH : cnt_h;
    if (cnt_h <= 0) return;
    const int n16 = round16(cnt_h);
    if (nl >= n16) return;
    float v[32];
    if (tok >= 0) {
        const float4* src = (const float4*)(p.x + (size_t)tok * p.ld_x + kb * GQ_KB + g * 32);
        #pragma unroll
        for (int j = 0; j < 8; ++j) { const float4 a = src[j]; v[4*j] = a.x; v[4*j+1] = a.y; v[4*j+2] = a.z; v[4*j+3] = a.w; }
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.0f;
    }
    int8_t qv[32];
    const float d = quant_q8_group(v, qv);
    uint8_t* tile = (uint8_t*)(p.bt + (((size_t)s * GQ_NKB + kb) * 2 + nh) * (GQ_B_HALF / 2));
    #pragma unroll
    for (int c = 0; c < 4; ++c) {                        // 4 k8 blocks of 8 fp16 (16 bytes) each
        uint32_t whi[4], wlo[4];
        #pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int j = c * 8 + 2 * h;
            const float a0 = (float)qv[j] * d, a1 = (float)qv[j + 1] * d;
            const __half h0 = __float2half_rn(a0), h1 = __float2half_rn(a1);
            const __half l0 = __float2half_rn(a0 - __half2float(h0)), l1 = __float2half_rn(a1 - __half2float(h1));
            whi[h] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            wlo[h] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        *(uint4*)(tile + btile_off(nl, g * 32 + c * 8, 2 * n16)) = make_uint4(whi[0], whi[1], whi[2], whi[3]);
        *(uint4*)(tile + btile_off(n16 + nl, g * 32 + c * 8, 2 * n16)) = make_uint4(wlo[0], wlo[1], wlo[2], wlo[3]);
    }
}

void launch_gate_up_q8(const GemmParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_gate_up_q8, cudaFuncAttributeMaxDynamicSharedMemorySize, GQ_SMEM); attr = true; }
    k_gate_b_tiles_q8<<<dim3(p.max_slots, GQ_NKB), GQ_BT_THREADS, 0, st>>>(p);
    k_gate_up_q8<<<grid, GQ_THREADS, GQ_SMEM, st>>>(p);
}

size_t gate_q8_tile_halfs(int max_slots) { return (size_t)max_slots * GQ_NKB * 2 * (GQ_B_HALF / 2); }

}  // namespace lk
