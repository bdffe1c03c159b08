// expert_kq.cu -- the down projection for K-quant experts (Q2_K, Q3_K, Q6_K): the real DeepSeek-R1
// IQ2_XXS model's routed down matrices and its shared expert's down (the reference's tc_matvec<F_Q2K / F_Q3K>, src/fused_layer.cu:203-254,
// launched at :608 and :550).
//
// Contract as k_down1 (expert_gemv1.cu): single-token slots, the slot's SwiGLU output as q8 (hq, hd),
// y[entry][row] = w * (W_down h)[row].  Same CTA shape: a producer thread streams units of 32 rows (one
// bulk copy each: 21 504 B for Q2_K, 28 160 B for Q3_K) into an 8-stage ring; 16 consumer warps in 4
// groups, a warp computes whole-row dot products of 8 rows.
// Lane l owns 64 weights of K: block b = l / 4, quarter q = l % 4, i.e. K [256b + 64q, +64): qs bytes
// 32n..32n+31 of the block (n = q / 2) at bit pairs 2j, j = 2(q % 2) + {0, 1}, and the four 16-weight
// sub-blocks 4q..4q+3 -- whose four scale bytes (Q2_K) or four unpacked 6-bit scales (Q3_K, word q of
// ggml's kmask unpacking) are one 32-bit word.  The lane keeps its 64 q8 activations, their two group
// scales and four 16-wide sums in registers for the whole slot.  Per sub-block:
//   Q2_K: isum = sum q_w * q_x (dp4a over 2-bit fields), v += dx * (d*sc*isum - dmin*m*sum q_x)
//   Q3_K: w3 = low2 | hbit << 2 (0..7, value w3 - 4), isum = dp4a(w3, x) - 4 * sum q_x,
//         v += dx * d * (scale - 32) * isum
//   Q6_K (the real model's shared down, :131-158): q6 = low4 | high2 << 4 (0..63, value q6 - 32),
//         isum = dp4a(q6, x) - 32 * sum q_x, v += dx * d * scale * isum (int8 scales, one word per quarter)
// the reference's per-16 arithmetic with exact integer sums.  Q3_K (110 B) and Q6_K (210 B) blocks are only
// 2-byte aligned in shared memory, so their words are read as aligned pairs and funnel-shifted.  Q6_K units
// rows are 1 680 B, so its warps take 4 rows each (units of 16 rows, 26 880 B).
// Shared-only mode (slot_expert == null, launch_shared_kq): slot j is the shared expert of token j: h from
// hq/hd row sh_row0 + j, written to y row sh_row0 + j with weight 1.
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

namespace {

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v; asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a)); return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint16_t v; asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a)); return v;
}

template <int FMT> struct KqFmt;
template <> struct KqFmt<FMT_Q2K> { static constexpr int BLK = BLK_Q2K; };
template <> struct KqFmt<FMT_Q3K> { static constexpr int BLK = BLK_Q3K; };
template <> struct KqFmt<FMT_Q6K> { static constexpr int BLK = BLK_Q6K; };

constexpr int KQ_WARPS = 16;
constexpr int KQ_THREADS = (KQ_WARPS + 1) * 32;
constexpr int KQ_GWARPS = 4;                         // warps per group: a unit is 4 warps x kq_wrows rows
constexpr int KQ_GROUPS = KQ_WARPS / KQ_GWARPS;      // 4 groups

// rows per warp: 8, or 4 for Q6_K (the shared expert's down: one matrix per token, so at T = 1 each SM
// has ~48 rows and shorter units keep more warps busy)
template <int FMT> constexpr int kq_wrows() { return FMT == FMT_Q6K ? 4 : 8; }
template <int FMT> constexpr int kq_urows() { return KQ_GWARPS * kq_wrows<FMT>(); }          // 32 / 16 rows per unit
template <int FMT> constexpr int kq_units_per_slot() { return HIDDEN / kq_urows<FMT>(); }    // 224 / 448
template <int FMT> constexpr int kq_rowb() { return (MOE_INTER / QK) * KqFmt<FMT>::BLK; }     // 672 / 880 / 1680
template <int FMT> constexpr int kq_ubytes() { return kq_urows<FMT>() * kq_rowb<FMT>(); }
// ring stages: group g uses stages g and g + 4
template <int FMT> constexpr int kq_nst() { return 2 * KQ_GROUPS; }
template <int FMT> constexpr int kq_off_bar() { return kq_nst<FMT>() * kq_ubytes<FMT>(); }
template <int FMT> constexpr int kq_smem() { return kq_off_bar<FMT>() + 2 * kq_nst<FMT>() * 8 + 16; }
static_assert(kq_smem<FMT_Q3K>() <= 232448 && kq_smem<FMT_Q6K>() <= 232448, "K-quant ring exceeds shared memory");
static_assert(kq_rowb<FMT_Q2K>() % 16 == 0 && kq_rowb<FMT_Q3K>() % 16 == 0 && kq_rowb<FMT_Q6K>() % 16 == 0,
              "bulk copies need 16-byte rows");

__device__ __forceinline__ const uint8_t* kq_down_matrix(const ExpertParams& p, int e) {
    return e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride;
}

// the four 16-weight partial dot products of one row for this lane, scaled and summed
template <int FMT>
__device__ __forceinline__ float kq_row_dot(uint32_t blk, uint32_t sh, int q, const uint32_t (&xr)[16], const float (&dx)[2],
                                            const int (&xs)[4]) {
    const int n = q >> 1, j0 = 2 * (q & 1);
    float v = 0.0f;
    if (FMT == FMT_Q2K) {                                // block 4-byte aligned (84 = 4 * 21, rows 16-aligned)
        const uint32_t sc = lds_u32(blk + 4 * q);        // scale bytes of sub-blocks 4q .. 4q+3 (= 8n + 2j0 ..)
        const uint32_t dd = lds_u32(blk + Q2K_D);
        const float d = __half2float(__ushort_as_half((uint16_t)(dd & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(dd >> 16)));
        uint32_t qs[8];
        #pragma unroll
        for (int w = 0; w < 8; ++w) qs[w] = lds_u32(blk + Q2K_QS + 32 * n + 4 * w);
        #pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = j0 + jj;
            #pragma unroll
            for (int s = 0; s < 2; ++s) {
                int isum = 0;
                #pragma unroll
                for (int w = 0; w < 4; ++w) isum = __dp4a((int)((qs[4 * s + w] >> (2 * j)) & 0x03030303u), (int)xr[8 * jj + 4 * s + w], isum);
                const uint32_t scb = (sc >> (8 * (2 * jj + s))) & 0xFFu;
                const float t = fmaf(d * (float)(scb & 15u), (float)isum, -(dmin * (float)(scb >> 4)) * (float)xs[2 * jj + s]);
                v = fmaf(dx[jj], t, v);
            }
        }
    } else if (FMT == FMT_Q6K) {                         // block 2-byte aligned: blk = aligned base, sh = 0 or 16
        // quarter q: ql bytes 64n..64n+63 at nibble q & 1, qh bytes 128+32n.. at bit pairs 4(q&1) + 2(s16>>1),
        // int8 scales 4q..4q+3 (one word), 16-weight sub-block s16 = weights 64q + 16 s16 ..
        const int hs = q & 1;
        uint32_t ql[16], qh[8];
        {
            uint32_t a[17];
            #pragma unroll
            for (int w = 0; w < 17; ++w) a[w] = lds_u32(blk + 64 * n + 4 * w);
            #pragma unroll
            for (int w = 0; w < 16; ++w) ql[w] = __funnelshift_r(a[w], a[w + 1], sh);
            #pragma unroll
            for (int w = 0; w < 9; ++w) a[w] = lds_u32(blk + Q6K_QH + 32 * n + 4 * w);
            #pragma unroll
            for (int w = 0; w < 8; ++w) qh[w] = __funnelshift_r(a[w], a[w + 1], sh);
        }
        const uint32_t scw = __funnelshift_r(lds_u32(blk + Q6K_SC + 4 * q), lds_u32(blk + Q6K_SC + 4 * q + 4), sh);
        const float d = __half2float(__ushort_as_half((uint16_t)lds_u16(blk + Q6K_D + (sh >> 3))));
        #pragma unroll
        for (int s16 = 0; s16 < 4; ++s16) {
            int isum = 0;
            #pragma unroll
            for (int w = 0; w < 4; ++w) {
                const uint32_t q6 = ((ql[4 * s16 + w] >> (4 * hs)) & 0x0F0F0F0Fu) |
                                    (((qh[4 * (s16 & 1) + w] >> (4 * hs + 2 * (s16 >> 1))) & 0x03030303u) << 4);
                isum = __dp4a((int)q6, (int)xr[4 * s16 + w], isum);
            }
            isum -= 32 * xs[s16];
            const int scale = (int)(int8_t)(uint8_t)((scw >> (8 * s16)) & 0xFFu);
            v = fmaf(dx[s16 >> 1] * (d * (float)scale), (float)isum, v);
        }
    } else {                                             // block 2-byte aligned: blk = aligned base, sh = 0 or 16
        uint32_t hm[8], qs[8];
        {
            uint32_t a[9];
            #pragma unroll
            for (int w = 0; w < 9; ++w) a[w] = lds_u32(blk + 4 * w);
            #pragma unroll
            for (int w = 0; w < 8; ++w) hm[w] = __funnelshift_r(a[w], a[w + 1], sh);
            #pragma unroll
            for (int w = 0; w < 9; ++w) a[w] = lds_u32(blk + Q3K_QS + 32 * n + 4 * w);
            #pragma unroll
            for (int w = 0; w < 8; ++w) qs[w] = __funnelshift_r(a[w], a[w + 1], sh);
        }
        uint32_t scw;                                    // 4 unpacked scales (+32) of sub-blocks 4q..4q+3
        {
            const uint32_t lo_a = lds_u32(blk + Q3K_SC + 4 * (q & 1)), lo_b = lds_u32(blk + Q3K_SC + 4 * (q & 1) + 4);
            const uint32_t hi_a = lds_u32(blk + Q3K_SC + 8), hi_b = lds_u32(blk + Q3K_SC + 12);
            const uint32_t lw = __funnelshift_r(lo_a, lo_b, sh), hw = __funnelshift_r(hi_a, hi_b, sh);
            const uint32_t low = (q < 2 ? lw : (lw >> 4)) & 0x0F0F0F0Fu;
            scw = low | (((hw >> (2 * q)) & 0x03030303u) << 4);
        }
        const uint32_t doff = Q3K_D + (sh >> 3);
        const float d = __half2float(__ushort_as_half((uint16_t)lds_u16(blk + doff)));
        #pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = j0 + jj;
            #pragma unroll
            for (int s = 0; s < 2; ++s) {
                int isum = 0;
                #pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const uint32_t w3 = ((qs[4 * s + w] >> (2 * j)) & 0x03030303u) | (((hm[4 * s + w] >> (4 * n + j)) & 0x01010101u) << 2);
                    isum = __dp4a((int)w3, (int)xr[8 * jj + 4 * s + w], isum);
                }
                isum -= 4 * xs[2 * jj + s];
                const int scale = (int)((scw >> (8 * (2 * jj + s))) & 0xFFu) - 32;
                v = fmaf(dx[jj] * (d * (float)scale), (float)isum, v);
            }
        }
    }
    return v;
}

template <int FMT>
__global__ void __launch_bounds__(KQ_THREADS, 1) k_down1_kq(ExpertParams p) {
    constexpr int RB = kq_rowb<FMT>(), UB = kq_ubytes<FMT>(), KQ_NST = kq_nst<FMT>();
    constexpr int WROWS = kq_wrows<FMT>(), UROWS = kq_urows<FMT>(), UPS = kq_units_per_slot<FMT>();
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = (uint64_t*)(smem + kq_off_bar<FMT>());
    uint64_t* empty = full + KQ_NST;
    volatile int* abort_flag = (volatile int*)(empty + KQ_NST);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < KQ_NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], KQ_GWARPS); }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const bool sh_only = p.slot_expert == nullptr;   // shared-only slots (launch_shared_kq)
    const int nslots = sh_only ? p.sh_count : *p.nslots;
    const int nunits = nslots * UPS;
    const int u0 = (int)((long long)blockIdx.x * nunits / gridDim.x);
    const int nu = (int)((long long)(blockIdx.x + 1) * nunits / gridDim.x) - u0;
    if (nu <= 0) return;
    if (warp == KQ_WARPS) {                           // ---------------- producer
        if (lane == 0) {
            int j = 0;
            for (; j < nu; ++j) {
                const int u = u0 + j, s = u / UPS, cu = u % UPS;
                const int st = j % KQ_NST;
                if (*abort_flag || !mbar_wait(&empty[st], ((j / KQ_NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                const uint8_t* dw = kq_down_matrix(p, sh_only ? SHARED_SLOT : p.slot_expert[s]);
                mbar_arrive_expect_tx(&full[st], UB);
                bulk_g2s(ring + st * UB, dw + (size_t)cu * UB, UB, &full[st]);
            }
            {   // every issued copy must land before the CTA may exit
                const int first = j > KQ_NST ? j - KQ_NST : 0;
                for (int i = first; i < j; ++i) mbar_wait(&full[i % KQ_NST], (i / KQ_NST) & 1, nullptr, 0);
            }
        }
        return;
    }

    const uint32_t ring_s = smem_u32(ring);
    const int b = lane >> 2, q = lane & 3;
    const uint32_t boff = (uint32_t)(b * KqFmt<FMT>::BLK);
    const uint32_t balign = boff & ~3u, bsh = (boff & 3u) * 8u;          // Q3_K: odd blocks sit 2 bytes past a word
    const int grp = warp / KQ_GWARPS, sub = warp % KQ_GWARPS;
    uint32_t xr[16]; float dx[2] = {0.0f, 0.0f}; int xs[4] = {0, 0, 0, 0};
    int xslot = -1, out = -1;
    float wv = 0.0f;
    float* yrow = nullptr;
    for (int j = grp; j < nu; j += KQ_GROUPS) {
        const int u = u0 + j, s = u / UPS, cu = u % UPS;
        if (s != xslot) {                             // this slot's h (q8): K [256b + 64q, +64)
            xslot = s; out = sh_only ? p.sh_row0 + s : p.slot_out[s]; wv = sh_only ? 1.0f : p.slot_w[s];
            yrow = out < 0 ? nullptr : (p.ydst && !sh_only ? p.ydst[s] : p.y + (size_t)out * HIDDEN);
            if (out >= 0) {
                const uint4* src = (const uint4*)(p.hq + (size_t)out * MOE_INTER + b * QK + 64 * q);
                #pragma unroll
                for (int c = 0; c < 4; ++c) { const uint4 a = src[c]; xr[4*c] = a.x; xr[4*c+1] = a.y; xr[4*c+2] = a.z; xr[4*c+3] = a.w; }
                const float* hdp = p.hd + (size_t)out * (MOE_INTER / 32) + b * 8 + 2 * q;
                dx[0] = hdp[0]; dx[1] = hdp[1];
            } else {
                #pragma unroll
                for (int w = 0; w < 16; ++w) xr[w] = 0u;
                dx[0] = dx[1] = 0.0f;
            }
            #pragma unroll
            for (int h = 0; h < 4; ++h) {
                int a = 0;
                #pragma unroll
                for (int w = 0; w < 4; ++w) a = __dp4a((int)xr[4 * h + w], 0x01010101, a);
                xs[h] = a;
            }
        }
        const int st = j % KQ_NST;
        if (!mbar_wait(&full[st], (j / KQ_NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { *abort_flag = 1; break; }
        const uint32_t ub = ring_s + st * UB + sub * WROWS * RB;
        float v[WROWS];
        #pragma unroll
        for (int r = 0; r < WROWS; ++r) v[r] = kq_row_dot<FMT>(ub + r * RB + (FMT == FMT_Q2K ? boff : balign), bsh, q, xr, dx, xs);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        const int row0 = cu * UROWS + sub * WROWS;
        if constexpr (WROWS == 8) {
            const float sum = warp_reduce8(*reinterpret_cast<float(*)[8]>(v), lane);   // lane l: row l >> 2, 4 replicas
            if ((lane & 3) == 0 && yrow) yrow[row0 + (lane >> 2)] = wv * sum;
        } else {
            const float sum = warp_reduce4(*reinterpret_cast<float(*)[4]>(v), lane);   // lane l: row l >> 3, 8 replicas
            if ((lane & 7) == 0 && yrow) yrow[row0 + (lane >> 3)] = wv * sum;
        }
        if (*abort_flag) break;
    }
}

template <int FMT> void kq_launch(const ExpertParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_down1_kq<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kq_smem<FMT>()); attr = true; }
    launch_pdl(k_down1_kq<FMT>, dim3(grid), dim3(KQ_THREADS), kq_smem<FMT>(), st, p);
}

}  // namespace

void launch_down1_kq(const ExpertParams& p, int grid, cudaStream_t st) {
    if (p.down_fmt == FMT_Q2K) kq_launch<FMT_Q2K>(p, grid, st);
    else if (p.down_fmt == FMT_Q6K) kq_launch<FMT_Q6K>(p, grid, st);
    else kq_launch<FMT_Q3K>(p, grid, st);
}

}  // namespace lk
