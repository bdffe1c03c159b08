// kq_mma.cu -- the K-quant (Q2_K / Q3_K) down projection for batches, on mma.sync: the real model's routed
// downs at T >= the mma threshold, after an IQ2_XXS gate/up phase that writes fp16 SwiGLU rows -- the
// register-fed one of slot_mma.cu, or from the GEMM threshold the tcgen05 one of prefill_gemm.cu.
//
// The single-token dp4a kernel (expert_kq.cu) decodes a down matrix once per (token, expert) entry; at T=512
// that makes the layer instruction-bound.  Here one warp owns 16 weight rows of one slot's expert (<= MM_NT =
// 16 tokens) and all of K = 2048: each 16-weight sub-block of its rows is decoded once -- scale and min folded
// in -- into an fp16 m16n8k16 A fragment and multiplied into both 8-token N tiles.  B is the slot tokens' fp16
// SwiGLU rows (hb, written by the gate/up phase), C accumulates in fp32 registers.  The numerics are those of
// the IQ2_XXS tensor-core paths: h stays fp16 instead of being re-quantised to q8.
//
// K order: a 16-deep mma step is one sub-block (n, j, s) of a 256-weight block -- weights 128n + 32j + 16s + l,
// l < 16 -- whose 2-bit fields sit in qs bytes 32n + 16s + l at bit pair j (Q3_K: plus hmask[16s + l] bit
// 4n + j).  Lane (g, c) needs l in {2c, 2c+1} and {2c+8, 2c+9} of rows g and g+8: two 16-bit words per row,
// shared by the four j of one (n, s); the B fragment reads the same feature indices of h.  A weight becomes
// fp16 as (1024 + q) by OR-ing q into 0x6400, then fma((1024 + q), ds, -1024 ds) = q ds exactly rounded (1024 ds
// is exact), minus dmin * min (Q2_K) or 4 ds (Q3_K: the value is q3 - 4 with q3 = low2 | hbit << 2).
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

namespace {

constexpr int KM_WARPS = 8;
constexpr int KM_ITEMS_PER_SLOT = HIDDEN / 16;         // 448 row blocks of 16

__device__ __forceinline__ void mma16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3]) : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d; asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d; asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b)); return d;
}
__device__ __forceinline__ uint32_t half2_bits(float v) {
    const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
}
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) { return (uint32_t)__ldg((const unsigned short*)p); }
__device__ __forceinline__ uint32_t ldg_u8(const uint8_t* p) { return (uint32_t)__ldg(p); }

// two fp16 (1024 + q) from the fields of a 16-bit word: q0 in bits 0..w-1 of t, q1 in bits 8..8+w-1
__device__ __forceinline__ uint32_t pair_1024(uint32_t t, uint32_t mask) {
    return 0x64006400u | (t & mask) | ((t >> 8) & mask) << 16;
}

// one row's per-block constants, loaded once per 256-weight block: d (and dmin), and the scale bytes -- Q2_K:
// scales[0..15] as four words; Q3_K: the 12 packed scale bytes as three words
struct RowBlk { float d, dmin; uint32_t sc[4]; };
template <int FMT>
__device__ __forceinline__ RowBlk load_rowblk(const uint8_t* blk) {
    RowBlk r;
    if (FMT == FMT_Q2K) {                             // 84-byte blocks: 4-byte aligned
        const uint32_t dd = __ldg((const unsigned*)(blk + Q2K_D));
        r.d = __half2float(__ushort_as_half((uint16_t)(dd & 0xFFFFu)));
        r.dmin = __half2float(__ushort_as_half((uint16_t)(dd >> 16)));
        #pragma unroll
        for (int w = 0; w < 4; ++w) r.sc[w] = __ldg((const unsigned*)(blk + 4 * w));
    } else {                                          // 110-byte blocks: 2-byte aligned
        r.d = __half2float(__ushort_as_half((uint16_t)ldg_u16(blk + Q3K_D)));
        r.dmin = 0.0f;
        #pragma unroll
        for (int w = 0; w < 3; ++w) r.sc[w] = ldg_u16(blk + Q3K_SC + 4 * w) | (ldg_u16(blk + Q3K_SC + 4 * w + 2) << 16);
        r.sc[3] = 0u;
    }
    return r;
}

// one row's A-fragment halves for sub-block (n, j, s): words w0 (l = 2c, 2c+1) and w1 (l = 2c+8, 2c+9) of qs
// (and hm0/hm1 of hmask for Q3_K) -> two fp16x2 of the weights
template <int FMT>
__device__ __forceinline__ void row_pair(const RowBlk& rb, uint32_t w0, uint32_t w1, uint32_t hm0, uint32_t hm1, int n, int j, int s,
                                         uint32_t& o0, uint32_t& o1) {
    const int is = 8 * n + 2 * j + s;
    if (FMT == FMT_Q2K) {
        const uint32_t sc = (rb.sc[is >> 2] >> (8 * (is & 3))) & 0xFFu;
        const float ds = rb.d * (float)(sc & 15u);
        const uint32_t ds2 = half2_bits(ds), c2 = half2_bits(-1024.0f * ds), dm2 = half2_bits(rb.dmin * (float)(sc >> 4));
        o0 = hsub2(hfma2(pair_1024(w0 >> (2 * j), 3u), ds2, c2), dm2);
        o1 = hsub2(hfma2(pair_1024(w1 >> (2 * j), 3u), ds2, c2), dm2);
    } else {                                          // Q3_K: the kmask unpacking of moe_format.h q3k_scale
        const uint32_t lob = (rb.sc[(is & 7) >> 2] >> (8 * (is & 3))) & 0xFFu;
        const int lo = is < 8 ? (int)(lob & 15u) : (int)(lob >> 4);
        const int hi = (int)((rb.sc[2] >> (8 * (is & 3) + 2 * (is >> 2))) & 3u);
        const float ds = rb.d * (float)((lo | (hi << 4)) - 32);
        const uint32_t ds2 = half2_bits(ds), c2 = half2_bits(-1024.0f * ds), f2 = half2_bits(4.0f * ds);
        const int hb = 4 * n + j;
        const uint32_t t0 = ((w0 >> (2 * j)) & 0x0303u) | (((hm0 >> hb) & 0x0101u) << 2);
        const uint32_t t1 = ((w1 >> (2 * j)) & 0x0303u) | (((hm1 >> hb) & 0x0101u) << 2);
        o0 = hsub2(hfma2(pair_1024(t0, 7u), ds2, c2), f2);
        o1 = hsub2(hfma2(pair_1024(t1, 7u), ds2, c2), f2);
    }
}

template <int FMT>
__global__ void __launch_bounds__(KM_WARPS * 32) k_kq_mma_down(MmaParams p) {
    constexpr int BLK = FMT == FMT_Q2K ? BLK_Q2K : BLK_Q3K;
    constexpr int QS = FMT == FMT_Q2K ? Q2K_QS : Q3K_QS;
    constexpr int ROWB = (MOE_INTER / QK) * BLK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int nitems = *p.nslots * KM_ITEMS_PER_SLOT;
    for (int item = blockIdx.x * KM_WARPS + warp; item < nitems; item += gridDim.x * KM_WARPS) {
        const int s = item / KM_ITEMS_PER_SLOT, rb = item % KM_ITEMS_PER_SLOT;
        int cnt = 0;                                  // the slot's tokens (counted here when no pre-pass ran)
        if (p.slot_cnt) cnt = p.slot_cnt[s];
        else while (cnt < MM_NT && p.slot_tok[s * MM_NT + cnt] >= 0) ++cnt;
        if (cnt <= 0) continue;
        const int e = p.slot_expert[s];
        const uint8_t* W = (e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride) + (size_t)rb * 16 * ROWB;
        const uint8_t* wa = W + (size_t)g * ROWB;
        const uint8_t* wb = W + (size_t)(g + 8) * ROWB;
        const __half* hrow[2];
        #pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            const int tn = 8 * nt + g;
            const int out = tn < cnt ? p.slot_out[s * MM_NT + tn] : -1;
            hrow[nt] = out >= 0 ? p.hb + (size_t)out * MOE_INTER : nullptr;
        }
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        for (int b = 0; b < MOE_INTER / QK; ++b) {
            const uint8_t* ba = wa + b * BLK;
            const uint8_t* bb = wb + b * BLK;
            const RowBlk ra = load_rowblk<FMT>(ba), rbk = load_rowblk<FMT>(bb);
            #pragma unroll
            for (int n = 0; n < 2; ++n) {
                #pragma unroll
                for (int sh = 0; sh < 2; ++sh) {
                    const int q0 = QS + 32 * n + 16 * sh + 2 * c;
                    const uint32_t wa0 = ldg_u16(ba + q0), wa1 = ldg_u16(ba + q0 + 8), wb0 = ldg_u16(bb + q0), wb1 = ldg_u16(bb + q0 + 8);
                    uint32_t ha0 = 0, ha1 = 0, hb0 = 0, hb1 = 0;
                    if (FMT == FMT_Q3K) {
                        const int m0 = 16 * sh + 2 * c;
                        ha0 = ldg_u16(ba + m0); ha1 = ldg_u16(ba + m0 + 8); hb0 = ldg_u16(bb + m0); hb1 = ldg_u16(bb + m0 + 8);
                    }
                    #pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t a0, a2, a1, a3;                   // rows g (a0, a2) and g+8 (a1, a3); l = 2c.. and 2c+8..
                        row_pair<FMT>(ra, wa0, wa1, ha0, ha1, n, j, sh, a0, a2);
                        row_pair<FMT>(rbk, wb0, wb1, hb0, hb1, n, j, sh, a1, a3);
                        const int k0 = b * QK + 128 * n + 32 * j + 16 * sh + 2 * c;
                        #pragma unroll
                        for (int nt = 0; nt < 2; ++nt) {
                            const uint32_t b0 = hrow[nt] ? __ldg((const unsigned*)(hrow[nt] + k0)) : 0u;
                            const uint32_t b1 = hrow[nt] ? __ldg((const unsigned*)(hrow[nt] + k0 + 8)) : 0u;
                            mma16816_f16(acc[nt], a0, a1, a2, a3, b0, b1);
                        }
                    }
                }
            }
        }
        // C fragment: acc[nt][0..1] = row g, tokens 8nt + 2c, +1; acc[nt][2..3] = row g + 8
        #pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int tn = 8 * nt + 2 * c + (i & 1);
                if (tn >= cnt) continue;
                const int out = p.slot_out[s * MM_NT + tn];
                if (out < 0) continue;
                const int row = rb * 16 + g + 8 * (i >> 1);
                p.y[(size_t)out * HIDDEN + row] = p.slot_w[s * MM_NT + tn] * acc[nt][i];
            }
        }
    }
}

}  // namespace

void launch_kq_mma_down(const MmaParams& p, int down_fmt, int nsm, cudaStream_t st) {
    const int grid = 4 * nsm;
    if (down_fmt == FMT_Q2K) k_kq_mma_down<FMT_Q2K><<<grid, KM_WARPS * 32, 0, st>>>(p);
    else k_kq_mma_down<FMT_Q3K><<<grid, KM_WARPS * 32, 0, st>>>(p);
}

}  // namespace lk
