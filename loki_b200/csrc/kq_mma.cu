// kq_mma.cu -- the K-quant (Q2_K / Q3_K) down projection for batches, on mma.sync: the real model's routed
// downs at T >= the mma threshold, after an IQ2_XXS gate/up phase that writes fp16 SwiGLU rows -- the
// register-fed one of slot_mma.cu, or from the GEMM threshold the tcgen05 one of prefill_gemm.cu.
//
// The single-token dp4a kernel (expert_kq.cu) decodes a down matrix once per (token, expert) entry; at T=512
// that makes the layer instruction-bound.  Here one warp owns 16 weight rows of one slot's expert (<= MM_NT =
// 16 tokens; the first two slots of an expert's run together, <= 32) and all of K = 2048: each 16-weight
// sub-block of its rows is decoded once -- scale and min folded in -- into an fp16 m16n8k16 A fragment and
// multiplied into every 8-token N tile.  B is the slot tokens' fp16
// SwiGLU rows (hb, written by the gate/up phase), C accumulates in fp32 registers.  The numerics are those of
// the IQ2_XXS tensor-core paths: h stays fp16 instead of being re-quantised to q8.
//
// K order: the k index of an mma step is free as long as A and B agree on it.  Lane (g, c) owns the sub-block
// half (n, sh) = (c >> 1, c & 1) of every 256-weight block -- weights 128n + 32j + 16sh + l, l < 16, j < 4 --
// whose 2-bit fields sit in qs bytes 32n + 16sh + l at bit pair j (Q3_K: plus hmask[16sh + l] bit 4n + j).  The
// 16-deep step (j, w) places weights l = 4w, 4w+1 of each lane's own sub-block at k slots 2c, 2c+1 and
// l = 4w+2, 4w+3 at 2c+8, 2c+9, so a lane's weights come from four consecutive qs bytes (one word) and its B
// fragments of two steps from eight consecutive h features (one 16-byte load); every weight of the block is still
// decoded exactly once per row.  A weight becomes fp16 as (1024 + q) by placing q under a 0x64 high byte, then
// fma((1024 + q), ds, -1024 ds) = q ds exactly rounded (1024 ds is exact), minus dmin * min (Q2_K) or 4 ds (Q3_K:
// the value is q3 - 4 with q3 = low2 | hbit << 2).
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

namespace {

constexpr int KM_WARPS = 8;
// resident blocks per SM the register budget is set for: Q2_K fits 64 registers without spills, Q3_K's extra
// hmask words need ~80
template <int FMT> constexpr int km_min_blocks() { return FMT == FMT_Q2K ? 3 : 2; }
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

// the lane's data of one row and 256-weight block: qs words q[w] (bytes l = 4w..4w+3 of its sub-block half),
// Q3_K's hmask words, the scale words covering sub-blocks 8n + 2j + sh (Q2_K: scales[8n..8n+7] as two words;
// Q3_K: the 12 packed scale bytes as three words), d and dmin
struct LaneBlk { uint32_t q[4], hm[4], sc[3]; float d, dmin; };
// four little-endian words from a 2-byte-aligned address by aligned loads: direct when p is 4-byte aligned,
// else funnel-shifted out of the five aligned words around the 16 bytes.  Every entry point takes 16-byte
// aligned arenas and strides, and a Q3_K row is 880 bytes, so only odd blocks sit at 2 mod 4; the word before
// their data lies in the previous block of the same row, and no load leaves the arena.  A warp's rows share
// their alignment, so the branch is uniform.
__device__ __forceinline__ void ldg_words4(const uint8_t* p, uint32_t (&o)[4]) {
    if (((uintptr_t)p & 3u) == 0) {
        #pragma unroll
        for (int w = 0; w < 4; ++w) o[w] = __ldg((const unsigned*)(p + 4 * w));
    } else {
        const unsigned* a = (const unsigned*)(p - 2);
        uint32_t v[5];
        #pragma unroll
        for (int i = 0; i < 5; ++i) v[i] = __ldg(a + i);
        #pragma unroll
        for (int w = 0; w < 4; ++w) o[w] = __funnelshift_r(v[w], v[w + 1], 16);
    }
}
template <int FMT>
__device__ __forceinline__ LaneBlk load_lane(const uint8_t* blk, int n, int sh) {
    LaneBlk r;
    if (FMT == FMT_Q2K) {                             // 84-byte blocks: 4-byte aligned
        const uint8_t* q = blk + Q2K_QS + 32 * n + 16 * sh;
        #pragma unroll
        for (int w = 0; w < 4; ++w) { r.q[w] = __ldg((const unsigned*)(q + 4 * w)); r.hm[w] = 0u; }
        r.sc[0] = __ldg((const unsigned*)(blk + 8 * n));
        r.sc[1] = __ldg((const unsigned*)(blk + 8 * n + 4));
        r.sc[2] = 0u;
        const uint32_t dd = __ldg((const unsigned*)(blk + Q2K_D));
        r.d = __half2float(__ushort_as_half((uint16_t)(dd & 0xFFFFu)));
        r.dmin = __half2float(__ushort_as_half((uint16_t)(dd >> 16)));
    } else {                                          // 110-byte blocks: 4-byte aligned for every other block
        ldg_words4(blk + Q3K_QS + 32 * n + 16 * sh, r.q);
        ldg_words4(blk + 16 * sh, r.hm);
        uint32_t dw;
        if (((uintptr_t)blk & 3u) == 0) {             // scale words at +96..+107, d at +108
            #pragma unroll
            for (int w = 0; w < 3; ++w) r.sc[w] = __ldg((const unsigned*)(blk + Q3K_SC + 4 * w));
            dw = ldg_u16(blk + Q3K_D);
        } else {                                      // aligned words at +94, +98, +102, +106 (d in the last one's high half)
            const unsigned* a = (const unsigned*)(blk + Q3K_SC - 2);
            uint32_t v[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __ldg(a + i);
            #pragma unroll
            for (int w = 0; w < 3; ++w) r.sc[w] = __funnelshift_r(v[w], v[w + 1], 16);
            dw = v[3] >> 16;
        }
        r.d = __half2float(__ushort_as_half((uint16_t)dw));
        r.dmin = 0.0f;
    }
    return r;
}

// the fp16x2 constants of the lane's sub-block 8n + 2j + sh in one row: scale ds, -1024 ds, and the offset
// subtracted after the fma (dmin * min for Q2_K, 4 ds for Q3_K)
struct SubScale { uint32_t ds2, c2, m2; };
template <int FMT>
__device__ __forceinline__ SubScale sub_scale(const LaneBlk& r, int n, int sh, int j) {
    const int bsh = 8 * (2 * (j & 1) + sh);          // byte (2j + sh) & 3 of word (2j + sh) >> 2 = j >> 1
    const uint32_t scw = (j & 2) ? r.sc[1] : r.sc[0];
    float ds, m;
    if (FMT == FMT_Q2K) {
        const uint32_t sc = (scw >> bsh) & 0xFFu;
        ds = r.d * (float)(sc & 15u);
        m = r.dmin * (float)(sc >> 4);
    } else {                                          // the kmask unpacking of moe_format.h q3k_scale, is = 8n + 2j + sh
        const uint32_t lob = (scw >> bsh) & 0xFFu;
        const int lo = n == 0 ? (int)(lob & 15u) : (int)(lob >> 4);
        const int hi = (int)((r.sc[2] >> (bsh + 2 * (2 * n + (j >> 1)))) & 3u);
        ds = r.d * (float)((lo | (hi << 4)) - 32);
        m = 4.0f * ds;
    }
    return SubScale{half2_bits(ds), half2_bits(-1024.0f * ds), half2_bits(m)};
}

// one row's two A-fragment words for step (j, w): weights l = 4w, 4w+1 (lo) and 4w+2, 4w+3 (hi) as fp16x2.  One
// shift and mask leave the four fields of qs word w in their bytes (Q3_K: the hmask bit ORed in as bit 2); a
// byte permute then puts each field under a 0x64 high byte, the fp16 (1024 + q).
template <int FMT>
__device__ __forceinline__ void lane_pair(const LaneBlk& r, const SubScale& s, int n, int j, int w, uint32_t& lo, uint32_t& hi) {
    uint32_t t = (r.q[w] >> (2 * j)) & 0x03030303u;
    if (FMT == FMT_Q3K) t |= ((r.hm[w] >> (4 * n + j)) & 0x01010101u) << 2;
    lo = hsub2(hfma2(__byte_perm(t, 0x64646464u, 0x4140u), s.ds2, s.c2), s.m2);
    hi = hsub2(hfma2(__byte_perm(t, 0x64646464u, 0x4342u), s.ds2, s.c2), s.m2);
}

// steps (j, 0..3) of one block: both rows' A fragments against the NT 8-token N tiles.  Token column g of
// tile nt is the fp16 h row at element offset hoff[nt] (negative: no token there, B = 0).  The A fragments of
// the two steps sharing a 16-byte h load are formed first, then h is loaded one tile pair at a time.
template <int FMT, int NT>
__device__ __forceinline__ void block_steps(const LaneBlk& ra, const LaneBlk& rbk, const __half* hb, const int (&hoff)[NT], int f, int n,
                                            int sh, int j, float (&acc)[NT][4]) {
    const SubScale sa = sub_scale<FMT>(ra, n, sh, j), sb = sub_scale<FMT>(rbk, n, sh, j);
    #pragma unroll
    for (int v = 0; v < 2; ++v) {
        uint32_t a[2][4];                             // step u: rows g (a[u][0], a[u][2]) and g+8 (a[u][1], a[u][3])
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
            lane_pair<FMT>(ra, sa, n, j, 2 * v + u, a[u][0], a[u][2]);
            lane_pair<FMT>(rbk, sb, n, j, 2 * v + u, a[u][1], a[u][3]);
        }
        #pragma unroll
        for (int tp = 0; tp < NT; tp += 2) {
            uint4 h[2];
            #pragma unroll
            for (int q = 0; q < 2; ++q)
                h[q] = hoff[tp + q] >= 0 ? __ldg((const uint4*)(hb + hoff[tp + q] + f + 32 * j + 8 * v)) : make_uint4(0u, 0u, 0u, 0u);
            #pragma unroll
            for (int u = 0; u < 2; ++u) {
                #pragma unroll
                for (int q = 0; q < 2; ++q)
                    mma16816_f16(acc[tp + q], a[u][0], a[u][1], a[u][2], a[u][3], u ? h[q].z : h[q].x, u ? h[q].w : h[q].y);
            }
        }
    }
}

// 16 rows (row block rb) of slot s's expert against NT 8-token N tiles: tiles 0, 1 hold slot s's tokens, tiles
// 2, 3 (NT = 4) slot s + 1's, so one decode of the rows serves both slots of the pair
template <int FMT, int NT>
__device__ __forceinline__ void item_rows(const MmaParams& p, const uint8_t* W, int s, const int (&cnt)[2], int rb, int g, int c) {
    constexpr int BLK = FMT == FMT_Q2K ? BLK_Q2K : BLK_Q3K;
    constexpr int ROWB = (MOE_INTER / QK) * BLK;
    const uint8_t* wa = W + (size_t)g * ROWB;
    const uint8_t* wb = W + (size_t)(g + 8) * ROWB;
    int hoff[NT];
    #pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int sl = s + (nt >> 1), tn = 8 * (nt & 1) + g;
        const int out = tn < cnt[nt >> 1] ? p.slot_out[sl * MM_NT + tn] : -1;
        hoff[nt] = out >= 0 ? out * MOE_INTER : -1;
    }
    float acc[NT][4];
    #pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
    const int n = c >> 1, sh = c & 1;
    for (int b = 0; b < MOE_INTER / QK; ++b) {
        const LaneBlk ra = load_lane<FMT>(wa + b * BLK, n, sh), rbk = load_lane<FMT>(wb + b * BLK, n, sh);
        const int f = b * QK + 128 * n + 16 * sh;    // h features of the lane's sub-block half, j = 0
        #pragma unroll 1
        for (int j = 0; j < 4; ++j) block_steps<FMT, NT>(ra, rbk, p.hb, hoff, f, n, sh, j, acc);
    }
    // C fragment: acc[nt][0..1] = row g, tokens 8(nt & 1) + 2c, +1 of slot s + (nt >> 1); acc[nt][2..3] = row g + 8
    #pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int sl = s + (nt >> 1);
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tn = 8 * (nt & 1) + 2 * c + (i & 1);
            if (tn >= cnt[nt >> 1]) continue;
            const int out = p.slot_out[sl * MM_NT + tn];
            if (out < 0) continue;
            const int row = rb * 16 + g + 8 * (i >> 1);
            p.y[(size_t)out * HIDDEN + row] = p.slot_w[sl * MM_NT + tn] * acc[nt][i];
        }
    }
}

__device__ __forceinline__ int slot_tokens(const MmaParams& p, int s) {
    if (p.slot_cnt) return p.slot_cnt[s];
    int cnt = 0;                                      // counted here when no pre-pass ran
    while (cnt < MM_NT && p.slot_tok[s * MM_NT + cnt] >= 0) ++cnt;
    return cnt;
}

// Items are (slot, row block).  An expert's slots are consecutive; the first slot of a run also takes the second
// (a decode of the rows feeds 4 N tiles), the second is then skipped, and later slots of a hot expert go alone.
template <int FMT>
__global__ void __launch_bounds__(KM_WARPS * 32, km_min_blocks<FMT>()) k_kq_mma_down(MmaParams p) {
    constexpr int BLK = FMT == FMT_Q2K ? BLK_Q2K : BLK_Q3K;
    constexpr int ROWB = (MOE_INTER / QK) * BLK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const int nslots = *p.nslots;
    const int nitems = nslots * KM_ITEMS_PER_SLOT;
    for (int item = blockIdx.x * KM_WARPS + warp; item < nitems; item += gridDim.x * KM_WARPS) {
        const int s = item / KM_ITEMS_PER_SLOT, rb = item % KM_ITEMS_PER_SLOT;
        const int e = p.slot_expert[s];
        const bool first = s == 0 || p.slot_expert[s - 1] != e;
        if (!first && (s == 1 || p.slot_expert[s - 2] != e)) continue;   // second of its run: done with the first
        const bool pair = first && s + 1 < nslots && p.slot_expert[s + 1] == e;
        const int cnt[2] = { slot_tokens(p, s), pair ? slot_tokens(p, s + 1) : 0 };
        if (cnt[0] <= 0 && cnt[1] <= 0) continue;
        const uint8_t* W = (e == SHARED_SLOT ? p.sh_down : p.down + (size_t)e * p.down_stride) + (size_t)rb * 16 * ROWB;
        if (pair) item_rows<FMT, 4>(p, W, s, cnt, rb, g, c);
        else item_rows<FMT, 2>(p, W, s, cnt, rb, g, c);
    }
}

}  // namespace

// one wave of resident blocks: items are grid-strided, so blocks beyond the resident ones would only form a tail
template <int FMT>
static void launch_fmt(const MmaParams& p, int nsm, cudaStream_t st) {
    static int per_sm = 0;
    if (per_sm <= 0 && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_kq_mma_down<FMT>, KM_WARPS * 32, 0) != cudaSuccess || per_sm <= 0))
        per_sm = km_min_blocks<FMT>();
    k_kq_mma_down<FMT><<<per_sm * nsm, KM_WARPS * 32, 0, st>>>(p);
}

void launch_kq_mma_down(const MmaParams& p, int down_fmt, int nsm, cudaStream_t st) {
    if (down_fmt == FMT_Q2K) launch_fmt<FMT_Q2K>(p, nsm, st);
    else launch_fmt<FMT_Q3K>(p, nsm, st);
}

}  // namespace lk
