// shared_kq.cu -- the real DeepSeek-R1 IQ2_XXS model's shared expert: Q5_K gate/up and a Q6_K down (the
// reference's mvg(F_Q5K, sh_gate / sh_up) + swiglu_q8 + mvg(F_Q6K, sh_down), src/fused_layer.cu:521-524, with
// tc_matvec's Q5_K and Q6_K arithmetic, :102-158).
//
// gate/up (k_sh_gate_up_q5k): the CTA shape of the IQ2_XXS single-token kernel -- 4 consumer streams of 224
// threads, one 32-weight K sub-block each, plus a producer warp that streams weight rows into an 8-stage ring
// with cp.async.bulk.  A tile is 32 rows of ONE matrix (gate or up) for one token, so a single token still
// has 128 tiles for the 148 SMs: 8 chunks of 4 rows (19 712 B each), chunk c in stage c.  Stream k takes
// chunks k and k + 4 (rows 4k..4k+3 and 16+4k..16+4k+3).  Per sub-block (block b = g / 8, sub-block
// s = g % 8 of the thread's K group g):
//   q = ((qs[32(s/2) + l] >> 4(s%2)) & 15) | (qh[l] bit s) << 4 (0..31), isum = sum q * q_x (dp4a),
//   v = dx * (d*scale*isum - dmin*min*sum q_x)
// -- the reference's per-32 integer arithmetic.  A block's header (d, dmin, 12 scale bytes), its 32 qh bytes
// and the thread's 32 qs bytes are five 16-byte shared loads (Q5_K blocks are 176 B: 16-byte aligned).  The
// tile's row sums (7 warps per row, fixed order) go to `gu` as fp32 [token][gate 2048 | up 2048].  The gate
// and up tiles of the same rows run on different CTAs: a per-(token, row tile) counter (fence, then atomic
// add) tells the CTA that finishes second, which forms SwiGLU and the q8 of those 32 h values (one q8 group,
// the reference's swiglu_q8) from its own sums and the partner's, and resets the counter.
// down: k_down1_kq<FMT_Q6K> (expert_kq.cu) in its shared-only mode, reading those q8 rows.
//
// Many tokens: shared_gemm.cu (the same expert as two dense tcgen05 GEMMs on fp16-dequantised weights).
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

namespace {

constexpr int S5_NS = 4;                             // consumer streams
constexpr int S5_KG = HIDDEN / 32;                   // 224 consumers per stream (one 32-weight sub-block each)
constexpr int S5_SW = S5_KG / 32;                    // 7 warps per stream
constexpr int S5_CONS = S5_NS * S5_KG;               // 896
constexpr int S5_THREADS = S5_CONS + 32;             // + producer warp
constexpr int S5_ROWB = (HIDDEN / QK) * BLK_Q5K;     // 4928
constexpr int S5_CROWS = 4;
constexpr int S5_CBYTES = S5_CROWS * S5_ROWB;        // 19712
constexpr int S5_TILE = 32;                          // rows per tile
constexpr int S5_CPT = S5_TILE / S5_CROWS;           // 8 chunks per tile; chunk c always uses stage c
constexpr int S5_TILES_PER_MAT = MOE_INTER / S5_TILE;     // 64
static_assert(S5_CPT == 2 * S5_NS, "each stream takes two chunks per tile");
static_assert(S5_ROWB % 16 == 0 && S5_CBYTES % 16 == 0, "bulk copies need 16-byte rows");

constexpr int S5_OFF_RING = 0;
constexpr int S5_OFF_RED = S5_OFF_RING + S5_CPT * S5_CBYTES;
constexpr int S5_OFF_BAR = S5_OFF_RED + 2 * S5_NS * S5_SW * 32 * 4;
constexpr int S5_OFF_ABORT = S5_OFF_BAR + 2 * S5_CPT * 8;
constexpr int S5_SMEM = S5_OFF_ABORT + 16;
static_assert(S5_SMEM <= 232448, "Q5_K gate/up shared-memory layout exceeds the 227 KB a CTA can have");

__device__ __forceinline__ uint4 lds_v4(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// q8 of the 32-wide group g of an fp32 row (global): 8 packed words, returns the scale
__device__ __forceinline__ float q8_group_row(const float* row, int g, uint32_t (&xr)[8]) {
    float xv[32];
    const float4* src = (const float4*)(row + g * 32);
    #pragma unroll
    for (int j = 0; j < 8; ++j) { const float4 v = src[j]; xv[4*j] = v.x; xv[4*j+1] = v.y; xv[4*j+2] = v.z; xv[4*j+3] = v.w; }
    int8_t q[32];
    const float d = quant_q8_group(xv, q);
    #pragma unroll
    for (int j = 0; j < 8; ++j)
        xr[j] = (uint32_t)(uint8_t)q[4*j] | ((uint32_t)(uint8_t)q[4*j+1] << 8) |
                ((uint32_t)(uint8_t)q[4*j+2] << 16) | ((uint32_t)(uint8_t)q[4*j+3] << 24);
    return d;
}

// one row's sub-block s (0..7) of the block at shared address bb: the partial dot product with this thread's
// 32 q8 activations (xr, their sum xs, scale dx).  Per 4 weights: the qs nibbles shifted down, qh bit s
// rotated into bit 4 of each byte (one funnel shift), the two merged by one LOP3; then dp4a.
__device__ __forceinline__ float q5k_dot(uint32_t bb, int s, const uint32_t (&xr)[8], int xs, float dx) {
    const uint4 hdr = lds_v4(bb);                    // d | dmin, scales[0..3], scales[4..7], scales[8..11]
    const uint4 h0 = lds_v4(bb + Q5K_QH), h1 = lds_v4(bb + Q5K_QH + 16);
    const uint32_t qo = bb + Q5K_QS + 32 * (s >> 1);
    const uint4 q0 = lds_v4(qo), q1 = lds_v4(qo + 16);
    const uint32_t qs[8] = { q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w };
    const uint32_t qh[8] = { h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w };
    const uint32_t nsh = 4u * (uint32_t)(s & 1), rot = (uint32_t)(4 - s) & 31u;
    int isum = 0;
    #pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t hi = __funnelshift_l(qh[w], qh[w], rot) & 0x10101010u;
        const uint32_t q5 = ((qs[w] >> nsh) & 0x0F0F0F0Fu) | hi;
        isum = __dp4a((int)q5, (int)xr[w], isum);
    }
    const uint32_t selk = 0x4440u | (uint32_t)(s & 3);     // byte s & 3 of a word, zero-extended
    const uint32_t A = __byte_perm(hdr.y, 0u, selk), B = __byte_perm(hdr.z, 0u, selk), C = __byte_perm(hdr.w, 0u, selk);
    const uint32_t sc = s < 4 ? (A & 63u) : ((C & 15u) | ((A >> 2) & 48u));
    const uint32_t mn = s < 4 ? (B & 63u) : ((C >> 4) | ((B >> 2) & 48u));
    const float2 dd = __half22float2(*reinterpret_cast<const __half2*>(&hdr.x));   // (d, dmin)
    return dx * fmaf(dd.x * (float)sc, (float)isum, -(dd.y * (float)mn) * (float)xs);
}

__global__ void __launch_bounds__(S5_THREADS, 1) k_sh_gate_up_q5k(SharedKqParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem + S5_OFF_RING;
    float* red = (float*)(smem + S5_OFF_RED);
    uint64_t* full = (uint64_t*)(smem + S5_OFF_BAR);
    uint64_t* empty = full + S5_CPT;
    volatile int* abort_flag = (volatile int*)(smem + S5_OFF_ABORT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        *abort_flag = 0;
        for (int c = 0; c < S5_CPT; ++c) { mbar_init(&full[c], 1); mbar_init(&empty[c], S5_SW); }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    const int ntiles = p.n * 2 * S5_TILES_PER_MAT;   // tile = (token j, matrix m, row tile rt), token-major
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x);
    const int t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    if (t0 >= t1) return;

    if (warp == S5_CONS / 32) {                       // ---------------- producer
        if (lane == 0) {
            uint32_t it = 0;                          // copies issued; copy it uses stage it % 8, phase it / 8
            for (int tile = t0; tile < t1; ++tile) {
                const int m = (tile / S5_TILES_PER_MAT) & 1, rt = tile % S5_TILES_PER_MAT;
                const uint8_t* mat = m ? p.up : p.gate;
                for (int c = 0; c < S5_CPT; ++c, ++it) {
                    if (*abort_flag || !mbar_wait(&empty[c], ((it / S5_CPT) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; goto drain; }
                    const uint8_t* src = mat + (size_t)(rt * S5_TILE + c * S5_CROWS) * S5_ROWB;
                    mbar_arrive_expect_tx(&full[c], S5_CBYTES);
                    bulk_g2s(ring + c * S5_CBYTES, src, S5_CBYTES, &full[c]);
                }
            }
        drain:
            {   // every issued copy must land before the CTA may exit
                const uint32_t first = it > S5_CPT ? it - S5_CPT : 0;
                for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S5_CPT], (j / S5_CPT) & 1, nullptr, 0);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int strm = tid / S5_KG, g = tid % S5_KG, sw = g >> 5;
    const int s = g & 7;
    const uint32_t boff = (uint32_t)(BLK_Q5K * (g >> 3));
    const uint32_t ring_s = smem_u32(ring);
    uint32_t xr[8];
    float dx = 0.0f;
    int xs = 0, xtok = -1;
    bool aborted = false;
    uint32_t ti = 0;
    for (int tile = t0; tile < t1; ++tile, ++ti) {
        const int jm = tile / S5_TILES_PER_MAT, rt = tile % S5_TILES_PER_MAT;
        const int tok = p.t0 + (jm >> 1);
        if (tok != xtok) {
            if (tok == 0 && p.xq) {                  // quantised by the router (one-token forward)
                const uint4 a0 = ((const uint4*)(p.xq + g * 32))[0], a1 = ((const uint4*)(p.xq + g * 32))[1];
                xr[0] = a0.x; xr[1] = a0.y; xr[2] = a0.z; xr[3] = a0.w; xr[4] = a1.x; xr[5] = a1.y; xr[6] = a1.z; xr[7] = a1.w;
                dx = p.xd[g];
            } else {
                dx = q8_group_row(p.x + (size_t)tok * p.ld_x, g, xr);
            }
            xs = 0;
            #pragma unroll
            for (int w = 0; w < 8; ++w) xs = __dp4a((int)xr[w], 0x01010101, xs);
            xtok = tok;
        }
        float kept = 0.0f;
        #pragma unroll
        for (int ch = 0; ch < 2; ++ch) {              // rows 4k.. and 16+4k..
            const int c = strm + S5_NS * ch;
            if (!aborted && !mbar_wait(&full[c], ti & 1, p.err, DEV_ERR_TIMEOUT_FULL)) { aborted = true; *abort_flag = 1; }
            const uint32_t base = ring_s + c * S5_CBYTES + boff;
            float v[4];
            #pragma unroll
            for (int rr = 0; rr < S5_CROWS; ++rr) v[rr] = aborted ? 0.0f : q5k_dot(base + rr * S5_ROWB, s, xr, xs, dx);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[c]);
            const float r = warp_reduce4(v, lane);    // lane l: row l >> 3 of the chunk
            if ((lane & 7) == ch) kept = r;
        }
        float* rb = red + (ti & 1) * (S5_NS * S5_SW * 32);
        rb[(strm * S5_SW + sw) * 32 + lane] = kept;
        if (named_bar_or(1, S5_CONS, aborted)) break;   // uniform: every consumer leaves here together
        if (warp == 0) {                              // row `lane` of the tile: stream (lane & 15) / 4, chunk lane / 16
            const int k = (lane & 15) >> 2, rr = lane & 3, hi = lane >> 4;
            const float* q = rb + k * S5_SW * 32 + rr * 8 + hi;
            float acc = q[0];
            #pragma unroll
            for (int w = 1; w < S5_SW; ++w) acc += q[w * 32];
            p.gu[(size_t)jm * MOE_INTER + rt * S5_TILE + lane] = acc;
            __threadfence();                          // this half visible before the count
            __syncwarp();
            const int j = jm >> 1;
            int* cnt = p.pair + (size_t)j * S5_TILES_PER_MAT + rt;
            int old = 0;
            if (lane == 0) old = atomicAdd(cnt, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == 1) {                           // the partner's half is done: SwiGLU + q8 of these 32 rows
                __threadfence();
                const float other = __ldcg(p.gu + (size_t)(jm ^ 1) * MOE_INTER + rt * S5_TILE + lane);
                const float hv = (jm & 1) ? lk_swiglu(other, acc) : lk_swiglu(acc, other);
                float amax = fabsf(hv);
                #pragma unroll
                for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
                const size_t out = (size_t)(p.row0 + j);
                p.hq[out * MOE_INTER + rt * S5_TILE + lane] = (int8_t)(int)rintf(hv * id);
                if (lane == 0) { p.hd[out * (MOE_INTER / 32) + rt] = d; *cnt = 0; }
            }
        }
    }
}

}  // namespace

void launch_shared_kq(const SharedKqParams& p, int grid, cudaStream_t st) {
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_sh_gate_up_q5k, cudaFuncAttributeMaxDynamicSharedMemorySize, S5_SMEM); attr = true; }
    if (p.n <= 0) return;
    const int tiles = p.n * 2 * S5_TILES_PER_MAT;
    launch_pdl(k_sh_gate_up_q5k, dim3(grid < tiles ? grid : tiles), dim3(S5_THREADS), S5_SMEM, st, p);
    ExpertParams e{};                                 // the down: k_down1_kq<Q6_K>, shared-only slots
    e.sh_down = p.down; e.hq = p.hq; e.hd = p.hd; e.y = p.y; e.err = p.err; e.down_fmt = FMT_Q6K;
    e.slot_expert = nullptr; e.sh_count = p.n; e.sh_row0 = p.row0;
    launch_down1_kq(e, grid, st);
}

}  // namespace lk
