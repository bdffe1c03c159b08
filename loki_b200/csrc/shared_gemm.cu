// shared_gemm.cu -- the real model's shared expert (Q5_K gate/up, Q6_K down) for many tokens: two dense GEMMs
// on tcgen05 (kind::f16, fp32 accumulators in tensor memory).  The per-token kernels of shared_kq.cu re-stream
// the 32 MB of weights once per token; from a few tokens on it pays to dequantise the three matrices once per
// call and run them as GEMMs.  The reference runs the same expert as tc_matvec, one token at a time, on the
// q8 of x and the q8 of the SwiGLU output (src/fused_layer.cu:40-47, 102-158, 334-341, 521-524).
//
// Numerics.  The q8 of h is a rounding step: a gate/up value a few 1e-4 off moves some h codes by one, and
// that alone puts a plain fp16 GEMM ~2.5e-3 (relative L2) from the reference's integer arithmetic.  So the
// gate/up operands are split: x's q8 value q*d (fp32) = hi + lo with hi = fp16(q*d), lo = fp16(q*d - hi), and
// each dequantised weight w (fp32, gguf-py arithmetic) = whi + wlo the same way.  The accumulator gets
// whi*xhi + wlo*xhi + whi*xlo (the dropped wlo*xlo is ~2^-22 relative): fp32 accuracy, like the reference's
// sums.  The down then needs no split: its input is the q8 of h (fp16(q*d), error <= 2^-12 per value) and
// nothing is rounded after it.
//
// Every operand is written by this file's own kernels straight into the UMMA canonical K-major layout
// (no swizzle: 8-row x 16-byte core matrices), tiled so that one (row tile, K block) is one contiguous run of
// bytes that a single 1-D bulk copy (cp.async.bulk) stages.  Element (r, k) of a tile of R rows sits at
// (k/8)*(R/8)*128 + (r/8)*128 + (r%8)*16 + (k%8)*2 bytes: LBO = R/8*128 between K core columns, SBO = 128
// between 8-row groups.
//   gate, up  [row tile of 128][K block of 32][whi tile 8 KB | wlo tile 8 KB]       (k_sh_w16, 16 x 224 blocks)
//   down      [row tile of 128][K block of 64][16 KB]                               (k_sh_w16, 56 x 32 blocks)
//   x         [token tile of NT][K block of 32][2NT rows: xhi rows, then xlo rows]  (k_sh_x16)
//   h         [token tile of NT][K block of 64][NT rows]                            (the gate/up epilogue)
//
// k_sh_gemm<GU, NT>: one CTA per (128-row tile, NT-token tile).  Warp 0 lane 0 streams the K blocks through
// a ring of stages with bulk copies; warp 1 issues the MMAs (whole warp, elect.sync) and commits each stage
// back to the producer; warps 2-5 (one TMEM lane quarter = 32 rows each) run the epilogue.
//   GU: per K step and per matrix (gate, up) two MMAs: whi x [xhi; xlo] (N = 2NT) into columns [0, 2NT) of
//       the matrix's accumulator, and wlo x xhi (N = NT) into columns [0, NT).  Epilogue: g = D[c] + D[NT+c],
//       likewise u, h = SwiGLU(g, u) in fp32, its q8 per 32 (quant_q8_group's arithmetic: a warp's 32 lanes
//       are one group of h indices) as fp16(q*d) into the h tiles.
//   down: y[row0 + n][row] = the accumulator.
// Every wait is bounded (2 s): on a timeout the error word is set, the producer drains the copies it issued,
// the MMA warp drains its MMAs, and the CTA exits.
#include "moe_internal.h"
#include "moe_device.cuh"
#include "tcgen05.cuh"

namespace lk {

constexpr int SG_M = 128;                            // rows per tile (MMA M)
constexpr int SG_THREADS = 192;                      // producer, MMA, 4 epilogue warps
constexpr int SG_GU_KB = 32, SG_DN_KB = 64;          // K per block
constexpr int SG_GU_KBN = HIDDEN / SG_GU_KB;         // 224
constexpr int SG_DN_KBN = MOE_INTER / SG_DN_KB;      // 32
constexpr int SG_GU_W = 2 * SG_M * SG_GU_KB * 2;     // whi + wlo tiles of one (row tile, K block): 16 KB
constexpr int SG_DN_W = SG_M * SG_DN_KB * 2;         // 16 KB
constexpr int SG_GU_TILES = MOE_INTER / SG_M;        // 16 row tiles of gate (and of up)
constexpr int SG_DN_TILES = HIDDEN / SG_M;           // 56 row tiles of down
constexpr size_t SG_GU_MAT = (size_t)SG_GU_TILES * SG_GU_KBN * SG_GU_W;   // bytes of gate (or up) in w16

__host__ __device__ constexpr int sg_kb(bool gu) { return gu ? SG_GU_KB : SG_DN_KB; }
__host__ __device__ constexpr int sg_a_bytes(bool gu) { return gu ? 2 * SG_GU_W : SG_DN_W; }
__host__ __device__ constexpr int sg_b_bytes(bool gu, int nt) { return gu ? 2 * nt * SG_GU_KB * 2 : nt * SG_DN_KB * 2; }
__host__ __device__ constexpr int sg_stage_bytes(bool gu, int nt) { return sg_a_bytes(gu) + sg_b_bytes(gu, nt); }
__host__ __device__ constexpr int sg_nst(bool gu, int nt) { return 200 * 1024 / sg_stage_bytes(gu, nt); }
__host__ __device__ constexpr int sg_smem(bool gu, int nt) { return sg_nst(gu, nt) * sg_stage_bytes(gu, nt) + 1024; }
__host__ __device__ constexpr int sg_tmem_cols(bool gu, int nt) { return gu ? 4 * nt : (nt < 32 ? 32 : nt); }

__device__ __forceinline__ uint32_t sg_off(int r, int k, int rows) {   // byte offset of (r, k) in a tile
    return (uint32_t)((k >> 3) * (rows >> 3) * 128 + (r >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// D[tmem] (+)= A[smem] x B[smem]^T, one 16-deep K step, issued by one elected lane of a converged warp
__device__ __forceinline__ void umma_f16_ss_warp(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void split_f16(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// ---------------------------------------------------------------- operand writers
// weights: one thread per 8 consecutive weights of a row, FMT = Q5_K (gate/up: whi and wlo tiles, 32-deep K
// blocks) or Q6_K (down: one fp16 tile, 64-deep K blocks); rows x K
template <int FMT>
__global__ void __launch_bounds__(256) k_sh_w16(const uint8_t* __restrict__ W, int rows, int K, uint8_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int per_row = K / 8;
    if (i >= (int64_t)rows * per_row) return;
    const int r = (int)(i / per_row), k0 = 8 * (int)(i % per_row);
    const uint8_t* blk = W + ((size_t)r * (K / QK) + k0 / QK) * fmt_block_bytes(FMT);
    const int w0 = k0 % QK;
    float v[8];
    if (FMT == FMT_Q5K) {
        const int j = w0 >> 6, u = (w0 >> 5) & 1, l0 = w0 & 31;
        int sc, mn;
        q5k_scale_min(blk + Q5K_SC, 2 * j + u, sc, mn);
        const float d = __half2float(__ushort_as_half((uint16_t)(blk[0] | (blk[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((uint16_t)(blk[2] | (blk[3] << 8))));
        const float dl = d * (float)sc, ml = dmin * (float)mn;
        #pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = ((blk[Q5K_QS + 32 * j + l0 + k] >> (4 * u)) & 15) | (((blk[Q5K_QH + l0 + k] >> (2 * j + u)) & 1) << 4);
            v[k] = dl * (float)q - ml;
        }
        __align__(16) __half hi[8];
        __align__(16) __half lo[8];
        #pragma unroll
        for (int k = 0; k < 8; ++k) split_f16(v[k], hi[k], lo[k]);
        uint8_t* tile = out + ((size_t)(r / SG_M) * (K / SG_GU_KB) + k0 / SG_GU_KB) * SG_GU_W;
        const uint32_t o = sg_off(r % SG_M, k0 % SG_GU_KB, SG_M);
        *(uint4*)(tile + o) = *(const uint4*)hi;
        *(uint4*)(tile + SG_GU_W / 2 + o) = *(const uint4*)lo;
    } else {                                          // Q6_K
        const int n = w0 >> 7, c = (w0 >> 5) & 3, l0 = w0 & 31;
        const float d = __half2float(__ushort_as_half((uint16_t)(blk[Q6K_D] | (blk[Q6K_D + 1] << 8))));
        const float dl = d * (float)(int8_t)blk[Q6K_SC + w0 / 16];
        #pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = ((blk[64 * n + 32 * (c & 1) + l0 + k] >> (4 * (c >> 1))) & 15) | (((blk[Q6K_QH + 32 * n + l0 + k] >> (2 * c)) & 3) << 4);
            v[k] = dl * (float)(q - 32);
        }
        __half2 h[4];
        #pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        uint8_t* tile = out + ((size_t)(r / SG_M) * (K / SG_DN_KB) + k0 / SG_DN_KB) * SG_DN_W;
        *(uint4*)(tile + sg_off(r % SG_M, k0 % SG_DN_KB, SG_M)) = *(const uint4*)h;
    }
}

// x rows [t0, t0 + n) (fp32, row stride ld) -> the gate/up B tiles of nt-token tiles: the q8 of x
// (quant_q8_group per 32) as q*d split into xhi / xlo rows, one thread per 32-wide group; rows n..n_pad-1 zero
// (the MMA columns of padding tokens are never read back, so h keeps whatever its padding rows held)
__global__ void __launch_bounds__(256) k_sh_x16(const float* __restrict__ x, int ld, int t0, int n, int n_pad, int nt,
                                                uint8_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    constexpr int per = HIDDEN / 32;
    if (i >= (int64_t)n_pad * per) return;
    const int r = (int)(i / per), c = 32 * (int)(i % per);
    __align__(16) __half hi[32];
    __align__(16) __half lo[32];
    if (r < n) {
        float v[32];
        const float4* src = (const float4*)(x + (size_t)(t0 + r) * ld + c);
        #pragma unroll
        for (int j = 0; j < 8; ++j) { const float4 a = src[j]; v[4*j] = a.x; v[4*j+1] = a.y; v[4*j+2] = a.z; v[4*j+3] = a.w; }
        int8_t q[32];
        const float d = quant_q8_group(v, q);
        #pragma unroll
        for (int j = 0; j < 32; ++j) split_f16((float)q[j] * d, hi[j], lo[j]);
    } else {
        #pragma unroll
        for (int j = 0; j < 32; ++j) { hi[j] = __float2half_rn(0.0f); lo[j] = hi[j]; }
    }
    uint8_t* tile = out + ((size_t)(r / nt) * SG_GU_KBN + c / SG_GU_KB) * (size_t)sg_b_bytes(true, nt);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
        *(uint4*)(tile + sg_off(r % nt, 8 * j, 2 * nt)) = *(const uint4*)(hi + 8 * j);
        *(uint4*)(tile + sg_off(nt + r % nt, 8 * j, 2 * nt)) = *(const uint4*)(lo + 8 * j);
    }
}

// ---------------------------------------------------------------- the GEMM
template <bool GU, int NT>
__global__ void __launch_bounds__(SG_THREADS, 1) k_sh_gemm(SharedGemmParams p) {
    constexpr int NST = sg_nst(GU, NT), STAGE = sg_stage_bytes(GU, NT), KB = sg_kb(GU);
    constexpr int NKB = GU ? SG_GU_KBN : SG_DN_KBN;
    constexpr int A_BYTES = sg_a_bytes(GU), B_BYTES = sg_b_bytes(GU, NT), W_TILE = GU ? SG_GU_W : SG_DN_W;
    constexpr uint32_t TMEM_COLS = sg_tmem_cols(GU, NT);
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = (uint64_t*)(smem + NST * STAGE);
    uint64_t* empty = full + NST;
    uint64_t* accfull = empty + NST;
    uint64_t* drain = accfull + 1;
    uint32_t* tmem_slot = (uint32_t*)(drain + 1);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles_m = GU ? SG_GU_TILES : SG_DN_TILES;
    const int m = blockIdx.x % ntiles_m, j = blockIdx.x / ntiles_m;        // row tile, token tile
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < NST; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(accfull, 1); mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer: one bulk copy per operand tile
        if (lane == 0) {
            const uint8_t* a0 = p.w16 + (GU ? 0 : 2 * SG_GU_MAT) + (size_t)m * NKB * W_TILE;
            const uint8_t* a1 = a0 + SG_GU_MAT;                                    // up (GU only)
            const uint8_t* b = (GU ? p.x16 : p.h16) + (size_t)j * NKB * B_BYTES;
            int kb = 0;
            for (; kb < NKB; ++kb) {
                const int st = kb % NST;
                if (*abort_flag || !mbar_wait_backoff(&empty[st], ((kb / NST) & 1) ^ 1, p.err, DEV_ERR_TIMEOUT_EMPTY)) { *abort_flag = 1; break; }
                uint8_t* dst = ring + st * STAGE;
                mbar_arrive_expect_tx(&full[st], STAGE);
                bulk_g2s(dst, a0 + (size_t)kb * W_TILE, W_TILE, &full[st]);
                if (GU) bulk_g2s(dst + W_TILE, a1 + (size_t)kb * W_TILE, W_TILE, &full[st]);
                bulk_g2s(dst + A_BYTES, b + (size_t)kb * B_BYTES, B_BYTES, &full[st]);
            }
            const int first = kb > NST ? kb - NST : 0;         // every issued copy lands before the CTA exits
            for (int i = first; i < kb; ++i) mbar_wait_backoff(&full[i % NST], (i / NST) & 1, nullptr, 0);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (whole warp)
        constexpr uint32_t lbo_a = (SG_M / 8) * 128;
        constexpr uint32_t lbo_b = ((GU ? 2 * NT : NT) / 8) * 128;
        constexpr uint32_t idesc_full = idesc_f16_f32(SG_M, GU ? 2 * NT : NT), idesc_hi = idesc_f16_f32(SG_M, NT);
        const uint32_t ring_s = smem_u32(ring);
        bool ok = true;
        int kb = 0;
        for (; kb < NKB; ++kb) {
            const int st = kb % NST;
            if (!__all_sync(0xffffffffu, mbar_wait_backoff(&full[st], (kb / NST) & 1, p.err, DEV_ERR_TIMEOUT_FULL))) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = ring_s + st * STAGE;
            const uint64_t bd = umma_desc(sa + A_BYTES, lbo_b, 128);
            #pragma unroll
            for (int ks = 0; ks < KB / 16; ++ks) {
                const uint32_t acc = (kb | ks) != 0;
                const uint64_t ka = (uint64_t)((ks * 2 * lbo_a) >> 4), kbd = (uint64_t)((ks * 2 * lbo_b) >> 4);
                if (GU) {
                    #pragma unroll
                    for (int mat = 0; mat < 2; ++mat) {
                        const uint32_t d = tmem + (uint32_t)(mat * 2 * NT);
                        const uint64_t whi = umma_desc(sa + mat * W_TILE, lbo_a, 128) + ka;
                        const uint64_t wlo = umma_desc(sa + mat * W_TILE + W_TILE / 2, lbo_a, 128) + ka;
                        umma_f16_ss_warp(d, whi, bd + kbd, idesc_full, acc);        // whi x [xhi; xlo]
                        umma_f16_ss_warp(d, wlo, bd + kbd, idesc_hi, 1u);           // + wlo x xhi
                    }
                } else {
                    umma_f16_ss_warp(tmem, umma_desc(sa, lbo_a, 128) + ka, bd + kbd, idesc_full, acc);
                }
            }
            umma_commit_warp(&empty[st]);
        }
        if (!ok && lane == 0) *abort_flag = 1;
        if (ok) umma_commit_warp(accfull);
        if (kb > 0) {                                 // every issued MMA has completed before teardown
            umma_commit_warp(drain);
            mbar_wait_backoff(drain, 0, nullptr, 0);
        }
    } else {
        // ---------------------------------------------------------------- epilogue: TMEM lane quarter q
        const int q = warp & 3;
        const int r = SG_M * m + 32 * q + lane;      // gate/up: h index; down: output row
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int ncols = min(NT, p.n - j * NT);
        bool ok = true;                               // wait until the accumulator is complete, the kernel
        const unsigned long long t0 = globaltimer_ns();   // aborts, or the deadline passes
        while (!mbar_try_wait_sleep(accfull, 0, WAIT_SLEEP_NS)) {
            if (*abort_flag) { ok = false; break; }
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) { if (p.err) atomicCAS(p.err, 0, DEV_ERR_TIMEOUT_FULL); ok = false; break; }
        }
        if (ok) {
            tc_fence_after();
            for (int c0 = 0; c0 < ncols; c0 += 16) {
                float v0[16];
                tmem_ld16(tmem + lane_base + (uint32_t)c0, v0);
                if (GU) {
                    float t[16];
                    tmem_ld16(tmem + lane_base + (uint32_t)(NT + c0), t);             // gate: whi x xlo
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) v0[i] += t[i];
                    float v1[16];
                    tmem_ld16(tmem + lane_base + (uint32_t)(2 * NT + c0), v1);        // up
                    tmem_ld16(tmem + lane_base + (uint32_t)(3 * NT + c0), t);
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) v1[i] += t[i];
                    // h[token j*NT + c0 + i][r] -> the down GEMM's B tiles (token tile j, K block r / 64)
                    uint8_t* hb = p.h16 + ((size_t)j * SG_DN_KBN + r / SG_DN_KB) * sg_b_bytes(false, NT);
                    #pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float hv = lk_swiglu(v0[i], v1[i]);
                        float amax = fabsf(hv);
                        #pragma unroll
                        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                        const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
                        const float hq = (float)(int)rintf(hv * id) * d;
                        if (c0 + i < ncols) *(__half*)(hb + sg_off(c0 + i, r % SG_DN_KB, NT)) = __float2half_rn(hq);
                    }
                } else {
                    #pragma unroll
                    for (int i = 0; i < 16; ++i)
                        if (c0 + i < ncols) p.y[(size_t)(p.row0 + j * NT + c0 + i) * HIDDEN + r] = v0[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) { tc_fence_after(); tmem_dealloc(tmem, TMEM_COLS); }
}

template <bool GU, int NT>
static void launch_sh_gemm(const SharedGemmParams& p, cudaStream_t st) {
    constexpr int smem = sg_smem(GU, NT);
    static bool attr = false;
    if (!attr) { cudaFuncSetAttribute(k_sh_gemm<GU, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); attr = true; }
    const int grid = (GU ? SG_GU_TILES : SG_DN_TILES) * ((p.n + NT - 1) / NT);
    k_sh_gemm<GU, NT><<<grid, SG_THREADS, smem, st>>>(p);
}
// one CTA per SM (more than half the shared memory), so a CTA never waits for another's tensor memory, and
// the gate/up accumulators (4 NT columns) fit the 512 columns
static_assert(sg_smem(true, 128) <= 232448 && sg_smem(false, 128) <= 232448, "stages exceed the 227 KB a CTA can have");
static_assert(sg_smem(true, 64) > 116224 && sg_smem(false, 64) > 116224 && sg_smem(true, 128) > 116224 &&
              sg_smem(false, 128) > 116224, "tile shapes must hold one CTA per SM");
static_assert(sg_nst(true, 128) >= 3 && sg_nst(false, 128) >= 3, "at least three stages");
static_assert(sg_tmem_cols(true, 128) <= 512, "tensor memory holds 512 columns");
static_assert(SH_GEMM_W16_BYTES == 2 * SG_GU_MAT + (size_t)SG_DN_TILES * SG_DN_KBN * SG_DN_W, "w16 size");

int sh_gemm_tile_tokens(int n) { return n > 512 ? 128 : 64; }

int launch_shared_gemm(const SharedGemmParams& p, cudaStream_t st) {
    if (p.n <= 0) return 0;
    const int nt = sh_gemm_tile_tokens(p.n);
    const int n_pad = (p.n + nt - 1) / nt * nt;
    const int64_t gw = (int64_t)MOE_INTER * (HIDDEN / 8), dw = (int64_t)HIDDEN * (MOE_INTER / 8);
    k_sh_w16<FMT_Q5K><<<(unsigned)((gw + 255) / 256), 256, 0, st>>>(p.gate, MOE_INTER, HIDDEN, p.w16);
    k_sh_w16<FMT_Q5K><<<(unsigned)((gw + 255) / 256), 256, 0, st>>>(p.up, MOE_INTER, HIDDEN, p.w16 + SG_GU_MAT);
    k_sh_w16<FMT_Q6K><<<(unsigned)((dw + 255) / 256), 256, 0, st>>>(p.down, HIDDEN, MOE_INTER, p.w16 + 2 * SG_GU_MAT);
    const int64_t nx = (int64_t)n_pad * (HIDDEN / 32);
    k_sh_x16<<<(unsigned)((nx + 255) / 256), 256, 0, st>>>(p.x, p.ld_x, p.t0, p.n, n_pad, nt, p.x16);
    if (nt == 128) { launch_sh_gemm<true, 128>(p, st); launch_sh_gemm<false, 128>(p, st); }
    else { launch_sh_gemm<true, 64>(p, st); launch_sh_gemm<false, 64>(p, st); }
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

}  // namespace lk
