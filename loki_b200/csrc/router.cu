// router.cu -- the DeepSeek-R1 router on sm_100a.
//
// k_router_logits: logits[t][e] = W[e] . x[t] (fp32 or fp16 weights), then probs = sigmoid(logits or an
//   override).  Replaces router_probs (reference src/fused_layer.cu:314-322).  One CTA = one expert x a
//   tile of up to 8 tokens; 256 threads each own the float4 chunks c = tid, tid+256, ... of the row (all
//   loads in flight at once; fmaf over the 4 components in order), then a warp xor-butterfly and
//   ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)) across the 8 warps.  The order is fixed and restated by the oracle
//   (orc_router_logits), so probabilities -- and with them the selected experts -- are bit-identical to it.
//   The last CTA to finish a token tile (an atomic count after a fence) runs the top-k for it, so the
//   router is one launch.
// k_router_batch (T >= 64): the same logits in the same order, with the data movement turned around: a CTA
//   keeps a tile of 8 tokens' rows in shared memory and streams expert rows past it, 4 experts at a time
//   against all 8 tokens (32 accumulators per thread, expert chunks 3 deep in registers), so each (token,
//   expert) pair costs ~3.5 KB of L2 traffic and each fmaf 1 B of shared-memory traffic.  Thread p still owns partial p (chunks p + 256 j
//   of every row, fmaf in the same order, the butterfly's pair sums and the same warp tree), so the results
//   are bit-identical to k_router_logits and the oracle.
// router_topk_token: one warp per token: top-k of p + bias with ties to the lower expert id (reference
//   router_topk, src/fused_layer.cu:323-332), or the DeepSeek-V3 grouped mode (n_group groups of 32
//   experts, group score = sum of the group's top-2, keep topk_group groups); weights p/max(sum, 2^-14)
//   * scale; then the engine's keep-KE compaction (src/server_core_fused.cpp:793-813: order by weight,
//   keep KE, rescale the kept weights to sum to `scale`).  For T == 1 it also writes the decode slot
//   table (one slot per kept expert + the shared expert), so no dispatch kernel is needed at decode.
#include "moe_internal.h"
#include "moe_device.cuh"
#include "ep_device.cuh"
#include <cuda_fp16.h>

namespace lk {

__device__ void router_topk_token(const RouterParams& p, int t, int lane);
__device__ void router_topk_cta(const RouterParams& p, int t);

__device__ __forceinline__ int atom_add_acq_rel_gpu(int* a, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
    return old;
}

// one CTA = one expert x a tile of NTT tokens; 256 threads, each owns float4 chunks c = tid + 256 j
template <int NTT>
__global__ void __launch_bounds__(256) k_router_logits(RouterParams p) {
    __shared__ float ws[8][NTT];
    __shared__ int last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e = blockIdx.x;
    const int t0 = blockIdx.y * NTT;
    const int nt = min(NTT, p.T - t0);
    constexpr int NCH = HIDDEN / 4;                 // 1792 float4 chunks, 7 per thread
    float4 w[NCH / 256];
    #pragma unroll
    for (int j = 0; j < NCH / 256; ++j) {
        const int c = tid + 256 * j;
        if (p.w_f16) {
            const uint2 raw = __ldg((const uint2*)((const __half*)p.W + (size_t)e * HIDDEN) + c);
            const float2 a = __half22float2(*(const __half2*)&raw.x), b = __half22float2(*(const __half2*)&raw.y);
            w[j] = make_float4(a.x, a.y, b.x, b.y);
        } else {
            w[j] = __ldg((const float4*)((const float*)p.W + (size_t)e * HIDDEN) + c);
        }
    }
    // the router weights are never written by a kernel: their loads are in flight before the wait for
    // the previous kernel (which may still be producing x)
    pdl_trigger();
    pdl_wait();
    if (NTT == 1 && p.xq && e < HIDDEN / 32 && warp == 0) {   // one token: q8 group e of x for the experts
        const float4 xv = lane < 8 ? ((const float4*)p.x)[e * 8 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        float amax = fmaxf(fmaxf(fabsf(xv.x), fabsf(xv.y)), fmaxf(fabsf(xv.z), fabsf(xv.w)));
        #pragma unroll
        for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;      // as quant_q8_group
        if (lane < 8) {
            const int q0 = (int)rintf(xv.x * id), q1 = (int)rintf(xv.y * id), q2 = (int)rintf(xv.z * id), q3 = (int)rintf(xv.w * id);
            ((uint32_t*)p.xq)[e * 8 + lane] = (uint32_t)(uint8_t)q0 | (uint32_t)(uint8_t)q1 << 8 |
                                              (uint32_t)(uint8_t)q2 << 16 | (uint32_t)(uint8_t)q3 << 24;
            ((uint32_t*)p.xqn)[e * 8 + lane] = (uint32_t)(uint8_t)-q0 | (uint32_t)(uint8_t)-q1 << 8 |
                                               (uint32_t)(uint8_t)-q2 << 16 | (uint32_t)(uint8_t)-q3 << 24;
            if (lane == 0) p.xd[e] = d;
        }
    }
    #pragma unroll
    for (int t = 0; t < NTT; ++t) {
        float a = 0.0f;
        if (t < nt) {
            const float4* xr = (const float4*)(p.x + (size_t)(t0 + t) * p.ld_x);
            #pragma unroll
            for (int j = 0; j < NCH / 256; ++j) {
                const float4 xv = xr[tid + 256 * j];
                a = fmaf(w[j].x, xv.x, a);
                a = fmaf(w[j].y, xv.y, a);
                a = fmaf(w[j].z, xv.z, a);
                a = fmaf(w[j].w, xv.w, a);
            }
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) ws[warp][t] = a;
    }
    __syncthreads();
    if (tid < nt) {
        const int t = tid;
        const float lg = __fadd_rn(__fadd_rn(__fadd_rn(ws[0][t], ws[1][t]), __fadd_rn(ws[2][t], ws[3][t])),
                                   __fadd_rn(__fadd_rn(ws[4][t], ws[5][t]), __fadd_rn(ws[6][t], ws[7][t])));
        const size_t o = (size_t)(t0 + t) * p.n_experts + e;
        p.logits[o] = lg;
        const float v = p.logits_override ? p.logits_override[o] : lg;
        p.probs[o] = lk_sigmoid(v);
    }
    // the last CTA of this token tile runs the top-k for it.  The count is an acquire-release atomic:
    // each CTA releases its probabilities (ordered before it by the barrier), and the last one acquires
    // everyone's before its barrier hands them to its other threads.
    if (!p.tile_count) return;
    __syncthreads();
    if (tid == 0) last = atom_add_acq_rel_gpu(&p.tile_count[blockIdx.y], 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    if (nt == 1) router_topk_cta(p, t0);          // one token: all 8 warps
    else if (warp < nt) router_topk_token(p, t0 + warp, lane);
    __syncthreads();
    if (tid == 0) p.tile_count[blockIdx.y] = 0;       // ready for the next call
    // expert-parallel decode: the token's rows to every rank (the other CTAs' q8 groups of x were acquired
    // with the count; this CTA's sel / w are ordered before the barrier above)
    if (NTT == 1 && p.send.n_ranks && p.xq) ep_send_token(p.send, p.sel + (size_t)t0 * p.keep, p.w + (size_t)t0 * p.keep, p.keep, p.xq, p.xd);
}

constexpr int RB_TT = 8;                          // tokens per CTA tile
constexpr int RB_EG = 4;                          // experts per group: 8 x 4 (token, expert) accumulators per thread
constexpr int RB_NP = RB_TT * RB_EG;              // 32 pairs per group: one per lane after the warp reduction
constexpr int RB_SMEM = RB_TT * HIDDEN * 4;       // the token tile: 224 KB, one CTA per SM
constexpr int RB_J = HIDDEN / 1024;               // 7 float4 chunks per thread and row
constexpr int RB_RING = 4;                        // expert chunks in flight per thread (registers)

// chunk j (float4 tid + 256 j) of the rows of experts e .. e + RB_EG - 1
__device__ __forceinline__ void rb_load_wc(const RouterParams& p, int e, int j, int tid, float4 (&w)[RB_EG]) {
    const int c = tid + 256 * j;
    #pragma unroll
    for (int k = 0; k < RB_EG; ++k) {
        if (p.w_f16) {
            const uint2 raw = __ldg((const uint2*)((const __half*)p.W + (size_t)(e + k) * HIDDEN) + c);
            const float2 a = __half22float2(*(const __half2*)&raw.x), b = __half22float2(*(const __half2*)&raw.y);
            w[k] = make_float4(a.x, a.y, b.x, b.y);
        } else {
            w[k] = __ldg((const float4*)((const float*)p.W + (size_t)(e + k) * HIDDEN) + c);
        }
    }
}

// acc[RB_EG t + k] += the 4 products of chunk w[k] with x chunk xv[t], in component order (fmaf), the 32 pairs
// interleaved component by component
__device__ __forceinline__ void rb_fma(float (&acc)[RB_NP], const float4 (&w)[RB_EG], const float4 (&xv)[RB_TT]) {
    #pragma unroll
    for (int t = 0; t < RB_TT; ++t)
        #pragma unroll
        for (int k = 0; k < RB_EG; ++k) acc[RB_EG * t + k] = fmaf(w[k].x, xv[t].x, acc[RB_EG * t + k]);
    #pragma unroll
    for (int t = 0; t < RB_TT; ++t)
        #pragma unroll
        for (int k = 0; k < RB_EG; ++k) acc[RB_EG * t + k] = fmaf(w[k].y, xv[t].y, acc[RB_EG * t + k]);
    #pragma unroll
    for (int t = 0; t < RB_TT; ++t)
        #pragma unroll
        for (int k = 0; k < RB_EG; ++k) acc[RB_EG * t + k] = fmaf(w[k].z, xv[t].z, acc[RB_EG * t + k]);
    #pragma unroll
    for (int t = 0; t < RB_TT; ++t)
        #pragma unroll
        for (int k = 0; k < RB_EG; ++k) acc[RB_EG * t + k] = fmaf(w[k].w, xv[t].w, acc[RB_EG * t + k]);
}

// one CTA = RB_TT tokens x experts [e0, e0 + n_experts / esplit) in groups of RB_EG; the top-k of a token
// tile runs in the CTA that finishes it (its only CTA when esplit == 1).
// Thread p owns partial p of every (token, expert) pair: chunks p + 256 j (j = 0..6) with fmaf over the 4
// components in order -- k_router_logits' order.  The token rows sit in shared memory (each thread reads only
// its own chunks, which it stored itself).  The expert chunks stream through registers as one sequence
// q = 7 * group + j, RB_RING chunks ahead of their use.  A warp's 32 partials of each of the 32 pairs of a group
// are summed by halving exchanges (offsets 16, 8, 4, 2, 1: at each step a lane keeps half of its values and
// adds the partner's copy of the same pair), which forms exactly the xor butterfly's pair sums and leaves pair
// `lane` in lane `lane`; the 8 warp sums as ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).  So the logits are
// bit-identical to k_router_logits and to the oracle.
__global__ void __launch_bounds__(256, 1) k_router_batch(RouterParams p) {
    const int esplit = p.esplit;
    extern __shared__ __align__(16) float4 xt[];  // [RB_TT][HIDDEN / 4]
    __shared__ float ws[2][8][RB_NP];             // warp sums, double-buffered by group parity
    __shared__ int last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NCH = HIDDEN / 4;
    const int t0 = blockIdx.x * RB_TT, nt = min(RB_TT, p.T - t0);
    const int per = p.n_experts / esplit, e0 = blockIdx.y * per;
    const int nq = per / RB_EG * RB_J;            // chunks of this CTA's expert rows, in use order
    float4 ring[RB_RING][RB_EG];
    #pragma unroll
    for (int r = 0; r < RB_RING; ++r)             // router weights are never written by a kernel
        if (r < nq) rb_load_wc(p, e0 + r / RB_J * RB_EG, r % RB_J, tid, ring[r]);
    int pf_g = e0 + RB_RING / RB_J * RB_EG, pf_j = RB_RING % RB_J;   // the chunk RB_RING ahead
    pdl_trigger();
    pdl_wait();
    #pragma unroll
    for (int t = 0; t < RB_TT; ++t)
        #pragma unroll
        for (int j = 0; j < RB_J; ++j)
            xt[t * NCH + tid + 256 * j] = t < nt ? ((const float4*)(p.x + (size_t)(t0 + t) * p.ld_x))[tid + 256 * j]
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
    float acc[RB_NP];                             // pair i = RB_EG * t + k
    #pragma unroll
    for (int i = 0; i < RB_NP; ++i) acc[i] = 0.0f;
    int j = 0, gi = 0;                            // chunk and group of q
    for (int q0 = 0; q0 < nq; q0 += RB_RING) {
        #pragma unroll
        for (int r = 0; r < RB_RING; ++r) {
            const int q = q0 + r;
            if (q >= nq) break;                   // uniform across the CTA
            float4 xv[RB_TT];
            #pragma unroll
            for (int t = 0; t < RB_TT; ++t) xv[t] = xt[t * NCH + tid + 256 * j];
            rb_fma(acc, ring[r], xv);
            if (q + RB_RING < nq) {               // refill this ring slot with the chunk RB_RING ahead
                rb_load_wc(p, pf_g, pf_j, tid, ring[r]);
                if (++pf_j == RB_J) { pf_j = 0; pf_g += RB_EG; }
            }
            if (j == RB_J - 1) {                  // the group's sums: warp reduction, then the warp tree
                #pragma unroll
                for (int o = 16, h = RB_NP / 2; o >= 1; o >>= 1, h >>= 1) {
                    const bool up = (lane & o) != 0;
                    #pragma unroll
                    for (int i = 0; i < h; ++i) {
                        const float send = up ? acc[i] : acc[i + h];
                        const float keep = up ? acc[i + h] : acc[i];
                        acc[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
                    }
                }
                // pair index bits 4..0 = lane bits 4..0.  One barrier per group: group n's sums go to buffer
                // n & 1 and are read by warp n % 8 after the barrier; buffer n & 1 is next written after the
                // following group's barrier, which that reader has passed only once it finished reading.
                float (*wb)[RB_NP] = ws[gi & 1];
                wb[warp][lane] = acc[0];
                __syncthreads();
                if (warp == (gi & 7)) {
                    const int t = lane / RB_EG, k = lane % RB_EG;
                    if (t < nt) {
                        const float lg = __fadd_rn(__fadd_rn(__fadd_rn(wb[0][lane], wb[1][lane]), __fadd_rn(wb[2][lane], wb[3][lane])),
                                                   __fadd_rn(__fadd_rn(wb[4][lane], wb[5][lane]), __fadd_rn(wb[6][lane], wb[7][lane])));
                        const size_t o = (size_t)(t0 + t) * p.n_experts + e0 + gi * RB_EG + k;
                        p.logits[o] = lg;
                        const float v = p.logits_override ? p.logits_override[o] : lg;
                        p.probs[o] = lk_sigmoid(v);
                    }
                }
                #pragma unroll
                for (int i = 0; i < RB_NP; ++i) acc[i] = 0.0f;
                j = 0; ++gi;
            } else {
                ++j;
            }
        }
    }
    __syncthreads();                              // every group's probabilities are written
    if (!p.tile_count) return;
    if (esplit > 1) {                             // as k_router_logits: acquire-release count per token tile
        if (tid == 0) last = atom_add_acq_rel_gpu(&p.tile_count[blockIdx.x], 1) == esplit - 1;
        __syncthreads();
        if (!last) return;
    }
    if (warp < nt) router_topk_token(p, t0 + warp, lane);
    if (esplit > 1) {
        __syncthreads();
        if (tid == 0) p.tile_count[blockIdx.x] = 0;   // ready for the next call
    }
}

// warp argmax over (value, index) pairs, ties -> lower index; every lane returns the winner
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
    }
}

__device__ __forceinline__ void router_finish(const RouterParams& p, int t, int lane, const int (&sel)[MAX_TOPK],
                                              const float (&ps)[MAX_TOPK]);

__device__ void router_topk_token(const RouterParams& p, int t, int lane) {
    const float* pr = p.probs + (size_t)t * p.n_experts;   // written by other CTAs: read past L1
    constexpr int PER = N_EXPERTS / 32;             // 8 experts per lane: e = lane + 32*i
    float sc[PER], pv[PER];
    bool allowed[PER];
    #pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        pv[i] = __ldcg(pr + e);
        sc[i] = __fadd_rn(pv[i], p.bias[e]);
        allowed[i] = true;
    }
    if (p.n_group > 1) {                            // n_group == 8 groups of 32: group g = register i
        float gs[PER];
        #pragma unroll
        for (int g = 0; g < PER; ++g) {
            float v1 = sc[g]; int i1 = lane + 32 * g;
            warp_argmax(v1, i1);
            float v2 = (lane + 32 * g == i1) ? -INFINITY : sc[g]; int i2 = (lane + 32 * g == i1) ? 0x7fffffff : lane + 32 * g;
            warp_argmax(v2, i2);
            gs[g] = __fadd_rn(v1, v2);
        }
        bool keepg[PER];
        #pragma unroll
        for (int g = 0; g < PER; ++g) keepg[g] = false;
        for (int r = 0; r < p.topk_group; ++r) {
            int bg = -1; float bv = 0.0f;
            #pragma unroll
            for (int g = 0; g < PER; ++g) if (!keepg[g] && (bg < 0 || gs[g] > bv)) { bg = g; bv = gs[g]; }
            #pragma unroll
            for (int g = 0; g < PER; ++g) if (g == bg) keepg[g] = true;
        }
        #pragma unroll
        for (int i = 0; i < PER; ++i) allowed[i] = keepg[i];
    }
    int sel[MAX_TOPK]; float ps[MAX_TOPK];
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) {
        sel[k] = 0; ps[k] = 0.0f;
        if (k >= p.topk) continue;
        float bv = -INFINITY; int bi = 0x7fffffff;
        #pragma unroll
        for (int i = 0; i < PER; ++i)
            if (allowed[i] && (bi == 0x7fffffff || sc[i] > bv)) { bv = sc[i]; bi = lane + 32 * i; }
        warp_argmax(bv, bi);
        sel[k] = bi;
        float mine = 0.0f;                          // the winner's probability, from its lane's registers
        #pragma unroll
        for (int i = 0; i < PER; ++i) if (lane + 32 * i == bi) { allowed[i] = false; mine = pv[i]; }
        ps[k] = __shfl_sync(0xffffffffu, mine, bi & 31);
    }
    router_finish(p, t, lane, sel, ps);
}

// weights of the selected experts (normalised, scaled), the engine's keep pass, and the outputs;
// sel / ps: the topk selected experts and their probabilities in selection order (all lanes alike)
__device__ __forceinline__ void router_finish(const RouterParams& p, int t, int lane, const int (&sel)[MAX_TOPK],
                                              const float (&ps)[MAX_TOPK]) {
    // every loop runs over the constant MAX_TOPK with predicates, so the arrays stay in registers
    float sum = 0.0f;
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) if (k < p.topk) sum = __fadd_rn(sum, ps[k]);
    sum = fmaxf(sum, 6.103515625e-5f);
    float pk = 0.0f;                                  // lane k divides entry k's probability, then all gather
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) if (k == lane) pk = ps[k];
    const float mine = __fmul_rn(__fdiv_rn(pk, sum), p.scale);
    float wt[MAX_TOPK];
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) wt[k] = __shfl_sync(0xffffffffu, mine, k);
    int osel[MAX_TOPK]; float ow[MAX_TOPK];
    const int keep = p.keep;
    if (keep >= p.topk) {
        #pragma unroll
        for (int k = 0; k < MAX_TOPK; ++k) { osel[k] = sel[k]; ow[k] = wt[k]; }
    } else {
        // the engine's stable sort by weight, descending: entry a goes to position
        // #{b : wt[b] > wt[a]} + #{b < a : wt[b] == wt[a]}
        #pragma unroll
        for (int r = 0; r < MAX_TOPK; ++r) { osel[r] = 0; ow[r] = 0.0f; }
        #pragma unroll
        for (int a = 0; a < MAX_TOPK; ++a) {
            int r = 0;
            #pragma unroll
            for (int b = 0; b < MAX_TOPK; ++b)
                if (b < p.topk && b != a && (wt[b] > wt[a] || (wt[b] == wt[a] && b < a))) ++r;
            #pragma unroll
            for (int q = 0; q < MAX_TOPK; ++q) if (a < p.topk && r == q) { osel[q] = sel[a]; ow[q] = wt[a]; }
        }
        float sw = 0.0f;
        #pragma unroll
        for (int k = 0; k < MAX_TOPK; ++k) if (k < keep) sw = __fadd_rn(sw, ow[k]);
        if (p.renorm && sw > 1e-6f) {
            const float f = __fdiv_rn(p.scale, sw);
            #pragma unroll
            for (int k = 0; k < MAX_TOPK; ++k) if (k < keep) ow[k] = __fmul_rn(ow[k], f);
        }
    }
    if (lane < keep) {
        int sv = 0; float wv = 0.0f;
        #pragma unroll
        for (int k = 0; k < MAX_TOPK; ++k) if (k == lane) { sv = osel[k]; wv = ow[k]; }
        p.sel[(size_t)t * keep + lane] = sv;
        p.w[(size_t)t * keep + lane] = wv;
        if (p.slot_expert && p.T == 1) {            // decode slot table, one token per slot
            p.slot_expert[lane] = sv; p.slot_tok[lane] = 0; p.slot_out[lane] = lane; p.slot_w[lane] = wv;
        }
    }
    if (p.slot_expert && p.T == 1 && lane == 0) {
        if (p.with_shared) {
            p.slot_expert[keep] = SHARED_SLOT; p.slot_tok[keep] = 0; p.slot_out[keep] = keep; p.slot_w[keep] = 1.0f;
        }
        *p.nslots = keep + (p.with_shared ? 1 : 0);
    }
}

// One token's top-k with the whole CTA (256 threads = 256 experts, group g = warp g).  Each warp sorts its
// 32 (score, id) pairs by a bitonic network over shuffles (descending score, ties to the lower id): a
// group's score is then lanes 0 + 1, and its best topk are lanes 0..topk-1.  The allowed groups' best
// topk are the candidates; each candidate's rank among them is its position in the selection.  The
// result (order included) is that of topk rounds of argmax over the allowed experts.
__device__ void router_topk_cta(const RouterParams& p, int t) {
    __shared__ float s_p[N_EXPERTS];
    __shared__ float s_gs[8];
    __shared__ float s_cv[8 * MAX_TOPK];
    __shared__ int s_ci[8 * MAX_TOPK];
    __shared__ int s_sel[MAX_TOPK];
    __shared__ float s_ps[MAX_TOPK];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const float pv = __ldcg(p.probs + (size_t)t * p.n_experts + tid);
    s_p[tid] = pv;
    float v = __fadd_rn(pv, p.bias[tid]);
    int i = tid;
    #pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
        #pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, j);
            const int oi = __shfl_xor_sync(0xffffffffu, i, j);
            const bool mine_better = v > ov || (v == ov && i < oi);
            const bool keep_mine = (((lane & j) == 0) == ((lane & k) == 0)) ? mine_better : !mine_better;
            if (!keep_mine) { v = ov; i = oi; }
        }
    }
    const float second = __shfl_sync(0xffffffffu, v, 1);
    if (lane == 0) s_gs[warp] = __fadd_rn(v, second);
    __syncthreads();
    unsigned allowed = 0xFFu;
    if (p.n_group > 1) {                              // top topk_group groups, ties -> lower group
        allowed = 0u;
        for (int r = 0; r < p.topk_group; ++r) {
            int bg = -1; float bv = 0.0f;
            #pragma unroll
            for (int g = 0; g < 8; ++g) if (!((allowed >> g) & 1u) && (bg < 0 || s_gs[g] > bv)) { bg = g; bv = s_gs[g]; }
            allowed |= 1u << bg;
        }
    }
    const int nc = __popc(allowed) * p.topk;
    if (((allowed >> warp) & 1u) && lane < p.topk) {
        const int pos = __popc(allowed & ((1u << warp) - 1u)) * p.topk + lane;
        s_cv[pos] = v; s_ci[pos] = i;
    }
    __syncthreads();
    if (tid < nc) {
        const float cv = s_cv[tid]; const int ci = s_ci[tid];
        int rank = 0;
        for (int c = 0; c < nc; ++c) { const float ov = s_cv[c]; const int oi = s_ci[c]; rank += (ov > cv || (ov == cv && oi < ci)) ? 1 : 0; }
        if (rank < p.topk) { s_sel[rank] = ci; s_ps[rank] = s_p[ci]; }
    }
    __syncthreads();
    if (warp == 0) {
        int sel[MAX_TOPK]; float ps[MAX_TOPK];
        #pragma unroll
        for (int k = 0; k < MAX_TOPK; ++k) { sel[k] = k < p.topk ? s_sel[k] : 0; ps[k] = k < p.topk ? s_ps[k] : 0.0f; }
        router_finish(p, t, lane, sel, ps);
    }
}

// p.tile_count: T zeroed ints (one per token tile of 8; left zeroed again)
void launch_router(const RouterParams& p, cudaStream_t st) {
    const int ne = p.n_experts;
    if (p.T <= 1) launch_pdl(k_router_logits<1>, dim3(ne, 1), dim3(256), 0, st, p);
    else if (p.T <= 2) launch_pdl(k_router_logits<2>, dim3(ne, 1), dim3(256), 0, st, p);
    else if (p.T <= 4) launch_pdl(k_router_logits<4>, dim3(ne, 1), dim3(256), 0, st, p);
    else if (p.T < 64) launch_pdl(k_router_logits<8>, dim3(ne, (p.T + 7) / 8), dim3(256), 0, st, p);
    else {                                        // batches: token tiles in shared memory, expert rows streamed
        static bool attr = false;
        if (!attr) { cudaFuncSetAttribute(k_router_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, RB_SMEM); attr = true; }
        int dev = 0; cudaGetDevice(&dev);
        const int tiles = (p.T + RB_TT - 1) / RB_TT, target = num_sms(dev);
        int esplit = 1;                           // split the experts until every SM has a CTA
        while (tiles * esplit < target && (ne / (2 * esplit)) % RB_EG == 0) esplit *= 2;
        RouterParams q = p;
        q.esplit = esplit;
        launch_pdl(k_router_batch, dim3(tiles, esplit), dim3(256), RB_SMEM, st, q);
    }
}

}  // namespace lk
