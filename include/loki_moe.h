/* loki_moe.h -- B200-native DeepSeek-R1 MoE layer: the device-pointer C ABI of libloki_moe.so.
 *
 * Every pointer argument is a device pointer unless stated otherwise; work is queued on the caller's
 * stream and the calls do not synchronise (lk_moe_get_error does).  Return values are status codes
 * (LK_OK = 0, negative = error; lk_moe_strerror names them); no call exits the process.
 *
 * What each entry point replaces in the reference (grimnier/loki):
 *   lk_moe_route     router_probs + router_topk        src/fused_layer.cu:314-332 (launched :506)
 *                    + the host keep-KE post-pass      src/server_core_fused.cpp:793-813
 *   lk_moe_dispatch  per-expert (row, k) lists          src/server_core_fused.cpp:937
 *   lk_moe_experts   fl_moe's expert products + combine src/fused_layer.cu:599-612 (gate/up :605,
 *                    swiglu_q8 :606, down :608, moe_combine :609) and the shared expert of fl_attn
 *                    src/fused_layer.cu:521-524
 *   lk_moe_forward   lk_moe_route + lk_moe_experts      (the MoE half of one layer)
 *   lk_gen_iq2       (no counterpart: seeded synthetic IQ2_XXS weights for tests and benchmarks)
 */
#ifndef LOKI_MOE_H
#define LOKI_MOE_H
#include <stdint.h>
#include <stddef.h>

#ifndef LK_API
#if defined(__GNUC__)
#define LK_API __attribute__((visibility("default")))
#else
#define LK_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* lk_stream_t;      /* == cudaStream_t */
typedef struct LkMoeCtx LkMoeCtx;

enum {
    LK_OK = 0,
    LK_ERR_ARG = -1,          /* bad argument (null pointer, size out of range, misaligned weights) */
    LK_ERR_CUDA = -2,         /* a CUDA runtime call failed */
    LK_ERR_UNSUPPORTED = -3,  /* configuration the kernels do not implement (e.g. a down format) */
    LK_ERR_CAPACITY = -4,     /* more tokens than the context was created for */
    LK_ERR_DEVICE = -5        /* a kernel recorded an error (bounded wait expired, bad slot) */
};

enum { LK_FMT_Q6K = 1, LK_FMT_Q5K = 3, LK_FMT_IQ2 = 4, LK_FMT_Q2K = 5, LK_FMT_Q3K = 6 };   /* numerically equal to FL_* */

typedef struct LkMoeConfig {
    int n_experts;      /* routed experts: 256, or an expert-parallel shard's count (the router needs 256) */
    int topk;           /* experts chosen by score (8) */
    int keep;           /* experts kept per token after ordering by weight (the engine's --experts; <= topk) */
    int renorm;         /* 1: kept weights rescaled to sum to `scale` (the engine's default) */
    int n_group;        /* 1: plain top-k (the reference); 8: DeepSeek-V3 grouped top-k */
    int topk_group;     /* groups kept in grouped mode (4) */
    float scale;        /* routed scaling factor (2.5) */
    int with_shared;    /* 1: run the shared expert and add it in the combine */
    int max_tokens;     /* capacity: tokens per call */
} LkMoeConfig;

typedef struct LkMoeWeights {
    /* routed experts in the engine's arena layout: expert e's matrix at base + e * stride (bytes) */
    const void* gate; const void* up; const void* down;
    int64_t gate_stride, up_stride, down_stride;
    int down_fmt;                 /* format of every routed down matrix: LK_FMT_IQ2, or the real model's
                                     LK_FMT_Q2K / LK_FMT_Q3K (fl_moe's down_fmt, src/fused_layer.h:45); the K-quants
                                     run the single-token matvec path at every T (q8 SwiGLU output, as the reference) */
    /* shared expert, same shapes as one routed expert; null when with_shared == 0.  Formats: sh_fmt 0 or
     * LK_FMT_IQ2 = IQ2_XXS gate/up with a down in down_fmt (run as extra slots of the routed launches);
     * LK_FMT_Q5K = the real model's Q5_K gate/up and Q6_K down (src/fused_layer.h:14; own launches, the
     * reference's shared-expert numerics: q8 x, per-32 / per-16 integer sums, q8 SwiGLU output) */
    const void* sh_gate; const void* sh_up; const void* sh_down;
    /* router: weights [n_experts][7168] fp32 (router_w_f16 = 0) or fp16 (1); bias [n_experts] fp32 */
    const void* router_w; int router_w_f16;
    const float* router_bias;
    int sh_fmt;
} LkMoeWeights;

LK_API int  lk_moe_create(const LkMoeConfig* cfg, int device, LkMoeCtx** out);
LK_API void lk_moe_destroy(LkMoeCtx* ctx);

/* router: x [T][7168] fp32 -> sel/w [T][keep] (+ probs [T][n_experts] if non-null).  logits_override
 * (optional, [T][n_experts]) replaces W.x in the selection; the GEMV still runs. */
LK_API int lk_moe_route(LkMoeCtx* ctx, const LkMoeWeights* W, const float* x, int T, const float* logits_override,
                 int* sel, float* w, float* probs, lk_stream_t stream);

/* dispatch: sel [T][keep] -> counts [n_experts], offsets [n_experts+1], perm [T*keep] (flat t*keep+k
 * entries grouped by expert, stable by (t, k)) */
LK_API int lk_moe_dispatch(LkMoeCtx* ctx, const int* sel, const float* w, int T, int keep,
                    int* counts, int* offsets, int* perm, lk_stream_t stream);

/* experts + combine for given routing: h = resid + shared(x) + sum_k w[t][k] * expert_{sel[t][k]}(x[t]),
 * moe = the routed sum.  h / moe may be null. */
LK_API int lk_moe_experts(LkMoeCtx* ctx, const LkMoeWeights* W, const float* x, const float* resid, int T,
                   const int* sel, const float* w, int keep, float* h, float* moe, lk_stream_t stream);

/* the whole MoE layer: route + experts + combine; sel/w (optional) receive the routing */
LK_API int lk_moe_forward(LkMoeCtx* ctx, const LkMoeWeights* W, const float* x, const float* resid, int T,
                   const float* logits_override, float* h, float* moe, int* sel, float* w, lk_stream_t stream);

/* per-slot weighted expert outputs of the last lk_moe_experts/lk_moe_forward call: [T*keep (+T shared)][7168] */
LK_API const float* lk_moe_slot_outputs(LkMoeCtx* ctx);

/* token count from which lk_moe_forward / lk_moe_experts (and the expert-parallel stages) use the
 * tensor-core GEMM path (tcgen05, slots of up to 128 tokens per expert; default 192) */
LK_API int lk_moe_set_gemm_threshold(LkMoeCtx* ctx, int min_tokens);
/* below the GEMM threshold (default 192), calls with at least min_tokens tokens (default 48) take the register-fed
 * mma.sync path (IQ2 decoded into tensor-core fragments, reused by up to 16 tokens per expert slot);
 * smaller calls take the single-token dp4a matvecs */
LK_API int lk_moe_set_mma_threshold(LkMoeCtx* ctx, int min_tokens);
/* calls with >= min_tokens tokens (default 16) run a Q5_K/Q6_K shared expert (sh_fmt = LK_FMT_Q5K) as two
 * dense tcgen05 GEMMs (its weights dequantised once per call; the q8 of x and of h as in the per-token path,
 * fp16 hi/lo operands, fp32 accumulation); fewer tokens take the per-token q8 kernels.  The dense path's
 * buffers (~147 MB + 32 KB per token) are allocated on its first use outside a stream capture. */
LK_API int lk_moe_set_shared_gemm_threshold(LkMoeCtx* ctx, int min_tokens);

/* optional per-kernel timing: events[0..3] (cudaEvent_t) recorded on the launch stream before the gate/up
 * kernel, after it, after the down kernel and after the combine of every following lk_moe_forward /
 * lk_moe_experts call (also inside CUDA-graph capture); null disables. */
LK_API int lk_moe_set_events(LkMoeCtx* ctx, void* const* events);

/* synchronise `stream`, then read and clear the context's device error word */
LK_API int lk_moe_get_error(LkMoeCtx* ctx, lk_stream_t stream);
LK_API const char* lk_moe_strerror(int code);
LK_API const char* lk_moe_last_error(LkMoeCtx* ctx);

/* lk_moe_experts_noalloc -- no counterpart in the reference.  The expert stage of lk_moe_experts
 * (dispatch, gate/up + SwiGLU, down, combine) for callers that cannot allocate device memory: an engine
 * that has already given all free HBM to resident expert shards and KV cache (a further cudaMalloc would
 * fail or evict), or a latency-critical caller that cannot take cudaMalloc's device-wide synchronisation.
 * No context: nothing is allocated or freed.  Its scratch is one static device array of
 * LK_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until exit, so it serves at most
 * LK_NOALLOC_MAX_TOKENS tokens and keep <= 8 per call; larger calls return LK_ERR_CAPACITY (with a message
 * on stderr).  The first call on a device looks the array's address up (cudaGetSymbolAddress, with that
 * device current): make that first call before any stream capture.  All calls share the array and it keeps
 * the last call's contents; calls that overlap on the GPU race on it, so serialise them.  The kernel error
 * word is cleared at the start of each call and, if `status` (a device int) is given, copied there at the
 * end (0 = no error).  Arguments as lk_moe_experts, plus with_shared (run the shared expert W->sh_*). */
#define LK_NOALLOC_MAX_TOKENS 8
#define LK_NOALLOC_SCRATCH_BYTES 2241536
LK_API int lk_moe_experts_noalloc(const LkMoeWeights* W, const float* x, const float* resid, int T, const int* sel,
                                  const float* w, int keep, int with_shared, float* h, float* moe, int* status,
                                  lk_stream_t stream);

/* seeded synthetic IQ2_XXS weights: n_exp consecutive experts [rows][K] of (layer, matrix 0 gate / 1 up
 * / 2 down), expert expert0+i written at dst + i * stride; the same bytes as the CPU generator. */
LK_API int lk_gen_iq2(void* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
               int64_t stride, lk_stream_t stream);
/* the same for any format: fmt LK_FMT_IQ2 (identical to lk_gen_iq2), LK_FMT_Q2K or LK_FMT_Q3K (every byte but the
 * fp16 scales uniform, d and dmin = fp16(|N(0,1)|*1e-3)); the same bytes as the CPU generator */
LK_API int lk_gen_weights(int fmt, void* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                          int64_t stride, lk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
