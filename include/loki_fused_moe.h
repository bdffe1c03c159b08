/* loki_fused_moe.h -- the MoE entry points of loki's fused-layer ABI, served by libloki_moe.so.
 *
 * The names, argument lists and meanings are those of the reference's src/fused_layer.h, so that
 * src/server_core_fused.cpp links against this library for its MoE calls without source changes; the
 * attention half of that header (fl_attn, fl_spec, fl_sketch) is out of scope and stays with the
 * reference build.  What replaces what (reference line numbers):
 *   fl_init          src/fused_layer.h:24     context: stream, buffers, pinned host mirrors
 *   fl_wide_init     src/fused_layer.h:29     buffers for a wide (prefill) pass of up to wmax rows
 *   fl_wide_moe      src/fused_layer.h:30     one arena batch of expert slots (<= 8 (row, k) pairs each)
 *   fl_wide_mark     src/fused_layer.h:31     record the parity's event
 *   fl_wide_wait     src/fused_layer.h:32     host wait on that event
 *   fl_wide_finish   src/fused_layer.h:33     h = base + sum_k out, moe = sum_k out, to pinned mirrors
 *   fl_moe_outs      src/fused_layer.h:35     one row's weighted expert pushes (narrow pass)
 *   fl_wide_outs     src/fused_layer.h:36     one row's weighted expert pushes (wide pass)
 *   fl_wide_skip     src/fused_layer.h:37     h = base + stored output (wide pass)
 *   fl_fetch         src/fused_layer.h:43     sel/wts/ncur/fi (what & 1) and h (what & 32) to the host
 *   fl_moe           src/fused_layer.h:45     narrow pass: routed experts for n <= 8 rows, combined
 *   fl_skip          src/fused_layer.h:47     h = stored output + shared + ffn_inp
 *   fl_h2d           src/fused_layer.h:49     host -> device on the context stream
 *   fl_wait_event    src/fused_layer.h:51     the context stream waits for an event
 *   fl_gpu_ms        src/fused_layer.h:52     accumulated GPU time (1: experts, 2: prepare)
 * Additive (no counterpart: it is the MoE half of fl_attn, src/fused_layer.cu:506-525):
 *   fl_moe_prepare   router + shared expert on the rows' normalised hidden state `ncur` with residual
 *                    `ffn_inp`; leaves the context as fl_attn does for the MoE calls that follow.
 * Additive (no counterpart: the engine's host routing post-pass, src/server_core_fused.cpp:793-818, done on
 * the device):
 *   fl_moe_auto      fl_fetch + host keep pass + fl_moe in one call, without the routing round trip.
 *
 * Behaviour kept from the reference: host arrays (ids, w, slot tables) are copied before the call
 * returns; FLOut points into library-owned pinned mirrors valid until the next call on the context;
 * fl_moe, fl_fetch, fl_wide_finish, fl_skip, fl_wide_skip block the host until their results are in
 * the mirrors.  Differences: errors are printed and recorded (fl_moe_error) instead of exit(7); the
 * down projection format is FL_IQ2, FL_Q2K or FL_Q3K (the real model's downs; other formats return
 * LK_ERR_UNSUPPORTED through fl_moe_error), with the routed arena's expert stride
 * ggml_row_size(down_fmt, 2048) * 7168 as in the engine's load_experts; the shared expert passed to
 * fl_moe_prepare is IQ2_XXS; with HBM-resident shards, ids may be global expert ids into the full
 * 256-expert arena.
 */
#ifndef LOKI_FUSED_MOE_H
#define LOKI_FUSED_MOE_H
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

struct FLCtx;
typedef struct FLCtx FLCtx;
typedef struct CUevent_st* fl_event_t;        /* == cudaEvent_t */
#ifndef LOKI_FL_NO_FORMAT_ENUM   /* a translation unit that already has src/fused_layer.h's identical enum defines this */
enum { FL_Q4K = 0, FL_Q6K = 1, FL_Q80 = 2, FL_Q5K = 3, FL_IQ2 = 4, FL_Q2K = 5, FL_Q3K = 6 };
#endif

/* host (pinned) mirrors filled by fl_fetch / fl_moe / fl_skip / fl_wide_finish; null where not produced.
 * Field order and meaning as the reference's FLOut. */
typedef struct FLOut {
    const int* sel; const float* wts; const float* ncur; const float* fi; const float* skt; const int* sel_s;
    const float* wts_s; const float* sc; const float* ccat; const float* h; const float* moe;
} FLOut;

/* the MoE weights fl_moe_prepare needs: router (F32 or F16 [256][7168]) + bias, shared expert (IQ2_XXS) */
typedef struct FLMoeW {
    const void* gate_inp; int gate_f16; const float* probs_b;
    const void* sh_gate; const void* sh_up; const void* sh_down;
    int sh_fmt;     /* 0 / FL_IQ2: IQ2_XXS shared expert (IQ2_XXS down); FL_Q5K: the real model's Q5_K gate/up + Q6_K down */
} FLMoeW;

LK_API FLCtx* fl_init(int kvp, int sc_cap);
LK_API int    fl_wide_init(FLCtx* c, int wmax, int KE);
LK_API void   fl_wide_moe(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int nexp,
                   const int* midx, const int* rows, const int* kidx, const float* wk, int nslots, int KE, int par);
LK_API void   fl_wide_mark(FLCtx* c, int par);
LK_API void   fl_wide_wait(FLCtx* c, int par);
LK_API void   fl_wide_finish(FLCtx* c, int n, int KE, FLOut* out);
LK_API void   fl_moe_outs(FLCtx* c, int b, const int* ids, const float* w, int KE, float* out);
LK_API void   fl_wide_outs(FLCtx* c, int row, int KE, float* out);
LK_API void   fl_wide_skip(FLCtx* c, const float* mo, int n, FLOut* out);
LK_API void   fl_fetch(FLCtx* c, int n, int what, FLOut* out);
LK_API void   fl_moe(FLCtx* c, const void* gate, const void* up, const void* down, int nexp, int down_fmt,
              const int* ids, const float* w, int KE, int n, FLOut* out);
LK_API void   fl_skip(FLCtx* c, const float* mo, int n, FLOut* out);
LK_API void   fl_h2d(FLCtx* c, void* dst, const void* src, size_t bytes);
LK_API void   fl_wait_event(FLCtx* c, fl_event_t ev);
LK_API double fl_gpu_ms(FLCtx* c, int which);

/* additive: the MoE half of fl_attn.  ncur / ffn_inp: N x 7168 fp32 rows, host pointers (host = 1) or
 * device pointers (host = 0).  wrow >= 0: these rows are rows wrow.. of a wide pass (their ncur and
 * ffn_inp + shared output go to the pass-wide buffers, as fl_attn's wrow does). */
LK_API void   fl_moe_prepare(FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow);
/* additive: the narrow pass for the first n <= 8 rows of the last fl_moe_prepare, routed on the device from
 * that call's router output: each row's KE highest-weight experts (equal weights in position order; renorm = 1
 * rescales them to sum to 2.5), as global expert ids into a 256-expert resident arena.  Results as fl_moe (h,
 * moe; fl_moe_outs sees this routing).  The engine's --share-experts choice depends on the rows beside each
 * other and stays on the host path (fl_fetch + keep pass + fl_moe). */
LK_API void   fl_moe_auto(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int KE, int renorm, int n,
                          FLOut* out);
/* additive: fl_moe_prepare, fl_moe and fl_moe_auto replay a CUDA graph for every call shape (weights, row
 * count, KE, format) seen before -- captured on its second occurrence -- instead of issuing their launches and
 * copies one by one (default on; enable = 0 issues them directly).  The results are the same either way. */
LK_API void   fl_use_graphs(FLCtx* c, int enable);
/* additive: last error recorded on the context (0 = none), cleared by the call */
LK_API int    fl_moe_error(FLCtx* c);
LK_API void   fl_free(FLCtx* c);

/* ---- The same entry points under the lkfl_ prefix (identical behaviour), and three calls for a bridge library
 * that re-exports all of src/fused_layer.h with its attention half from the reference's own fused_layer.cu
 * (loki_b200/csrc/fl_bridge.cu, built as libloki_fused.so).  No counterpart in the reference: the prefix lets the
 * bridge define fl_* itself and still reach this library in the same process. */
LK_API FLCtx* lkfl_init(int kvp, int sc_cap);
LK_API void   lkfl_free(FLCtx* c);
LK_API int    lkfl_moe_error(FLCtx* c);
LK_API void   lkfl_h2d(FLCtx* c, void* dst, const void* src, size_t bytes);
LK_API void   lkfl_wait_event(FLCtx* c, fl_event_t ev);
LK_API double lkfl_gpu_ms(FLCtx* c, int which);
LK_API void   lkfl_moe_prepare(FLCtx* c, const FLMoeW* W, const float* ncur, const float* ffn_inp, int N, int host, int wrow);
LK_API void   lkfl_fetch(FLCtx* c, int n, int what, FLOut* out);
LK_API void   lkfl_moe(FLCtx* c, const void* gate, const void* up, const void* down, int nexp, int down_fmt,
                       const int* ids, const float* w, int KE, int n, FLOut* out);
LK_API void   lkfl_moe_auto(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int KE, int renorm, int n,
                            FLOut* out);
LK_API void   lkfl_use_graphs(FLCtx* c, int enable);
LK_API void   lkfl_skip(FLCtx* c, const float* mo, int n, FLOut* out);
LK_API void   lkfl_moe_outs(FLCtx* c, int b, const int* ids, const float* w, int KE, float* out);
LK_API int    lkfl_wide_init(FLCtx* c, int wmax, int KE);
LK_API void   lkfl_wide_moe(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int nexp,
                            const int* midx, const int* rows, const int* kidx, const float* wk, int nslots, int KE, int par);
LK_API void   lkfl_wide_mark(FLCtx* c, int par);
LK_API void   lkfl_wide_wait(FLCtx* c, int par);
LK_API void   lkfl_wide_finish(FLCtx* c, int n, int KE, FLOut* out);
LK_API void   lkfl_wide_skip(FLCtx* c, const float* mo, int n, FLOut* out);
LK_API void   lkfl_wide_outs(FLCtx* c, int row, int KE, float* out);
/* bridge: a context that runs on `stream` (a cudaStream_t it does not own: the attention context's), so the two
 * halves of a layer are ordered without events */
LK_API FLCtx* lkfl_init_on_stream(void* stream);
/* bridge: take over the MoE inputs that the attention half left on the device for N rows -- ncur, ffn_inp
 * ([N][7168]), the router's top-8 ids / weights ([N][8]) and the shared expert's output as n_parts partial sums
 * shared_parts[k][row] (k < n_parts, part_rows rows apart) -- instead of recomputing them (fl_moe_prepare's role);
 * wrow >= 0 places the rows in the wide pass's buffers as fl_moe_prepare does.  Stream-ordered, no host wait. */
LK_API void   lkfl_moe_adopt(FLCtx* c, const float* ncur, const float* ffn_inp, const float* shared_parts, int n_parts,
                             size_t part_rows, const int* sel, const float* wts, int N, int wrow);
/* bridge: the device rows of h written by the last fl_moe / fl_moe_auto / fl_skip ([n][7168]) */
LK_API const float* lkfl_device_h(FLCtx* c);

#ifdef __cplusplus
}
#endif
#endif
