// fl_bridge.cu -- libloki_fused.so: all of the reference's src/fused_layer.h in one library, so that an unchanged
// src/server_core_fused.cpp links against it instead of the reference's fused_layer.cu.
//
//   attention half   fl_attn, fl_spec, fl_sketch, fl_fetch, fl_h2d, fl_wait_event, fl_gpu_ms (but 1): the
//                    reference's own src/fused_layer.cu, compiled here from the reference checkout (#included at
//                    build time from -I<checkout>/src; nothing of it is copied into this repository) with every name
//                    it exports moved aside (ref_fl_*, RefFLCtx, RefFLOut) and kept internal to this library;
//   MoE half         fl_moe, fl_skip, fl_wide_*, fl_moe_outs, fl_wide_outs, fl_gpu_ms(1): libloki_moe.so through its
//                    lkfl_* names (loki_b200/csrc/fl_abi.cu).
//
// The hand-off between the halves (the reference keeps both in one context, src/fused_layer.cu:509-527): fl_init
// creates the reference's context and a MoE context on the reference's stream (lkfl_init_on_stream), so both
// halves are stream-ordered without events.  After the reference's fl_attn of a MoE layer the MoE context adopts
// what it left on the device -- ncur, ffn_inp, the router's top-8 ids and weights, and the shared expert's output
// as the two partial sums of its down projection -- instead of recomputing them (lkfl_moe_adopt); a wide pass's
// rows (wrow >= 0) go to the MoE context's pass buffers as well.  After fl_moe / fl_skip the MoE context's device
// h is copied into the reference context's output rows (lo2), which the next layer's fl_attn reads when the engine
// passes hin = null.  fl_wide_init sets up both contexts: the reference's fl_attn writes its own wide buffers too.
//
// Built by loki_b200/build.py (build_bridge) when a reference checkout is given; the reference's internal layout
// that the hand-off reads (the context fields above, two shared-expert partial sums laid out [k][R rows][7168] with
// R = round_g((N + 7) / 8) * 8) is that checkout's src/fused_layer.cu:441-527.
#include <cstring>
#include <cstdio>

#define FLCtx RefFLCtx
#define FLOut RefFLOut
#define fl_init ref_fl_init
#define fl_attn ref_fl_attn
#define fl_wide_init ref_fl_wide_init
#define fl_wide_moe ref_fl_wide_moe
#define fl_wide_mark ref_fl_wide_mark
#define fl_wide_wait ref_fl_wide_wait
#define fl_wide_finish ref_fl_wide_finish
#define fl_moe_outs ref_fl_moe_outs
#define fl_wide_outs ref_fl_wide_outs
#define fl_wide_skip ref_fl_wide_skip
#define fl_spec ref_fl_spec
#define fl_sketch ref_fl_sketch
#define fl_fetch ref_fl_fetch
#define fl_moe ref_fl_moe
#define fl_skip ref_fl_skip
#define fl_h2d ref_fl_h2d
#define fl_wait_event ref_fl_wait_event
#define fl_gpu_ms ref_fl_gpu_ms
#include "fused_layer.cu"
#undef FLCtx
#undef FLOut
#undef fl_init
#undef fl_attn
#undef fl_wide_init
#undef fl_wide_moe
#undef fl_wide_mark
#undef fl_wide_wait
#undef fl_wide_finish
#undef fl_moe_outs
#undef fl_wide_outs
#undef fl_wide_skip
#undef fl_spec
#undef fl_sketch
#undef fl_fetch
#undef fl_moe
#undef fl_skip
#undef fl_h2d
#undef fl_wait_event
#undef fl_gpu_ms

#define LOKI_FL_NO_FORMAT_ENUM
#include "../../include/loki_fused_moe.h"

namespace {

struct Bridge {
    RefFLCtx* a = nullptr;            // the reference's context: attention, router, shared expert
    FLCtx* m = nullptr;               // this library's MoE context, on a->st
};
Bridge* br(FLCtx* c) { return reinterpret_cast<Bridge*>(c); }

static_assert(sizeof(RefFLOut) == sizeof(FLOut), "FLOut field order and meaning are the reference's");
void out_of(const RefFLOut& r, FLOut* o) { std::memcpy(o, &r, sizeof(FLOut)); }

// the MoE context's device h rows -> the reference context's output rows, for a following fl_attn(hin = null)
void h_to_attention(Bridge* b, int n) {
    const float* h = lkfl_device_h(b->m);
    if (h && n > 0) CK(cudaMemcpyAsync(b->a->lo2, h, (size_t)n * E * sizeof(float), cudaMemcpyDeviceToDevice, b->a->st));
}

}  // namespace

extern "C" {

LK_API FLCtx* fl_init(int kvp, int sc_cap) {
    Bridge* b = new Bridge();
    b->a = ref_fl_init(kvp, sc_cap);
    b->m = lkfl_init_on_stream((void*)b->a->st);
    if (!b->m) { std::fprintf(stderr, "[loki_fused] MoE context: allocation failed\n"); std::exit(7); }
    return reinterpret_cast<FLCtx*>(b);
}

LK_API void fl_attn(FLCtx* c, const FLW* W, int N, int pos0, const int* pos, void* KC, void* VC, const float* hin, int dense,
                    int last_row, int wrow) {
    Bridge* b = br(c);
    ref_fl_attn(b->a, W, N, pos0, pos, KC, VC, hin, dense, last_row, wrow);
    if (dense) return;
    const RefFLCtx* a = b->a;
    const int R = round_g((N + NB - 1) / NB) * NB;
    lkfl_moe_adopt(b->m, a->ncur, a->ffn_inp, a->partSD, 2, (size_t)R, a->sel, a->wts, N, wrow);
}

LK_API void fl_spec(FLCtx* c, const FLW* W1, void* KC1, void* VC1) { ref_fl_spec(br(c)->a, W1, KC1, VC1); }
LK_API void fl_sketch(FLCtx* c, const float* TPROJ, const void* GSKT, int K) { ref_fl_sketch(br(c)->a, TPROJ, GSKT, K); }

LK_API void fl_fetch(FLCtx* c, int n, int what, FLOut* out) {
    RefFLOut r;
    ref_fl_fetch(br(c)->a, n, what, &r);
    out_of(r, out);
}

LK_API void fl_moe(FLCtx* c, const void* gate, const void* up, const void* down, int nexp, int down_fmt, const int* ids,
                   const float* w, int KE, int n, FLOut* out) {
    Bridge* b = br(c);
    lkfl_moe(b->m, gate, up, down, nexp, down_fmt, ids, w, KE, n, out);
    h_to_attention(b, n);
}

LK_API void fl_skip(FLCtx* c, const float* mo, int n, FLOut* out) {
    Bridge* b = br(c);
    lkfl_skip(b->m, mo, n, out);
    h_to_attention(b, n);
}

LK_API void fl_h2d(FLCtx* c, void* dst, const void* src, size_t bytes) { ref_fl_h2d(br(c)->a, dst, src, bytes); }
LK_API void fl_wait_event(FLCtx* c, fl_event_t ev) { ref_fl_wait_event(br(c)->a, (cudaEvent_t)ev); }
LK_API double fl_gpu_ms(FLCtx* c, int which) { return which == 1 ? lkfl_gpu_ms(br(c)->m, 1) : ref_fl_gpu_ms(br(c)->a, which); }

LK_API int fl_wide_init(FLCtx* c, int wmax, int KE) {
    Bridge* b = br(c);
    return ref_fl_wide_init(b->a, wmax, KE) && lkfl_wide_init(b->m, wmax, KE) ? 1 : 0;
}
LK_API void fl_wide_moe(FLCtx* c, const void* gate, const void* up, const void* down, int down_fmt, int nexp, const int* midx,
                        const int* rows, const int* kidx, const float* wk, int nslots, int KE, int par) {
    lkfl_wide_moe(br(c)->m, gate, up, down, down_fmt, nexp, midx, rows, kidx, wk, nslots, KE, par);
}
LK_API void fl_wide_mark(FLCtx* c, int par) { lkfl_wide_mark(br(c)->m, par); }
LK_API void fl_wide_wait(FLCtx* c, int par) { lkfl_wide_wait(br(c)->m, par); }
LK_API void fl_wide_finish(FLCtx* c, int n, int KE, FLOut* out) { lkfl_wide_finish(br(c)->m, n, KE, out); }
LK_API void fl_wide_skip(FLCtx* c, const float* mo, int n, FLOut* out) { lkfl_wide_skip(br(c)->m, mo, n, out); }
LK_API void fl_moe_outs(FLCtx* c, int b, const int* ids, const float* w, int KE, float* out) { lkfl_moe_outs(br(c)->m, b, ids, w, KE, out); }
LK_API void fl_wide_outs(FLCtx* c, int row, int KE, float* out) { lkfl_wide_outs(br(c)->m, row, KE, out); }

}  // extern "C"
