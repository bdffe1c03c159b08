// ref_harness.cu -- TEST INFRASTRUCTURE, not product.  Builds the reference's own MoE code
// (src/fused_layer.cu of the reference checkout, included from where it lies by `make -C oracle ref`; nothing
// of it is copied here) into oracle/_ref/libref_moe.so with the reference's own flags (nvcc -O3 -arch=sm_89,
// build.bat:13; the sm_89 PTX is JIT-compiled for the B200), and exposes entry points that run ITS kernels:
//   refh_router  router_probs + router_topk as attn_block launches them (fused_layer.cu:506)
//   refh_moe     the shared expert as fl_attn runs it (quant_x, Q5_K gate/up, swiglu_q8, Q6_K down;
//                fused_layer.cu:521-524), then the narrow MoE pass fl_moe (:599-612) with its combine
//   refh_ctx / refh_wide_rows   the context and the rows fl_attn leaves for the exported wide pass
//   refh_bench   the device time of the first two, for the timing beside the pin
// The GPU tests compare these with the CPU oracle: they pin the oracle's routing and layer arithmetic
// against the reference itself.  Every call is synchronous; inputs and outputs are host arrays.
#include <chrono>
#include "fused_layer.cu"

namespace {

FLCtx* g_ctx = nullptr;
FLCtx* ref_ctx() {
    if (!g_ctx) g_ctx = fl_init(64, 64);          // attention-side sizes kept small: only the MoE buffers are used
    return g_ctx;
}

// device copy of a host array, with 4 KB of zeroed slack after it (no read of the reference's staging loops
// can leave the allocation)
template <class T> T* upload(const void* host, size_t bytes) {
    T* d = nullptr;
    CK(cudaMalloc((void**)&d, bytes + 4096));
    CK(cudaMemset(d, 0, bytes + 4096));
    if (bytes) CK(cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice));
    return d;
}

}  // namespace

extern "C" {

// x [n][7168] fp32, gate_inp [256][7168] fp32 (f16 = 0) or fp16 (f16 = 1), bias [256] -> probs [n][256],
// sel [n][8], wts [n][8]; n <= 64
int refh_router(const float* x, int n, const void* gate_inp, int f16, const float* bias, float* probs, int* sel, float* wts) {
    if (n < 1 || n > RMAX) return 1;
    FLCtx* c = ref_ctx();
    cudaStream_t st = c->st;
    float* xd = upload<float>(x, (size_t)n * E * 4);
    void* wd = upload<uint8_t>(gate_inp, (size_t)256 * E * (f16 ? 2 : 4));
    float* bd = upload<float>(bias, 256 * 4);
    float *pd = nullptr, *wtd = nullptr; int* sd = nullptr;
    CK(cudaMalloc((void**)&pd, (size_t)n * 256 * 4)); CK(cudaMalloc((void**)&sd, (size_t)n * 8 * 4)); CK(cudaMalloc((void**)&wtd, (size_t)n * 8 * 4));
    router_probs<<<blocks_for((size_t)n * 256 * 32), 256, 0, st>>>(xd, wd, f16, pd, n);
    router_topk<<<n, 256, 0, st>>>(pd, bd, sd, wtd);
    CK(cudaStreamSynchronize(st));
    CK(cudaMemcpy(probs, pd, (size_t)n * 256 * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(sel, sd, (size_t)n * 8 * 4, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(wts, wtd, (size_t)n * 8 * 4, cudaMemcpyDeviceToHost));
    void* fr[] = { xd, wd, bd, pd, sd, wtd };
    for (void* p : fr) cudaFree(p);
    return 0;
}

// One narrow MoE pass of n <= 8 rows through the reference: x (ncur) and resid (ffn_inp) [n][7168]; arenas
// of nexp experts (gate/up IQ2_XXS, down Q2_K (down_fmt 5) or Q3_K (6)), slot ids / weights [n][KE];
// optional shared expert (Q5_K gate, Q5_K up, Q6_K down; all three null = none) -> h, moe [n][7168]
int refh_moe(const float* x, const float* resid, int n, const uint8_t* gate, const uint8_t* up, const uint8_t* down, int nexp,
             int down_fmt, const int* ids, const float* w, int KE, const uint8_t* sh_gate, const uint8_t* sh_up,
             const uint8_t* sh_down, float* h, float* moe) {
    if (n < 1 || n > NB || nexp < 1 || KE < 1 || KE > 8 || (down_fmt != FL_Q2K && down_fmt != FL_Q3K)) return 1;
    FLCtx* c = ref_ctx();
    cudaStream_t st = c->st;
    const size_t wsg = (size_t)HSH * (E / QK) * BLK_IQ2;
    const size_t wsd = (size_t)E * (HSH / QK) * (down_fmt == FL_Q3K ? BLK_Q3 : BLK_Q2);
    uint8_t* gd = upload<uint8_t>(gate, nexp * wsg);
    uint8_t* ud = upload<uint8_t>(up, nexp * wsg);
    uint8_t* dd = upload<uint8_t>(down, nexp * wsd);
    CK(cudaMemset(c->ncur, 0, (size_t)NB * E * 4));
    CK(cudaMemset(c->ffn_inp, 0, (size_t)NB * E * 4));
    CK(cudaMemcpy(c->ncur, x, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->ffn_inp, resid, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    uint8_t *sg = nullptr, *su = nullptr, *sdn = nullptr;
    if (sh_gate && sh_up && sh_down) {            // fl_attn's shared expert on ncur, one row-block (G = 1, R = NB)
        sg = upload<uint8_t>(sh_gate, (size_t)HSH * (E / QK) * BLK_Q5);
        su = upload<uint8_t>(sh_up, (size_t)HSH * (E / QK) * BLK_Q5);
        sdn = upload<uint8_t>(sh_down, (size_t)E * (HSH / QK) * BLK_Q6);
        const int G = 1;
        quant_x<<<blocks_for((size_t)NB * (E / 32)), 256, 0, st>>>(c->ncur, E, G, E, NB * E, c->xcur);
        mvg(c, F_Q5K, sg, 0, HSH, E, 1, c->xcur, 7, c->partS, G);
        mvg(c, F_Q5K, su, 0, HSH, E, 1, c->xcur, 7, c->partS + (size_t)7 * NB * HSH, G);
        swiglu_q8<<<blocks_for((size_t)NB * (HSH / 32)), 256, 0, st>>>(c->partS, c->partS + (size_t)7 * NB * HSH, 7, G, HSH, c->xh);
        mvg(c, F_Q6K, sdn, 0, E, HSH, 1, c->xh, 2, c->partSD, G);
    } else {
        CK(cudaMemsetAsync(c->partSD, 0, (size_t)2 * NB * E * 4, st));
    }
    FLOut out;
    fl_moe(c, gd, ud, dd, nexp, down_fmt, ids, w, KE, n, &out);
    std::memcpy(h, out.h, (size_t)n * E * 4);
    std::memcpy(moe, out.moe, (size_t)n * E * 4);
    void* fr[] = { gd, ud, dd, sg, su, sdn };
    for (void* p : fr) if (p) cudaFree(p);
    return 0;
}

// The reference's context, for driving its exported wide pass (fl_wide_init / fl_wide_moe / fl_wide_mark /
// fl_wide_wait / fl_wide_finish, fused_layer.cu:528-561) the way the engine does (engine:930-950)
void* refh_ctx() { return ref_ctx(); }

// What fl_attn(wrow = 0) leaves for a wide pass of n rows without a shared expert: ncur_all = x and
// base_all = resid (fused_layer.cu:525, base_rows with zero shared partials).  Call after fl_wide_init.
int refh_wide_rows(const float* x, const float* resid, int n) {
    FLCtx* c = ref_ctx();
    if (!c->ncur_all || n < 1 || n > c->wmax) return 1;
    CK(cudaMemcpy(c->ncur_all, x, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->base_all, resid, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    return 0;
}

// Device time of the reference on one decode layer's MoE work, per call, over `iters` calls after 3 warm-up
// calls, with every input resident: the shared expert as fl_attn launches it (events around its four
// launches) and fl_moe (its own em0/em1 events, fl_gpu_ms(c, 1)).  Before each call `flush` (device,
// flush_bytes) is overwritten so no weight is served from L2.  Returns 0; *moe_us / *shared_us / *wall_us
// receive the mean per call (wall: fl_moe's host call, which includes its synchronisation).
int refh_bench(const float* x, const float* resid, int n, const uint8_t* gate, const uint8_t* up, const uint8_t* down, int nexp,
               int down_fmt, const int* ids, const float* w, int KE, const uint8_t* sh_gate, const uint8_t* sh_up,
               const uint8_t* sh_down, void* flush, size_t flush_bytes, int iters, double* moe_us, double* shared_us, double* wall_us) {
    if (n < 1 || n > NB || nexp < 1 || KE < 1 || KE > 8 || iters < 1 || (down_fmt != FL_Q2K && down_fmt != FL_Q3K)) return 1;
    FLCtx* c = ref_ctx();
    cudaStream_t st = c->st;
    const size_t wsg = (size_t)HSH * (E / QK) * BLK_IQ2;
    const size_t wsd = (size_t)E * (HSH / QK) * (down_fmt == FL_Q3K ? BLK_Q3 : BLK_Q2);
    uint8_t* gd = upload<uint8_t>(gate, nexp * wsg);
    uint8_t* ud = upload<uint8_t>(up, nexp * wsg);
    uint8_t* dd = upload<uint8_t>(down, nexp * wsd);
    uint8_t* sg = upload<uint8_t>(sh_gate, (size_t)HSH * (E / QK) * BLK_Q5);
    uint8_t* su = upload<uint8_t>(sh_up, (size_t)HSH * (E / QK) * BLK_Q5);
    uint8_t* sdn = upload<uint8_t>(sh_down, (size_t)E * (HSH / QK) * BLK_Q6);
    CK(cudaMemset(c->ncur, 0, (size_t)NB * E * 4));
    CK(cudaMemset(c->ffn_inp, 0, (size_t)NB * E * 4));
    CK(cudaMemcpy(c->ncur, x, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->ffn_inp, resid, (size_t)n * E * 4, cudaMemcpyHostToDevice));
    cudaEvent_t s0, s1;
    CK(cudaEventCreate(&s0)); CK(cudaEventCreate(&s1));
    double sh_ms = 0.0, wall = 0.0;
    const double moe0 = c->ms_moe;
    FLOut out;
    for (int it = -3; it < iters; ++it) {
        if (it == 0) { sh_ms = 0.0; wall = 0.0; }
        const double m_before = c->ms_moe;
        if (flush) CK(cudaMemsetAsync(flush, it & 0xFF, flush_bytes, st));
        CK(cudaEventRecord(s0, st));
        const int G = 1;
        quant_x<<<blocks_for((size_t)NB * (E / 32)), 256, 0, st>>>(c->ncur, E, G, E, NB * E, c->xcur);
        mvg(c, F_Q5K, sg, 0, HSH, E, 1, c->xcur, 7, c->partS, G);
        mvg(c, F_Q5K, su, 0, HSH, E, 1, c->xcur, 7, c->partS + (size_t)7 * NB * HSH, G);
        swiglu_q8<<<blocks_for((size_t)NB * (HSH / 32)), 256, 0, st>>>(c->partS, c->partS + (size_t)7 * NB * HSH, 7, G, HSH, c->xh);
        mvg(c, F_Q6K, sdn, 0, E, HSH, 1, c->xh, 2, c->partSD, G);
        CK(cudaEventRecord(s1, st));
        if (flush) CK(cudaMemsetAsync(flush, (it + 1) & 0xFF, flush_bytes, st));
        const auto t0 = std::chrono::steady_clock::now();
        fl_moe(c, gd, ud, dd, nexp, down_fmt, ids, w, KE, n, &out);
        const auto t1 = std::chrono::steady_clock::now();
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, s0, s1));
        if (it >= 0) { sh_ms += ms; wall += std::chrono::duration<double, std::micro>(t1 - t0).count(); }
        if (it < 0) c->ms_moe = m_before;         // warm-up calls do not count
        (void)moe0;
    }
    *moe_us = (c->ms_moe - moe0) * 1e3 / iters;
    *shared_us = sh_ms * 1e3 / iters;
    *wall_us = wall / iters;
    CK(cudaEventDestroy(s0)); CK(cudaEventDestroy(s1));
    void* fr[] = { gd, ud, dd, sg, su, sdn };
    for (void* p : fr) cudaFree(p);
    return 0;
}

}  // extern "C"
