// fl_replay.cpp -- the engine side of the fused-layer MoE calls, in C++: the host keep-KE pass and the
// per-token call sequence of src/server_core_fused.cpp, driving libloki_moe.so exactly as the engine
// drives src/fused_layer.h.  Built as libloki_replay.so (linked against libloki_moe.so); bench.py's
// end-to-end figure and the fl ABI tests run through it, so that number is the ABI's cost with host
// buffers, not a Python interpreter's.
//
//   lkr_keep    the keep-KE compaction of server_core_fused.cpp:793-813 (weight order with ties in position
//               order, the --share-experts variant of :799-807, renormalisation to 2.5 of :811)
//   lkr_decode  per layer: fl_moe_prepare (host ncur / ffn_inp) -> fl_fetch(what = 1) -> lkr_keep ->
//               fl_moe with global expert ids into HBM-resident arenas (the sequence of engine:753-953 for
//               the narrow pass; mode 0), or fl_moe_prepare -> fl_moe_auto (the routing post-pass on the
//               device; mode 1), for `steps` timed tokens after `warmup` untimed ones; wall clock
#include <algorithm>
#include <chrono>
#include <cstring>
#include <set>
#include <vector>
#include "../../include/loki_fused_moe.h"

extern "C" {

__attribute__((visibility("default")))
int lkr_keep(const int* sel8, const float* w8, int n, int KE, int renorm, int share, int n_pad_from, int* sel, float* w) {
    if (!sel8 || !w8 || !sel || !w || n < 0 || KE < 1 || KE > 8) return -1;
    if (KE == 8) {                                    // the engine compacts only for KE < 8
        std::memcpy(sel, sel8, (size_t)n * 8 * sizeof(int));
        std::memcpy(w, w8, (size_t)n * 8 * sizeof(float));
        return 0;
    }
    std::vector<std::vector<int>> ords(n, std::vector<int>(8));
    for (int i = 0; i < n; ++i) {
        for (int k = 0; k < 8; ++k) ords[i][k] = k;
        std::stable_sort(ords[i].begin(), ords[i].end(), [&](int a, int b) { return w8[i * 8 + a] > w8[i * 8 + b]; });
    }
    if (share && n > 1) {
        const int own = std::min(2, KE);
        std::set<int> U;
        for (int i = 0; i < n && i < n_pad_from; ++i)
            for (int k = 0; k < own; ++k) U.insert(sel8[i * 8 + ords[i][k]]);
        for (int i = 0; i < n; ++i) {
            std::vector<int> pick(ords[i].begin(), ords[i].begin() + own);
            for (int k = own; k < 8 && (int)pick.size() < KE; ++k)
                if (U.count(sel8[i * 8 + ords[i][k]])) pick.push_back(ords[i][k]);
            for (int k = own; k < 8 && (int)pick.size() < KE; ++k)
                if (std::find(pick.begin(), pick.end(), ords[i][k]) == pick.end()) {
                    pick.push_back(ords[i][k]);
                    U.insert(sel8[i * 8 + ords[i][k]]);
                }
            for (int k = 0; k < KE; ++k) { sel[i * KE + k] = sel8[i * 8 + pick[k]]; w[i * KE + k] = w8[i * 8 + pick[k]]; }
        }
    } else {
        for (int i = 0; i < n; ++i)
            for (int k = 0; k < KE; ++k) { sel[i * KE + k] = sel8[i * 8 + ords[i][k]]; w[i * KE + k] = w8[i * 8 + ords[i][k]]; }
    }
    if (renorm)
        for (int i = 0; i < n; ++i) {
            float sw = 0.0f;
            for (int k = 0; k < KE; ++k) sw += w[i * KE + k];
            if (sw > 1e-6f) { const float f = 2.5f / sw; for (int k = 0; k < KE; ++k) w[i * KE + k] *= f; }
        }
    return 0;
}

// x, resid: [layers][n][7168] host rows; gate/up/down: per layer the 256-expert arenas; mw: per layer the
// router and shared expert.  h_last (optional): the last timed step's h of the last layer [n][7168].
// Returns the seconds of the timed steps, or a negative value when a call recorded an error.
__attribute__((visibility("default")))
double lkr_decode(FLCtx* c, int layers, const FLMoeW* mw, const void* const* gate, const void* const* up, const void* const* down,
                  int down_fmt, const float* x, const float* resid, int n, int KE, int warmup, int steps, float* h_last, int mode) {
    if (!c || layers < 1 || n < 1 || n > 8 || KE < 1 || KE > 8 || warmup < 0 || steps < 1) return -1.0;
    std::vector<int> sel((size_t)n * KE);
    std::vector<float> w((size_t)n * KE);
    const size_t row = 7168;
    FLOut o{};
    auto step = [&](bool last) {
        for (int l = 0; l < layers; ++l) {
            fl_moe_prepare(c, &mw[l], x + (size_t)l * n * row, resid + (size_t)l * n * row, n, 1, -1);
            if (mode == 1) {
                fl_moe_auto(c, gate[l], up[l], down[l], down_fmt, KE, 1, n, &o);
            } else {
                fl_fetch(c, n, 1, &o);
                lkr_keep(o.sel, o.wts, n, KE, 1, 0, n, sel.data(), w.data());
                fl_moe(c, gate[l], up[l], down[l], 256, down_fmt, sel.data(), w.data(), KE, n, &o);
            }
            if (last && l == layers - 1 && h_last && o.h) std::memcpy(h_last, o.h, (size_t)n * row * sizeof(float));
        }
    };
    for (int s = 0; s < warmup; ++s) step(false);
    if (fl_moe_error(c)) return -2.0;
    const auto t0 = std::chrono::steady_clock::now();
    for (int s = 0; s < steps; ++s) step(s == steps - 1);
    const auto t1 = std::chrono::steady_clock::now();
    if (fl_moe_error(c)) return -2.0;
    return std::chrono::duration<double>(t1 - t0).count();
}

}  // extern "C"
