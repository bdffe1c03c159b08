// engine_standin.cpp -- TEST INFRASTRUCTURE: a stand-in for the engine's translation unit (src/server_core_fused.cpp)
// in what it needs from the fused layer.  It includes the reference's own src/fused_layer.h (from the checkout, -I)
// and makes every call the engine makes, in the engine's order -- attention + router + shared expert (fl_attn,
// engine:746-753), the routing fetch (fl_fetch, :753), the narrow MoE pass (fl_moe, :953) or a wide pass in arena
// batches (fl_wide_init / fl_wide_wait / fl_wide_moe / fl_wide_mark / fl_wide_finish, :930-950), the memory paths
// (fl_skip, fl_wide_skip), attribution (fl_moe_outs, fl_wide_outs), the speculative pass and sketch (fl_spec,
// fl_sketch), the loader hooks (fl_h2d, fl_wait_event) and the timers (fl_gpu_ms) -- so linking it against
// libloki_fused.so alone shows the engine binds to that one library without source changes.  Without arguments
// it only reports that it linked and loaded; it touches no GPU.
#include <cstdio>
#include <vector>
#include "fused_layer.h"

static void one_layer(FLCtx* FL, const FLW* w, int n, int KE, bool wide, void* KC, void* VC, const void* arena[3]) {
    std::vector<int> pos(n);
    for (int i = 0; i < n; ++i) pos[i] = i;
    FLOut fo{};
    fl_attn(FL, w, n, 0, pos.data(), KC, VC, nullptr, 0, 0, wide ? 0 : -1);
    fl_fetch(FL, n, 1, &fo);
    std::vector<int> ids((size_t)n * KE, 0);
    std::vector<float> wts((size_t)n * KE, 0.f);
    if (!wide) {
        fl_moe(FL, arena[0], arena[1], arena[2], 1, FL_Q2K, ids.data(), wts.data(), KE, n, &fo);
        std::vector<float> pushes((size_t)KE * 7168);
        fl_moe_outs(FL, 0, ids.data(), wts.data(), KE, pushes.data());
        return;
    }
    fl_wide_init(FL, n, KE);
    std::vector<int> midx(1, 0), rows(8, -1), kidx(8, 0);
    std::vector<float> wk(8, 0.f);
    fl_wide_wait(FL, 0);
    fl_wide_moe(FL, arena[0], arena[1], arena[2], FL_Q2K, 1, midx.data(), rows.data(), kidx.data(), wk.data(), 1, KE, 0);
    fl_wide_mark(FL, 0);
    fl_wide_finish(FL, n, KE, &fo);
    std::vector<float> pushes((size_t)KE * 7168);
    fl_wide_outs(FL, 0, KE, pushes.data());
}

int main(int argc, char** argv) {
    (void)argv;
    if (argc < 2) {                    // link and load only
        std::printf("engine stand-in linked against the fused-layer ABI\n");
        return 0;
    }
    FLCtx* FL = fl_init(64, 64);
    FLW w{};
    const void* arena[3] = { nullptr, nullptr, nullptr };
    one_layer(FL, &w, 1, 8, false, nullptr, nullptr, arena);
    one_layer(FL, &w, 16, 8, true, nullptr, nullptr, arena);
    FLOut fo{};
    std::vector<float> mo(7168, 0.f);
    fl_skip(FL, mo.data(), 1, &fo);
    fl_wide_skip(FL, mo.data(), 1, &fo);
    fl_spec(FL, &w, nullptr, nullptr);
    fl_sketch(FL, nullptr, nullptr, 0);
    fl_h2d(FL, nullptr, nullptr, 0);
    fl_wait_event(FL, nullptr);
    std::printf("gpu ms %.3f %.3f\n", fl_gpu_ms(FL, 0), fl_gpu_ms(FL, 1));
    return 0;
}
