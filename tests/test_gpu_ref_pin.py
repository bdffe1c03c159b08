"""The CPU oracle pinned against the reference's OWN kernels on the GPU.

oracle/_ref/libref_moe.so is src/fused_layer.cu of the reference, built from its sources with its own flags
(nvcc -O3 -arch=sm_89; `make -C oracle ref`, oracle/ref_harness.cu) and JIT-compiled for the B200.  It runs the
reference's router (router_probs / router_topk, fused_layer.cu:314-332), its shared expert as fl_attn runs it
(Q5_K gate/up, swiglu_q8, Q6_K down; :521-524) and its narrow MoE pass fl_moe (IQ2_XXS gate/up, Q2_K / Q3_K
down, moe_combine; :599-612).  The oracle must agree with it, and so must this library's GPU path."""
import ctypes
import os

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, MAT, RTOL_L2, rel_l2, FMT_Q5K, FMT_Q6K

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REF_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref", "libref_moe.so")
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_moe.so not built (make -C oracle ref needs the reference checkout)")
    L = ctypes.CDLL(REF_LIB)
    L.refh_router.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P, P, P, P]
    L.refh_moe.argtypes = [P, P, ctypes.c_int, P, P, P, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, P, P, P, P, P]
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


@pytest.mark.parametrize("f16", [False, True])
def test_router_matches_reference_kernels(native, oracle, ref, f16):
    rng = np.random.default_rng(501 + f16)
    T = 6
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    if f16:
        W = W.astype(np.float16)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    probs, sel, wts = np.empty((T, 256), np.float32), np.empty((T, 8), np.int32), np.empty((T, 8), np.float32)
    assert ref.refh_router(_p(x), T, _p(np.ascontiguousarray(W)), int(f16), _p(bias), _p(probs), _p(sel), _p(wts)) == 0
    op, osel, ow = oracle.router(x, W.astype(np.float32), bias, oracle.route_cfg(8, 8))
    np.testing.assert_allclose(probs, op, rtol=2e-6, atol=1e-7)
    np.testing.assert_array_equal(sel, osel)
    np.testing.assert_allclose(wts, ow, rtol=2e-6)


def _arena(oracle, down_fmt, NE):
    gate = np.concatenate([oracle.gen_iq2(SEED, 14, 0, e, INTER, HIDDEN) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 14, 1, e, INTER, HIDDEN) for e in range(NE)])
    down = np.concatenate([oracle.gen_kq(down_fmt, SEED, 14, 2, e, HIDDEN, INTER) for e in range(NE)])
    sh = (oracle.gen_kq(FMT_Q5K, SEED, 14, 0, 256, INTER, HIDDEN), oracle.gen_kq(FMT_Q5K, SEED, 14, 1, 256, INTER, HIDDEN),
          oracle.gen_kq(FMT_Q6K, SEED, 14, 2, 256, HIDDEN, INTER))
    return gate, up, down, sh


@pytest.mark.parametrize("down_fmt,n,KE,shared", [(5, 1, 4, True), (6, 3, 4, True), (5, 8, 2, False), (6, 2, 6, False)])
def test_moe_layer_matches_reference_kernels(native, oracle, ref, down_fmt, n, KE, shared):
    """fl_moe of the reference (with fl_attn's Q5_K/Q6_K shared expert) vs the oracle and vs this library."""
    from loki_b200 import moe as M
    NE = 6
    gate, up, down, sh = _arena(oracle, down_fmt, NE)
    DS = HIDDEN * 8 * oracle.BLOCK_BYTES[down_fmt]
    rng = np.random.default_rng(100 * down_fmt + n)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    ids = np.stack([rng.choice(NE, KE, replace=False) for _ in range(n)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (n, KE)).astype(np.float32)
    h_ref, moe_ref = np.empty((n, HIDDEN), np.float32), np.empty((n, HIDDEN), np.float32)
    shp = sh if shared else (None, None, None)
    assert ref.refh_moe(_p(x), _p(r), n, _p(gate), _p(up), _p(down), NE, down_fmt, _p(ids), _p(w), KE,
                        _p(shp[0]), _p(shp[1]), _p(shp[2]), _p(h_ref), _p(moe_ref)) == 0
    # the oracle (the reference's q8 scheme and per-sub-block integer sums)
    o = oracle.moe_layer(x, r, gate, up, down, MAT, ids, w, *shp, down_fmt=down_fmt, down_stride=DS,
                         sh_gu_fmt=FMT_Q5K, sh_down_fmt=FMT_Q6K)
    e_moe, e_h = rel_l2(o["moe"], moe_ref), rel_l2(o["h"], h_ref)
    e_sh = rel_l2(o["h"] - o["moe"] - r, h_ref - moe_ref - r) if shared else 0.0
    print("oracle vs reference kernels: moe %.2e  h %.2e  shared %.2e" % (e_moe, e_h, e_sh))
    assert e_moe < 1e-4 and e_h < 1e-4 and e_sh < 1e-4, (e_moe, e_h, e_sh)
    # this library's expert stage on the same arenas
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    g_d, u_d, d_d = dev(gate), dev(up), dev(down)
    s_d = [dev(m) for m in sh] if shared else [None, None, None]
    ws = native.LkMoeWeights(g_d.data_ptr(), u_d.data_ptr(), d_d.data_ptr(), MAT, MAT, DS, down_fmt,
                             *(m.data_ptr() if m is not None else None for m in s_d), None, 0, None, FMT_Q5K if shared else 0)
    layer = M.MoeLayer(0, topk=KE, keep=KE, max_tokens=n, n_experts=NE, with_shared=shared)
    h, mo = layer.experts(ws, dev(x), dev(r), dev(ids), dev(w))
    layer.device_error()
    assert rel_l2(mo.cpu().numpy(), moe_ref) < RTOL_L2 and rel_l2(h.cpu().numpy(), h_ref) < RTOL_L2


def test_reference_kernels_timing(native, oracle, ref):
    """Timing beside the pin: the reference's own kernels (fl_attn's shared expert + fl_moe) and this library's
    expert stage on the same decode-layer work -- the real model's formats (IQ2_XXS gate/up, Q2_K downs,
    Q5_K/Q6_K shared expert), one row, 8 experts -- with every input resident and L2 overwritten (256 MB)
    before each call.  Device time per call from CUDA events on each side; printed, not asserted."""
    from loki_b200 import moe as M
    NE, KE, n, iters = 8, 8, 1, 20
    gate, up, down, sh = _arena(oracle, 5, NE)
    DS = HIDDEN * 8 * 84
    rng = np.random.default_rng(7)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    ids = np.arange(KE, dtype=np.int32).reshape(1, KE)
    w = rng.uniform(0.1, 1.0, (1, KE)).astype(np.float32)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    moe_us, sh_us, wall_us = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    assert ref.refh_bench(_p(x), _p(r), n, _p(gate), _p(up), _p(down), NE, 5, _p(ids), _p(w), KE, _p(sh[0]), _p(sh[1]), _p(sh[2]),
                          P(flush.data_ptr()), ctypes.c_size_t(flush.numel()), iters, ctypes.byref(moe_us), ctypes.byref(sh_us),
                          ctypes.byref(wall_us)) == 0
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    g_d, u_d, d_d = dev(gate), dev(up), dev(down)
    s_d = [dev(m) for m in sh]
    ws = native.LkMoeWeights(g_d.data_ptr(), u_d.data_ptr(), d_d.data_ptr(), MAT, MAT, DS, 5, *(m.data_ptr() for m in s_d),
                             None, 0, None, FMT_Q5K)
    layer = M.MoeLayer(0, topk=KE, keep=KE, max_tokens=n, n_experts=NE)
    xd, rd, idd, wd = dev(x), dev(r), dev(ids), dev(w)
    h = torch.empty(n, HIDDEN, device="cuda")
    mo = torch.empty(n, HIDDEN, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for it in range(3 + iters):
        flush.fill_(it & 0xFF)
        e0.record()
        layer.experts(ws, xd, rd, idd, wd, h=h, moe=mo)
        e1.record()
        torch.cuda.synchronize()
        if it >= 3:
            times.append(e0.elapsed_time(e1) * 1e3)
    layer.device_error()
    ours = float(np.mean(times))
    refs = moe_us.value + sh_us.value
    print("reference kernels on B200: fl_moe %.1f us + shared expert %.1f us = %.1f us (fl_moe wall %.1f us); "
          "this library: %.1f us (%.2fx)" % (moe_us.value, sh_us.value, refs, wall_us.value, ours, refs / ours))


def _wide_lib(ref, native):
    ref.refh_ctx.restype = P
    ref.refh_wide_rows.argtypes = [P, P, ctypes.c_int]
    ref.fl_wide_init.argtypes = [P, ctypes.c_int, ctypes.c_int]
    ref.fl_wide_moe.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    ref.fl_wide_mark.argtypes = [P, ctypes.c_int]
    ref.fl_wide_wait.argtypes = [P, ctypes.c_int]
    ref.fl_wide_finish.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(native.FLOut)]
    return ref.refh_ctx()


def _run_reference_wide(ref, native, c, gate, up, down, down_fmt, nexp, ids, w, KE, n, eb):
    """The engine's wide-pass driver (src/server_core_fused.cpp:930-950) over the reference's exported calls."""
    from loki_b200 import fused as F
    used = sorted(set(int(e) for e in ids.reshape(-1)))
    plan = []
    for batch, midx, rows, kidx, wk in F.wide_slots(ids, w, KE, used, eb=eb):
        plan.append((np.array([batch[u] for u in midx], np.int32), np.array(rows, np.int32), np.array(kidx, np.int32),
                     np.array(wk, np.float32)))
    for i, (gm, rows, kidx, wk) in enumerate(plan):
        par = i & 1
        if i >= 2:
            ref.fl_wide_wait(c, par)
        ref.fl_wide_moe(c, P(gate), P(up), P(down), down_fmt, nexp, _p(gm), _p(rows), _p(kidx), _p(wk), len(gm), KE, par)
        ref.fl_wide_mark(c, par)
    out = native.FLOut()
    ref.fl_wide_finish(c, n, KE, ctypes.byref(out))
    h = np.ctypeslib.as_array(ctypes.cast(out.h, ctypes.POINTER(ctypes.c_float)), (n * HIDDEN,)).reshape(n, HIDDEN).copy()
    moe = np.ctypeslib.as_array(ctypes.cast(out.moe, ctypes.POINTER(ctypes.c_float)), (n * HIDDEN,)).reshape(n, HIDDEN).copy()
    return h, moe


@pytest.mark.parametrize("down_fmt,n,KE", [(5, 20, 4), (6, 13, 3)])
def test_wide_pass_matches_reference_kernels(native, oracle, ref, down_fmt, n, KE):
    """The reference's wide (prefill) pass -- slots of <= 8 (row, k) pairs per expert, arena batches of <= 4
    experts, double-buffered parities, wide_finish -- against the oracle and this library."""
    from loki_b200 import moe as M
    NE = 12
    gate, up, down, _ = _arena(oracle, down_fmt, NE)
    DS = HIDDEN * 8 * oracle.BLOCK_BYTES[down_fmt]
    rng = np.random.default_rng(900 + n)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    ids = np.stack([rng.choice(NE, KE, replace=False) for _ in range(n)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (n, KE)).astype(np.float32)
    c = _wide_lib(ref, native)
    assert ref.fl_wide_init(c, 64, KE) == 1
    assert ref.refh_wide_rows(_p(x), _p(r), n) == 0
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    g_d, u_d, d_d = dev(gate), dev(up), dev(down)
    h_ref, moe_ref = _run_reference_wide(ref, native, c, g_d.data_ptr(), u_d.data_ptr(), d_d.data_ptr(), down_fmt, NE, ids, w, KE, n, 4)
    o = oracle.moe_layer(x, r, gate, up, down, MAT, ids, w, down_fmt=down_fmt, down_stride=DS)
    e_moe, e_h = rel_l2(o["moe"], moe_ref), rel_l2(o["h"], h_ref)
    print("oracle vs reference wide pass: moe %.2e  h %.2e" % (e_moe, e_h))
    assert e_moe < 1e-4 and e_h < 1e-4, (e_moe, e_h)
    ws = native.LkMoeWeights(g_d.data_ptr(), u_d.data_ptr(), d_d.data_ptr(), MAT, MAT, DS, down_fmt, None, None, None, None, 0, None, 0)
    layer = M.MoeLayer(0, topk=KE, keep=KE, max_tokens=n, n_experts=NE, with_shared=False)
    h, mo = layer.experts(ws, dev(x), dev(r), dev(ids), dev(w))
    layer.device_error()
    assert rel_l2(mo.cpu().numpy(), moe_ref) < RTOL_L2 and rel_l2(h.cpu().numpy(), h_ref) < RTOL_L2


def test_reference_wide_pass_timing(native, oracle, ref):
    """Timing beside the pin, prefill: the reference's wide pass (the engine's driver over fl_wide_moe, arena
    batches of 16 experts) and this library's expert stage, T=512 rows, top-8 of 256 experts, Q2_K downs (the
    reference's wide pass takes only K-quant downs), no shared expert; host wall time of one pass each.  Both of
    this library's passes (device API and fl_wide_*) must land within 2e-3 of the reference's own wide pass."""
    import time
    from loki_b200 import fused as F
    from loki_b200 import moe as M
    T, KE = 512, 8
    W = M.LayerWeights("cuda", SEED, 40, down_fmt=5, with_shared=False)
    rng = np.random.default_rng(512)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    ids = np.argsort(-rng.uniform(-1, 1, (T, 256)), axis=1)[:, :KE].astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, KE)).astype(np.float32)
    c = _wide_lib(ref, native)
    assert ref.fl_wide_init(c, T, KE) == 1
    assert ref.refh_wide_rows(_p(x), _p(r), T) == 0
    used = sorted(set(int(e) for e in ids.reshape(-1)))
    plan = [(np.array([b[u] for u in mi], np.int32), np.array(ro, np.int32), np.array(ki, np.int32), np.array(wk, np.float32))
            for b, mi, ro, ki, wk in F.wide_slots(ids, w, KE, used, eb=16)]
    out = native.FLOut()

    def ref_pass():
        for i, (gm, rows, kidx, wk) in enumerate(plan):
            par = i & 1
            if i >= 2:
                ref.fl_wide_wait(c, par)
            ref.fl_wide_moe(c, P(W.gate), P(W.up), P(W.down), 5, 256, _p(gm), _p(rows), _p(kidx), _p(wk), len(gm), KE, par)
            ref.fl_wide_mark(c, par)
        ref.fl_wide_finish(c, T, KE, ctypes.byref(out))

    layer = M.MoeLayer(0, keep=KE, max_tokens=T, with_shared=False)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xd, rd, idd, wd = dev(x), dev(r), dev(ids), dev(w)
    h = torch.empty(T, HIDDEN, device="cuda")
    mo = torch.empty(T, HIDDEN, device="cuda")

    def our_pass():
        layer.experts(W, xd, rd, idd, wd, h=h, moe=mo)
        torch.cuda.synchronize()

    # this library's engine-facing wide pass: the same plan through fl_wide_moe / fl_wide_finish
    fc = F.FusedCtx()
    assert fc.wide_init(T, KE) == 1
    mw = native.FLMoeW(W.router_w.data_ptr(), 0, W.router_bias.data_ptr(), None, None, None, 0)
    for g0 in range(0, T, 8):
        fc.prepare(mw, x[g0:g0 + 8], r[g0:g0 + 8], wrow=g0)
    fl_out = {}

    def fl_pass():
        for i, (gm, rows, kidx, wk) in enumerate(plan):
            par = i & 1
            if i >= 2:
                fc.wide_wait(par)
            fc.wide_moe(W.gate, W.up, W.down, 256, gm, rows, kidx, wk, KE, par, down_fmt=5)
            fc.wide_mark(par)
        fl_out["h"], fl_out["moe"] = fc.wide_finish(T, KE)

    res = {}
    for name, fn in (("reference", ref_pass), ("ours", our_pass), ("ours_fl", fl_pass)):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        res[name] = (time.perf_counter() - t0) / 3 * 1e3
    layer.device_error()
    h_ref = np.ctypeslib.as_array(ctypes.cast(out.h, ctypes.POINTER(ctypes.c_float)), (T * HIDDEN,)).reshape(T, HIDDEN)
    hn = h.cpu().numpy()
    err = rel_l2(hn, h_ref)
    # both sides re-quantise h to q8 (the reference's swiglu_q8, :334-341); each against the oracle and, on
    # every row, against each other
    from moe_helpers import oracle_layer
    tok = [0, 1, 255, 511]
    o8 = oracle_layer(oracle, SEED, 40, x, r, ids, w, with_shared=False, tokens=tok, hq8=True, down_fmt=5)
    e_ours, e_ref = rel_l2(hn[tok], o8["h"]), rel_l2(h_ref[tok], o8["h"])
    e_fl = rel_l2(fl_out["h"][tok], o8["h"])
    err_fl = rel_l2(fl_out["h"], h_ref)
    assert fc.error() == 0
    fc.close()
    print("wide pass T=512, Q2_K downs: reference %.2f ms, this library %.2f ms (%.2fx), through its fl_wide_* ABI "
          "%.2f ms (%.2fx); vs the oracle: ours %.1e, fl %.1e, reference %.1e; vs the reference's wide pass (all rows): "
          "ours %.1e, fl %.1e"
          % (res["reference"], res["ours"], res["reference"] / res["ours"], res["ours_fl"], res["reference"] / res["ours_fl"],
             e_ours, e_fl, e_ref, err, err_fl))
    assert e_ours < RTOL_L2 and e_fl < RTOL_L2 and e_ref < 1e-4
    assert err < RTOL_L2 and err_fl < RTOL_L2
