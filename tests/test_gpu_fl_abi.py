"""GPU parity of the engine-facing fused-layer ABI (include/loki_fused_moe.h), driven the way
src/server_core_fused.cpp drives src/fused_layer.h: fl_moe_prepare -> fl_fetch -> host keep pass ->
fl_moe (narrow, n <= 8 rows), and fl_moe_prepare(wrow) per group -> fl_wide_moe per arena batch ->
fl_wide_finish (wide pass; its routed products on the mma.sync path).  Host buffers in and out; every down format the ABI accepts."""
import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, RTOL_L2, rel_l2, oracle_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[4, 5, 6], ids=["iq2", "q2k", "q3k"])
def fl_layer(request, native):
    from loki_b200 import moe as M
    fmt = request.param
    W = M.LayerWeights("cuda", SEED, 5, down_fmt=fmt)
    torch.cuda.synchronize()
    yield fmt, W
    del W
    torch.cuda.empty_cache()


def _mw(native, W, fmt):
    # fl_moe_prepare's shared expert is IQ2_XXS: with K-quant layers the test runs without it
    sh = (W.sh_gate, W.sh_up, W.sh_down) if fmt == 4 else (None, None, None)
    return native.FLMoeW(W.router_w.data_ptr(), 0, W.router_bias.data_ptr(), *sh)


@pytest.mark.parametrize("n,KE,share", [(1, 8, False), (3, 2, False), (8, 8, False), (8, 3, True)])
def test_fl_narrow(native, oracle, fl_layer, n, KE, share):
    from loki_b200 import fused as F
    fmt, W = fl_layer
    rng = np.random.default_rng(n * 10 + KE)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        fc.prepare(_mw(native, W, fmt), x, r)
        got = fc.fetch(n, 1)
        _, osel, ow = oracle.router(x, W.router_w.float().cpu().numpy(), W.router_bias.cpu().numpy(),
                                    oracle.route_cfg(8, 8, 0))
        np.testing.assert_array_equal(got["sel"], osel)
        np.testing.assert_array_equal(got["wts"], ow)
        ids, w = F.keep_pass(got["sel"], got["wts"], KE, share=share)
        h, mo = fc.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=fmt)
        assert fc.error() == 0
        ref = oracle_layer(oracle, SEED, 5, x, r, ids, w, with_shared=fmt == 4, down_fmt=fmt)
        assert rel_l2(mo, ref["moe"]) < RTOL_L2
        assert rel_l2(h, ref["h"]) < RTOL_L2
    finally:
        fc.close()


def test_fl_wide(native, oracle, fl_layer):
    from loki_b200 import fused as F
    fmt, W = fl_layer
    n, KE = 20, 4
    rng = np.random.default_rng(2020 + fmt)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        assert fc.wide_init(32, KE) == 1
        sel = np.empty((n, 8), np.int32)
        wts = np.empty((n, 8), np.float32)
        for g0 in range(0, n, 8):
            g1 = min(n, g0 + 8)
            fc.prepare(_mw(native, W, fmt), x[g0:g1], r[g0:g1], wrow=g0)
            got = fc.fetch(g1 - g0, 1)
            sel[g0:g1], wts[g0:g1] = got["sel"], got["wts"]
        ids, w = F.keep_pass(sel, wts, KE)
        used = sorted(set(int(e) for e in ids.reshape(-1)))
        for i, (batch, midx, rows, kidx, wk) in enumerate(F.wide_slots(ids, w, KE, used, eb=4)):
            par = i & 1
            if i >= 2:
                fc.wide_wait(par)                     # the engine's order: this parity's tables are free again
            gmidx = [batch[u] for u in midx]          # resident arenas: global expert ids
            fc.wide_moe(W.gate, W.up, W.down, 256, gmidx, rows, kidx, wk, KE, par, down_fmt=fmt)
            fc.wide_mark(par)
        h, mo = fc.wide_finish(n, KE)
        assert fc.error() == 0
        # routed products and the shared expert of fl_moe_prepare both with the reference's numerics (q8 x and h)
        ref = oracle_layer(oracle, SEED, 5, x, r, ids, w, with_shared=fmt == 4, down_fmt=fmt)
        assert rel_l2(mo, ref["moe"]) < RTOL_L2
        assert rel_l2(h, ref["h"]) < RTOL_L2
    finally:
        fc.close()


def test_fl_replay_decode(native, oracle, fl_layer):
    """The C++ engine replay (lkr_decode) over two layers: the last layer's h equals the oracle's."""
    from loki_b200 import fused as F
    fmt, W = fl_layer
    if fmt != 4:
        pytest.skip("the replay drives fl_moe_prepare's IQ2_XXS shared expert")
    rng = np.random.default_rng(31)
    x = rng.standard_normal((2, 1, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((2, 1, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        sec, h = F.replay_decode(fc, [W, W], x, r, 8, 1, 2, down_fmt=fmt)
        assert sec > 0 and fc.error() == 0
    finally:
        fc.close()
    _, osel, ow = oracle.router(x[1], W.router_w.float().cpu().numpy(), W.router_bias.cpu().numpy(), oracle.route_cfg(8, 8, 0))
    ref = oracle_layer(oracle, SEED, 5, x[1], r[1], osel, ow, down_fmt=fmt)
    assert rel_l2(h, ref["h"]) < RTOL_L2


@pytest.mark.parametrize("n,KE", [(1, 8), (3, 2), (8, 3)])
def test_fl_moe_auto_equals_host_keep_path(native, oracle, fl_layer, n, KE):
    """fl_moe_auto (routing post-pass on the device) gives exactly the outputs of fl_fetch + host keep pass +
    fl_moe, and fl_moe_outs sees its routing."""
    from loki_b200 import fused as F
    fmt, W = fl_layer
    rng = np.random.default_rng(700 + n * 10 + KE)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        fc.prepare(_mw(native, W, fmt), x, r)
        got = fc.fetch(n, 1)
        ids, w = F.keep_pass(got["sel"], got["wts"], KE)
        h1, m1 = [a.copy() for a in fc.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=fmt)]
        outs1 = fc.moe_outs(0, ids[0], w[0]).copy()
        fc.prepare(_mw(native, W, fmt), x, r)
        h2, m2 = [a.copy() for a in fc.moe_auto(W.gate, W.up, W.down, n, KE, down_fmt=fmt)]
        outs2 = fc.moe_outs(0, ids[0], w[0])
        assert fc.error() == 0
        np.testing.assert_array_equal(h1, h2)
        np.testing.assert_array_equal(m1, m2)
        np.testing.assert_array_equal(outs1, outs2)
    finally:
        fc.close()


def test_fl_replay_decode_device_keep(native, oracle, fl_layer):
    """The C++ replay through fl_moe_auto: the last layer's h equals the oracle's (keep 2 of 8, renormalised)."""
    from loki_b200 import fused as F
    fmt, W = fl_layer
    if fmt != 4:
        pytest.skip("the replay drives fl_moe_prepare's IQ2_XXS shared expert")
    rng = np.random.default_rng(32)
    x = rng.standard_normal((2, 1, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((2, 1, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        sec, h = F.replay_decode(fc, [W, W], x, r, 2, 1, 2, down_fmt=fmt, device_keep=True)
        assert sec > 0 and fc.error() == 0
    finally:
        fc.close()
    _, osel, ow = oracle.router(x[1], W.router_w.float().cpu().numpy(), W.router_bias.cpu().numpy(), oracle.route_cfg(8, 2, 1))
    ref = oracle_layer(oracle, SEED, 5, x[1], r[1], osel, ow, down_fmt=fmt)
    assert rel_l2(h, ref["h"]) < RTOL_L2


@pytest.mark.parametrize("device_keep", [False, True])
def test_fl_graphs_match_direct_launches(native, fl_layer, device_keep):
    """Repeated call shapes replay captured CUDA graphs: the same h as issuing every launch directly."""
    from loki_b200 import fused as F
    fmt, W = fl_layer
    if fmt != 4:
        pytest.skip("the replay drives fl_moe_prepare's IQ2_XXS shared expert")
    rng = np.random.default_rng(33)
    x = rng.standard_normal((3, 2, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((3, 2, HIDDEN)).astype(np.float32)
    hs = []
    for graphs in (False, True):
        fc = F.FusedCtx()
        try:
            fc.use_graphs(graphs)
            _, h = F.replay_decode(fc, [W, W, W], x, r, 4, 2, 3, device_keep=device_keep)   # shapes repeat
            assert fc.error() == 0
            hs.append(h)
        finally:
            fc.close()
    np.testing.assert_array_equal(hs[0], hs[1])


def oracle_layer_slots(oracle, x, r, ids, w, fmt):
    """The oracle layer with its per-entry pushes (y_slot [T][KE][7168]) and shared-expert output."""
    from moe_helpers import host_arena, down_bytes, shared_fmts, MAT
    used = sorted(set(int(e) for e in ids.reshape(-1)))
    remap = {e: i for i, e in enumerate(used)}
    cids = np.vectorize(lambda e: remap[int(e)])(ids).astype(np.int32)
    gate, up, down, sh = host_arena(oracle, SEED, 5, used, fmt, 4)
    shg, shu, shd = sh if fmt == 4 else (None, None, None)
    gf, df = shared_fmts(fmt, 4)
    return oracle.moe_layer(x, r, gate, up, down, MAT, cids, w, shg, shu, shd, want_slots=True, down_fmt=fmt,
                            down_stride=down_bytes(fmt), sh_gu_fmt=gf, sh_down_fmt=df)


def test_fl_attribution_and_skip_vs_oracle(native, oracle, fl_layer):
    """fl_moe_outs (narrow pass) and fl_wide_outs (wide pass) return each row's weighted expert pushes -- the
    reference's out_all rows (src/fused_layer.cu:569-576) -- and fl_skip / fl_wide_skip add a stored output to the
    shared expert and residual (:562-566, :613-618); all against the oracle's per-entry outputs."""
    from loki_b200 import fused as F
    fmt, W = fl_layer
    n, KE = 6, 4
    rng = np.random.default_rng(77 + fmt)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    mo_stored = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        assert fc.wide_init(8, KE) == 1
        fc.prepare(_mw(native, W, fmt), x, r)
        got = fc.fetch(n, 1)
        ids, w = F.keep_pass(got["sel"], got["wts"], KE)
        fc.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=fmt)
        ref = oracle_layer_slots(oracle, x, r, ids, w, fmt)
        for b in range(n):
            pushes = fc.moe_outs(b, ids[b], w[b])
            assert rel_l2(pushes, ref["y_slot"][b]) < RTOL_L2, b
        # fl_skip: h = stored output + shared expert + residual of the last prepare's rows
        h = fc.skip(mo_stored)
        want = mo_stored + r + (ref["shared"] if fmt == 4 else 0.0)
        assert rel_l2(h, want) < RTOL_L2
        # the same rows as a wide pass (one group), then its attribution and the wide skip
        fc.prepare(_mw(native, W, fmt), x, r, wrow=0)
        used = sorted(set(int(e) for e in ids.reshape(-1)))
        for i, (batch, midx, rows, kidx, wk) in enumerate(F.wide_slots(ids, w, KE, used, eb=4)):
            par = i & 1
            if i >= 2:
                fc.wide_wait(par)
            fc.wide_moe(W.gate, W.up, W.down, 256, [batch[u] for u in midx], rows, kidx, wk, KE, par, down_fmt=fmt)
            fc.wide_mark(par)
        hw, mw_ = fc.wide_finish(n, KE)
        assert rel_l2(mw_, ref["moe"]) < RTOL_L2
        for row in range(n):
            assert rel_l2(fc.wide_outs(row, KE), ref["y_slot"][row]) < RTOL_L2, row
        hs = fc.wide_skip(mo_stored)
        assert rel_l2(hs, mo_stored + r + (ref["shared"] if fmt == 4 else 0.0)) < RTOL_L2
        assert fc.error() == 0
    finally:
        fc.close()


def test_adopt_matches_prepare(native, oracle, fl_layer):
    """The bridge's hand-off (libloki_fused.so): a context on a given stream that adopts ncur, ffn_inp, the router's
    top-8 and the shared expert's output as two partial sums [2][8 rows][7168] (the layout the reference's fl_attn
    leaves, src/fused_layer.cu:521-525) gives the narrow pass's h / moe of a context that ran fl_moe_prepare on
    the same rows; lkfl_device_h holds the h rows the bridge hands to the next layer's attention."""
    import ctypes
    from loki_b200 import fused as F
    fmt, W = fl_layer
    n, KE = 5, 8
    rng = np.random.default_rng(99 + fmt)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fa = F.FusedCtx()
    stream = torch.cuda.Stream()
    fb = F.FusedCtx(stream=stream.cuda_stream)
    try:
        fa.prepare(_mw(native, W, fmt), x, r)
        got = fa.fetch(n, 1)
        ids, w = F.keep_pass(got["sel"], got["wts"], KE)
        h1, mo1 = [a.copy() for a in fa.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=fmt)]
        shared = (h1 - mo1 - r).astype(np.float32)
        parts = np.zeros((2, 8, HIDDEN), np.float32)
        parts[0, :n] = shared * np.float32(0.5)
        parts[1, :n] = shared - parts[0, :n]
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        xd, rd, pd, sd, wd = dev(x), dev(r), dev(parts), dev(got["sel"]), dev(got["wts"])
        torch.cuda.synchronize()
        fb.adopt(xd.data_ptr(), rd.data_ptr(), pd.data_ptr(), 2, 8, sd.data_ptr(), wd.data_ptr(), n)
        h2, mo2 = fb.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=fmt)
        assert fa.error() == 0 and fb.error() == 0
        assert rel_l2(mo2, mo1) < 1e-6 and rel_l2(h2, h1) < 1e-6
        hdev = np.empty((n, HIDDEN), np.float32)
        cu = ctypes.CDLL("libcuda.so.1")                   # the driver's copy, on the context torch made current
        cu.cuMemcpyDtoH_v2.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t]
        assert cu.cuMemcpyDtoH_v2(hdev.ctypes.data, fb.device_h(), n * HIDDEN * 4) == 0
        assert np.array_equal(hdev, h2)
    finally:
        fa.close()
        fb.close()
