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
