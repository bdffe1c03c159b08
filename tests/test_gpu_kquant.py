"""GPU parity of the K-quant down projections (Q2_K, Q3_K: the real DeepSeek-R1 model's down formats,
the reference's tc_matvec<F_Q2K / F_Q3K>) through libloki_moe.so's C ABI, against the CPU oracle.

Bit-exact: the seeded K-quant generator.  Layer outputs: relative L2 <= RTOL_L2 of the oracle with the
same q8 scheme (the K-quant path keeps the reference's q8 SwiGLU output at every T)."""
import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, MAT, RTOL_L2, rel_l2, oracle_layer, down_bytes

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

KQ = [5, 6]                          # FMT_Q2K, FMT_Q3K


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt", KQ)
@pytest.mark.parametrize("key", [(0, 2, 0), (9, 2, 255), (57, 2, 256)])
def test_kq_generator_bitexact(native, oracle, fmt, key):
    from loki_b200 import moe as M
    layer, m, e = key
    DS = down_bytes(fmt)
    buf = torch.empty(DS, dtype=torch.uint8, device="cuda")
    M.gen_weights(fmt, buf, SEED, layer, m, e, 1, HIDDEN, INTER, DS)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(buf.cpu().numpy(), oracle.gen_kq(fmt, SEED, layer, m, e, HIDDEN, INTER))


def _small_arena(native, M, fmt, NE, layer_id, with_shared=True):
    DS = down_bytes(fmt)
    nb = 2 * NE * MAT + NE * DS + (2 * MAT + DS if with_shared else 0)
    buf = torch.empty(nb, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    g, u, d = base, base + NE * MAT, base + 2 * NE * MAT
    M.gen_iq2(g, SEED, layer_id, 0, 0, NE, INTER, HIDDEN, MAT)
    M.gen_iq2(u, SEED, layer_id, 1, 0, NE, INTER, HIDDEN, MAT)
    M.gen_weights(fmt, d, SEED, layer_id, 2, 0, NE, HIDDEN, INTER, DS)
    sg = su = sd = None
    if with_shared:
        sg = base + 2 * NE * MAT + NE * DS
        su, sd = sg + MAT, sg + 2 * MAT
        M.gen_iq2(sg, SEED, layer_id, 0, 256, 1, INTER, HIDDEN, MAT)
        M.gen_iq2(su, SEED, layer_id, 1, 256, 1, INTER, HIDDEN, MAT)
        M.gen_weights(fmt, sd, SEED, layer_id, 2, 256, 1, HIDDEN, INTER, DS)
    ws = native.LkMoeWeights(g, u, d, MAT, MAT, DS, fmt, sg, su, sd, None, 0, None)
    return buf, ws


@pytest.mark.parametrize("fmt", KQ)
@pytest.mark.parametrize("T,keep", [(1, 8), (1, 2), (3, 4), (8, 8), (47, 2), (64, 2), (200, 8)])
def test_kq_experts_small_arena(native, oracle, fmt, T, keep):
    """lk_moe_experts with K-quant downs: the single-token q8 matvecs below the mma threshold (48), from there
    the q8 gate/up on tcgen05 (h re-quantised to q8) and kq_mma.cu's Q2_K/Q3_K down; both against the oracle
    with the reference's numerics."""
    from loki_b200 import moe as M
    NE, layer_id = 10, 21
    buf, ws = _small_arena(native, M, fmt, NE, layer_id)
    rng = np.random.default_rng(T * 31 + keep + fmt)
    sel = np.stack([rng.choice(NE, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = M.MoeLayer(0, keep=keep, max_tokens=T)
    h, mo = layer.experts(ws, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    tok = list(range(T)) if T <= 8 else [0, 1, T // 2, T - 1]
    ref = oracle_layer(oracle, SEED, layer_id, x, r, sel, w, tokens=tok, down_fmt=fmt, hq8=True)
    e_moe, e_h = rel_l2(mo.cpu().numpy()[tok], ref["moe"]), rel_l2(h.cpu().numpy()[tok], ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)
    del buf


@pytest.mark.parametrize("fmt", KQ)
def test_kq_layer_forward_T1(native, oracle, fmt):
    """The one-token forward (router-written slots, router-quantised x) with a 256-expert K-quant layer."""
    from loki_b200 import moe as M
    W = M.LayerWeights("cuda", SEED, 3, down_fmt=fmt)
    try:
        rng = np.random.default_rng(fmt)
        x = rng.standard_normal((1, HIDDEN)).astype(np.float32)
        r = rng.standard_normal((1, HIDDEN)).astype(np.float32)
        layer = M.MoeLayer(0, keep=8, n_group=8, topk_group=4, max_tokens=1)
        h, mo, sel, w = layer.forward(W, _dev(x), _dev(r))
        layer.device_error()
        sel, w = sel.cpu().numpy(), w.cpu().numpy()
        _, osel, ow = oracle.router(x, W.router_w.float().cpu().numpy(), W.router_bias.cpu().numpy(),
                                    oracle.route_cfg(8, 8, 1, 8, 4))
        np.testing.assert_array_equal(sel, osel)
        np.testing.assert_array_equal(w, ow)
        ref = oracle_layer(oracle, SEED, 3, x, r, sel, w, down_fmt=fmt)
        assert rel_l2(mo.cpu().numpy(), ref["moe"]) < RTOL_L2
        assert rel_l2(h.cpu().numpy(), ref["h"]) < RTOL_L2
    finally:
        del W
        torch.cuda.empty_cache()
