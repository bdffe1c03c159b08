"""GPU parity of the real DeepSeek-R1 model's shared expert (Q5_K gate/up, Q6_K down; the reference's
mvg(F_Q5K) / mvg(F_Q6K) path, src/fused_layer.cu:521-524) through libloki_moe.so's C ABIs, against the CPU
oracle: the seeded generator bit for bit, then layer outputs within RTOL_L2 in every expert regime (the
single-token matvecs, the mma.sync path, the tcgen05 GEMMs), the one-token forward, the expert-parallel
shared stage and the fused-layer ABI (fl_moe_prepare with FL_Q5K)."""
import ctypes

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, RTOL_L2, rel_l2, oracle_layer, FMT_Q5K, FMT_Q6K

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("fmt,rows,K,m", [(FMT_Q5K, INTER, HIDDEN, 0), (FMT_Q5K, INTER, HIDDEN, 1), (FMT_Q6K, HIDDEN, INTER, 2)])
def test_shared_generator_bitexact(native, oracle, fmt, rows, K, m):
    from loki_b200 import moe as M
    nb = rows * (K // 256) * oracle.BLOCK_BYTES[fmt]
    buf = torch.empty(nb, dtype=torch.uint8, device="cuda")
    M.gen_weights(fmt, buf, SEED, 4, m, 256, 1, rows, K, nb)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(buf.cpu().numpy(), oracle.gen_kq(fmt, SEED, 4, m, 256, rows, K))


@pytest.fixture(scope="module", params=[4, 6], ids=["iq2down", "q3kdown"])
def small_layer(request, native):
    """10 routed experts (ids 0..9) and the model-format shared expert."""
    from loki_b200 import moe as M
    W = M.LayerWeights("cuda", SEED, 23, n_experts=10, down_fmt=request.param, sh_fmt=FMT_Q5K)
    torch.cuda.synchronize()
    yield request.param, W
    del W
    torch.cuda.empty_cache()


def _shared_float_ref(oracle, W, x):
    """The shared expert on fp32 x with the gguf-py-pinned dequantised weights, in float64 (the dense path's
    reference: no q8 of x or of the SwiGLU output)."""
    G = oracle.kq_dequant(FMT_Q5K, W.expert_bytes(W.n_experts, 0)).reshape(INTER, HIDDEN).astype(np.float64)
    U = oracle.kq_dequant(FMT_Q5K, W.expert_bytes(W.n_experts, 1)).reshape(INTER, HIDDEN).astype(np.float64)
    D = oracle.kq_dequant(FMT_Q6K, W.expert_bytes(W.n_experts, 2)).reshape(HIDDEN, INTER).astype(np.float64)
    g, u = x.astype(np.float64) @ G.T, x.astype(np.float64) @ U.T
    return ((g / (1.0 + np.exp(-g))) * u) @ D.T


@pytest.mark.parametrize("T,keep", [(1, 8), (1, 2), (3, 4), (8, 8), (20, 3)])
def test_shared_model_fmt_experts(native, oracle, small_layer, T, keep):
    """lk_moe_experts with the routed experts in the single-token regime and the Q5_K/Q6_K shared expert on
    its per-token q8 kernels (the dense path held off)."""
    from loki_b200 import moe as M
    fmt, W = small_layer
    rng = np.random.default_rng(T * 13 + keep + fmt)
    sel = np.stack([rng.choice(10, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = M.MoeLayer(0, keep=keep, max_tokens=T)
    layer.set_shared_gemm_threshold(1 << 20)
    h, mo = layer.experts(W, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    tok = list(range(T)) if T <= 8 else [0, 7, T - 1]
    ref = oracle_layer(oracle, SEED, 23, x, r, sel, w, tokens=tok, down_fmt=fmt, sh_fmt=FMT_Q5K)
    hn, mn = h.cpu().numpy()[tok], mo.cpu().numpy()[tok]
    e_moe, e_h = rel_l2(mn, ref["moe"]), rel_l2(hn, ref["h"])
    e_sh = rel_l2(hn - mn - r[tok], ref["h"] - ref["moe"] - r[tok])        # the shared expert's part alone
    assert e_moe < RTOL_L2 and e_h < RTOL_L2 and e_sh < RTOL_L2, (e_moe, e_h, e_sh)


@pytest.mark.parametrize("T,regime", [(64, "mma"), (256, "gemm")])
def test_shared_model_fmt_tensor_core_regimes(native, oracle, small_layer, T, regime):
    """The routed experts on the batch regimes (the q8 gate/up, then the mma.sync / tcgen05 IQ2_XXS down: the
    reference's numerics), the shared expert on its own launches."""
    from loki_b200 import moe as M
    fmt, W = small_layer
    if fmt != 4:
        pytest.skip("K-quant downs take the single-token matvecs at every T")
    keep = 4
    rng = np.random.default_rng(T + 5)
    sel = np.stack([rng.choice(10, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = M.MoeLayer(0, keep=keep, max_tokens=T)
    if regime == "mma":
        layer.set_gemm_threshold(1 << 20)
        layer.set_mma_threshold(1)
    else:
        layer.set_gemm_threshold(1)
    h, mo = layer.experts(W, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    tok = [0, 1, T // 2, T - 1]
    ref = oracle_layer(oracle, SEED, 23, x, r, sel, w, tokens=tok, hq8=True, sh_fmt=FMT_Q5K)
    hn, mn = h.cpu().numpy()[tok], mo.cpu().numpy()[tok]
    e_moe = rel_l2(mn, ref["moe"])
    # the shared expert took the dense tcgen05 path (>= 16 tokens): against the reference's q8 numerics
    e_sh = rel_l2(hn - mn - r[tok], ref["h"] - ref["moe"] - r[tok])
    assert e_moe < RTOL_L2 and e_sh < RTOL_L2, (e_moe, e_sh)


@pytest.mark.parametrize("T", [16, 40, 600])
def test_shared_model_fmt_dense_path(native, oracle, small_layer, T):
    """Calls of >= 16 tokens: the Q5_K/Q6_K shared expert dequantised to fp16 once and run as two tcgen05 GEMMs
    (shared_gemm.cu: q8 of x and of h as fp16 operands, fp32 accumulation; 64-token tiles, and 128-token tiles
    from 513 tokens), the routed experts on their usual regime; twice, the second call reusing the buffers.
    The shared part within RTOL_L2 of the reference's q8 numerics; its distance from float64 with unquantised
    x and h is printed for scale."""
    from loki_b200 import moe as M
    fmt, W = small_layer
    keep = 2
    rng = np.random.default_rng(T * 3 + fmt)
    sel = np.stack([rng.choice(10, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = M.MoeLayer(0, keep=keep, max_tokens=T)
    layer.set_mma_threshold(1 << 20)
    for _ in range(2):
        h, mo = layer.experts(W, _dev(x), _dev(r), _dev(sel), _dev(w))
        layer.device_error()
    tok = [0, T // 3, 127, T - 1] if T > 128 else [0, T // 3, T - 1]
    ref = oracle_layer(oracle, SEED, 23, x, r, sel, w, tokens=tok, down_fmt=fmt, sh_fmt=FMT_Q5K)
    hn, mn = h.cpu().numpy()[tok], mo.cpu().numpy()[tok]
    e_moe = rel_l2(mn, ref["moe"])
    e_sh = rel_l2(hn - mn - r[tok], ref["h"] - ref["moe"] - r[tok])
    e_f64 = rel_l2(hn - mn - r[tok], _shared_float_ref(oracle, W, x[tok]))   # unquantised x and h, for scale
    print("\n[shared dense T=%d] vs reference q8 numerics %.3e, vs float64 %.3e" % (T, e_sh, e_f64))
    assert e_moe < RTOL_L2 and e_sh < RTOL_L2, (e_moe, e_sh, e_f64)


def test_shared_model_fmt_forward_T1(native, oracle):
    """The real model's layer formats end to end at T=1: grouped routing, IQ2_XXS gate/up, Q2_K downs, the
    Q5_K/Q6_K shared expert reading the router's q8 of x."""
    from loki_b200 import moe as M
    W = M.LayerWeights("cuda", SEED, 8, down_fmt=5, sh_fmt=FMT_Q5K)
    try:
        rng = np.random.default_rng(81)
        x = rng.standard_normal((1, HIDDEN)).astype(np.float32)
        r = rng.standard_normal((1, HIDDEN)).astype(np.float32)
        layer = M.MoeLayer(0, keep=8, n_group=8, topk_group=4, max_tokens=1)
        h, mo, sel, w = layer.forward(W, _dev(x), _dev(r))
        layer.device_error()
        sel, w = sel.cpu().numpy(), w.cpu().numpy()
        _, osel, ow = oracle.router(x, W.router_w.float().cpu().numpy(), W.router_bias.cpu().numpy(), oracle.route_cfg(8, 8, 1, 8, 4))
        np.testing.assert_array_equal(sel, osel)
        np.testing.assert_array_equal(w, ow)
        ref = oracle_layer(oracle, SEED, 8, x, r, sel, w, down_fmt=5, sh_fmt=FMT_Q5K)
        assert rel_l2(mo.cpu().numpy(), ref["moe"]) < RTOL_L2
        assert rel_l2(h.cpu().numpy(), ref["h"]) < RTOL_L2
    finally:
        del W
        torch.cuda.empty_cache()


def test_shared_model_fmt_ep_shared(native, oracle, small_layer):
    """lk_ep_shared (the expert-parallel home rank's shared stage) with the model-format shared expert:
    h_partial = resid + shared."""
    from loki_b200 import moe as M
    fmt, W = small_layer
    T = 5
    rng = np.random.default_rng(55)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = M.MoeLayer(0, keep=2, max_tokens=T)
    hp = torch.empty(T, HIDDEN, device="cuda")
    ws = W.struct()
    xd, rd = _dev(x), _dev(r)
    rc = native.lib().lk_ep_shared(layer.ctx, ctypes.byref(ws), ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(rd.data_ptr()), T,
                                   ctypes.c_void_p(hp.data_ptr()), None)
    assert rc == 0
    layer.device_error()
    sel = np.zeros((T, 1), np.int32)
    ref = oracle_layer(oracle, SEED, 23, x, r, sel, np.zeros((T, 1), np.float32), down_fmt=fmt, sh_fmt=FMT_Q5K)
    assert rel_l2(hp.cpu().numpy(), ref["h"]) < RTOL_L2


@pytest.fixture(scope="module")
def model_layer(native):
    """A 256-expert layer in the real model's formats (Q2_K downs, Q5_K/Q6_K shared expert)."""
    from loki_b200 import moe as M
    W = M.LayerWeights("cuda", SEED, 6, down_fmt=5, sh_fmt=FMT_Q5K)
    torch.cuda.synchronize()
    yield W
    del W
    torch.cuda.empty_cache()


def _mw(native, W):
    return native.FLMoeW(W.router_w.data_ptr(), 0, W.router_bias.data_ptr(), W.sh_gate, W.sh_up, W.sh_down, FMT_Q5K)


@pytest.mark.parametrize("n,KE,auto", [(1, 8, False), (5, 4, False), (1, 8, True), (8, 8, True)])
def test_fl_shared_model_fmt(native, oracle, model_layer, n, KE, auto):
    """fl_moe_prepare with FL_Q5K, then fl_moe (host keep pass) or fl_moe_auto (keep on the device), twice so
    the second call replays the captured CUDA graph."""
    from loki_b200 import fused as F
    W = model_layer
    rng = np.random.default_rng(n * 7 + KE)
    x = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((n, HIDDEN)).astype(np.float32)
    fc = F.FusedCtx()
    try:
        for _ in range(2):
            fc.prepare(_mw(native, W), x, r)
            got = fc.fetch(n, 1)
            ids, w = F.keep_pass(got["sel"], got["wts"], KE)
            if auto:
                h, mo = fc.moe_auto(W.gate, W.up, W.down, n, KE, down_fmt=5)
            else:
                h, mo = fc.moe(W.gate, W.up, W.down, 256, ids, w, down_fmt=5)
            assert fc.error() == 0
            ref = oracle_layer(oracle, SEED, 6, x, r, ids, w, down_fmt=5, sh_fmt=FMT_Q5K)
            assert rel_l2(mo, ref["moe"]) < RTOL_L2
            assert rel_l2(h, ref["h"]) < RTOL_L2
    finally:
        fc.close()


def test_gguf_layer_model_shared(native, oracle, tmp_path):
    """A GGUF file in the real model's tensor types (IQ2_XXS gate/up, Q3_K down, Q5_K/Q6_K shared expert)
    loads into resident arenas and runs the expert stage like the seeded layer."""
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as QT
    from loki_b200 import moe as M
    from loki_b200.gguf_experts import GgufLayer
    NE = 2
    path = str(tmp_path / "model.gguf")
    wr = gguf.GGUFWriter(path, "deepseek2")
    gate = np.concatenate([oracle.gen_iq2(SEED, 0, 0, e, INTER, HIDDEN) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 0, 1, e, INTER, HIDDEN) for e in range(NE)])
    down = np.concatenate([oracle.gen_kq(6, SEED, 0, 2, e, HIDDEN, INTER) for e in range(NE)])
    shg, shu = oracle.gen_kq(FMT_Q5K, SEED, 0, 0, 256, INTER, HIDDEN), oracle.gen_kq(FMT_Q5K, SEED, 0, 1, 256, INTER, HIDDEN)
    shd = oracle.gen_kq(FMT_Q6K, SEED, 0, 2, 256, HIDDEN, INTER)
    wr.add_tensor("blk.0.ffn_gate_exps.weight", gate.reshape(NE, INTER, -1), raw_shape=[NE, INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
    wr.add_tensor("blk.0.ffn_up_exps.weight", up.reshape(NE, INTER, -1), raw_shape=[NE, INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
    wr.add_tensor("blk.0.ffn_down_exps.weight", down.reshape(NE, HIDDEN, -1), raw_shape=[NE, HIDDEN, 8 * 110], raw_dtype=QT.Q3_K)
    wr.add_tensor("blk.0.ffn_gate_shexp.weight", shg.reshape(INTER, -1), raw_shape=[INTER, 28 * 176], raw_dtype=QT.Q5_K)
    wr.add_tensor("blk.0.ffn_up_shexp.weight", shu.reshape(INTER, -1), raw_shape=[INTER, 28 * 176], raw_dtype=QT.Q5_K)
    wr.add_tensor("blk.0.ffn_down_shexp.weight", shd.reshape(HIDDEN, -1), raw_shape=[HIDDEN, 8 * 210], raw_dtype=QT.Q6_K)
    wr.add_tensor("blk.0.ffn_gate_inp.weight", np.zeros((256, HIDDEN), np.float32))
    wr.add_tensor("blk.0.exp_probs_b.bias", np.zeros(256, np.float32))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    L = GgufLayer(path, 0)
    assert L.with_shared and L.sh_fmt == FMT_Q5K and L.down_fmt == 6
    rng = np.random.default_rng(4)
    T, keep = 2, 2
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    sel = np.array([[0, 1], [1, 0]], np.int32)
    w = rng.uniform(0.1, 1.0, (T, keep)).astype(np.float32)
    ctx = M.MoeLayer(0, topk=keep, keep=keep, max_tokens=T, n_experts=NE)
    h, mo = ctx.experts(L, _dev(x), _dev(r), _dev(sel), _dev(w))
    ctx.device_error()
    ref = oracle.moe_layer(x, r, gate, up, down, 28 * 66 * INTER, sel, w, shg, shu, shd, down_fmt=6, down_stride=HIDDEN * 8 * 110,
                           sh_gu_fmt=FMT_Q5K, sh_down_fmt=FMT_Q6K)
    assert rel_l2(mo.cpu().numpy(), ref["moe"]) < RTOL_L2 and rel_l2(h.cpu().numpy(), ref["h"]) < RTOL_L2
