"""CPU tests of the oracle (the checker): pinned against gguf-py's IQ2_XXS decode, the committed golden
fixtures, and pure-Python restatements of the reference's routing semantics."""
import math
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SEED = 0x10C1


def test_iq2_dequant_matches_gguf_fixture(oracle):
    f = np.load(os.path.join(GOLD, "iq2_xxs_gguf.npz"))
    out = oracle.iq2_dequant(f["blocks"])
    np.testing.assert_array_equal(out, f["dequant"])


def test_iq2_dequant_matches_gguf_live(oracle):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    blk = oracle.gen_iq2(SEED, 5, 2, 200, 16, 2048)
    np.testing.assert_array_equal(oracle.iq2_dequant(blk), dequantize(blk, gguf.GGMLQuantizationType.IQ2_XXS).reshape(-1))


def test_grid_table_matches_gguf():
    pytest.importorskip("gguf")
    from loki_b200.csrc.gen_iq2_tables import iq2xxs_grid_u64
    path = os.path.join(os.path.dirname(GOLD), "..", "loki_b200", "csrc", "iq2_grid.inc")
    txt = open(path).read()
    vals = [int(t[:-3], 16) for t in txt.replace(",", " ").split() if t.startswith("0x")]
    assert vals == iq2xxs_grid_u64()


def test_generator_kat(oracle):
    f = np.load(os.path.join(GOLD, "generator_kat.npz"))
    for (l, m, e), ref in zip(f["keys"], f["bytes"]):
        np.testing.assert_array_equal(oracle.gen_iq2(SEED, int(l), int(m), int(e), 2, 7168)[: 2 * 66], ref)


def test_generator_distribution(oracle):
    blk = oracle.gen_iq2(SEED, 1, 0, 0, 2048, 7168).reshape(-1, 66)
    d = blk[:, :2].copy().view(np.float16).astype(np.float64).ravel()
    assert (d >= 0).all()
    assert abs(d.mean() - 0.7979e-3) < 0.02e-3          # E|N(0,1)| * 1e-3
    qs = blk[:, 2:].reshape(-1, 8)
    scales = (qs[:, 4:8].copy().view(np.uint32).ravel() >> 28)
    counts = np.bincount(scales, minlength=16)
    assert counts.min() > 0.9 * counts.mean()


def test_expf_accuracy(oracle):
    xs = np.linspace(-85.0, 87.0, 20011).astype(np.float32)
    worst = 0.0
    for v in xs:
        r = oracle.lib().orc_expf(float(v))
        worst = max(worst, abs(r / math.exp(float(v)) - 1.0))
    assert worst < 2.5e-7                                 # ~2 ulp


def test_fp16_conversion(oracle):
    rng = np.random.default_rng(3)
    v = (rng.standard_normal(4000) * 10.0 ** rng.integers(-9, 6, 4000)).astype(np.float32)
    v = np.concatenate([v, np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 6e-8, 2.9802322e-08, -1e-10], np.float32)])
    mine = np.array([oracle.lib().orc_f2h(float(a)) for a in v], np.uint16)
    with np.errstate(over="ignore"):
        ref = v.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(mine, ref)


def test_quant_q8(oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(7168).astype(np.float32)
    x[:32] = 0.0
    q, d = oracle.quant_q8(x)
    assert d[0] == 0.0 and (q[:32] == 0).all()
    g = x.reshape(-1, 32)
    dd = (np.abs(g).max(1) / np.float32(127.0)).astype(np.float32)
    np.testing.assert_array_equal(d, dd)
    idv = np.where(dd > 0, np.float32(1.0) / np.maximum(dd, np.float32(1e-30)), 0).astype(np.float32)
    qq = np.rint((g * idv[:, None]).astype(np.float32)).astype(np.int8)
    np.testing.assert_array_equal(q.reshape(-1, 32), qq)


# ---------------------------------------------------------------- routing semantics
def py_route(p, bias, topk=8, keep=8, renorm=True, n_group=1, topk_group=1, scale=2.5):
    """Pure-Python restatement: reference router_topk (fused_layer.cu:323-332), grouped mode, and the
    engine's keep-KE pass (server_core_fused.cpp:793-813), in float32 arithmetic."""
    f = np.float32
    sc = [f(p[e]) + f(bias[e]) for e in range(len(p))]
    allowed = [True] * len(p)
    if n_group > 1:
        gs = len(p) // n_group
        gsc = []
        for g in range(n_group):
            vals = sorted(((sc[e], e) for e in range(g * gs, (g + 1) * gs)), key=lambda t: (-t[0], t[1]))
            gsc.append(f(vals[0][0]) + f(vals[1][0]))
        order = sorted(range(n_group), key=lambda g: (-gsc[g], g))[:topk_group]
        allowed = [(e // gs) in order for e in range(len(p))]
    cand = sorted((e for e in range(len(p)) if allowed[e]), key=lambda e: (-sc[e], e))[:topk]
    s = f(0.0)
    for e in cand:
        s = f(s + f(p[e]))
    s = max(s, f(6.103515625e-5))
    w = [f(f(f(p[e]) / s) * f(scale)) for e in cand]
    if keep >= topk:
        return cand, w
    order = sorted(range(topk), key=lambda k: -w[k])       # stable: ties keep position order
    kept = [cand[k] for k in order[:keep]]
    kw = [w[k] for k in order[:keep]]
    sw = f(0.0)
    for v in kw:
        sw = f(sw + v)
    if renorm and sw > 1e-6:
        fac = f(f(scale) / sw)
        kw = [f(v * fac) for v in kw]
    return kept, kw


@pytest.mark.parametrize("mode", [dict(keep=8), dict(keep=2), dict(keep=2, renorm=False), dict(keep=8, n_group=8, topk_group=4),
                                  dict(keep=2, n_group=8, topk_group=4)])
def test_router_matches_python_restatement(oracle, mode):
    rng = np.random.default_rng(11)
    T = 6
    logits = rng.uniform(-1, 1, (T, 256)).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    cfg = oracle.route_cfg(8, mode.get("keep", 8), int(mode.get("renorm", True)), mode.get("n_group", 1), mode.get("topk_group", 1))
    probs, sel, w = oracle.router(None, None, bias, cfg, logits=logits)
    for t in range(T):
        s, ww = py_route(probs[t], bias, keep=cfg.keep, renorm=bool(cfg.renorm), n_group=cfg.n_group, topk_group=cfg.topk_group)
        assert list(sel[t]) == s
        np.testing.assert_array_equal(w[t], np.array(ww, np.float32))


def test_router_ties_go_to_lower_id(oracle):
    logits = np.zeros((1, 256), np.float32)
    logits[0, [200, 3, 100, 50, 7, 9, 250, 1, 2]] = 1.0    # nine equal maxima: the eight lowest ids win
    bias = np.zeros(256, np.float32)
    _, sel, w = oracle.router(None, None, bias, oracle.route_cfg(8, 8), logits=logits)
    assert list(sel[0]) == [1, 2, 3, 7, 9, 50, 100, 200]
    assert np.allclose(w[0], 2.5 / 8)


def test_router_logits_order_close_to_float64(oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 7168)).astype(np.float32)
    W = (rng.standard_normal((256, 7168)) * 0.02).astype(np.float32)
    lg = oracle.router_logits(x, W)
    ref = x.astype(np.float64) @ W.astype(np.float64).T
    assert np.abs(lg - ref).max() < 1e-4


def test_router_kat(oracle):
    f = np.load(os.path.join(GOLD, "router_kat.npz"))
    rng = np.random.default_rng(2024)
    x = rng.standard_normal((5, 7168)).astype(np.float32)
    W = (rng.standard_normal((256, 7168)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    p8, s8, w8 = oracle.router(x, W, bias, oracle.route_cfg(8, 8))
    np.testing.assert_array_equal(p8, f["probs"])
    np.testing.assert_array_equal(s8, f["sel8"]); np.testing.assert_array_equal(w8, f["w8"])
    _, s2, w2 = oracle.router(x, W, bias, oracle.route_cfg(8, 2))
    np.testing.assert_array_equal(s2, f["sel2"]); np.testing.assert_array_equal(w2, f["w2"])
    _, sg, wg = oracle.router(x, W, bias, oracle.route_cfg(8, 8, n_group=8, topk_group=4))
    np.testing.assert_array_equal(sg, f["selg"]); np.testing.assert_array_equal(wg, f["wg"])


def test_permute_stable(oracle):
    rng = np.random.default_rng(6)
    sel = rng.integers(0, 256, (300, 8)).astype(np.int32)
    counts, offsets, perm = oracle.permute(sel)
    assert counts.sum() == sel.size and offsets[-1] == sel.size
    flat = sel.reshape(-1)
    for e in range(256):
        seg = perm[offsets[e]:offsets[e + 1]]
        assert (flat[seg] == e).all()
        assert (np.diff(seg) > 0).all()                     # stable by (t, k)


# ---------------------------------------------------------------- expert products
def _q8_dequant(oracle, x):
    q, d = oracle.quant_q8(x)
    return (q.reshape(-1, 32).astype(np.float64) * d[:, None].astype(np.float64)).reshape(-1)


def test_iq2_matvec_vs_float64(oracle):
    rng = np.random.default_rng(8)
    rows, K = 64, 7168
    W = oracle.gen_iq2(SEED, 2, 0, 9, rows, K)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = oracle.quant_q8(x)
    y = oracle.iq2_matvec(W, rows, K, q, d)
    Wd = oracle.iq2_dequant(W).reshape(rows, K).astype(np.float64)
    ref = Wd @ _q8_dequant(oracle, x)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


def test_moe_layer_vs_numpy_restatement(oracle):
    """The oracle layer against a numpy float64 restatement of fl_moe's math on the same q8 operands."""
    NE, T, KE = 3, 2, 2
    S = 2048 * 28 * 66
    gate = np.concatenate([oracle.gen_iq2(SEED, 4, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 4, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([oracle.gen_iq2(SEED, 4, 2, e, 7168, 2048) for e in range(NE)])
    rng = np.random.default_rng(12)
    x = rng.standard_normal((T, 7168)).astype(np.float32)
    r = rng.standard_normal((T, 7168)).astype(np.float32)
    ids = np.array([[2, 0], [1, 2]], np.int32)
    w = np.array([[0.7, 1.8], [1.1, 1.4]], np.float32)
    out = oracle.moe_layer(x, r, gate, up, down, S, ids, w)
    for t in range(T):
        xq = _q8_dequant(oracle, x[t])
        acc = np.zeros(7168)
        for k in range(KE):
            e = ids[t, k]
            G = oracle.iq2_dequant(gate[e * S:(e + 1) * S]).reshape(2048, 7168).astype(np.float64)
            U = oracle.iq2_dequant(up[e * S:(e + 1) * S]).reshape(2048, 7168).astype(np.float64)
            D = oracle.iq2_dequant(down[e * S:(e + 1) * S]).reshape(7168, 2048).astype(np.float64)
            g = (G @ xq).astype(np.float32)
            u = (U @ xq).astype(np.float32)
            h = np.array([oracle_swiglu(a, b) for a, b in zip(g, u)], np.float32)
            acc += float(w[t, k]) * (D @ _q8_dequant(oracle, h))
        rel = np.linalg.norm(out["moe"][t] - acc) / np.linalg.norm(acc)
        assert rel < 1e-5, rel
        np.testing.assert_allclose(out["h"][t], out["moe"][t] + r[t], rtol=1e-6, atol=1e-5)


def oracle_swiglu(g, u):
    from oracle import oracle as O
    e = O.lib().orc_expf(float(-g))
    return np.float32(np.float32(g) / np.float32(np.float32(1.0) + np.float32(e)) * np.float32(u))


def test_moe_layer_kat(oracle):
    f = np.load(os.path.join(GOLD, "moe_layer_kat.npz"))
    NE = 6
    S = 2048 * 28 * 66
    gate = np.concatenate([oracle.gen_iq2(SEED, 9, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 9, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([oracle.gen_iq2(SEED, 9, 2, e, 7168, 2048) for e in range(NE)])
    shg, shu, shd = (oracle.gen_iq2(SEED, 9, 0, 256, 2048, 7168), oracle.gen_iq2(SEED, 9, 1, 256, 2048, 7168),
                     oracle.gen_iq2(SEED, 9, 2, 256, 7168, 2048))
    rng = np.random.default_rng(99)
    xs = rng.standard_normal((3, 7168)).astype(np.float32)
    rs = rng.standard_normal((3, 7168)).astype(np.float32)
    out = oracle.moe_layer(xs, rs, gate, up, down, S, f["ids"], f["w"], shg, shu, shd)
    np.testing.assert_array_equal(out["h"], f["h"])
    np.testing.assert_array_equal(out["moe"], f["moe"])


# ---------------------------------------------------------------- K-quant down formats (Q2_K, Q3_K)
KQ = [(5, "q2k", "Q2_K"), (6, "q3k", "Q3_K")]


@pytest.mark.parametrize("fmt,tag,name", KQ)
def test_kq_dequant_matches_gguf_fixture(oracle, fmt, tag, name):
    f = np.load(os.path.join(GOLD, "kquant_gguf.npz"))
    out = oracle.kq_dequant(fmt, f[tag + "_blocks"])
    np.testing.assert_array_equal(out, f[tag + "_dequant"])


@pytest.mark.parametrize("fmt,tag,name", KQ)
def test_kq_dequant_matches_gguf_live(oracle, fmt, tag, name):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    blk = oracle.gen_kq(fmt, SEED, 7, 2, 100, 32, 2048)
    np.testing.assert_array_equal(oracle.kq_dequant(fmt, blk), dequantize(blk, getattr(gguf.GGMLQuantizationType, name)).reshape(-1))


def test_q3k_scale_unpack_matches_kmask_restatement(oracle):
    """The 6-bit scale unpacking against a word-level restatement of ggml's kmask1/kmask2 shuffle
    (dequantize_row_q3_K; the reference's q3_scales, fused_layer.cu:34-37)."""
    rng = np.random.default_rng(21)
    blk = rng.integers(0, 256, (64, 110), dtype=np.uint8)
    blk[:, 108:110] = np.frombuffer(np.array([1.0] * 64, np.float16).tobytes(), np.uint8).reshape(64, 2)
    blk[:, 32:96] = 0x55                        # every low 2-bit field = 1
    blk[:, 0:32] = 0xFF                         # every high bit set: q = 1
    deq = oracle.kq_dequant(6, blk.reshape(-1)).reshape(64, 16, 16)
    for b in range(64):
        a0, a1, tmp = (int.from_bytes(bytes(blk[b, 96 + 4 * i: 100 + 4 * i]), "little") for i in range(3))
        aux = [(a0 & 0x0F0F0F0F) | (((tmp >> 0) & 0x03030303) << 4), (a1 & 0x0F0F0F0F) | (((tmp >> 2) & 0x03030303) << 4),
               ((a0 >> 4) & 0x0F0F0F0F) | (((tmp >> 4) & 0x03030303) << 4), ((a1 >> 4) & 0x0F0F0F0F) | (((tmp >> 6) & 0x03030303) << 4)]
        sc = [((aux[i // 4] >> (8 * (i % 4))) & 0xFF) - 32 for i in range(16)]
        np.testing.assert_array_equal(deq[b, :, 0], np.array(sc, np.float32))


@pytest.mark.parametrize("fmt,tag,name", KQ)
def test_kq_matvec_vs_float64(oracle, fmt, tag, name):
    rng = np.random.default_rng(9)
    rows, K = 96, 2048
    W = oracle.gen_kq(fmt, SEED, 2, 2, 9, rows, K)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = oracle.quant_q8(x)
    y = oracle.kq_matvec(fmt, W, rows, K, q, d)
    Wd = oracle.kq_dequant(fmt, W).reshape(rows, K).astype(np.float64)
    ref = Wd @ _q8_dequant(oracle, x)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


@pytest.mark.parametrize("fmt,tag,name", KQ)
def test_kq_moe_layer_kat(oracle, fmt, tag, name):
    f = np.load(os.path.join(GOLD, "kquant_gguf.npz"))
    NE, nb = 4, oracle.BLOCK_BYTES[fmt]
    S, DS = 2048 * 28 * 66, 7168 * 8 * nb
    gate = np.concatenate([oracle.gen_iq2(SEED, 11, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 11, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([oracle.gen_kq(fmt, SEED, 11, 2, e, 7168, 2048) for e in range(NE)])
    shg, shu = oracle.gen_iq2(SEED, 11, 0, 256, 2048, 7168), oracle.gen_iq2(SEED, 11, 1, 256, 2048, 7168)
    shd = oracle.gen_kq(fmt, SEED, 11, 2, 256, 7168, 2048)
    rng = np.random.default_rng(77)
    xs = rng.standard_normal((2, 7168)).astype(np.float32)
    rs = rng.standard_normal((2, 7168)).astype(np.float32)
    out = oracle.moe_layer(xs, rs, gate, up, down, S, f[tag + "_layer_ids"], f[tag + "_layer_w"], shg, shu, shd,
                           down_fmt=fmt, down_stride=DS)
    np.testing.assert_array_equal(out["h"], f[tag + "_layer_h"])
    np.testing.assert_array_equal(out["moe"], f[tag + "_layer_moe"])
    # the layer's down projection against the dequantised K-quant matrix (float64 restatement)
    D = oracle.kq_dequant(fmt, down[:DS]).reshape(7168, 2048).astype(np.float64)
    assert np.isfinite(D).all() and np.abs(D).max() > 0


# ---------------------------------------------------------------- the shared expert's formats (Q5_K, Q6_K)
SKQ = [(3, "q5k", "Q5_K", 7168), (1, "q6k", "Q6_K", 2048)]


@pytest.mark.parametrize("fmt,tag,name,K", SKQ)
def test_shared_kq_dequant_matches_gguf_fixture(oracle, fmt, tag, name, K):
    f = np.load(os.path.join(GOLD, "shared_kq_gguf.npz"))
    np.testing.assert_array_equal(oracle.kq_dequant(fmt, f[tag + "_blocks"]), f[tag + "_dequant"])


@pytest.mark.parametrize("fmt,tag,name,K", SKQ)
def test_shared_kq_dequant_matches_gguf_live(oracle, fmt, tag, name, K):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    blk = oracle.gen_kq(fmt, SEED, 7, 0, 256, 16, K)
    np.testing.assert_array_equal(oracle.kq_dequant(fmt, blk), dequantize(blk, getattr(gguf.GGMLQuantizationType, name)).reshape(-1))


@pytest.mark.parametrize("fmt,tag,name,K", SKQ)
def test_shared_kq_matvec_vs_float64(oracle, fmt, tag, name, K):
    """The reference's per-sub-block integer arithmetic (Q5_K per 32 with the min term, Q6_K per 16) equals
    the dequantised matrix times the q8 activations."""
    rng = np.random.default_rng(10)
    rows = 64
    W = oracle.gen_kq(fmt, SEED, 2, 0, 256, rows, K)
    x = rng.standard_normal(K).astype(np.float32)
    q, d = oracle.quant_q8(x)
    y = oracle.kq_matvec(fmt, W, rows, K, q, d)
    ref = oracle.kq_dequant(fmt, W).reshape(rows, K).astype(np.float64) @ _q8_dequant(oracle, x)
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


def test_q5k_scale_min_matches_restatement(oracle):
    """Q5_K's packed (scale, min) pairs against a bit-level restatement of ggml's get_scale_min_k4: with q = 1
    everywhere (qs nibbles 1, qh bits 0), d = 1 and dmin = 0 each sub-block's weights equal its scale."""
    rng = np.random.default_rng(22)
    blk = rng.integers(0, 256, (64, 176), dtype=np.uint8)
    blk[:, 0:2] = np.frombuffer(np.array([1.0] * 64, np.float16).tobytes(), np.uint8).reshape(64, 2)
    blk[:, 2:4] = 0
    blk[:, 16:48] = 0
    blk[:, 48:176] = 0x11
    deq = oracle.kq_dequant(3, blk.reshape(-1)).reshape(64, 8, 32)
    for b in range(64):
        q = blk[b, 4:16].astype(int)
        sc = [q[j] & 63 if j < 4 else (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4) for j in range(8)]
        np.testing.assert_array_equal(deq[b, :, 0], np.array(sc, np.float32))


def test_shared_kq_moe_layer_kat(oracle):
    """IQ2_XXS routed gate/up, Q3_K routed downs and the real model's Q5_K / Q6_K shared expert."""
    f = np.load(os.path.join(GOLD, "shared_kq_gguf.npz"))
    NE = 3
    S, DS = 2048 * 28 * 66, 7168 * 8 * 110
    gate = np.concatenate([oracle.gen_iq2(SEED, 12, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 12, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([oracle.gen_kq(6, SEED, 12, 2, e, 7168, 2048) for e in range(NE)])
    shg = oracle.gen_kq(3, SEED, 12, 0, 256, 2048, 7168)
    shu = oracle.gen_kq(3, SEED, 12, 1, 256, 2048, 7168)
    shd = oracle.gen_kq(1, SEED, 12, 2, 256, 7168, 2048)
    rng = np.random.default_rng(78)
    xs = rng.standard_normal((2, 7168)).astype(np.float32)
    rs = rng.standard_normal((2, 7168)).astype(np.float32)
    out = oracle.moe_layer(xs, rs, gate, up, down, S, f["layer_ids"], f["layer_w"], shg, shu, shd, want_slots=True,
                           down_fmt=6, down_stride=DS, sh_gu_fmt=3, sh_down_fmt=1)
    np.testing.assert_array_equal(out["h"], f["layer_h"])
    np.testing.assert_array_equal(out["moe"], f["layer_moe"])
    np.testing.assert_array_equal(out["shared"], f["layer_shared"])
    # the shared part against a float64 restatement from the gguf-py-pinned dequantisation
    G = oracle.kq_dequant(3, shg).reshape(2048, 7168).astype(np.float64)
    U = oracle.kq_dequant(3, shu).reshape(2048, 7168).astype(np.float64)
    D = oracle.kq_dequant(1, shd).reshape(7168, 2048).astype(np.float64)
    xq = _q8_dequant(oracle, xs[0])
    g, u = G @ xq, U @ xq
    hsw = (g / (1 + np.exp(-g))) * u
    ref = D @ _q8_dequant(oracle, hsw.astype(np.float32))
    assert np.linalg.norm(out["shared"][0] - ref) / np.linalg.norm(ref) < 1e-3
    # shared and routed parts have comparable magnitudes with the generator's scales
    r = np.linalg.norm(out["shared"]) / np.linalg.norm(out["moe"])
    assert 0.05 < r < 20
