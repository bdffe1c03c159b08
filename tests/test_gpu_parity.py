"""GPU parity of the CUDA path (through libloki_moe.so's C ABI) against the CPU oracle.

Bit-exact: generated weights, router probabilities, selected expert ids and weights, dispatch
permutations.  Layer outputs h / moe: relative L2 <= 2e-3 (RTOL_L2) of the oracle using the same q8 scheme.
"""
import ctypes

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, MAT, RTOL_L2, rel_l2, oracle_layer, host_arena

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def moe(native):
    from loki_b200 import moe as M
    return M


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def router_only_weights(native, W, bias, f16=False):
    ws = native.LkMoeWeights()
    ws.router_w = W.data_ptr()
    ws.router_w_f16 = 1 if f16 else 0
    ws.router_bias = bias.data_ptr()
    ws.down_fmt = native.FMT_IQ2
    return ws


# ---------------------------------------------------------------- generator
@pytest.mark.parametrize("key", [(0, 0, 0), (3, 1, 77), (57, 2, 255), (7, 0, 256)])
def test_generator_bitexact(native, moe, oracle, key):
    layer, m, e = key
    rows, K = (INTER, HIDDEN) if m < 2 else (HIDDEN, INTER)
    buf = torch.empty(MAT, dtype=torch.uint8, device="cuda")
    moe.gen_iq2(buf, SEED, layer, m, e, 1, rows, K, MAT)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(buf.cpu().numpy(), oracle.gen_iq2(SEED, layer, m, e, rows, K))


# ---------------------------------------------------------------- router
ROUTE_MODES = {
    "top8": dict(keep=8), "keep2": dict(keep=2), "keep2_norenorm": dict(keep=2, renorm=False),
    "grouped": dict(keep=8, n_group=8, topk_group=4), "grouped_keep2": dict(keep=2, n_group=8, topk_group=4),
}


@pytest.mark.parametrize("T", [1, 3, 16, 100, 512, 4096])
@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("mode", list(ROUTE_MODES))
def test_router_bitexact(native, moe, oracle, T, f16, mode):
    """Probabilities, ids and weights bit-identical to the oracle: the per-expert kernel (T < 64) and the
    token-tile batch kernel (T >= 64; T = 100 ends on a partial tile of 4 tokens, T = 512 splits the experts
    over 4 CTAs per tile, T = 4096 does not split)."""
    md = ROUTE_MODES[mode]
    rng = np.random.default_rng(100 + T)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    if f16:
        W = W.astype(np.float16)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    layer = moe.MoeLayer(0, keep=md["keep"], renorm=md.get("renorm", True), n_group=md.get("n_group", 1),
                         topk_group=md.get("topk_group", 1), max_tokens=T)
    Wd, bd = _dev(W), _dev(bias)
    probs, sel, w = layer.route(router_only_weights(native, Wd, bd, f16), _dev(x))
    torch.cuda.synchronize()
    cfg = oracle.route_cfg(8, md["keep"], int(md.get("renorm", True)), md.get("n_group", 1), md.get("topk_group", 1))
    op, osel, ow = oracle.router(x, W.astype(np.float32), bias, cfg)
    np.testing.assert_array_equal(probs.cpu().numpy(), op)
    np.testing.assert_array_equal(sel.cpu().numpy(), osel)
    np.testing.assert_array_equal(w.cpu().numpy(), ow)
    layer.device_error()


def test_router_logits_override(native, moe, oracle):
    rng = np.random.default_rng(7)
    T = 64
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    logits = rng.uniform(-1, 1, (T, 256)).astype(np.float32)
    layer = moe.MoeLayer(0, max_tokens=T)
    Wd, bd, xd, ld = _dev(W), _dev(bias), _dev(x), _dev(logits)      # kept alive: the struct holds raw pointers
    probs, sel, w = layer.route(router_only_weights(native, Wd, bd), xd, logits_override=ld)
    op, osel, ow = oracle.router(None, None, bias, oracle.route_cfg(8, 8), logits=logits)
    np.testing.assert_array_equal(probs.cpu().numpy(), op)
    np.testing.assert_array_equal(sel.cpu().numpy(), osel)
    np.testing.assert_array_equal(w.cpu().numpy(), ow)


@pytest.mark.parametrize("T", [1, 3])
@pytest.mark.parametrize("grouped", [False, True])
def test_router_ties(native, moe, oracle, T, grouped):
    """Logits on a 5-value grid and a zero bias: many experts (and groups) score exactly alike, so the
    order of the selection rests on the lower-id tie rule (one-token CTA path and per-warp path)."""
    rng = np.random.default_rng(11 + T)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    bias = np.zeros(256, np.float32)
    logits = rng.integers(-2, 3, (T, 256)).astype(np.float32) * 0.5
    ng, tg = (8, 4) if grouped else (1, 1)
    layer = moe.MoeLayer(0, n_group=ng, topk_group=tg, max_tokens=T)
    Wd, bd, xd, ld = _dev(W), _dev(bias), _dev(x), _dev(logits)
    probs, sel, w = layer.route(router_only_weights(native, Wd, bd), xd, logits_override=ld)
    op, osel, ow = oracle.router(None, None, bias, oracle.route_cfg(8, 8, 1, ng, tg), logits=logits)
    np.testing.assert_array_equal(sel.cpu().numpy(), osel)
    np.testing.assert_array_equal(w.cpu().numpy(), ow)


# ---------------------------------------------------------------- dispatch
def zipf_sel(rng, T, keep, s=1.2):
    p = 1.0 / np.arange(1, 257) ** s
    p /= p.sum()
    out = np.empty((T, keep), np.int32)
    for t in range(T):
        out[t] = rng.choice(256, keep, replace=False, p=p)
    return out


@pytest.mark.parametrize("T,keep,skew", [(1, 8, False), (5, 2, False), (512, 8, False), (4096, 8, False), (512, 2, True), (3000, 8, True)])
def test_dispatch_bitexact(native, moe, oracle, T, keep, skew):
    rng = np.random.default_rng(T + keep)
    sel = zipf_sel(rng, T, keep) if skew else np.stack([rng.choice(256, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0, 1, (T, keep)).astype(np.float32)
    layer = moe.MoeLayer(0, keep=keep, max_tokens=T)
    counts, offsets, perm = layer.dispatch(_dev(sel), _dev(w))
    oc, oo, op = oracle.permute(sel)
    np.testing.assert_array_equal(counts.cpu().numpy(), oc)
    np.testing.assert_array_equal(offsets.cpu().numpy(), oo)
    np.testing.assert_array_equal(perm.cpu().numpy(), op)


# ---------------------------------------------------------------- experts on a small arena
@pytest.mark.parametrize("T,keep", [(1, 8), (1, 2), (3, 2), (8, 8), (20, 4)])
def test_experts_small_arena(native, moe, oracle, T, keep):
    NE = 12
    layer_id = 11
    buf = torch.empty(3 * NE * MAT + 3 * MAT, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    for m in range(3):
        rows, K = (INTER, HIDDEN) if m < 2 else (HIDDEN, INTER)
        moe.gen_iq2(base + m * NE * MAT, SEED, layer_id, m, 0, NE, rows, K, MAT)
        moe.gen_iq2(base + 3 * NE * MAT + m * MAT, SEED, layer_id, m, 256, 1, rows, K, MAT)
    ws = native.LkMoeWeights(base, base + NE * MAT, base + 2 * NE * MAT, MAT, MAT, MAT, native.FMT_IQ2,
                             base + 3 * NE * MAT, base + 3 * NE * MAT + MAT, base + 3 * NE * MAT + 2 * MAT, None, 0, None)
    rng = np.random.default_rng(T * 10 + keep)
    sel = np.stack([rng.choice(NE, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = moe.MoeLayer(0, keep=keep, max_tokens=T)
    layer.set_mma_threshold(1 << 20)                  # the single-token dp4a matvecs (q8 h, as the reference)
    h, mo = layer.experts(ws, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    ref = oracle_layer(oracle, SEED, layer_id, x, r, sel, w)
    e_moe, e_h = rel_l2(mo.cpu().numpy(), ref["moe"]), rel_l2(h.cpu().numpy(), ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)


@pytest.mark.parametrize("T,keep", [(2, 8), (5, 2), (16, 8), (40, 4), (100, 8)])
def test_experts_mma_path(native, moe, oracle, T, keep):
    """The mid-size regime (forced on for any T): the q8 gate/up on tcgen05 (h re-quantised to q8, the
    reference's numerics), then the mma.sync IQ2_XXS down, against the oracle with the reference's numerics."""
    NE = 12
    layer_id = 17
    buf = torch.empty(3 * NE * MAT + 3 * MAT, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    for m in range(3):
        rows, K = (INTER, HIDDEN) if m < 2 else (HIDDEN, INTER)
        moe.gen_iq2(base + m * NE * MAT, SEED, layer_id, m, 0, NE, rows, K, MAT)
        moe.gen_iq2(base + 3 * NE * MAT + m * MAT, SEED, layer_id, m, 256, 1, rows, K, MAT)
    ws = native.LkMoeWeights(base, base + NE * MAT, base + 2 * NE * MAT, MAT, MAT, MAT, native.FMT_IQ2,
                             base + 3 * NE * MAT, base + 3 * NE * MAT + MAT, base + 3 * NE * MAT + 2 * MAT, None, 0, None)
    rng = np.random.default_rng(T * 13 + keep)
    sel = np.stack([rng.choice(NE, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = moe.MoeLayer(0, keep=keep, max_tokens=T)
    layer.set_mma_threshold(2)
    layer.set_gemm_threshold(1 << 20)
    h, mo = layer.experts(ws, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    tok = list(range(T)) if T <= 40 else [0, 1, T // 2, T - 2, T - 1]
    ref = oracle_layer(oracle, SEED, layer_id, x, r, sel, w, tokens=tok, hq8=True)
    e_moe, e_h = rel_l2(mo.cpu().numpy()[tok], ref["moe"]), rel_l2(h.cpu().numpy()[tok], ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)


@pytest.mark.parametrize("T,keep", [(2, 8), (40, 8), (70, 2), (130, 8)])
def test_experts_tensor_core_path(native, moe, oracle, T, keep):
    """The tcgen05 regime (forced on for any T): the q8 gate/up, then the tcgen05 IQ2_XXS down, against the
    oracle with the reference's numerics (h re-quantised to q8) on a small arena."""
    NE = 12
    layer_id = 13
    buf = torch.empty(3 * NE * MAT + 3 * MAT, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    for m in range(3):
        rows, K = (INTER, HIDDEN) if m < 2 else (HIDDEN, INTER)
        moe.gen_iq2(base + m * NE * MAT, SEED, layer_id, m, 0, NE, rows, K, MAT)
        moe.gen_iq2(base + 3 * NE * MAT + m * MAT, SEED, layer_id, m, 256, 1, rows, K, MAT)
    ws = native.LkMoeWeights(base, base + NE * MAT, base + 2 * NE * MAT, MAT, MAT, MAT, native.FMT_IQ2,
                             base + 3 * NE * MAT, base + 3 * NE * MAT + MAT, base + 3 * NE * MAT + 2 * MAT, None, 0, None)
    rng = np.random.default_rng(T * 7 + keep)
    sel = np.stack([rng.choice(NE, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = moe.MoeLayer(0, keep=keep, max_tokens=T)
    layer.set_gemm_threshold(1)
    h, mo = layer.experts(ws, _dev(x), _dev(r), _dev(sel), _dev(w))
    layer.device_error()
    tok = list(range(T)) if T <= 40 else [0, 1, T // 2, T - 2, T - 1]
    ref = oracle_layer(oracle, SEED, layer_id, x, r, sel, w, tokens=tok, hq8=True)
    e_moe = rel_l2(mo.cpu().numpy()[tok], ref["moe"])
    e_h = rel_l2(h.cpu().numpy()[tok], ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)


# ---------------------------------------------------------------- the whole layer (256 experts resident)
@pytest.fixture(scope="module")
def layer_weights(moe):
    W = moe.LayerWeights("cuda", SEED, 0)
    torch.cuda.synchronize()
    yield W
    del W
    torch.cuda.empty_cache()


def _layer_case(moe, oracle, W, T, keep=8, n_group=1, topk_group=1, logits=None, sample=None, seed=0, bf16=False):
    """One layer through lk_moe_forward against the oracle with the reference's numerics (q8 x and h) on the
    tokens of `sample` (default: all).  bf16: hidden states rounded to bf16, as BASELINE configs 2 and 3 state."""
    rng = np.random.default_rng(1000 + T + seed)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    if bf16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    layer = moe.MoeLayer(0, keep=keep, n_group=n_group, topk_group=topk_group, max_tokens=T)
    h, mo, sel, w = layer.forward(W, _dev(x), _dev(r), logits_override=None if logits is None else _dev(logits))
    layer.device_error()
    sel, w = sel.cpu().numpy(), w.cpu().numpy()
    Wr = W.router_w.float().cpu().numpy()
    bias = W.router_bias.cpu().numpy()
    cfg = oracle.route_cfg(8, keep, 1, n_group, topk_group)
    _, osel, ow = oracle.router(x, Wr, bias, cfg, logits=logits)
    np.testing.assert_array_equal(sel, osel)
    np.testing.assert_array_equal(w, ow)
    ref = oracle_layer(oracle, SEED, 0, x, r, sel, w, tokens=sample, hq8=True)
    tok = list(range(T)) if sample is None else list(sample)
    e_moe = rel_l2(mo.cpu().numpy()[tok], ref["moe"])
    e_h = rel_l2(h.cpu().numpy()[tok], ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)
    return e_moe, e_h


def test_layer_config0_T16(moe, oracle, layer_weights):
    """T=16, hidden 7168, 256 experts, top-8 with grouped routing (8 groups, top 4), shared expert."""
    _layer_case(moe, oracle, layer_weights, 16, n_group=8, topk_group=4)


@pytest.mark.parametrize("keep,n_group", [(8, 1), (2, 1), (8, 8), (2, 8)])
def test_layer_decode_T1(moe, oracle, layer_weights, keep, n_group):
    _layer_case(moe, oracle, layer_weights, 1, keep=keep, n_group=n_group, topk_group=4 if n_group > 1 else 1)


def _sample(T, n, seed):
    """n distinct token positions of T, first and last included (sorted)."""
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(1, T - 1), n - 2, replace=False)
    return sorted({0, T - 1, *map(int, mid)})


def test_layer_prefill_T512_uniform_logits(moe, oracle, layer_weights):
    """T=512, bf16 N(0,1) hidden states, uniform-random router logits, top-8 of 256 with the
    shared expert; the oracle (reference numerics) on 64 sampled tokens."""
    rng = np.random.default_rng(512)
    logits = rng.uniform(-1, 1, (512, 256)).astype(np.float32)
    _layer_case(moe, oracle, layer_weights, 512, logits=logits, sample=_sample(512, 64, 5), bf16=True)


def test_layer_batch_T4096_grouped(moe, oracle, layer_weights):
    """BASELINE config 3's single-GPU shape: T=4096 bf16 N(0,1) hidden states through the grouped router
    (8 groups, top 4) and top-8 of 256 experts (slots of up to 128 tokens: both token halves of the gate/up);
    the oracle on 64 sampled tokens."""
    _layer_case(moe, oracle, layer_weights, 4096, n_group=8, topk_group=4, sample=_sample(4096, 64, 6), bf16=True)


def test_layer_deterministic(moe, layer_weights):
    rng = np.random.default_rng(3)
    x = _dev(rng.standard_normal((64, HIDDEN)).astype(np.float32))
    r = _dev(rng.standard_normal((64, HIDDEN)).astype(np.float32))
    layer = moe.MoeLayer(0, max_tokens=64)
    h1 = layer.forward(layer_weights, x, r)[0].clone()
    h2 = layer.forward(layer_weights, x, r)[0].clone()
    assert torch.equal(h1, h2)


# ---------------------------------------------------------------- load imbalance
@pytest.mark.parametrize("T", [8, 64, 200])
def test_layer_zipf_bias_keep2(moe, oracle, T):
    """keep 2 of top-8 with a Zipf-calibrated router bias (hottest expert ~10x the mean entries): routing
    bit-exact, outputs within RTOL_L2 (T >= 64 takes the tensor-core path with its hot, multi-slot experts)."""
    from loki_b200 import synthetic as S
    bias = S.zipf_bias(S.calibrate_zipf_lambda())
    W = moe.LayerWeights("cuda", SEED, 0, router_bias=torch.from_numpy(bias))
    try:
        rng = np.random.default_rng(4000 + T)
        x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
        r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
        layer = moe.MoeLayer(0, keep=2, max_tokens=T)
        h, mo, sel, w = layer.forward(W, _dev(x), _dev(r))
        layer.device_error()
        sel, w = sel.cpu().numpy(), w.cpu().numpy()
        _, osel, ow = oracle.router(x, W.router_w.float().cpu().numpy(), bias, oracle.route_cfg(8, 2, 1, 1, 1))
        np.testing.assert_array_equal(sel, osel)
        np.testing.assert_array_equal(w, ow)
        counts = np.bincount(sel.reshape(-1), minlength=256)
        assert counts.max() >= 4 * max(counts.mean(), 1e-9)          # the bias does concentrate the routing
        tok = list(range(T)) if T <= 64 else [0, 1, 50, 99, 150, T - 1]
        ref = oracle_layer(oracle, SEED, 0, x, r, sel, w, tokens=tok, hq8=True)
        assert rel_l2(mo.cpu().numpy()[tok], ref["moe"]) < RTOL_L2
        assert rel_l2(h.cpu().numpy()[tok], ref["h"]) < RTOL_L2
    finally:
        del W
        torch.cuda.empty_cache()


@pytest.mark.parametrize("T", [64, 256])
def test_layer_default_paths(moe, oracle, layer_weights, T):
    """The default thresholds route T=64 to the mma.sync path and T=256 to the tcgen05 path."""
    _layer_case(moe, oracle, layer_weights, T, sample=[0, 1, T // 2, T - 1])
