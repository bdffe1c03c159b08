"""Selection margins of the routing parity inputs (CPU, oracle only).

The GPU router and the oracle agree bit for bit because both compute the router dot in one fixed order (the
selection itself follows src/fused_layer.cu:323-332: score = p + bias, argmax rounds, ties to the lower id). This
test measures how much that agreement rests on, for the seeded inputs of the GPU routing tests
(test_gpu_parity.py test_router_bitexact). Per row it takes the gap between the 8th and 9th selection scores among
the allowed experts, and in grouped mode (8 groups, top 4) the gap between the 4th and 5th group scores. Each gap is
measured in float32 ulps at the score above it. A gap under 4 ulp would let a last-bit difference in the dot flip
an id. The fixed seeds must have none.
"""
import numpy as np
import pytest

HIDDEN = 7168
NEAR_ULP = 4


def selection_gaps(p, bias, n_group, topk_group, topk=8):
    """Per-row (expert gap, group gap) in ulps; the group gap is nan without grouping."""
    sc = (p + bias).astype(np.float32)
    T, NE = sc.shape
    eg = np.empty(T)
    gg = np.full(T, np.nan)
    for t in range(T):
        s = sc[t]
        allowed = np.ones(NE, bool)
        if n_group > 1:
            gs = NE // n_group
            top2 = np.sort(s.reshape(n_group, gs), axis=1)[:, ::-1]
            gsc = (top2[:, 0] + top2[:, 1]).astype(np.float32)      # larger + smaller, as the selection sums them
            order = np.argsort(-gsc, kind="stable")
            above, below = gsc[order[topk_group - 1]], gsc[order[topk_group]]
            gg[t] = (above - below) / np.spacing(above)
            allowed = np.repeat(np.isin(np.arange(n_group), order[:topk_group]), gs)
        a = np.sort(s[allowed])[::-1]
        eg[t] = (a[topk - 1] - a[topk]) / np.spacing(a[topk - 1])
    return eg, gg


@pytest.mark.parametrize("T", [1, 3, 16, 512])
@pytest.mark.parametrize("f16", [False, True])
def test_router_inputs_have_no_near_ties(oracle, T, f16):
    rng = np.random.default_rng(100 + T)                     # the inputs of test_router_bitexact
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    W = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    if f16:
        W = W.astype(np.float16).astype(np.float32)
    p, _, _ = oracle.router(x, W, bias, oracle.route_cfg(8, 8))
    for n_group, topk_group in ((1, 1), (8, 4)):
        eg, gg = selection_gaps(p, bias, n_group, topk_group)
        near_e = int((eg < NEAR_ULP).sum())
        near_g = int(np.nansum(gg < NEAR_ULP))
        print("T=%d f16=%d n_group=%d: smallest 8th/9th gap %.0f ulp, rows under %d ulp: %d; smallest group gap %s"
              % (T, f16, n_group, eg.min(), NEAR_ULP, near_e, "-" if n_group == 1 else "%.0f ulp" % np.nanmin(gg)))
        assert near_e == 0 and near_g == 0


def test_gap_measure_sees_a_planted_tie(oracle):
    """The measure itself: scores with the 8th and 9th one ulp apart, and groups 4 and 5 tied, read as near."""
    p = np.linspace(0.9, 0.1, 256, dtype=np.float32)[None, :].copy()
    bias = np.zeros(256, np.float32)
    p[0, 8] = np.nextafter(p[0, 7], np.float32(0))             # experts 0..7 first; the 8th and 9th one ulp apart
    eg, _ = selection_gaps(p, bias, 1, 1)
    assert eg[0] < NEAR_ULP
    q = np.full((1, 256), 0.5, np.float32)                     # every group scores alike: groups 4 and 5 tie
    _, gg = selection_gaps(q, bias, 8, 4)
    assert gg[0] < NEAR_ULP
