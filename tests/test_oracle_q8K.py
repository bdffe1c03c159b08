"""The oracle's ggml CPU mode: q8_K activations (one scale per 256 values) as ggml's published
quantize_row_q8_K states them, and the distance of the reference's fused numerics (q8 per 32) from it.

ggml is not vendored in the reference and gguf-py has no Q8_K, so the q8_K restatement is unpinned: these
tests hold it to the algorithm's definition on hand-built blocks and to an independent numpy statement."""
import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, MAT, rel_l2, host_arena, oracle_layer, oracle_layer_ggml


def _np_q8K(x):
    """quantize_row_q8_K restated with numpy: max = the largest-magnitude value (first on ties),
    iscale = -127/max, q = min(127, rint(iscale*x)), d = 1/iscale; zero blocks give d = 0."""
    x = np.asarray(x, np.float32).reshape(-1, 256)
    i = np.argmax(np.abs(x), axis=1)
    mx = x[np.arange(len(x)), i]
    zero = mx == 0
    with np.errstate(divide="ignore"):
        iscale = np.where(zero, np.float32(0), np.float32(-127.0) / np.where(zero, np.float32(1), mx)).astype(np.float32)
    q = np.minimum(127, np.rint((iscale[:, None] * x).astype(np.float32))).astype(np.int8)
    with np.errstate(divide="ignore"):
        d = np.where(zero, np.float32(0), (np.float32(1) / np.where(zero, np.float32(1), iscale)).astype(np.float32))
    return q.reshape(-1), d.astype(np.float32)


def test_q8K_known_answers(oracle):
    x = np.zeros((4, 256), np.float32)
    x[0, 5], x[0, 9] = 2.0, -1.0                 # positive max: d = -2/127, q[5] = -127
    x[1, 3], x[1, 4] = -127.0, 2.5               # negative max: iscale = 1, halves round to even
    x[1, 6], x[1, 7], x[1, 8] = 3.5, -0.5, 1.5
    x[2, 10], x[2, 11] = -4.0, 4.0               # equal magnitudes: the first (negative) sets the sign
    q, d = oracle.quant_q8_K(x.reshape(-1))
    q, d = q.reshape(4, 256), d
    assert d[0] == np.float32(1) / (np.float32(-127) / np.float32(2)) and q[0, 5] == -127 and q[0, 9] == 64
    assert d[1] == 1.0 and list(q[1, 3:9]) == [-127, 2, 0, 4, 0, 2]
    assert d[2] > 0 and q[2, 10] == -127 and q[2, 11] == 127
    assert d[3] == 0 and not q[3].any()          # all-zero block


def test_q8K_matches_numpy_statement(oracle):
    rng = np.random.default_rng(11)
    x = np.concatenate([rng.standard_normal(256 * 64), rng.standard_normal(256 * 16) * 1e-30,
                        np.round(rng.standard_normal(256 * 16) * 4) / 4, rng.uniform(-1, 1, 256 * 16) * 1e20]).astype(np.float32)
    q, d = oracle.quant_q8_K(x)
    nq, nd = _np_q8K(x)
    np.testing.assert_array_equal(q, nq)
    np.testing.assert_array_equal(d.view(np.uint32), nd.view(np.uint32))
    # reconstruction within half a step per element
    err = np.abs(q.astype(np.float64).reshape(-1, 256) * d[:, None].astype(np.float64) - x.reshape(-1, 256).astype(np.float64))
    assert (err <= np.abs(d)[:, None] * 0.5 * (1 + 1e-5) + 1e-45).all()


def test_reference_numerics_distance_from_ggml(oracle):
    """Two tokens through the whole layer: the reference's fused numerics (q8 per 32 for x and h) and ggml's
    CPU numerics (q8_K) are two quantisation schemes of the same layer, about 1.9e-2 apart in relative L2 --
    ten times the 2e-3 parity gate, which is why parity is defined against the reference's own kernels."""
    rng = np.random.default_rng(7)
    x = rng.standard_normal((2, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((2, HIDDEN)).astype(np.float32)
    sel = np.array([[3, 17, 40, 77, 100, 150, 200, 255], [5, 17, 41, 78, 101, 151, 201, 254]], np.int32)
    w = rng.uniform(0.1, 0.5, (2, 8)).astype(np.float32)
    a = oracle_layer(oracle, SEED, 0, x, r, sel, w)
    b = oracle_layer_ggml(oracle, SEED, 0, x, r, sel, w)
    e = rel_l2(a["moe"], b["moe"])
    print("reference (q8 per 32) vs ggml (q8_K) numerics: moe %.3e  h %.3e" % (e, rel_l2(a["h"], b["h"])))
    assert 5e-3 < e < 4e-2
    # the slots are combined in fp32 in k order; routing weights scale linearly
    b2 = oracle_layer_ggml(oracle, SEED, 0, x, r, sel, w * 2)
    assert rel_l2(b2["moe"], 2 * b["moe"]) < 1e-6
