"""What the reference's q8 numerics cost (CPU, oracle only; informational numbers with loose bounds).

The parity gate compares the CUDA paths with an oracle that uses the reference's own arithmetic: q8-per-32
activations (src/fused_layer.cu:40-47) and SwiGLU followed by a q8 of h (src/fused_layer.cu:334-341). This test
reports the other two numbers for one layer. Both compare against the same layer computed in float64 from the
dequantised weights, with x and h unquantised:
* the oracle with the reference's numerics (x and h in q8);
* the oracle of the tensor-core paths (x in q8, h unquantised).
The gaps are the activations' quantisation noise: about 1e-2 relative L2 with h in q8 and 7e-3 without. A comparison
against an unquantised computation therefore cannot hold the 2e-3 tolerance, which is why the gate uses the same-q8
oracle.
"""
import numpy as np

from moe_helpers import HIDDEN, INTER, SEED, oracle_layer, rel_l2

LAYER = 3


def swiglu64(g, u):
    return g / (1.0 + np.exp(-g)) * u


def layer_fp64(oracle, x, sel, w):
    """(routed = sum_k w_k * expert_k, shared expert), every product in float64 on fp32 x."""
    x64 = x.astype(np.float64)
    T = x.shape[0]
    moe = np.zeros((T, HIDDEN))
    shared = np.zeros((T, HIDDEN))

    def expert(e):
        G = oracle.iq2_dequant(oracle.gen_iq2(SEED, LAYER, 0, e, INTER, HIDDEN)).reshape(INTER, HIDDEN).astype(np.float64)
        U = oracle.iq2_dequant(oracle.gen_iq2(SEED, LAYER, 1, e, INTER, HIDDEN)).reshape(INTER, HIDDEN).astype(np.float64)
        D = oracle.iq2_dequant(oracle.gen_iq2(SEED, LAYER, 2, e, HIDDEN, INTER)).reshape(HIDDEN, INTER).astype(np.float64)
        return lambda v: D @ swiglu64(G @ v, U @ v)

    for e in sorted(set(int(i) for i in sel.reshape(-1))):
        f = expert(e)
        for t, k in zip(*np.nonzero(sel == e)):
            moe[t] += w[t, k] * f(x64[t])
    f = expert(256)                                          # the shared expert (generator slot 256)
    for t in range(T):
        shared[t] = f(x64[t])
    return moe, shared


def test_q8_activation_noise_against_float64(oracle):
    rng = np.random.default_rng(2024)
    T, KE = 2, 8
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    resid = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    sel = np.stack([rng.choice(256, KE, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 0.6, (T, KE)).astype(np.float32)
    routed64, shared64 = layer_fp64(oracle, x, sel, w)
    q8 = oracle_layer(oracle, SEED, LAYER, x, resid, sel, w, hq8=True)        # moe = routed; h = resid + routed + shared
    f16h = oracle_layer(oracle, SEED, LAYER, x, resid, sel, w, hq8=False)
    e_q8, e_h = rel_l2(q8["moe"], routed64), rel_l2(f16h["moe"], routed64)
    h64 = resid.astype(np.float64) + routed64 + shared64
    print("routed experts vs float64 on unquantised activations: reference numerics (x, h in q8) %.2e; "
          "tensor-core numerics (x in q8, h unquantised) %.2e; between the two %.2e. Layer output h (with the shared "
          "expert and the residual): %.2e / %.2e" % (e_q8, e_h, rel_l2(q8["moe"], f16h["moe"]), rel_l2(q8["h"], h64), rel_l2(f16h["h"], h64)))
    # the structure agrees (an error of order 1 would mean a different layer), and the noise is that of q8
    assert 5e-4 < e_q8 < 2e-2 and e_h < e_q8
