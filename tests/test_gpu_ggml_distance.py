"""Every regime's distance from ggml's CPU numerics (the oracle's q8_K mode), beside the reference's own.

The reference's fused kernels and ggml's CPU mul_mat_id quantise activations differently (q8 per 32 vs q8_K
per 256), which puts them about 1.9e-2 apart in relative L2.  Each regime of the CUDA path runs one layer; on
the sampled tokens its distance from the q8_K oracle must equal the reference numerics' own distance from it
to within the 2e-3 parity gate (the CUDA path is within 2e-3 of the reference numerics, so by the triangle
inequality this holds whenever parity does).  The printed lines are the figures quoted in the documentation."""
import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, RTOL_L2, rel_l2, oracle_layer, oracle_layer_ggml

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def moe(native):
    from loki_b200 import moe as M
    return M


@pytest.fixture(scope="module")
def layer_weights(moe):
    W = moe.LayerWeights("cuda", SEED, 0)
    torch.cuda.synchronize()
    yield W
    del W
    torch.cuda.empty_cache()


# (T, regime name, sampled tokens)
REGIMES = [(1, "decode matvec (T=1)", None), (16, "narrow matvec (T=16)", [0, 7, 15]),
           (64, "q8 gate/up + mma.sync down (T=64)", [0, 31, 63]),
           (512, "q8 gate/up + tcgen05 down (T=512)", [0, 200, 511])]


@pytest.mark.parametrize("T,name,tok", REGIMES)
def test_regime_distance_from_ggml(moe, oracle, layer_weights, T, name, tok):
    rng = np.random.default_rng(4000 + T)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    layer = moe.MoeLayer(0, max_tokens=T)
    h, mo, sel, w = layer.forward(layer_weights, torch.from_numpy(x).cuda(), torch.from_numpy(r).cuda())
    layer.device_error()
    sel, w = sel.cpu().numpy(), w.cpu().numpy()
    tok = list(range(T)) if tok is None else tok
    ref = oracle_layer(oracle, SEED, 0, x, r, sel, w, tokens=tok)
    gg = oracle_layer_ggml(oracle, SEED, 0, x, r, sel, w, tokens=tok)
    mo = mo.cpu().numpy()[tok]
    d_gpu, d_ref, d_par = rel_l2(mo, gg["moe"]), rel_l2(ref["moe"], gg["moe"]), rel_l2(mo, ref["moe"])
    print("\n[ggml distance] %-36s cuda-vs-ggml %.3e  reference-vs-ggml %.3e  cuda-vs-reference %.3e"
          % (name, d_gpu, d_ref, d_par))
    assert d_par < RTOL_L2
    assert abs(d_gpu - d_ref) < RTOL_L2
