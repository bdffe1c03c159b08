"""Shared helpers of the GPU parity tests: host arenas for the oracle, relative errors, tolerances."""
import numpy as np

SEED = 0x10C1
HIDDEN, INTER = 7168, 2048
MAT = 2048 * 28 * 66                 # bytes of one expert matrix (gate, up or down)
# north_star tolerance: layer outputs within relative L2 2e-3 of the oracle that uses the same q8 scheme
RTOL_L2 = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def host_arena(oracle, seed, layer, experts):
    """Compact host arenas (gate, up, down) holding `experts` in order, plus the shared expert."""
    gate = np.concatenate([oracle.gen_iq2(seed, layer, 0, e, INTER, HIDDEN) for e in experts])
    up = np.concatenate([oracle.gen_iq2(seed, layer, 1, e, INTER, HIDDEN) for e in experts])
    down = np.concatenate([oracle.gen_iq2(seed, layer, 2, e, HIDDEN, INTER) for e in experts])
    sh = tuple(oracle.gen_iq2(seed, layer, m, 256, *((INTER, HIDDEN) if m < 2 else (HIDDEN, INTER))) for m in range(3))
    return gate, up, down, sh


def oracle_layer(oracle, seed, layer, x, resid, sel, w, with_shared=True, tokens=None, hq8=True):
    """Oracle h/moe for routing (sel, w) with global expert ids, on the given tokens (default: all)."""
    tokens = list(range(x.shape[0])) if tokens is None else list(tokens)
    sel = np.asarray(sel)[tokens]
    used = sorted(set(int(e) for e in sel.reshape(-1)))
    remap = {e: i for i, e in enumerate(used)}
    ids = np.vectorize(lambda e: remap[int(e)])(sel).astype(np.int32)
    gate, up, down, sh = host_arena(oracle, seed, layer, used)
    shg, shu, shd = sh if with_shared else (None, None, None)
    return oracle.moe_layer(x[tokens], resid[tokens], gate, up, down, MAT, ids, np.asarray(w)[tokens], shg, shu, shd, hq8=hq8)
