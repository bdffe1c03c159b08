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


FMT_Q6K, FMT_Q5K = 1, 3              # the real model's shared-expert formats


def shared_fmts(down_fmt, sh_fmt):
    """(gate/up, down) formats of the shared expert: IQ2_XXS with the routed down format (sh_fmt 4), or
    the real model's Q5_K / Q6_K (sh_fmt 3)."""
    return (FMT_Q5K, FMT_Q6K) if sh_fmt == FMT_Q5K else (4, down_fmt)


def host_arena(oracle, seed, layer, experts, down_fmt=4, sh_fmt=4):
    """Compact host arenas (gate, up, down) holding `experts` in order, plus the shared expert; the routed
    down matrices in down_fmt (4 IQ2_XXS, 5 Q2_K, 6 Q3_K), the shared expert's formats from shared_fmts."""
    gate = np.concatenate([oracle.gen_iq2(seed, layer, 0, e, INTER, HIDDEN) for e in experts])
    up = np.concatenate([oracle.gen_iq2(seed, layer, 1, e, INTER, HIDDEN) for e in experts])
    down = np.concatenate([oracle.gen_matrix(down_fmt, seed, layer, 2, e, HIDDEN, INTER) for e in experts])
    gf, df = shared_fmts(down_fmt, sh_fmt)
    sh = (oracle.gen_matrix(gf, seed, layer, 0, 256, INTER, HIDDEN), oracle.gen_matrix(gf, seed, layer, 1, 256, INTER, HIDDEN),
          oracle.gen_matrix(df, seed, layer, 2, 256, HIDDEN, INTER))
    return gate, up, down, sh


def down_bytes(down_fmt):
    """Bytes of one expert's down matrix in down_fmt."""
    return HIDDEN * (INTER // 256) * {4: 66, 5: 84, 6: 110}[down_fmt]


def oracle_layer(oracle, seed, layer, x, resid, sel, w, with_shared=True, tokens=None, hq8=True, down_fmt=4, sh_fmt=4):
    """Oracle h/moe for routing (sel, w) with global expert ids, on the given tokens (default: all)."""
    tokens = list(range(x.shape[0])) if tokens is None else list(tokens)
    sel = np.asarray(sel)[tokens]
    used = sorted(set(int(e) for e in sel.reshape(-1)))
    remap = {e: i for i, e in enumerate(used)}
    ids = np.vectorize(lambda e: remap[int(e)])(sel).astype(np.int32)
    gate, up, down, sh = host_arena(oracle, seed, layer, used, down_fmt, sh_fmt)
    shg, shu, shd = sh if with_shared else (None, None, None)
    gf, df = shared_fmts(down_fmt, sh_fmt)
    return oracle.moe_layer(x[tokens], resid[tokens], gate, up, down, MAT, ids, np.asarray(w)[tokens], shg, shu, shd, hq8=hq8,
                            down_fmt=down_fmt, down_stride=down_bytes(down_fmt), sh_gu_fmt=gf, sh_down_fmt=df)


def oracle_layer_ggml(oracle, seed, layer, x, resid, sel, w, tokens=None, down_fmt=4, sh_fmt=4):
    """The oracle's ggml CPU mode (q8_K activations and h) for routing (sel, w) on the given tokens."""
    tokens = list(range(x.shape[0])) if tokens is None else list(tokens)
    sel = np.asarray(sel)[tokens]
    used = sorted(set(int(e) for e in sel.reshape(-1)))
    remap = {e: i for i, e in enumerate(used)}
    ids = np.vectorize(lambda e: remap[int(e)])(sel).astype(np.int32)
    gate, up, down, sh = host_arena(oracle, seed, layer, used, down_fmt, sh_fmt)
    gf, df = shared_fmts(down_fmt, sh_fmt)
    return oracle.moe_layer_ggml(x[tokens], resid[tokens], gate, up, down, MAT, ids, np.asarray(w)[tokens], *sh,
                                 down_fmt=down_fmt, down_stride=down_bytes(down_fmt), sh_gu_fmt=gf, sh_down_fmt=df)
