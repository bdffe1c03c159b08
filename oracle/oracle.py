"""ctypes binding of the CPU oracle (oracle.cpp).  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import this module; it is
the checker the CUDA path is compared against, never part of the product path.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

HIDDEN = 7168
MOE_INTER = 2048
N_EXPERTS = 256
QK = 256
BLK_IQ2 = 66
FMT_Q6K, FMT_Q5K, FMT_IQ2, FMT_Q2K, FMT_Q3K = 1, 3, 4, 5, 6
BLOCK_BYTES = {FMT_IQ2: 66, FMT_Q2K: 84, FMT_Q3K: 110, FMT_Q5K: 176, FMT_Q6K: 210}


def build(force=False):
    """Compile liboracle.so with the committed Makefile (g++, OpenMP)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


class RouteCfg(ctypes.Structure):
    _fields_ = [("n_experts", ctypes.c_int), ("topk", ctypes.c_int), ("keep", ctypes.c_int),
                ("renorm", ctypes.c_int), ("n_group", ctypes.c_int), ("topk_group", ctypes.c_int),
                ("scale", ctypes.c_float)]


class LayerW(ctypes.Structure):
    _fields_ = [("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("gate_stride", ctypes.c_int64), ("up_stride", ctypes.c_int64), ("down_stride", ctypes.c_int64),
                ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p), ("sh_down", ctypes.c_void_p)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        L.orc_iq2_dequant.argtypes = [P, ctypes.c_int64, P]
        L.orc_gen_iq2.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.orc_gen_d_only.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, P]
        L.orc_expf.argtypes = [ctypes.c_float]; L.orc_expf.restype = ctypes.c_float
        L.orc_f2h.argtypes = [ctypes.c_float]; L.orc_f2h.restype = ctypes.c_uint16
        L.orc_h2f.argtypes = [ctypes.c_uint16]; L.orc_h2f.restype = ctypes.c_float
        L.orc_quant_q8.argtypes = [P, ctypes.c_int64, P, P]
        L.orc_router_logits.argtypes = [P, ctypes.c_int, P, ctypes.c_int, ctypes.c_int, P]
        L.orc_router.argtypes = [P, ctypes.c_int, P, P, P, ctypes.POINTER(RouteCfg), P, P, P]
        L.orc_permute.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P]
        L.orc_iq2_matvec.argtypes = [P, ctypes.c_int, ctypes.c_int, P, P, P]
        L.orc_moe_layer.argtypes = [P, P, ctypes.c_int, ctypes.POINTER(LayerW), P, P, ctypes.c_int, P, P, P, P]
        L.orc_moe_layer.restype = ctypes.c_int
        L.orc_moe_layer_ex.argtypes = [P, P, ctypes.c_int, ctypes.POINTER(LayerW), P, P, ctypes.c_int, P, P, P, P, ctypes.c_int]
        L.orc_moe_layer_ex.restype = ctypes.c_int
        L.orc_moe_layer_fmt.argtypes = [P, P, ctypes.c_int, ctypes.POINTER(LayerW), P, P, ctypes.c_int, P, P, P, P, ctypes.c_int,
                                        ctypes.c_int]
        L.orc_moe_layer_fmt.restype = ctypes.c_int
        L.orc_moe_layer_fmt2.argtypes = L.orc_moe_layer_fmt.argtypes + [ctypes.c_int, ctypes.c_int]
        L.orc_moe_layer_fmt2.restype = ctypes.c_int
        L.orc_kq_dequant.argtypes = [ctypes.c_int, P, ctypes.c_int64, P]
        L.orc_gen_kq.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, P]
        L.orc_kq_matvec.argtypes = [ctypes.c_int, P, ctypes.c_int, ctypes.c_int, P, P, P]
        L.orc_quant_q8_K.argtypes = [P, ctypes.c_int64, P, P]
        L.orc_moe_layer_ggml.argtypes = [P, P, ctypes.c_int, ctypes.POINTER(LayerW), P, P, ctypes.c_int, P, P, P,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_moe_layer_ggml.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def iq2_dequant(blocks):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nblk = blocks.size // BLK_IQ2
    out = np.empty(nblk * QK, np.float32)
    lib().orc_iq2_dequant(_p(blocks), nblk, _p(out))
    return out


def gen_iq2(seed, layer, matrix, expert, rows, K):
    out = np.empty(rows * (K // QK) * BLK_IQ2, np.uint8)
    lib().orc_gen_iq2(seed, layer, matrix, expert, rows, K, _p(out))
    return out


def kq_dequant(fmt, blocks):
    """Q2_K (fmt 5), Q3_K (6), Q5_K (3) or Q6_K (1) blocks -> fp32 weights (gguf-py dequantize semantics)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nblk = blocks.size // BLOCK_BYTES[fmt]
    out = np.empty(nblk * QK, np.float32)
    lib().orc_kq_dequant(fmt, _p(blocks), nblk, _p(out))
    return out


def gen_kq(fmt, seed, layer, matrix, expert, rows, K):
    out = np.empty(rows * (K // QK) * BLOCK_BYTES[fmt], np.uint8)
    lib().orc_gen_kq(fmt, seed, layer, matrix, expert, rows, K, _p(out))
    return out


def gen_matrix(fmt, seed, layer, matrix, expert, rows, K):
    """Seeded matrix in any supported format (IQ2_XXS uses the IQ2 generator)."""
    return gen_iq2(seed, layer, matrix, expert, rows, K) if fmt == FMT_IQ2 else gen_kq(fmt, seed, layer, matrix, expert, rows, K)


def kq_matvec(fmt, W, rows, K, xq, xd):
    y = np.empty(rows, np.float32)
    lib().orc_kq_matvec(fmt, _p(np.ascontiguousarray(W, np.uint8)), rows, K, _p(np.ascontiguousarray(xq, np.int8)),
                        _p(np.ascontiguousarray(xd, np.float32)), _p(y))
    return y


def quant_q8(x):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 32, np.float32)
    lib().orc_quant_q8(_p(x), x.size, _p(q), _p(d))
    return q, d


def router_logits(x, W):
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.float32)
    T = x.shape[0]
    out = np.empty((T, W.shape[0]), np.float32)
    lib().orc_router_logits(_p(x), T, _p(W), W.shape[0], x.shape[1], _p(out))
    return out


def route_cfg(topk=8, keep=8, renorm=1, n_group=1, topk_group=1, scale=2.5, n_experts=N_EXPERTS):
    return RouteCfg(n_experts, topk, keep, renorm, n_group, topk_group, scale)


def router(x, W, bias, cfg, logits=None):
    """Returns (probs [T,NE], sel [T,keep], w [T,keep])."""
    bias = np.ascontiguousarray(bias, np.float32)
    if logits is not None:
        logits = np.ascontiguousarray(logits, np.float32)
        T = logits.shape[0]
        xs = None
    else:
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        xs = x
    W = None if W is None else np.ascontiguousarray(W, np.float32)
    probs = np.empty((T, cfg.n_experts), np.float32)
    sel = np.empty((T, cfg.keep), np.int32)
    w = np.empty((T, cfg.keep), np.float32)
    lib().orc_router(_p(xs), T, _p(W), _p(logits), _p(bias), ctypes.byref(cfg), _p(probs), _p(sel), _p(w))
    return probs, sel, w


def permute(sel, n_experts=N_EXPERTS):
    sel = np.ascontiguousarray(sel, np.int32)
    T, KE = sel.shape
    counts = np.empty(n_experts, np.int32)
    offsets = np.empty(n_experts + 1, np.int32)
    perm = np.empty(T * KE, np.int32)
    lib().orc_permute(_p(sel), T, KE, n_experts, _p(counts), _p(offsets), _p(perm))
    return counts, offsets, perm


def iq2_matvec(W, rows, K, xq, xd):
    y = np.empty(rows, np.float32)
    lib().orc_iq2_matvec(_p(np.ascontiguousarray(W, np.uint8)), rows, K, _p(np.ascontiguousarray(xq, np.int8)),
                         _p(np.ascontiguousarray(xd, np.float32)), _p(y))
    return y


def moe_layer(x, resid, gate, up, down, stride, ids, w, sh_gate=None, sh_up=None, sh_down=None, want_slots=False, hq8=True,
              down_fmt=FMT_IQ2, down_stride=None, sh_gu_fmt=FMT_IQ2, sh_down_fmt=None):
    """Reference MoE layer on arena-layout weights (expert m at m*stride bytes of each arena).

    Returns dict(h, moe[, y_slot, shared]).  ids/w: [T, KE] expert ids (arena slots) and weights.
    hq8: re-quantise the SwiGLU output to q8 before the down projection (reference semantics; the
    tensor-core prefill path keeps it at 16-bit precision: hq8=False).  down_fmt: format of every down
    matrix (routed and shared); down_stride: the down arena's expert stride (default `stride`).
    sh_gu_fmt / sh_down_fmt: the shared expert's formats (default IQ2_XXS and down_fmt; the real model's are
    FMT_Q5K and FMT_Q6K)."""
    x = np.ascontiguousarray(x, np.float32)
    resid = np.ascontiguousarray(resid, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    T, KE = ids.shape
    lw = LayerW(_p(gate).value, _p(up).value, _p(down).value, stride, stride, stride if down_stride is None else down_stride,
                None if sh_gate is None else _p(sh_gate).value,
                None if sh_up is None else _p(sh_up).value,
                None if sh_down is None else _p(sh_down).value)
    h = np.empty((T, HIDDEN), np.float32)
    moe = np.empty((T, HIDDEN), np.float32)
    ys = np.empty((T, KE, HIDDEN), np.float32) if want_slots else None
    sh = np.empty((T, HIDDEN), np.float32) if want_slots else None
    rc = lib().orc_moe_layer_fmt2(_p(x), _p(resid), T, ctypes.byref(lw), _p(ids), _p(w), KE, _p(h), _p(moe), _p(ys), _p(sh),
                                  1 if hq8 else 0, down_fmt, sh_gu_fmt, down_fmt if sh_down_fmt is None else sh_down_fmt)
    assert rc == 0
    out = {"h": h, "moe": moe}
    if want_slots:
        out["y_slot"] = ys
        out["shared"] = sh
    return out


def quant_q8_K(x):
    """ggml's q8_K of x (len % 256 == 0): codes int8 [n], scales float32 [n/256] (orc_quant_q8_K)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 256, np.float32)
    lib().orc_quant_q8_K(_p(x), x.size, _p(q), _p(d))
    return q, d


def moe_layer_ggml(x, resid, gate, up, down, stride, ids, w, sh_gate=None, sh_up=None, sh_down=None, down_fmt=FMT_IQ2,
                   down_stride=None, sh_gu_fmt=FMT_IQ2, sh_down_fmt=None):
    """moe_layer's arguments in ggml's CPU numerics (q8_K activations and h, fp32 combine in k order;
    orc_moe_layer_ggml).  Returns dict(h, moe, shared)."""
    x = np.ascontiguousarray(x, np.float32)
    resid = np.ascontiguousarray(resid, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    w = np.ascontiguousarray(w, np.float32)
    T, KE = ids.shape
    lw = LayerW(_p(gate).value, _p(up).value, _p(down).value, stride, stride, stride if down_stride is None else down_stride,
                None if sh_gate is None else _p(sh_gate).value,
                None if sh_up is None else _p(sh_up).value,
                None if sh_down is None else _p(sh_down).value)
    h = np.empty((T, HIDDEN), np.float32)
    moe = np.empty((T, HIDDEN), np.float32)
    sh = np.empty((T, HIDDEN), np.float32)
    rc = lib().orc_moe_layer_ggml(_p(x), _p(resid), T, ctypes.byref(lw), _p(ids), _p(w), KE, _p(h), _p(moe), _p(sh),
                                  down_fmt, sh_gu_fmt, down_fmt if sh_down_fmt is None else sh_down_fmt)
    assert rc == 0
    return {"h": h, "moe": moe, "shared": sh}
