"""Python mirror of loki's fused-layer MoE calls (include/loki_fused_moe.h), the engine-facing ABI.

Host arrays in, host arrays out, exactly as server_core_fused.cpp drives src/fused_layer.h: per layer
fl_moe_prepare (the MoE half of fl_attn) -> fl_fetch(what=1) -> host keep-KE pass -> fl_moe, or for a wide
(prefill) pass fl_moe_prepare(wrow=...) per group -> fl_wide_moe per arena batch -> fl_wide_finish.
"""
import ctypes
import os

import numpy as np

from . import native as N
from .native import HIDDEN, lib

FL_IQ2, FL_Q2K, FL_Q3K = 4, 5, 6      # down formats (src/fused_layer.h:11)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _view(addr, n, dtype):
    if not addr:
        return None
    ct = {np.float32: ctypes.c_float, np.int32: ctypes.c_int32}[dtype]
    return np.ctypeslib.as_array(ctypes.cast(addr, ctypes.POINTER(ct)), shape=(n,))


def keep_pass(sel, wts, KE, renorm=True, scale=2.5, share=False, n_pad_from=None):
    """The engine's keep-KE compaction (src/server_core_fused.cpp:793-813) on host arrays [n][8]: each row's
    experts ordered by weight (descending; equal weights keep their position), the first KE kept, and with
    renorm their weights rescaled to sum to `scale`.

    share: the engine's --share-experts variant (server_core_fused.cpp:799-807), for n > 1 rows: every row
    keeps its own top min(2, KE); its remaining slots take, in weight order, experts that the set U already
    holds, then the highest-weight rest, each of which joins U.  U starts as the own top experts of the rows
    before n_pad_from (the engine's N_PAD_FROM; default every row).  The choice of a row depends on the rows
    beside it, so the engine turns it off for fixed-width passes; callers decide likewise."""
    sel = np.asarray(sel)
    wts = np.asarray(wts, np.float32)
    n = sel.shape[0]
    if KE >= sel.shape[1]:
        return sel.astype(np.int32), wts.astype(np.float32)
    order = np.argsort(-wts, axis=1, kind="stable")
    if share and n > 1:
        own = min(2, KE)
        npf = n if n_pad_from is None else min(n, n_pad_from)
        U = {int(sel[i, order[i, k]]) for i in range(npf) for k in range(own)}
        idx = np.empty((n, KE), np.int64)
        for i in range(n):
            pick = [int(order[i, k]) for k in range(own)]
            for k in range(own, sel.shape[1]):
                if len(pick) >= KE:
                    break
                if int(sel[i, order[i, k]]) in U:
                    pick.append(int(order[i, k]))
            for k in range(own, sel.shape[1]):
                if len(pick) >= KE:
                    break
                if int(order[i, k]) not in pick:
                    pick.append(int(order[i, k]))
                    U.add(int(sel[i, order[i, k]]))
            idx[i] = pick
    else:
        idx = order[:, :KE]
    s = np.take_along_axis(sel, idx, 1).astype(np.int32)
    w = np.take_along_axis(wts, idx, 1).astype(np.float32)
    if renorm:
        sw = np.zeros(w.shape[0], np.float32)
        for k in range(KE):
            sw = (sw + w[:, k]).astype(np.float32)
        f = np.where(sw > 1e-6, np.float32(scale) / np.where(sw > 1e-6, sw, 1), 1).astype(np.float32)
        w = (w * f[:, None]).astype(np.float32)
    return s, w


def pad_rows(sel, w, n_pad_from):
    """The engine's pad rows (src/server_core_fused.cpp:815): rows from n_pad_from on take row 0's experts at
    weight 0, so a fixed-width pass computes them without changing any output."""
    sel = np.array(sel, np.int32, copy=True)
    w = np.array(w, np.float32, copy=True)
    sel[n_pad_from:] = sel[0]
    w[n_pad_from:] = 0.0
    return sel, w


def union_remap(sel):
    """The engine's expert union and slot remap (src/server_core_fused.cpp:816-818): the sorted distinct
    expert ids of the pass (the arena's load list) and every entry's index into it (fl_moe's ids)."""
    sel = np.asarray(sel, np.int32)
    used = np.unique(sel)
    remap = np.full(256, -1, np.int32)
    remap[used] = np.arange(len(used), dtype=np.int32)
    return used.astype(np.int32), remap[sel]


_replay = None


def replay_lib():
    """libloki_replay.so: the engine-side C++ harness (keep pass, per-token call sequence) over this ABI."""
    global _replay
    if _replay is None:
        lib()
        L = ctypes.CDLL(os.path.join(os.path.dirname(N.LIB_PATH), "libloki_replay.so"))
        P, I = ctypes.c_void_p, ctypes.c_int
        L.lkr_keep.argtypes = [P, P, I, I, I, I, I, P, P]
        L.lkr_keep.restype = I
        L.lkr_decode.argtypes = [P, I, P, P, P, P, I, P, P, I, I, I, I, P, I]
        L.lkr_decode.restype = ctypes.c_double
        _replay = L
    return _replay


def keep_pass_native(sel, wts, KE, renorm=True, share=False, n_pad_from=None):
    """lkr_keep (the C++ keep pass the replay harness uses) on host arrays [n][8]."""
    sel = np.ascontiguousarray(sel, np.int32)
    wts = np.ascontiguousarray(wts, np.float32)
    n = sel.shape[0]
    s = np.empty((n, KE), np.int32)
    w = np.empty((n, KE), np.float32)
    rc = replay_lib().lkr_keep(_p(sel), _p(wts), n, KE, int(renorm), int(share), n if n_pad_from is None else n_pad_from,
                               _p(s), _p(w))
    assert rc == 0
    return s, w


def replay_decode(fc, layers, x, resid, KE, warmup, steps, down_fmt=FL_IQ2, device_keep=False):
    """The engine's per-token MoE call sequence over `layers` (LayerWeights with 256-expert arenas), driven
    from C++ (lkr_decode): fl_moe_prepare -> fl_fetch -> host keep pass -> fl_moe per layer, or with
    device_keep fl_moe_prepare -> fl_moe_auto.  x, resid: [L][n][7168] host arrays.  Returns (seconds of the
    timed steps, the last layer's h of the last step)."""
    L = len(layers)
    x = np.ascontiguousarray(x, np.float32)
    resid = np.ascontiguousarray(resid, np.float32)
    n = x.shape[1]
    mw = (N.FLMoeW * L)(*[N.FLMoeW(l.router_w.data_ptr(), 0, l.router_bias.data_ptr(), l.sh_gate, l.sh_up, l.sh_down,
                                   N.FMT_Q5K if getattr(l, "sh_fmt", N.FMT_IQ2) == N.FMT_Q5K else 0)
                          for l in layers])
    ptrs = lambda attr: (ctypes.c_void_p * L)(*[getattr(l, attr) for l in layers])
    h = np.empty((n, HIDDEN), np.float32)
    sec = replay_lib().lkr_decode(fc.c, L, mw, ptrs("gate"), ptrs("up"), ptrs("down"), down_fmt, _p(x), _p(resid), n, KE,
                                  warmup, steps, _p(h), 1 if device_keep else 0)
    if sec < 0:
        raise N.NativeError("lkr_decode failed (%g): fl_moe_error %d" % (sec, fc.error()))
    return sec, h


class FusedCtx:
    def __init__(self, kvp=512, sc_cap=64, stream=None):
        """stream: a cudaStream_t (int) the context runs on without owning it (lkfl_init_on_stream, the bridge's
        way of putting the MoE half on the attention context's stream); default: a stream of its own."""
        self.c = lib().fl_init(kvp, sc_cap) if stream is None else lib().lkfl_init_on_stream(ctypes.c_void_p(stream))
        if not self.c:
            raise N.NativeError("fl_init failed")
        self.out = N.FLOut()

    def adopt(self, ncur_ptr, ffn_ptr, parts_ptr, n_parts, part_rows, sel_ptr, wts_ptr, n, wrow=-1):
        """lkfl_moe_adopt: take over device rows left by an attention half (ncur, ffn_inp, top-8 ids / weights, the
        shared expert's output as n_parts partial sums [k][part_rows][7168]) instead of fl_moe_prepare."""
        P = ctypes.c_void_p
        lib().lkfl_moe_adopt(self.c, P(ncur_ptr), P(ffn_ptr), P(parts_ptr), n_parts, part_rows, P(sel_ptr), P(wts_ptr), n, wrow)

    def device_h(self):
        return lib().lkfl_device_h(self.c)

    def close(self):
        if self.c:
            lib().fl_free(self.c)
            self.c = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def error(self):
        return lib().fl_moe_error(self.c)

    def use_graphs(self, enable):
        lib().fl_use_graphs(self.c, int(enable))

    def prepare(self, mw, ncur, ffn_inp, wrow=-1):
        ncur = np.ascontiguousarray(ncur, np.float32)
        ffn_inp = np.ascontiguousarray(ffn_inp, np.float32)
        lib().fl_moe_prepare(self.c, ctypes.byref(mw), _p(ncur), _p(ffn_inp), ncur.shape[0], 1, wrow)

    def prepare_device(self, mw, ncur_ptr, ffn_ptr, n, wrow=-1):
        lib().fl_moe_prepare(self.c, ctypes.byref(mw), ctypes.c_void_p(ncur_ptr), ctypes.c_void_p(ffn_ptr), n, 0, wrow)

    def fetch(self, n, what=1):
        lib().fl_fetch(self.c, n, what, ctypes.byref(self.out))
        o = self.out
        r = {}
        if o.sel:
            r["sel"] = _view(o.sel, n * 8, np.int32).reshape(n, 8).copy()
            r["wts"] = _view(o.wts, n * 8, np.float32).reshape(n, 8).copy()
            r["ncur"] = _view(o.ncur, n * HIDDEN, np.float32).reshape(n, HIDDEN)
            r["fi"] = _view(o.fi, n * HIDDEN, np.float32).reshape(n, HIDDEN)
        if o.h:
            r["h"] = _view(o.h, n * HIDDEN, np.float32).reshape(n, HIDDEN)
        return r

    def moe(self, gate, up, down, nexp, ids, w, down_fmt=FL_IQ2):
        ids = np.ascontiguousarray(ids, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        n, KE = ids.shape
        lib().fl_moe(self.c, ctypes.c_void_p(gate), ctypes.c_void_p(up), ctypes.c_void_p(down), nexp, down_fmt, _p(ids), _p(w),
                     KE, n, ctypes.byref(self.out))
        o = self.out
        return (_view(o.h, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.h else None,
                _view(o.moe, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.moe else None)

    def moe_auto(self, gate, up, down, n, KE, renorm=True, down_fmt=FL_IQ2):
        """fl_moe_auto: the narrow pass routed on the device from the last prepare's router output."""
        lib().fl_moe_auto(self.c, ctypes.c_void_p(gate), ctypes.c_void_p(up), ctypes.c_void_p(down), down_fmt, KE, int(renorm), n,
                          ctypes.byref(self.out))
        o = self.out
        return (_view(o.h, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.h else None,
                _view(o.moe, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.moe else None)

    def skip(self, mo):
        mo = np.ascontiguousarray(mo, np.float32)
        lib().fl_skip(self.c, _p(mo), mo.shape[0], ctypes.byref(self.out))
        return _view(self.out.h, mo.shape[0] * HIDDEN, np.float32).reshape(-1, HIDDEN) if self.out.h else None

    def moe_outs(self, b, ids, w):
        ids = np.ascontiguousarray(ids, np.int32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty((len(ids), HIDDEN), np.float32)
        lib().fl_moe_outs(self.c, b, _p(ids), _p(w), len(ids), _p(out))
        return out

    def wide_init(self, wmax, KE):
        return lib().fl_wide_init(self.c, wmax, KE)

    def wide_moe(self, gate, up, down, nexp, midx, rows, kidx, wk, KE, par, down_fmt=FL_IQ2):
        midx = np.ascontiguousarray(midx, np.int32)
        rows = np.ascontiguousarray(rows, np.int32)
        kidx = np.ascontiguousarray(kidx, np.int32)
        wk = np.ascontiguousarray(wk, np.float32)
        lib().fl_wide_moe(self.c, ctypes.c_void_p(gate), ctypes.c_void_p(up), ctypes.c_void_p(down), down_fmt, nexp,
                          _p(midx), _p(rows), _p(kidx), _p(wk), len(midx), KE, par)

    def wide_mark(self, par):
        lib().fl_wide_mark(self.c, par)

    def wide_wait(self, par):
        lib().fl_wide_wait(self.c, par)

    def wide_finish(self, n, KE):
        lib().fl_wide_finish(self.c, n, KE, ctypes.byref(self.out))
        o = self.out
        return (_view(o.h, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.h else None,
                _view(o.moe, n * HIDDEN, np.float32).reshape(n, HIDDEN) if o.moe else None)

    def wide_skip(self, mo):
        mo = np.ascontiguousarray(mo, np.float32)
        lib().fl_wide_skip(self.c, _p(mo), mo.shape[0], ctypes.byref(self.out))
        return _view(self.out.h, mo.shape[0] * HIDDEN, np.float32).reshape(-1, HIDDEN) if self.out.h else None

    def wide_outs(self, row, KE):
        out = np.empty((KE, HIDDEN), np.float32)
        lib().fl_wide_outs(self.c, row, KE, _p(out))
        return out

    def gpu_ms(self, which):
        return lib().fl_gpu_ms(self.c, which)


def wide_slots(sel, w, KE, used, eb=16):
    """The engine's wide-pass batching (src/server_core_fused.cpp:937-946): per arena batch of <= eb experts
    from `used`, slots of <= 8 (row, k) pairs; returns [(batch_experts, midx, rows, kidx, wk)]."""
    byexp = {e: [] for e in used}
    n = sel.shape[0]
    for i in range(n):
        for k in range(KE):
            byexp[int(sel[i, k])].append((i, k))
    out = []
    for b0 in range(0, len(used), eb):
        batch = used[b0:b0 + eb]
        midx, rows, kidx, wk = [], [], [], []
        for u, e in enumerate(batch):
            lst = byexp[e]
            for i0 in range(0, len(lst), 8):
                midx.append(u)
                for j in range(8):
                    if i0 + j < len(lst):
                        r, k = lst[i0 + j]
                        rows.append(r); kidx.append(k); wk.append(w[r, k])
                    else:
                        rows.append(-1); kidx.append(0); wk.append(0.0)
        out.append((batch, midx, rows, kidx, wk))
    return out
