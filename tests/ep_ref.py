"""Test-side pieces of the expert-parallel protocol tests (not part of the package).

RefEpOps: the per-rank stages of loki_b200.ep.EpMoeLayer restated on the CPU with numpy and the oracle
(the checker), on the same row format as the CUDA path (include/loki_ep.h), so that the exchange logic of
EpMoeLayer.forward runs unchanged over gloo.
ThreadComm: an in-process all-to-all between threads, one per emulated rank, for running several ranks'
CUDA stages on one GPU.
"""
import threading

import numpy as np
import torch

from moe_helpers import HIDDEN, INTER, MAT

ROW_HDR = 64
ROW_Q = ROW_HDR                       # int8 q8 codes [HIDDEN]
ROW_D = ROW_HDR + HIDDEN              # fp32 scales [HIDDEN / 32]
ROW_BYTES = ROW_D + HIDDEN // 32 * 4
N_EXPERTS = 256


def _row_x(rows):
    """fp32 activations of rows: q * d per 32 (what the CUDA path's experts read back)."""
    q = rows[:, ROW_Q:ROW_D].copy().view(np.int8).astype(np.float32)
    d = rows[:, ROW_D:].copy().view(np.float32)
    return (q.reshape(len(rows), HIDDEN // 32, 32) * d[:, :, None]).reshape(len(rows), HIDDEN)


class RefShard:
    """Rank `rank`'s view of one layer: router, shared expert and experts [rank*E, (rank+1)*E)."""

    def __init__(self, oracle, seed, layer, rank, n_ranks, router_w, router_bias):
        self.oracle, self.seed, self.layer = oracle, seed, layer
        self.n_local = N_EXPERTS // n_ranks
        self.expert0 = rank * self.n_local
        self.router_w, self.router_bias = router_w, router_bias
        self._cache = {}

    def matrices(self, e):
        """(gate, up, down) bytes of global expert e (256 = shared)."""
        if e not in self._cache:
            g = self.oracle.gen_iq2
            self._cache[e] = (g(self.seed, self.layer, 0, e, INTER, HIDDEN), g(self.seed, self.layer, 1, e, INTER, HIDDEN),
                              g(self.seed, self.layer, 2, e, HIDDEN, INTER))
        return self._cache[e]


class RefEpOps:
    def __init__(self, oracle, n_ranks, cfg):
        self.oracle, self.n_ranks, self.cfg = oracle, n_ranks, cfg

    def route(self, W, x, logits_override=None):
        lo = None if logits_override is None else logits_override.numpy()
        _, sel, w = self.oracle.router(x.numpy(), W.router_w, W.router_bias, self.cfg, logits=lo)
        return torch.from_numpy(sel), torch.from_numpy(w)

    def pack(self, sel, w, x, cap, self_rank):
        sel, w, x = sel.numpy(), w.numpy(), x.numpy()
        T, keep = sel.shape
        NR, epr = self.n_ranks, N_EXPERTS // self.n_ranks
        q, dq = self.oracle.quant_q8(x) if T else (np.zeros(0, np.int8), np.zeros(0, np.float32))
        q, dq = q.reshape(T, HIDDEN), dq.reshape(T, HIDDEN // 32)
        owner = sel // epr
        lists = [[t for t in range(T) if d == self_rank or (owner[t] == d).any()] for d in range(NR)]
        counts = np.array([len(l) for l in lists], np.int32)
        offs = np.concatenate([[0], np.cumsum([cap if cap else c for c in counts])]).astype(np.int64)
        rows = NR * cap if cap else T * NR
        send = np.zeros((max(rows, 1), ROW_BYTES), np.uint8)
        row_map = np.full((T, NR), -1, np.int32)
        for d in range(NR):
            if cap:
                for r in range(counts[d], cap):
                    send[offs[d] + r, :32] = np.full(8, -1, np.int32).view(np.uint8)
            for j, t in enumerate(lists[d]):
                row = offs[d] + j
                row_map[t, d] = row
                mine = owner[t] == d
                hs = np.full(8, -1, np.int32)
                hw = np.zeros(8, np.float32)
                hs[:keep] = np.where(mine, sel[t] - d * epr, -1)
                hw[:keep] = np.where(mine, w[t], 0)
                send[row, :32] = hs.view(np.uint8)
                send[row, 32:64] = hw.view(np.uint8)
                send[row, ROW_Q:ROW_D] = q[t].view(np.uint8)
                send[row, ROW_D:] = dq[t].view(np.uint8)
        return torch.from_numpy(send), torch.from_numpy(counts), torch.from_numpy(row_map)

    def _shared(self, W, x):
        T = x.shape[0]
        g, u, dn = W.matrices(W.expert0)
        sg, su, sd = W.matrices(N_EXPERTS)
        out = self.oracle.moe_layer(x, np.zeros_like(x), g, u, dn, MAT, np.zeros((T, 1), np.int32),
                                    np.zeros((T, 1), np.float32), sg, su, sd)
        return out["h"]

    def experts(self, W, recv, R, keep, shared_row0=0, shared_rows=0):
        recv = recv.numpy()
        ret = np.zeros((R, HIDDEN), np.float32)
        shared = np.zeros((shared_rows, HIDDEN), np.float32)
        if shared_rows:
            shared = self._shared(W, _row_x(recv[shared_row0:shared_row0 + shared_rows]))
        ret, shared = self._routed(W, recv, R, keep, ret), torch.from_numpy(shared)
        return ret, shared

    def _routed(self, W, recv, R, keep, ret):
        if R == 0:
            return torch.from_numpy(ret)
        sel = recv[:, :32].copy().view(np.int32)[:, :keep]
        w = recv[:, 32:64].copy().view(np.float32)[:, :keep]
        x = _row_x(recv)
        live = [r for r in range(R) if (sel[r] >= 0).any()]
        if not live:
            return torch.from_numpy(ret)
        used = sorted(set(int(e) for e in sel[live].reshape(-1) if e >= 0))
        slot = {e: i for i, e in enumerate(used)}
        ids = np.array([[slot.get(int(e), 0) for e in sel[r]] for r in live], np.int32)
        ww = np.where(sel[live] >= 0, w[live], 0).astype(np.float32)
        mats = [W.matrices(W.expert0 + e) for e in used]
        g, u, dn = (np.concatenate([m[i] for m in mats]) for i in range(3))
        out = self.oracle.moe_layer(x[live], np.zeros((len(live), HIDDEN), np.float32), g, u, dn, MAT, ids, ww)
        ret[live] = out["moe"]
        return torch.from_numpy(ret)

    def combine(self, ret_home, row_map, hpart, shared=None):
        ret_home, row_map, hpart = ret_home.numpy(), row_map.numpy(), hpart.numpy()
        T = row_map.shape[0]
        acc = np.zeros((T, HIDDEN), np.float32)
        for d in range(self.n_ranks):
            for t in range(T):
                if row_map[t, d] >= 0:
                    acc[t] += ret_home[row_map[t, d]]
        base = hpart if shared is None else hpart + shared.numpy()
        return torch.from_numpy(base + acc), torch.from_numpy(acc)


class _Done:
    def wait(self):
        pass


class ThreadComm:
    """all_to_all among `size` threads of one process (emulated ranks on one device, one CUDA stream)."""

    class _Hub:
        def __init__(self, size):
            self.size = size
            self.barrier = threading.Barrier(size)
            self.slots = [None] * size

    def __init__(self, hub, rank):
        self.hub, self.rank, self.size = hub, rank, hub.size

    @classmethod
    def group(cls, size):
        hub = cls._Hub(size)
        return [cls(hub, r) for r in range(size)]

    def all_to_all(self, out, inp, out_splits=None, in_splits=None, async_op=False):
        n = self.size
        if in_splits is None:
            in_splits = [inp.shape[0] // n] * n
        if out_splits is None:
            out_splits = [out.shape[0] // n] * n
        self.hub.slots[self.rank] = (inp, list(in_splits))
        self.hub.barrier.wait()
        o = 0
        for src in range(n):
            sinp, ssplits = self.hub.slots[src]
            s0 = sum(ssplits[:self.rank])
            k = ssplits[self.rank]
            assert k == out_splits[src]
            if k:
                out[o:o + k].copy_(sinp[s0:s0 + k])
            o += k
        self.hub.barrier.wait()
        return _Done()
