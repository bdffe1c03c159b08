"""Expert-parallel MoE layer: 256 routed experts sharded over the GPUs of one node (include/loki_ep.h).

No counterpart in the reference, which runs one GPU and streams experts from NVMe
(src/moe_stream_buffer.h).  Rank r keeps experts [r*E, (r+1)*E) (E = 256 / n_ranks) resident, plus
the router and the shared expert.  Tokens stay on their home rank; one layer is

    home   route -> pack rows per owner rank (every token also gets a row to its own rank)
    exchange #1: rows (all-to-all)
    owner  expert stage on the received rows -> per-row partial sums; the rows from this rank itself also
           get the shared expert, in the same launches
    exchange #2: partial sums (all-to-all, the transpose of #1)
    home   combine: h = resid + shared + sum over ranks, moe = sum over ranks

The exchanges go through a communicator with torch.distributed's all_to_all_single signature: NativeComm
(the library's own NCCL communicator, grouped send/recv over NVLink, capturable in a CUDA graph), TorchComm
(a torch.distributed process group: NCCL, or gloo in the CPU protocol tests).  Two row layouts: fixed capacity (block d holds up to
`cap` rows, so no count exchange and no host synchronisation: decode, CUDA-graph friendly) and compact
(block sizes exchanged first; the host learns them with one device->host copy: batch prefill).

`ops` supplies the per-rank stages.  `NativeEpOps` runs them in libloki_moe.so on one GPU; it is the only
implementation the package ships.
"""
import ctypes

import torch
import torch.distributed as dist

from . import native as N
from .moe import MoeLayer, _ptr, _stream
from .native import HIDDEN, N_EXPERTS, EP_ROW_BYTES, EP_IPC_HANDLE_BYTES, check, lib


class TorchComm:
    """all-to-all over a torch.distributed process group (NCCL on GPUs)."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    def all_to_all(self, out, inp, out_splits=None, in_splits=None, async_op=False):
        return dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group, async_op=async_op)


class _Done:
    def wait(self):
        pass


class NativeComm:
    """all-to-all through libloki_moe.so's NCCL communicator (include/loki_ep.h lk_ep_all_to_all): stream-ordered
    on the current CUDA stream, so it can sit inside a captured CUDA graph.  The NCCL id is made on rank 0
    and broadcast over the default torch.distributed group."""

    def __init__(self, device):
        self.rank, self.size = dist.get_rank(), dist.get_world_size()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        idb = ctypes.create_string_buffer(N.EP_COMM_ID_BYTES)
        if self.rank == 0:
            check(lib().lk_ep_comm_id(idb))
        obj = [idb.raw if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, device=self.device)
        idb = ctypes.create_string_buffer(obj[0], N.EP_COMM_ID_BYTES)
        h = ctypes.c_void_p()
        check(lib().lk_ep_comm_create(idb, self.size, self.rank, self.device.index or 0, ctypes.byref(h)))
        self.comm = h

    def close(self):
        if self.comm:
            lib().lk_ep_comm_destroy(self.comm)
            self.comm = None

    def all_to_all(self, out, inp, out_splits=None, in_splits=None, async_op=False):
        n = self.size
        if in_splits is None and out_splits is None:
            assert out.numel() * out.element_size() == inp.numel() * inp.element_size()
            block = inp.numel() * inp.element_size() // n
            check(lib().lk_ep_all_to_all(self.comm, _ptr(inp), _ptr(out), None, None, None, None, block, _stream()))
            return _Done()
        rin = inp[0].numel() * inp.element_size() if inp.dim() > 1 else inp.element_size()
        rout = out[0].numel() * out.element_size() if out.dim() > 1 else out.element_size()
        arr = ctypes.c_int64 * n
        sb = arr(*[s * rin for s in in_splits])
        so = arr(*[sum(in_splits[:d]) * rin for d in range(n)])
        rb = arr(*[s * rout for s in out_splits])
        ro = arr(*[sum(out_splits[:d]) * rout for d in range(n)])
        check(lib().lk_ep_all_to_all(self.comm, _ptr(inp) if inp.numel() else None, _ptr(out) if out.numel() else None,
                                     so, sb, ro, rb, 0, _stream()))
        return _Done()


class P2PExchange:
    """The peer-memory exchange of fixed-capacity (decode) layers: a mailbox per rank in HBM, exported with
    CUDA IPC and mapped by every peer (include/loki_ep.h lk_ep_mailbox_* / lk_ep_p2p_*).  `cap`: the largest
    per-rank token count it serves.  Collective: every rank of the default group constructs it."""

    def __init__(self, device, cap):
        self.rank, self.size = dist.get_rank(), dist.get_world_size()
        self.cap = cap
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        h = ctypes.create_string_buffer(EP_IPC_HANDLE_BYTES)
        mb = ctypes.c_void_p()
        check(lib().lk_ep_mailbox_create(self.size, self.rank, cap, dev.index or 0, ctypes.byref(mb), h))
        self.mb = mb
        handles = [None] * self.size
        dist.all_gather_object(handles, h.raw)
        check(lib().lk_ep_mailbox_connect(self.mb, b"".join(handles)))
        dist.barrier()                                  # every mailbox mapped everywhere before any traffic

    def close(self):
        if self.mb:
            torch.cuda.synchronize()
            dist.barrier()                              # no peer still writes into our mailbox
            lib().lk_ep_mailbox_destroy(self.mb)
            self.mb = None


class NativeEpOps:
    """The per-rank stages on one GPU: a 256-expert home context (router, shared expert) and an expert
    context over this rank's shard."""

    def __init__(self, device, n_ranks, max_local_tokens, topk=8, keep=8, renorm=True, n_group=1, topk_group=1,
                 scale=2.5):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.n_ranks, self.keep = n_ranks, keep
        self.home = MoeLayer(self.device, topk, keep, renorm, n_group, topk_group, scale, with_shared=True,
                             max_tokens=max_local_tokens)
        # the shard context never routes (rows arrive with their experts chosen), so it takes the plain
        # routing configuration whatever the home context's grouped mode
        self.expert = MoeLayer(self.device, topk, keep, renorm, 1, 1, scale, with_shared=True,
                               max_tokens=max(1, n_ranks * max_local_tokens), n_experts=N_EXPERTS // n_ranks)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def set_gemm_threshold(self, min_tokens):
        self.home.set_gemm_threshold(min_tokens)
        self.expert.set_gemm_threshold(min_tokens)

    def set_mma_threshold(self, min_tokens):
        self.home.set_mma_threshold(min_tokens)
        self.expert.set_mma_threshold(min_tokens)

    def route(self, W, x, logits_override=None):
        _, sel, w = self.home.route(W, x, logits_override=logits_override)
        return sel, w

    def pack(self, sel, w, x, cap, self_rank):
        T = x.shape[0]
        rows = self.n_ranks * cap if cap else T * self.n_ranks
        send = torch.empty(max(rows, 1), EP_ROW_BYTES, dtype=torch.uint8, device=self.device)
        counts = torch.empty(self.n_ranks, dtype=torch.int32, device=self.device)
        row_map = torch.empty(T, self.n_ranks, dtype=torch.int32, device=self.device)
        check(lib().lk_ep_pack(_ptr(sel), _ptr(w), _ptr(x), T, sel.shape[1], self.n_ranks, self_rank, cap, _ptr(send),
                               _ptr(counts), _ptr(row_map), _ptr(self.err), _stream()))
        return send, counts, row_map

    def shared(self, W, x, resid):
        hpart = torch.empty(x.shape[0], HIDDEN, device=self.device)
        ws = W.struct()
        self.home._check(lib().lk_ep_shared(self.home.ctx, ctypes.byref(ws), _ptr(x), _ptr(resid), x.shape[0], _ptr(hpart),
                                            _stream()))
        return hpart

    def experts(self, W, recv, R, keep, shared_row0=0, shared_rows=0):
        """Routed partial sums of the R received rows (a tensor or a device address), and the shared expert
        of rows [shared_row0, +shared_rows)."""
        ret = torch.empty(max(R, 1), HIDDEN, device=self.device)
        shared = torch.empty(max(shared_rows, 1), HIDDEN, device=self.device)
        ws = W.struct()
        rows = recv if isinstance(recv, ctypes.c_void_p) else _ptr(recv)
        self.expert._check(lib().lk_ep_experts(self.expert.ctx, ctypes.byref(ws), rows, R, keep, shared_row0,
                                               shared_rows, _ptr(ret), _ptr(shared), _stream()))
        return ret[:R], shared[:shared_rows]

    def p2p_route_dispatch(self, p2p, W, x, logits_override=None):
        """Routing and the peer-memory send as the router's one launch (one token): (sel, w, row_map), or None
        where that path does not apply (then route + p2p_layer)."""
        T = x.shape[0]
        sel = torch.empty(T, self.home.keep, dtype=torch.int32, device=self.device)
        w = torch.empty(T, self.home.keep, device=self.device)
        row_map = torch.empty(T, self.n_ranks, dtype=torch.int32, device=self.device)
        ws = W.struct()
        rc = lib().lk_ep_p2p_route_dispatch(p2p.mb, self.home.ctx, ctypes.byref(ws), _ptr(x), T, _ptr(logits_override),
                                            _ptr(sel), _ptr(w), _ptr(row_map), _ptr(self.err), _stream())
        if rc == N.LK_ERR_UNSUPPORTED:
            return None
        self.home._check(rc)
        return sel, w, row_map

    def p2p_layer(self, p2p, W, x, resid, sel, w, row_map=None):
        """One fixed-capacity layer over the peer-memory exchange (after routing; row_map given: after the
        dispatch too): h, moe."""
        T, keep, NR = x.shape[0], sel.shape[1], self.n_ranks
        if row_map is None:
            row_map = torch.empty(T, NR, dtype=torch.int32, device=self.device)
            check(lib().lk_ep_p2p_dispatch(p2p.mb, _ptr(sel), _ptr(w), _ptr(x), T, keep, _ptr(row_map), _ptr(self.err),
                                           _stream()))
        shared = torch.empty(max(T, 1), HIDDEN, device=self.device)
        ws = W.struct()
        rc = lib().lk_ep_p2p_experts(p2p.mb, self.expert.ctx, ctypes.byref(ws), keep, T, _ptr(shared), _ptr(self.err),
                                     _stream())
        h = torch.empty(T, HIDDEN, device=self.device)
        moe = torch.empty(T, HIDDEN, device=self.device)
        if rc == N.LK_ERR_UNSUPPORTED:                 # a batch-sized or K-quant-shared expert stage: separate calls
            rows = ctypes.c_void_p()
            check(lib().lk_ep_p2p_rows(p2p.mb, ctypes.byref(rows), _ptr(self.err), _stream()))
            partial, shared = self.experts(W, rows, NR * p2p.cap, keep, p2p.rank * p2p.cap, T)
            check(lib().lk_ep_p2p_return(p2p.mb, _ptr(partial), _stream()))
            check(lib().lk_ep_p2p_combine(p2p.mb, _ptr(row_map), T, _ptr(resid), _ptr(shared), _ptr(h), _ptr(moe),
                                          _ptr(self.err), _stream()))
        else:                                          # the direct return: entry rows in this rank's mailbox
            self.expert._check(rc)
            check(lib().lk_ep_p2p_combine_entries(p2p.mb, _ptr(sel), keep, _ptr(row_map), T, _ptr(resid), _ptr(shared),
                                                  _ptr(h), _ptr(moe), _ptr(self.err), _stream()))
        return h, moe

    def combine(self, ret_home, row_map, hpart, shared=None):
        T = row_map.shape[0]
        h = torch.empty(T, HIDDEN, device=self.device)
        moe = torch.empty(T, HIDDEN, device=self.device)
        check(lib().lk_ep_combine(_ptr(ret_home), _ptr(row_map), T, self.n_ranks, _ptr(hpart), _ptr(shared), _ptr(h),
                                  _ptr(moe), _stream()))
        return h, moe

    def device_error(self):
        self.home.device_error()
        self.expert.device_error()
        e = int(self.err.item())
        if e:
            self.err.zero_()
            raise N.NativeError("expert-parallel pack: device error code %d" % e)


class EpMoeLayer:
    """One expert-parallel MoE layer call per rank.

    comm: TorchComm (or any object with its all_to_all); ops: NativeEpOps.  `fixed_cap_max`: calls with at
    most this many local tokens use the fixed-capacity layout (every rank must then pass the same T).
    `p2p`: a P2PExchange -- fixed-capacity calls of at most p2p.cap tokens then use the peer-memory exchange
    instead of the communicator."""

    def __init__(self, comm, ops, fixed_cap_max=8, p2p=None):
        self.comm, self.ops, self.p2p = comm, ops, p2p
        self.n_ranks = comm.size
        self.fixed_cap_max = fixed_cap_max
        self.last_counts = None          # (rows sent per rank, rows received per rank) of the last compact call

    def forward(self, W, x, resid, logits_override=None):
        """W: this rank's LayerWeights shard (router + shared expert + experts [r*E, (r+1)*E)); x, resid:
        [T][7168] fp32 home tokens.  Returns h, moe ([T][7168]), sel, w ([T][keep] global ids)."""
        ops, comm, NR = self.ops, self.comm, self.n_ranks
        T = x.shape[0]
        me = comm.rank
        if self.p2p is not None and T <= self.p2p.cap:
            fused = ops.p2p_route_dispatch(self.p2p, W, x, logits_override) if T == 1 else None
            if fused is not None:
                sel, w, row_map = fused
                h, moe = ops.p2p_layer(self.p2p, W, x, resid, sel, w, row_map)
            else:
                sel, w = ops.route(W, x, logits_override)
                h, moe = ops.p2p_layer(self.p2p, W, x, resid, sel, w)
            return h, moe, sel, w
        sel, w = ops.route(W, x, logits_override)
        keep = sel.shape[1]
        fixed = T <= self.fixed_cap_max
        cap = T if fixed else 0
        send, counts, row_map = ops.pack(sel, w, x, cap, me)
        if fixed:
            recv = torch.empty(NR * cap, EP_ROW_BYTES, dtype=torch.uint8, device=send.device)
            comm.all_to_all(recv, send[:NR * cap])
            sent, got = None, None
            own0 = me * cap                                            # this rank's own rows in the receive buffer
        else:
            rcounts = torch.empty_like(counts)
            comm.all_to_all(rcounts, counts)
            both = torch.cat([counts, rcounts]).cpu().tolist()          # the one host synchronisation
            sent, got = both[:NR], both[NR:]
            self.last_counts = (sent, got)
            recv = torch.empty(sum(got), EP_ROW_BYTES, dtype=torch.uint8, device=send.device)
            comm.all_to_all(recv, send[:sum(sent)], got, sent)
            own0 = sum(got[:me])
        R = recv.shape[0]
        ret, shared = ops.experts(W, recv, R, keep, own0, T)           # + the shared expert of the own T rows
        ret_home = torch.empty(NR * cap if fixed else sum(sent), HIDDEN, dtype=ret.dtype, device=ret.device)
        comm.all_to_all(ret_home, ret, sent, got)
        h, moe = ops.combine(ret_home, row_map, resid, shared)
        return h, moe, sel, w
