"""Expert-parallel layer on the CUDA path (include/loki_ep.h through loki_b200.ep) against the oracle.

* emulated ranks: 2 or 4 ranks as threads on one GPU (ThreadComm), each with its own 256/N-expert shard
  and contexts: the pack / expert / shared / combine kernels and the exchange logic, on one device;
* NCCL: 2 processes on 2 GPUs (skipped with fewer), the real all-to-all over NVLink, through the library's
  own communicator (NativeComm, also replayed from a captured CUDA graph) and through torch.distributed.
Routing must match the oracle bit-exactly; h / moe within RTOL_L2 of the single-GPU oracle layer.
"""
import os
import socket
import threading

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, RTOL_L2, rel_l2, oracle_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _inputs(T_loc, rank):
    rng = np.random.default_rng(500 + 7 * T_loc + rank)
    return (rng.standard_normal((T_loc, HIDDEN)).astype(np.float32),
            rng.standard_normal((T_loc, HIDDEN)).astype(np.float32))


def _check_rank(oracle, W, x, r, h, moe, sel, w, keep=8, n_group=1):
    sel, w = sel.cpu().numpy(), w.cpu().numpy()
    Wr = W.router_w.float().cpu().numpy()
    bias = W.router_bias.cpu().numpy()
    _, osel, ow = oracle.router(x, Wr, bias, oracle.route_cfg(8, keep, 1, n_group, 4 if n_group > 1 else 1))
    np.testing.assert_array_equal(sel, osel)
    np.testing.assert_array_equal(w, ow)
    ref = oracle_layer(oracle, SEED, 0, x, r, sel, w)
    e_moe, e_h = rel_l2(moe.cpu().numpy(), ref["moe"]), rel_l2(h.cpu().numpy(), ref["h"])
    assert e_moe < RTOL_L2 and e_h < RTOL_L2, (e_moe, e_h)


@pytest.mark.parametrize("n_ranks,T_loc,fixed_cap_max,n_group", [(2, 1, 8, 1), (2, 5, 8, 1), (4, 3, 8, 1), (2, 12, 4, 1),
                                                                 (2, 5, 8, 8), (4, 1, 8, 8)])
def test_ep_emulated_ranks_one_gpu(native, oracle, n_ranks, T_loc, fixed_cap_max, n_group):
    """n_group = 8: the DeepSeek-V3 grouped routing on the home rank (the shard contexts never route)."""
    from loki_b200.moe import LayerWeights
    from loki_b200.ep import EpMoeLayer, NativeEpOps
    from ep_ref import ThreadComm
    E = 256 // n_ranks
    comms = ThreadComm.group(n_ranks)
    shards = [LayerWeights("cuda", SEED, 0, n_experts=E, expert0=r * E) for r in range(n_ranks)]
    ops = [NativeEpOps(0, n_ranks, T_loc, n_group=n_group, topk_group=4 if n_group > 1 else 1) for _ in range(n_ranks)]
    for o in ops:
        o.set_gemm_threshold(1 << 20)              # the matvec path: same q8 scheme as the oracle
        o.set_mma_threshold(1 << 20)
    inputs = [_inputs(T_loc, r) for r in range(n_ranks)]
    torch.cuda.synchronize()
    out, errs = [None] * n_ranks, []

    def run(rank):
        try:
            layer = EpMoeLayer(comms[rank], ops[rank], fixed_cap_max=fixed_cap_max)
            x, r = (torch.from_numpy(a).cuda() for a in inputs[rank])
            out[rank] = layer.forward(shards[rank], x, r)
        except Exception as e:                     # surfaced below
            errs.append(e)
            comms[rank].hub.barrier.abort()

    th = [threading.Thread(target=run, args=(k,)) for k in range(n_ranks)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=600)
    assert not errs, errs
    torch.cuda.synchronize()
    for rank in range(n_ranks):
        ops[rank].device_error()
        _check_rank(oracle, shards[rank], *inputs[rank], *out[rank], n_group=n_group)


@pytest.mark.parametrize("n_ranks,T_loc", [(2, 256), (4, 96)])
def test_ep_emulated_ranks_batch_regime(native, oracle, n_ranks, T_loc):
    """BASELINE config 3's path on emulated ranks with the default thresholds: every shard receives a few hundred
    rows, so its experts run the batch regime (the q8 gate/up on tcgen05, then the tcgen05 or mma.sync down) on
    the compact row layout; routing bit-exact, h / moe within RTOL_L2 of the oracle with the reference's numerics
    on sampled tokens of every rank."""
    from loki_b200.moe import LayerWeights
    from loki_b200.ep import EpMoeLayer, NativeEpOps
    from ep_ref import ThreadComm
    E = 256 // n_ranks
    comms = ThreadComm.group(n_ranks)
    shards = [LayerWeights("cuda", SEED, 0, n_experts=E, expert0=r * E) for r in range(n_ranks)]
    ops = [NativeEpOps(0, n_ranks, T_loc) for _ in range(n_ranks)]
    inputs = [_inputs(T_loc, r) for r in range(n_ranks)]
    torch.cuda.synchronize()
    out, errs = [None] * n_ranks, []

    def run(rank):
        try:
            layer = EpMoeLayer(comms[rank], ops[rank], fixed_cap_max=8)
            x, r = (torch.from_numpy(a).cuda() for a in inputs[rank])
            out[rank] = layer.forward(shards[rank], x, r)
        except Exception as e:                     # surfaced below
            errs.append(e)
            comms[rank].hub.barrier.abort()

    th = [threading.Thread(target=run, args=(k,)) for k in range(n_ranks)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=600)
    assert not errs, errs
    torch.cuda.synchronize()
    tok = [0, 1, 17, T_loc // 2, T_loc - 2, T_loc - 1]
    for rank in range(n_ranks):
        ops[rank].device_error()
        x, r = inputs[rank]
        h, moe, sel, w = out[rank]
        sel, w = sel.cpu().numpy(), w.cpu().numpy()
        _, osel, ow = oracle.router(x, shards[rank].router_w.float().cpu().numpy(), shards[rank].router_bias.cpu().numpy(),
                                    oracle.route_cfg(8, 8, 1, 1, 1))
        np.testing.assert_array_equal(sel, osel)
        np.testing.assert_array_equal(w, ow)
        ref = oracle_layer(oracle, SEED, 0, x, r, sel, w, tokens=tok)
        e_moe, e_h = rel_l2(moe.cpu().numpy()[tok], ref["moe"]), rel_l2(h.cpu().numpy()[tok], ref["h"])
        assert e_moe < RTOL_L2 and e_h < RTOL_L2, (rank, e_moe, e_h)


def _nccl_worker(rank, port, T_loc, fixed_cap_max, comm_kind, out_dir):
    import torch.distributed as dist
    from loki_b200.moe import LayerWeights
    from loki_b200.ep import EpMoeLayer, NativeEpOps, TorchComm, NativeComm, P2PExchange
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank))
    try:
        W = LayerWeights("cuda:%d" % rank, SEED, 0, n_experts=128, expert0=rank * 128)
        ops = NativeEpOps(rank, 2, T_loc)
        ops.set_gemm_threshold(1 << 20)
        ops.set_mma_threshold(1 << 20)
        comm = NativeComm(rank) if comm_kind in ("native", "p2p") else TorchComm()
        p2p = P2PExchange(rank, T_loc) if comm_kind == "p2p" else None
        layer = EpMoeLayer(comm, ops, fixed_cap_max=fixed_cap_max, p2p=p2p)
        x, r = (torch.from_numpy(a).cuda() for a in _inputs(T_loc, rank))
        h, moe, sel, w = layer.forward(W, x, r)
        torch.cuda.synchronize()
        if comm_kind in ("native", "p2p") and T_loc <= fixed_cap_max:
            # the same layer captured in a CUDA graph (exchanges included) and replayed: identical outputs
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                out_g = layer.forward(W, x, r)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out_g[0], h) and torch.equal(out_g[1], moe)
            del g
        if p2p is not None:
            p2p.close()
        if comm_kind in ("native", "p2p"):
            comm.close()
        ops.device_error()
        np.savez(os.path.join(out_dir, "r%d.npz" % rank), h=h.cpu().numpy(), moe=moe.cpu().numpy(),
                 sel=sel.cpu().numpy(), w=w.cpu().numpy(), Wr=W.router_w.float().cpu().numpy(),
                 b=W.router_bias.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_loc,fixed_cap_max,comm_kind", [(1, 8, "native"), (12, 4, "native"), (3, 8, "torch"),
                                                             (12, 4, "torch"), (1, 8, "p2p"), (5, 8, "p2p")])
def test_ep_nccl_two_gpus(native, oracle, tmp_path, T_loc, fixed_cap_max, comm_kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_nccl_worker, args=(port, T_loc, fixed_cap_max, comm_kind, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for rank in range(2):
        got = np.load(os.path.join(str(tmp_path), "r%d.npz" % rank))
        x, r = _inputs(T_loc, rank)
        _, osel, ow = oracle.router(x, got["Wr"], got["b"], oracle.route_cfg(8, 8, 1, 1, 1))
        np.testing.assert_array_equal(got["sel"], osel)
        np.testing.assert_array_equal(got["w"], ow)
        ref = oracle_layer(oracle, SEED, 0, x, r, osel, ow)
        assert rel_l2(got["moe"], ref["moe"]) < RTOL_L2
        assert rel_l2(got["h"], ref["h"]) < RTOL_L2


def test_p2p_wait_runs_out_with_error_status(native):
    """A rank that never sends: rank 0 of a 2-rank mailbox, nothing ever publishes its flags.  The rows wait
    and the returns wait each give up after their bounded spin (2 s of globaltimer) and leave their error word
    (1: rows never arrived, 2: returns never arrived); the context stays usable for the next launches."""
    import ctypes
    from loki_b200.native import lib, check, EP_IPC_HANDLE_BYTES
    L = lib()
    mb, h = ctypes.c_void_p(), ctypes.create_string_buffer(EP_IPC_HANDLE_BYTES)
    check(L.lk_ep_mailbox_create(2, 0, 4, torch.cuda.current_device(), ctypes.byref(mb), h))
    try:
        st = torch.cuda.current_stream()
        err = torch.zeros(2, dtype=torch.int32, device="cuda")
        rows = ctypes.c_void_p()
        check(L.lk_ep_p2p_rows(mb, ctypes.byref(rows), ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(st.cuda_stream)))
        row_map = torch.full((1, 2), -1, dtype=torch.int32, device="cuda")
        resid = torch.ones(1, HIDDEN, device="cuda")
        hh, moe = torch.empty_like(resid), torch.empty_like(resid)
        check(L.lk_ep_p2p_combine(mb, ctypes.c_void_p(row_map.data_ptr()), 1, ctypes.c_void_p(resid.data_ptr()), None,
                                  ctypes.c_void_p(hh.data_ptr()), ctypes.c_void_p(moe.data_ptr()),
                                  ctypes.c_void_p(err.data_ptr() + 4), ctypes.c_void_p(st.cuda_stream)))
        torch.cuda.synchronize()
        assert err.tolist() == [1, 2]
        assert torch.equal(hh, resid) and not moe.any()       # nothing returned: h = resid, moe = 0
        assert float(torch.ones(1 << 20, device="cuda").sum()) == float(1 << 20)
    finally:
        L.lk_ep_mailbox_destroy(mb)


def _one_rank_worker(rank, port, T_loc, out_dir):
    import torch.distributed as dist
    from loki_b200.moe import LayerWeights
    from loki_b200.ep import EpMoeLayer, NativeEpOps, NativeComm, P2PExchange
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        W = LayerWeights("cuda:0", SEED, 0)
        ops = NativeEpOps(0, 1, T_loc)
        comm = NativeComm(0)
        p2p = P2PExchange(0, T_loc)
        layer = EpMoeLayer(comm, ops, p2p=p2p)
        x, r = (torch.from_numpy(a).cuda() for a in _inputs(T_loc, 0))
        outs = [layer.forward(W, x, r) for _ in range(3)]          # three layers: the epoch advances
        torch.cuda.synchronize()
        for o in outs[1:]:
            assert torch.equal(o[0], outs[0][0]) and torch.equal(o[1], outs[0][1])
        h, moe, sel, w = outs[0]
        p2p.close()
        comm.close()
        ops.device_error()
        extra = {}
        if T_loc == 1:                                              # the single-GPU forward on the same layer
            from loki_b200.moe import MoeLayer
            one = MoeLayer(0, max_tokens=1)
            h1, moe1, _, _ = one.forward(W, x, r)
            torch.cuda.synchronize()
            extra = {"h1": h1.cpu().numpy(), "moe1": moe1.cpu().numpy()}
            one.close()
        np.savez(os.path.join(out_dir, "r0.npz"), h=h.cpu().numpy(), moe=moe.cpu().numpy(), sel=sel.cpu().numpy(),
                 w=w.cpu().numpy(), Wr=W.router_w.float().cpu().numpy(), b=W.router_bias.cpu().numpy(), **extra)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_loc", [1, 3])
def test_ep_p2p_one_rank(native, oracle, tmp_path, T_loc):
    """The peer-memory exchange with a single rank (every expert local, the rows sent to itself) on one GPU:
    dispatch, the fused lk_ep_p2p_experts (rows wait + slot tables, the expert kernels reading the rows' q8
    codes, the down kernel storing each entry's row into the home mailbox, the return flags) and the waiting
    combine, three layers in a row; routing bit-exact and h / moe within RTOL_L2 of the oracle.  At one token
    the exchange runs the single-GPU kernels on the same q8 codes and sums in the same order, so h and moe
    equal lk_moe_forward's bit for bit."""
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_one_rank_worker, args=(port, T_loc, str(tmp_path)), nprocs=1, join=True, start_method="spawn")
    got = np.load(os.path.join(str(tmp_path), "r0.npz"))
    x, r = _inputs(T_loc, 0)
    _, osel, ow = oracle.router(x, got["Wr"], got["b"], oracle.route_cfg(8, 8, 1, 1, 1))
    np.testing.assert_array_equal(got["sel"], osel)
    np.testing.assert_array_equal(got["w"], ow)
    ref = oracle_layer(oracle, SEED, 0, x, r, osel, ow)
    assert rel_l2(got["moe"], ref["moe"]) < RTOL_L2
    assert rel_l2(got["h"], ref["h"]) < RTOL_L2
    if T_loc == 1:
        np.testing.assert_array_equal(got["moe"], got["moe1"])
        np.testing.assert_array_equal(got["h"], got["h1"])
