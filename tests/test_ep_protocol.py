"""The expert-parallel exchange protocol (loki_b200.ep.EpMoeLayer) over gloo, world_size 2, on the CPU.

Each rank owns 128 experts; the per-rank stages are the oracle restatements (ep_ref.RefEpOps) on the
CUDA path's row format.  Every rank's h / moe must equal the single-process oracle of the whole layer
for its tokens up to fp32 summation order (the home rank sums per-rank partial sums), in both row
layouts: fixed capacity (decode) and compact (count exchange first).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from moe_helpers import SEED, HIDDEN, rel_l2, oracle_layer

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(T_loc, rank):
    rng = np.random.default_rng(77 + rank)
    return (rng.standard_normal((T_loc, HIDDEN)).astype(np.float32),
            rng.standard_normal((T_loc, HIDDEN)).astype(np.float32))


def _router():
    rng = np.random.default_rng(5)
    return (rng.normal(0, 0.02, (256, HIDDEN)).astype(np.float32), rng.normal(0, 0.01, 256).astype(np.float32))


def _worker(rank, port, T_loc, fixed_cap_max, n_group, out_dir):
    import torch.distributed as dist
    from oracle import oracle as O
    from ep_ref import RefEpOps, RefShard
    from loki_b200.ep import EpMoeLayer, TorchComm
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=WORLD)
    try:
        Wr, b = _router()
        cfg = O.route_cfg(8, 8, 1, n_group, 4 if n_group > 1 else 1)
        ops = RefEpOps(O, WORLD, cfg)
        W = RefShard(O, SEED, 0, rank, WORLD, Wr, b)
        layer = EpMoeLayer(TorchComm(), ops, fixed_cap_max=fixed_cap_max)
        x, r = _inputs(T_loc, rank)
        h, moe, sel, w = layer.forward(W, torch.from_numpy(x), torch.from_numpy(r))
        np.savez(os.path.join(out_dir, "r%d.npz" % rank), h=h.numpy(), moe=moe.numpy(), sel=sel.numpy(), w=w.numpy(),
                 counts=np.array(layer.last_counts if layer.last_counts else [[-1], [-1]]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_loc,fixed_cap_max,n_group", [(3, 8, 1), (9, 4, 8)])
def test_ep_protocol_gloo(oracle, tmp_path, T_loc, fixed_cap_max, n_group):
    mp.start_processes(_worker, args=(_free_port(), T_loc, fixed_cap_max, n_group, str(tmp_path)), nprocs=WORLD,
                       join=True, start_method="spawn")
    Wr, b = _router()
    total_sent = 0
    for rank in range(WORLD):
        got = np.load(os.path.join(str(tmp_path), "r%d.npz" % rank))
        x, r = _inputs(T_loc, rank)
        cfg = oracle.route_cfg(8, 8, 1, n_group, 4 if n_group > 1 else 1)
        _, osel, ow = oracle.router(x, Wr, b, cfg)
        np.testing.assert_array_equal(got["sel"], osel)
        np.testing.assert_array_equal(got["w"], ow)
        ref = oracle_layer(oracle, SEED, 0, x, r, osel, ow)
        assert rel_l2(got["moe"], ref["moe"]) < 1e-5
        assert rel_l2(got["h"], ref["h"]) < 1e-5
        if T_loc > fixed_cap_max:                  # compact layout: tokens with an expert there, all to the own rank
            sent = got["counts"][0]
            owners = osel // 128
            assert list(sent) == [T_loc if d == rank else int((owners == d).any(axis=1).sum()) for d in range(WORLD)]
            total_sent += int(np.sum(sent))
    if T_loc > fixed_cap_max:
        assert total_sent > 0
