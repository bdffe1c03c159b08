"""The GGUF expert loader (loki_b200/gguf_experts.py) and the engine's --dump-moe records
(loki_b200/moe_dump.py): CPU checks of the container parser and the record layout against files written by
gguf-py / in the engine's byte order, and GPU runs of the expert stage on loaded layers and replayed records
against the oracle."""
import os

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, MAT, RTOL_L2, rel_l2, down_bytes

NE = 2            # experts in the test files (a DeepSeek layer has 256; the loader reads the count from the file)


def _write_layer_file(path, oracle, down_fmt, f16_router=False, model_shared=False):
    gguf = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as QT
    qt = {4: QT.IQ2_XXS, 5: QT.Q2_K, 6: QT.Q3_K}[down_fmt]
    nb = {4: 66, 5: 84, 6: 110}[down_fmt]
    w = gguf.GGUFWriter(path, "deepseek2")
    w.add_uint32("deepseek2.expert_count", NE)
    gate = np.concatenate([oracle.gen_iq2(SEED, 0, 0, e, INTER, HIDDEN) for e in range(NE)])
    up = np.concatenate([oracle.gen_iq2(SEED, 0, 1, e, INTER, HIDDEN) for e in range(NE)])
    down = np.concatenate([oracle.gen_matrix(down_fmt, SEED, 0, 2, e, HIDDEN, INTER) for e in range(NE)])
    w.add_tensor("blk.0.ffn_gate_exps.weight", gate.reshape(NE, INTER, -1), raw_shape=[NE, INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
    w.add_tensor("blk.0.ffn_up_exps.weight", up.reshape(NE, INTER, -1), raw_shape=[NE, INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
    w.add_tensor("blk.0.ffn_down_exps.weight", down.reshape(NE, HIDDEN, -1), raw_shape=[NE, HIDDEN, 8 * nb], raw_dtype=qt)
    rng = np.random.default_rng(3)
    router = (rng.standard_normal((256, HIDDEN)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    if f16_router:
        router = router.astype(np.float16)
        w.add_tensor("blk.0.ffn_gate_inp_f16.weight", router)
    else:
        w.add_tensor("blk.0.ffn_gate_inp.weight", router)
    w.add_tensor("blk.0.exp_probs_b.bias", bias)
    if model_shared:                      # the real model's shared expert types (Q5_K gate/up, Q6_K down)
        w.add_tensor("blk.0.ffn_gate_shexp.weight", np.zeros((INTER, 28 * 176), np.uint8), raw_shape=[INTER, 28 * 176], raw_dtype=QT.Q5_K)
        w.add_tensor("blk.0.ffn_up_shexp.weight", np.zeros((INTER, 28 * 176), np.uint8), raw_shape=[INTER, 28 * 176], raw_dtype=QT.Q5_K)
        w.add_tensor("blk.0.ffn_down_shexp.weight", np.zeros((HIDDEN, 8 * 210), np.uint8), raw_shape=[HIDDEN, 8 * 210], raw_dtype=QT.Q6_K)
        sh = None
    else:
        sh = (oracle.gen_iq2(SEED, 0, 0, 256, INTER, HIDDEN), oracle.gen_iq2(SEED, 0, 1, 256, INTER, HIDDEN),
              oracle.gen_matrix(down_fmt, SEED, 0, 2, 256, HIDDEN, INTER))
        w.add_tensor("blk.0.ffn_gate_shexp.weight", sh[0].reshape(INTER, -1), raw_shape=[INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
        w.add_tensor("blk.0.ffn_up_shexp.weight", sh[1].reshape(INTER, -1), raw_shape=[INTER, 28 * 66], raw_dtype=QT.IQ2_XXS)
        w.add_tensor("blk.0.ffn_down_shexp.weight", sh[2].reshape(HIDDEN, -1), raw_shape=[HIDDEN, 8 * nb], raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return gate, up, down, sh, router, bias


@pytest.mark.parametrize("down_fmt", [4, 6])
def test_gguf_index_and_bytes(oracle, tmp_path, down_fmt):
    from loki_b200.gguf_experts import GgufFile, GGML_IQ2_XXS, GGML_Q3_K, GGML_F32
    path = str(tmp_path / "layer.gguf")
    gate, up, down, sh, router, bias = _write_layer_file(path, oracle, down_fmt)
    g = GgufFile(path)
    assert g.meta["general.architecture"] == "deepseek2" and g.meta["deepseek2.expert_count"] == NE
    t, ne, _, nbytes = g.info("blk.0.ffn_gate_exps.weight")
    assert t == GGML_IQ2_XXS and ne == [HIDDEN, INTER, NE] and nbytes == NE * MAT
    t, ne, _, nbytes = g.info("blk.0.ffn_down_exps.weight")
    assert t == (GGML_IQ2_XXS if down_fmt == 4 else GGML_Q3_K) and ne == [INTER, HIDDEN, NE] and nbytes == NE * down_bytes(down_fmt)
    np.testing.assert_array_equal(np.asarray(g.bytes("blk.0.ffn_gate_exps.weight")), gate)
    np.testing.assert_array_equal(np.asarray(g.bytes("blk.0.ffn_up_exps.weight")), up)
    np.testing.assert_array_equal(np.asarray(g.bytes("blk.0.ffn_down_exps.weight")), down)
    np.testing.assert_array_equal(np.asarray(g.bytes("blk.0.ffn_down_shexp.weight")), sh[2])
    assert g.info("blk.0.ffn_gate_inp.weight")[:2] == (GGML_F32, [HIDDEN, 256])
    np.testing.assert_array_equal(np.frombuffer(g.bytes("blk.0.ffn_gate_inp.weight"), np.float32).reshape(256, HIDDEN), router)
    np.testing.assert_array_equal(np.frombuffer(g.bytes("blk.0.exp_probs_b.bias"), np.float32), bias)


def test_gguf_rejects_non_gguf(tmp_path):
    from loki_b200.gguf_experts import GgufFile, GgufError
    p = tmp_path / "x.bin"
    p.write_bytes(b"GGML" + bytes(64))
    with pytest.raises(GgufError):
        GgufFile(str(p))


def test_moe_dump_roundtrip(tmp_path):
    """Records in the engine's byte order (server_core_fused.cpp:814) read back exactly."""
    from loki_b200.moe_dump import read_moe_dump, write_moe_dump
    rng = np.random.default_rng(8)
    recs = [{"layer": L, "sel": rng.choice(256, ke, replace=False), "w": rng.uniform(0, 1, ke).astype(np.float32),
             "x": rng.standard_normal(HIDDEN).astype(np.float32)} for L, ke in ((3, 8), (4, 2), (60, 1))]
    path = str(tmp_path / "moe.bin")
    write_moe_dump(path, recs)
    # the engine's layout, written field by field
    raw = open(path, "rb").read()
    r0 = recs[0]
    expect0 = (np.array([3, 8], np.int32).tobytes() + np.asarray(r0["sel"], np.int32).tobytes() + r0["w"].tobytes() + r0["x"].tobytes())
    assert raw[:len(expect0)] == expect0
    back = read_moe_dump(path)
    assert [b["layer"] for b in back] == [3, 4, 60] and [b["keep"] for b in back] == [8, 2, 1]
    for a, b in zip(recs, back):
        np.testing.assert_array_equal(b["sel"], a["sel"])
        np.testing.assert_array_equal(b["w"], a["w"])
        np.testing.assert_array_equal(b["x"], a["x"])
    with open(path, "ab") as f:
        f.write(b"\x01\x00")
    with pytest.raises(ValueError):
        read_moe_dump(path)


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("down_fmt,f16_router", [(4, False), (6, True)])
def test_gguf_layer_on_gpu(native, oracle, tmp_path, down_fmt, f16_router):
    """A layer loaded from a GGUF file runs the expert stage (and its router) like generated weights."""
    import torch
    from loki_b200 import moe as M
    from loki_b200.gguf_experts import GgufLayer
    path = str(tmp_path / "layer.gguf")
    gate, up, down, sh, router, bias = _write_layer_file(path, oracle, down_fmt, f16_router=f16_router)
    L = GgufLayer(path, 0)
    assert L.n_experts == NE and L.down_fmt == down_fmt and L.with_shared
    rng = np.random.default_rng(41)
    T, keep = 3, 2
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    sel = np.array([[0, 1], [1, 0], [0, 1]], np.int32)
    w = rng.uniform(0.1, 1.0, (T, keep)).astype(np.float32)
    ctx = M.MoeLayer(0, topk=keep, keep=keep, max_tokens=T, n_experts=NE)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    h, mo = ctx.experts(L.struct(), dev(x), dev(r), dev(sel), dev(w))
    ctx.device_error()
    ref = oracle.moe_layer(x, r, gate, up, down, MAT, sel, w, *sh, down_fmt=down_fmt, down_stride=down_bytes(down_fmt))
    assert rel_l2(mo.cpu().numpy(), ref["moe"]) < RTOL_L2 and rel_l2(h.cpu().numpy(), ref["h"]) < RTOL_L2
    # the router tensors as loaded: the routing of the 256-expert router equals the oracle's
    route = M.MoeLayer(0, keep=8, max_tokens=T)
    probs, s8, w8 = route.route(L.struct(), dev(x))
    _, osel, ow = oracle.router(x, router.astype(np.float32), bias, oracle.route_cfg(8, 8))
    np.testing.assert_array_equal(s8.cpu().numpy(), osel)
    np.testing.assert_array_equal(w8.cpu().numpy(), ow)


@pytest.mark.gpu
def test_gguf_model_shared_expert_loaded(native, oracle, tmp_path):
    """The real model's shared-expert types (Q5_K gate/up, Q6_K down) load as the model-format shared expert."""
    from loki_b200.gguf_experts import GgufLayer, GGML_Q5_K, GGML_Q6_K
    path = str(tmp_path / "layer.gguf")
    _write_layer_file(path, oracle, 5, model_shared=True)
    L = GgufLayer(path, 0)
    assert L.down_fmt == 5 and L.with_shared and L.sh_fmt == 3 and L.shared_types == (GGML_Q5_K, GGML_Q5_K, GGML_Q6_K)


@pytest.mark.gpu
def test_moe_dump_replay(native, oracle, tmp_path):
    """Dump records replayed through the expert stage (the engine's row-0 inputs and routing) match the oracle."""
    import torch
    from loki_b200 import moe as M
    from loki_b200.moe_dump import read_moe_dump, write_moe_dump
    from moe_helpers import oracle_layer
    rng = np.random.default_rng(12)
    recs = [{"layer": 0, "sel": rng.choice(256, ke, replace=False), "w": rng.uniform(0.1, 1, ke).astype(np.float32),
             "x": rng.standard_normal(HIDDEN).astype(np.float32)} for ke in (8, 2)]
    path = str(tmp_path / "moe.bin")
    write_moe_dump(path, recs)
    W = M.LayerWeights("cuda", SEED, 0)
    try:
        for rec in read_moe_dump(path):
            ke = rec["keep"]
            ctx = M.MoeLayer(0, keep=ke, max_tokens=1)
            x = torch.from_numpy(rec["x"][None]).cuda()
            zero = torch.zeros_like(x)
            h, mo = ctx.experts(W, x, zero, torch.from_numpy(rec["sel"][None]).cuda(), torch.from_numpy(rec["w"][None]).cuda())
            ctx.device_error()
            ref = oracle_layer(oracle, SEED, 0, rec["x"][None], np.zeros((1, HIDDEN), np.float32), rec["sel"][None], rec["w"][None])
            assert rel_l2(mo.cpu().numpy(), ref["moe"]) < RTOL_L2
    finally:
        del W
        torch.cuda.empty_cache()
