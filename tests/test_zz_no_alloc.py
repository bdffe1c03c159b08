"""lk_moe_experts_noalloc: the expert stage for callers that cannot allocate device memory (an engine whose
HBM is already fully given to resident expert shards and KV cache, or a latency-critical caller that cannot
take cudaMalloc's device-wide synchronisation).  It runs on one static device array instead of context
scratch.  Checked through the C ABI against the existing entry point (lk_moe_experts) on two calls in a
row with different inputs, so the second call also shows that nothing stale from the first leaks through.

Collected last (file name), so a run that stops at the first failure has run every other test first; it
builds and loads the library itself, so it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from moe_helpers import SEED, HIDDEN, INTER, MAT, RTOL_L2, rel_l2, oracle_layer

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
LAYER = 21


@pytest.fixture(scope="module")
def arena(native):
    from loki_b200 import moe as M
    NE, layer_id = 10, LAYER
    buf = torch.empty(3 * NE * MAT + 3 * MAT, dtype=torch.uint8, device="cuda")
    base = buf.data_ptr()
    for m in range(3):
        rows, K = (INTER, HIDDEN) if m < 2 else (HIDDEN, INTER)
        M.gen_iq2(base + m * NE * MAT, SEED, layer_id, m, 0, NE, rows, K, MAT)
        M.gen_iq2(base + 3 * NE * MAT + m * MAT, SEED, layer_id, m, 256, 1, rows, K, MAT)
    ws = native.LkMoeWeights(base, base + NE * MAT, base + 2 * NE * MAT, MAT, MAT, MAT, native.FMT_IQ2,
                             base + 3 * NE * MAT, base + 3 * NE * MAT + MAT, base + 3 * NE * MAT + 2 * MAT, None, 0, None)
    torch.cuda.synchronize()
    return buf, ws, NE


def _case(rng, NE, T, keep):
    sel = np.stack([rng.choice(NE, keep, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, keep)).astype(np.float32)
    x = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    r = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    return [torch.from_numpy(a).cuda() for a in (sel, w, x, r)]


def _noalloc(native, ws, sel, w, x, r, with_shared=1, want_h=True):
    T, keep = sel.shape
    h = torch.empty(T, HIDDEN, device="cuda") if want_h else None
    mo = torch.empty(T, HIDDEN, device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    rc = native.lib().lk_moe_experts_noalloc(ctypes.byref(ws), p(x), p(r), T, p(sel), p(w), keep, with_shared, p(h), p(mo),
                                             p(status), s)
    assert rc == native.LK_OK, rc
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return h, mo


def _existing(ws, sel, w, x, r, with_shared=True):
    """The context entry point (lk_moe_experts) on the same single-token matvec path."""
    from loki_b200 import moe as M
    T, keep = sel.shape
    ref = M.MoeLayer(0, keep=keep, max_tokens=T, with_shared=with_shared)
    ref.set_mma_threshold(1 << 20)
    h_ref, mo_ref = ref.experts(ws, x, r, sel, w)
    ref.device_error()
    return h_ref.cpu().numpy(), mo_ref.cpu().numpy()


def test_noalloc_matches_existing_entry_point_twice(native, arena, oracle):
    _, ws, NE = arena
    rng = np.random.default_rng(4242)
    for T, keep in ((3, 8), (8, 2)):                       # two calls in a row, different shapes
        sel, w, x, r = _case(rng, NE, T, keep)
        h, mo = _noalloc(native, ws, sel, w, x, r)
        h_ref, mo_ref = _existing(ws, sel, w, x, r)
        e_h = rel_l2(h.cpu().numpy(), h_ref)
        e_m = rel_l2(mo.cpu().numpy(), mo_ref)
        assert e_h < RTOL_L2 and e_m < RTOL_L2, (T, keep, e_h, e_m)
        # and straight against the CPU oracle (the reference's q8 numerics)
        ref = oracle_layer(oracle, SEED, LAYER, x.cpu().numpy(), r.cpu().numpy(), sel.cpu().numpy(), w.cpu().numpy())
        e_o = rel_l2(h.cpu().numpy(), ref["h"])
        assert e_o < RTOL_L2, (T, keep, e_o)


def test_noalloc_absent_entries_moe_only_and_no_shared(native, arena):
    """Absent entries (negative ids) after a call that left other data in the static array: their stale y rows
    must not reach the outputs.  Also a call without the shared expert and a moe-only call (h = null)."""
    _, ws, NE = arena
    rng = np.random.default_rng(77)
    sel, w, x, r = _case(rng, NE, 8, 8)
    _noalloc(native, ws, sel, w, x, r)                     # fills every y row of the array
    sel2, w2, x2, r2 = _case(rng, NE, 5, 8)
    s2 = sel2.cpu().numpy()
    s2[:, 5:] = -1                                         # the last three entries of every token absent
    s2[2, :] = -1                                          # and one token with no routed entry at all
    sel2 = torch.from_numpy(s2).cuda()
    for with_shared in (1, 0):
        h, mo = _noalloc(native, ws, sel2, w2, x2, r2, with_shared=with_shared)
        h_ref, mo_ref = _existing(ws, sel2, w2, x2, r2, with_shared=bool(with_shared))
        assert rel_l2(h.cpu().numpy(), h_ref) < RTOL_L2 and rel_l2(mo.cpu().numpy(), mo_ref) < RTOL_L2, with_shared
        if not with_shared:
            assert np.abs(mo.cpu().numpy()[2]).max() == 0.0          # token 2 has nothing routed and no shared expert
    _, mo = _noalloc(native, ws, sel2, w2, x2, r2, with_shared=1, want_h=False)
    _, mo_ref = _existing(ws, sel2, w2, x2, r2)
    assert rel_l2(mo.cpu().numpy(), mo_ref) < RTOL_L2


def test_noalloc_rejects_sizes_above_its_limit(native, arena):
    _, ws, NE = arena
    T = 9                                                  # LK_NOALLOC_MAX_TOKENS + 1
    rng = np.random.default_rng(5)
    sel, w, x, r = _case(rng, NE, T, 2)
    h = torch.empty(T, HIDDEN, device="cuda")
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = native.lib().lk_moe_experts_noalloc(ctypes.byref(ws), p(x), p(r), T, p(sel), p(w), 2, 1, p(h), None, None,
                                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == native.LK_ERR_CAPACITY
