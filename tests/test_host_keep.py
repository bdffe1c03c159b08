"""CPU tests of the engine-side host logic around fl_moe (loki_b200/fused.py): the keep-KE compaction with
and without --share-experts, pad rows and the expert union/remap, each against a line-by-line
restatement of src/server_core_fused.cpp:793-818."""
import numpy as np
import pytest

from loki_b200 import fused as F


def ref_keep(selh, wh, KE, share, n_pad_from, renorm=True):
    """Loop restatement of server_core_fused.cpp:793-813 (ties: equal weights keep position order)."""
    n = len(selh)
    ords = [sorted(range(8), key=lambda k: (-float(wh[i][k]), k)) for i in range(n)]
    sk, wk = [], []
    if share and n > 1:
        own = min(2, KE)
        U = set()
        for i in range(min(n, n_pad_from)):
            for k in range(own):
                U.add(int(selh[i][ords[i][k]]))
        for i in range(n):
            pick = [ords[i][k] for k in range(own)]
            k = own
            while k < 8 and len(pick) < KE:
                if int(selh[i][ords[i][k]]) in U:
                    pick.append(ords[i][k])
                k += 1
            k = own
            while k < 8 and len(pick) < KE:
                if ords[i][k] not in pick:
                    pick.append(ords[i][k])
                    U.add(int(selh[i][ords[i][k]]))
                k += 1
            sk.append([int(selh[i][p]) for p in pick])
            wk.append([np.float32(wh[i][p]) for p in pick])
    else:
        for i in range(n):
            sk.append([int(selh[i][ords[i][k]]) for k in range(KE)])
            wk.append([np.float32(wh[i][ords[i][k]]) for k in range(KE)])
    if renorm:
        for i in range(n):
            sw = np.float32(0)
            for v in wk[i]:
                sw = np.float32(sw + v)
            if sw > 1e-6:
                f = np.float32(np.float32(2.5) / sw)
                wk[i] = [np.float32(v * f) for v in wk[i]]
    return np.array(sk, np.int32), np.array(wk, np.float32)


def _rows(rng, n, pool=256):
    sel = np.stack([rng.choice(pool, 8, replace=False) for _ in range(n)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (n, 8)).astype(np.float32)
    return sel, w


@pytest.mark.parametrize("KE", [1, 2, 3, 4, 6])
@pytest.mark.parametrize("share", [False, True])
def test_keep_pass_matches_engine(KE, share):
    rng = np.random.default_rng(KE * 7 + share)
    for n in (1, 2, 5, 8):
        for pool in (12, 256):                          # a small pool makes rows share experts
            sel, w = _rows(rng, n, pool)
            got_s, got_w = F.keep_pass(sel, w, KE, share=share)
            ref_s, ref_w = ref_keep(sel, w, KE, share, n)
            np.testing.assert_array_equal(got_s, ref_s)
            np.testing.assert_array_equal(got_w, ref_w)


def test_share_experts_prefers_experts_other_rows_keep():
    # row 0 keeps 10, 11; row 1 keeps 20, 21 and then prefers 10 (kept by row 0) over its own 22
    sel = np.array([[10, 11, 12, 13, 14, 15, 16, 17], [20, 21, 22, 10, 23, 24, 25, 26]], np.int32)
    w = np.array([[.9, .8, .7, .6, .5, .4, .3, .2], [.9, .8, .7, .6, .5, .4, .3, .2]], np.float32)
    s, _ = F.keep_pass(sel, w, 3, share=True)
    assert list(s[0]) == [10, 11, 12] and list(s[1]) == [20, 21, 10]
    s_plain, _ = F.keep_pass(sel, w, 3)
    assert list(s_plain[1]) == [20, 21, 22]


def test_share_experts_pad_rows_do_not_seed_the_set():
    # row 1 is padding (n_pad_from=1): its own top-2 (30, 31) do not seed U, but the expert it takes to fill
    # its third slot (32) joins U, and row 2 then prefers 32 over its own 22; 30 stays out of U
    sel = np.array([[10, 11, 12, 13, 14, 15, 16, 17], [30, 31, 32, 33, 34, 35, 36, 37],
                    [20, 21, 22, 30, 32, 24, 25, 26]], np.int32)
    w = np.tile(np.linspace(0.9, 0.2, 8, dtype=np.float32), (3, 1))
    s, _ = F.keep_pass(sel, w, 3, share=True, n_pad_from=1)
    ref_s, _ = ref_keep(sel, w, 3, True, 1)
    np.testing.assert_array_equal(s, ref_s)
    assert list(s[1]) == [30, 31, 32] and list(s[2]) == [20, 21, 32]


def test_pad_rows_and_union_remap():
    sel = np.array([[5, 9], [7, 5], [1, 2], [3, 4]], np.int32)
    w = np.array([[1.0, 1.5], [2.0, 0.5], [1.0, 1.0], [1.0, 1.0]], np.float32)
    ps, pw = F.pad_rows(sel, w, 2)
    assert (ps[2:] == ps[0]).all() and (pw[2:] == 0).all() and (ps[:2] == sel[:2]).all()
    used, idsc = F.union_remap(ps)
    assert list(used) == [5, 7, 9]
    np.testing.assert_array_equal(used[idsc], ps)


@pytest.mark.parametrize("share", [False, True])
def test_native_keep_matches_python(share):
    """lkr_keep (the C++ keep pass of the engine-replay harness) equals keep_pass."""
    rng = np.random.default_rng(5 + share)
    for KE in (1, 2, 3, 5, 8):
        for pool in (10, 256):
            sel, w = _rows(rng, 7, pool)
            a = F.keep_pass(sel, w, KE, share=share)
            b = F.keep_pass_native(sel, w, KE, share=share)
            np.testing.assert_array_equal(a[0], b[0])
            np.testing.assert_array_equal(a[1], b[1])
