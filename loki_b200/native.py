"""ctypes binding of libloki_moe.so (include/loki_moe.h, include/loki_fused_moe.h, include/loki_ep.h).

The library is the product: every call here goes straight to the CUDA kernels.  There is no CPU or
PyTorch fallback; a missing library raises at first use.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libloki_moe.so")
REPO = os.path.dirname(HERE)

HIDDEN = 7168
MOE_INTER = 2048
N_EXPERTS = 256
QK = 256
BLK_IQ2 = 66
EXPERT_MATRIX_BYTES = MOE_INTER * (HIDDEN // QK) * BLK_IQ2          # 3 784 704 (gate, up and down alike)

LK_OK, LK_ERR_ARG, LK_ERR_CUDA, LK_ERR_UNSUPPORTED, LK_ERR_CAPACITY, LK_ERR_DEVICE = 0, -1, -2, -3, -4, -5
FMT_Q6K, FMT_Q5K, FMT_IQ2, FMT_Q2K, FMT_Q3K = 1, 3, 4, 5, 6
BLOCK_BYTES = {FMT_IQ2: 66, FMT_Q2K: 84, FMT_Q3K: 110, FMT_Q5K: 176, FMT_Q6K: 210}
# one expert's down matrix [7168 rows][2048] per format: 3 784 704 / 4 816 896 / 6 307 840 bytes
DOWN_MATRIX_BYTES = {f: HIDDEN * (MOE_INTER // QK) * b for f, b in BLOCK_BYTES.items()}
# bytes of one gate (or up) matrix [MOE_INTER][HIDDEN] per format
GU_MATRIX_BYTES = {f: MOE_INTER * (HIDDEN // QK) * b for f, b in BLOCK_BYTES.items()}
EP_ROW_HDR_BYTES = 64
EP_ROW_BYTES = EP_ROW_HDR_BYTES + HIDDEN + HIDDEN // 32 * 4   # 8 128: header, q8 codes, fp32 scales
EP_MAX_RANKS = 8
EP_COMM_ID_BYTES = 128
EP_IPC_HANDLE_BYTES = 64


class LkMoeConfig(ctypes.Structure):
    _fields_ = [("n_experts", ctypes.c_int), ("topk", ctypes.c_int), ("keep", ctypes.c_int), ("renorm", ctypes.c_int),
                ("n_group", ctypes.c_int), ("topk_group", ctypes.c_int), ("scale", ctypes.c_float),
                ("with_shared", ctypes.c_int), ("max_tokens", ctypes.c_int)]


class LkMoeWeights(ctypes.Structure):
    _fields_ = [("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("gate_stride", ctypes.c_int64), ("up_stride", ctypes.c_int64), ("down_stride", ctypes.c_int64),
                ("down_fmt", ctypes.c_int),
                ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p), ("sh_down", ctypes.c_void_p),
                ("router_w", ctypes.c_void_p), ("router_w_f16", ctypes.c_int), ("router_bias", ctypes.c_void_p),
                ("sh_fmt", ctypes.c_int)]


class FLOut(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("sel", "wts", "ncur", "fi", "skt", "sel_s", "wts_s", "sc", "ccat", "h", "moe")]


class FLMoeW(ctypes.Structure):
    _fields_ = [("gate_inp", ctypes.c_void_p), ("gate_f16", ctypes.c_int), ("probs_b", ctypes.c_void_p),
                ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p), ("sh_down", ctypes.c_void_p), ("sh_fmt", ctypes.c_int)]


# exported symbol -> (restype, argtypes)
_P, _I, _I64, _F, _D, _S = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_double, ctypes.c_size_t
SIGNATURES = {
    "lk_moe_create": (_I, [ctypes.POINTER(LkMoeConfig), _I, ctypes.POINTER(_P)]),
    "lk_moe_destroy": (None, [_P]),
    "lk_moe_route": (_I, [_P, ctypes.POINTER(LkMoeWeights), _P, _I, _P, _P, _P, _P, _P]),
    "lk_moe_dispatch": (_I, [_P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "lk_moe_experts": (_I, [_P, ctypes.POINTER(LkMoeWeights), _P, _P, _I, _P, _P, _I, _P, _P, _P]),
    "lk_moe_forward": (_I, [_P, ctypes.POINTER(LkMoeWeights), _P, _P, _I, _P, _P, _P, _P, _P, _P]),
    "lk_moe_slot_outputs": (_P, [_P]),
    "lk_moe_set_events": (_I, [_P, _P]),
    "lk_moe_set_gemm_threshold": (_I, [_P, _I]),
    "lk_moe_set_mma_threshold": (_I, [_P, _I]),
    "lk_moe_set_shared_gemm_threshold": (_I, [_P, _I]),
    "lk_moe_get_error": (_I, [_P, _P]),
    "lk_moe_strerror": (ctypes.c_char_p, [_I]),
    "lk_moe_last_error": (ctypes.c_char_p, [_P]),
    "lk_moe_experts_noalloc": (_I, [ctypes.POINTER(LkMoeWeights), _P, _P, _I, _P, _P, _I, _I, _P, _P, _P, _P]),
    "lk_gen_iq2": (_I, [_P, ctypes.c_uint64, _I, _I, _I, _I, _I, _I, _I64, _P]),
    "lk_gen_weights": (_I, [_I, _P, ctypes.c_uint64, _I, _I, _I, _I, _I, _I, _I64, _P]),
    "lk_ep_pack": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "lk_ep_experts": (_I, [_P, ctypes.POINTER(LkMoeWeights), _P, _I, _I, _I, _I, _P, _P, _P]),
    "lk_ep_shared": (_I, [_P, ctypes.POINTER(LkMoeWeights), _P, _P, _I, _P, _P]),
    "lk_ep_combine": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "lk_ep_comm_id": (_I, [_P]),
    "lk_ep_comm_create": (_I, [_P, _I, _I, _I, ctypes.POINTER(_P)]),
    "lk_ep_comm_destroy": (None, [_P]),
    "lk_ep_all_to_all": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _P]),
    "lk_ep_mailbox_create": (_I, [_I, _I, _I, _I, ctypes.POINTER(_P), _P]),
    "lk_ep_mailbox_connect": (_I, [_P, _P]),
    "lk_ep_mailbox_destroy": (None, [_P]),
    "lk_ep_p2p_dispatch": (_I, [_P, _P, _P, _P, _I, _I, _P, _P, _P]),
    "lk_ep_p2p_rows": (_I, [_P, ctypes.POINTER(_P), _P, _P]),
    "lk_ep_p2p_return": (_I, [_P, _P, _P]),
    "lk_ep_p2p_combine": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _P]),
    "lk_ep_p2p_experts": (_I, [_P, _P, _P, _I, _I, _P, _P, _P]),
    "lk_ep_p2p_combine_entries": (_I, [_P, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P]),
    "lk_ep_p2p_route_dispatch": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P]),
    "fl_init": (_P, [_I, _I]),
    "fl_wide_init": (_I, [_P, _I, _I]),
    "fl_wide_moe": (None, [_P, _P, _P, _P, _I, _I, _P, _P, _P, _P, _I, _I, _I]),
    "fl_wide_mark": (None, [_P, _I]),
    "fl_wide_wait": (None, [_P, _I]),
    "fl_wide_finish": (None, [_P, _I, _I, ctypes.POINTER(FLOut)]),
    "fl_moe_outs": (None, [_P, _I, _P, _P, _I, _P]),
    "fl_wide_outs": (None, [_P, _I, _I, _P]),
    "fl_wide_skip": (None, [_P, _P, _I, ctypes.POINTER(FLOut)]),
    "fl_fetch": (None, [_P, _I, _I, ctypes.POINTER(FLOut)]),
    "fl_moe": (None, [_P, _P, _P, _P, _I, _I, _P, _P, _I, _I, ctypes.POINTER(FLOut)]),
    "fl_skip": (None, [_P, _P, _I, ctypes.POINTER(FLOut)]),
    "fl_h2d": (None, [_P, _P, _P, _S]),
    "fl_wait_event": (None, [_P, _P]),
    "fl_gpu_ms": (_D, [_P, _I]),
    "fl_moe_prepare": (None, [_P, ctypes.POINTER(FLMoeW), _P, _P, _I, _I, _I]),
    "fl_moe_error": (_I, [_P]),
    "fl_moe_auto": (None, [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.POINTER(FLOut)]),
    "fl_use_graphs": (None, [_P, _I]),
    "fl_free": (None, [_P]),
    "lkfl_init_on_stream": (_P, [_P]),
    "lkfl_moe_adopt": (None, [_P, _P, _P, _P, _I, _S, _P, _P, _I, _I]),
    "lkfl_device_h": (_P, [_P]),
}
# the fused-layer entry points also under the lkfl_ prefix (what a bridge library that re-exports fl_* calls)
SIGNATURES.update({"lk" + k: v for k, v in list(SIGNATURES.items()) if k.startswith("fl_")})

_lib = None


class NativeError(RuntimeError):
    pass


def lib():
    """Load libloki_moe.so (built by loki_b200.build); raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeError("libloki_moe.so not built: run `python -m loki_b200.build` (no fallback exists)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, ctx=None):
    if rc != LK_OK:
        msg = lib().lk_moe_strerror(rc).decode()
        if ctx is not None:
            msg += ": " + lib().lk_moe_last_error(ctx).decode()
        raise NativeError("loki_moe error %d (%s)" % (rc, msg))
    return rc
