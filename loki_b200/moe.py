"""Host-side API of the B200 MoE layer: HBM-resident expert shards and the layer call.

Mirrors the reference's MoE interface (src/fused_layer.h fl_moe / fl_wide_moe and the engine's arena
layout, src/server_core_fused.cpp:301-317) with device-resident tensors: one layer's routed experts live
in three arenas (gate, up, down), expert e at byte e * stride, every matrix in GGUF IQ2_XXS layout.
torch supplies device memory and streams; every computation runs in libloki_moe.so.
"""
import ctypes

import torch

from . import native as N
from .native import HIDDEN, MOE_INTER, N_EXPERTS, EXPERT_MATRIX_BYTES, FMT_IQ2, check, lib

ALIGN = 256


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def gen_iq2(dst, seed, layer, matrix, expert0, n_exp, rows, K, stride, stream=None):
    """Fill dst (a uint8 CUDA tensor or a raw device address) with seeded IQ2_XXS matrices."""
    addr = dst if isinstance(dst, int) else dst.data_ptr()
    check(lib().lk_gen_iq2(ctypes.c_void_p(addr), seed, layer, matrix, expert0, n_exp, rows, K, stride, _stream(stream)))


def gen_weights(fmt, dst, seed, layer, matrix, expert0, n_exp, rows, K, stride, stream=None):
    """Seeded matrices in any supported format (IQ2_XXS, Q2_K, Q3_K, Q5_K, Q6_K); the CPU generator's bytes."""
    addr = dst if isinstance(dst, int) else dst.data_ptr()
    check(lib().lk_gen_weights(fmt, ctypes.c_void_p(addr), seed, layer, matrix, expert0, n_exp, rows, K, stride, _stream(stream)))


class LayerWeights:
    """One MoE layer's weights, resident in HBM.

    buf layout (bytes): [gate x n_experts][up x n_experts][down x n_experts][shared gate][shared up][shared down],
    each gate/up matrix EXPERT_MATRIX_BYTES (3 784 704, a multiple of 256) of seeded IQ2_XXS, each down matrix
    DOWN_MATRIX_BYTES[down_fmt] in down_fmt (IQ2_XXS, or the real model's Q2_K / Q3_K), all from the seeded
    generators (matrix ids 0/1/2, shared expert id 256).  The shared expert is IQ2_XXS with a down in down_fmt
    (sh_fmt = FMT_IQ2), or in the real model's formats (sh_fmt = FMT_Q5K: Q5_K gate/up, Q6_K down).
    An expert-parallel shard holds the n_experts
    consecutive global experts starting at expert0 (arena slot i = global expert expert0 + i).  Router weights/bias are given or drawn from
    torch's generator: W ~ N(0, 0.02) [n_experts][7168] fp32 (or fp16), bias ~ N(0, 0.01)."""

    def __init__(self, device, seed, layer, n_experts=N_EXPERTS, with_shared=True, router_w=None, router_bias=None,
                 router_f16=False, stream=None, buf=None, expert0=0, down_fmt=FMT_IQ2, sh_fmt=FMT_IQ2):
        self.device = torch.device(device)
        self.seed, self.layer, self.n_experts, self.with_shared = seed, layer, n_experts, with_shared
        self.expert0 = expert0
        self.down_fmt = down_fmt
        self.sh_fmt = sh_fmt
        S, DS = EXPERT_MATRIX_BYTES, N.DOWN_MATRIX_BYTES[down_fmt]
        sh_gu_fmt, sh_dn_fmt = (N.FMT_Q5K, N.FMT_Q6K) if sh_fmt == N.FMT_Q5K else (FMT_IQ2, down_fmt)
        self.sh_sizes = (N.GU_MATRIX_BYTES[sh_gu_fmt], N.GU_MATRIX_BYTES[sh_gu_fmt], N.DOWN_MATRIX_BYTES[sh_dn_fmt])
        self.nbytes = (2 * S + DS) * n_experts + (sum(self.sh_sizes) if with_shared else 0)
        self.buf = buf if buf is not None else torch.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        base = self.buf.data_ptr()
        self.gate, self.up, self.down = base, base + n_experts * S, base + 2 * n_experts * S
        self.stride, self.down_stride = S, DS
        gen_iq2(self.gate, seed, layer, 0, expert0, n_experts, MOE_INTER, HIDDEN, S, stream)
        gen_iq2(self.up, seed, layer, 1, expert0, n_experts, MOE_INTER, HIDDEN, S, stream)
        gen_weights(down_fmt, self.down, seed, layer, 2, expert0, n_experts, HIDDEN, MOE_INTER, DS, stream)
        if with_shared:
            sh = base + n_experts * (2 * S + DS)
            SG = self.sh_sizes[0]
            self.sh_gate, self.sh_up, self.sh_down = sh, sh + SG, sh + 2 * SG
            gen_weights(sh_gu_fmt, self.sh_gate, seed, layer, 0, N_EXPERTS, 1, MOE_INTER, HIDDEN, SG, stream)
            gen_weights(sh_gu_fmt, self.sh_up, seed, layer, 1, N_EXPERTS, 1, MOE_INTER, HIDDEN, SG, stream)
            gen_weights(sh_dn_fmt, self.sh_down, seed, layer, 2, N_EXPERTS, 1, HIDDEN, MOE_INTER, self.sh_sizes[2], stream)
        else:
            self.sh_gate = self.sh_up = self.sh_down = None
        if router_w is None:
            g = torch.Generator(device=self.device).manual_seed(seed * 1000003 + layer)
            router_w = torch.randn(N_EXPERTS, HIDDEN, generator=g, device=self.device) * 0.02
            if router_bias is None:
                router_bias = torch.randn(N_EXPERTS, generator=g, device=self.device) * 0.01
        self.router_w = router_w.to(self.device).contiguous()
        if router_f16:
            self.router_w = self.router_w.half()
        self.router_bias = router_bias.to(self.device, torch.float32).contiguous()

    def struct(self):
        return N.LkMoeWeights(self.gate, self.up, self.down, self.stride, self.stride, self.down_stride, self.down_fmt,
                              self.sh_gate, self.sh_up, self.sh_down, self.router_w.data_ptr(),
                              1 if self.router_w.dtype == torch.float16 else 0, self.router_bias.data_ptr(),
                              self.sh_fmt if self.sh_fmt == N.FMT_Q5K else 0)

    def expert_bytes(self, expert, matrix):
        """Host copy of one expert matrix (matrix 0 gate, 1 up, 2 down; expert == n_experts: shared)."""
        size = self.down_stride if matrix == 2 else self.stride
        if expert == self.n_experts:
            off = self.n_experts * (2 * self.stride + self.down_stride) + sum(self.sh_sizes[:matrix])
            size = self.sh_sizes[matrix]
        else:
            off = matrix * self.n_experts * self.stride + expert * size
        return self.buf[off:off + size].cpu().numpy()


class MoeLayer:
    """A B200 MoE-layer context (scratch buffers for up to max_tokens tokens) bound to one device."""

    def __init__(self, device=0, topk=8, keep=8, renorm=True, n_group=1, topk_group=1, scale=2.5, with_shared=True,
                 max_tokens=512, n_experts=N_EXPERTS):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.cfg = N.LkMoeConfig(n_experts, topk, keep, int(renorm), n_group, topk_group, scale, int(with_shared),
                                 max_tokens)
        h = ctypes.c_void_p()
        check(lib().lk_moe_create(ctypes.byref(self.cfg), self.device.index or 0, ctypes.byref(h)))
        self.ctx = h
        self.keep = keep

    def close(self):
        if self.ctx:
            lib().lk_moe_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        return check(rc, self.ctx)

    def forward(self, W, x, resid, logits_override=None, h=None, moe=None, sel=None, w=None, stream=None):
        """h, moe, sel, w = layer(x, resid): all CUDA tensors; outputs allocated when not given."""
        T = x.shape[0]
        dev = x.device
        h = torch.empty(T, HIDDEN, device=dev) if h is None else h
        moe = torch.empty(T, HIDDEN, device=dev) if moe is None else moe
        sel = torch.empty(T, self.keep, dtype=torch.int32, device=dev) if sel is None else sel
        w = torch.empty(T, self.keep, device=dev) if w is None else w
        ws = W.struct() if hasattr(W, "struct") else W
        self._check(lib().lk_moe_forward(self.ctx, ctypes.byref(ws), _ptr(x), _ptr(resid), T, _ptr(logits_override),
                                         _ptr(h), _ptr(moe), _ptr(sel), _ptr(w), _stream(stream)))
        return h, moe, sel, w

    def route(self, W, x, logits_override=None, stream=None):
        T = x.shape[0]
        sel = torch.empty(T, self.keep, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.keep, device=x.device)
        probs = torch.empty(T, N_EXPERTS, device=x.device)
        ws = W.struct() if hasattr(W, "struct") else W
        self._check(lib().lk_moe_route(self.ctx, ctypes.byref(ws), _ptr(x), T, _ptr(logits_override), _ptr(sel), _ptr(w),
                                       _ptr(probs), _stream(stream)))
        return probs, sel, w

    def dispatch(self, sel, w, stream=None):
        T, keep = sel.shape
        counts = torch.empty(N_EXPERTS, dtype=torch.int32, device=sel.device)
        offsets = torch.empty(N_EXPERTS + 1, dtype=torch.int32, device=sel.device)
        perm = torch.empty(T * keep, dtype=torch.int32, device=sel.device)
        self._check(lib().lk_moe_dispatch(self.ctx, _ptr(sel), _ptr(w), T, keep, _ptr(counts), _ptr(offsets), _ptr(perm),
                                          _stream(stream)))
        return counts, offsets, perm

    def experts(self, W, x, resid, sel, w, h=None, moe=None, stream=None):
        T, keep = sel.shape
        h = torch.empty(T, HIDDEN, device=x.device) if h is None else h
        moe = torch.empty(T, HIDDEN, device=x.device) if moe is None else moe
        ws = W.struct() if hasattr(W, "struct") else W
        self._check(lib().lk_moe_experts(self.ctx, ctypes.byref(ws), _ptr(x), _ptr(resid), T, _ptr(sel), _ptr(w), keep,
                                         _ptr(h), _ptr(moe), _stream(stream)))
        return h, moe

    def set_gemm_threshold(self, min_tokens):
        """Use the tensor-core GEMM path for calls with at least min_tokens tokens (default 192)."""
        self._check(lib().lk_moe_set_gemm_threshold(self.ctx, min_tokens))

    def set_mma_threshold(self, min_tokens):
        """Below the GEMM threshold, use the register-fed mma.sync path for calls with >= min_tokens tokens."""
        self._check(lib().lk_moe_set_mma_threshold(self.ctx, min_tokens))

    def set_shared_gemm_threshold(self, min_tokens):
        """Run a Q5_K/Q6_K shared expert as dense fp16 GEMMs for calls with >= min_tokens tokens (default 16)."""
        self._check(lib().lk_moe_set_shared_gemm_threshold(self.ctx, min_tokens))

    def device_error(self, stream=None):
        """Synchronise and return the device error status (0 = none); raises on a recorded error."""
        return self._check(lib().lk_moe_get_error(self.ctx, _stream(stream)))
