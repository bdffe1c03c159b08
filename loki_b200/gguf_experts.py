"""A DeepSeek-R1 GGUF file's MoE tensors, loaded into HBM-resident arenas for the B200 kernels.

Replaces the engine's expert indexing and NVMe streaming (src/server_core_fused.cpp:97-110 index the
tensors by name with their file offsets and ggml types; :289-332 `load_experts` copies selected experts into a
VRAM arena): with 180 GB of HBM a layer's experts stay resident, so a layer loads once.  In GGUF an expert
tensor such as `blk.L.ffn_gate_exps.weight` is [n_expert][rows][K] with K innermost (ggml ne = [K, rows,
n_expert]), expert-major -- exactly the arena layout the kernels read (expert e at e * rows * row_bytes), so
each tensor is one contiguous copy.

Tensors per layer L (names as the engine's, server_core_fused.cpp:413, 451, 554-555):
  blk.L.ffn_gate_exps.weight, ffn_up_exps.weight     IQ2_XXS  [256][2048][7168]
  blk.L.ffn_down_exps.weight                          IQ2_XXS / Q2_K / Q3_K  [256][7168][2048]
  blk.L.ffn_gate_inp.weight (F32) or ffn_gate_inp_f16.weight (F16)   router [256][7168]
  blk.L.exp_probs_b.bias                              F32 [256]
  blk.L.ffn_{gate,up,down}_shexp.weight               the shared expert (the real model: Q5_K / Q6_K)

The GGUF container is parsed here (header, key/value metadata, tensor index, aligned data section); no
ggml or gguf-py code is used.
"""
import ctypes
import struct

import numpy as np
import torch

from . import native as N
from .native import HIDDEN, MOE_INTER, N_EXPERTS, FMT_IQ2, FMT_Q2K, FMT_Q3K, FMT_Q5K

GGML_F32, GGML_F16, GGML_Q2_K, GGML_Q3_K, GGML_Q5_K, GGML_Q6_K, GGML_IQ2_XXS = 0, 1, 10, 11, 13, 14, 16
# ggml type -> (weights per block, bytes per block)
TYPE_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q2_K: (256, 84), GGML_Q3_K: (256, 110), GGML_Q5_K: (256, 176),
              GGML_Q6_K: (256, 210), GGML_IQ2_XXS: (256, 66)}
DOWN_FMT = {GGML_IQ2_XXS: FMT_IQ2, GGML_Q2_K: FMT_Q2K, GGML_Q3_K: FMT_Q3K}

# GGUF metadata value types
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GgufError(ValueError):
    pass


class GgufFile:
    """The tensor index of a GGUF (v2/v3) file: name -> (ggml type, ne, absolute offset, bytes)."""

    def __init__(self, path):
        self.path = path
        self.meta = {}
        self.tensors = {}
        with open(path, "rb") as f:
            if f.read(4) != b"GGUF":
                raise GgufError("%s: not a GGUF file" % path)
            version, = struct.unpack("<I", f.read(4))
            if version not in (2, 3):
                raise GgufError("%s: GGUF version %d" % (path, version))
            n_tensors, n_kv = struct.unpack("<QQ", f.read(16))
            for _ in range(n_kv):
                key = self._string(f)
                vtype, = struct.unpack("<I", f.read(4))
                self.meta[key] = self._value(f, vtype)
            infos = []
            for _ in range(n_tensors):
                name = self._string(f)
                n_dims, = struct.unpack("<I", f.read(4))
                ne = list(struct.unpack("<%dQ" % n_dims, f.read(8 * n_dims)))
                ttype, off = struct.unpack("<IQ", f.read(12))
                infos.append((name, ttype, ne, off))
            align = int(self.meta.get("general.alignment", 32))
            pos = f.tell()
            data0 = (pos + align - 1) // align * align
        for name, ttype, ne, off in infos:
            if ttype not in TYPE_BLOCK:
                nbytes = None                     # a type this loader never reads
            else:
                per, bpb = TYPE_BLOCK[ttype]
                if ne[0] % per:
                    raise GgufError("%s: row of %d not a whole number of %d-weight blocks" % (name, ne[0], per))
                nbytes = ne[0] // per * bpb * int(np.prod(ne[1:], dtype=np.int64))
            self.tensors[name] = (ttype, ne, data0 + off, nbytes)

    @staticmethod
    def _string(f):
        n, = struct.unpack("<Q", f.read(8))
        return f.read(n).decode("utf-8", errors="replace")

    def _value(self, f, vtype):
        if vtype in _SCALAR:
            fmt = _SCALAR[vtype]
            return struct.unpack(fmt, f.read(struct.calcsize(fmt)))[0]
        if vtype == _STRING:
            return self._string(f)
        if vtype == _ARRAY:
            etype, n = struct.unpack("<IQ", f.read(12))
            return [self._value(f, etype) for _ in range(n)]
        raise GgufError("unknown metadata value type %d" % vtype)

    def info(self, name):
        if name not in self.tensors:
            raise GgufError("tensor %s not in %s" % (name, self.path))
        return self.tensors[name]

    def bytes(self, name):
        """The tensor's data as a uint8 memmap (copy-on-write: the file is never modified)."""
        ttype, ne, off, nbytes = self.info(name)
        if nbytes is None:
            raise GgufError("%s: ggml type %d is not one this loader reads" % (name, ttype))
        return np.memmap(self.path, dtype=np.uint8, mode="c", offset=off, shape=(nbytes,))   # copy-on-write: never written back


def _expect(g, name, types, ne):
    ttype, tne, _, _ = g.info(name)
    if ttype not in types:
        raise GgufError("%s: ggml type %d, expected one of %s" % (name, ttype, sorted(types)))
    if list(tne[:len(ne)]) != list(ne):
        raise GgufError("%s: ne %s, expected %s.." % (name, tne, ne))
    return ttype, tne


class GgufLayer:
    """One MoE layer of a GGUF file resident in HBM, with the interface of moe.LayerWeights (arenas,
    strides, down format, shared expert, router) for lk_moe_* calls.

    The shared expert is loaded in the real model's formats (Q5_K gate/up, Q6_K down: sh_fmt = FMT_Q5K), or as
    IQ2_XXS gate/up with a down in the routed down's format (sh_fmt = FMT_IQ2).  Any other combination is not
    loaded: `shared_types` records its ggml types and `sh_gate` is None, so the context must run with_shared = 0."""

    def __init__(self, gguf, layer, device="cuda"):
        g = gguf if isinstance(gguf, GgufFile) else GgufFile(gguf)
        self.device = torch.device(device)
        self.layer = layer
        p = "blk.%d." % layer
        _, gne = _expect(g, p + "ffn_gate_exps.weight", {GGML_IQ2_XXS}, [HIDDEN, MOE_INTER])
        self.n_experts = int(gne[2]) if len(gne) > 2 else 1
        self.expert0 = 0
        _expect(g, p + "ffn_up_exps.weight", {GGML_IQ2_XXS}, [HIDDEN, MOE_INTER, self.n_experts])
        dtype_, _ = _expect(g, p + "ffn_down_exps.weight", set(DOWN_FMT), [MOE_INTER, HIDDEN, self.n_experts])
        self.down_fmt = DOWN_FMT[dtype_]
        self.stride = N.EXPERT_MATRIX_BYTES
        self.down_stride = N.DOWN_MATRIX_BYTES[self.down_fmt]
        names = [p + "ffn_gate_exps.weight", p + "ffn_up_exps.weight", p + "ffn_down_exps.weight"]
        self.arenas = [self._upload(g.bytes(n)) for n in names]
        self.gate, self.up, self.down = (a.data_ptr() for a in self.arenas)
        # shared expert
        sh = [p + "ffn_gate_shexp.weight", p + "ffn_up_shexp.weight", p + "ffn_down_shexp.weight"]
        self.shared_types = tuple(g.info(n)[0] for n in sh) if all(n in g.tensors for n in sh) else None
        self.sh_gate = self.sh_up = self.sh_down = None
        self.shared = None
        self.sh_fmt = FMT_IQ2
        if self.shared_types in ((GGML_IQ2_XXS, GGML_IQ2_XXS, dtype_), (GGML_Q5_K, GGML_Q5_K, GGML_Q6_K)):
            model = self.shared_types[0] == GGML_Q5_K
            for n, ne in zip(sh, ([HIDDEN, MOE_INTER], [HIDDEN, MOE_INTER], [MOE_INTER, HIDDEN])):
                _expect(g, n, {self.shared_types[0] if "down" not in n else self.shared_types[2]}, ne)
            self.shared = [self._upload(g.bytes(n)) for n in sh]
            self.sh_gate, self.sh_up, self.sh_down = (a.data_ptr() for a in self.shared)
            self.sh_fmt = FMT_Q5K if model else FMT_IQ2
        # router: F32 [256][7168], or the F16 copy of the engine's trimmed file
        if p + "ffn_gate_inp_f16.weight" in g.tensors:
            _expect(g, p + "ffn_gate_inp_f16.weight", {GGML_F16}, [HIDDEN, N_EXPERTS])
            w = np.frombuffer(g.bytes(p + "ffn_gate_inp_f16.weight"), np.float16).reshape(N_EXPERTS, HIDDEN)
        else:
            _expect(g, p + "ffn_gate_inp.weight", {GGML_F32}, [HIDDEN, N_EXPERTS])
            w = np.frombuffer(g.bytes(p + "ffn_gate_inp.weight"), np.float32).reshape(N_EXPERTS, HIDDEN)
        _expect(g, p + "exp_probs_b.bias", {GGML_F32}, [N_EXPERTS])
        self.router_w = torch.from_numpy(np.array(w)).to(self.device)
        self.router_bias = torch.from_numpy(np.frombuffer(g.bytes(p + "exp_probs_b.bias"), np.float32).copy()).to(self.device)
        torch.cuda.synchronize(self.device)

    def _upload(self, mm):
        t = torch.empty(mm.size, dtype=torch.uint8, device=self.device)
        t.copy_(torch.from_numpy(np.asarray(mm)))
        return t

    @property
    def with_shared(self):
        return self.sh_gate is not None

    def struct(self):
        return N.LkMoeWeights(self.gate, self.up, self.down, self.stride, self.stride, self.down_stride, self.down_fmt,
                              self.sh_gate, self.sh_up, self.sh_down, self.router_w.data_ptr(),
                              1 if self.router_w.dtype == torch.float16 else 0, self.router_bias.data_ptr(),
                              FMT_Q5K if self.sh_fmt == FMT_Q5K else 0)
