"""The engine's `--dump-moe` records (src/server_core_fused.cpp:359, 814): real activations and routing.

With `--dump-moe FILE` the engine appends, after every MoE layer of a pass, one record for row 0:
  int32 layer, int32 KE, int32 sel[KE] (global expert ids, kept order), float32 w[KE] (kept weights), float32
  x[7168] (the layer's post-ffn_norm hidden state, the MoE input).
Replaying such records through the B200 expert stage next to the oracle pins parity on real activations
and routing once a dump and the model's weights are at hand.
"""
import numpy as np

from .native import HIDDEN


def read_moe_dump(path):
    """All records of a dump file: a list of dicts (layer, keep, sel [KE] int32, w [KE] float32, x [7168] float32)."""
    raw = np.fromfile(path, dtype=np.uint8)
    out, pos = [], 0
    while pos < raw.size:
        if raw.size - pos < 8:
            raise ValueError("%s: truncated record header at byte %d" % (path, pos))
        layer, ke = np.frombuffer(raw[pos:pos + 8].tobytes(), np.int32)
        if not 1 <= ke <= 8:
            raise ValueError("%s: record at byte %d has KE=%d" % (path, pos, ke))
        n = 8 + 4 * (2 * int(ke) + HIDDEN)
        if raw.size - pos < n:
            raise ValueError("%s: truncated record at byte %d" % (path, pos))
        body = raw[pos + 8:pos + n].tobytes()
        sel = np.frombuffer(body, np.int32, int(ke)).copy()
        w = np.frombuffer(body, np.float32, int(ke), 4 * int(ke)).copy()
        x = np.frombuffer(body, np.float32, HIDDEN, 8 * int(ke)).copy()
        out.append({"layer": int(layer), "keep": int(ke), "sel": sel, "w": w, "x": x})
        pos += n
    return out


def write_moe_dump(path, records, append=True):
    """Append records in the engine's byte layout (tests and tools that produce dumps without the engine)."""
    with open(path, "ab" if append else "wb") as f:
        for r in records:
            sel = np.asarray(r["sel"], np.int32)
            f.write(np.array([r["layer"], sel.size], np.int32).tobytes())
            f.write(sel.tobytes())
            f.write(np.asarray(r["w"], np.float32).tobytes())
            f.write(np.asarray(r["x"], np.float32).reshape(HIDDEN).tobytes())
