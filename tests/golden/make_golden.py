"""Generate the committed golden fixtures (tests/golden/*.npz).

The reference ships no kernel tests or vectors for its MoE path, so the fixtures pin the oracle against an
independent implementation of the same format and against itself over time:

  iq2_xxs_gguf.npz   IQ2_XXS blocks (seeded + hand-built edge blocks covering every grid index, sign index
                     and scale, plus zero / subnormal / negative / large d) and their dequantisation by
                     gguf-py 0.19.0 (gguf.quants.dequantize, the Python port of ggml's
                     dequantize_row_iq2_xxs) -- the independent decode reference.
  generator_kat.npz  the first bytes of seeded weight matrices (seed 0x10C1) for several (layer, matrix,
                     expert) keys -- pins the counter-based generator shared by CPU and GPU.
  router_kat.npz     router outputs (probs, top-8 ids/weights; keep-2 ids/weights; grouped mode) of the
                     oracle on numpy-seeded inputs -- pins routing semantics.
  moe_layer_kat.npz  h / moe of the oracle layer on a small arena (6 experts, T=3) -- pins the layer math.
  kquant_gguf.npz    Q2_K and Q3_K blocks (seeded, uniform random bytes, and edge blocks with zero /
                     subnormal / negative / large d and dmin) and their dequantisation by gguf-py 0.19.0
                     (the Python port of ggml's dequantize_row_q2_K / q3_K), plus the oracle layer with
                     each K-quant down format on a small arena (4 experts, T=2).
  shared_kq_gguf.npz Q5_K and Q6_K blocks (the real model's shared-expert formats; seeded and edge blocks)
                     and their dequantisation by gguf-py 0.19.0, plus the oracle layer with IQ2_XXS routed
                     gate/up, Q3_K routed downs and a Q5_K / Q6_K shared expert (3 experts, T=2).

Run from the repository root:  python tests/golden/make_golden.py [name ...]   (no name: every fixture)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

SEED = 0x10C1


def edge_blocks():
    """Blocks whose groups walk every grid index (256), sign index (128) and scale (16)."""
    rng = np.random.default_rng(7)
    blocks = []
    ds = [0.0, 1e-3, -2.5e-3, 6.0e-8, 1.0, 65504.0, 3.0517578125e-05, 0.5]
    gi = 0
    si = 0
    for b in range(40):
        blk = bytearray(66)
        d = np.float16(ds[b % len(ds)]) if b < len(ds) else np.float16(abs(rng.standard_normal()) * 1e-3)
        blk[0:2] = np.array([d], np.float16).tobytes()
        for g in range(8):
            idx = [(gi + j) % 256 for j in range(4)]
            gi += 4
            sg = [(si + j) % 128 for j in range(4)]
            si += 4
            scale = (b * 8 + g) % 16
            aux1 = sg[0] | (sg[1] << 7) | (sg[2] << 14) | (sg[3] << 21) | (scale << 28)
            blk[2 + 8 * g: 6 + 8 * g] = bytes(idx)
            blk[6 + 8 * g: 10 + 8 * g] = int(aux1).to_bytes(4, "little")
        blocks.append(bytes(blk))
    return np.frombuffer(b"".join(blocks), np.uint8)


def kquant_blocks(fmt, nb):
    """Uniform random blocks whose fp16 scale fields walk the edge values (finite only)."""
    rng = np.random.default_rng(11 + fmt)
    blocks = rng.integers(0, 256, (48, nb), dtype=np.uint8)
    ds = [0.0, 1e-3, -2.5e-3, 6.0e-8, 1.0, 65504.0, 3.0517578125e-05, 0.5, -0.75]
    off = nb - 4 if fmt == O.FMT_Q2K else nb - 2
    for b in range(48):
        d = np.float16(ds[b % len(ds)]) if b < 2 * len(ds) else np.float16(rng.standard_normal() * 1e-3)
        blocks[b, off:off + 2] = np.frombuffer(np.array([d], np.float16).tobytes(), np.uint8)
        if fmt == O.FMT_Q2K:
            m = np.float16(ds[(b + 3) % len(ds)]) if b < 2 * len(ds) else np.float16(abs(rng.standard_normal()) * 1e-3)
            blocks[b, nb - 2:nb] = np.frombuffer(np.array([m], np.float16).tobytes(), np.uint8)
    return blocks.reshape(-1)


def make_kquant():
    from gguf.quants import dequantize
    from gguf import GGMLQuantizationType as QT
    out = {}
    for fmt, qt, tag in ((O.FMT_Q2K, QT.Q2_K, "q2k"), (O.FMT_Q3K, QT.Q3_K, "q3k")):
        nb = O.BLOCK_BYTES[fmt]
        seeded = O.gen_kq(fmt, SEED, 0, 2, 3, 8, 2048)              # 8 rows x 8 blocks
        blocks = np.concatenate([kquant_blocks(fmt, nb), seeded])
        out[tag + "_blocks"] = blocks
        out[tag + "_dequant"] = dequantize(blocks, qt).reshape(-1).astype(np.float32)
        NE = 4
        S = 2048 * 28 * 66
        DS = 7168 * 8 * nb
        gate = np.concatenate([O.gen_iq2(SEED, 11, 0, e, 2048, 7168) for e in range(NE)])
        up = np.concatenate([O.gen_iq2(SEED, 11, 1, e, 2048, 7168) for e in range(NE)])
        down = np.concatenate([O.gen_kq(fmt, SEED, 11, 2, e, 7168, 2048) for e in range(NE)])
        shg, shu = O.gen_iq2(SEED, 11, 0, 256, 2048, 7168), O.gen_iq2(SEED, 11, 1, 256, 2048, 7168)
        shd = O.gen_kq(fmt, SEED, 11, 2, 256, 7168, 2048)
        rng = np.random.default_rng(77)
        xs = rng.standard_normal((2, 7168)).astype(np.float32)
        rs = rng.standard_normal((2, 7168)).astype(np.float32)
        ids = np.array([[0, 3, 1], [2, 0, 3]], np.int32)
        wk = rng.uniform(0.1, 1.0, (2, 3)).astype(np.float32)
        lay = O.moe_layer(xs, rs, gate, up, down, S, ids, wk, shg, shu, shd, down_fmt=fmt, down_stride=DS)
        out[tag + "_layer_ids"] = ids
        out[tag + "_layer_w"] = wk
        out[tag + "_layer_h"] = lay["h"]
        out[tag + "_layer_moe"] = lay["moe"]
    np.savez_compressed(os.path.join(HERE, "kquant_gguf.npz"), **out)


def shared_kq_blocks(fmt, nb):
    """Uniform random Q5_K / Q6_K blocks whose fp16 d (and Q5_K dmin) walk the edge values (finite only)."""
    rng = np.random.default_rng(31 + fmt)
    blocks = rng.integers(0, 256, (48, nb), dtype=np.uint8)
    ds = [0.0, 1e-3, -2.5e-3, 6.0e-8, 1.0, 65504.0, 3.0517578125e-05, 0.5, -0.75]
    doff = 0 if fmt == O.FMT_Q5K else nb - 2
    for b in range(48):
        d = np.float16(ds[b % len(ds)]) if b < 2 * len(ds) else np.float16(rng.standard_normal() * 4e-5)
        blocks[b, doff:doff + 2] = np.frombuffer(np.array([d], np.float16).tobytes(), np.uint8)
        if fmt == O.FMT_Q5K:
            m = np.float16(ds[(b + 3) % len(ds)]) if b < 2 * len(ds) else np.float16(abs(rng.standard_normal()) * 4e-5)
            blocks[b, 2:4] = np.frombuffer(np.array([m], np.float16).tobytes(), np.uint8)
    return blocks.reshape(-1)


def make_shared_kq():
    """The real model's shared-expert formats: Q5_K (gate/up) and Q6_K (down) blocks dequantised by gguf-py,
    and a layer KAT with IQ2_XXS routed gate/up, Q3_K routed downs and a Q5_K / Q6_K shared expert."""
    from gguf.quants import dequantize
    from gguf import GGMLQuantizationType as QT
    out = {}
    for fmt, qt, tag in ((O.FMT_Q5K, QT.Q5_K, "q5k"), (O.FMT_Q6K, QT.Q6_K, "q6k")):
        seeded = O.gen_kq(fmt, SEED, 0, 0 if fmt == O.FMT_Q5K else 2, 256, 8, 2048)
        blocks = np.concatenate([shared_kq_blocks(fmt, O.BLOCK_BYTES[fmt]), seeded])
        out[tag + "_blocks"] = blocks
        out[tag + "_dequant"] = dequantize(blocks, qt).reshape(-1).astype(np.float32)
    lay = shared_kq_layer()
    out.update({"layer_" + k: v for k, v in lay.items()})
    np.savez_compressed(os.path.join(HERE, "shared_kq_gguf.npz"), **out)


def shared_kq_layer():
    """The layer KAT's inputs and outputs (the test rebuilds the weights from the same seeds)."""
    NE = 3
    S, DS = 2048 * 28 * 66, 7168 * 8 * O.BLOCK_BYTES[O.FMT_Q3K]
    gate = np.concatenate([O.gen_iq2(SEED, 12, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([O.gen_iq2(SEED, 12, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([O.gen_kq(O.FMT_Q3K, SEED, 12, 2, e, 7168, 2048) for e in range(NE)])
    shg = O.gen_kq(O.FMT_Q5K, SEED, 12, 0, 256, 2048, 7168)
    shu = O.gen_kq(O.FMT_Q5K, SEED, 12, 1, 256, 2048, 7168)
    shd = O.gen_kq(O.FMT_Q6K, SEED, 12, 2, 256, 7168, 2048)
    rng = np.random.default_rng(78)
    xs = rng.standard_normal((2, 7168)).astype(np.float32)
    rs = rng.standard_normal((2, 7168)).astype(np.float32)
    ids = np.array([[0, 2], [1, 0]], np.int32)
    wk = rng.uniform(0.1, 1.0, (2, 2)).astype(np.float32)
    lay = O.moe_layer(xs, rs, gate, up, down, S, ids, wk, shg, shu, shd, want_slots=True, down_fmt=O.FMT_Q3K, down_stride=DS,
                      sh_gu_fmt=O.FMT_Q5K, sh_down_fmt=O.FMT_Q6K)
    return {"ids": ids, "w": wk, "h": lay["h"], "moe": lay["moe"], "shared": lay["shared"]}


def main(names):
    from gguf.quants import dequantize
    from gguf import GGMLQuantizationType as QT
    if names == ["kquant"]:
        make_kquant()
        print("kquant_gguf.npz written to", HERE)
        return
    if names == ["sharedkq"]:
        make_shared_kq()
        print("shared_kq_gguf.npz written to", HERE)
        return

    seeded = O.gen_iq2(SEED, 0, 0, 3, 8, 7168)            # 8 rows x 28 blocks
    blocks = np.concatenate([edge_blocks(), seeded[: 66 * 64]])
    deq = dequantize(blocks, QT.IQ2_XXS).reshape(-1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "iq2_xxs_gguf.npz"), blocks=blocks, dequant=deq)

    keys = [(0, 0, 0), (0, 1, 0), (0, 2, 0), (1, 0, 255), (57, 2, 256), (3, 1, 17)]
    kat = np.stack([O.gen_iq2(SEED, l, m, e, 2, 7168)[: 2 * 66] for (l, m, e) in keys])
    np.savez_compressed(os.path.join(HERE, "generator_kat.npz"), keys=np.array(keys, np.int32), bytes=kat)

    rng = np.random.default_rng(2024)
    T = 5
    x = rng.standard_normal((T, 7168)).astype(np.float32)
    W = (rng.standard_normal((256, 7168)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    p8, s8, w8 = O.router(x, W, bias, O.route_cfg(8, 8))
    _, s2, w2 = O.router(x, W, bias, O.route_cfg(8, 2))
    _, sg, wg = O.router(x, W, bias, O.route_cfg(8, 8, n_group=8, topk_group=4))
    np.savez_compressed(os.path.join(HERE, "router_kat.npz"), probs=p8, sel8=s8, w8=w8, sel2=s2, w2=w2, selg=sg, wg=wg)

    NE = 6
    S = 2048 * 28 * 66
    gate = np.concatenate([O.gen_iq2(SEED, 9, 0, e, 2048, 7168) for e in range(NE)])
    up = np.concatenate([O.gen_iq2(SEED, 9, 1, e, 2048, 7168) for e in range(NE)])
    down = np.concatenate([O.gen_iq2(SEED, 9, 2, e, 7168, 2048) for e in range(NE)])
    shg, shu, shd = (O.gen_iq2(SEED, 9, 0, 256, 2048, 7168), O.gen_iq2(SEED, 9, 1, 256, 2048, 7168),
                     O.gen_iq2(SEED, 9, 2, 256, 7168, 2048))
    rng = np.random.default_rng(99)
    T, KE = 3, 4
    xs = rng.standard_normal((T, 7168)).astype(np.float32)
    rs = rng.standard_normal((T, 7168)).astype(np.float32)
    ids = np.array([[0, 2, 5, 1], [3, 2, 4, 0], [5, 1, 0, 3]], np.int32)
    wk = rng.uniform(0.1, 1.0, (T, KE)).astype(np.float32)
    out = O.moe_layer(xs, rs, gate, up, down, S, ids, wk, shg, shu, shd)
    np.savez_compressed(os.path.join(HERE, "moe_layer_kat.npz"), ids=ids, w=wk, h=out["h"], moe=out["moe"])
    make_kquant()
    make_shared_kq()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main(sys.argv[1:])
