"""Build libloki_moe.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension machinery).

    python -m loki_b200.build            # incremental: per-file objects under loki_b200/_build/
    python -m loki_b200.build --force    # rebuild everything

The library links the CUDA runtime statically (nvcc's default), so it does not depend on which
libcudart the host process (e.g. torch) loaded.
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libloki_moe.so")
# the engine-side replay harness (csrc/fl_replay.cpp): plain C++ against the fl_* ABI of LIB
REPLAY_SRC = os.path.join(CSRC, "fl_replay.cpp")
REPLAY_LIB = os.path.join(HERE, "libloki_replay.so")
SOURCES = ["expert_gemv.cu", "expert_gemv1.cu", "aux_kernels.cu", "router.cu", "dispatch.cu", "prefill_gemm.cu", "gate_up_q8.cu", "moe_api.cu", "fl_abi.cu", "noalloc.cu", "ep.cu", "ep_comm.cu", "slot_mma.cu", "ep_p2p.cu", "expert_kq.cu", "shared_kq.cu", "shared_gemm.cu", "kq_mma.cu"]
HEADERS = ["moe_format.h", "moe_device.cuh", "moe_internal.h", "ep_device.cuh", "tcgen05.cuh", "iq2_tc.cuh", "iq2_grid.inc",
           os.path.join("..", "..", "include", "loki_moe.h"), os.path.join("..", "..", "include", "loki_fused_moe.h"),
           os.path.join("..", "..", "include", "loki_ep.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc():
    for cand in (os.environ.get("NVCC"), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or shutil.which(cand)):
            return cand
    raise RuntimeError("nvcc not found")


def host_cxx():
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, ptxas_verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    hdrs = [os.path.join(CSRC, h) for h in HEADERS]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        if not os.path.exists(s):
            continue
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s, __file__] + hdrs):
            cmd = [nv, "-ccbin", host_cxx()] + ARCH + FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0 or verbose or ptxas_verbose:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError("nvcc failed on %s" % src)
    if force or _stale(LIB, objs):
        cuda_lib = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64")
        # --no-undefined: a symbol declared but defined nowhere fails the link instead of the first dlopen
        cmd = [nv, "-ccbin", host_cxx()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda", "-ldl",
                                                                                "-Xlinker", "-rpath=" + cuda_lib,
                                                                                "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    if force or _stale(REPLAY_LIB, [REPLAY_SRC, LIB, os.path.join(CSRC, "..", "..", "include", "loki_fused_moe.h")]):
        cmd = [host_cxx(), "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-o", REPLAY_LIB, REPLAY_SRC,
               "-L" + HERE, "-lloki_moe", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("replay harness build failed")
    return LIB


BRIDGE_SRC = os.path.join(CSRC, "fl_bridge.cu")
BRIDGE_LIB = os.path.join(HERE, "libloki_fused.so")


def build_bridge(ref, force=False, verbose=False):
    """libloki_fused.so: the engine-facing library exporting all of the reference's src/fused_layer.h -- its
    attention half compiled from the reference checkout `ref` (src/fused_layer.cu, included at build time), its MoE
    half this library (csrc/fl_bridge.cu).  Needs LIB built first."""
    src_ref = os.path.join(ref, "src", "fused_layer.cu")
    deps = [BRIDGE_SRC, LIB, src_ref, os.path.join(CSRC, "..", "..", "include", "loki_fused_moe.h")]
    if not force and not _stale(BRIDGE_LIB, deps):
        return BRIDGE_LIB
    cmd = [nvcc(), "-ccbin", host_cxx()] + ARCH + ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                                                "-w", "-shared", "-I" + os.path.join(ref, "src"), BRIDGE_SRC, "-o", BRIDGE_LIB,
                                                "-L" + HERE, "-lloki_moe", "-Xlinker", "-rpath=$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("bridge build failed")
    return BRIDGE_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/spill/smem reports")
    ap.add_argument("--reference", default=os.environ.get("LOKI_REFERENCE"),
                    help="reference checkout: also build libloki_fused.so (the engine-facing bridge)")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas))
    if a.reference:
        print(build_bridge(a.reference, a.force, a.verbose))
