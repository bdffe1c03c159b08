"""The engine binding links: a stand-in for the engine's translation unit (tests/engine_standin.cpp: every
fused-layer call src/server_core_fused.cpp makes, compiled against the reference's own src/fused_layer.h) links
against libloki_fused.so alone -- the reference's attention half from its checkout, this library's MoE half --
with every symbol resolved at load time (LD_BIND_NOW).  CPU only: nothing is called on a GPU.  Skipped where no
reference checkout is available (the bridge is built from it)."""
import os
import re
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _checkout():
    sys.path.insert(0, REPO)
    import __graft_entry__ as g
    return g.reference_checkout()


@pytest.fixture(scope="module")
def bridge(native):
    ref = _checkout()
    if not ref:
        pytest.skip("no reference checkout: the bridge is built from its src/fused_layer.cu")
    from loki_b200 import build as B
    return ref, B.build_bridge(ref)


def _exports(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if l.strip()}


def test_bridge_exports_the_whole_fused_layer_header(bridge):
    ref, lib = bridge
    header = open(os.path.join(ref, "src", "fused_layer.h")).read()
    declared = set(re.findall(r"\b(fl_[a-z0-9_]+)\s*\(", header))
    assert declared, "no fl_* declarations found in the reference header"
    got = {s for s in _exports(lib) if s.startswith("fl_")}
    assert declared == got, (sorted(declared - got), sorted(got - declared))


def test_engine_standin_links_and_loads(bridge, tmp_path):
    ref, lib = bridge
    exe = tmp_path / "engine"
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    libdir = os.path.dirname(lib)
    cmd = ["g++", "-std=c++17", "-O1", "-I" + os.path.join(ref, "src"), "-I" + cuda_inc,
           os.path.join(REPO, "tests", "engine_standin.cpp"), "-o", str(exe), "-L" + libdir, "-lloki_fused",
           "-Wl,-rpath," + libdir, "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    # only libloki_fused.so is named at link time; every fl_* the engine calls resolves in it
    needed = subprocess.run(["readelf", "-d", str(exe)], capture_output=True, text=True).stdout
    assert "libloki_fused.so" in needed and "libloki_moe.so" not in needed
    env = dict(os.environ, LD_BIND_NOW="1")
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "linked" in r.stdout
