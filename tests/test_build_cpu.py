"""The build covers the sources: every CUDA and C++ file under
neurons_b200/csrc is compiled into libnq.so or libnq_dist.so, and every header
is tracked as a rebuild dependency; the build targets sm_100a alone."""
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "neurons_b200", "csrc")


def test_every_source_is_built():
    from neurons_b200 import build
    files = {os.path.relpath(os.path.join(d, f), CSRC)
             for d, _, fs in os.walk(CSRC) if "_build" not in d for f in fs}
    compiled = set(build.CU_SOURCES) | set(build.CPP_SOURCES) | {build.DIST_SOURCE}
    assert {f for f in files if f.endswith((".cu", ".cpp"))} == compiled
    assert {f for f in files if f.endswith((".h", ".cuh"))} == set(build.HEADERS)


def test_build_targets_sm100a_only(nqlib):
    from neurons_b200 import build
    flags = " ".join(build.ARCH)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert "sm_90" not in flags and "compute_90" not in flags
    for path in (build.LIB, build.DIST_LIB):
        assert os.path.exists(path), path
