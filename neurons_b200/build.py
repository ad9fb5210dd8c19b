"""Build libnq.so (the C-ABI library) and libnq_dist.so (its multi-GPU
sharding over NCCL) in-tree for sm_100a with nvcc.

    python -m neurons_b200.build [--force] [-v]

Each .cu under csrc/ is compiled to an object with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, the C++ backend
(csrc/cuda_backend.cpp) with g++ -std=c++23, and everything is linked into
neurons_b200/libnq.so.  Only the CUDA runtime is linked; the driver entry
point for TMA descriptors is resolved at run time through
cudaGetDriverEntryPoint.  `-v` prints ptxas register/spill reports.
libnq_dist.so (csrc/dist.cu) links libnq.so and the NCCL that ships with
torch (the same libnccl.so.2 a torch process has already loaded).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libnq.so")
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")

CU_SOURCES = ["abi.cu", "quant.cu", "gemv.cu", "gemm_tc.cu", "gemm_tc_moe.cu", "moe.cu",
              "moe_small.cu", "llama.cu"]
CPP_SOURCES = ["cuda_backend.cpp", "model_loader.cpp"]
HEADERS = ["nq_common.cuh", "nq_internal.h", "cuda_backend.h", "iface/compute_types.h",
           "iface/compute_backend.h", "model_loader.h"]
# The reference's interface headers, restated, for building libnq on its own
# (inside the reference tree its own core/ headers take their place).
IFACE = os.path.join(CSRC, "iface")

DIST_LIB = os.path.join(HERE, "libnq_dist.so")
DIST_SOURCE = "dist.cu"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def nccl_home():
    """Directory holding include/nccl.h and lib/libnccl.so.2 (torch's NCCL)."""
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is None or not spec.submodule_search_locations:
        raise RuntimeError("NCCL (the nvidia-nccl package torch depends on) was not found")
    return list(spec.submodule_search_locations)[0]
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + INCLUDE]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "nq.h")]
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or verbose or _newer(o, [s] + hdrs):
            cmd = [NVCC] + ARCH + NVFLAGS + ["-c", s, "-o", o]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            subprocess.run(cmd, check=True)
    for src in CPP_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            subprocess.run(["g++", "-O2", "-std=c++23", "-fPIC", "-Wall", "-I" + INCLUDE,
                            "-I" + IFACE,
                            "-I" + os.path.join(CUDA_HOME, "include"), "-c", s, "-o", o],
                           check=True)
    if force or _newer(LIB, objs):
        tmp = LIB + ".tmp%d" % os.getpid()
        subprocess.run([NVCC] + ARCH + ["-shared", "-o", tmp] + objs +
                       ["-lcudart", "-Xlinker", "-rpath," + os.path.join(CUDA_HOME, "lib64")],
                       check=True)
        os.replace(tmp, LIB)
    build_dist(force, verbose)
    return LIB


def build_dist(force: bool = False, verbose: bool = False) -> str:
    nccl = nccl_home()
    s = os.path.join(CSRC, DIST_SOURCE)
    o = os.path.join(BUILD, DIST_SOURCE + ".o")
    deps = [s, os.path.join(INCLUDE, "nq.h"), os.path.join(INCLUDE, "nq_dist.h")]
    if force or verbose or _newer(o, deps):
        subprocess.run([NVCC] + ARCH + NVFLAGS + ["-I" + os.path.join(nccl, "include"), "-c", s,
                                                  "-o", o], check=True)
    if force or _newer(DIST_LIB, [o, LIB]):
        tmp = DIST_LIB + ".tmp%d" % os.getpid()
        subprocess.run([NVCC] + ARCH + ["-shared", "-o", tmp, o, "-L" + HERE, "-lnq",
                                        "-L" + os.path.join(nccl, "lib"), "-l:libnccl.so.2",
                                        "-lcudart", "-Xlinker", "-rpath,$ORIGIN",
                                        "-Xlinker", "-rpath," + os.path.join(nccl, "lib"),
                                        "-Xlinker", "-rpath," + os.path.join(CUDA_HOME, "lib64")],
                       check=True)
        os.replace(tmp, DIST_LIB)
    return DIST_LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
