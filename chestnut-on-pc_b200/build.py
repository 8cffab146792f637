"""Build libchestnut.so and libcncomm.so (sm_100a) in-tree with nvcc.

    python chestnut-on-pc_b200/build.py [--force]

libchestnut.so is the engine's only compute path; libcncomm.so is the
clip-end NCCL gather (kept apart so the engine does not load NCCL).  Both are
cross-compiled here (no GPU needed) and the built .so files travel with the
source tree.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "chestnut_b200", "libchestnut.so")
COMM_LIB = os.path.join(HERE, "chestnut_b200", "libcncomm.so")
COMM_SRC = os.path.join(CSRC, "comm", "cn_comm.cu")
SOURCES = ["cn_lib.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
    "--expt-relaxed-constexpr",
    # No f16 arithmetic operators: every half value is converted to f32 before
    # arithmetic, so no half division (run_pinned2.py:622-632 lowers half a/b
    # to a * f16(rcp_f32(b))) can appear in the engine without an explicit
    # intrinsic; tests/test_f16_divide.py checks that none is used.
    "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF2_OPERATORS__",
]


def _stale(lib, deps):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = list(deps) + [os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def nccl_paths():
    """(include dir, lib dir) of the NCCL the image ships with PyTorch (the same
    library torch.distributed loads), else the system one."""
    try:
        import nvidia.nccl
        base = list(nvidia.nccl.__path__)[0]
        if os.path.exists(os.path.join(base, "lib", "libnccl.so.2")):
            return os.path.join(base, "include"), os.path.join(base, "lib")
    except ImportError:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def build_comm(force=False, verbose=False):
    if not force and not _stale(COMM_LIB, [COMM_SRC, os.path.join(HERE, "..", "include", "chestnut_comm.h")]):
        return COMM_LIB
    inc, libdir = nccl_paths()
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", "-I", inc, COMM_SRC, "-o", COMM_LIB, "-L", libdir, "-l:libnccl.so.2",
           "-Xlinker", "-rpath=" + libdir, "-Xlinker", "--exclude-libs,ALL"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode:
        raise RuntimeError("nvcc failed on cn_comm.cu")
    return COMM_LIB


def build(force=False, verbose=False):
    build_comm(force, verbose)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh"))]
    deps.append(os.path.join(HERE, "..", "include", "chestnut.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    objs = []
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    for src in SOURCES:
        obj = os.path.join(bdir, src.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(obj)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB, *objs,
           "-Xlinker", "--exclude-libs,ALL"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
