"""Build libmlxturbo_b200.so in-tree with nvcc for sm_100a.

    python -m mlxturbo_b200.build [--debug]

The library is plain C ABI (include/mlxturbo_b200.h) over CUDA; it links the
CUDA runtime statically so it loads next to any PyTorch build.  Objects go to
mlxturbo_b200/_build/, the library to mlxturbo_b200/libmlxturbo_b200.so.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmlxturbo_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

SOURCES = ["capi.cu", "qmv.cu", "qmv_sk.cu", "moe.cu", "prefill.cu", "layout.cu", "tmap.cu", "noalloc.cu", "floor.cu", "qmv_i8.cu", "argmax.cu", "moe_decode.cu", "hostcopy.cu"]


def _flags(debug: bool) -> list[str]:
    f = ARCH + ["-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", "-I", os.path.join(os.path.dirname(HERE), "include")]
    f += ["-O0", "-G"] if debug else ["-O3"]
    if os.environ.get("QMM_PTXAS_VERBOSE"):
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, debug: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "mlxturbo_b200.h"))
    if os.path.exists(obj) and all(os.path.getmtime(obj) >= os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *_flags(debug), "-c", path, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip():
        sys.stderr.write(res.stderr)
    return obj


TORCH_BUILD = os.path.join(HERE, "_build_torch")
TORCH_OPS_LIB = os.path.join(HERE, "libmlxturbo_b200_torch.so")


def build_torch_ops() -> str:
    """The PyTorch custom operators (csrc/torch_ops.cpp) over the C ABI, linked
    against libmlxturbo_b200.so (found next to it at run time)."""
    import shutil

    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, LIB, os.path.join(os.path.dirname(HERE), "include", "mlxturbo_b200.h")]
    if os.path.exists(TORCH_OPS_LIB) and all(os.path.getmtime(TORCH_OPS_LIB) >= os.path.getmtime(d) for d in deps):
        return TORCH_OPS_LIB
    from torch.utils import cpp_extension

    os.makedirs(TORCH_BUILD, exist_ok=True)
    # ninja reads `$$` as a literal `$` and the quotes keep the shell from
    # expanding it: the runpath is $ORIGIN, where the library is copied next to
    # libmlxturbo_b200.so below.  cpp_extension loads the freshly built copy
    # too, so the C ABI library (soname libmlxturbo_b200.so) is preloaded.
    import ctypes

    ctypes.CDLL(LIB, mode=ctypes.RTLD_GLOBAL)
    built = cpp_extension.load(
        name="mlxturbo_b200_torch", sources=[src], build_directory=TORCH_BUILD, with_cuda=True,
        is_python_module=False, is_standalone=False, verbose=False,
        extra_cflags=["-O2", "-std=c++17"],
        extra_ldflags=[f"-L{HERE}", "-l:libmlxturbo_b200.so", "'-Wl,-rpath,$$ORIGIN'"])
    path = built if isinstance(built, str) else os.path.join(TORCH_BUILD, "mlxturbo_b200_torch.so")
    shutil.copyfile(path, TORCH_OPS_LIB)
    return TORCH_OPS_LIB


def build(debug: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, debug), SOURCES))
    if os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(o) for o in objs):
        return LIB
    # the soname lets the torch operator library (which names it as NEEDED)
    # resolve to the copy already loaded by the Python layer
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-Xlinker", "-soname=libmlxturbo_b200.so", "-o", LIB, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(debug="--debug" in sys.argv))
    print(build_torch_ops())
