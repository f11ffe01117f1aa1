"""Build libtgcb.so in-tree with nvcc for sm_100a.

The library holds the runtime (NVRTC compilation, module loading, plan execution) and the
ahead-of-time kernels (long sums, the int8 quantiser). Generated kernels are compiled at
``compile_graph`` time by the library itself, so only this one shared object is built here.
"""

from __future__ import annotations

import os
import subprocess
import sys

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
SOURCE_DIR = os.path.join(os.path.dirname(PACKAGE_DIR), "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(os.path.dirname(PACKAGE_DIR)), "include")
LIBRARY = os.path.join(PACKAGE_DIR, "libtgcb.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
SOURCES = ("runtime.cu", "reductions.cu", "attention.cu", "peer.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_command(output: str = LIBRARY) -> list[str]:
    return [
        os.path.join(CUDA_HOME, "bin", "nvcc"),
        *ARCH,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        f"-I{INCLUDE_DIR}",
        *[os.path.join(SOURCE_DIR, s) for s in SOURCES],
        "-o",
        output,
        f"-L{os.path.join(CUDA_HOME, 'lib64')}",
        "-lnvrtc",
        "-Xlinker",
        f"-rpath={os.path.join(CUDA_HOME, 'lib64')}",
    ]


def is_stale() -> bool:
    if not os.path.exists(LIBRARY):
        return True
    built = os.path.getmtime(LIBRARY)
    deps = [os.path.join(SOURCE_DIR, f) for f in os.listdir(SOURCE_DIR)] + [os.path.join(INCLUDE_DIR, "tgcb.h")]
    return any(os.path.getmtime(d) > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not is_stale():
        return LIBRARY
    tmp = LIBRARY + ".tmp"
    cmd = nvcc_command(tmp)
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
