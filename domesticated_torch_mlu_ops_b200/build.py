"""Build recipe for ``libgdn_b200.so`` (nvcc, sm_100a, in-tree).

``python -m domesticated_torch_mlu_ops_b200.build`` compiles every ``.cu``
file under ``csrc/`` into one shared library next to this file.  nvcc
cross-compiles without a GPU.  The library links the CUDA runtime
statically and exports only the C ABI declared in ``include/gdn_b200.h``.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libgdn_b200.so")

NVCC_FLAGS = [
    "-O3", "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgdn_b200.so")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path.

    Each ``.cu`` file is compiled to an object file on its own process (in
    parallel), then the objects are linked into the shared library."""
    if not force and not _stale():
        return LIB
    import concurrent.futures
    import tempfile

    tmp = LIB + ".tmp"
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    with tempfile.TemporaryDirectory() as objdir:
        objs, cmds = [], []
        for src in sources():
            obj = os.path.join(objdir, os.path.basename(src) + ".o")
            cmd = [_nvcc(), *compile_flags, "-I", INCLUDE, "-I", CSRC, "-c", "-o", obj, src]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            objs.append(obj)
            cmds.append(cmd)
        workers = max(1, min(len(cmds), os.cpu_count() or 1))
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            for f in [pool.submit(_run, c, verbose) for c in cmds]:
                f.result()
        _run([_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp, *objs], verbose)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
