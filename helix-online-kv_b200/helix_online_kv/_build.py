"""Build libhokv.so in-tree with nvcc for sm_100a (no JIT cache, no torch headers)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
OUT = os.path.join(HERE, "_lib", "libhokv.so")
# profiling variant: the same sources with phase stamps in the decode kernels
VARIANTS = {"": (OUT, []), "stamps": (os.path.join(HERE, "_lib", "libhokv_stamps.so"), ["-DHOKV_STAMPS"])}

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr", "--extended-lambda"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def up_to_date(out: str = OUT) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    deps = sources() + [os.path.join(INCLUDE, "hokv.h")]
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, nvcc: str = "nvcc", verbose: bool = True, variant: str = "") -> str:
    out, extra = VARIANTS[variant]
    if not force and up_to_date(out):
        return out
    os.makedirs(os.path.dirname(out), exist_ok=True)
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-I", CSRC, "-o", out + ".tmp", os.path.join(CSRC, "hokv_lib.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(out + ".tmp", out)
    return out


def build_all(force: bool = False, verbose: bool = True):
    """The product library and the profiling variant, compiled in parallel."""
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(len(VARIANTS)) as ex:
        return list(ex.map(lambda v: build(force=force, verbose=verbose, variant=v), VARIANTS))


if __name__ == "__main__":
    build_all(force=True)
