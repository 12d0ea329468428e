"""Build libmonarch_attn.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (include/ma_api.h): no torch
headers, cudart linked statically, the driver's cuTensorMapEncodeTiled
resolved at run time through cudaGetDriverEntryPoint.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "libmonarch_attn.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return (sources() + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)])


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, out: str = OUT,
          defines: tuple = ()) -> str:
    """Compile every .cu under csrc/ (one nvcc per file, in parallel) and link
    libmonarch_attn.so; returns its path.

    ``defines`` adds -D flags (e.g. ("MA_TC_TRACE",) for the per-item timeline
    build, written to a separate ``out`` path).
    """
    if not force and out == OUT and up_to_date():
        return out
    from concurrent.futures import ThreadPoolExecutor
    import tempfile
    objdir = tempfile.mkdtemp(prefix="ma_build_")
    dflags = [f"-D{d}" for d in defines]
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *compile_flags, *dflags, "-I", INCLUDE, "-c", "-o", obj, src]
        return obj, cmd, subprocess.run(cmd, capture_output=True, text=True)

    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, srcs))
    log = os.path.join(HERE, "build.log")
    tmp = out + ".tmp"
    link = [nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *[r[0] for r in results]]
    with open(log, "w") as f:
        for obj, cmd, res in results:
            f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        bad = [r for r in results if r[2].returncode != 0]
        if bad:
            shutil.rmtree(objdir, ignore_errors=True)
            raise RuntimeError(f"nvcc failed (see {log}):\n" +
                               "\n".join(r[2].stderr[-4000:] for r in bad))
        res = subprocess.run(link, capture_output=True, text=True)
        f.write(" ".join(link) + "\n" + res.stdout + res.stderr)
    shutil.rmtree(objdir, ignore_errors=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed (see {log}):\n{res.stderr[-4000:]}")
    if verbose:
        print(open(log).read())
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force=True, verbose=True))
