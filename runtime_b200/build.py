"""Build libmfcuda.so (sm_100a) in-tree with nvcc.

    python -m runtime_b200.build [--force] [-j N]

Objects go to runtime_b200/_build/, the shared library to
runtime_b200/libmfcuda.so (both git-ignored).  Compilation is
cross-compilation: no GPU is needed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmfcuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2,-Wall",
          "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(ROOT, "include", "mfcuda.h"))
    return sorted(hs)


def _digest(paths: list[str], extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in paths:
        with open(p, "rb") as fh:
            h.update(p.encode())
            h.update(fh.read())
    return h.hexdigest()


def _compile(src: str, obj: str, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd[-4:-4] = ["-x", "cu"]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr_digest = _digest(headers(), " ".join(ARCH + COMMON))
    objs = []
    todo = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        stamp = obj + ".sha"
        dig = _digest([src], hdr_digest)
        objs.append(obj)
        fresh = (not force and os.path.exists(obj) and os.path.exists(stamp)
                 and open(stamp).read() == dig)
        if not fresh:
            todo.append((src, obj, stamp, dig))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose): (s, o, st, d) for s, o, st, d in todo}
            for fut in cf.as_completed(futs):
                fut.result()
                _, _, stamp, dig = futs[fut]
                with open(stamp, "w") as fh:
                    fh.write(dig)
    if todo or force or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="pass -Xptxas -v")
    a = ap.parse_args(argv)
    print(build(a.force, a.j, a.verbose))


if __name__ == "__main__":
    main()
