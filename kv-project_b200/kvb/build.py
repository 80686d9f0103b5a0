"""Build libkvb.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m kvb.build            # from kv-project_b200/, or through __graft_entry__.build()

The library is written next to this file (``kvb/libkvb.so``) so that it travels with the source
tree; nothing is installed into site-packages and no JIT cache is used.  The units of csrc/ are
compiled in parallel, each into its own device module, and linked into the one shared library
(object files under kv-project_b200/_build/, which is not part of the sources).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parents[1] / "include"
LIB = PKG / "libkvb.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# every translation unit is its own device module (whole-program compilation: relocatable device code
# cost the kernels up to 60 % more registers and the compress kernels 20 % of their speed); the host
# reads every unit's status words (KVB_STATUS_WORDS)
COMPILE_FLAGS = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                 "-Xptxas", "-v", "--expt-relaxed-constexpr"]
LINK_FLAGS = [*ARCH, "--shared", "-Xcompiler", "-fPIC", "-lcudart"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def sources():
    return sorted(CSRC.glob("*.cu"))


def deps():
    return sorted(CSRC.glob("*.cu*")) + [INCLUDE / "kvb.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in deps())


def _compile(src: Path, obj: Path, extra) -> subprocess.CompletedProcess:
    cmd = [nvcc(), *COMPILE_FLAGS, *extra, "-I", str(INCLUDE), "-c", "-o", str(obj), str(src)]
    return subprocess.run(cmd, capture_output=True, text=True)


def build(force: bool = False, verbose: bool = False, extra=(), out: Path | None = None,
          jobs: int | None = None) -> Path:
    """Compile every csrc/*.cu (in parallel, `jobs` at a time) and link them into `out`
    (default kvb/libkvb.so).  `extra`: additional nvcc flags for every unit (e.g. -D switches)."""
    out = Path(out) if out else LIB
    if not force and out == LIB and up_to_date():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    objdir = PKG.parent / "_build" / out.stem
    objdir.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    objs = [objdir / (s.stem + ".o") for s in srcs]
    jobs = jobs or max(1, min(len(srcs), os.cpu_count() or 1))
    with ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda so: _compile(so[0], so[1], list(extra)), zip(srcs, objs)))
    log = "".join(f"=== {s.name}\n{r.stdout}{r.stderr}" for s, r in zip(srcs, results))
    bad = [s.name for s, r in zip(srcs, results) if r.returncode != 0]
    if bad:
        (PKG / "build.log").write_text(log)
        raise RuntimeError(f"nvcc failed on {bad}:\n{log[-6000:]}")
    tmp = out.with_suffix(".so.tmp")
    res = subprocess.run([nvcc(), *LINK_FLAGS, "-o", str(tmp), *map(str, objs)], capture_output=True, text=True)
    log += "=== link\n" + res.stdout + res.stderr
    (PKG / "build.log").write_text(log)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{log[-6000:]}")
    os.replace(tmp, out)
    if verbose:
        print(log)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
