"""Build the in-tree sm_100a shared library ``libcxlsparse_b200.so`` with nvcc.

The library holds every CUDA kernel of the package behind the C ABI declared
in ``include/cxlsparse.h``. It is built in place (next to this file) so it
travels with the source tree; there is no JIT cache.
"""

import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
SOURCES = ["capi.cu", "planner.cu", "attend.cu", "select.cu", "glue.cu", "exchange.cu"]
LIBRARY = PACKAGE / "libcxlsparse_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else "nvcc"


def build(force=False, verbose=False):
    """Compile all sources into one shared library; skip when up to date."""
    csrc = PACKAGE / "csrc"
    inputs = [csrc / s for s in SOURCES] + list(csrc.glob("*.cuh")) + [ROOT / "include" / "cxlsparse.h"]
    if (not force and LIBRARY.exists()
            and LIBRARY.stat().st_mtime >= max(p.stat().st_mtime for p in inputs)):
        return LIBRARY
    build_dir = PACKAGE / "_build"
    build_dir.mkdir(exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-I", str(ROOT / "include"), "-I", str(csrc)]
    if verbose:
        common += ["-Xptxas", "-v"]
    objects = []
    for source in SOURCES:
        obj = build_dir / (source + ".o")
        cmd = common + ["-c", str(csrc / source), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objects], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
