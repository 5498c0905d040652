"""Build libcubutterfly_b200.so in-tree for sm_100a.

Run ``python -m cubutterfly_b200._build`` (or ``__graft_entry__.build()``).
Objects go to ``cubutterfly_b200/_build/``, the library to
``cubutterfly_b200/lib/libcubutterfly_b200.so``.  Compilation units are built
in parallel and only when their sources changed.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libcubutterfly_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

# (operator, storage) units of the FWHT / zeta tile kernels
BW_UNITS = [(0, 0), (0, 1), (0, 2), (1, 3), (1, 4), (2, 3), (2, 4)]


def _json_include() -> str:
    cands = []
    for base in sys.path + [os.path.dirname(os.__file__)]:
        cands += glob.glob(os.path.join(base, "include", "cudnn_frontend", "thirdparty"))
    cands += glob.glob("/usr/include/nlohmann/..")
    for c in cands:
        if os.path.exists(os.path.join(c, "nlohmann", "json.hpp")):
            return os.path.abspath(c)
    raise RuntimeError("nlohmann/json.hpp not found (needed to build the C ABI)")


def _units():
    common = [NVCC, "-std=c++17", *ARCH, "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{_json_include()}"]
    units = []
    for name in ("c_api.cpp", "descriptor.cpp", "planner.cpp", "rns_api.cpp", "launch_bitwise_dispatch.cpp",
                 "launch_ntt_dispatch.cpp", "launch_fft.cu", "noalloc.cu", "fourstep.cu", "bitrev.cu", "fwht_tc.cu",
                 "real_adapter.cu", "real_fft.cu", "calibrate.cu", "fourstep_peer.cu", "unaligned.cu", "structured.cu", "fwht_native.cu", "fft64.cu", "fft_chain.cu",
                 "heongpu_adapter.cpp", "bluestein.cu"):
        src = CSRC / name
        obj = OBJ / (src.stem + ".o")
        units.append((common + ["-c", str(src), "-o", str(obj)], src, obj))
    for word in (64, 32):  # NTT storage words
        src = CSRC / "launch_ntt.cu"
        obj = OBJ / f"ntt_w{word}.o"
        units.append((common + [f"-DCUBF_NTT_WORD={word}", "-c", str(src), "-o", str(obj)], src, obj))
    for op, ty in BW_UNITS:
        src = CSRC / "launch_bitwise.cu"
        obj = OBJ / f"bitwise_{op}_{ty}.o"
        units.append((common + [f"-DCUBF_BW_OP={op}", f"-DCUBF_BW_TYPE={ty}", "-c", str(src), "-o", str(obj)],
                      src, obj))
    return units


def _stale(obj: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    deps = list(CSRC.glob("*")) + list((ROOT / "include").rglob("*.h*")) + [Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    units = _units()
    todo = [u for u in units if _stale(u[2])]

    def run(u):
        cmd, src, obj = u
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("built", obj.name, flush=True)
        return obj

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or max(2, os.cpu_count() or 2)) as ex:
            list(ex.map(run, todo))
    if todo or not LIB.exists():
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *[str(u[2]) for u in units], "-cudart", "static",
               "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
