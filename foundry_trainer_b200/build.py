"""Builds the sm_100a shared libraries in-tree (no JIT cache, no pip install).

    python -m foundry_trainer_b200.build            # build what is stale
    python -m foundry_trainer_b200.build --force    # rebuild everything

Outputs (git-ignored, shipped with the tree to the GPU box):
    foundry_trainer_b200/lib/libfoundry_attn.so   the C ABI of include/foundry_attn.h
    foundry_trainer_b200/lib/test_attn_op         C++ host-mirror driver (tests only)
    tests/lib/libfa_selftest.so                   tcgen05 known-answer kernels of
                                                  tests/csrc/ (tests only)
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-I", str(CSRC),
]

LIB_SOURCES = ["capi.cu", "attn_fwd_sm100.cu", "attn_bwd_sm100.cu", "attn_f32.cu", "misc.cu", "peer.cu",
               "qk_prologue.cu",
               "noalloc.cu"]
# test infrastructure: the descriptor / operand-layout known-answer kernels
SELFTEST_SOURCES = [ROOT / "tests" / "csrc" / "umma_selftest.cu"]
SELFTEST_LIB = ROOT / "tests" / "lib" / "libfa_selftest.so"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = OBJ / (src.stem + ".o")
    if _stale(obj, [src] + _headers()) or verbose_ptxas:
        cmd = [nvcc()] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(r.stderr)
            if r.returncode != 0:
                raise RuntimeError(r.stdout + r.stderr)
        else:
            _run(cmd)
    return obj


def _link(objs: list[Path], out: Path) -> None:
    if _stale(out, objs):
        _run([nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC"]
             + [str(o) for o in objs] + ["-o", str(out)])


def build_cpp_driver(force: bool = False) -> Path:
    """C++ mirror of the reference's CustomOp3 surface, exercised on the GPU."""
    src = ROOT / "tests" / "cpp" / "test_attn_op.cpp"
    out = LIB / "test_attn_op"
    deps = [src, ROOT / "include" / "foundry_attn.h", ROOT / "include" / "foundry_attn_op.hpp",
            LIB / "libfoundry_attn.so"]
    if src.exists() and (force or _stale(out, deps)):
        _run(["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
              str(src), "-o", str(out), "-L", str(LIB), "-lfoundry_attn",
              "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{LIB}",
              "-Wl,-rpath,$ORIGIN", "-Wl,-rpath,/usr/local/cuda/lib64"])
    return out


def build_all(force: bool = False, verbose_ptxas: bool = False) -> dict[str, Path]:
    OBJ.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    if force:
        for p in OBJ.glob("*.o"):
            p.unlink()
    SELFTEST_LIB.parent.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in LIB_SOURCES] + SELFTEST_SOURCES
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = dict(zip([s.name for s in srcs], ex.map(lambda s: _compile(s, verbose_ptxas), srcs)))
    lib = LIB / "libfoundry_attn.so"
    st = SELFTEST_LIB
    if force:
        for p in (lib, st):
            if p.exists():
                p.unlink()
    _link([objs[s] for s in LIB_SOURCES], lib)
    _link([objs[s.name] for s in SELFTEST_SOURCES], st)
    drv = build_cpp_driver(force)
    return {"lib": lib, "selftest": st, "cpp_driver": drv}


if __name__ == "__main__":
    out = build_all(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    for k, v in out.items():
        print(f"{k}: {v}")
