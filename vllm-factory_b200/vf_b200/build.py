"""Builds libvf_b200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is a plain shared object: no torch headers, no torch ABI.  It is written
next to this file so that it travels with the source tree and is the one loaded by
`vf_b200._lib`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parent.parent / "include"
LIB_PATH = PKG_DIR / "libvf_b200.so"
TORCH_LIB_PATH = PKG_DIR / "libvf_b200_torch.so"
SOURCES = [CSRC / "vf_attention.cu", CSRC / "vf_deberta_fused.cu", CSRC / "vf_ffn.cu", CSRC / "vf_layernorm.cu",
           CSRC / "vf_span.cu", CSRC / "vf_gemm.cu"]
DEPS = SOURCES + [CSRC / "vf_ptx.cuh", CSRC / "vf_internal.h", INCLUDE / "vf_b200.h"]
TORCH_SOURCES = [CSRC / "vf_torch_ops.cpp"]
TORCH_DEPS = TORCH_SOURCES + [INCLUDE / "vf_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
    "-shared",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libvf_b200.so")
    return cand


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def is_stale() -> bool:
    return _stale(LIB_PATH, DEPS) or _stale(TORCH_LIB_PATH, TORCH_DEPS + [LIB_PATH])


def system_cxx() -> str:
    """The C++ compiler for the torch op layer: VF_CXX if set, else the system g++ (the GCC
    13 that torch itself was built with, linking the shared libstdc++.so.6).  $CXX is not
    used: a toolchain that links libstdc++ statically into the library gives the process a
    second copy of the C++ runtime, and then formatting a number into an exception message
    (any TORCH_CHECK with a value in its text) crashes on the duplicated locale facets."""
    cand = os.environ.get("VF_CXX") or shutil.which("g++", path="/usr/bin:/bin") or shutil.which("g++")
    if not cand:
        raise RuntimeError("no C++ compiler found for the torch op layer (set VF_CXX)")
    return cand


def embedded_cxx_runtime(lib: Path) -> list[str]:
    """libstdc++ internals that `lib` defines itself (empty for a library that uses the
    process's shared libstdc++.so.6)."""
    res = subprocess.run(["nm", "-D", "-C", "--defined-only", str(lib)], capture_output=True, text=True)
    if res.returncode != 0:
        return []
    bad = ("std::locale::id::_M_id", "std::locale::facet::_M_cow_shim", "std::ios_base::Init::Init")
    return [l for l in res.stdout.splitlines() if any(b in l for b in bad)]


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the torch op layer (csrc/vf_torch_ops.cpp) against torch's headers and the
    C ABI library; the result is loaded with torch.ops.load_library."""
    if not force and not _stale(TORCH_LIB_PATH, TORCH_DEPS + [LIB_PATH]):
        return TORCH_LIB_PATH
    import torch
    from torch.utils import cpp_extension as ce
    cxx = system_cxx()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + [f"-I{INCLUDE}"]
    libdirs = ce.library_paths(device_type="cuda")
    tmp = TORCH_LIB_PATH.with_suffix(".so.tmp")
    # The flags torch.utils.cpp_extension gives an extension (same compiler family as torch's
    # own build: GCC 13), with hidden visibility so that no template instantiation of this
    # library interposes on torch's.
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *incs, *map(str, TORCH_SOURCES), "-o", str(tmp),
           *[f"-L{d}" for d in libdirs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           f"-L{PKG_DIR}", "-lvf_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"torch op layer build failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    embedded = embedded_cxx_runtime(tmp)
    if embedded:
        tmp.unlink()
        raise RuntimeError(f"{cxx} linked its own copy of libstdc++ into the torch op layer "
                           f"(e.g. {embedded[0].strip()}); build with the system g++ (VF_CXX)")
    os.replace(tmp, TORCH_LIB_PATH)
    return TORCH_LIB_PATH


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles whatever is missing or older than its sources; returns the kernel library."""
    build_kernels(force=force, verbose=verbose)
    build_torch_ops(force=force, verbose=verbose)
    return LIB_PATH


def build_kernels(force: bool = False, verbose: bool = False) -> Path:
    """nvcc: the sm_100a kernels and the C ABI -> libvf_b200.so."""
    if not force and not _stale(LIB_PATH, DEPS):
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(INCLUDE), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
