"""Build and load the native parts: libfrn_b200.so (C ABI + sm_100a kernels)
and the ``denominator_cuda`` pybind11 module layered on it.

Both artefacts are built in-tree under ``<project>/lib`` so that they travel
with the source tree; a content hash of the sources and flags is stored next
to each one, and a stale or missing artefact is rebuilt on first use (the
reference also JIT-builds ``denominator_cuda`` at import time, reference
src/load_cuda.py:11-20).  Nothing here falls back to a CPU or pure-PyTorch
implementation: if the library cannot be built or loaded, loading raises.
"""

from __future__ import annotations

import concurrent.futures
import contextlib
import ctypes
import fcntl
import hashlib
import importlib.machinery
import importlib.util
import os
import subprocess
import sys
import threading

PROJECT_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO_DIR = os.path.dirname(PROJECT_DIR)
CSRC_DIR = os.path.join(PROJECT_DIR, "csrc")
LIB_DIR = os.path.join(PROJECT_DIR, "lib")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")

LIB_NAME = "libfrn_b200.so"
LIB_PATH = os.path.join(LIB_DIR, LIB_NAME)

CU_SOURCES = [
    "frn_capi.cu",
    "frn_fused_linear.cu",
    "frn_fused_linear_pair.cu",
    "frn_decode.cu",
    "frn_fused_linear_w8.cu",
    "frn_normalize.cu",
    "frn_gqa_decode.cu",
    "frn_gqa_decode_mma.cu",
]
HEADERS = ["frn_ptx.cuh", "frn_internal.h", "frn_pair_common.cuh"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    f"-I{INCLUDE_DIR}",
]

_lock = threading.Lock()
_lib_handle = None
_ext_module = None


def _nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _digest(paths, extra: str) -> str:
    h = hashlib.sha256()
    for p in paths:
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(extra.encode())
    return h.hexdigest()


def _read(path: str) -> str:
    try:
        with open(path) as f:
            return f.read().strip()
    except OSError:
        return ""


def _lib_inputs():
    files = [os.path.join(CSRC_DIR, s) for s in CU_SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE_DIR, "frn_b200.h"))
    return files


def _flags_key() -> str:
    # The include path is absolute; the tree may be copied elsewhere (another
    # machine, a scratch directory), so the stamp records it relative.
    return " ".join(f.replace(REPO_DIR, "<repo>") for f in NVCC_FLAGS)


@contextlib.contextmanager
def _build_lock():
    """Inter-process lock around check-and-build: several ranks of one job
    import the package at once and must not build (or load a half-written
    library) concurrently."""
    os.makedirs(LIB_DIR, exist_ok=True)
    with open(os.path.join(LIB_DIR, ".build.lock"), "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        try:
            yield
        finally:
            fcntl.flock(f, fcntl.LOCK_UN)


def library_is_fresh() -> bool:
    want = _digest(_lib_inputs(), _flags_key())
    return os.path.exists(LIB_PATH) and _read(LIB_PATH + ".sha256") == want


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu for sm_100a and link libfrn_b200.so (in-tree)."""
    with _build_lock():
        return _build_library_locked(force, verbose)


def _build_library_locked(force: bool, verbose: bool) -> str:
    want = _digest(_lib_inputs(), _flags_key())
    if not force and os.path.exists(LIB_PATH) and _read(LIB_PATH + ".sha256") == want:
        return LIB_PATH
    obj_dir = os.path.join(LIB_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = _nvcc()

    def compile_one(src):
        obj = os.path.join(obj_dir, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc] + NVCC_FLAGS + ["-c", os.path.join(CSRC_DIR, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, file=sys.stderr)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(CU_SOURCES))) as ex:
        objs = list(ex.map(compile_one, CU_SOURCES))
    tmp = f"{LIB_PATH}.{os.getpid()}.tmp"
    cmd = [nvcc] + ARCH_FLAGS + ["-rdc=true", "-shared", "-Xlinker", f"-soname={LIB_NAME}",
                                 "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    with open(LIB_PATH + ".sha256", "w") as f:
        f.write(want + "\n")
    return LIB_PATH


def load_library() -> ctypes.CDLL:
    """dlopen libfrn_b200.so (building it first if missing or stale).

    Loaded RTLD_GLOBAL so that the pybind11 module, which links against the
    same soname, resolves to this very copy.
    """
    global _lib_handle
    with _lock:
        if _lib_handle is None:
            path = build_library()
            _lib_handle = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        return _lib_handle


def _ext_build_dir() -> str:
    return os.path.join(LIB_DIR, "denominator_cuda_build")


def _ext_inputs():
    return [os.path.join(CSRC_DIR, "denominator.cpp"), os.path.join(INCLUDE_DIR, "frn_b200.h")]


def _ext_digest() -> str:
    import torch

    return _digest(_ext_inputs(), f"torch={torch.__version__} py={sys.version_info[:2]}")


def _ext_so_path() -> str:
    return os.path.join(_ext_build_dir(), "denominator_cuda.so")


def _import_so(name: str, path: str):
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def build_denominator_cuda(force: bool = False, verbose: bool = False):
    """Build (if needed) and import the ``denominator_cuda`` module."""
    import torch  # noqa: F401  (the module links against torch's libraries)
    import torch.utils.cpp_extension as ext

    load_library()
    with _build_lock():
        return _build_denominator_cuda_locked(force, verbose)


def _build_denominator_cuda_locked(force: bool, verbose: bool):
    import torch.utils.cpp_extension as ext

    so = _ext_so_path()
    want = _ext_digest()
    if not force and os.path.exists(so) and _read(so + ".sha256") == want:
        return _import_so("denominator_cuda", so)
    os.makedirs(_ext_build_dir(), exist_ok=True)
    # Same bypass as the reference loader (src/load_cuda.py:5-7): the
    # toolkit here (12.9) is newer than torch's CUDA build (12.8).
    orig_check = ext._check_cuda_version
    ext._check_cuda_version = lambda *a, **k: None
    try:
        mod = ext.load(
            name="denominator_cuda",
            sources=[os.path.join(CSRC_DIR, "denominator.cpp")],
            extra_cflags=["-O3", "-std=c++17"],
            extra_include_paths=[INCLUDE_DIR],
            extra_ldflags=[f"-L{LIB_DIR}", "-lfrn_b200"],
            build_directory=_ext_build_dir(),
            with_cuda=True,
            verbose=verbose,
        )
    finally:
        ext._check_cuda_version = orig_check
    with open(so + ".sha256", "w") as f:
        f.write(want + "\n")
    return mod


def load_denominator_cuda():
    global _ext_module
    with _lock:
        if _ext_module is not None:
            return _ext_module
    mod = build_denominator_cuda()
    with _lock:
        _ext_module = mod
    return mod


def build_all(force: bool = True, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_denominator_cuda(force=force, verbose=verbose)
