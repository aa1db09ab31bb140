"""Build ``libnespec.so`` (the C-ABI library of include/nespec.h) in-tree for sm_100a.

    python "inference-engine-from-scratch_b200/build.py"      # or __graft_entry__.build()

nvcc compiles every ``csrc/*.cu`` with ``-gencode arch=compute_100a,code=sm_100a`` and links the
CUDA runtime statically, so the library needs only the NVIDIA driver at run time (it resolves the
driver's ``cuTensorMapEncodeTiled`` through ``cudaGetDriverEntryPoint``). The build is skipped when
the SHA-256 of every source, header and flag, recorded next to the library at its last build
(``libnespec.so.sha256``), still matches: a prebuilt library whose sources changed is rebuilt,
whatever the files' modification times say. The sources compile in parallel.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO / "include"
LIBRARY = PACKAGE_DIR / "libnespec.so"
LIBRARY_HASH = PACKAGE_DIR / "libnespec.so.sha256"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-v",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the B200 kernels need the CUDA toolkit to build")


def nccl_include() -> list[str]:
    """NCCL's public header (types only: the library is dlopen'ed at run time, tp.cu)."""
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
        for root in (spec.submodule_search_locations or []) if spec else []:
            if (Path(root) / "include" / "nccl.h").exists():
                return [f"-I{Path(root) / 'include'}"]
    except Exception:
        pass
    return []  # the system include path (/usr/include/nccl.h)


def nccl_library() -> str | None:
    """The NCCL shared library PyTorch loads (tensor parallelism uses the same one)."""
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
        for root in (spec.submodule_search_locations or []) if spec else []:
            lib = Path(root) / "lib" / "libnccl.so.2"
            if lib.exists():
                return str(lib)
    except Exception:
        pass
    return None


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def source_hash() -> str:
    """SHA-256 over the build inputs: every source and header (name and bytes) and the flags."""
    h = hashlib.sha256()
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    for path in sources() + headers():
        h.update(path.name.encode() + b"\0")
        h.update(path.read_bytes())
        h.update(b"\0")
    return h.hexdigest()


def is_stale() -> bool:
    if not LIBRARY.exists() or not LIBRARY_HASH.exists():
        return True
    return LIBRARY_HASH.read_text().strip() != source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Build if stale. Concurrent callers (several ranks of one job) serialise on a lock file; the
    first builds, the others then find the library fresh."""
    if not force and not is_stale():
        return LIBRARY
    import fcntl

    build_dir = PACKAGE_DIR / "_build"
    build_dir.mkdir(exist_ok=True)
    with open(build_dir / ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not is_stale():
            return LIBRARY
        return _build(build_dir, verbose)


def _build(build_dir: Path, verbose: bool) -> Path:
    from concurrent.futures import ThreadPoolExecutor

    nvcc = nvcc_path()
    digest = source_hash()
    srcs = sources()
    objects = [str(build_dir / (src.stem + ".o")) for src in srcs]

    def compile_one(src: Path, obj: str):
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *nccl_include(), "-c", str(src), "-o", obj]
        return src, subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as pool:
        results = list(pool.map(compile_one, srcs, objects))
    for src, proc in results:
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stderr}")
        if verbose:
            sys.stderr.write(proc.stderr)
    tmp = LIBRARY.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *objects, "-ldl"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{proc.stderr}")
    os.replace(tmp, LIBRARY)
    LIBRARY_HASH.write_text(digest + "\n")
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
