"""Build libsx.so (sm_100a) in-tree with nvcc.

Each csrc/*.cu is compiled to an object in parallel, then linked into
ai-research_b200/sx/libsx.so next to this file.  The .so is git-ignored but travels
with the repository snapshot to the GPU box.  A stamp file beside the library holds a
SHA-256 of every source and header, the compiler flags and the nvcc version; the library is
rebuilt whenever that digest differs (file times are not trusted: a checkout or a copy can
make an old library look newer than its sources).
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parents[1] / "include"
BUILD_DIR = PKG_DIR.parents[1] / "_build" / "sx"
LIB_PATH = PKG_DIR / "libsx.so"
STAMP_PATH = PKG_DIR / "libsx.so.stamp"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "sx.h"]


def source_digest(nvcc: str) -> str:
    h = hashlib.sha256()
    ver = subprocess.run([nvcc, "--version"], capture_output=True, text=True).stdout
    h.update(ver.encode())
    h.update(" ".join(ARCH + NVCC_FLAGS).encode())
    for p in _deps():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def up_to_date(digest: str) -> bool:
    return LIB_PATH.exists() and STAMP_PATH.exists() and STAMP_PATH.read_text().strip() == digest


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link libsx.so unless the stamp matches; returns its path.  `built` on the
    returned module attribute LAST_BUILD records whether this call compiled."""
    global LAST_BUILD
    nvcc = _nvcc()
    digest = source_digest(nvcc)
    if not force and up_to_date(digest):
        LAST_BUILD = "up to date (stamp " + digest[:12] + ")"
        return LIB_PATH
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    LAST_BUILD = "compiled (stamp " + digest[:12] + ")"
    return LIB_PATH


LAST_BUILD = "not built in this process"


if __name__ == "__main__":
    print(build(force=True, verbose=True))
