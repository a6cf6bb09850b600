"""Builds libjxattn.so (the sm_100a decode-attention library) in-tree.

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the CUDA
12.9 toolkit is installed.  Objects go to jxai_b200/_build/, the library to
jxai_b200/libjxattn.so; a rebuild happens only when a source or the header is
newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import fcntl
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libjxattn.so")
STAMP = os.path.join(BUILD, "libjxattn.sources.sha256")
# Same sources with every device-side index checked (JX_DEVICE_CHECKS=1): a
# diagnostic build, selected at load time with JXAI_B200_CHECKED=1.
LIB_CHECKED = os.path.join(PKG, "libjxattn_checked.so")
STAMP_CHECKED = os.path.join(BUILD, "checked", "libjxattn.sources.sha256")

SOURCES = ["jx_lib.cu", "jx_decode_f32.cu", "jx_decode_bf16.cu", "jx_decode_f16.cu",
           "jx_noalloc.cu", "jx_prefill_tc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (CUDA toolkit required to build libjxattn.so)")


def _deps() -> list[str]:
    files = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC))
    files.append(os.path.join(INCLUDE, "jx_attn.h"))
    files.append(os.path.abspath(__file__))
    return files


def sources_digest() -> str:
    h = hashlib.sha256()
    for f in _deps():
        h.update(os.path.basename(f).encode())
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def up_to_date(checked: bool = False) -> bool:
    """True when the library exists and was built from the current sources."""
    lib, stamp = (LIB_CHECKED, STAMP_CHECKED) if checked else (LIB, STAMP)
    if not os.path.exists(lib) or not os.path.exists(stamp):
        return False
    with open(stamp) as fh:
        return fh.read().strip() == sources_digest()


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False,
          checked: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    lib, stamp = (LIB_CHECKED, STAMP_CHECKED) if checked else (LIB, STAMP)
    objdir = os.path.join(BUILD, "checked") if checked else BUILD
    os.makedirs(objdir, exist_ok=True)
    with open(os.path.join(BUILD, ".lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)  # one builder at a time (e.g. several ranks)
        if not force and up_to_date(checked):
            return lib
        cc = nvcc()
        extra = ["-Xptxas", "-v"] if ptxas_info else []
        if checked:
            extra += ["-DJX_DEVICE_CHECKS=1"]

        def compile_one(src: str) -> str:
            obj = os.path.join(objdir, src.replace(".cu", ".o"))
            cmd = [cc, *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
            if verbose or ptxas_info:
                sys.stderr.write(r.stderr)
            return obj

        digest = sources_digest()
        with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
            objs = list(ex.map(compile_one, SOURCES))
        tmp = f"{lib}.{os.getpid()}.tmp"
        cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, lib)
        with open(stamp, "w") as fh:
            fh.write(digest + "\n")
        return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv,
                checked="--checked" in sys.argv))
