"""Build libwamb.so in-tree with nvcc for sm_100a (B200).

Usage: python wam-egale_b200/build.py   (also called by __graft_entry__.build()).
The output lands in wam-egale_b200/lib/ so that it travels with the source
tree; nothing is installed into site-packages.
"""
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
OUT = ROOT / "lib" / "libwamb.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def sources():
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cuh", ".h")) + \
        [ROOT.parent / "include" / "wamb.h"]


def fingerprint():
    """sha256 of the nvcc flags and of every source file's bytes: the build
    is reused only when this matches the one recorded beside the library
    (a binary copied from elsewhere, or built from other sources, never is)."""
    h = hashlib.sha256()
    h.update("\0".join(NVCC_FLAGS).encode())
    for p in sources():
        h.update(p.name.encode() + b"\0" + p.read_bytes() + b"\0")
    return h.hexdigest()


STAMP = OUT.with_suffix(".so.sha256")


def up_to_date():
    if not OUT.exists() or not STAMP.exists():
        return False
    return STAMP.read_text().strip() == fingerprint()


def build(force=False, verbose=False):
    if not force and up_to_date():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "wamb.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, OUT)
    STAMP.write_text(fingerprint() + "\n")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
