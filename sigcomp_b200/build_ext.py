"""Build libsigcomp_b200.so in-tree with nvcc for sm_100a."""

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libsigcomp_b200.so"
SOURCES = ["sc_capi.cu", "sc_codec.cu", "sc_frames.cu", "sc_mlp_simple.cu", "sc_mlp_tc.cu", "sc_signal.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-ccbin", "/usr/bin/g++",
]


# Kernels whose tcgen05.ld results land in registers asynchronously (until tcgen05.wait::ld):
# a register spill placed between a load and its wait would store values not yet written, so the
# build refuses any spill in them.  ptxas -v reports stack and spills per entry function.
NO_SPILL_KERNELS = ("k_fused2", "k_small_decode")
NO_SPILL_SOURCE = "sc_mlp_tc.cu"


def spilling_kernels(ptxas_log, names=NO_SPILL_KERNELS):
    """[(mangled name, spill store bytes, spill load bytes)] of the entry functions in a
    `ptxas -v` log whose name contains one of `names` and that spill."""
    bad, current = [], None
    for line in ptxas_log.splitlines():
        if "Function properties for" in line:
            current = line.split("Function properties for", 1)[1].strip()
        elif current is not None and "spill stores" in line:
            parts = line.replace(",", "").split()
            stores = int(parts[parts.index("spill") - 2])
            loads = int(parts[parts.index("loads") - 3])
            if any(n in current for n in names) and (stores or loads):
                bad.append((current, stores, loads))
            current = None
    return bad


def _stale():
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        [PKG.parent / "include" / "sigcomp_b200.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force=False, verbose=False, jobs=4):
    if not force and not _stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = build_dir / (src + ".o")
        extra = ["-Xptxas", "-v"] if src == NO_SPILL_SOURCE else []
        cmd = [NVCC, *FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(str(obj))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((src, out.decode()))
            continue
        if src == NO_SPILL_SOURCE:
            spills = spilling_kernels(out.decode())
            if spills:
                failed.append((src, "register spills in kernels that must not spill: " + "; ".join(
                    f"{name}: {st} B stored, {ld} B loaded" for name, st, ld in spills)))
                continue
        if verbose and out:
            print(out.decode())
    if failed:
        for src, out in failed:
            sys.stderr.write(f"--- {src}\n{out}\n")
        raise RuntimeError("nvcc failed for " + ", ".join(s for s, _ in failed))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-ccbin", "/usr/bin/g++",
                    *objs, "-o", str(tmp), "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
