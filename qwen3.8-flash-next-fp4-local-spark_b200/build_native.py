"""Build libfp4x.so (the sm_100a kernels and their C ABI) in place, next to this file.

    python build_native.py [--jobs N] [--force] [--timeline]

Each csrc/*.cu translation unit is compiled with nvcc for sm_100a only, then linked into one shared library
that has no dependency on torch.  The build is skipped when the library is newer than every source.
`--timeline` builds the diagnostic twin libfp4x_timeline.so instead: the same kernels with the launch-timeline
stamps compiled in (-DFP4X_TIMELINE), which the product library leaves out because they slow every launch.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "libfp4x.so")
BUILD = os.path.join(HERE, "_build")
TIMELINE_OUT = os.path.join(HERE, "libfp4x_timeline.so")
TIMELINE_BUILD = os.path.join(HERE, "_build_timeline")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "-I" + INCLUDE, "-I" + CSRC,
]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date(out=OUT):
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps())


def build(jobs=None, force=False, verbose=False, timeline=False):
    out, bdir = (TIMELINE_OUT, TIMELINE_BUILD) if timeline else (OUT, BUILD)
    flags = NVCC_FLAGS + (["-DFP4X_TIMELINE"] if timeline else [])
    if not force and up_to_date(out):
        return out
    os.makedirs(bdir, exist_ok=True)
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(bdir, os.path.basename(src) + ".o")
        cmd = [cc] + flags + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr))
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
        return obj

    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = out + ".tmp"
    cmd = [cc, "-shared", "-o", tmp] + objs + ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr))
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--timeline", action="store_true", help="build the diagnostic libfp4x_timeline.so")
    a = ap.parse_args()
    print(build(a.jobs, a.force, a.verbose, a.timeline))
