"""Build the flash_attn_b200 CUDA library in-tree for sm_100a.

    python flash-attn-mps_b200/build.py [--jobs N] [--force]

Compiles every ``csrc/*.cu`` with nvcc (``-gencode arch=compute_100a,code=sm_100a``)
into ``flash_attn_b200/_lib/libflash_attn_b200.so``. The CUDA runtime is linked
statically and the CUDA driver API is reached through
``cudaGetDriverEntryPoint``, so the library loads on a host without a GPU
driver (it only fails when a kernel is launched there).

Every object is rebuilt when the content of its source, of any header or of
the compiler flags changes (a hash stamp beside the object, not file times).
The library carries the hash of all its compiled sources and the flags
(``fa_build_id()``, the same value ``source_hash()`` computes from the files
on disk), so a prebuilt library that does not match the checked-out sources
is detected at run time.
"""

import argparse
import concurrent.futures
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "flash_attn_b200", "_lib")
LIB = os.path.join(LIBDIR, "libflash_attn_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-I", os.path.join(ROOT, "include"), "-I", CSRC,
]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    paths = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cuh", ".h"))]
    include = os.path.join(ROOT, "include")
    paths += [os.path.join(include, f) for f in sorted(os.listdir(include)) if f.endswith(".h")]
    return paths


def _digest(paths, flags):
    h = hashlib.sha256()
    # Paths inside the repository enter the hash relative to its root, so a
    # copy of the tree elsewhere hashes the same.
    h.update("\0".join(f.replace(ROOT, "<root>") for f in flags).encode())
    for path in paths:
        h.update(b"\0" + os.path.relpath(path, ROOT).encode() + b"\0")
        with open(path, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def source_hash():
    """Hash of every compiled source, header and the compiler flags (16 hex digits)."""
    paths = [os.path.join(CSRC, f) for f in _sources()] + _headers()
    return _digest(paths, FLAGS)[:16]


def _compile(src, force, extra, build_id):
    obj = os.path.join(BUILD, src[:-3] + ".o")
    path = os.path.join(CSRC, src)
    defines = [f"-DFAB_BUILD_ID=\"{build_id}\""] if src == "build_id.cu" else []
    stamp = _digest([path] + _headers(), FLAGS + defines)
    stamp_path = obj + ".stamp"
    if not force and os.path.exists(obj) and os.path.exists(stamp_path):
        with open(stamp_path) as f:
            if f.read().strip() == stamp:
                return obj, None, False
    cmd = [NVCC, *FLAGS, *defines, *extra, "-c", path, "-o", obj]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{proc.stdout}{proc.stderr}", True
    if extra:
        sys.stdout.write(proc.stdout + proc.stderr)
    with open(stamp_path, "w") as f:
        f.write(stamp + "\n")
    return obj, None, True


def build(jobs=None, force=False, verbose_ptxas=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = _sources()
    build_id = source_hash()
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as pool:
        results = list(pool.map(lambda s: _compile(s, force, extra, build_id), srcs))
    errors = [e for _, e, _ in results if e]
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    objs = [o for o, _, _ in results]
    rebuilt = any(r for _, _, r in results)
    if (force or rebuilt or not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
               *objs, "-o", LIB]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}{proc.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.jobs, args.force, args.ptxas_verbose))
