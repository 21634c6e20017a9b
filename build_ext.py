"""Build the in-tree CUDA extension `modded_nanogpt_b200/_C*.so` for sm_100a.

    python build_ext.py            # incremental
    python build_ext.py --force    # rebuild everything
    python build_ext.py --debug    # also build `_Cdbg*.so` with -DMNG_BOUNDS_CHECK (index checks that record, never trap)

Each .cu file is compiled by nvcc with `-gencode arch=compute_100a,code=sm_100a -lineinfo` (no
PyTorch headers, so this takes seconds and cross-compiles without a GPU); `binding.cpp` is the
only translation unit that includes torch.  Objects are cached under `build/`.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
SRC = ROOT / "modded_nanogpt_b200" / "csrc"
BUILD = ROOT / "build" / "ext"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _digest(paths, extra="") -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(Path(p).read_bytes())
    return h.hexdigest()[:16]


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(map(str, cmd)) + "\n" + r.stdout)
    return r.stdout


def target_path(name: str = "_C") -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return ROOT / "modded_nanogpt_b200" / f"{name}{suffix}"


def build(force: bool = False, verbose: bool = True, debug: bool = False) -> Path:
    """`debug=True` builds the bounds-checked variant `_Cdbg` (same sources, -DMNG_BOUNDS_CHECK) next to `_C`."""
    name = "_Cdbg" if debug else "_C"
    defs = ["-DMNG_BOUNDS_CHECK"] if debug else []
    import torch
    from torch.utils import cpp_extension as ce

    BUILD.mkdir(parents=True, exist_ok=True)
    headers = list(SRC.glob("*.h")) + list(SRC.glob("*.cuh"))
    cu_files = sorted(SRC.glob("*.cu"))
    cpp_files = sorted(SRC.glob("*.cpp"))
    hdr_digest = _digest(headers)
    jobs, objs = [], []
    for f in cu_files:
        tag = _digest([f], hdr_digest + "nvcc" + name)
        o = BUILD / f"{f.stem}.{tag}.o"
        objs.append(o)
        if force or not o.exists():
            jobs.append([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "--use_fast_math", "-Xcompiler", "-fPIC", *defs,
                         "-I", str(SRC), "-c", str(f), "-o", str(o)])
    inc = [a for p in ce.include_paths("cuda") for a in ("-I", p)]
    for f in cpp_files:
        tag = _digest([f], hdr_digest + torch.__version__ + name)
        o = BUILD / f"{f.stem}.{tag}.o"
        objs.append(o)
        if force or not o.exists():
            jobs.append(["g++", "-O2", "-std=c++17", "-fPIC", f"-DTORCH_EXTENSION_NAME={name}", "-DTORCH_API_INCLUDE_EXTENSION_H", *defs,
                         f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}", *inc,
                         "-I", sysconfig.get_paths()["include"], "-I", str(SRC), "-c", str(f), "-o", str(o)])
    if jobs:
        if verbose:
            print(f"[build_ext] compiling {len(jobs)} file(s) for sm_100a", flush=True)
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    out = target_path(name)
    stamp = BUILD / f"link{name}.stamp"
    want = " ".join(o.name for o in objs)
    if force or jobs or not out.exists() or not stamp.exists() or stamp.read_text() != want:
        libdirs = ce.library_paths("cuda")
        link = ["g++", "-shared", "-o", str(out), *map(str, objs)]
        for d in libdirs:
            link += ["-L", d, f"-Wl,-rpath,{d}"]
        link += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-ltorch_python", "-lcudart"]
        _run(link)
        stamp.write_text(want)
        live = {n for st in BUILD.glob("link*.stamp") for n in st.read_text().split()}
        for o in BUILD.glob("*.o"):                          # objects of earlier source versions
            if o.name not in live:
                o.unlink()
        if verbose:
            print(f"[build_ext] linked {out.name}", flush=True)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    if "--debug" in sys.argv:
        build(force="--force" in sys.argv, debug=True)
