"""Build step: compiles csrc/*.cu for sm_100a into _build/libqwen3_b200.so, and (where the
reference sources are available) the drop-in engine: the reference's unchanged host code
(src/forward.cu, main.cu, loader.cu, dump.cu and its vendored cJSON) linked against this
library in place of src/kernels.cu.

    python llm-inference_b200/build.py [--dropin REF_DIR] [-v]

Sources are compiled in parallel, one object per .cu, and only when a source or header
changed. Nothing here needs a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = BUILD / "libqwen3_b200.so"
DROPIN = BUILD / "dropin_engine"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = Path(cuda) / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _run(cmd, verbose):
    if verbose:
        print("$ " + " ".join(map(str, cmd)), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(map(str, cmd))}\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout + r.stderr)
    return r


def build(verbose: bool = False, force: bool = False, extra_flags=()) -> Path:
    """Compile the library if any source or header is newer than it."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    hdr_time = _newest(headers)
    nvcc = _nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            _run([nvcc, *NVCC_FLAGS, *extra_flags, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)], verbose)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    if force or not LIB.exists() or LIB.stat().st_mtime < _newest(objs):
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"], verbose)
        os.replace(tmp, LIB)
    return LIB


def build_dropin(ref_dir, verbose: bool = False) -> Path | None:
    """Link the reference's host code, unchanged, against libqwen3_b200.so.

    Compiles src/forward.cu, main.cu, loader.cu and dump.cu and third_party/cjson/cJSON.c where
    they lie in ``ref_dir`` (read-only) into objects under _build/, and links them with this
    library instead of src/kernels.cu. Returns None when ``ref_dir`` has no sources.
    """
    ref = Path(ref_dir)
    host = [ref / "src" / f for f in ("forward.cu", "main.cu", "loader.cu", "dump.cu")]
    cjson = ref / "third_party" / "cjson" / "cJSON.c"
    if not all(p.exists() for p in host + [cjson]):
        return None
    lib = build(verbose)
    obj_dir = BUILD / "dropin_obj"
    obj_dir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src in host:
        obj = obj_dir / (src.stem + ".o")
        if not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime:
            _run([nvcc, *ARCH, "-O3", "-I", str(ref / "src"), "-I", str(cjson.parent), "-c", str(src),
                  "-o", str(obj)], verbose)
        objs.append(obj)
    cobj = obj_dir / "cJSON.o"
    if not cobj.exists():
        _run(["gcc", "-O2", "-c", str(cjson), "-o", str(cobj)], verbose)
    objs.append(cobj)
    if not DROPIN.exists() or DROPIN.stat().st_mtime < max(_newest(objs), lib.stat().st_mtime):
        _run([nvcc, *ARCH, "-o", str(DROPIN), *map(str, objs), "-L", str(BUILD), "-lqwen3_b200",
              "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN"], verbose)
    return DROPIN


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--dropin", metavar="REF_DIR", help="also link the reference host code from REF_DIR")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(args.verbose, args.force))
    if args.dropin:
        print(build_dropin(args.dropin, args.verbose))


if __name__ == "__main__":
    sys.exit(main())
