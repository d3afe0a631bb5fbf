"""Build recipe for libklab_b200.so (sm_100a) and the standalone prefetch cubin.

Runs nvcc directly (no JIT, no torch extension machinery) and writes everything
in-tree under klab_b200/_lib/, so the built files travel with the repository
snapshot. Objects are rebuilt only when a source or header is newer.

    python -m klab_b200.build            # build (incremental)
    python -m klab_b200.build --clean    # rebuild everything
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT = HERE / "_lib"
OBJ = OUT / "obj"
LIBRARY = OUT / "libklab_b200.so"
ALIAS = OUT / "libkernel_lab.so"  # the reference's library name (native/build/libkernel_lab.so)
PREFETCH_CUBIN = OUT / "prefetch_kernels.cubin"
LAUNCHER = HERE.parent / "bin" / "klab"   # the reference's bin/klab (native/cli.cpp)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler",
                     "-fvisibility=hidden", f"-I{INCLUDE}"]
CUDA_SOURCES = ("capi.cu", "aux_kernels.cu", "prefetch_kernels.cu", "gemv_half.cu", "gemv_cbf16.cu",
                "gemv_int8.cu", "gemv_fp4a.cu", "gemv_fp4b.cu", "noalloc.cu", "peer.cu", "chain_kernel.cu",
                "gemv_lossless.cu", "tc_gemm.cu", "tile_mma.cu", "decode_ops.cu", "decode_attn.cu")
CXX_SOURCES = ("driver_abi.cpp", "codec_host.cpp")
EXPORTS = OUT / "exports.map"


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; klab_b200 builds with the CUDA toolkit's nvcc")


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > mtime for s in sources)


def _run(cmd):
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"command failed ({result.returncode}): {' '.join(map(str, cmd))}\n"
                           f"{result.stdout}\n{result.stderr}")
    return result


def _compile(source: Path, headers, verbose=False) -> Path:
    obj = OBJ / (source.name + ".o")
    if _stale(obj, [source, *headers]):
        if source.suffix == ".cu":
            cmd = [nvcc(), *NVCC_FLAGS, "-c", str(source), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
        else:
            cmd = [nvcc(), "-std=c++17", "-O2", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                   f"-I{INCLUDE}", "-c", str(source), "-o", str(obj)]
        result = _run(cmd)
        if verbose and result.stderr:
            print(result.stderr, file=sys.stderr)
    return obj


def build(clean: bool = False, verbose: bool = False, out_dir: Path | None = None, defines=()) -> Path:
    """Compile every kernel for sm_100a and link libklab_b200.so; return its path.
    out_dir/defines build a variant (e.g. defines=("KLAB_DEPTH=4",)) elsewhere."""
    global OUT, OBJ, LIBRARY, ALIAS, PREFETCH_CUBIN, EXPORTS, NVCC_FLAGS
    if out_dir is not None:
        OUT = Path(out_dir)
        OBJ, LIBRARY, ALIAS = OUT / "obj", OUT / "libklab_b200.so", OUT / "libkernel_lab.so"
        PREFETCH_CUBIN, EXPORTS = OUT / "prefetch_kernels.cubin", OUT / "exports.map"
    NVCC_FLAGS = NVCC_FLAGS + [f"-D{d}" for d in defines]
    if clean and OUT.exists():
        shutil.rmtree(OUT)
    OBJ.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    sources = [CSRC / s for s in CUDA_SOURCES] + [CSRC / s for s in CXX_SOURCES]
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(lambda s: _compile(s, headers, verbose), sources))
    EXPORTS.write_text("{ global: klab_*; lab_*; local: *; };\n")
    if _stale(LIBRARY, objects + [EXPORTS]):
        _run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIBRARY), *map(str, objects),
              "-Xlinker", f"--version-script={EXPORTS}", "-ldl"])
    if _stale(PREFETCH_CUBIN, [CSRC / "prefetch_kernels.cu", *headers]):
        _run([nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", f"-I{INCLUDE}", "-cubin",
              str(CSRC / "prefetch_kernels.cu"), "-o", str(PREFETCH_CUBIN)])
    if ALIAS.is_symlink() or ALIAS.exists():
        ALIAS.unlink()
    ALIAS.symlink_to(LIBRARY.name)
    if out_dir is None:
        build_launcher()
    return LIBRARY


def build_launcher() -> Path:
    """bin/klab from csrc/cli.cpp (g++, no CUDA): execs `python -m klab_b200.cli`."""
    source = CSRC / "cli.cpp"
    if _stale(LAUNCHER, [source]):
        LAUNCHER.parent.mkdir(exist_ok=True)
        cxx = shutil.which(os.environ.get("CXX", "g++")) or "g++"
        tmp = LAUNCHER.with_suffix(".new")
        _run([cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-Werror",
              f'-DKLAB_PROJECT_ROOT="{HERE.parent}"', f'-DKLAB_PYTHON="{sys.executable}"', str(source), "-o",
              str(tmp)])
        tmp.replace(LAUNCHER)
    return LAUNCHER


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--clean", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = parser.parse_args(argv)
    print(build(clean=args.clean, verbose=args.verbose))


if __name__ == "__main__":
    main()
