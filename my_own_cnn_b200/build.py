"""In-tree build of the b200q CUDA library and of the reference-facing C++ shim.

Everything is compiled for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) and
written next to the sources, so the built files travel with the source tree:

* ``my_own_cnn_b200/libb200q.so``            -- kernels + C ABI (include/b200q.h)
* ``my_own_cnn_b200/libb200q_refshim.so``    -- the reference's own C++ entry points
  (conv_quant_detail::launch_*_qi32_*, bmm_matmul_i32) defined over the C ABI; needs the
  reference headers (src/conv_types.h, src/nnalgebra_quantization.h, bmm.h) at build time
* ``oracle/_ref/quant_conv_test_b200``       -- the reference's unmodified quant_conv_test.cu
  linked against the shim instead of the reference kernels (drop-in proof)
* ``oracle/_ref/conv_bench_b200``            -- the reference's own fp32 conv_bench driver, unmodified,
  linked against the shim (its fp32 launchers come from this library)
* ``oracle/_ref/qconv_bench_b200``           -- shim/qconv_bench.cu, the reference's conv_bench
  driver pattern for the quantized path, with the reference's src/bench.cpp, src/cuda_utils.cpp and
  src/cpu_ref.cpp compiled from their sources

The reference checkout is taken from ``B200Q_REFERENCE`` or, when that is unset, from a
``reference`` directory beside this repository; without one only the library is built.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libb200q.so"
SHIM_LIB = PKG / "libb200q_refshim.so"
REF_TEST_BIN = ROOT / "oracle" / "_ref" / "quant_conv_test_b200"
QCONV_BENCH_BIN = ROOT / "oracle" / "_ref" / "qconv_bench_b200"
CONV_BENCH_BIN = ROOT / "oracle" / "_ref" / "conv_bench_b200"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def reference_root() -> Path:
    """Reference checkout: $B200Q_REFERENCE, else a `reference` directory beside this repository."""
    env = os.environ.get("B200Q_REFERENCE")
    return Path(env) if env else ROOT.parent / "reference"


def build_library(force: bool = False) -> Path:
    deps = sorted(CSRC.glob("*.cu*")) + [ROOT / "include" / "b200q.h"]
    if force or _stale(LIB, deps):
        _run([_nvcc(), *ARCH, *NVCC_FLAGS, "-shared", "-Xlinker", "-soname,libb200q.so",
              "-o", str(LIB), str(CSRC / "b200q.cu")])
    return LIB


def build_reference_shim(ref_root: str | os.PathLike | None = None, force: bool = False) -> bool:
    """Build the shim and the reference's quant_conv_test against it.

    Returns False (and builds nothing) when the reference sources are not present,
    e.g. on a GPU box, where the prebuilt files are used.
    """
    ref = Path(ref_root) if ref_root else reference_root()
    if not (ref / "src" / "conv_types.h").exists():
        return False
    build_library()
    shim_src = PKG / "shim" / "reference_shim.cpp"
    inc = ["-I", str(ref), "-I", str(ref / "src"), "-I", str(ROOT / "include")]
    if force or _stale(SHIM_LIB, [shim_src, LIB]):
        _run([_nvcc(), *ARCH, *NVCC_FLAGS, "-shared", *inc, "-o", str(SHIM_LIB), str(shim_src),
              "-L", str(PKG), "-lb200q", "-Xlinker", "-rpath,$ORIGIN"])
    REF_TEST_BIN.parent.mkdir(parents=True, exist_ok=True)
    if force or _stale(REF_TEST_BIN, [SHIM_LIB]):
        _run([_nvcc(), *ARCH, "-O2", "-std=c++17", *inc, "-o", str(REF_TEST_BIN),
              str(ref / "quant_conv_test.cu"), str(ref / "src" / "cpu_ref.cpp"),
              str(ref / "src" / "cuda_utils.cpp"),
              "-L", str(PKG), "-lb200q_refshim", "-lb200q",
              "-Xlinker", "-rpath,$ORIGIN/../../my_own_cnn_b200"])
    bench_src = PKG / "shim" / "qconv_bench.cu"
    if force or _stale(QCONV_BENCH_BIN, [bench_src, SHIM_LIB]):
        _run([_nvcc(), *ARCH, "-O2", "-std=c++17", *inc, "-o", str(QCONV_BENCH_BIN), str(bench_src),
              str(ref / "src" / "bench.cpp"), str(ref / "src" / "cuda_utils.cpp"),
              str(ref / "src" / "cpu_ref.cpp"),
              "-L", str(PKG), "-lb200q_refshim", "-lb200q",
              "-Xlinker", "-rpath,$ORIGIN/../../my_own_cnn_b200"])
    # The reference's own fp32 conv_bench driver (src/main.cpp, bench.cpp, verify.cpp, cpu_ref.cpp,
    # cudnn_ref.cpp without cuDNN), unmodified, linked against the shim instead of the reference's
    # src/cuda_kernels.cu and bmm.cu.
    if force or _stale(CONV_BENCH_BIN, [SHIM_LIB]):
        srcs = [str(ref / "src" / f) for f in ("main.cpp", "bench.cpp", "verify.cpp", "cpu_ref.cpp", "cudnn_ref.cpp",
                                               "cuda_utils.cpp")]
        _run([_nvcc(), *ARCH, "-O2", "-std=c++17", *inc, "-o", str(CONV_BENCH_BIN), *srcs,
              "-L", str(PKG), "-lb200q_refshim", "-lb200q",
              "-Xlinker", "-rpath,$ORIGIN/../../my_own_cnn_b200"])
    return True


def build_oracle() -> None:
    """CPU oracle (test infrastructure): oracle/liboracle.so and, with the reference present,
    oracle/_ref/libref_oracle.so."""
    ref = reference_root()
    target = "all" if (ref / "src" / "cpu_ref.cpp").exists() else "liboracle.so"
    _run(["make", "-s", "-C", str(ROOT / "oracle"), f"REF={ref}", target])


def build_all() -> None:
    build_library()
    build_oracle()
    build_reference_shim()
