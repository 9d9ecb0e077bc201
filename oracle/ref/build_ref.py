"""TEST INFRASTRUCTURE ONLY: build the reference's own CUDA kernels for sm_100a.

Compiles, from the reference checkout where the sources lie (read-only), into
oracle/_ref/ (git-ignored; it travels to the GPU box with the snapshot):
  * libref_linear.so — kernel/csrc/turing/{convrot_quant,bf16_epilogue,w4a8,
    segmented_rms_adaln}.cu
    with the reference's nvcc flags (kernel/setup.py:398-412, no fast-math) and
    the CUTLASS 2.x headers vendored in site-packages, plus
    oracle/ref/ref_linear_shim.cu (C entry points);
  * ref_sage*.so — kernel/csrc/turing/sage/{fused,qk_preprocess,
    qk_int_sv_f16_cuda_sm75,sol_sparse_cuda_sm75,quant_v_int8_cuda_sm75}.cu
    with the reference's attention flags (adds --use_fast_math,
    kernel/setup.py:483-497), as a torch extension built here with
    torch.utils.cpp_extension (not the reference's own setup.py).
Only tests/golden/make_golden.py and the gpu tests use the results.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE.parent / "_ref"
# The reference checkout: TB_REFERENCE_ROOT, else a `reference` directory
# beside this repository.
REF = Path(os.environ.get("TB_REFERENCE_ROOT", Path(__file__).resolve().parents[3] / "reference"))
CSRC = REF / "kernel" / "csrc"

COMMON = ["-DENABLE_BF16=1", "-std=c++17", "-O3", "--expt-relaxed-constexpr",
          "--expt-extended-lambda", "--ptxas-options=--allow-expensive-optimizations=true",
          "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
          "-U__CUDA_NO_HALF2_OPERATORS__", "-U__CUDA_NO_HALF2_CONVERSIONS__",
          "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
          "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cutlass_include() -> Path:
    import site

    for base in site.getsitepackages():
        p = Path(base) / "flashinfer" / "data" / "cutlass" / "include"
        if (p / "cutlass" / "cutlass.h").exists():
            return p
    raise FileNotFoundError("CUTLASS headers not found in site-packages")


def build_linear() -> Path:
    lib = OUT / "libref_linear.so"
    objdir = OUT / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    cut = cutlass_include()
    srcs = [CSRC / "turing" / "convrot_quant.cu", CSRC / "turing" / "bf16_epilogue.cu",
            CSRC / "turing" / "w4a8.cu", CSRC / "turing" / "segmented_rms_adaln.cu",
            HERE / "ref_linear_shim.cu"]
    procs, objs = [], []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        objs.append(o)
        if o.exists() and o.stat().st_mtime > s.stat().st_mtime:
            continue
        cmd = ["nvcc", *ARCH, *COMMON, "-Xcompiler", "-fPIC", f"-I{CSRC}", f"-I{cut}",
               "-c", str(s), "-o", str(o)]
        procs.append(subprocess.Popen(cmd))
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("reference linear build failed")
    subprocess.check_call(["nvcc", *ARCH, "-shared", "-o", str(lib), *map(str, objs), "-lcudart"])
    return lib


def build_sage() -> None:
    from torch.utils.cpp_extension import load

    bdir = OUT / "sage_build"
    bdir.mkdir(parents=True, exist_ok=True)
    sage = CSRC / "turing" / "sage"
    load(name="ref_sage",
         sources=[str(HERE / "ref_sage_shim.cpp"), str(sage / "fused.cu"),
                  str(sage / "qk_preprocess.cu"), str(sage / "qk_int_sv_f16_cuda_sm75.cu"),
                  str(sage / "sol_sparse_cuda_sm75.cu"), str(sage / "quant_v_int8_cuda_sm75.cu")],
         extra_include_paths=[str(CSRC / "turing"), str(sage)],
         extra_cflags=["-O3", "-DENABLE_BF16=1", "-std=c++17"],
         extra_cuda_cflags=[*ARCH, *COMMON, "--use_fast_math"],
         build_directory=str(bdir), verbose=False)
    for so in bdir.glob("ref_sage*.so"):
        (OUT / so.name).write_bytes(so.read_bytes())


def main() -> int:
    if not CSRC.exists():
        print(f"reference sources not found at {CSRC}; skipping oracle/_ref")
        return 0
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    build_linear()
    build_sage()
    print(f"built reference kernels into {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
