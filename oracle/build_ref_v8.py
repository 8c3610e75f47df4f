"""Builds the reference's own CUDA op (v8) for sm_100a, for a GPU side-by-side with the
sm_100a kernels of this repository. Test and benchmark infrastructure only.

The source stays where it lies (``flash_attention_backend/toy_flash_attn/v8/flash_attn_func.cu``
and ``helper.h`` in the reference tree); it is compiled as the reference itself does
(``flash_attention_func.py:226-240``: a torch extension with CuTe headers and
``--extended-lambda``), with the CuTe headers of this image (flashinfer's copy of CUTLASS)
``-gencode arch=compute_100a,code=sm_100a``. The module is written to ``oracle/_ref/``
(not committed; it travels to the GPU box with the working tree).

Usage (where the reference tree is mounted)::

    python oracle/build_ref_v8.py <path of the reference tree>
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
V8 = "flash_attention_backend/toy_flash_attn/v8"
NAME = "toy_ref_v8"
# nvcc 12.9 stops with an internal compiler error on v8/flash_attn_func.cu:367
# ("unsupported float variant": glibc's _Float32 constant M_LOG2Ef32 under GCC >= 13) for
# any target; ref_v8_prelude.h, pre-included, restates that constant as a plain float.
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a", "--pre-include", str(HERE / "ref_v8_prelude.h")]


def cute_include() -> Path:
    import flashinfer  # noqa: F401 - only to locate its CUTLASS headers

    return Path(flashinfer.__file__).resolve().parent / "data" / "cutlass" / "include"


def build(ref_root: str) -> Path:
    from torch.utils.cpp_extension import load

    src = Path(ref_root) / V8
    build_dir = OUT / "build_v8"
    build_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    load(
        name=NAME,
        sources=[str(src / "flash_attn_func.cu")],
        extra_include_paths=[str(src), str(cute_include())],
        extra_cflags=["-O2"],
        extra_cuda_cflags=["-O2", "--extended-lambda"] + GENCODE,
        build_directory=str(build_dir),
        is_python_module=False,
        verbose=False,
    )
    so = build_dir / f"{NAME}.so"
    dst = OUT / f"{NAME}.so"
    shutil.copy2(so, dst)
    shutil.rmtree(build_dir, ignore_errors=True)  # objects only; the module is the copy above
    return dst


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/build_ref_v8.py <path of the reference tree>")
    print(build(sys.argv[1]))
