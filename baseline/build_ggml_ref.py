"""Build the reference's own GGUF matvec extension (tinyserve/csrc/ggml_ops.cu,
registered as torch.ops.tinyserve_ggml.ggml_mul_mat_vec) unmodified, for
sm_100a, into baseline/_ref/ggml/ -- the same-box A/B that bench.py times
beside tsb_quant_matvec.  Its source is read from the reference checkout given
as the first argument (it is not part of the installed package).  Output
stays in the git-ignored baseline/_ref/ and travels with the tree to the GPU
box; nothing here is imported by the product.

    python baseline/build_ggml_ref.py <reference checkout>
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "_ref" / "ggml"


def main(ref_root: str) -> Path:
    src = Path(ref_root) / "tinyserve" / "csrc" / "ggml_ops.cu"
    if not src.exists():
        raise SystemExit(f"{src} not found")
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load
    load(name="tinyserve_ggml", sources=[str(src)], build_directory=str(OUT),
         extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"], verbose=False)
    for junk in list(OUT.glob("*.o")) + [OUT / "build.ninja", OUT / ".ninja_log", OUT / ".ninja_deps"]:
        if junk.exists():
            junk.unlink()
    so = sorted(OUT.glob("tinyserve_ggml*.so"))
    print(so[0] if so else "no .so produced")
    return OUT


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
