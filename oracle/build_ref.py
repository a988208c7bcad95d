"""Build the reference CompactLogic CUDA extensions (the GPU oracle) from their own sources.

Test infrastructure only: the product path never imports anything built here.

The reference ships two torch extensions, ``difflogic_cuda`` (compactlogic/cuda/difflogic.cpp +
difflogic_kernel.cu) and ``convlogic_cuda`` (compactlogic/cuda/convlogic.cpp + convlogic_kernel.cu).
Its setup.py (setup.py:25-50) compiles each pair with nvcc ``-lineinfo`` and nothing else; the target
arch comes from TORCH_CUDA_ARCH_LIST.  This script compiles the same source files, unmodified and
read in place, for sm_100 with the same flags, writing only into ``oracle/_ref/``.  It needs the
reference tree, so it runs in the build container; the resulting ``.so`` files travel to the GPU box.

Usage: python oracle/build_ref.py [--ref /path/to/reference]
"""
import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_root: str) -> None:
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    src = os.path.join(ref_root, "compactlogic", "cuda")
    for name, files in (("difflogic_cuda", ["difflogic.cpp", "difflogic_kernel.cu"]),
                        ("convlogic_cuda", ["convlogic.cpp", "convlogic_kernel.cu"])):
        if os.path.exists(os.path.join(OUT, name + ".so")):
            print(f"[build_ref] {name}.so present, skipping")
            continue
        bdir = os.path.join(OUT, "build_" + name)
        os.makedirs(bdir, exist_ok=True)
        load(name=name, sources=[os.path.join(src, f) for f in files], build_directory=bdir,
             extra_cuda_cflags=["-lineinfo"], with_cuda=True, verbose=False, is_python_module=True)
        shutil.copy2(os.path.join(bdir, name + ".so"), os.path.join(OUT, name + ".so"))
        print(f"[build_ref] built {name}.so")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("COMPACTLOGIC_REF"),
                    help="reference checkout (default: $COMPACTLOGIC_REF)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(os.path.join(args.ref, "compactlogic", "cuda")):
        print("[build_ref] reference tree not present; nothing to build")
        sys.exit(0)
    os.makedirs(OUT, exist_ok=True)
    build(args.ref)
