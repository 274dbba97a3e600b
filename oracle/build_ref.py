"""Builds the reference's own CUDA extensions from their sources, for the
parity tests only (TEST INFRASTRUCTURE: nothing in the product loads them).

    python oracle/build_ref.py --reference <path of the reference checkout>

Compiles, where they lie in the reference checkout (read only), the two
extensions its loaders build (src/load_cuda.py:11-20, src/load_gqa_attention.py):

* csrc/denominator.cpp + csrc/denominator_kernel.cu -> ``ref_denominator_cuda``
  (rmsnorm_normalize(_512), rmsnorm_swiglu(_512), ...),
* csrc/gqa_attention.cpp + csrc/gqa_attention_kernel.cu -> ``ref_gqa_attention_cuda``
  (gqa_decode_v2 / gqa_decode_v3),

with the reference's own nvcc flags (-O3 --use_fast_math), for sm_100a
instead of its sm_90, through torch.utils.cpp_extension.  The module names
carry a ``ref_`` prefix so that they can be imported beside this library's
``denominator_cuda``.  Output goes to oracle/_ref/ only (kept out of git, but
shipped with the tree to a GPU machine, where there is no reference checkout
and the tests import the built files).  No reference source is copied.
"""

from __future__ import annotations

import argparse
import glob
import importlib.machinery
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")

EXTENSIONS = {
    "ref_denominator_cuda": ("csrc/denominator.cpp", "csrc/denominator_kernel.cu"),
    "ref_gqa_attention_cuda": ("csrc/gqa_attention.cpp", "csrc/gqa_attention_kernel.cu"),
}
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math"]


def build(reference: str, verbose: bool = False) -> list[str]:
    import torch.utils.cpp_extension as ext

    built = []
    # The toolkit here (12.9) is newer than torch's CUDA (12.8); the reference's
    # own loader skips the same check (src/load_cuda.py:5-7).
    orig = ext._check_cuda_version
    ext._check_cuda_version = lambda *a, **k: None
    try:
        for name, sources in EXTENSIONS.items():
            srcs = [os.path.join(reference, s) for s in sources]
            for s in srcs:
                if not os.path.exists(s):
                    raise FileNotFoundError(s)
            bdir = os.path.join(OUT_DIR, name)
            os.makedirs(bdir, exist_ok=True)
            ext.load(name=name, sources=srcs, extra_cflags=["-O3"],
                     extra_cuda_cflags=NVCC_FLAGS, build_directory=bdir, verbose=verbose)
            built.append(so_path(name))
    finally:
        ext._check_cuda_version = orig
    return built


def so_path(name: str) -> str | None:
    hits = glob.glob(os.path.join(OUT_DIR, name, f"{name}*.so"))
    return hits[0] if hits else None


def load(name: str):
    """Imports a built extension from oracle/_ref (None when it was not built)."""
    path = so_path(name)
    if path is None:
        return None
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    for p in build(args.reference, args.verbose):
        print(p)


if __name__ == "__main__":
    main()
