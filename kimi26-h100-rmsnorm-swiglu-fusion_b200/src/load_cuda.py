"""Load the ``denominator_cuda`` extension, building it in-tree if needed.

Same entry point as the reference (src/load_cuda.py:1-22): importing this
module yields ``denominator_cuda``.  Here the module is a pybind11 layer over
libfrn_b200.so, whose kernels are compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``).  There is no fallback: a
missing toolchain or a failed build raises at import.
"""
from src._build import load_denominator_cuda

denominator_cuda = load_denominator_cuda()
