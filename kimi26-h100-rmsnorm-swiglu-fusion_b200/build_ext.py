"""Build the native parts in-tree (same entry point as the reference's
build_ext.py): libfrn_b200.so for sm_100a and the ``denominator_cuda`` module.

    python build_ext.py
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from src._build import LIB_PATH, build_all, load_denominator_cuda  # noqa: E402

if __name__ == "__main__":
    build_all(force=True, verbose="-v" in sys.argv)
    module = load_denominator_cuda()
    print("Build successful!")
    print(f"Library: {LIB_PATH}")
    print(f"Module: {module}")
    print(f"Functions: {[n for n in dir(module) if not n.startswith('_')]}")
