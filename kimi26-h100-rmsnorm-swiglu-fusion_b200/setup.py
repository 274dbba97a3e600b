"""setuptools entry point kept for parity with the reference's setup.py.

``python setup.py build_ext --inplace`` builds the same in-tree artefacts as
build_ext.py (libfrn_b200.so + denominator_cuda); nothing is installed into
site-packages, so the loaded extension is always the one in this tree.
"""
import os
import sys

from setuptools import Command, setup

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


class BuildInTree(Command):
    description = "build libfrn_b200.so (sm_100a) and denominator_cuda in-tree"
    user_options = [("inplace", "i", "ignored: the build is always in-tree")]

    def initialize_options(self):
        self.inplace = 1

    def finalize_options(self):
        pass

    def run(self):
        from src._build import build_all

        build_all(force=True)


setup(name="denominator_cuda", version="0.1.0", cmdclass={"build_ext": BuildInTree})
