"""CPU: the shipped package never reaches the test-only checkers -- no module
under seedvr2_ncnn_b200/ imports the oracle, no C/C++/CUDA source includes or
links anything from oracle/ -- and every native source the build compiles
exists."""
import os
import re

from tests.conftest import ROOT

PKG = os.path.join(ROOT, "seedvr2_ncnn_b200")


def _files(root, exts):
    for d, _, fs in os.walk(root):
        if "_build" in d.split(os.sep):
            continue
        for f in fs:
            if f.endswith(exts):
                yield os.path.join(d, f)


def test_package_python_does_not_import_oracle():
    for path in _files(PKG, (".py",)):
        text = open(path).read()
        assert not re.search(r"^\s*(from|import)\s+oracle\b", text, re.M), path


def test_native_sources_do_not_use_oracle():
    for path in _files(PKG, (".cu", ".cuh", ".cpp", ".h")):
        text = open(path).read()
        assert "s2_oracle" not in text and "oracle/" not in text, path


def test_build_sources_exist():
    from seedvr2_ncnn_b200 import build

    for src in build.SOURCES:
        assert os.path.exists(os.path.join(build.CSRC, src)), src
    for src in build.LAYER_SOURCES:
        assert os.path.exists(os.path.join(build.CSRC, "layers", src)), src
