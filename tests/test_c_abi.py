"""The C ABI from plain C (tests/c/enhance_demo.c): the header compiles as C99
and every entry point the program uses resolves against libgcdr_cuda.so (CPU);
on a B200 the program enhances an image in place through the pooled enhancer
and checks the Enhance contract (GPU)."""
import os
import subprocess

import pytest

import golden_data as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "enhance_demo.c")


def _build(tmp_path):
    from sdcb.gcdrnet_b200 import library_path
    exe = str(tmp_path / "enhance_demo")
    libdir = os.path.dirname(library_path)
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC, "-o", exe,
           "-L", libdir, "-l:" + os.path.basename(library_path), "-Wl,-rpath," + libdir]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_header_compiles_as_c_and_links(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_c_caller_enhances_in_place(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe, G.GC_PATH, G.DR_PATH, "250", "170"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
