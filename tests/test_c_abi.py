"""The C ABI from C: tests/c/abi_check.c is compiled with gcc against
include/tgsample.h alone (its static asserts pin the struct layouts) and linked
to libtgsample.so and the CUDA runtime.  On a GPU it samples the committed
fixture (tests/golden/c_abi_case.bin, oracle outputs) through tg_sample and
tg_sample_host and must match bit for bit."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build(tmp_path, cuda_lib):
    exe = str(tmp_path / "abi_check")
    libdir = os.path.join(ROOT, "tinygpt_b200")
    cmd = ["gcc", "-std=c11", "-Wall", "-Werror", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c", "abi_check.c"),
           "-L", libdir, "-ltgsample", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_program_compiles_against_header(tmp_path, cuda_lib):
    assert os.path.exists(build(tmp_path, cuda_lib))


@pytest.mark.gpu
def test_c_program_samples_fixture(tmp_path, cuda_lib):
    exe = build(tmp_path, cuda_lib)
    r = subprocess.run([exe, os.path.join(ROOT, "tests", "golden", "c_abi_case.bin"), "0"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "rows equal" in r.stdout
