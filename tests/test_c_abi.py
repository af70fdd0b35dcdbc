"""The C ABI from C: tests/c_abi_demo.c is built with plain gcc against
include/flexkv_b200.h and libflexkv_b200.so (no Python, no torch in the
caller).  Building and linking is checked on the CPU; running it (a KV
round trip through a page-locked pool, block hashes of a token range
checked against the oracle, and a put / match / get through the CPU-tier
cache index, checked by the program itself) needs a GPU."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from flexkv_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_demo(out_dir: str) -> str:
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lib_dir = os.path.dirname(_lib.lib_path())
    exe = os.path.join(out_dir, "c_abi_demo")
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "c_abi_demo.c"), "-o", exe,
           "-L", lib_dir, "-lflexkv_b200", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_header_compiles_as_c_and_links(tmp_path):
    assert os.path.exists(build_demo(str(tmp_path)))


@pytest.mark.gpu
@pytest.mark.parametrize("n_tok,tpb", [(256, 16), (1000, 7)])
def test_c_caller_round_trip_and_hashes(tmp_path, n_tok, tpb):
    from oracle import oracle as O
    exe = build_demo(str(tmp_path))
    r = subprocess.run([exe, str(n_tok), str(tpb)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.array([int(x) for x in r.stdout.split()], dtype=np.uint64)
    want = O.gen_hashes(np.arange(n_tok, dtype=np.int64), tpb)
    assert np.array_equal(got, want)
