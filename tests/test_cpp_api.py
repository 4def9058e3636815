"""The public C++ API (include/engine/*.h) from a compiled C++ caller.

tests/native/engine_api.cpp is a program written against the headers the way a reference C++
caller is (reference tests/native/smoke.cpp): NeuralEngine construction, step, pack/unpack,
CorticalColumnV2::load/step through make_backend("cuda"), and the refusal of a "cpu" backend.
On CPU it is compiled and linked against libneurogen_native.so (the headers match the library's
exported C++ symbols); on a GPU it runs against the reference's own native CPU library.
"""
import shutil
import subprocess

import pytest

from conftest import ROOT, gpu_available

LIB_DIR = ROOT / 'neurogen-2.5_b200' / 'lib'
REF_LIB = ROOT / 'oracle' / '_ref' / 'libneurogen_ref.so'


def build(tmp_path):
    exe = tmp_path / 'engine_api'
    cmd = ['g++', '-std=c++17', '-O2', '-Wall', '-Werror', f'-I{ROOT / "include"}',
           str(ROOT / 'tests' / 'native' / 'engine_api.cpp'), f'-L{LIB_DIR}', '-lneurogen_native',
           f'-Wl,-rpath,{LIB_DIR}', '-ldl', '-o', str(exe)]
    out = subprocess.run(cmd, capture_output=True, text=True)
    assert out.returncode == 0, out.stderr[-3000:]
    return exe


@pytest.mark.skipif(shutil.which('g++') is None, reason='no C++ compiler')
def test_cpp_caller_compiles_and_links(tmp_path):
    exe = build(tmp_path)
    assert exe.is_file()


@pytest.mark.gpu
def test_cpp_caller_runs_against_the_reference_library(tmp_path):
    assert gpu_available()
    if not REF_LIB.is_file():
        pytest.skip('reference library not built (oracle/_ref)')
    exe = build(tmp_path)
    out = subprocess.run([str(exe), str(REF_LIB)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:] + out.stdout[-2000:]
    assert 'Passed: cuda' in out.stdout
