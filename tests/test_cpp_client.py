"""The C ABI from C++, as a ggml CUDA-backend bridge would use it: tests/cpp/
abi_client.cpp includes only include/acefa.h and the CUDA runtime, builds the
descriptors of acestep.cpp's batched decode node (views into a KV cache, the
validity mask) and links libacefa.so.  On the CPU it checks descriptor
validation; on a B200 it runs the node and checks the output against a naive
double-precision loop (max-abs 2e-3)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIBDIR = os.path.join(ROOT, "acestep.cpp_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build():
    out_dir = os.path.join(HERE, "cpp", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "abi_client")
    src = os.path.join(HERE, "cpp", "abi_client.cpp")
    lib = os.path.join(LIBDIR, "libacefa.so")
    if not os.path.exists(lib):
        pytest.skip("libacefa.so is not built")
    if shutil.which("g++") is None:
        pytest.skip("no g++")
    cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           src, "-o", exe, "-L", LIBDIR, "-lacefa", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_client_validates_descriptors():
    exe = _build()
    r = subprocess.run([exe, "validate"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "validate ok" in r.stdout


@pytest.mark.gpu
def test_cpp_client_runs_decode_node():
    exe = _build()
    r = subprocess.run([exe, "run"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "run ok" in r.stdout
