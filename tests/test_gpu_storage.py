"""om::TensorStorage on the device (include/om_tensor_storage.hpp), the engine storage with a
dtype, a layout tag, a device id and a stream.

tests/cpp/storage_check.cpp is compiled here against the header and libomcuda.so and run: the
reference's byte-buffer contract (host and device buffers, copies in all directions), the
NCHW fp32 <-> NHWC bf16/fp16 round trip (bit-exact on values bf16 and fp16 hold exactly;
copyTo(CPU) always yields NCHW fp32), the device-side contiguous copy of strided views (equal to
the host walk of the same view), and errors for misuse.
"""
import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_tensor_storage_on_device(gpu, tmp_path):
    from omnimatchdeeplearningtool_b200 import _lib
    exe = tmp_path / "storage_check"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "storage_check.cpp"), "-L", libdir,
                    "-lomcuda", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "storage ok" in r.stdout
