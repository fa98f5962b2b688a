"""CPU-only: the C++ om::CUDABackend mirror (include/om_cuda_backend.hpp) compiles against
the C ABI, links against libomcuda.so and throws on a failing status."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_mirror_compiles_links_and_throws(tmp_path):
    from omnimatchdeeplearningtool_b200 import _lib
    exe = tmp_path / "mirror"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "backend_mirror.cpp"), "-L", libdir,
                    "-lomcuda", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "threw -4" in r.stdout


def test_python_mirror_has_every_reference_method():
    """The Python CUDABackend carries the same method names as the C++ mirror's list of the
    reference wrapper's methods (tests/cpp/backend_mirror.cpp)."""
    import re
    from omnimatchdeeplearningtool_b200.backend import CUDABackend
    src = open(os.path.join(ROOT, "tests", "cpp", "backend_mirror.cpp")).read()
    names = re.findall(r"OMB_HAS\((\w+)\)", src.split("reference_methods_exist() {")[1])
    assert len(names) == 71
    missing = [n for n in names if not callable(getattr(CUDABackend, n, None))]
    assert not missing, missing
