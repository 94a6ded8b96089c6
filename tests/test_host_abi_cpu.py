"""The public headers as a C or C++ host sees them (no GPU needed): each header compiles alone as
C11, all of them together in a C++17 host that links libiq4xs_b200.so and exercises the calls that
return before any CUDA work (tests/host_abi_check.cpp)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
INC = ROOT / "include"
CUDA_INC = Path("/usr/local/cuda/include")
HEADERS = ["iq4xs.h", "iq4xs_bench.h", "iq4xs_decoder.h", "iq4xs_peer.h"]

needs_toolchain = pytest.mark.skipif(shutil.which("gcc") is None or shutil.which("g++") is None
                                     or not CUDA_INC.exists(), reason="needs gcc, g++ and the CUDA headers")


@needs_toolchain
@pytest.mark.parametrize("header", HEADERS)
def test_header_compiles_as_c(header, tmp_path):
    src = tmp_path / "use.c"
    src.write_text(f'#include "{header}"\nint main(void) {{ return 0; }}\n')
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", str(INC), "-I", str(CUDA_INC),
                        "-c", str(src), "-o", str(tmp_path / "use.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@needs_toolchain
def test_cpp_host_links_and_validates(pkg, tmp_path):
    lib = Path(pkg.LIB_PATH)
    exe = tmp_path / "host_abi_check"
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I", str(INC), "-I", str(CUDA_INC),
                        str(ROOT / "tests" / "host_abi_check.cpp"), "-o", str(exe), f"-L{lib.parent}",
                        "-l:" + lib.name, f"-Wl,-rpath,{lib.parent}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
