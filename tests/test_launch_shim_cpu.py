"""The C++ drop-in header compiles against the reference's own headers and
links against the library (CPU only; skipped where the reference sources are
absent)."""
import os
import subprocess

import pytest

import blog_b200 as Q

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference checkout (its local-llm directory): QL_REFERENCE_SRC, by default a
# checkout of the reference repository next to this one
REF = os.path.join(os.environ.get("QL_REFERENCE_SRC", os.path.join(os.path.dirname(ROOT), "reference", "AI", "codes",
                                                                       "local-llm")), "src")


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference sources not present")
def test_launch_shim_links_with_reference_headers(tmp_path):
    src = tmp_path / "bridge.cpp"
    src.write_text('#include "tensor/TensorCommon.h"\n#include "backend/cuda/common.h"\n'
                   '#define QLINEAR_B200_DEFINE_LAUNCH\n#include "qlinear_b200_launch.hpp"\n'
                   '#include "backend/cuda/ops/kernel.cuh"\n'  # the reference's declarations must agree
                   'cudaStream_t get_current_cuda_stream() { return nullptr; }\n'
                   'int main() { return &launch_quant_gemv == nullptr; }\n')
    if not os.path.exists(Q.LIB_PATH):
        pytest.skip("library not built")
    cmd = ["g++", "-std=c++20", "-I" + REF, "-I" + os.path.join(ROOT, "include"), "-I/usr/local/cuda/include",
           str(src), "-o", str(tmp_path / "bridge"), Q.LIB_PATH, "-L/usr/local/cuda/lib64", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
