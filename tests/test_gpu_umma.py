"""Self-test of the tcgen05 operand layouts and descriptors used by the
tensor-core chunk path: one MMA per layout combination, against torch."""

import ctypes
import os
import subprocess

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CASES = {0: (64, 64, 128, False, False), 1: (64, 128, 64, False, True),
         2: (128, 32, 64, True, True), 3: (64, 32, 128, False, True),
         4: (128, 128, 64, True, True), 5: (64, 64, 64, False, True),
         # 128-byte swizzled (TMA-written) operands
         6: (64, 64, 128, False, False), 7: (64, 128, 64, False, True),
         8: (128, 32, 64, True, True), 9: (64, 32, 128, False, True),
         10: (128, 128, 64, True, True),
         # stacked M=128 operands, N=256 with spread-out atoms
         11: (128, 64, 128, False, False), 12: (128, 256, 64, False, True),
         13: (128, 32, 128, False, True), 14: (128, 32, 64, False, True),
         15: (128, 128, 128, False, True)}


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    assert torch.cuda.is_available()
    out = tmp_path_factory.mktemp("umma") / "libumma_selftest.so"
    src = os.path.join(ROOT, "tests", "csrc", "umma_selftest.cu")
    inc = os.path.join(ROOT, "domesticated_torch_mlu_ops_b200", "csrc")
    subprocess.run(["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-Xcompiler", "-fPIC", "-shared", "-I", inc, "-o", str(out), src], check=True)
    l = ctypes.CDLL(str(out))
    l.umma_selftest.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 4
    return l


@pytest.mark.parametrize("which", sorted(CASES))
def test_umma_layout(lib, which):
    M, N, K, amn, bmn = CASES[which]
    g = torch.Generator().manual_seed(which)
    A = torch.randn(M, K, generator=g).bfloat16()
    B = torch.randn(N, K, generator=g).bfloat16()
    ref = A.float() @ B.float().T
    a_src = (A.T if amn else A).contiguous().cuda()
    b_src = (B.T if bmn else B).contiguous().cuda()
    D = torch.full((M, N), float("nan"), device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.umma_selftest(which, a_src.data_ptr(), b_src.data_ptr(), D.data_ptr(), st.data_ptr())
    assert rc == 0 and int(st.item()) == 0
    torch.testing.assert_close(D.cpu(), ref, rtol=1e-3, atol=1e-2)
