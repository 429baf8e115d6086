"""GPU check of the node-linear GEMM kernels against a float64 torch product.

Error metric: |C - C_fp64| / (|A| |B|)  (elementwise), which is scale-free; FP32 SIMT
accumulation stays near 1e-7, and the tensor-core kernel (3-term fp16 split with per-row
exponents for A and one exponent per B matrix) must stay within the same 1e-6 bound, also for
rows of very different magnitudes.
"""
import ctypes as ct

import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(1000, 128, 128, 1), (300, 256, 2048, 3), (10000, 512, 512, 1), (130, 2048, 128, 2), (77, 128, 32, 7),
          (5000, 1280, 64, 1), (3000, 512, 64, 2),  # edge-projection shapes (K = 64)
          (200, 384, 96, 9)]  # grouped mode: 18 problems, two launches


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4],
                         ids=["simt", "tcgen05", "tcgen05-grouped", "tcgen05-ksegments", "tcgen05-presplit"])
def test_gemm_matches_fp64(library, shape, mode):
    import torch
    if mode == 3 and shape[2] < 64:
        pytest.skip("K segments need K >= 64")
    if mode == 4 and shape[2] % 64:
        pytest.skip("a split operand needs K a multiple of 64")
    lib = ct.CDLL(str(library))
    lib.mace_debug_gemm.argtypes = [ct.c_int] * 4 + [ct.c_void_p] * 3 + [ct.c_int, ct.c_int]
    lib.mace_last_error.restype = ct.c_char_p
    M, N, K, batch = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(batch, M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    C0 = torch.randn(batch, M, N, device="cuda", generator=g)
    for accumulate in (0, 1):
        C = C0.clone()
        assert lib.mace_debug_gemm(M, N, K, batch, A.data_ptr(), B.data_ptr(), C.data_ptr(), accumulate, mode) == 0, \
            lib.mace_last_error()
        ref = A.double() @ B.double() + (C0.double() if accumulate else 0)
        scale = A.double().abs() @ B.double().abs() + (C0.double().abs() if accumulate else 0)
        err = ((C.double() - ref).abs() / scale).max().item()
        assert err < 1e-6, (shape, mode, accumulate, err)


def test_tensor_core_error_close_to_fp32(library):
    """RMS error of the tensor-core GEMM within 4x that of the FP32 SIMT kernel (K = 2048)."""
    import torch
    lib = ct.CDLL(str(library))
    lib.mace_debug_gemm.argtypes = [ct.c_int] * 4 + [ct.c_void_p] * 3 + [ct.c_int, ct.c_int]
    M, N, K = 2000, 256, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(1, M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
    ref = A.double() @ B.double()
    rms = []
    for mode in (0, 1):
        C = torch.zeros(1, M, N, device="cuda")
        assert lib.mace_debug_gemm(M, N, K, 1, A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, mode) == 0
        rms.append(((C.double() - ref) ** 2).mean().sqrt().item() / ref.abs().mean().item())
    print("relative rms error simt %.3e tcgen05 %.3e" % tuple(rms))
    assert rms[1] <= 4 * rms[0] + 1e-8, rms


@pytest.mark.parametrize("mode", [1, 2, 3, 4], ids=["tcgen05", "tcgen05-grouped", "tcgen05-ksegments", "tcgen05-presplit"])
def test_tensor_core_rows_of_any_magnitude(library, mode):
    """Row magnitudes from 1e-25 to 1e25, every 7th row mixing in values 2^-20 smaller, B of
    magnitude 1e-3: the fp16 split scales each row (and B) into fp16's range, so every row
    keeps the same scale-free error."""
    import torch
    lib = ct.CDLL(str(library))
    lib.mace_debug_gemm.argtypes = [ct.c_int] * 4 + [ct.c_void_p] * 3 + [ct.c_int, ct.c_int]
    lib.mace_last_error.restype = ct.c_char_p
    M, N, K, batch = 640, 256, 192, 2
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(batch, M, K, device="cuda", generator=g, dtype=torch.float64)
    A *= 10.0 ** torch.linspace(-25, 25, M, device="cuda", dtype=torch.float64)[None, :, None]
    A[:, ::7, 1::2] *= 2.0 ** -20
    A = A.float()
    B = (torch.randn(K, N, device="cuda", generator=g) * 1e-3).float()
    C = torch.zeros(batch, M, N, device="cuda")
    assert lib.mace_debug_gemm(M, N, K, batch, A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, mode) == 0, \
        lib.mace_last_error()
    ref = A.double() @ B.double()
    scale = A.double().abs() @ B.double().abs()
    err = ((C.double() - ref).abs() / scale).max().item()
    assert err < 1e-6, err


def test_tensor_core_product_is_unbiased(library):
    """The mean signed relative error of the tensor-core GEMM is at the FP32 SIMT kernel's level
    (|bias| < 2e-8), for one slab (K = 64) and many (K = 1024): the drain compensates the
    tensor pipe's truncation toward zero, which would otherwise shrink every output by about
    one ulp (-8.7e-8) and coherently bias the forces and the virial."""
    import torch
    lib = ct.CDLL(str(library))
    lib.mace_debug_gemm.argtypes = [ct.c_int] * 4 + [ct.c_void_p] * 3 + [ct.c_int, ct.c_int]
    for K in (64, 1024):
        M, N = 16384, 256
        g = torch.Generator(device="cuda").manual_seed(K)
        A = torch.randn(1, M, K, device="cuda", generator=g)
        B = torch.randn(K, N, device="cuda", generator=g) / K ** 0.5
        ref = A.double() @ B.double()
        C = torch.zeros(1, M, N, device="cuda")
        assert lib.mace_debug_gemm(M, N, K, 1, A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, 1) == 0
        bias = ((C.double() - ref) * ref.sign()).mean().item() / ref.abs().mean().item()
        assert abs(bias) < 2e-8, (K, bias)
