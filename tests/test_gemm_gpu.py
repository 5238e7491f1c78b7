"""GEMM, batched GEMM and SYRK on the B200 kernels (through the C ABI via the
public API) against the oracle / an fp64 product of the same inputs.

Gates (the path's accuracy targets): relative Frobenius error <= 1e-5 for fp32
(3xTF32), <= 1e-2 for bf16; fp16 is held to 2e-3 (its output rounding).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import trnblas_b200 as tb
from oracle import blas3

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float16: 2e-3}
DEV = "cuda"


def relf(x, ref):
    x, ref = x.double().cpu(), torch.as_tensor(ref).double().cpu()
    return float((x - ref).norm() / max(float(ref.norm()), 1e-300))


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert tb.device_status(0) == 0, "a kernel gave up a bounded wait"


# The last: 81 CTA-pair tiles (at least one per SM pair) and K >= 1024, the
# pair kernel, with ragged edges; the others run on the one-CTA kernel.
SHAPES = [(128, 128, 64), (256, 512, 128), (127, 129, 65), (300, 200, 17), (1, 1, 1), (640, 384, 1000), (1000, 33, 257),
          (130, 520, 96), (1500, 700, 333), (2300, 2100, 1100)]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("ta,tbb", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_matches_fp64(dt, M, N, K, ta, tbb):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(*((K, M) if ta else (M, K)), device=DEV, generator=g).to(dt)
    B = torch.randn(*((N, K) if tbb else (K, N)), device=DEV, generator=g).to(dt)
    C = torch.randn(M, N, device=DEV, generator=g).to(dt)
    out = tb.gemm(0.7, A, B, 0.5, C, transA=ta, transB=tbb)
    assert out.dtype == dt and out.shape == (M, N) and out.device.type == "cuda"
    ref = blas3.gemm(0.7, A.double().cpu().numpy(), B.double().cpu().numpy(), 0.5, C.double().cpu().numpy(), ta, tbb)
    assert relf(out, ref) <= TOL[dt]


def test_gemm_golden_reference_cases():
    g = np.load("tests/golden/gemm.npz")
    for case in ("g0", "g1", "g2", "g3", "g5"):
        M, K, N, ta, tbb, alpha, beta, _ = g[f"{case}_meta"]
        A, B, C = (torch.from_numpy(g[f"{case}_{k}"]).to(DEV) for k in "ABC")
        out = tb.gemm(alpha, A, B, beta, C, transA=bool(ta), transB=bool(tbb))
        assert relf(out, g[f"{case}_R"]) <= 1e-5, case


def test_config1_against_reference_samples():
    """Benchmark case 1 (fp32 1024^3, transA, beta 0.5, seed 0) vs the reference's output."""
    c = np.load("tests/golden/config1.npz")
    gen = torch.Generator().manual_seed(0)
    A, B, C = (2 * torch.rand(1024, 1024, generator=gen) - 1 for _ in range(3))
    out = tb.gemm(1.0, A.to(DEV), B.to(DEV), 0.5, C.to(DEV), transA=True).cpu().numpy()
    idx = c["idx"]
    np.testing.assert_allclose(out[idx[:, 0], idx[:, 1]], c["vals"], rtol=1e-4, atol=1e-5)
    assert abs(np.linalg.norm(out.astype(np.float64)) - float(c["fro"])) / float(c["fro"]) < 1e-6


def test_host_tensors_round_trip():
    """CPU operands are uploaded, computed on the GPU, returned on the host."""
    g = np.load("tests/golden/gemm.npz")
    A, B, C = (torch.from_numpy(g[f"g1_{k}"]) for k in "ABC")
    out = tb.gemm(0.7, A, B, 0.5, C, transA=True)
    assert out.device.type == "cpu"
    assert relf(out, g["g1_R"]) <= 1e-5


def test_fp32_error_flat_in_k():
    """K-chunked promotion: the 3xTF32 error does not grow with K."""
    errs = []
    for K in (256, 4096, 16384):
        A = torch.randn(256, K, device=DEV)
        B = torch.randn(K, 256, device=DEV)
        errs.append(relf(tb.gemm(1.0, A, B), A.double() @ B.double()))
    assert max(errs) <= 2e-6 and errs[-1] <= 2.5 * errs[0]


def test_beta_zero_ignores_nan_c_and_no_alias():
    A = torch.randn(64, 32, device=DEV)
    B = torch.randn(32, 48, device=DEV)
    C = torch.full((64, 48), float("nan"), device=DEV)
    A0, B0 = A.clone(), B.clone()
    out = tb.gemm(1.0, A, B, 0.0, C)
    assert torch.isfinite(out).all()
    assert torch.equal(A, A0) and torch.equal(B, B0)
    assert out.data_ptr() not in (A.data_ptr(), B.data_ptr(), C.data_ptr())


def test_zero_sizes_and_broadcast_c():
    out = tb.gemm(1.0, torch.randn(5, 0, device=DEV), torch.randn(0, 7, device=DEV), 2.0, torch.ones(5, 7, device=DEV))
    assert torch.equal(out, torch.full((5, 7), 2.0, device=DEV))
    assert tb.gemm(1.0, torch.randn(0, 3, device=DEV), torch.randn(3, 4, device=DEV)).shape == (0, 4)
    A, B = torch.randn(10, 20, device=DEV), torch.randn(20, 30, device=DEV)
    row = torch.randn(30, device=DEV)
    out = tb.gemm(2.0, A, B, 0.5, row)
    assert relf(out, 2.0 * A.double() @ B.double() + 0.5 * row.double()) <= 1e-5


def test_mixed_dtypes_raise():
    with pytest.raises(RuntimeError):
        tb.gemm(1.0, torch.randn(4, 4, device=DEV), torch.randn(4, 4, device=DEV, dtype=torch.bfloat16))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_batched_config2(dt):
    """Benchmark case 2a: batch 64 of 512^3 (N(0,1), seed 1), one launch."""
    gen = torch.Generator().manual_seed(1)
    A = torch.randn(64, 512, 512, generator=gen).to(dt)
    B = torch.randn(64, 512, 512, generator=gen).to(dt)
    out = tb.batched_gemm(1.0, A.to(DEV), B.to(DEV))
    assert out.shape == (64, 512, 512) and out.dtype == dt
    assert relf(out, A.double() @ B.double()) <= TOL[dt]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_batched_on_cta_pairs(dt):
    """20 x (512 x 520 x 1100), transposed B, fused C: 20 x 2 x 3 pair tiles
    with K >= 1024 run the CTA-pair kernel with the batch in its tile walk."""
    g = torch.Generator(device=DEV).manual_seed(21)
    A = torch.randn(20, 512, 1100, device=DEV, generator=g).to(dt)
    Bt = torch.randn(20, 520, 1100, device=DEV, generator=g).to(dt)
    C = torch.randn(20, 512, 520, device=DEV, generator=g).to(dt)
    out = tb.batched_gemm(0.5, A, Bt, 2.0, C, transB=True)
    ref = 0.5 * A.double() @ Bt.double().transpose(1, 2) + 2.0 * C.double()
    assert out.dtype == dt and relf(out, ref) <= TOL[dt]


def test_batched_broadcast_trans_and_c():
    g = np.load("tests/golden/gemm.npz")
    A, B, B2, C = (torch.from_numpy(g[f"b0_{k}"]).to(DEV) for k in ("A", "B", "B2", "C"))
    assert relf(tb.batched_gemm(0.9, A, B, 0.4, C), g["b0_R"]) <= 1e-5
    assert relf(tb.batched_gemm(1.0, A, B2), g["b0_R2"]) <= 1e-5
    assert relf(tb.batched_gemm(1.0, A, B.transpose(-2, -1).contiguous(), transB=True), g["b0_R3"]) <= 1e-5
    A4 = torch.randn(2, 3, 40, 24, device=DEV)
    B4 = torch.randn(3, 24, 16, device=DEV)
    assert relf(tb.batched_gemm(1.0, A4, B4), A4.double() @ B4.double()) <= 1e-5


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
# (3000, 1100): 78 lower-triangle 256 x 256 tiles and k >= 1024, the fp32
# CTA-pair kernel plus the mirror pass (upper-stored C keeps the one-CTA kernel)
@pytest.mark.parametrize("n,k", [(128, 64), (300, 200), (1000, 512), (129, 1), (3000, 1100)])
@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
def test_syrk_exactly_symmetric(dt, n, k, trans, uplo):
    A = (torch.randn(k, n, device=DEV) if trans else torch.randn(n, k, device=DEV)).to(dt)
    C0 = torch.randn(n, n, device=DEV).to(dt)
    C = torch.tril(C0) if uplo == "lower" else torch.triu(C0)
    out = tb.syrk(0.9, A, 0.3, C, trans=trans, uplo=uplo)
    assert torch.equal(out, out.T)
    ref = blas3.syrk(0.9, A.double().cpu().numpy(), 0.3, C.double().cpu().numpy(), trans=trans, uplo=uplo)
    assert relf(out, ref) <= TOL[dt]


def test_syrk_golden_reference_cases():
    s = np.load("tests/golden/syrk.npz")
    A, C0, At = (torch.from_numpy(s[k]).to(DEV) for k in ("A", "C0", "At"))
    assert relf(tb.syrk(0.7, A, 0.3, torch.tril(C0), uplo="lower"), s["lower"]) <= 1e-5
    assert relf(tb.syrk(0.7, A, 0.3, torch.triu(C0), uplo="upper"), s["upper"]) <= 1e-5
    assert relf(tb.syrk(0.7, A, 0.3, C0, uplo="lower"), s["both_lower"]) <= 1e-5
    assert relf(tb.syrk(1.0, At, trans=True), s["trans"]) <= 1e-5
    assert relf(tb.syrk(2.0, A), s["noc"]) <= 1e-5
    assert relf(tb.syrk(1.0, A, 0.5, torch.arange(30.0, device=DEV)), s["bcast"]) <= 1e-5
    with pytest.warns(DeprecationWarning):
        r = tb.syrk(0.7, A, 0.3, torch.tril(C0), uplo="upper")  # only the other triangle stored
    assert relf(r, s["lower"]) <= 1e-5


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,k", [(256, 96), (640, 130), (1100, 64), (2176, 200)])
@pytest.mark.parametrize("trans", [False, True])
def test_syrk_without_c_every_tile_walk(dt, n, k, trans):
    """No C: off-diagonal blocks take the vector row stores and the
    transposed mirror stores; 16-bit types walk 128 x 256 tiles over the
    lower triangle's column-block pairs (odd and even tile-row counts, a
    ragged last row block at n = 1100)."""
    A = (torch.randn(k, n, device=DEV) if trans else torch.randn(n, k, device=DEV)).to(dt)
    out = tb.syrk(0.75, A, trans=trans, uplo="lower")
    assert torch.equal(out, out.T)
    a = A.double().T if trans else A.double()
    assert relf(out, 0.75 * a @ a.T) <= TOL[dt]


def test_syrk_config2_lower():
    """Benchmark case 2b: n = k = 4096, uplo lower, A ~ N(0, 1/k), seed 2."""
    gen = torch.Generator().manual_seed(2)
    A = (torch.randn(4096, 4096, generator=gen) / 64.0).to(DEV)
    out = tb.syrk(1.0, A, uplo="lower")
    assert torch.equal(out, out.T)
    ref = A.double() @ A.double().T
    assert relf(out, ref) <= 1e-5


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_host_operands_streamed_match_device_path(dt):
    """Large host operands stream through the GPU in row blocks (uploads,
    GEMMs and downloads overlapped); the result equals the one-shot device
    product bit for bit (same kernel, same per-element K order), with and
    without a fused C."""
    from trnblas_b200 import level3

    g = torch.Generator().manual_seed(11)
    M, K, N = 3000, 2048, 1536  # M not a multiple of the row block
    A = torch.randn(M, K, generator=g).to(dt).pin_memory()
    B = torch.randn(K, N, generator=g).to(dt).pin_memory()
    C = torch.randn(M, N, generator=g).to(dt).pin_memory()
    assert 2.0 * M * N * K >= level3.STREAM_MIN_FLOPS
    old = level3.STREAM_BLOCK_BYTES
    level3.STREAM_BLOCK_BYTES = 1 << 20  # several blocks at this size
    try:
        R = tb.gemm(1.5, A, B)
        R2 = tb.gemm(0.5, A, B, 2.0, C)
    finally:
        level3.STREAM_BLOCK_BYTES = old
    assert R.device.type == "cpu" and R.dtype == dt
    ref = tb.gemm(1.5, A.cuda(), B.cuda()).cpu()
    ref2 = tb.gemm(0.5, A.cuda(), B.cuda(), 2.0, C.cuda()).cpu()
    assert torch.equal(R, ref)
    assert torch.equal(R2, ref2)
