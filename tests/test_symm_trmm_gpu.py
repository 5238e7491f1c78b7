"""symm and trmm on the GEMM kernel against the reference's outputs
(tests/golden/symm_trmm.npz) and the fp64 oracle: relF <= 1e-5 (fp32 as
3xTF32), bf16 <= 1e-2."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import trnblas_b200 as tb
from oracle import blas3

pytestmark = pytest.mark.gpu
D = np.load(Path(__file__).resolve().parent / "golden" / "symm_trmm.npz")


def _t(name, dev="cuda"):
    return torch.from_numpy(D[name]).to(dev)


@pytest.mark.parametrize("uplo", ["upper", "lower"])
def test_symm_matches_reference(uplo):
    L = tb.symm(1.5, _t("A"), _t("B"), 0.5, _t("C"), side="left", uplo=uplo)
    R = tb.symm(-0.75, _t("A"), _t("Br"), 2.0, _t("Cr"), side="right", uplo=uplo)
    assert L.dtype == torch.float32 and L.is_cuda
    assert blas3.relf(L.cpu().numpy(), D[f"symm_left_{uplo}"]) <= 1e-5
    assert blas3.relf(R.cpu().numpy(), D[f"symm_right_{uplo}"]) <= 1e-5
    # only the uplo triangle is read: garbage in the other one changes nothing
    A = _t("A").clone()
    junk = torch.full_like(A, float("nan"))
    A = torch.where(torch.ones_like(A, dtype=torch.bool).triu() if uplo == "upper" else torch.ones_like(A, dtype=torch.bool).tril(), A, junk)
    L2 = tb.symm(1.5, A, _t("B"), 0.5, _t("C"), side="left", uplo=uplo)
    assert torch.equal(L2, L)
    # host operands: result on the host
    Lh = tb.symm(1.5, _t("A", "cpu"), _t("B", "cpu"), 0.5, _t("C", "cpu"), side="left", uplo=uplo)
    assert Lh.device.type == "cpu" and torch.equal(Lh, L.cpu())


@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["upper", "lower"])
@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("diag", ["nonunit", "unit"])
def test_trmm_matches_reference(side, uplo, trans, diag):
    X = _t("B") if side == "left" else _t("Br")
    R = tb.trmm(0.5, _t("A"), X, side=side, uplo=uplo, trans=trans, diag=diag)
    ref = D[f"trmm_{side}_{uplo}_{int(trans)}_{diag}"]
    assert blas3.relf(R.cpu().numpy(), ref) <= 1e-5
    exact = blas3.trmm(0.5, D["A"], X.cpu().numpy(), side, uplo, trans, diag)
    assert blas3.relf(R.cpu().numpy(), exact) <= 1e-5


def test_symm_trmm_bf16_and_large():
    g = torch.Generator(device="cuda").manual_seed(2)
    A = torch.randn(1000, 1000, device="cuda", generator=g)
    B = torch.randn(1000, 777, device="cuda", generator=g)
    for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 1e-2)):
        S = tb.symm(1.0, A.to(dt), B.to(dt), uplo="lower")
        ref = blas3.symm(1.0, A.to(dt).float().cpu().numpy(), B.to(dt).float().cpu().numpy(), uplo="lower")
        assert S.dtype == dt and blas3.relf(S.float().cpu().numpy(), ref) <= tol
        T = tb.trmm(2.0, A.to(dt), B.to(dt), uplo="upper", trans=True)
        ref = blas3.trmm(2.0, A.to(dt).float().cpu().numpy(), B.to(dt).float().cpu().numpy(), "left", "upper", True)
        assert T.dtype == dt and blas3.relf(T.float().cpu().numpy(), ref) <= tol


@pytest.mark.parametrize("dt,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("n,m", [(1300, 520), (2600, 1900)])
def test_trmm_triangle_blocks_every_case(dt, tol, n, m):
    """The GEMM kernel skips the K blocks outside the triangle (triangular
    op(A) on the left, triangular op(B) on the right, lower or upper): every
    case at ragged sizes spanning many K blocks against the fp64 product of
    the masked triangle; 1300 x 520 runs on one-CTA tiles, 2600 x 1900 on
    CTA pairs (88 pair tiles)."""
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(n, n, device="cuda", generator=g).to(dt)
    for side in ("left", "right"):
        X = torch.randn(*((n, m) if side == "left" else (m, n)), device="cuda", generator=g).to(dt)
        for uplo in ("lower", "upper"):
            for trans in (False, True):
                R = tb.trmm(0.5, A, X, side=side, uplo=uplo, trans=trans)
                T = torch.tril(A.double()) if uplo == "lower" else torch.triu(A.double())
                T = T.T if trans else T
                ref = 0.5 * (T @ X.double() if side == "left" else X.double() @ T)
                assert R.dtype == dt
                assert blas3.relf(R.double().cpu().numpy(), ref.cpu().numpy()) <= tol, (side, uplo, trans)


@pytest.mark.parametrize("dt,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("n,m", [(300, 130), (2600, 1900)])
def test_symm_reads_only_the_triangle(dt, tol, n, m):
    """symm runs trnblas_symm: the fp32 split pass (or the 16-bit fill pass)
    reads the symmetric operand from its stored triangle (the other one holds
    NaN here and is never read). Both sides and triangles, a column-major A
    (its stored triangle is the other one of the memory), a strided B and a
    broadcasting C, at a one-CTA size and at a CTA-pair size (2600 x 1900:
    88 pair tiles), against fp64."""
    g = torch.Generator(device="cuda").manual_seed(11)
    S = torch.randn(n, n, device="cuda", generator=g, dtype=torch.float64)
    S = S + S.T
    for side in ("left", "right"):
        X = torch.randn(*((n, m) if side == "left" else (m, n)), device="cuda", generator=g).to(dt)
        ref_core = (S @ X.double()) if side == "left" else (X.double() @ S)
        for uplo in ("lower", "upper"):
            keep = torch.ones(n, n, dtype=torch.bool, device="cuda")
            keep = keep.tril() if uplo == "lower" else keep.triu()
            A = torch.where(keep, S, torch.full_like(S, float("nan"))).to(dt)
            R = tb.symm(0.5, A, X, 2.0, ref_core.to(dt), side=side, uplo=uplo)
            assert R.dtype == dt
            assert blas3.relf(R.double().cpu().numpy(), (2.5 * ref_core).cpu().numpy()) <= tol, (side, uplo)
            # column-major storage of the same logical A
            Acm = A.T.contiguous().T
            R2 = tb.symm(1.0, Acm, X, side=side, uplo=uplo)
            assert blas3.relf(R2.double().cpu().numpy(), ref_core.cpu().numpy()) <= tol, (side, uplo, "cm")
    # strided B (every other column of a wider tensor) and a row-vector C
    Xw = torch.randn(n, 2 * m, device="cuda", generator=g).to(dt)[:, ::2]
    Crow = torch.randn(1, m, device="cuda", generator=g).to(dt)
    S16 = S.to(dt)
    R3 = tb.symm(1.0, S16, Xw, 0.25, Crow, side="left", uplo="lower")
    ref3 = S16.double() @ Xw.double() + 0.25 * Crow.double()
    assert blas3.relf(R3.double().cpu().numpy(), ref3.cpu().numpy()) <= tol
