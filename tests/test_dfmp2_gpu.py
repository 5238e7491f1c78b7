"""trsm, metric_inv_half and the end-to-end DF-MP2 energy on one GPU, against
the reference's outputs (tests/golden/dfmp2.npz) and the fp64 oracle.

Bars: trsm / metric factor relF <= 1e-5 (fp32 class: 3xTF32 GEMM updates,
fp32 panel solves); DF-MP2 energy within 1e-5 relative of the reference's
fp64 energy (the whole pipeline is fp32, as the reference's; its own fp32
result is 1e-7 off)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import trnblas_b200 as tb
from oracle import blas3, dfmp2

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD / "dfmp2.npz")


def _ins(d, dev=None):
    t = [torch.from_numpy(d["in_" + k]) for k in ("C_occ", "C_vir", "eri", "J", "eo", "ev")]
    return [x.to(dev) for x in t] if dev else t


@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["upper", "lower"])
@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("diag", ["nonunit", "unit"])
def test_trsm_matches_reference(gold, side, uplo, trans, diag):
    A = torch.from_numpy(gold["trsm_A"]).cuda()
    B = torch.from_numpy(gold["trsm_B"]).cuda()
    Bm = B if side == "left" else B.T.contiguous()
    X = tb.trsm(0.5, A, Bm, side=side, uplo=uplo, trans=trans, diag=diag)
    assert X.dtype == torch.float32 and X.device == A.device
    ref = gold[f"trsm_{side}_{uplo}_{int(trans)}_{diag}"]
    assert blas3.relf(X.cpu().numpy(), ref) <= 1e-5
    exact = dfmp2.trsm(0.5, gold["trsm_A"], Bm.cpu().numpy(), side, uplo, trans, diag)
    assert blas3.relf(X.cpu().numpy(), exact) <= 1e-5


@pytest.mark.parametrize("n,m", [(700, 96), (1031, 17)])
@pytest.mark.parametrize("uplo,trans", [("lower", False), ("upper", True), ("upper", False)])
def test_trsm_blocked_panels(n, m, uplo, trans):
    """n > the 256-row panel: the blocked path with GEMM trailing updates."""
    rng = np.random.default_rng(n + m)
    A = (rng.standard_normal((n, n)) / n + 2.0 * np.eye(n)).astype(np.float32)
    B = rng.standard_normal((n, m)).astype(np.float32)
    X = tb.trsm(1.5, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), uplo=uplo, trans=trans)
    assert blas3.relf(X.cpu().numpy(), dfmp2.trsm(1.5, A, B, "left", uplo, trans)) <= 1e-5
    # host operands: result back on the host
    Xh = tb.trsm(1.5, torch.from_numpy(A), torch.from_numpy(B), uplo=uplo, trans=trans)
    assert Xh.device.type == "cpu" and torch.equal(Xh, X.cpu())


def test_trsm_vector_and_fp64_and_errors():
    rng = np.random.default_rng(3)
    A = (rng.standard_normal((300, 300)) / 300 + 2 * np.eye(300)).astype(np.float32)
    b = rng.standard_normal(300).astype(np.float32)
    x = tb.trsm(1.0, torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda(), uplo="lower")
    assert x.shape == (300,)
    assert blas3.relf(x.cpu().numpy(), dfmp2.trsm(1.0, A, b[:, None], "left", "lower")[:, 0]) <= 1e-5
    Ad = torch.from_numpy(A.astype(np.float64)).cuda()
    xd = tb.trsm(1.0, Ad, torch.from_numpy(b.astype(np.float64)).cuda(), uplo="lower")
    assert xd.dtype == torch.float64
    with pytest.raises(ValueError):
        tb.trsm(1.0, Ad, Ad, side="middle")
    with pytest.raises(ValueError):
        tb.trsm(1.0, Ad[:, :10], Ad)


def test_metric_inv_half(gold):
    J = torch.from_numpy(gold["in_J"])
    X = tb.metric_inv_half(J.cuda())
    assert X.dtype == torch.float32
    assert blas3.relf(X.cpu().numpy(), gold["X32"]) <= 1e-5
    rng = np.random.default_rng(8)
    R = rng.standard_normal((900, 900)) * 0.01
    Jb = (R @ R.T + 900 * np.eye(900)).astype(np.float32)
    Xb = tb.metric_inv_half(torch.from_numpy(Jb))  # host in, host out
    assert Xb.device.type == "cpu"
    assert blas3.relf(Xb.numpy(), dfmp2.metric_inv_half(Jb)) <= 1e-5
    with pytest.raises(NotImplementedError):
        tb.metric_inv_half(torch.ones(3, 3, dtype=torch.int32))


def test_df_mp2_energy_single_gpu(gold):
    from trnblas_b200 import parallel

    ref = float(gold["E64"])
    t = {}
    e_host = parallel.df_mp2_energy(*_ins(gold), timings=t)
    assert abs(e_host - ref) <= 1e-5 * abs(ref)
    assert sorted(t) == sorted(["chol_upload_2a", "rs_iv_bcast_X", "local_2b_3", "ag_B", "energy"])
    e_dev = parallel.df_mp2_energy(*_ins(gold, "cuda"))
    assert e_dev == e_host
    assert tb.device_status(0) == 0


def test_df_mp2_energy_symmetric_packed(gold):
    from trnblas_b200 import parallel

    C_occ, C_vir, eri, J, eo, ev = _ins(gold)
    eri_s = 0.5 * (eri + eri.transpose(0, 1))
    ref = float(gold["E64_sym"])
    e_sym = parallel.df_mp2_energy(C_occ, C_vir, eri_s, J, eo, ev, eri_symmetric=True)
    e_pack = parallel.df_mp2_energy(C_occ, C_vir, parallel.pack_tril(eri_s), J, eo, ev, eri_symmetric=True)
    for e in (e_sym, e_pack):
        assert abs(e - ref) <= 1e-5 * abs(ref)
    with pytest.raises(ValueError):
        parallel.df_mp2_energy(C_occ, C_vir, parallel.pack_tril(eri_s), J, eo, ev)


def test_df_mp2_energy_medium_vs_oracle():
    """A larger case (nocc not a multiple of anything, nvir > 128, naux > one
    K slab) against the fp64 oracle."""
    from trnblas_b200 import parallel

    ins = dfmp2.make_inputs(200, 23, 260, seed=5)
    ref = dfmp2.df_mp2_energy(*ins)
    e = parallel.df_mp2_energy(*[torch.from_numpy(x) for x in ins])
    assert abs(e - ref) <= 1e-5 * abs(ref)
