"""Parity at the benchmark's own sizes (the shapes bench.py times), on the
inputs bench.py draws (device generator, the benchmark seeds):

* config 5a, C = A @ B at M = N = K = 32768 in bf16 and fp32 (3xTF32): a
  sample of whole rows against an fp64 product of those rows, and every
  column through the size-independent checksum 1^T C = (1^T A) B in fp64;
* config 5b, the pair energy at nocc / nvir / naux = 96 / 2208 / 6912: pair
  ranges at the start, middle and end of the i <= j list against the
  reference's chunked energy arithmetic in fp64 on the GPU
  (`oracle.pair_energy.pair_range_energy_torch`), and the reference's
  `multicore.aten_rows` split (occupied rows (0, 2) with every j,
  `oracle.pair_energy.aten_rows_torch`) against the kernel's per-pair energies;
* config 2b in bf16: SYRK n = k = 4096 against fp64.

Gates: relative Frobenius error <= 1e-2 (bf16) / 1e-5 (fp32); pair energy
relative <= 1e-9.
"""

from __future__ import annotations

import pytest
import torch

import trnblas_b200 as tb
from oracle import pair_energy as PE
from trnblas_b200 import energy

pytestmark = pytest.mark.gpu
DEV = "cuda"


def relf(x, ref):
    x, ref = x.double(), ref.double()
    return float((x - ref).norm() / ref.norm())


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    torch.cuda.empty_cache()
    assert tb.device_status(0) == 0


@pytest.mark.parametrize("dt,tol", [(torch.bfloat16, 1e-2), (torch.float32, 1e-5)])
def test_config5a_gemm_32768(dt, tol):
    n = 32768
    g = torch.Generator(device=DEV).manual_seed(5)  # bench.py's config-5a draw at one GPU
    A = (2 * torch.rand(n, n, device=DEV, generator=g) - 1).to(dt)
    B = (2 * torch.rand(n, n, device=DEV, generator=g) - 1).to(dt)
    C = tb.gemm(1.0, A, B)
    assert C.dtype == dt and C.shape == (n, n)
    rows = torch.cat([torch.tensor([0, 1, n - 1]), torch.randperm(n, generator=torch.Generator().manual_seed(5))[:45]])
    rows = rows.to(DEV)
    Bd = B.double()
    ref = A[rows].double() @ Bd
    assert relf(C[rows], ref) <= tol
    # checksum of every column: 1^T C against (1^T A) B, both in fp64
    colsum = C.double().sum(0)
    ref_cs = A.double().sum(0) @ Bd
    assert relf(colsum, ref_cs) <= tol
    del C, Bd, A, B


@pytest.fixture(scope="module")
def cfg5b():
    nocc, nvir, naux = 96, 2208, 6912
    g = torch.Generator(device=DEV).manual_seed(6)  # bench.py's config-5b draw
    B = 0.05 * torch.randn(nocc, nvir, naux, device=DEV, generator=g)
    eo = torch.sort(-20 + 19.7 * torch.rand(nocc, device=DEV, generator=g)).values
    ev = torch.sort(0.1 + 4.9 * torch.rand(nvir, device=DEV, generator=g)).values
    yield B, eo, ev
    del B


@pytest.mark.parametrize("p0,p1", [(0, 120), (2300, 2420), (4560, 4656)])
def test_config5b_pair_ranges_vs_fp64(cfg5b, p0, p1):
    B, eo, ev = cfg5b
    got = float(energy.pair_range_energy(B, eo, ev, p0, p1))
    ref = PE.pair_range_energy_torch(B, eo, ev, p0, p1, dtype=torch.float64)
    assert abs(got - ref) <= 1e-9 * abs(ref), (got, ref)


def test_config5b_aten_rows_vs_kernel(cfg5b):
    """The reference's row split: rows (0, 2) of the chunked energy (every
    ordered pair (i, j) with i in {0, 1}) equal the kernel's pair energies
    e_0j, e_1j summed with the ordered-pair multiplicities."""
    B, eo, ev = cfg5b
    nocc = B.shape[0]
    ref = PE.aten_rows_torch(B, eo, ev, (0, 2), dtype=torch.float64)
    tot = 0.0
    for i in (0, 1):
        for j in range(nocc):
            a, b = min(i, j), max(i, j)
            if i == 1 and j == 0:
                continue  # (1, 0) is pair (0, 1), counted below with weight 2
            p = b * (b + 1) // 2 + a
            w = float(energy.pair_range_energy(B, eo, ev, p, p + 1))  # w_p e_ab
            # ordered pairs with i in {0, 1}: e_00, e_11 once; e_01 and e_10 both; e_0j, e_1j (j >= 2) once
            if a == b:
                tot += w
            elif (a, b) == (0, 1):
                tot += w  # w = 2: e_01 + e_10
            else:
                tot += w / 2.0
    assert abs(tot - ref) <= 1e-9 * abs(ref), (tot, ref)


def test_syrk_config2_bf16():
    """Benchmark case 2b in bf16: n = k = 4096, uplo lower, A ~ N(0, 1/k), seed 2."""
    gen = torch.Generator().manual_seed(2)
    A = (torch.randn(4096, 4096, generator=gen) / 64.0).to(torch.bfloat16).to(DEV)
    out = tb.syrk(1.0, A, uplo="lower")
    assert out.dtype == torch.bfloat16 and torch.equal(out, out.T)
    assert relf(out, A.double() @ A.double().T) <= 1e-2
