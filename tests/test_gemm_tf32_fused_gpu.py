"""The fp32 GEMM with the 3xTF32 split fused into the kernel, which
TRNBLAS_B200_TF32_FUSED=1 selects for operands the TMA can read in place of
the split pass (the default, covered by test_gemm_gpu.py), against fp64
products: K-major and MN-major operands (every transpose pair), ragged
edges, a long K, batched calls, SYRK and a triangular (trmm) product, whose
tiles run fewer K blocks than the others. The selection is read once per
process, so the products run in a child process."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import json, torch
import trnblas_b200 as tb
g = torch.Generator(device="cuda").manual_seed(5)
out = []
def relf(x, r):
    return float((x.double() - r).norm() / r.norm())
for (M, N, K) in [(128, 128, 64), (300, 200, 516), (1500, 700, 332), (1024, 1024, 8192)]:
    for ta in (False, True):
        for tbb in (False, True):
            A = torch.randn(*((K, M) if ta else (M, K)), device="cuda", generator=g)
            B = torch.randn(*((N, K) if tbb else (K, N)), device="cuda", generator=g)
            C = torch.randn(M, N, device="cuda", generator=g)
            r = tb.gemm(0.5, A, B, 2.0, C, transA=ta, transB=tbb)
            a = A.double().T if ta else A.double()
            b = B.double().T if tbb else B.double()
            out.append(["gemm %d%d" % (ta, tbb), M, N, K, relf(r, 0.5 * a @ b + 2.0 * C.double())])
gen = torch.Generator().manual_seed(0)
A1, B1, C1 = (2 * torch.rand(1024, 1024, generator=gen) - 1 for _ in range(3))
r = tb.gemm(1.0, A1.cuda(), B1.cuda(), 0.5, C1.cuda(), transA=True)
out.append(["config1", 1024, 1024, 1024, relf(r, (A1.double().T @ B1.double() + 0.5 * C1.double()).cuda())])
A2 = torch.randn(64, 512, 512, device="cuda", generator=g)
B2 = torch.randn(64, 512, 512, device="cuda", generator=g)
out.append(["batched 2a", 512, 512, 512, relf(tb.batched_gemm(1.0, A2, B2), A2.double() @ B2.double())])
A3 = torch.randn(6, 384, 256, device="cuda", generator=g)
B3 = torch.randn(6, 320, 256, device="cuda", generator=g)
r = tb.batched_gemm(1.0, A3, B3, transB=True)
out.append(["batched", 0, 0, 0, relf(r, A3.double() @ B3.double().transpose(1, 2))])
S = torch.randn(700, 900, device="cuda", generator=g)
out.append(["syrk", 700, 700, 900, relf(tb.syrk(1.0, S), S.double() @ S.double().T)])
T = torch.randn(640, 640, device="cuda", generator=g)
X = torch.randn(384, 640, device="cuda", generator=g)
for uplo in ("lower", "upper"):
    for trans in (False, True):
        ref_t = torch.tril(T.double()) if uplo == "lower" else torch.triu(T.double())
        ref = X.double() @ (ref_t.T if trans else ref_t)
        r = tb.trmm(1.0, T, X, side="right", uplo=uplo, trans=trans)
        out.append(["trmm " + uplo + (" T" if trans else ""), 384, 640, 640, relf(r, ref)])
out.append(["status", tb.device_status(0)])
print(json.dumps(out))
"""


def test_fused_split_matches_fp64():
    env = dict(os.environ, TRNBLAS_B200_TF32_FUSED="1", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res[-1] == ["status", 0]
    for name, M, N, K, err in res[:-1]:
        assert err <= 1e-5, (name, M, N, K, err)
