"""The one-CTA GEMM kernel, which TRNBLAS_B200_GEMM_PAIR=0 selects for 16-bit
GEMMs in place of the default CTA-pair kernel (tcgen05 cta_group::2, 256 x 256
tiles; covered by test_gemm_gpu.py), against fp64 products: K-major and
MN-major operands, ragged edges, a batched call and a long K with the wave
synchronisation. The selection is read once per process, so the products run
in a child process."""

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
g = torch.Generator(device="cuda").manual_seed(4)
out = []
def relf(x, r):
    return float((x.double() - r).norm() / r.norm())
for dt in (torch.bfloat16, torch.float16):
    for (M, N, K, ta, tbb) in [(256, 512, 128, False, False), (130, 520, 96, True, False),
                               (1500, 700, 333, False, True), (640, 384, 1000, True, True),
                               (2048, 2048, 8192, False, False)]:
        A = torch.randn(*((K, M) if ta else (M, K)), device="cuda", generator=g).to(dt)
        B = torch.randn(*((N, K) if tbb else (K, N)), device="cuda", generator=g).to(dt)
        C = torch.randn(M, N, device="cuda", generator=g).to(dt)
        r = tb.gemm(0.5, A, B, 2.0, C, transA=ta, transB=tbb)
        a = A.double().T if ta else A.double()
        b = B.double().T if tbb else B.double()
        out.append([str(dt), M, N, K, relf(r, 0.5 * a @ b + 2.0 * C.double())])
    A3 = torch.randn(8, 512, 512, device="cuda", generator=g).to(dt)
    B3 = torch.randn(8, 512, 512, device="cuda", generator=g).to(dt)
    out.append([str(dt), "batched", 0, 0, relf(tb.batched_gemm(1.0, A3, B3), A3.double() @ B3.double())])
out.append(["status", tb.device_status(0)])
print(json.dumps(out))
"""


def test_one_cta_kernel_matches_fp64():
    env = dict(os.environ, TRNBLAS_B200_GEMM_PAIR="0", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res[-1] == ["status", 0]
    for dt, M, N, K, err in res[:-1]:
        tol = 1e-2 if "bfloat16" in dt else 2e-3
        assert err <= tol, (dt, M, N, K, err)
