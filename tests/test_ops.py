"""The kernel boundary as torch ops (`torch.ops.trnblas.*`, the analogue of
the reference's `trnblas/nki/_native.py` op table): fake implementations give
the output shapes and dtypes without a GPU, the op table applies the
reference's operand dtype check (TypeError), and on a B200 each op passes
`torch.library.opcheck` and matches the public API."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import trnblas_b200 as tb
from trnblas_b200 import ops

T = torch.ops.trnblas


def test_fake_shapes_without_gpu():
    bf = torch.bfloat16
    with FakeTensorMode():
        a = torch.empty(64, 32, device="cuda", dtype=bf)
        b = torch.empty(32, 48, device="cuda", dtype=bf)
        r = T.gemm(a, b, 1.0, 0.0, None, False, False)
        assert r.shape == (64, 48) and r.dtype == bf
        assert T.gemm(a.mT.contiguous(), b, 1.0, 0.0, None, True, False).shape == (64, 48)
        assert T.gemm(a, b.mT.contiguous(), 1.0, 0.0, None, False, True).shape == (64, 48)
        x = T.batched_gemm(torch.empty(3, 64, 32, device="cuda"), torch.empty(1, 32, 16, device="cuda"))
        assert x.shape == (3, 64, 16) and x.dtype == torch.float32
        assert T.syrk(a).shape == (64, 64) and T.syrk(a, trans=True).shape == (32, 32)
        d, e = T.ozaki_split(torch.empty(10, 20, device="cuda", dtype=torch.float64), 8)
        assert d.shape == (8, 10, 20) and d.dtype == torch.int8 and e.shape == (10,) and e.dtype == torch.int32
        g = T.ozaki_gemm(torch.empty(10, 20, device="cuda", dtype=torch.float64),
                         torch.empty(20, 5, device="cuda", dtype=torch.float64), 8)
        assert g.shape == (10, 5) and g.dtype == torch.float64
        E = T.pair_energy(torch.empty(4, 10, 32, device="cuda"), torch.empty(4, device="cuda"),
                          torch.empty(10, device="cuda"), 0, 10)
        assert E.shape == () and E.dtype == torch.float64


def test_op_table_dtype_check():
    assert sorted(ops.OPS) == ["batched_gemm", "gemm", "ozaki_gemm", "ozaki_split", "pair_energy", "syrk"]
    f64 = torch.ones(2, 2, dtype=torch.float64)
    for name in ("gemm", "batched_gemm"):
        with pytest.raises(TypeError, match=f"trnblas::{name}"):
            ops.OPS[name](f64, f64)
    with pytest.raises(TypeError, match="trnblas::syrk"):
        ops.OPS["syrk"](torch.ones(2, 2, dtype=torch.int32))
    with pytest.raises(TypeError, match="trnblas::ozaki_gemm"):
        ops.OPS["ozaki_gemm"](torch.ones(2, 2, dtype=torch.complex64), f64)


def test_schemas_are_functional():
    for name in ops.OPS:
        schema = getattr(T, name).default._schema
        assert not any(a.alias_info is not None and a.alias_info.is_write for a in schema.arguments), name


@pytest.mark.gpu
def test_opcheck_and_parity_on_gpu():
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(3)
    for dt in (torch.float32, torch.bfloat16):
        a = torch.randn(300, 200, device=dev, generator=g).to(dt)
        b = torch.randn(200, 260, device=dev, generator=g).to(dt)
        c = torch.randn(300, 260, device=dev, generator=g).to(dt)
        torch.library.opcheck(T.gemm, (a, b, 0.5, 2.0, c, False, False))
        assert torch.equal(T.gemm(a, b, 0.5, 2.0, c, False, False), tb.gemm(0.5, a, b, 2.0, c))
        assert torch.equal(T.gemm(a.mT.contiguous(), b, 1.0, 0.0, None, True, False),
                           tb.gemm(1.0, a.mT.contiguous(), b, transA=True))
        A3 = torch.randn(4, 64, 96, device=dev, generator=g).to(dt)
        B3 = torch.randn(4, 96, 80, device=dev, generator=g).to(dt)
        torch.library.opcheck(T.batched_gemm, (A3, B3, 1.0, 0.0, None, False, False))
        assert torch.equal(T.batched_gemm(A3, B3), tb.batched_gemm(1.0, A3, B3))
        torch.library.opcheck(T.syrk, (a, 1.0, 0.0, None, True, False))
        assert torch.equal(T.syrk(a), tb.syrk(1.0, a, uplo="lower"))
    x = torch.randn(50, 70, device=dev, dtype=torch.float64, generator=g)
    y = torch.randn(70, 30, device=dev, dtype=torch.float64, generator=g)
    torch.library.opcheck(T.ozaki_split, (x, 8))
    torch.library.opcheck(T.ozaki_gemm, (x, y, 8))
    assert torch.equal(T.ozaki_gemm(x, y, 8), tb.gemm_fp64(x, y))
    from oracle import pair_energy as PE

    B, eo, ev = (t.to(dev) for t in PE.make_inputs(5, 70, 64, 3))
    torch.library.opcheck(T.pair_energy, (B, eo, ev, 0, 15))
    assert float(T.pair_energy(B, eo, ev, 2, 9)) == float(tb.pair_range_energy(B, eo, ev, 2, 9))
    assert tb.device_status(0) == 0
