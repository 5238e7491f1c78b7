"""Generate the golden fixtures in this folder from the reference trnblas itself.

Run where the reference source is available (it is not on the GPU hosts):

    PYTHONPATH=<path to trnsci/trnblas checkout> python tests/golden/make_golden.py

It imports the reference package (trnsci/trnblas 0.13.0, CPU path: HAS_NKI is
False, so every op is the reference's torch route) and records inputs and
outputs of the hot-path functions:
- trnblas.gemm / batched_gemm / syrk on small seeded fp32 / bf16 inputs;
- config 1 (gemm fp32 1024^3, transA, alpha 1, beta 0.5, seed 0): a
  checksum of the output and 512 sampled entries;
- trnblas.ozaki.split digits and exponents (per row, per column, extreme
  rows), trnblas.ozaki.reference_gemm, trnblas.gemm_fp64;
- the pair energy: _torch_chunked_pair_energy (fp64 and fp32),
  _torch_batched_pair_energy, _pair_sym_reference, multicore.aten_rows row
  ranges, on a small case and on config 3 (48/432/1152, seed 3);
- DF-MP2 end to end (dfmp2.npz): examples/df_mp2.df_mp2_energy in fp32 and
  fp64 on the example's own synthetic inputs, trnblas.parallel.df_mp2_energy
  on one gloo rank (full and packed-symmetric integrals), trnblas.trsm over
  side / uplo / trans / diag, trnblas.metric_inv_half.
- trnblas.symm (side x uplo, with beta and C) and trnblas.trmm (side x uplo
  x trans x diag) on seeded fp32 inputs (symm_trmm.npz).
`--only dfmp2` / `--only symm_trmm` writes just that file.
Inputs that tests can regenerate from a seed are not stored when large.
The torch / numpy versions used are written into meta.json.
"""

from __future__ import annotations

import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _ref():
    import trnblas  # the reference package (PYTHONPATH)
    from trnblas import ozaki
    from trnblas.nki import dispatch, multicore

    if not hasattr(trnblas, "__version__") or "trnblas_b200" in trnblas.__name__:
        raise SystemExit("make_golden.py must import the reference trnblas")
    return trnblas, ozaki, dispatch, multicore


def config1_inputs():
    g = torch.Generator().manual_seed(0)
    n = 1024
    A = 2 * torch.rand(n, n, generator=g) - 1  # stored K x M (transA)
    B = 2 * torch.rand(n, n, generator=g) - 1
    C = 2 * torch.rand(n, n, generator=g) - 1
    return A, B, C


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def gemm_cases(trnblas):
    out = {}
    cases = [
        ("g0", 64, 48, 80, False, False, 1.0, 0.0, torch.float32),
        ("g1", 33, 17, 65, True, False, 0.7, 0.5, torch.float32),
        ("g2", 40, 70, 30, False, True, -1.3, 2.0, torch.float32),
        ("g3", 25, 25, 25, True, True, 1.0, 1.0, torch.float32),
        ("g4", 64, 48, 80, False, False, 0.5, 0.25, torch.bfloat16),
        ("g5", 1, 1, 1, False, False, 1.0, 0.0, torch.float32),
    ]
    for seed, (name, M, K, N, ta, tb, alpha, beta, dt) in enumerate(cases):
        g = torch.Generator().manual_seed(100 + seed)
        A = torch.randn(*(K, M) if ta else (M, K), generator=g).to(dt)
        B = torch.randn(*(N, K) if tb else (K, N), generator=g).to(dt)
        C = torch.randn(M, N, generator=g).to(dt)
        R = trnblas.gemm(alpha, A, B, beta, C, transA=ta, transB=tb)
        for k, v in (("A", A), ("B", B), ("C", C), ("R", R)):
            out[f"{name}_{k}"] = v.float().numpy()
        out[f"{name}_meta"] = np.array([M, K, N, int(ta), int(tb), alpha, beta, dt == torch.bfloat16], dtype=np.float64)
    g = torch.Generator().manual_seed(11)
    A = torch.randn(4, 24, 16, generator=g)
    B = torch.randn(4, 16, 20, generator=g)
    B2 = torch.randn(16, 20, generator=g)
    C = torch.randn(4, 24, 20, generator=g)
    out["b0_A"], out["b0_B"], out["b0_B2"], out["b0_C"] = A.numpy(), B.numpy(), B2.numpy(), C.numpy()
    out["b0_R"] = trnblas.batched_gemm(0.9, A, B, 0.4, C).numpy()
    out["b0_R2"] = trnblas.batched_gemm(1.0, A, B2).numpy()
    out["b0_R3"] = trnblas.batched_gemm(1.0, A, B.transpose(-2, -1).contiguous(), transB=True).numpy()
    return out


def syrk_cases(trnblas):
    out = {}
    g = torch.Generator().manual_seed(21)
    A = torch.randn(30, 20, generator=g)
    C0 = torch.randn(30, 30, generator=g)
    At = torch.randn(20, 30, generator=g)
    out["A"], out["C0"], out["At"] = A.numpy(), C0.numpy(), At.numpy()
    out["lower"] = trnblas.syrk(0.7, A, 0.3, torch.tril(C0), uplo="lower").numpy()
    out["upper"] = trnblas.syrk(0.7, A, 0.3, torch.triu(C0), uplo="upper").numpy()
    out["both_lower"] = trnblas.syrk(0.7, A, 0.3, C0, uplo="lower").numpy()
    out["trans"] = trnblas.syrk(1.0, At, trans=True).numpy()
    out["noc"] = trnblas.syrk(2.0, A).numpy()
    out["bcast"] = trnblas.syrk(1.0, A, 0.5, torch.arange(30.0)).numpy()
    return out


def ozaki_cases(trnblas, ozaki):
    out = {}
    torch.manual_seed(0)
    X = torch.randn(20, 37, dtype=torch.float64) * torch.logspace(-5, 5, 37, dtype=torch.float64)
    out["X"] = X.numpy()
    for per in ("row", "col"):
        for k in (1, 3, 8, 12):
            d, e = ozaki.split(X, k, per=per, pad=(1, 1))
            out[f"split_{per}_{k}_d"] = d.to(torch.float64).numpy().astype(np.int8)
            out[f"split_{per}_{k}_e"] = e
    Xe = torch.zeros(4, 300, dtype=torch.float64)
    Xe[0] = torch.linspace(-1e300, 1e300, 300, dtype=torch.float64)
    Xe[1] = torch.linspace(-1e-300, 1e-300, 300, dtype=torch.float64)
    Xe[2, 5] = 5e-324
    out["Xe"] = Xe.numpy()
    d, e = ozaki.split(Xe, 8, per="row", pad=(1, 1))
    out["split_extreme_d"] = d.to(torch.float64).numpy().astype(np.int8)
    out["split_extreme_e"] = e
    rng = np.random.default_rng(4)
    for name, (M, K, N) in {"r0": (37, 300, 29), "r1": (64, 130, 48), "r2": (5, 4100, 7)}.items():
        A = rng.standard_normal((M, K)) * np.exp2(rng.integers(-10, 11, (M, K)))
        B = rng.standard_normal((K, N)) * np.exp2(rng.integers(-10, 11, (K, N)))
        out[f"{name}_A"], out[f"{name}_B"] = A, B
        for k in (4, 8):
            out[f"{name}_ref{k}"] = ozaki.reference_gemm(torch.from_numpy(A), torch.from_numpy(B), k).numpy()
        out[f"{name}_host"] = trnblas.gemm_fp64(torch.from_numpy(A), torch.from_numpy(B)).numpy()
    # the reference's k = 1 exactness known answer (tests/test_ozaki.py:197-203 pattern)
    rng = np.random.default_rng(3)
    A = rng.integers(-63, 64, (40, 500)).astype(np.float64) * 2.0**-6
    B = rng.integers(-63, 64, (500, 30)).astype(np.float64)
    A[:, 0] = 63 * 2.0**-6
    B[0] = 63
    out["k1_A"], out["k1_B"] = A, B
    out["k1_ref"] = ozaki.reference_gemm(torch.from_numpy(A), torch.from_numpy(B), 1).numpy()
    out["consts"] = np.array([ozaki.n_products(8), ozaki.exponent_offset(8), ozaki.SLICE_BITS,
                              ozaki.TILE_K, ozaki.GROUP_TERMS])
    return out


def energy_inputs(nocc, nvir, naux, seed):
    g = torch.Generator().manual_seed(seed)
    B = (0.05 * torch.randn(nocc * nvir, naux, generator=g)).reshape(nocc, nvir, naux)
    eo = torch.sort(-20.0 + 19.7 * torch.rand(nocc, generator=g)).values
    ev = torch.sort(0.1 + 4.9 * torch.rand(nvir, generator=g)).values
    return B, eo, ev


def energy_cases(dispatch, multicore, full: bool):
    out = {}
    B, eo, ev = energy_inputs(6, 20, 32, 3)
    out["small_B"], out["small_eo"], out["small_ev"] = B.numpy(), eo.numpy(), ev.numpy()
    out["small_chunked64"] = np.array(float(dispatch._torch_chunked_pair_energy(B.double(), eo.double(), ev.double())))
    out["small_chunked32"] = np.array(float(dispatch._torch_chunked_pair_energy(B, eo, ev)))
    out["small_batched64"] = np.array(float(dispatch._torch_batched_pair_energy(B.double(), eo.double(), ev.double())))
    out["small_sym"] = np.array(float(dispatch._pair_sym_reference(B, eo, ev)))
    cpu = torch.device("cpu")
    for r0, r1 in ((0, 2), (2, 6), (3, 4)):
        out[f"small_rows_{r0}_{r1}"] = np.array(float(multicore.aten_rows(B.double(), eo.double(), ev.double(), (r0, r1), cpu)))
    out["small_occ_chunks_6_4"] = np.array(multicore.occ_chunks(6, 4))
    B2, eo2, ev2 = energy_inputs(5, 37, 45, 7)
    out["odd_B"], out["odd_eo"], out["odd_ev"] = B2.numpy(), eo2.numpy(), ev2.numpy()
    out["odd_chunked64"] = np.array(float(dispatch._torch_chunked_pair_energy(B2.double(), eo2.double(), ev2.double())))
    B4, eo4, ev4 = energy_inputs(7, 300, 200, 9)  # several 128 / 64 blocks, ragged
    out["mid_sha_B"] = np.array(sha(B4))
    out["mid_chunked64"] = np.array(float(dispatch._torch_chunked_pair_energy(B4.double(), eo4.double(), ev4.double())))
    if full:
        B3, eo3, ev3 = energy_inputs(48, 432, 1152, 3)
        out["cfg3_sha_B"] = np.array(sha(B3))
        t0 = time.time()
        out["cfg3_E64"] = np.array(float(dispatch._torch_chunked_pair_energy(B3.double(), eo3.double(), ev3.double())))
        t1 = time.time()
        out["cfg3_E32"] = np.array(float(dispatch._torch_chunked_pair_energy(B3, eo3, ev3)))
        t2 = time.time()
        out["cfg3_seconds"] = np.array([t1 - t0, t2 - t1])
    return out


def dfmp2_cases(trnblas):
    """DF-MP2 pipeline and trsm outputs of the reference (CPU, torch route)."""
    import os

    import torch.distributed as dist

    import examples.df_mp2 as ex  # the reference's example driver (PYTHONPATH)
    from trnblas import parallel as rpar

    out = {}
    nbasis, nocc, naux, seed = 40, 6, 48, 11
    C_occ, C_vir, eri, J, eo, ev = ex._make_inputs(nbasis, nocc, naux, seed=seed)
    for k, v in dict(C_occ=C_occ, C_vir=C_vir, eri=eri, J=J, eo=eo, ev=ev).items():
        out["in_" + k] = v.numpy()
    out["E32"] = np.array(ex.df_mp2_energy(C_occ, C_vir, eri, J, eo, ev))
    out["E64"] = np.array(ex.df_mp2_energy(*(x.double() for x in (C_occ, C_vir, eri, J, eo, ev))))
    eri_s = 0.5 * (eri + eri.transpose(0, 1))
    out["E64_sym"] = np.array(ex.df_mp2_energy(*(x.double() for x in (C_occ, C_vir, eri_s, J, eo, ev))))
    out["X32"] = trnblas.metric_inv_half(J).numpy()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        out["E32_par"] = np.array(rpar.df_mp2_energy(C_occ, C_vir, eri, J, eo, ev))
        packed = rpar.pack_tril(eri_s)
        out["E32_par_sym"] = np.array(rpar.df_mp2_energy(C_occ, C_vir, packed, J, eo, ev, eri_symmetric=True))
        out["packed_sha"] = np.array(sha(packed))
    finally:
        dist.destroy_process_group()
    g = torch.Generator().manual_seed(21)
    n, m = 200, 24
    # off-diagonal entries small enough that unit-diagonal solves stay
    # well conditioned too
    A = torch.randn(n, n, generator=g) / n + 2.0 * torch.eye(n)
    B = torch.randn(n, m, generator=g)
    out["trsm_A"], out["trsm_B"] = A.numpy(), B.numpy()
    for side in ("left", "right"):
        Bm = B if side == "left" else B.T.contiguous()
        for uplo in ("upper", "lower"):
            for trans in (False, True):
                for diag in ("nonunit", "unit"):
                    X = trnblas.trsm(0.5, A, Bm, side=side, uplo=uplo, trans=trans, diag=diag)
                    out[f"trsm_{side}_{uplo}_{int(trans)}_{diag}"] = X.numpy()
    return out


def symm_trmm_cases(trnblas):
    """symm and trmm of the reference on seeded fp32 inputs (CPU torch route)."""
    out = {}
    g = torch.Generator().manual_seed(31)
    n, m = 96, 80
    A = torch.randn(n, n, generator=g)
    B = torch.randn(n, m, generator=g)
    Br = torch.randn(m, n, generator=g)
    C = torch.randn(n, m, generator=g)
    Cr = torch.randn(m, n, generator=g)
    out.update(A=A.numpy(), B=B.numpy(), Br=Br.numpy(), C=C.numpy(), Cr=Cr.numpy())
    for uplo in ("upper", "lower"):
        out[f"symm_left_{uplo}"] = trnblas.symm(1.5, A, B, 0.5, C, side="left", uplo=uplo).numpy()
        out[f"symm_right_{uplo}"] = trnblas.symm(-0.75, A, Br, 2.0, Cr, side="right", uplo=uplo).numpy()
        for side in ("left", "right"):
            X = B if side == "left" else Br
            for trans in (False, True):
                for diag in ("nonunit", "unit"):
                    out[f"trmm_{side}_{uplo}_{int(trans)}_{diag}"] = trnblas.trmm(
                        0.5, A, X, side=side, uplo=uplo, trans=trans, diag=diag).numpy()
    return out


def main():
    trnblas, ozaki, dispatch, multicore = _ref()
    only = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
    if only == "dfmp2":
        np.savez_compressed(HERE / "dfmp2.npz", **dfmp2_cases(trnblas))
        print("dfmp2.npz written")
        return
    if only == "symm_trmm":
        np.savez_compressed(HERE / "symm_trmm.npz", **symm_trmm_cases(trnblas))
        print("symm_trmm.npz written")
        return
    full = "--quick" not in sys.argv
    meta = {
        "reference": "trnsci/trnblas " + trnblas.__version__,
        "torch": torch.__version__,
        "numpy": np.__version__,
        "threads": torch.get_num_threads(),
    }
    np.savez_compressed(HERE / "gemm.npz", **gemm_cases(trnblas))
    np.savez_compressed(HERE / "syrk.npz", **syrk_cases(trnblas))
    np.savez_compressed(HERE / "ozaki.npz", **ozaki_cases(trnblas, ozaki))
    A, B, C = config1_inputs()
    R = trnblas.gemm(1.0, A, B, 0.5, C, transA=True, transB=False)
    rng = np.random.default_rng(123)
    idx = rng.integers(0, 1024, (512, 2))
    np.savez_compressed(
        HERE / "config1.npz",
        sha_inputs=np.array(sha(torch.cat([A, B, C]))),
        sha_out=np.array(sha(R)),
        fro=np.array(float(R.double().norm())),
        idx=idx,
        vals=R.numpy()[idx[:, 0], idx[:, 1]],
    )
    np.savez_compressed(HERE / "energy.npz", **energy_cases(dispatch, multicore, full))
    (HERE / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("golden fixtures written:", meta)


if __name__ == "__main__":
    main()
