"""GPU tier: the tcgen05 GEMM through the C ABI against the oracle.

Tolerances (written here, per the north star):
  * integer pairs: bit-exact;
  * Float32 output: relative Frobenius <= 1e-3 and per-element |Δ| <= 1e-2 against the
    float64 product of the same fp16/bf16 inputs (K <= 8192);
  * Float16 / BFloat16 output: within 1 unit in the last place of the output type of the
    float64 product rounded once (one output ulp at |C| ~ 30-100 exceeds 1e-2, so the
    absolute bound is stated on the Float32-output variant of the same kernel), plus
    relative Frobenius <= 1e-3 against the unrounded float64 product.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import vocab
from oracle.gemm import (gemm_ref, rel_frobenius, max_abs, ulp_distance_f16,
                         ulp_distance_bf16)
from oracle.inputs import gemm_inputs, GEMM_CONFIGS

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
TNAME = {"Float16": "float16", "BFloat16": "bfloat16", "Float32": "float32", "Int8": "int8",
         "UInt8": "uint8", "Int32": "int32", "UInt32": "uint32"}


def _tdt(torch, T):
    return getattr(torch, TNAME[T])


def to_dev(torch, x, T):
    t = torch.from_numpy(np.ascontiguousarray(x))
    if T == "BFloat16":
        t = t.to(torch.bfloat16)       # float32 values that are exact bf16
    return t.cuda()


def run(lvb, torch, A, Bt, ab, out, c_rowmajor=False, lda=None, ldb=None, ldc=None):
    """A (M,K) and Bt (N,K) storage arrays -> C (M,N) as numpy (float32 for bf16 out)."""
    M, K = A.shape
    N = Bt.shape[0]
    dA = to_dev(torch, A, ab)
    dB = to_dev(torch, Bt, ab)
    if lda is not None:     # pad the leading dimension
        big = torch.zeros(M, lda, dtype=dA.dtype, device="cuda")
        big[:, :K] = dA
        dA = big[:, :K]
    if ldb is not None:
        big = torch.zeros(N, ldb, dtype=dB.dtype, device="cuda")
        big[:, :K] = dB
        dB = big[:, :K]
    cdt = _tdt(torch, out) if out != "UInt32" else torch.int32
    if c_rowmajor:
        w = ldc or N
        dC = torch.full((M, w), 7, dtype=cdt, device="cuda")[:, :N]
    else:
        w = ldc or M
        dC = torch.full((N, w), 7, dtype=cdt, device="cuda")[:, :M].t()
    lvb.gemm(dC, dA, dB.t(), c_type=lvb.U32 if out == "UInt32" else None)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    res = dC.cpu()
    if out == "BFloat16":
        return res.float().numpy()
    if out == "UInt32":
        return res.numpy().view(np.uint32)
    return res.numpy()


def out_ulp(x, out):
    """Spacing of the output type at |x| (fp16: np.spacing; bf16: 2^(e-7))."""
    ax = np.abs(np.asarray(x, dtype=np.float64))
    if out == "Float16":
        return np.spacing(np.minimum(ax, 65504).astype(np.float16)).astype(np.float64)
    if out == "BFloat16":
        e = np.floor(np.log2(np.maximum(ax, 2.0 ** -126)))
        return 2.0 ** (e - 7)
    return np.spacing(ax.astype(np.float32)).astype(np.float64)


def check(C, A, B, out):
    ref = gemm_ref(A, B, out)
    if out in ("Int32", "UInt32"):
        assert np.array_equal(C, ref)
        return
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    exact = A64 @ B64
    C64 = np.asarray(C, dtype=np.float64)
    # against the oracle rounded once to the output type (a bf16 output rounded exactly
    # already sits ~1.7e-3 from the exact product, so the exact product is no yardstick there)
    assert rel_frobenius(C64, ref) <= 1e-3
    if out == "Float32":
        assert rel_frobenius(C64, exact) <= 1e-3
        assert max_abs(C64, exact) <= 1e-2
    # per element: one unit of the output type plus the fp32 accumulation bound
    K = A.shape[1]
    acc = 4.0 * np.sqrt(max(K, 1)) * 2.0 ** -24 * (np.abs(A64) @ np.abs(B64))
    err = np.abs(C64 - exact)
    bound = out_ulp(exact, out) + acc
    bad = err > bound
    assert not bad.any(), (f"{int(bad.sum())} elements out of bound; worst excess "
                           f"{float((err - bound).max()):.3e}")


def test_golden_fixtures(lvb, torch_cuda):
    torch = torch_cuda
    files = sorted(f for f in GOLDEN.glob("gemm_*.npz"))
    assert len(files) >= 6
    for f in files:
        z = np.load(f)
        ab, out = str(z["ab"]), str(z["out"])
        A, B, Cg = z["A"], z["B"], z["C"]
        if ab == "BFloat16":
            A, B = vocab.bf16_bits_to_f32(A), vocab.bf16_bits_to_f32(B)
        Bt = np.ascontiguousarray(B.T)
        for crm in (False, True):
            C = run(lvb, torch, A, Bt, ab, out, c_rowmajor=crm)
            if out in ("Int32", "UInt32"):
                assert np.array_equal(C, Cg), f.name
                continue
            if out == "BFloat16":
                Cg = vocab.bf16_bits_to_f32(Cg) if Cg.dtype == np.uint16 else Cg
            # the fixture is the float64 product rounded once; the kernel may differ from it
            # by its fp32 accumulation, bounded in check()
            check(C, A, Bt.T, out)
            assert rel_frobenius(C, Cg) <= 1e-3, f.name


def test_config1_fp16_512_fp32(lvb, torch_cuda):
    cfg = GEMM_CONFIGS["C1"]
    A, Bt = gemm_inputs(cfg["M"], cfg["N"], cfg["K"], cfg["ab"], cfg["seed"])
    C = run(lvb, torch_cuda, A, Bt, "Float16", "Float32")
    check(C, A, Bt.T, "Float32")


@pytest.mark.parametrize("M,N,K", [(1, 1, 8), (127, 129, 72), (300, 520, 200),
                                   (129, 257, 1000), (128, 256, 64), (640, 64, 4096)])
@pytest.mark.parametrize("ab,out", [("Float16", "Float32"), ("Float16", "Float16"),
                                    ("BFloat16", "BFloat16"), ("BFloat16", "Float32"),
                                    ("Float16", "BFloat16")])
def test_ragged_float(lvb, torch_cuda, M, N, K, ab, out):
    A, Bt = gemm_inputs(M, N, K, ab, seed=M * 7 + N * 3 + K)
    for crm in (False, True):
        C = run(lvb, torch_cuda, A, Bt, ab, out, c_rowmajor=crm)
        check(C, A, Bt.T, out)


@pytest.mark.parametrize("M,N,K", [(1, 1, 16), (130, 300, 272), (257, 129, 1040), (512, 512, 8192)])
@pytest.mark.parametrize("ab,out", [("Int8", "Int32"), ("UInt8", "UInt32")])
def test_integer_exact(lvb, torch_cuda, M, N, K, ab, out):
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + N + K)
    for crm in (False, True):
        C = run(lvb, torch_cuda, A, Bt, ab, out, c_rowmajor=crm)
        check(C, A, Bt.T, out)


def test_extreme_int8_values_exact(lvb, torch_cuda):
    # all -128: every product is 16384, K=8192 -> 2^27, exact in int32
    M, N, K = 256, 256, 8192
    A = np.full((M, K), -128, dtype=np.int8)
    Bt = np.full((N, K), -128, dtype=np.int8)
    C = run(lvb, torch_cuda, A, Bt, "Int8", "Int32")
    assert np.all(C == 128 * 128 * K)


def test_leading_dimensions_and_zero_k(lvb, torch_cuda):
    torch = torch_cuda
    A, Bt = gemm_inputs(200, 136, 120, "Float16", seed=9)
    C = run(lvb, torch, A, Bt, "Float16", "Float32", lda=128, ldb=192, ldc=256)
    check(C, A, Bt.T, "Float32")
    C = run(lvb, torch, A, Bt, "Float16", "Float32", c_rowmajor=True, ldc=200)
    check(C, A, Bt.T, "Float32")
    # K = 0: C is the empty sum, zero
    dA = torch.empty(5, 0, dtype=torch.float16, device="cuda")
    dB = torch.empty(0, 7, dtype=torch.float16, device="cuda")
    dC = torch.full((5, 7), 3.0, device="cuda")
    lvb.gemm(dC, dA, dB)
    torch.cuda.synchronize()
    assert torch.all(dC == 0)


def test_unaligned_base_and_odd_strides_repacked(lvb, torch_cuda):
    """Bases and leading dimensions TMA cannot address go through the device repack."""
    torch = torch_cuda
    M, N, K = 96, 80, 70
    A, Bt = gemm_inputs(M, N, K, "Float16", seed=21)
    buf = torch.zeros(M * 75 + 1, dtype=torch.float16, device="cuda")
    dA = buf[1:].view(M, 75)[:, :K]               # 2-byte offset, lda = 75
    dA.copy_(torch.from_numpy(A))
    dB = to_dev(torch, Bt, "Float16")             # ldb = 70 (140 bytes)
    dC = torch.empty(N, M, device="cuda").t()
    lvb.gemm(dC, dA, dB.t())
    torch.cuda.synchronize()
    check(dC.cpu().numpy(), A, Bt.T, "Float32")
    # a pointer not aligned to its element size is an argument error
    raw = torch.zeros(64 * 64 + 8, dtype=torch.uint8, device="cuda")
    with pytest.raises(lvb.LavaError) as e:
        lvb.lib.lvb_gemm  # noqa: B018
        d = lvb.gemm_desc(torch.zeros(64, 64, device="cuda"), torch.zeros(64, 64, dtype=torch.float16, device="cuda"),
                          torch.zeros(64, 64, dtype=torch.float16, device="cuda").t())
        lvb.check(lvb.lib.lvb_gemm(lvb.C.byref(d), raw.data_ptr() + 1, raw.data_ptr() + 1,
                                   torch.zeros(64, 64, device="cuda").data_ptr(), None))
    assert e.value.status == lvb.LVB_ERR_INVALID_ARG


def test_deterministic_and_canary(lvb, torch_cuda):
    torch = torch_cuda
    A, Bt = gemm_inputs(333, 777, 1000, "Float16", seed=4)
    dA, dB = to_dev(torch, A, "Float16"), to_dev(torch, Bt, "Float16")
    # column-major C inside a larger buffer: the rows past M must keep their canary value
    big = torch.full((777, 400), -5.0, device="cuda")
    C = big[:, :333].t()
    lvb.gemm(C, dA, dB.t())
    first = big.clone()
    lvb.gemm(C, dA, dB.t())
    torch.cuda.synchronize()
    assert torch.equal(first, big)
    assert torch.all(big[:, 333:] == -5.0)


def row_checksum_bound(C, out):
    """Bound on |sum_n C[m,n] - sum_n exact[m,n]| per row m, for a C rounded once to `out`
    from an fp32 accumulator. Each element's rounding error is uniform within half an output
    ulp (variance ulp^2/12) and independent of the others, so the row's error has standard
    deviation sqrt(sum_n ulp^2/12); 8 of those, plus 2^-16 of sum_n |C| for the fp32
    accumulation (whose error per element is ~2^-24·sqrt(K)·|C|, under 2^-16·|C| for K <= 2^16).
    A single element off by one part in a thousand of a typical |C| already exceeds it."""
    C64 = np.asarray(C, dtype=np.float64)
    ulp = out_ulp(C64, out) if out != "Float32" else np.zeros_like(C64)
    return 8.0 * np.sqrt((ulp ** 2).sum(axis=1) / 12.0) + 2.0 ** -16 * np.abs(C64).sum(axis=1) + 1e-9


def check_row_checksums(C, A_rows_f64, colsum_f64, out):
    """Every row at once: sum_n C[m,n] against A[m,:]·(sum_n B[:,n]) in float64 (exact for
    fp16/bf16 inputs up to float64 rounding of the row sums)."""
    got = np.asarray(C, dtype=np.float64).sum(axis=1)
    want = A_rows_f64 @ colsum_f64
    bound = row_checksum_bound(C, out)
    bad = np.abs(got - want) > bound
    assert not bad.any(), (f"{int(bad.sum())} row checksums off; worst "
                           f"{float(np.max(np.abs(got - want) - bound)):.3e} over the bound")


def band_rows(M, bands, seed, band=256):
    """First and last row of `bands` randomly chosen `band`-row tile bands, plus rows 0 and
    M-1: the rows at the edges of the kernel's output tiles."""
    starts = np.random.default_rng(seed).choice(M // band, bands, replace=False) * band
    return np.unique(np.concatenate([starts, starts + band - 1, [0, M - 1]]))


@pytest.mark.slow
def test_config2_fp16_8192_sampled_rows_and_row_checksums(lvb, torch_cuda):
    """C2 at full size: 130 sampled rows (both edges of 64 128-row tile bands) checked element by
    element against the float64 oracle, and every row through its checksum."""
    torch = torch_cuda
    cfg = GEMM_CONFIGS["C2"]
    A, Bt = gemm_inputs(cfg["M"], cfg["N"], cfg["K"], cfg["ab"], cfg["seed"])
    C = run(lvb, torch, A, Bt, "Float16", "Float16", c_rowmajor=True)
    rows = band_rows(cfg["M"], 64, seed=0, band=128)
    assert len(rows) >= 128
    check(C[rows], A[rows], Bt.T, "Float16")
    colsum = Bt.astype(np.float64).sum(axis=0)
    check_row_checksums(C, A.astype(np.float64), colsum, "Float16")


@pytest.mark.slow
@pytest.mark.parametrize("out,c_rowmajor", [("BFloat16", True), ("Float32", False)])
def test_config5_bf16_gemm_65536_full(lvb, torch_cuda, out, c_rowmajor):
    """C5's GEMM at its stated size: A 65536x8192 row-major, B 8192x8192 column-major,
    U[-1,1) from PCG64 seed 5 rounded to bf16, on the CTA-pair kernel (row-major C: the
    65536 rows are the kernel's tile rows; column-major C: its tile columns). 130 rows at
    the edges of 64 tile bands are checked element by element against the float64 oracle
    (rounded once to bf16, or exact for the fp32 variant with the north star's |Δ| <= 1e-2),
    every row through its checksum."""
    torch = torch_cuda
    cfg = GEMM_CONFIGS["C5g"]
    M, N, K = cfg["M"], cfg["N"], cfg["K"]
    from oracle.inputs import gemm_inputs_stored
    Abits, Btbits = gemm_inputs_stored(M, N, K, "BFloat16", cfg["seed"])
    plan = lvb.gemm_plan(M, N, K, lvb.BF16, lvb.BF16 if out == "BFloat16" else lvb.F32,
                         c_rowmajor=c_rowmajor)
    assert plan.cta_pair == 1
    dA = torch.from_numpy(Abits.view(np.int16)).cuda().view(torch.bfloat16)
    dB = torch.from_numpy(Btbits.view(np.int16)).cuda().view(torch.bfloat16)
    odt = torch.bfloat16 if out == "BFloat16" else torch.float32
    dC = (torch.empty((M, N), dtype=odt, device="cuda") if c_rowmajor
          else torch.empty((N, M), dtype=odt, device="cuda").t())
    lvb.gemm(dC, dA, dB.t())
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    del dA, dB
    C = dC.float().cpu().numpy()
    del dC
    rows = band_rows(M, 64, seed=5)
    assert len(rows) >= 128
    Bv = vocab.bf16_bits_to_f32(Btbits)           # (N, K) values
    check(C[rows], vocab.bf16_bits_to_f32(Abits[rows]), Bv.T, out)
    colsum = Bv.astype(np.float64).sum(axis=0)
    for r0 in range(0, M, 8192):
        A64 = vocab.bf16_bits_to_f32(Abits[r0:r0 + 8192]).astype(np.float64)
        check_row_checksums(C[r0:r0 + 8192], A64, colsum, out)


@pytest.mark.slow
def test_config3_int8_8192_exact_sampled_rows(lvb, torch_cuda):
    torch = torch_cuda
    cfg = GEMM_CONFIGS["C3"]
    A, Bt = gemm_inputs(cfg["M"], cfg["N"], cfg["K"], cfg["ab"], cfg["seed"])
    C = run(lvb, torch, A, Bt, "Int8", "Int32")
    rows = np.random.default_rng(1).choice(cfg["M"], 96, replace=False)
    rows = np.concatenate([rows, [0, cfg["M"] - 1]])
    # float64 BLAS is exact here: every partial sum is an integer below 2^53
    ref = (A[rows].astype(np.float64) @ Bt.T.astype(np.float64)).astype(np.int64)
    assert np.array_equal(C[rows].astype(np.int64), ref)
    # a checksum of every row: sum_n C[m,n] == A[m,:] · (sum_n B[:,n])
    colsum = Bt.astype(np.int64).sum(axis=0)            # (K,)
    assert np.array_equal(C.astype(np.int64).sum(axis=1), A.astype(np.int64) @ colsum)


@pytest.mark.parametrize("c_rowmajor", [False, True])
def test_small_k_many_tiles_exact(lvb, torch_cuda, c_rowmajor):
    """8192 x 8192 x 32 int8: 1,024 output tiles, ~14 per CTA pair, whose epilogue (the whole
    run time at this K) hands each accumulator back to the MMA warp as soon as it has been
    read. Every element is compared exactly, so an accumulator overwritten before it was
    read would show."""
    torch = torch_cuda
    M = N = 8192
    K = 32
    A, Bt = gemm_inputs(M, N, K, "Int8", seed=31)
    C = run(lvb, torch, A, Bt, "Int8", "Int32", c_rowmajor=c_rowmajor)
    B64 = Bt.T.astype(np.float64)
    for r0 in range(0, M, 1024):     # float64 BLAS is exact: partial sums below 2^53
        ref = (A[r0:r0 + 1024].astype(np.float64) @ B64).astype(np.int64)
        assert np.array_equal(C[r0:r0 + 1024].astype(np.int64), ref), r0


@pytest.mark.parametrize("M,N,K,ab,out", [(2048, 7000, 512, "Int8", "Int32"),
                                          (1000, 5000, 300, "BFloat16", "Float32"),
                                          (1024, 8192, 1024, "Float16", "Float32"),
                                          (2048, 6000, 384, "UInt8", "UInt32")])
def test_pair_tile_224(lvb, torch_cuda, M, N, K, ab, out):
    """CTA pairs with 256×224 tiles (32-bit outputs; the planner takes them when the
    224-wide columns fill the waves better): seven 32-column chunks per drained accumulator, a
    ragged last column tile (7000 = 31·224 + 56), every element checked."""
    t = {"Int8": lvb.I8, "UInt8": lvb.U8, "BFloat16": lvb.BF16, "Float16": lvb.F16}[ab]
    o = {"Int32": lvb.I32, "UInt32": lvb.U32, "Float32": lvb.F32}[out]
    plan = lvb.gemm_plan(M, N, K, t, o, c_rowmajor=True)
    assert plan.cta_pair == 1 and plan.tile_n == 224, (plan.cta_pair, plan.tile_n)
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + N)
    C = run(lvb, torch_cuda, A, Bt, ab, out, c_rowmajor=True)
    check(C, A, Bt.T, out)


@pytest.mark.slow
def test_split_shard_int8_1024_rows_exact(lvb, torch_cuda):
    """One rank's share of C3 row-sharded over 8 GPUs: 1024×8192×8192 int8, 148 tiles of
    256×224 (exactly two waves of 74 CTA pairs), 96 sampled rows exactly and every row's
    exact checksum."""
    plan = lvb.gemm_plan(1024, 8192, 8192, lvb.I8, lvb.I32, c_rowmajor=True)
    assert plan.tile_n == 224 and plan.tiles == 148
    A, Bt = gemm_inputs(1024, 8192, 8192, "Int8", seed=22)
    C = run(lvb, torch_cuda, A, Bt, "Int8", "Int32", c_rowmajor=True)
    rows = np.random.default_rng(2).choice(1024, 96, replace=False)
    ref = (A[rows].astype(np.float64) @ Bt.T.astype(np.float64)).astype(np.int64)
    assert np.array_equal(C[rows].astype(np.int64), ref)
    colsum = Bt.astype(np.int64).sum(axis=0)
    assert np.array_equal(C.astype(np.int64).sum(axis=1), A.astype(np.int64) @ colsum)


@pytest.mark.parametrize("M,N,K,ab,out,c_rowmajor", [(4000, 4000, 256, "Float16", "Float16", True),
                                                     (3000, 5000, 1000, "BFloat16", "BFloat16", False),
                                                     (4000, 4000, 256, "Float16", "BFloat16", True)])
def test_tall_pair_tile(lvb, torch_cuda, M, N, K, ab, out, c_rowmajor):
    """CTA pairs with 512×256 tiles (two 256-row blocks sharing each B stage, one TMEM
    accumulator each, the next tile's first block started while the second drains): ragged
    rows (4000 = 7·512 + 416) and columns, both orientations of the product, every element
    checked."""
    t = {"BFloat16": lvb.BF16, "Float16": lvb.F16}[ab]
    o = {"Float16": lvb.F16, "BFloat16": lvb.BF16}[out]
    plan = lvb.gemm_plan(M, N, K, t, o, c_rowmajor=c_rowmajor)
    assert plan.cta_pair == 1 and plan.tile_m == 512, (plan.tile_m, plan.tile_n)
    A, Bt = gemm_inputs(M, N, K, ab, seed=M + K)
    C = run(lvb, torch_cuda, A, Bt, ab, out, c_rowmajor=c_rowmajor)
    check(C, A, Bt.T, out)


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (1024, 8192, 1024)])
def test_prepared_call_matches_one_shot_call(lvb, torch_cuda, M, N, K):
    """lvb.prepare_gemm (descriptor built once, one foreign call per launch; the one-CTA kernel
    at 512³ and the pair kernel at the larger shape, both launched with programmatic stream
    serialization) gives exactly lvb.gemm's result, call after call, with a dependent kernel
    (torch's add_) between launches on the same stream."""
    torch = torch_cuda
    A, Bt = gemm_inputs(M, N, K, "Float16", 11)
    dA = torch.from_numpy(A).half().cuda()
    dB = torch.from_numpy(np.ascontiguousarray(Bt)).half().cuda().t()   # K x N, column-major
    ref = torch.empty(M, N, dtype=torch.float32, device="cuda")
    lvb.gemm(ref, dA, dB)
    C = torch.full((M, N), 3.0, dtype=torch.float32, device="cuda")
    g = lvb.prepare_gemm(C, dA, dB)
    for _ in range(5):
        g()
        C.add_(1.0)          # reads the GEMM's output: ordered after it on the stream
        g()                  # overwrites C: ordered after the add_
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    assert torch.equal(C, ref)
