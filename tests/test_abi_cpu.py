"""CPU tier: the C ABI library loads, exports every symbol include/lvb.h declares, and
answers the host-only questions (caps, shapes, bestshape, argument validation, planning)
without a GPU — the reference's GPU-free test style (test/runtests.jl:1-20)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "lvb.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lvb_[a-z0-9_]+)\s*\(", text)))


def test_exports_every_declared_symbol(lvb):
    syms = declared_symbols()
    assert len(syms) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", str(lvb.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (lvb_\w+)", out))
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    assert sorted(lvb.EXPORTS) == syms          # the Python binding covers the header
    for s in syms:
        assert hasattr(lvb.lib, s)


def test_struct_layouts_match_header(lvb, tmp_path):
    """The ctypes mirrors (and so the Julia structs written field for field like them) have
    the C structs' sizes and field offsets, compiled from include/lvb.h by the host gcc."""
    structs = {"lvb_matrix_shape": lvb.lvb_matrix_shape, "lvb_device_caps": lvb.lvb_device_caps,
               "lvb_gemm_desc": lvb.lvb_gemm_desc, "lvb_gemm_plan": lvb.lvb_gemm_plan,
               "lvb_attn_desc": lvb.lvb_attn_desc, "lvb_epilogue": lvb.lvb_epilogue,
               "lvb_attn_plan": lvb.lvb_attn_plan, "lvb_comm_id": lvb.lvb_comm_id}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "lvb.h"', "int main(void){"]
    for name, cls in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{name}.{f} %zu\\n", offsetof({name}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True,
                                                         text=True, check=True).stdout.split("\n") if l)
    for name, cls in structs.items():
        assert int(out[name]) == C.sizeof(cls), name
        for f, _ in cls._fields_:
            assert int(out[f"{name}.{f}"]) == getattr(cls, f).offset, f"{name}.{f}"


def test_library_needs_no_libcuda_at_load(lvb):
    out = subprocess.run(["ldd", str(lvb.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out
    assert lvb.abi_version() == 5


def test_static_caps_answer(lvb):
    c = lvb.caps()   # static sm_100a table, no GPU
    assert c.coopmat and c.tile == 16 and c.subgroup == 32 and c.coopmatsubgroup == 32
    assert c.cores == 148 and c.sharedbudget == 227 * 1024 and c.workgrouplimit == 1024
    assert lvb.wggranularity(c, 128) == (128, 16, 16)
    assert lvb.wggranularity(c, 64) is None
    # `tile` is one entry of `shapes` (caps.jl:84-96)
    assert lvb.MatrixShape(lvb.F16, lvb.F32, 16, 16, 16) in c.shapes


def test_bestshape_squarest_then_largest(lvb):
    c = lvb.caps()
    s = lvb.bestshape(c, lvb.F16, lvb.F32)
    assert (s.M, s.N, s.K) == (16, 16, 16)
    s = lvb.bestshape(c, lvb.I8, lvb.I32)
    assert (s.M, s.N, s.K) == (16, 16, 32)
    assert lvb.bestshape(c, lvb.F32, lvb.F32) is None        # Lava returns `nothing`
    # The library's own answer agrees, and the workgroup-scope table gives tcgen05 tiles.
    assert lvb.bestshape_native(lvb.F16, lvb.F32) == lvb.bestshape(c, lvb.F16, lvb.F32)
    w = lvb.bestshape_native(lvb.BF16, lvb.F32, lvb.WORKGROUP_SCOPE)
    assert (w.M, w.K) == (128, 16) and w.N in (64, 128, 256)
    # coopmat=false empties the table but keeps the record (caps.jl:98-108,158-159)
    import dataclasses
    off = dataclasses.replace(c, coopmat=False)
    assert lvb.matrix_shapes(off) == [] and off.shapes
    assert not lvb.supports(off, lvb.MatrixShape(lvb.F16, lvb.F32, 16, 16, 16))


def _desc(lvb, **kw):
    d = lvb.lvb_gemm_desc(lvb.F16, lvb.F16, lvb.F32, 1, 0, 0, 256, 256, 256, 256, 256, 256)
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,status,needle", [
    (dict(M=-1), 1, "negative"),
    (dict(c_type=5), 2, "no kernel for Float16 x Float16 -> Int32"),
    (dict(a_type=3, b_type=3, c_type=2), 2, "no kernel"),
    (dict(a_type=0, b_type=1), 2, "no kernel"),
    (dict(a_rowmajor=0, lda=255), 1, "lda < M"),
    (dict(b_rowmajor=1, ldb=100), 1, "ldb < N"),
    (dict(lda=100), 1, "lda < K"),
    (dict(ldb=255), 1, "ldb < K"),
    (dict(ldc=10), 1, "ldc < M"),
    (dict(c_rowmajor=1, ldc=10), 1, "ldc < N"),
    (dict(M=2 ** 31), 2, "2^31"),
])
def test_gemm_validation(lvb, kw, status, needle):
    d = _desc(lvb, **kw)
    st = lvb.lib.lvb_gemm_check(C.byref(d))
    assert st == status
    msg = lvb.lib.lvb_last_error().decode()
    assert needle in msg and msg.startswith("lvb_gemm: ")


def test_gemm_null_pointers_rejected_before_device(lvb):
    d = _desc(lvb)
    st = lvb.lib.lvb_gemm(C.byref(d), None, None, None, None)
    assert st == lvb.LVB_ERR_INVALID_ARG
    with pytest.raises(lvb.LavaError) as e:
        lvb.check(st)
    assert e.value.operation == "lvb_gemm" and "NULL" in e.value.message
    # empty problems are a no-op even without a device
    d = _desc(lvb, M=0)
    assert lvb.lib.lvb_gemm(C.byref(d), None, None, None, None) == 0


def test_gemm_without_device_fails_loudly(lvb):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    d = _desc(lvb)
    st = lvb.lib.lvb_gemm(C.byref(d), 256, 256, 256, None)
    assert st == lvb.LVB_ERR_NO_DEVICE
    assert "no CUDA device" in lvb.lib.lvb_last_error().decode()


def test_plans(lvb):
    p = lvb.gemm_plan(8192, 8192, 8192, lvb.F16, lvb.F16)
    # large problems: 512x256 tiles on CTA pairs (cta_group::2: two 256x256 MMA chains, one
    # per 256-row block), 74 pairs on 148 SMs
    assert p.cta_pair == 1
    assert (p.tile_m, p.tile_n, p.tile_k, p.instr_m, p.instr_k) == (512, 256, 64, 256, 16)
    # column-major C that can take TMA stores: computed as Cᵀ = BᵀAᵀ so the kernel's
    # n is C's contiguous dimension (each thread's columns are one contiguous run)
    assert p.tiles == 16 * 32 and p.ctas == 148 and p.swap_ab == 1
    assert p.tmem_cols == 512 and p.smem_bytes <= 232448 and p.stages == 4
    # fewer row blocks than pairs can fill in whole waves: 256x256 tiles on the pairs
    sq = lvb.gemm_plan(4096, 8192, 8192, lvb.F16, lvb.F16, c_rowmajor=True)
    assert (sq.tile_m, sq.tile_n, sq.stages) == (256, 256, 6)
    q = lvb.gemm_plan(8192, 8192, 8192, lvb.I8, lvb.I32)
    assert q.tile_k == 128 and q.instr_k == 32
    # a problem with fewer 256x256 tiles than SM pairs uses 1-CTA tiles
    s = lvb.gemm_plan(1024, 1024, 8192, lvb.F16, lvb.F32)
    assert s.cta_pair == 0 and s.tiles > 16
    r = lvb.gemm_plan(512, 512, 512, lvb.F16, lvb.F32)
    assert r.tile_n == 64 and r.tiles == 32          # latency-bound size: more CTAs
    s = lvb.gemm_plan(1000, 300, 64, lvb.F16, lvb.F32, c_rowmajor=True)
    assert s.swap_ab == 0 and s.repack_a == 0 and s.repack_b == 0
    # a C leading dimension TMA cannot store to (N = 301 fp16 = 602 bytes): the other
    # orientation, so direct stores of one column by a warp are contiguous
    u = lvb.gemm_plan(1000, 301, 64, lvb.F16, lvb.F16, c_rowmajor=True)
    assert u.swap_ab == 1
    # a leading dimension TMA cannot address (K=70 fp16 = 140 bytes) is repacked, not refused
    t = lvb.gemm_plan(64, 64, 70, lvb.F16, lvb.F32)
    assert t.repack_a == 1 and t.repack_b == 1
    assert lvb.gemm_plan(64, 64, 72, lvb.I8, lvb.I32).repack_a == 1    # 72 bytes
    assert lvb.gemm_plan(64, 64, 80, lvb.I8, lvb.I32).repack_a == 0    # 80 = 5·16 bytes


def test_plans_transposed_operands(lvb):
    """MN-contiguous operands (Lava's transposing view): 16-bit ones are read MN-major in
    place, 8-bit ones are copied K-major first."""
    p = lvb.gemm_plan(4096, 4096, 4096, lvb.F16, lvb.F16, a_rowmajor=False, b_rowmajor=True)
    assert (p.a_mnmajor, p.b_mnmajor, p.repack_a, p.repack_b) == (1, 1, 0, 0)
    p = lvb.gemm_plan(4096, 4096, 4096, lvb.BF16, lvb.F32, b_rowmajor=True)
    assert (p.a_mnmajor, p.b_mnmajor, p.repack_a, p.repack_b) == (0, 1, 0, 0)
    q = lvb.gemm_plan(4096, 4096, 4096, lvb.I8, lvb.I32, a_rowmajor=False)
    assert (q.a_mnmajor, q.repack_a, q.b_mnmajor, q.repack_b) == (0, 1, 0, 0)
    # an MN-major leading dimension TMA cannot address (M=100 fp16 = 200 bytes) is copied
    r = lvb.gemm_plan(100, 64, 64, lvb.F16, lvb.F32, a_rowmajor=False)
    assert (r.a_mnmajor, r.repack_a) == (0, 1)


def _epi(lvb, **kw):
    e = lvb.lvb_epilogue()
    for k, v in kw.items():
        setattr(e, k, v)
    return e


@pytest.mark.parametrize("dkw,ekw,status,needle", [
    (dict(), dict(activation=7), 1, "unknown activation"),
    (dict(a_type=3, b_type=3, c_type=5), dict(activation=1), 2, "integer output"),
    (dict(), dict(bias=256, bias_type=5), 2, "bias type"),
    (dict(), dict(bias=256, bias_type=2, bias_axis=2), 1, "bias_axis"),
    (dict(), dict(bias=258, bias_type=2), 1, "bias not aligned"),
    (dict(), dict(residual=256, residual_type=3, ldr=256), 2, "residual type"),
    (dict(), dict(residual=256, residual_type=0, ldr=100), 1, "ldr < M"),
    (dict(c_rowmajor=1), dict(residual=256, residual_type=0, ldr=100), 1, "ldr < N"),
    (dict(), dict(residual=257, residual_type=0, ldr=256), 1, "residual not aligned"),
])
def test_gemm_epilogue_validation(lvb, dkw, ekw, status, needle):
    d = _desc(lvb, **dkw)
    e = _epi(lvb, **ekw)
    assert lvb.lib.lvb_gemm_ex_check(C.byref(d), C.byref(e)) == status
    msg = lvb.lib.lvb_last_error().decode()
    assert needle in msg and msg.startswith("lvb_gemm_ex: ")
    # a valid epilogue passes; NULL is plain lvb_gemm
    ok = _epi(lvb, bias=256, bias_type=lvb.F16, residual=512, residual_type=lvb.BF16, ldr=256,
              activation=lvb.ACT_GELU_ERF)
    assert lvb.lib.lvb_gemm_ex_check(C.byref(_desc(lvb)), C.byref(ok)) == 0
    assert lvb.lib.lvb_gemm_ex_check(C.byref(_desc(lvb)), None) == 0



def test_layout_from_strides(lvb):
    import torch
    A = torch.empty(64, 32, dtype=torch.float16)          # row-major (M,K)
    Bt = torch.empty(48, 32, dtype=torch.float16)         # storage of column-major B
    Ccol = torch.empty(48, 64, dtype=torch.float32).t()   # column-major (M,N)
    d = lvb.gemm_desc(Ccol, A, Bt.t())
    assert (d.a_rowmajor, d.lda, d.b_rowmajor, d.ldb, d.c_rowmajor, d.ldc) == (1, 32, 0, 32, 0, 64)
    Crow = torch.empty(64, 48, dtype=torch.float32)
    d = lvb.gemm_desc(Crow, A, Bt.t())
    assert (d.c_rowmajor, d.ldc) == (1, 48)
    with pytest.raises(lvb.LavaError):
        lvb.gemm_desc(Crow, A, torch.empty(33, 48, dtype=torch.float16))


def test_attention_validation(lvb):
    d = lvb.lvb_attn_desc()
    d.dtype, d.causal = lvb.F16, 1
    d.batch, d.heads_q, d.heads_kv, d.seq_q, d.seq_kv, d.head_dim = 2, 8, 2, 128, 128, 128
    d.scale = 0.088
    assert lvb.lib.lvb_attention_check(C.byref(d)) == 0
    d.heads_kv = 3
    assert lvb.lib.lvb_attention_check(C.byref(d)) == lvb.LVB_ERR_INVALID_ARG
    d.heads_kv = 2
    d.head_dim = 96
    assert lvb.lib.lvb_attention_check(C.byref(d)) == lvb.LVB_ERR_UNSUPPORTED
    d.head_dim = 128
    d.dtype = lvb.F32
    assert lvb.lib.lvb_attention_check(C.byref(d)) == lvb.LVB_ERR_UNSUPPORTED
    d.dtype = lvb.BF16
    d.scale = float("nan")
    assert lvb.lib.lvb_attention_check(C.byref(d)) == lvb.LVB_ERR_INVALID_ARG


def test_status_strings(lvb):
    assert lvb.lib.lvb_status_string(4) == b"LVB_ERR_TIMEOUT"
    assert lvb.lib.lvb_set_wait_timeout_ms(0) == lvb.LVB_ERR_INVALID_ARG


def test_plan_routes_vectors_to_gemv(lvb):
    """N == 1 or M == 1: the matrix-vector kernel, with k split across CTAs when the rows
    alone cannot fill the GPU."""
    p = lvb.gemm_plan(8192, 1, 8192, lvb.I8, lvb.I32)
    assert p.gemv == 1 and p.instr_m == 0 and p.gemv_ksplit == 1
    p = lvb.gemm_plan(1, 8192, 8192, lvb.F16, lvb.F32)
    assert p.gemv == 1
    p = lvb.gemm_plan(64, 1, 1 << 20, lvb.F16, lvb.F32)      # few rows: k split across CTAs
    assert p.gemv == 1 and p.gemv_ksplit > 1
    assert lvb.gemm_plan(8192, 2, 8192, lvb.F16, lvb.F32).gemv == 0
    assert lvb.gemm_plan(8192, 1, 8192, lvb.I8, lvb.I32).launches == 1
    assert lvb.gemm_plan(64, 1, 1 << 20, lvb.F16, lvb.F32).launches == 2     # + the split sums
    assert lvb.gemm_plan(8192, 8192, 8192, lvb.F16, lvb.F16).launches == 1
    assert lvb.gemm_plan(64, 64, 72, lvb.I8, lvb.I32).launches == 3          # + repacks of A and B
    assert lvb.gemm_plan(0, 64, 72, lvb.I8, lvb.I32).launches == 0


def test_attention_plans(lvb):
    """Few query rows per KV head take the decoding kernel, split over a long cache; long
    query sequences the flash kernel; an empty key sequence the fill kernel."""
    p = lvb.attention_plan(8, 64, 8, 1, 16384)              # C5's cache, one new token
    assert p.kernel == lvb.ATTN_DECODE and p.splits > 1 and p.launches == 2 and p.ctas == 148
    p = lvb.attention_plan(64, 32, 32, 1, 2048)              # many heads: no split needed
    assert p.kernel == lvb.ATTN_DECODE and p.splits == 1 and p.launches == 1
    assert lvb.attention_plan(1, 32, 1, 1, 300).kernel == lvb.ATTN_DECODE   # 32 rows
    assert lvb.attention_plan(1, 64, 1, 1, 300).kernel == lvb.ATTN_FLASH    # 64 rows
    assert lvb.attention_plan(1, 8, 8, 1, 300, D=64).kernel == lvb.ATTN_FLASH
    p = lvb.attention_plan(4, 32, 32, 4096, 4096, dtype=lvb.F16)
    assert p.kernel == lvb.ATTN_FLASH and p.ctas == 148 and p.launches == 1   # persistent
    assert lvb.attention_plan(2, 4, 4, 10, 0).kernel == lvb.ATTN_EMPTY
    assert lvb.attention_plan(0, 4, 4, 10, 10).launches == 0
