"""GPU tier: the tcgen05 flash-attention forward through the C ABI against the oracle.

Tolerances (per element, written from the error sources of the kernel's arithmetic):
  P is rounded to the input type before P·V and O is rounded to it at the store, so
  |ΔO| <= u·(max|V| + |O|) with u the unit roundoff of the type (2^-11 fp16, 2^-8 bf16);
  the fp32 accumulation and the hardware exp2 add far less. Stated bounds:
    Float16:  max|Δ| <= 1e-2 and relative Frobenius <= 1e-3
    BFloat16: max|Δ| <= 2^-8·(max|V| + max|O|) and relative Frobenius <= 1e-2
  lse (fp32) within 1e-3 absolute.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle.attention import attention_ref, attention_blockwise
from oracle.inputs import attention_inputs, ATTN_CONFIGS

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"


def tdt(torch, T):
    return torch.float16 if T == "Float16" else torch.bfloat16


def run(lvb, torch, Q, K, V, T, causal, scale, want_lse=False):
    dQ, dK, dV = (torch.from_numpy(np.ascontiguousarray(x)).to(tdt(torch, T)).cuda()
                  for x in (Q, K, V))
    dO = torch.full_like(dQ, 7.0)
    lse = torch.empty(Q.shape[:3], dtype=torch.float32, device="cuda") if want_lse else None
    lvb.attention(dO, dQ, dK, dV, causal=causal, scale=scale, lse=lse)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    O = dO.float().cpu().numpy()
    return (O, lse.cpu().numpy()) if want_lse else O


def check(O, ref, V, T):
    d = np.abs(O.astype(np.float64) - ref)
    rf = np.linalg.norm(O - ref) / max(np.linalg.norm(ref), 1e-30)
    if T == "Float16":
        assert d.max() <= 1e-2 and rf <= 1e-3, (d.max(), rf)
    else:
        bound = 2.0 ** -8 * (np.abs(V).max() + np.abs(ref).max())
        assert d.max() <= bound and rf <= 1e-2, (d.max(), bound, rf)


def test_golden_fixture(lvb, torch_cuda):
    z = np.load(GOLDEN / "attn_f16_gqa_causal.npz")
    O = run(lvb, torch_cuda, z["Q"], z["K"], z["V"], "Float16", bool(z["causal"]),
            float(z["scale"]))
    check(O, z["O"].astype(np.float64), z["V"], "Float16")


@pytest.mark.parametrize("T", ["Float16", "BFloat16"])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv", [
    (1, 2, 2, 256, 256),      # one tile pair, square
    (2, 4, 1, 300, 300),      # ragged query/key tails, GQA 4:1
    (1, 8, 2, 200, 333),      # Sq < Skv: causal mask offset by Skv - Sq
    (1, 2, 2, 640, 128),      # Sq > Skv: early rows see no key under the causal mask
    (1, 1, 1, 1, 1000),       # decode-like single query
])
def test_small(lvb, torch_cuda, T, D, causal, B, Hq, Hkv, Sq, Skv):
    Q, K, V = attention_inputs(B, Hq, Hkv, Sq, D, T, seed=Sq + Skv + D, Skv=Skv)
    scale = D ** -0.5
    O, lse = run(lvb, torch_cuda, Q, K, V, T, causal, scale, want_lse=True)
    ref, lref = attention_ref(Q, K, V, causal, scale, return_lse=True)
    check(O, ref, V, T)
    fin = np.isfinite(lref)
    assert np.array_equal(np.isfinite(lse), fin)
    assert np.abs(lse[fin] - lref[fin]).max(initial=0) <= 1e-3


def test_large_scores_stay_finite(lvb, torch_cuda):
    # scores of several hundred (a 20x scale): the running max moves often and far, which
    # exercises the lazy O rescale
    Q, K, V = attention_inputs(1, 2, 2, 512, 128, "Float16", seed=77)
    O = run(lvb, torch_cuda, Q, K, V, "Float16", True, 20 * 128 ** -0.5)
    ref = attention_ref(Q, K, V, True, 20 * 128 ** -0.5)
    assert np.isfinite(O).all()
    check(O, ref, V, "Float16")


def test_strided_views(lvb, torch_cuda):
    # Q/K/V as [B][S][H][D] storage viewed as [B][H][S][D] (non-packed strides)
    torch = torch_cuda
    Q, K, V = attention_inputs(2, 4, 2, 192, 128, "Float16", seed=5)
    def bshd(x):
        t = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3))).half().cuda()
        return t.transpose(1, 2)
    dQ, dK, dV = bshd(Q), bshd(K), bshd(V)
    dO = torch.empty(2, 192, 4, 128, dtype=torch.float16, device="cuda").transpose(1, 2)
    lvb.attention(dO, dQ, dK, dV, causal=True)
    torch.cuda.synchronize()
    ref = attention_ref(Q, K, V, True, 128 ** -0.5)
    check(dO.float().cpu().numpy(), ref, V, "Float16")



def test_output_rows_16_byte_aligned(lvb, torch_cuda):
    """Output rows 272 bytes apart from a base 16 bytes past a 32-byte boundary: rows alternate
    between the epilogue's 32-byte stores and its 16-byte stores; the padding between rows
    stays untouched."""
    torch = torch_cuda
    Q, K, V = attention_inputs(1, 4, 2, 300, 128, "Float16", seed=95)
    dQ, dK, dV = (torch.from_numpy(x).cuda() for x in (Q, K, V))
    buf = torch.full((4 * 300 * 136 + 8,), 7.0, dtype=torch.float16, device="cuda")
    rows = buf[8:].view(1, 4, 300, 136)
    assert rows.data_ptr() % 32 == 16
    dO = rows[..., :128]
    lvb.attention(dO, dQ, dK, dV, causal=True)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    ref = attention_ref(Q, K, V, True, 128 ** -0.5)
    check(dO.float().cpu().numpy(), ref, V, "Float16")
    assert bool((rows[..., 128:] == 7).all()) and bool((buf[:8] == 7).all())

def _full_config(lvb, torch, name, units):
    """A benchmark configuration at its stated size, inputs from its PCG64 seed. For each
    (b, h) unit listed, the rows of the first query tile, of a mid-sequence tile pair and of
    the last tile pair (the heaviest causal work item) are checked against the float64
    definition, output and lse; every row is checked for |O| <= max|V| and finiteness."""
    from oracle.inputs import attention_inputs_stored
    from oracle.attention import attention_rows
    from oracle.vocab import bf16_bits_to_f32
    cfg = ATTN_CONFIGS[name]
    T = cfg["dtype"]
    Bn, Hq, Hkv, S, D = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["S"], cfg["D"]
    Qs, Ks, Vs = attention_inputs_stored(Bn, Hq, Hkv, S, D, T, cfg["seed"])

    def dev(x):
        if T == "Float16":
            return torch.from_numpy(x).cuda()
        return torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)

    def vals(x):
        return x.astype(np.float32) if T == "Float16" else bf16_bits_to_f32(x)
    dQ, dK, dV = dev(Qs), dev(Ks), dev(Vs)
    dO = torch.empty_like(dQ)
    lse = torch.empty((Bn, Hq, S), dtype=torch.float32, device="cuda")
    lvb.attention(dO, dQ, dK, dV, causal=True, lse=lse)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    g = Hq // Hkv
    mid = (S // 2 // 256) * 256
    rows = np.concatenate([np.arange(0, 128), np.arange(mid - 128, mid + 128),
                           np.arange(S - 256, S)])
    for (b, h) in units:
        q = vals(Qs[b, h][rows])
        k = vals(Ks[b, h // g])
        v = vals(Vs[b, h // g])
        ref, lref = attention_rows(q, k, v, rows, True, D ** -0.5, sq=S)
        O = dO[b, h].float().cpu().numpy()[rows]
        check(O, ref, v, T)
        got = lse[b, h].cpu().numpy()[rows]
        assert np.abs(got - lref).max() <= 1e-3, (b, h, float(np.abs(got - lref).max()))
    # every row is a convex combination of V rows: |O| <= max|V| everywhere
    assert float(dO.float().abs().max()) <= float(dV.float().abs().max()) + 1e-2
    assert torch.isfinite(dO.float()).all()
    assert torch.isfinite(lse).all()


def _units(B, Hq, Hkv, n):
    """n (b, h) units: both ends, a whole GQA group of one KV head, and evenly spread others."""
    g = Hq // Hkv
    u = {(0, 0), (B - 1, Hq - 1), (B // 2, Hq // 2)}
    u |= {(B // 2, (Hkv // 2) * g + i) for i in range(min(g, 8))}
    k = 0
    while len(u) < n:
        u.add(((7 * k) % B, (13 * k + 5) % Hq))
        k += 1
    return sorted(u)


@pytest.mark.slow
def test_config4_fp16_full(lvb, torch_cuda):
    _full_config(lvb, torch_cuda, "C4", _units(4, 32, 32, 16))


@pytest.mark.slow
def test_config5_bf16_gqa_full(lvb, torch_cuda):
    _full_config(lvb, torch_cuda, "C5", _units(8, 64, 8, 16))


def test_prepared_call_matches_one_shot_call(lvb, torch_cuda):
    """lvb.prepare_attention (descriptor built once) gives exactly lvb.attention's result."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(5)
    Q = torch.randn(2, 8, 1024, 128, device="cuda", dtype=torch.float16, generator=g)
    K = torch.randn(2, 4, 1024, 128, device="cuda", dtype=torch.float16, generator=g)
    V = torch.randn(2, 4, 1024, 128, device="cuda", dtype=torch.float16, generator=g)
    ref = torch.empty_like(Q)
    lvb.attention(ref, Q, K, V, causal=True)
    O = torch.zeros_like(Q)
    a = lvb.prepare_attention(O, Q, K, V, causal=True)
    for _ in range(3):
        a()
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    assert torch.equal(O, ref)
