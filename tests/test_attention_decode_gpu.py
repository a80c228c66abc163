"""GPU tier: attention with few query rows per KV head (decoding) — the HBM-bound kernel that
lvb_attention_fwd takes when group·seq_q <= 32 and head_dim == 128 — through the C ABI
against the oracle. Tolerances are those of the flash-attention tests:
    Float16:  max|Δ| <= 1e-2 and relative Frobenius <= 1e-3
    BFloat16: max|Δ| <= 2^-8·(max|V| + max|O|) and relative Frobenius <= 1e-2
    lse (fp32) within 1e-3 absolute; rows that see no key: O = 0, lse = -inf.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import vocab
from oracle.attention import attention_ref
from oracle.inputs import attention_inputs
from test_attention_gpu import check, run, tdt

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"


def test_golden_fixture(lvb, torch_cuda):
    """A GQA group of 8 decoding against a 700-key cache (bf16): the fixture's inputs and its
    oracle output (tests/golden/make_golden.py)."""
    z = np.load(GOLDEN / "attn_bf16_decode_gqa.npz")
    Q, K, V = (vocab.bf16_bits_to_f32(z[k]) for k in ("Q", "K", "V"))
    O = run(lvb, torch_cuda, Q, K, V, "BFloat16", bool(z["causal"]), float(z["scale"]))
    check(O, z["O"].astype(np.float64), V, "BFloat16")


@pytest.mark.parametrize("T", ["Float16", "BFloat16"])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv", [
    (2, 64, 8, 1, 16384),    # the C5 KV cache, one new token per sequence: split over keys
    (1, 8, 8, 1, 1),         # one key
    (3, 16, 2, 2, 777),      # two positions, ragged last key block
    (1, 32, 1, 1, 300),      # a group of 32 query heads (32 rows)
    (2, 4, 4, 4, 129),       # MHA, four positions
    (1, 12, 4, 3, 4099),     # 9 rows of 16
    (1, 2, 1, 16, 16),       # square causal block
    (2, 8, 1, 4, 2),         # seq_q > seq_kv: under the causal mask early rows see no key
    (1, 4, 2, 1, 70000),     # long cache, few heads
])
def test_decode(lvb, torch_cuda, T, causal, B, Hq, Hkv, Sq, Skv):
    Q, K, V = attention_inputs(B, Hq, Hkv, Sq, 128, T, seed=Sq + Skv + Hq, Skv=Skv)
    scale = 128 ** -0.5
    O, lse = run(lvb, torch_cuda, Q, K, V, T, causal, scale, want_lse=True)
    ref, lref = attention_ref(Q, K, V, causal, scale, return_lse=True)
    check(O, ref, V, T)
    fin = np.isfinite(lref)
    assert np.array_equal(np.isfinite(lse), fin)
    assert np.abs(lse[fin] - lref[fin]).max(initial=0) <= 1e-3
    assert (O[~fin] == 0).all()


def test_decode_large_scores(lvb, torch_cuda):
    """Scores of several hundred: the running max moves far between key blocks and splits,
    which exercises the lazy rescale and the merge of the splits."""
    Q, K, V = attention_inputs(1, 8, 1, 1, 128, "Float16", seed=91, Skv=9000)
    O = run(lvb, torch_cuda, Q, K, V, "Float16", True, 20 * 128 ** -0.5)
    ref = attention_ref(Q, K, V, True, 20 * 128 ** -0.5)
    assert np.isfinite(O).all()
    check(O, ref, V, "Float16")


def test_decode_strided_cache(lvb, torch_cuda):
    """A KV cache stored [batch][seq][kv head][head_dim] and a query [batch][1][head][dim],
    viewed as [B][H][S][D] (non-packed strides)."""
    torch = torch_cuda
    Q, K, V = attention_inputs(2, 16, 4, 1, 128, "BFloat16", seed=92, Skv=5000)
    def bshd(x):
        t = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3))).to(torch.bfloat16).cuda()
        return t.transpose(1, 2)
    dQ, dK, dV = bshd(Q), bshd(K), bshd(V)
    dO = torch.empty(2, 1, 16, 128, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    lvb.attention(dO, dQ, dK, dV, causal=True)
    torch.cuda.synchronize()
    assert lvb.device_status() == (0, 0, 0)
    ref = attention_ref(Q, K, V, True, 128 ** -0.5)
    check(dO.float().cpu().numpy(), ref, V, "BFloat16")


def test_decode_repeatable(lvb, torch_cuda):
    """The splits are merged in a fixed order: two calls give identical bits."""
    torch = torch_cuda
    Q, K, V = attention_inputs(4, 32, 8, 1, 128, "BFloat16", seed=93, Skv=12345)
    dQ, dK, dV = (torch.from_numpy(x).to(tdt(torch, "BFloat16")).cuda() for x in (Q, K, V))
    outs = []
    for _ in range(2):
        dO = torch.empty_like(dQ)
        lvb.attention(dO, dQ, dK, dV, causal=True)
        torch.cuda.synchronize()
        outs.append(dO.float().cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
