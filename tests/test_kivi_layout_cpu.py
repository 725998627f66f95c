"""Index algebra of the fused KIVI decode's K-in-registers path, on the CPU.

The transposed tile computes S^T = K Q^T with ``mma.m16n8k16`` (A = the
warp's 16 keys x 16 k-columns, B = 16 k-columns x 8 q-heads).  It feeds k
in a permuted order -- logical column ``2c + e + 8h`` of k-step ``kk`` is
head-dim column ``c*D/4 + 4kk + 2h + e`` -- so thread ``(g, c)`` holds one
quantisation group of rows g and g + 8.  These tests model the MMA
fragment layout (PTX ISA, ``mma.m16n8k16`` with 16-bit A/B: a0/a1/a2/a3 =
rows g, g+8, g, g+8 x columns 2c..2c+1, 2c..2c+1, 2c+8..2c+9, 2c+8..2c+9;
b0/b1 = rows 2c..2c+1, 2c+8..2c+9 x column g) and the packed 2-bit
code-word order, and check that the permuted product equals K Q^T.
"""
from __future__ import annotations

import numpy as np
import pytest


def _logical_to_head_dim(D: int, kk: int, kin: int) -> int:
    h, c, e = int(kin >= 8), (kin % 8) // 2, kin % 2
    return (D // 4) * c + 4 * kk + 2 * h + e


@pytest.mark.parametrize("D", [64, 128])
def test_permutation_is_a_bijection(D):
    cols = sorted(_logical_to_head_dim(D, kk, kin) for kk in range(D // 16) for kin in range(16))
    assert cols == list(range(D))


@pytest.mark.parametrize("D", [64, 128])
def test_thread_span_is_one_group(D):
    """Each thread's D/4 columns of a row sit in one quantisation group of
    32, so one value table per row serves all of its fragments."""
    for c in range(4):
        cols = {(D // 4) * c + 4 * kk + 2 * h + e
                for kk in range(D // 16) for h in (0, 1) for e in (0, 1)}
        assert len({d // 32 for d in cols}) == 1


@pytest.mark.parametrize("D", [64, 128])
def test_permuted_fragments_give_k_q_transpose(D):
    rng = np.random.default_rng(D)
    K = rng.standard_normal((16, D))
    Q = rng.standard_normal((8, D))
    S = np.zeros((16, 8))
    for kk in range(D // 16):
        A = np.full((16, 16), np.nan)
        B = np.full((16, 8), np.nan)
        for lane in range(32):
            g, c = lane >> 2, lane & 3
            base = (D // 4) * c + 4 * kk
            # A: rows g, g + 8; pair h holds span elements 4kk + 2h + {0, 1}
            for r in (g, g + 8):
                for h in (0, 1):
                    for e in (0, 1):
                        A[r, 2 * c + 8 * h + e] = K[r, base + 2 * h + e]
            # B: q-head g, k rows 2c + 8h + e, read from the same columns
            for h in (0, 1):
                for e in (0, 1):
                    B[2 * c + 8 * h + e, g] = Q[g, base + 2 * h + e]
        assert not np.isnan(A).any() and not np.isnan(B).any()   # every slot owned once
        S += A @ B
    np.testing.assert_allclose(S, K @ Q.T, rtol=1e-12, atol=1e-12)


def test_code_pairs_decode_through_16_bit_exponent_magic():
    """Packed 2-bit format: element 16w + e of a group at bit 16*(e & 1) +
    2*(e >> 1) of word w, so pair q = (2q, 2q+1) sits at bit 2q of both
    16-bit halves.  The decoder's LOP3 ((w & (0x00030003 << 2q)) | M_q),
    with M_q a 16-bit float whose exponent makes bit 2q worth 1, gives
    E_q + c in each half; subtracting E_q leaves c exactly.  Pairs past the
    mantissa (q >= 5 for fp16, q >= 3 for bf16) are read from the word
    shifted right by 10 (fp16) or 6 (bf16) bits, in steps.  k-step kk of a
    thread uses pairs 2kk and 2kk + 1 of its span: word kk / 4."""
    rng = np.random.default_rng(7)
    codes = rng.integers(0, 4, 32)
    words = [0, 0]
    for j, code in enumerate(codes):
        w, e = divmod(j, 16)
        words[w] |= int(code) << (16 * (e & 1) + 2 * (e >> 1))
    for name, mant, per, shift, bias in (("f16", 10, 5, 10, 15), ("bf16", 7, 3, 6, 127)):
        dt = np.float16 if name == "f16" else None
        for p in range(16):
            w, q8 = divmod(p, 8)
            seg, q = divmod(q8, per)
            word = words[w] >> (seg * shift)
            m = (bias + mant - 2 * q) << mant            # 2^(mant - 2q) as 16-bit bits
            bits = (word & (0x00030003 << (2 * q))) | (m | (m << 16))
            lo, hi = bits & 0xFFFF, bits >> 16
            if name == "f16":
                vals = [float(np.array([x], dtype=np.uint16).view(dt)[0]) for x in (lo, hi)]
            else:
                vals = [float(np.array([x << 16], dtype=np.uint32).view(np.float32)[0])
                        for x in (lo, hi)]
            E = 2.0 ** (mant - 2 * q)
            assert [v - E for v in vals] == [codes[2 * p], codes[2 * p + 1]], (name, p)
    # k-step kk: pairs 2kk + h of the span (h = 0 -> a0/a1, h = 1 -> a2/a3)
    for kk in range(8):
        for h in (0, 1):
            p = 2 * kk + h
            assert p // 8 == kk // 4 and 2 * p == 4 * kk + 2 * h
