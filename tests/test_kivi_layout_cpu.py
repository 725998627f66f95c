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


def test_code_word_selectors_follow_the_packed_order():
    """Packed 2-bit format: element 16w + 4k + b of a group at bit 8b + 2k of
    word w.  The selector ``((word >> 2k) & 0x03030303) * 0x22 + 0x10101010``
    then names, per byte, the two table bytes of elements 4k .. 4k+3 --
    k-step kk of a thread uses shift k = kk % 4 of word kk / 4."""
    rng = np.random.default_rng(7)
    codes = rng.integers(0, 4, 32)
    words = [0, 0]
    for j, code in enumerate(codes):
        w, rem = divmod(j, 16)
        k, b = divmod(rem, 4)
        words[w] |= int(code) << (8 * b + 2 * k)
    for kk in range(8):
        w, k = divmod(kk, 4)
        sel = ((words[w] >> (2 * k)) & 0x03030303) * 0x22 + 0x10101010
        for b in range(4):
            lo, hi = (sel >> (8 * b)) & 0xF, (sel >> (8 * b + 4)) & 0xF
            assert (lo, hi) == (2 * codes[4 * kk + b], 2 * codes[4 * kk + b] + 1)
