"""The arithmetic of the chained stack's LayerNorm statistics, restated in float32 numpy: the residual GEMM's
per-256-column (mean, M2) blocks of a bf16 row, summed about the row block's first value, and the next up_conv
kernel's equal-count merge (Chan et al.) into rstd.  Checked against two-pass float64 statistics on rows where a
naive sum of squares would cancel (a large mean next to a small spread) and on constant rows."""
import numpy as np
import pytest

from oracle import conv_module as O

BLOCK = 256


def _blocks(row):
    """(mean, M2) of each 256-column block, as the epilogue forms them in fp32."""
    out = []
    for b in range(row.size // BLOCK):
        x = row[b * BLOCK:(b + 1) * BLOCK].astype(np.float32)
        k = x[0]
        d = (x - k).astype(np.float32)
        s = np.float32(0)
        q = np.float32(0)
        for v in d:
            s = np.float32(s + v)
            q = np.float32(q + np.float32(v * v))
        mt = np.float32(s / np.float32(BLOCK))
        out.append((np.float32(k + mt), max(np.float32(q - s * mt), np.float32(0))))
    return out


def _merged_rstd(blocks, eps):
    mean, m2 = blocks[0]
    for j, (mj, m2j) in enumerate(blocks[1:], start=1):
        delta = np.float32(mj - mean)
        mean = np.float32(mean + delta * np.float32(1.0 / (j + 1)))
        m2 = np.float32(m2 + np.float32(delta * delta * np.float32(BLOCK * j / (j + 1)) + m2j))
    d = BLOCK * len(blocks)
    return np.float32(1.0 / np.sqrt(np.float32(m2 / np.float32(d) + np.float32(eps)))), mean


@pytest.mark.parametrize("D", [256, 512, 1024, 2048])
@pytest.mark.parametrize("loc,scale", [(0.0, 1.0), (5.0, 1.0), (300.0, 0.5), (-40.0, 30.0), (1.0, 1e-3)])
def test_block_merge_matches_two_pass(D, loc, scale):
    rng = np.random.default_rng(D + int(abs(loc)))
    eps = 1e-5
    for _ in range(4):
        row = O.bf16_round((rng.standard_normal(D) * scale + loc).astype(np.float32))
        rstd, mean = _merged_rstd(_blocks(row), eps)
        x = row.astype(np.float64)
        ref_mean = x.mean()
        ref_rstd = 1.0 / np.sqrt(((x - ref_mean) ** 2).mean() + eps)
        assert abs(float(mean) - ref_mean) <= 1e-6 * max(1.0, abs(ref_mean))
        assert abs(float(rstd) - ref_rstd) <= 2e-5 * ref_rstd


def test_constant_row():
    row = np.full(1024, 3.5, dtype=np.float32)
    rstd, mean = _merged_rstd(_blocks(row), 1e-5)
    assert float(mean) == 3.5
    assert abs(float(rstd) - 1.0 / np.sqrt(1e-5)) <= 1e-3
