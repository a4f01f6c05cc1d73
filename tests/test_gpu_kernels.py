"""Kernel-level parity on the GPU (B200): the 8-bit cut and the 4-bit table kernel against the oracle, bit for bit.
Integer block dots and 8-bit codes are integer work: bit-exact. The float outputs of the table kernel are also
bit-exact, because the kernel keeps imi's per-row accumulation order (tables.cpp:127-143)."""
import numpy as np
import pytest

import nunchi_b200 as nb
import oracle
from nunchi_b200 import synth

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_cut_bit_exact():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4096), rng.standard_normal(4096) * 1e-3, rng.standard_normal(4096) * 50,
                        np.zeros(32), np.linspace(-3, 3, 32), 127.0 * np.arange(32) / 31.0, np.full(32, 1e-30)])
    x = x.astype(np.float32)
    q, d, s = nb.q8_cut(x)
    qo, do, so = oracle.cut(x)
    assert np.array_equal(q, qo)
    assert np.array_equal(bits(d), bits(do)) and np.array_equal(bits(s), bits(so))


@pytest.mark.parametrize("rows,cols,ncol", [(8, 256, 1), (64, 512, 1), (2048, 2048, 1), (300, 8192, 1), (1003, 512, 1),
                                            (2048, 2048, 2), (1000, 512, 3), (97, 2048, 8), (5, 1024, 5)])
def test_q4_table_bit_exact(rows, cols, ncol):
    rng = np.random.default_rng(rows * 7 + cols + ncol)
    q4 = synth._q4_0(rng, rows, cols).reshape(-1)
    x = rng.standard_normal((ncol, cols)).astype(np.float32)
    cuts = [oracle.cut(v) for v in x]
    cq, cd, cs = (np.concatenate([c[k] for c in cuts]) for k in range(3))
    want = oracle.q4_matvec(q4, rows, cols, cq, cd, cs)
    if ncol == 1:
        out, dots = nb.q4_matvec(q4, rows, cols, cq, cd, cs, dots=True)
        assert np.array_equal(dots, oracle.block_dots(q4, rows, cols, cq)), "integer block dots differ"
    else:
        out = nb.q4_matvec(q4, rows, cols, cq, cd, cs)
    assert np.array_equal(bits(out), bits(want))


def test_q4_table_matches_reference_golden():
    """The reference's own imi_q4_group / group2 / group_batch outputs (committed golden) on the device."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_tiny.npz"))
    rows, cols = 64, 512
    q, d, s = (np.concatenate([g[k][i] for i in range(5)]) for k in ("kat_q", "kat_d", "kat_s"))
    out = nb.q4_matvec(g["kat_q4"], rows, cols, q, d, s)
    assert np.array_equal(bits(out), bits(g["kat_out5"]))
    assert np.array_equal(bits(nb.q4_matvec(g["kat_q4"], rows, cols, q[:cols], d[:16], s[:16])), bits(g["kat_out1"]))


# ---- the Q6_K word table (the product's own word-table format): device word scores against the oracle ----

def _q6k_rows(rng, rows, cols, scale_lo=-64, scale_hi=64):
    """Random Q6_K rows: any bytes form valid blocks; int8 scales in [scale_lo, scale_hi), fp16 d in real ranges."""
    nbk = cols // 256
    b = rng.integers(0, 256, size=(rows, nbk, 210), dtype=np.uint8)
    b[:, :, 192:208] = rng.integers(scale_lo, scale_hi, size=(rows, nbk, 16)).astype(np.int8).view(np.uint8)
    b[:, :, 208:210] = rng.uniform(1e-4, 4e-3, size=(rows, nbk)).astype(np.float16).view(np.uint8).reshape(rows, nbk, 2)
    return b.reshape(rows, nbk * 210)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,seed", [(1000, 256, 0), (1000, 2048, 1), (333, 8192, 2), (97496, 2048, 3)])
def test_q6k_word_scores_bit_exact(rows, cols, seed):
    """imi_q8k::from and imi_q6k_row on the device (imi_cuda_q6k_scores) against the oracle (itself pinned to the
    reference's own AVX2 code): the input cut identical, every word score bit for bit; seed 2 pushes the scales to
    the int8 ends and the input to large magnitudes, and one input block is zero (scale 0)."""
    rng = np.random.default_rng(seed)
    W = _q6k_rows(rng, rows, cols, *((-128, 128) if seed == 2 else (-64, 64)))
    x = (rng.standard_normal(cols) * (40.0 if seed == 2 else 1.0)).astype(np.float32)
    x[:256] = 0.0 if seed == 1 else x[:256]
    got, cut = nb.q6k_scores(W, x)
    for mine, want in zip(cut, oracle.q8k_from(x)):
        assert np.array_equal(mine, want)
    want = oracle.q6k_rows(W, x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- the tensor-core batched read (tcgen05, fp16 codes, exact block dots; imi's chains per (row, input)) ----

@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,ncol", [(128, 256, 16), (2048, 2048, 64), (300, 8192, 32), (1003, 512, 48),
                                            (2048, 2048, 128), (3104, 2048, 40), (97496, 2048, 64), (16384, 2048, 64),
                                            (2048, 8192, 64), (77, 1024, 1), (129, 256, 256)])
def test_tc_table_bit_exact(rows, cols, ncol):
    """imi_cuda_q4_matmul against the oracle (imi_q4_group's per-row result for each input), bit for bit: block dots
    from fp16 x fp16 -> fp32 MMAs are exact, and the epilogue keeps the per-row fma order"""
    rng = np.random.default_rng(rows + 3 * cols + 7 * ncol)
    q4 = synth._q4_0(rng, rows, cols).reshape(-1)
    x = rng.standard_normal((ncol, cols)).astype(np.float32) * rng.uniform(0.1, 4.0, (ncol, 1)).astype(np.float32)
    x[0, :64] = 0.0                                      # zero blocks: scale 0
    cuts = [oracle.cut(v) for v in x]
    cq, cd, cs = (np.concatenate([c[k] for c in cuts]) for k in range(3))
    want = np.asarray(oracle.q4_matvec(q4, rows, cols, cq, cd, cs), np.float32).reshape(ncol, rows)
    got = nb.q4_matmul(q4, rows, cols, cq, cd, cs)
    assert np.array_equal(bits(got), bits(want)), f"max rel {np.abs(got - want).max() / np.abs(want).max():.3g}"
