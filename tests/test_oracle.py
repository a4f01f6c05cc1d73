"""The oracle pinned to the reference: its C restatement against the reference's own code (built from the reference
tree into oracle/_ref) and against committed golden outputs of that code and of the reference's fp64 truth key.
CPU only."""
import os

import numpy as np
import pytest

import oracle
from nunchi_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
needs_ref = pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built (no reference tree)")


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gold(kind, name):
    return np.load(os.path.join(GOLD, f"{kind}_{name}.npz"))


# ---------------- small math ----------------

def test_f2h_round_to_nearest_even_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(20000) * s for s in (1e-8, 1e-6, 1e-4, 1, 100, 3e4)]).astype(np.float32)
    edge = np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, np.inf, -np.inf],
                    np.float32)
    ties = (np.arange(1, 2048, dtype=np.float32) + 0.5) * np.float32(2.0 ** -10)   # exact halfway cases
    for x in np.concatenate([vals, edge, ties]):
        assert oracle.f2h(x) == int(np.float32(x).astype(np.float16).view(np.uint16)), x


def test_cut_edge_cases():
    x = np.zeros(128, np.float32)
    x[32:64] = 1e-30                      # tiny block (its scale's reciprocal still finite)
    x[64:96] = np.linspace(-3, 3, 32)     # includes exact .5 products
    x[96:128] = 127.0 * np.arange(32) / 31.0
    q, d, s = oracle.cut(x)
    assert (q[:32] == 0).all() and d[0] == 0 and s[0] == 0
    assert np.abs(q).max() <= 127
    for j in range(4):
        qq = np.rint(x[32 * j:32 * j + 32] * (np.float32(1) / d[j] if d[j] else 0)).astype(np.int64)
        assert (qq == q[32 * j:32 * j + 32]).all()


# ---------------- against the golden outputs of the reference's own code ----------------

@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_kernels_match_reference_golden(name):
    g = gold("ref", name)
    rows, cols = 64, 512
    for i, v in enumerate(g["kat_x"]):
        q, d, s = oracle.cut(v)
        assert np.array_equal(q, g["kat_q"][i]) and np.array_equal(bits(d), bits(g["kat_d"][i]))
        assert np.array_equal(bits(s), bits(g["kat_s"][i]))
    q = np.concatenate([oracle.cut(v)[0] for v in g["kat_x"]])
    d = np.concatenate([oracle.cut(v)[1] for v in g["kat_x"]])
    s = np.concatenate([oracle.cut(v)[2] for v in g["kat_x"]])
    out = oracle.q4_matvec(g["kat_q4"], rows, cols, q, d, s)
    assert np.array_equal(bits(out[:1]), bits(g["kat_out1"]))   # imi_q4_group
    assert np.array_equal(bits(out[:2]), bits(g["kat_out2"]))   # imi_q4_group2
    assert np.array_equal(bits(out), bits(g["kat_out5"]))       # imi_q8b + imi_q4_group_batch


@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_steps_match_reference_golden(name):
    g = gold("ref", name)
    o = oracle.Oracle(synth.cached_gguf(name), n_ctx=256)
    for i, t in enumerate(g["tokens"]):
        assert o.step(int(t)) == 0
        assert np.array_equal(bits(o.hidden), bits(g["hidden"][i])), f"hidden differs at position {i}"
        lg = o.logits
        if i < len(g["logits_full"]):
            assert np.array_equal(bits(lg), bits(g["logits_full"][i])), f"logits differ at position {i}"
        assert np.array_equal(np.argsort(-lg, kind="stable")[:16], g["logits_top_ids"][i])


def test_seoul_steps_match_reference_golden(seoul_path):
    g = gold("ref", "seoul")
    o = oracle.Oracle(seoul_path, n_ctx=64)
    for i, t in enumerate(g["tokens"]):
        o.step(int(t))
        assert np.array_equal(bits(o.hidden), bits(g["hidden"][i])), f"hidden differs at position {i}"
        lg = o.logits
        if i < len(g["logits_full"]):
            assert np.array_equal(bits(lg), bits(g["logits_full"][i]))
        assert np.array_equal(np.argsort(-lg, kind="stable")[:16], g["logits_top_ids"][i])
        assert lg.astype(np.float64).sum() == pytest.approx(g["logits_sum"][i], rel=1e-12)


@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_step_batch_matches_reference_golden(name):
    g = gold("ref", name)
    o = oracle.Oracle(synth.cached_gguf(name), n_ctx=256)
    ha = o.step_batch(embd=g["batch_embd"], want_logits=True, hidden_all=True)
    assert np.array_equal(bits(ha), bits(g["batch_hidden"]))
    assert np.array_equal(bits(o.logits), bits(g["batch_logits_full"][0]))


@pytest.mark.parametrize("name", ["tiny", "wide_heads", "seoul"])
def test_oracle_error_budget_against_truth_key(name):
    """imi's own error against the fp64 truth key (the reference's ref_exact.py, compare.py metrics): the oracle must
    sit at exactly the reference's budget; it is recorded here so the GPU tests can hold the engine to it."""
    g, t = gold("ref", name), gold("truth", name)
    eh = np.linalg.norm(g["hidden"] - t["hidden"], axis=1) / np.linalg.norm(t["hidden"], axis=1)
    assert eh.max() < 0.15, eh   # 8-bit input cuts: a few percent (seoul_check.cpp:36-43 metrics)
    full = min(len(t["logits_full"]), len(g["logits_full"]))
    lg_ref, lg_t = g["logits_full"][:full], t["logits_full"][:full]
    el = np.linalg.norm(lg_ref - lg_t, axis=1) / np.linalg.norm(lg_t, axis=1)
    assert el.max() < 0.15, el


# ---------------- live against the reference build (where the reference tree is present) ----------------

@needs_ref
@pytest.mark.parametrize("name", ["tiny", "small", "wide_heads"])
def test_steps_match_reference_live(name):
    path = synth.cached_gguf(name)
    o, r = oracle.Oracle(path, n_ctx=128), oracle.Reference(path, n_ctx=128)
    for t in synth.random_ids(20, o.n_vocab, 5):
        o.step(int(t))
        r.step(int(t))
        assert np.array_equal(bits(o.hidden), bits(r.hidden)) and np.array_equal(bits(o.logits), bits(r.logits))


@needs_ref
def test_riding_and_state_swap_match_reference_live(tiny_path):
    """The reference's step2 gives each conversation the numbers of its own step (seoul.cpp:222-224)."""
    r = oracle.Reference(tiny_path, n_ctx=64)
    o = oracle.Oracle(tiny_path, n_ctx=64)
    ob = o.new_state()
    b = r.new_state()
    ta, tb = synth.random_ids(12, r.n_vocab, 1), synth.random_ids(12, r.n_vocab, 2)
    for i in range(12):
        r.step2(int(ta[i]), None, True, b, int(tb[i]), None, True)
        o.step(int(ta[i]))
        ob.step(int(tb[i]))
        assert np.array_equal(bits(r.hidden), bits(o.hidden)) and np.array_equal(bits(b.logits), bits(ob.logits))


@needs_ref
def test_context_full_is_refused_like_the_reference(tiny_path):
    o = oracle.Oracle(tiny_path, n_ctx=3)
    for t in (1, 2, 3):
        assert o.step(t) == 0
    assert o.step(4) == 1 and o.pos == 3          # seoul.cpp:353: no step
    o.reset()
    with pytest.raises(RuntimeError):
        o.step_batch(tokens=np.arange(4, dtype=np.int32))   # seoul.cpp:498


# ---- the Q6_K word table of the product's own files: the restatement against the reference's own AVX2 code ----

def _q6k_rows(rng, rows, cols, scale_lo=-64, scale_hi=64):
    """Random Q6_K rows (210 B per 256 values: ql[128], qh[64], int8 scales[16], fp16 d): any bytes form a valid
    block; scales and d kept in the ranges real files use (or pushed to the int8 ends)."""
    nbk = cols // 256
    b = rng.integers(0, 256, size=(rows, nbk, 210), dtype=np.uint8)
    b[:, :, 192:208] = rng.integers(scale_lo, scale_hi, size=(rows, nbk, 16)).astype(np.int8).view(np.uint8)
    d = rng.uniform(1e-4, 4e-3, size=(rows, nbk)).astype(np.float16)
    b[:, :, 208:210] = d.view(np.uint8).reshape(rows, nbk, 2)
    return b.reshape(rows, nbk * 210)


@needs_ref
@pytest.mark.parametrize("cols,seed", [(256, 0), (2048, 1), (2048, 2), (8192, 3)])
def test_q6k_word_scores_match_reference(cols, seed):
    """imi_q8k::from and imi_q6k_row (tables.cpp:200-278): codes, scales and code sums identical, word scores bit
    for bit, including the saturating ends of the int8 scales and a large-magnitude input."""
    rng = np.random.default_rng(seed)
    W = _q6k_rows(rng, 96, cols, *((-128, 128) if seed == 2 else (-64, 64)))
    x = (rng.standard_normal(cols) * (40.0 if seed == 3 else 1.0)).astype(np.float32)
    for mine, ref in zip(oracle.q8k_from(x), oracle.q8k_from(x, reference=True)):
        assert np.array_equal(mine, ref)
    got, want = oracle.q6k_rows(W, x), oracle.q6k_rows(W, x, reference=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
def test_q6k_zero_input_and_lookup_match_reference():
    """A zero input block (scale 0, inverse 0: all codes 0) and the row lookup (tables.cpp:216-233)."""
    rng = np.random.default_rng(9)
    W = _q6k_rows(rng, 8, 2048)
    x = rng.standard_normal(2048).astype(np.float32)
    x[256:512] = 0.0
    q, d, bs = oracle.q8k_from(x)
    assert d[1] == 0.0 and not q[256:512].any() and not bs[16:32].any()
    got, want = oracle.q6k_rows(W, x), oracle.q6k_rows(W, x, reference=True)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for r in range(8):
        a, b = oracle.q6k_dequant_row(W[r], 8), oracle.q6k_dequant_row(W[r], 8, reference=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


needs_ref_q6k = pytest.mark.skipif(not oracle.reference_q6k_available(), reason="oracle/_ref not built")


@needs_ref_q6k
def test_q6k_word_table_steps_match_reference_live():
    """A model with the product's own Q6_K word table (lookup and word scores): the oracle's steps and prefill against
    the reference's own imi_seoul built without the Q4_0 word-table renames, bit for bit."""
    path = synth.cached_gguf("tiny_q6k")
    o, r = oracle.Oracle(path, n_ctx=96), oracle.ReferenceQ6K(path, n_ctx=96)
    ids = synth.random_ids(24, o.n_vocab, 6)
    o.step_batch(tokens=ids[:16], want_logits=True)
    r.step_batch(tokens=ids[:16], want_logits=True)
    assert np.array_equal(bits(o.logits), bits(r.logits))
    for t in ids[16:]:
        o.step(int(t))
        r.step(int(t))
        assert np.array_equal(bits(o.hidden), bits(r.hidden)) and np.array_equal(bits(o.logits), bits(r.logits))


@needs_ref
def test_q41_layer_tables_steps_match_reference_live():
    """Q4_1 layer tables (a minimum m per block: out = acc + cor with cor = fma(m, s_j, cor), group_avx2<true>,
    tables.cpp:127-143): the oracle's prefill and steps against the reference's own code, bit for bit."""
    path = synth.cached_gguf("tiny_q41")
    o, r = oracle.Oracle(path, n_ctx=96), oracle.Reference(path, n_ctx=96)
    ids = synth.random_ids(24, o.n_vocab, 7)
    o.step_batch(tokens=ids[:16], want_logits=True)
    r.step_batch(tokens=ids[:16], want_logits=True)
    assert np.array_equal(bits(o.logits), bits(r.logits))
    for t in ids[16:]:
        o.step(int(t))
        r.step(int(t))
        assert np.array_equal(bits(o.hidden), bits(r.hidden)) and np.array_equal(bits(o.logits), bits(r.logits))


def test_oracle_memory_import_continues_identically(tiny_path):
    """The parity harness's state import (or_state_import): a conversation given another conversation's memory
    (position, K/V caches, conv memory) steps to bit for bit the same numbers as the original."""
    o = oracle.Oracle(tiny_path, n_ctx=64)
    ids = synth.random_ids(12, o.n_vocab, 21)
    o.step_batch(tokens=ids[:10], want_logits=False)
    s = o.state
    conv = np.stack([s.conv_state(il) for il in range(o.n_layer) if il not in (1, 3)])   # tiny: attention at 1, 3
    k = np.stack([s.k_cache(a)[:10] for a in range(o.n_attn)])
    v = np.stack([s.v_cache(a)[:10] for a in range(o.n_attn)])
    t = o.new_state()
    t.import_memory(10, k, v, conv)
    assert t.pos == 10
    for tok in ids[10:]:
        s.step(int(tok))
        t.step(int(tok))
        assert np.array_equal(bits(s.logits), bits(t.logits)) and np.array_equal(bits(s.hidden), bits(t.hidden))
    with pytest.raises(ValueError):
        t.import_memory(65, np.zeros((2, 65, 128), np.uint16), np.zeros((2, 65, 128), np.uint16), conv)


def test_oracle_builds_differ_only_in_the_exponential(tiny_path):
    """liboracle_cr.so (correctly rounded exponential, as the engine computes it) against liboracle.so (the C library's
    expf, as imi): the same code otherwise, so steps without any exponential in play agree bit for bit and steps with
    it differ at most by what a few 1-ulp expf differences do."""
    a, b = oracle.Oracle(tiny_path, n_ctx=32), oracle.Oracle(tiny_path, n_ctx=32, exp="cr")
    assert a.L is not b.L
    diff = 0.0
    for t in synth.random_ids(8, a.n_vocab, 3):
        a.step(int(t))
        b.step(int(t))
        diff = max(diff, float(np.abs(a.logits - b.logits).max() / np.abs(a.logits).max()))
    assert diff < 1e-2
    x = np.random.default_rng(1).standard_normal(512).astype(np.float32)
    qa = [np.asarray(v) for v in oracle.cut(x)]
    L = oracle.Oracle.lib("cr")
    q, d, s = np.zeros(512, np.int8), np.zeros(16, np.float32), np.zeros(16, np.float32)
    L.or_cut(x.ctypes.data, 512, q.ctypes.data, d.ctypes.data, s.ctypes.data)
    assert np.array_equal(q, qa[0]) and np.array_equal(bits(d), bits(qa[1])) and np.array_equal(bits(s), bits(qa[2]))
