"""Parity at the context lengths the benchmarks run (B200), against the oracle and against stepping alone.

* Long-context attention: the engine's attention stages cached V rows in shared-memory tiles of 512 positions
  (head_dim 64) or 256 (head_dim 128), two tiles in flight; lengths just below, at and above a tile edge and several
  tiles long exercise the refill and the alternating tile buffers. At each length the oracle is given exactly the
  engine's memory (checkpoint image: K/V caches, conv memory, position) and both take one step, so the comparison
  isolates the step at that length from drift accumulated before it (seoul.cpp:425-456, 589-621).
* configs[1] (BASELINE): the Seoul shape, conversation A after 1024 ids (seed 1), B after 256 (seed 2), 128 greedy
  steps riding (one table read for both): tokens, scores, hidden states and memory byte-identical to running each
  alone; steps at positions 1024+ checked against the oracle from imported memory.
* sessions at contexts 1500-2048 stepped together equal stepping each alone, byte for byte, and one of them
  against the oracle."""
import numpy as np
import pytest

import nunchi_b200 as nb
import oracle
from nunchi_b200 import synth
from parity import TOL, bits, close, follow_greedy, import_memory, record, rel, same_bits

pytestmark = pytest.mark.gpu

LENGTHS = (511, 512, 513, 1025, 2047)


def step_both(g, o, token, where):
    """one step of the engine state g and the oracle state o (same memory beforehand); returns (rel hidden, rel
    scores, bit-identical)"""
    g.step(int(token))
    o.step(int(token))
    hg, ho, lg, lo = g.hidden, o.hidden, g.logits, o.logits
    rh = close(hg, ho, where + " hidden")
    rl = close(lg, lo, where + " scores")
    return rh, rl, same_bits(hg, ho) and same_bits(lg, lo)


@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_long_context_step_vs_oracle(name):
    """tiny: head_dim 64, full attention; wide_heads: head_dim 128, rope_freqs on the full layers, one layer with a
    window of 8 (window layers read only their last 8 positions at every length)."""
    path = synth.cached_gguf(name)
    n_ctx = 2304
    e = nb.Engine(path, n_ctx=n_ctx)
    o = oracle.Oracle(path, n_ctx=n_ctx)
    g = e.new_state()
    ids = synth.random_ids(n_ctx, e.n_vocab, 31)
    exact = 0
    for L in LENGTHS:
        g.step_batch(tokens=ids[g.pos:L], want_logits=False)
        assert g.pos == L
        assert import_memory(g, o.state) == L
        rh, rl, same = step_both(g, o.state, ids[L], f"{name} cached length {L}")
        exact += same
        record(f"long_context_{name}", cached=L, rel_hidden=rh, rel_scores=rl, bit_identical=bool(same))
    assert exact >= len(LENGTHS) - 1, f"only {exact} of {len(LENGTHS)} long-context steps bit-identical"


@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_long_context_prefill_chunk_vs_oracle(name):
    """a prefill chunk whose positions straddle a V tile edge (the batched read writes K/V before its attention)"""
    path = synth.cached_gguf(name)
    e = nb.Engine(path, n_ctx=1100)
    o = oracle.Oracle(path, n_ctx=1100)
    g = e.new_state()
    ids = synth.random_ids(1040, e.n_vocab, 32)
    g.step_batch(tokens=ids[:1020], want_logits=False)
    import_memory(g, o.state)
    hg = g.step_batch(tokens=ids[1020:], want_logits=True, hidden_all=True)
    ho = o.state.step_batch(tokens=ids[1020:], want_logits=True, hidden_all=True)
    worst = max(rel(hg[i], ho[i]) for i in range(len(hg)))
    record(f"long_prefill_{name}", rel_hidden=worst, rel_scores=rel(g.logits, o.state.logits))
    assert worst <= TOL
    close(g.logits, o.state.logits, f"{name} prefill chunk at 1020..1039 scores")


def test_configs1_riding_equals_alone_seoul(seoul_path, record_property):
    """BASELINE configs[1]'s own check: riding gives each conversation exactly what running it alone gives."""
    e = nb.Engine(seoul_path, n_ctx=1024 + 128 + 16)
    a, b = e.new_state(), e.new_state()
    a.step_batch(synth.random_ids(1024, e.n_vocab, 1), want_logits=True)
    b.step_batch(synth.random_ids(256, e.n_vocab, 2), want_logits=True)
    a1, b1 = e.new_state(), e.new_state()
    a1.load(a.save())
    b1.load(b.save())
    # the oracle from A's memory at position 1024: its first greedy steps against the riding engine's
    o = oracle.Oracle(seoul_path, n_ctx=1024 + 16)
    import_memory(a, o.state)
    o.state.step(int(a.argmax()[0]))   # the oracle's own step at position 1024 needs the prompt's last pick
    ride = nb.greedy([a, b], 128)
    alone_a = nb.greedy([a1], 128)[:, 0]
    alone_b = nb.greedy([b1], 128)[:, 0]
    assert np.array_equal(ride[:, 0], alone_a) and np.array_equal(ride[:, 1], alone_b)
    assert a.pos == a1.pos == 1024 + 128 and b.pos == b1.pos == 256 + 128
    for x, y in ((a, a1), (b, b1)):
        assert same_bits(x.logits, y.logits) and same_bits(x.hidden, y.hidden)
        assert x.save() == y.save(), "riding and alone left different memory"
    record("configs1_riding_vs_alone", steps=128, identical=True)
    # the oracle's scores at position 1024 against the engine's first riding step (a's pick there is ride[0, 0])
    lo = o.state.logits
    assert int(np.argmax(lo)) == int(ride[0, 0]) or np.sort(lo)[-1] - np.sort(lo)[-2] <= 1e-4 * np.abs(lo).max()
    record_property("configs1_first_pick_oracle", int(np.argmax(lo)))


def test_configs1_steps_vs_oracle_seoul(seoul_path, record_property):
    """configs[1]'s conversation A at positions 1024..1031 against the oracle given its memory, then 8 greedy picks
    of the oracle's own loop beside the device's."""
    e = nb.Engine(seoul_path, n_ctx=1024 + 32)
    a = e.new_state()
    a.step_batch(synth.random_ids(1024, e.n_vocab, 1), want_logits=True)
    o = oracle.Oracle(seoul_path, n_ctx=1024 + 32)
    import_memory(a, o.state)
    worst = 0.0
    toks = synth.random_ids(4, e.n_vocab, 41)
    for k, t in enumerate(toks):
        rh, rl, _ = step_both(a, o.state, t, f"seoul configs[1] A position {1024 + k}")
        worst = max(worst, rl)
    ids = nb.greedy([a], 8)[:, 0]
    n, tie = follow_greedy(o.state, ids, "seoul configs[1] A greedy from 1028", record_property)
    record("configs1_A_vs_oracle", rel_scores_max=worst, greedy_identical=n, tie=tie)
    if tie is None:
        close(a.logits, o.state.logits, "seoul configs[1] A after 8 greedy steps")


def test_configs3_long_sessions_multi_equals_alone(seoul_path):
    """sessions with 1500-2048 cached positions (configs[3]'s upper range), several steps of all together equal each
    stepping alone, byte for byte; one of them against the oracle from its memory."""
    rng = np.random.default_rng(44)
    lens = [int(x) for x in rng.integers(1500, 2049, 6)]
    e = nb.Engine(seoul_path, n_ctx=2048 + 8, max_batch=8)
    multi = [e.new_state() for _ in lens]
    for i, (s, n) in enumerate(zip(multi, lens)):
        s.step_batch(synth.random_ids(n, e.n_vocab, 200 + i), want_logits=True)
    alone = []
    for s in multi:
        c = e.new_state()
        c.load(s.save())
        alone.append(c)
    o = oracle.Oracle(seoul_path, n_ctx=2048 + 8)
    import_memory(multi[0], o.state)
    for k in range(4):
        toks = np.array([s.argmax()[0] for s in multi], np.int32)
        nb.step_multi(multi, toks)
        for s, t in zip(alone, toks):
            s.step(int(t))
        if k == 0:
            o.state.step(int(toks[0]))
            r = close(multi[0].logits, o.state.logits, f"configs[3] session at {lens[0]} scores")
            record("configs3_session_vs_oracle", cached=lens[0], rel_scores=r,
                   bit_identical=same_bits(multi[0].logits, o.state.logits))
    for m, a in zip(multi, alone):
        assert m.pos == a.pos
        assert same_bits(m.logits, a.logits) and same_bits(m.hidden, a.hidden)
