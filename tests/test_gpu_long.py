"""Parity at the context lengths the benchmarks run (B200), against the oracle and against stepping alone.

* Long-context attention: at head_dim 64 the attention streams each kv head's cached K and then V rows through a
  ring of shared-memory slots of 256 positions (2-6 slots); at head_dim 128 it stages V in tiles of 256 positions, two
  in flight. Lengths just below, at and above a tile edge and several tiles long exercise the ring's refills and the
  partial last tiles. At each length the oracle is given exactly the
  engine's memory (checkpoint image: K/V caches, conv memory, position) and both take one step, bit for bit with the
  "cr" oracle (tests/parity.py), imi's own numbers ("libc") recorded (seoul.cpp:425-456, 589-621).
* configs[1] (BASELINE): the Seoul shape, conversation A after 1024 ids (seed 1), B after 256 (seed 2), 128 greedy
  steps riding (one table read for both): picks, scores, hidden states and memory byte-identical to running each
  alone; A's steps at positions 1024+ bit for bit the oracle's from its memory.
* sessions at contexts 1500-2048 stepped together equal stepping each alone, byte for byte, and one of them
  the oracle's from its memory."""
import numpy as np
import pytest

import nunchi_b200 as nb
import oracle
from nunchi_b200 import synth
from parity import follow_greedy, import_memory, paired_step, record, same_bits

pytestmark = pytest.mark.gpu

LENGTHS = (511, 512, 513, 1025, 2047)


@pytest.mark.parametrize("name", ["tiny", "wide_heads", "tiny_g2"])
def test_long_context_step_vs_oracle(name):
    """tiny: head_dim 64, full attention; wide_heads: head_dim 128, rope_freqs on the full layers, one layer with a
    window of 8 (window layers read only their last 8 positions at every length); tiny_g2: head_dim 64 with two query
    heads per kv head and a window of 8 on one layer."""
    path = synth.cached_gguf(name)
    n_ctx = 2304
    e = nb.Engine(path, n_ctx=n_ctx)
    cr, lc = oracle.Oracle(path, n_ctx=n_ctx, exp="cr"), oracle.Oracle(path, n_ctx=n_ctx)
    g = e.new_state()
    ids = synth.random_ids(n_ctx, e.n_vocab, 31)
    for L in LENGTHS:
        if L > g.pos:
            g.step_batch(tokens=ids[g.pos:L], want_logits=False)
        assert g.pos == L
        rh, rl = paired_step(g, cr.state, ids[L], where=f"{name} cached length {L}", libc=lc.state)
        record(f"long_context_{name}", cached=L, bit_exact_vs_cr=True, libc_rel_hidden=rh, libc_rel_scores=rl)


@pytest.mark.parametrize("name", ["tiny", "wide_heads"])
def test_long_context_prefill_chunk(name):
    """a batched read whose positions straddle a V tile edge (the batched read writes K/V before its attention): bit
    for bit the oracle's batched read from the same memory"""
    path = synth.cached_gguf(name)
    e = nb.Engine(path, n_ctx=1100)
    cr = oracle.Oracle(path, n_ctx=1100, exp="cr")
    g = e.new_state()
    ids = synth.random_ids(1040, e.n_vocab, 32)
    g.step_batch(tokens=ids[:1020], want_logits=False)
    import_memory(g, cr.state)
    hg = g.step_batch(tokens=ids[1020:], want_logits=True, hidden_all=True)
    ho = cr.state.step_batch(tokens=ids[1020:], want_logits=True, hidden_all=True)
    assert np.array_equal(hg.view(np.uint32), ho.view(np.uint32))
    assert same_bits(g.logits, cr.state.logits)
    record(f"long_prefill_{name}", bit_exact_vs_cr=True)


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
    o = oracle.Oracle(seoul_path, n_ctx=1024 + 16, exp="cr")
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
    # the oracle's pick at position 1024 against the engine's first riding step's (a's pick there is ride[0, 0])
    assert int(np.argmax(o.state.logits)) == int(ride[0, 0])
    record_property("configs1_first_pick_oracle", int(np.argmax(o.state.logits)))


def test_configs1_steps_vs_oracle_seoul(seoul_path, record_property):
    """configs[1]'s conversation A at positions 1024..1027 against the oracle given its memory, bit for bit ("cr"),
    imi's own numbers recorded ("libc"); then 8 greedy picks of the oracle's own loop beside the device's."""
    e = nb.Engine(seoul_path, n_ctx=1024 + 32)
    a = e.new_state()
    a.step_batch(synth.random_ids(1024, e.n_vocab, 1), want_logits=True)
    cr, lc = oracle.Oracle(seoul_path, n_ctx=1024 + 32, exp="cr"), oracle.Oracle(seoul_path, n_ctx=1024 + 32)
    worst_h, worst_s = 0.0, 0.0
    for k, t in enumerate(synth.random_ids(4, e.n_vocab, 41)):
        rh, rl = paired_step(a, cr.state, t, where=f"seoul configs[1] A position {1024 + k}", libc=lc.state)
        worst_h, worst_s = max(worst_h, rh), max(worst_s, rl)
    ids = nb.greedy([a], 8)[:, 0]
    n, _ = follow_greedy(cr.state, ids, "seoul configs[1] A greedy from 1028 vs cr", record_property)
    assert n == 8 and same_bits(a.logits, cr.state.logits)
    record("configs1_A_vs_oracle", bit_exact_vs_cr=True, libc_rel_hidden_max=worst_h, libc_rel_scores_max=worst_s)


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
    o = oracle.Oracle(seoul_path, n_ctx=2048 + 8, exp="cr")
    import_memory(multi[0], o.state)
    for k in range(4):
        toks = np.array([s.argmax()[0] for s in multi], np.int32)
        nb.step_multi(multi, toks)
        for s, t in zip(alone, toks):
            s.step(int(t))
        if k == 0:
            o.state.step(int(toks[0]))
            assert same_bits(multi[0].logits, o.state.logits) and same_bits(multi[0].hidden, o.state.hidden)
            record("configs3_session_vs_oracle", cached=lens[0], bit_exact_vs_cr=True)
    for m, a in zip(multi, alone):
        assert m.pos == a.pos
        assert same_bits(m.logits, a.logits) and same_bits(m.hidden, a.hidden)


def test_many_conversations_two_heads_per_group_equal_alone():
    """11 conversations decoded together (the batched attention with two query heads per kv head, one layer
    windowed) equal decoding each alone, byte for byte, at contexts on both sides of the window and of a ring slot"""
    path = synth.cached_gguf("tiny_g2")
    e = nb.Engine(path, n_ctx=640, max_batch=16)
    lens = [5, 9, 40, 255, 256, 257, 300, 511, 3, 120, 600]
    multi = [e.new_state() for _ in lens]
    alone = [e.new_state() for _ in lens]
    for i, L in enumerate(lens):
        ids = synth.random_ids(L, e.n_vocab, 40 + i)
        multi[i].step_batch(tokens=ids, want_logits=False)
        alone[i].step_batch(tokens=ids, want_logits=False)
    toks = np.stack([synth.random_ids(len(lens), e.n_vocab, 60 + k) for k in range(4)])
    for k in range(4):
        nb.step_multi(multi, toks[k])
        for i in range(len(lens)):
            alone[i].step(int(toks[k, i]))
    for m, a in zip(multi, alone):
        assert m.pos == a.pos
        assert np.array_equal(m.logits.view(np.uint32), a.logits.view(np.uint32))
        assert np.array_equal(m.hidden.view(np.uint32), a.hidden.view(np.uint32))


def test_batched_read_beyond_the_ring_vs_oracle():
    """a context so long (n_ctx 10,240, 4 query heads per kv head) that neither form of the batched attention fits its
    score rows in shared memory: the batched read runs the per-column attention over all its columns; the read and the
    next step bit for bit the oracle's"""
    path = synth.cached_gguf("tiny")
    n_ctx = 10240
    e = nb.Engine(path, n_ctx=n_ctx)
    cr = oracle.Oracle(path, n_ctx=n_ctx, exp="cr")
    g = e.new_state()
    ids = synth.random_ids(300, e.n_vocab, 33)
    hg = g.step_batch(tokens=ids[:290], want_logits=True, hidden_all=True)
    ho = cr.step_batch(tokens=ids[:290], want_logits=True, hidden_all=True)
    assert np.array_equal(hg.view(np.uint32), ho.view(np.uint32))
    assert same_bits(g.logits, cr.logits)
    g.step(int(ids[290]))
    cr.step(int(ids[290]))
    assert same_bits(g.logits, cr.logits)
    record("batched_read_beyond_ring_tiny", bit_exact_vs_cr=True)
