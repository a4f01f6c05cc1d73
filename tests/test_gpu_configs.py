"""The measurement configurations other than the benchmarked ones, as parity cases on the GPU (B200), at their full
sizes where the check does not need the oracle to run the whole model:

  * table sweep (N x K in {2048x2048, 8192x2048, 2048x8192, 97,496x2048}, 1 / 2 / 8 inputs): the 4-bit table kernel
    against the oracle, bit for bit (integer block dots are exact and the per-row float chain keeps imi's order);
  * prefill (400 input vectors ~ N(0,1)*0.5 then 16 word ids, read in chunks): the batched read gives bit for bit the
    hidden state and word scores that reading the same inputs one position at a time gives (imi's run_batch and
    run compute every position in the same float order, seoul.cpp:490-517 vs 352-357);
  * many sessions (64 conversations of different lengths on one GPU): one multi-session step gives every conversation
    exactly the bytes its own step gives.
Batch widths above 8 (32, 128) are read as several 8-wide groups by the engine; a tensor-core path for them is not
built."""
import numpy as np
import pytest

import nunchi_b200 as nb
import oracle
from nunchi_b200 import synth

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("rows,cols", [(2048, 2048), (8192, 2048), (2048, 8192), (97496, 2048)])
@pytest.mark.parametrize("ncol", [1, 2, 8])
def test_table_sweep_bit_exact(rows, cols, ncol):
    rng = np.random.default_rng(5)
    q4 = synth._q4_0(rng, rows, cols).reshape(-1)
    x = rng.standard_normal((ncol, cols)).astype(np.float32)
    cuts = [oracle.cut(v) for v in x]
    cq, cd, cs = (np.concatenate([c[k] for c in cuts]) for k in range(3))
    want = oracle.q4_matvec(q4, rows, cols, cq, cd, cs)
    got = nb.q4_matvec(q4, rows, cols, cq, cd, cs)
    assert np.array_equal(bits(got), bits(np.asarray(want, np.float32).reshape(got.shape)))


def test_prefill_equals_position_by_position(seoul_path):
    e = nb.Engine(seoul_path, n_ctx=448)
    rng = np.random.default_rng(3)
    vecs = (rng.standard_normal((400, e.n_embd)) * 0.5).astype(np.float32)
    ids = synth.random_ids(16, e.n_vocab, 3)
    batched, single = e.new_state(), e.new_state()
    batched.step_batch(embd=vecs, want_logits=False)
    batched.step_batch(tokens=ids, want_logits=True)
    for v in vecs:
        single.step(-1, v, want_logits=False)
    for k, t in enumerate(ids):
        single.step(int(t), want_logits=k == len(ids) - 1)
    assert batched.pos == single.pos == 416
    assert np.array_equal(bits(batched.hidden), bits(single.hidden))
    assert np.array_equal(bits(batched.logits), bits(single.logits))


def test_64_sessions_multi_step_equals_alone(seoul_path):
    e = nb.Engine(seoul_path, n_ctx=64, max_batch=64)
    rng = np.random.default_rng(4)
    lens = rng.integers(4, 33, size=64)
    multi = [e.new_state() for _ in range(64)]
    alone = [e.new_state() for _ in range(64)]
    for i, n in enumerate(lens):
        prompt = synth.random_ids(int(n), e.n_vocab, 100 + i)
        multi[i].step_batch(tokens=prompt, want_logits=True)
        alone[i].step_batch(tokens=prompt, want_logits=True)
    for k in range(3):
        toks = np.array([int(np.argmax(s.logits)) for s in multi], np.int32)
        nb.step_multi(multi, toks)
        for i in range(64):
            alone[i].step(int(toks[i]))
    for m, a in zip(multi, alone):
        assert m.pos == a.pos
        assert np.array_equal(bits(m.logits), bits(a.logits)) and np.array_equal(bits(m.hidden), bits(a.hidden))
