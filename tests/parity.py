"""Shared checks of the parity tests (engine on the GPU against the oracle, the C restatement of imi's step that
tests/test_oracle.py pins bit for bit to the reference's own code).

The engine keeps imi's float order everywhere. The one operation whose rounding it does not share is expf: imi calls
the C library's expf, the engine computes the correctly rounded exponential (they differ on ~0.06% of inputs). The
oracle comes in two builds (oracle.Oracle(exp=...)): "libc" calls the C library's expf and is the reference bit for bit;
"cr" uses the correctly rounded exponential and is otherwise the same code. Hence:
  * against the "cr" oracle the engine is bit-exact: every step from identical memory (paired_step: the oracle is given
    the engine's K/V caches, conv memory and position from its checkpoint image) and whole free-running sequences;
  * against the "libc" oracle (= imi) a 1-ulp expf difference can move one 8-bit activation code by one step (1/127 of
    its block's maximum), which then stays in the attention cache and the conv memory. That difference is imi's own
    expf against the correctly rounded one; it is recorded per step, and the north star's bound holds at every
    position: against the reference's fp64 truth key the engine's max-abs error (relative to max|truth|) is at most
    imi's own plus TOL = 1e-3; greedy picks are identical except at logged ties (the top two scores within TIE = 1e-4
    of max|score|)."""
from __future__ import annotations

import json
import os
import warnings

import numpy as np

TOL = 1e-3
TIE = 1e-4
LOG = os.environ.get("IMI_PARITY_LOG")   # optional JSON-lines file receiving every recorded parity figure


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def rel(a, b):
    """max-abs difference relative to max|b|"""
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(float(np.abs(b).max()), 1e-30))


def same_bits(a, b) -> bool:
    return np.array_equal(bits(a), bits(b))


def record(what: str, **kv):
    """A parity figure worth keeping: appended to IMI_PARITY_LOG when set (the GPU runs set it)."""
    if LOG:
        with open(LOG, "a") as f:
            f.write(json.dumps({"test": what, **kv}) + "\n")


def is_tie(scores) -> bool:
    top2 = np.sort(scores)[-2:]
    return bool(top2[1] - top2[0] <= TIE * np.abs(scores).max())


def close(got, want, where: str, tol: float = TOL) -> float:
    r = rel(got, want)
    assert r <= tol, f"{where}: differs by {r:.3g} of max (tolerance {tol})"
    return r


def follow_greedy(o, ids, where: str, record_property=None):
    """Run the oracle's greedy loop beside the device's picks: step k reads the previous pick (the first step reads
    the pick after the prompt) and ids[k] is the pick step k makes. Every pick must match the oracle's, except where
    the oracle's top two scores are within TIE of max|score| (a tie: the paths may part there; the comparison stops).
    Returns (picks compared and identical, tie position or None); a tie is reported as a warning, recorded with
    record_property when given, and in IMI_PARITY_LOG."""
    t = int(np.argmax(o.logits))
    for k, got in enumerate(ids):
        o.step(t)
        lo = o.logits
        t = int(np.argmax(lo))
        if int(got) != t:
            assert is_tie(lo), f"{where}: greedy pick {k}: device {int(got)}, oracle {t}, not a tie"
            top2 = np.sort(lo)[-2:]
            msg = f"{where}: greedy picks identical for {k} steps, then a near-tie (gap {top2[1] - top2[0]:.3g})"
            warnings.warn(msg)
            if record_property:
                record_property("greedy_tie", msg)
            record(where, identical=k, tie_at=k, steps=len(ids))
            return k, k
    record(where, identical=len(ids), tie_at=None, steps=len(ids))
    if record_property:
        record_property("greedy_identical", len(ids))
    return len(ids), None


def import_memory(state, o_state):
    """Give the oracle conversation o_state exactly the engine conversation's memory (position, K/V caches, conv
    memory), read from the engine's checkpoint image, so one step of each starts from identical memory."""
    m = state.unpack()
    o_state.import_memory(m["pos"], m["k"], m["v"], m["conv"])
    return m["pos"]


def paired_step(g, o_state, token=-1, embd=None, want_logits=True, where="step", libc=None):
    """One step of the engine state g and the "cr" oracle state o_state from identical memory (the engine's, imported
    into the oracle first): hidden state and (when wanted) scores bit for bit. With libc (a "libc" oracle state, i.e.
    imi's own float results) the same step is taken there too and its max-abs relative difference recorded.
    Returns (rel hidden vs libc, rel scores vs libc) (zeros without libc)."""
    import_memory(g, o_state)
    if libc is not None:
        import_memory(g, libc)
    g.step(int(token), embd, want_logits)
    o_state.step(int(token), embd, want_logits)
    assert same_bits(g.hidden, o_state.hidden), f"{where}: hidden state differs ({rel(g.hidden, o_state.hidden):.3g})"
    if want_logits:
        assert same_bits(g.logits, o_state.logits), f"{where}: scores differ ({rel(g.logits, o_state.logits):.3g})"
    if libc is None:
        return 0.0, 0.0
    libc.step(int(token), embd, want_logits)
    return rel(g.hidden, libc.hidden), (rel(g.logits, libc.logits) if want_logits else 0.0)
