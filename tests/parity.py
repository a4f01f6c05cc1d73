"""Shared checks of the parity tests (engine on the GPU against the oracle, the C restatement of imi's step that
tests/test_oracle.py pins bit for bit to the reference's own code).

Tolerance (north star): word scores and hidden states within TOL = 1e-3 of max|value| (max-abs relative). The engine
keeps imi's float order everywhere, so most steps are bit-identical; the one operation that can differ is expf
(correctly rounded on the device, glibc's differs on ~0.06% of inputs). A 1-ulp difference there can move one 8-bit
activation code by one step (1/127 of its block's maximum), which then stays in the attention cache.
Greedy picks are identical except at logged ties (oracle's top two scores within TIE = 1e-4 of max|score|)."""
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
