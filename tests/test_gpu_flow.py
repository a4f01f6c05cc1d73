"""The riding caller (include/imi_flow_cuda.h, flow.cpp:114-126's step order): a voice conversation stepping frames
beside a text conversation stepping greedy words, each word riding a frame's step when both have work. The C++
program tests/flow_check.cpp runs it through the C-ABI with riding on and off and checks the two agree bit for bit;
here its text picks are also replayed on the oracle."""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle
from nunchi_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "nunchi_b200")


def build_flow_check(tmp_path) -> str:
    exe = str(tmp_path / "flow_check")
    r = subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "flow_check.cpp"), "-o", exe, "-L", LIBDIR, "-limi_cuda",
                        "-Wl,-rpath," + LIBDIR], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_flow_caller_compiles_and_links(tmp_path):
    """The caller header and its check program build against the engine library (no device needed)."""
    assert os.path.exists(build_flow_check(tmp_path))


@pytest.mark.gpu
def test_flow_riding_equals_alone_and_oracle(tmp_path, tiny_path):
    exe = build_flow_check(tmp_path)
    cap1, cap2, frames = 14, 10, 30
    r = subprocess.run([exe, tiny_path, str(frames), str(cap1), str(cap2), "5"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["same"]
    # riding: every text word while the voice speaks rides a frame (30 frames, 24 words: all but the voice's last 6)
    assert out["ride"]["shared"] == min(frames, cap1 + cap2) and out["alone"]["shared"] == 0
    assert out["ride"]["shared"] + out["ride"]["voice_alone"] == frames == out["alone"]["voice_alone"]
    assert out["alone"]["text_alone"] == cap1 + cap2
    # the text conversation's picks against the oracle's greedy loop (prompt, cap1 words, re-prompt, cap2 words)
    picks = out["picks"]
    assert len(picks) == cap1 + cap2
    _, text_prompt, re_prompt = out["prompts"]
    o = oracle.Oracle(tiny_path, n_ctx=128, exp="cr")   # the engine's exponential: every pick identical
    at = 0
    for prompt, cap in ((text_prompt, cap1), (re_prompt, cap2)):
        s = o.new_state()
        s.step_batch(tokens=np.array(prompt, np.int32), want_logits=True)
        for k in range(cap):
            t = int(np.argmax(s.logits))
            assert picks[at + k] == t, f"pick {at + k}: flow {picks[at + k]} oracle {t}"
            s.step(t)
        at += cap
