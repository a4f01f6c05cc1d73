"""Drop-in on the GPU (B200): the reference's own callers of imi's brain, compiled against the engine.

* imi/core/seoul_check.cpp, the reference's truth-key check tool, unmodified (oracle/Makefile compiles a byte-for-byte
  copy against include/drop_in, so its `#include "seoul.h"` is the engine's imi_seoul), run on the fp64 truth key of
  the reference's ref_exact.py (tests/golden) beside the same tool on the reference's own CPU brain (oracle/_ref): the
  same "same next word" count and, per position, errors against the truth key within 1e-3 of imi's own
  (seoul_check.cpp:17-43); with IMI_DUMP the engine's answers are the oracle's ("cr" build) bit for bit.
* imi_brain (brain.h:33-64) through include/drop_in/brain.h: the same numbers, and the model file's keys through
  brain.f with the gguf accessors the tokenizer uses."""
import os
import re
import struct
import subprocess

import numpy as np
import pytest

import oracle
from nunchi_b200 import synth
from parity import same_bits

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
GOLD = os.path.join(ROOT, "tests", "golden")


def write_key(path, tokens, hidden, logits):
    """imi's REF.bin layout (imi/ref/ref_llama.cpp:5)"""
    with open(path, "wb") as f:
        f.write(struct.pack("3i", hidden.shape[1], logits.shape[1], len(tokens)))
        for i, t in enumerate(tokens):
            f.write(struct.pack("i", int(t)))
            f.write(np.asarray(hidden[i], np.float32).tobytes())
            f.write(np.asarray(logits[i], np.float32).tobytes())


def read_key(path):
    with open(path, "rb") as f:
        ne, nv, n = struct.unpack("3i", f.read(12))
        T, H, L = [], [], []
        for _ in range(n):
            T.append(struct.unpack("i", f.read(4))[0])
            H.append(np.frombuffer(f.read(4 * ne), np.float32))
            L.append(np.frombuffer(f.read(4 * nv), np.float32))
    return np.array(T), np.array(H), np.array(L)


CHECK = re.compile(r"check: (\d+) positions, hidden error mean ([\d.e+-]+) max ([\d.e+-]+), score error mean "
                   r"([\d.e+-]+) max ([\d.e+-]+), same next word (\d+)/(\d+)")


def run_check(exe, model, key, env=None):
    r = subprocess.run([exe, model, key, "16"], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, IMI_REPS="1", **(env or {})))
    assert r.returncode == 0, r.stdout + r.stderr
    m = CHECK.search(r.stdout)
    assert m, r.stdout
    return [float(x) for x in m.groups()], r.stdout


@pytest.mark.parametrize("name", ["tiny", "seoul"])
def test_reference_check_tool_on_the_engine(name, tmp_path, record_property):
    exe_gpu, exe_cpu = os.path.join(REF, "seoul_check_cuda"), os.path.join(REF, "seoul_check_ref")
    if not (os.path.exists(exe_gpu) and os.path.exists(exe_cpu)):
        pytest.skip("the check tool builds where the reference tree is (oracle/Makefile)")
    t = np.load(os.path.join(GOLD, f"truth_{name}.npz"))
    n = len(t["logits_full"])
    key = str(tmp_path / "REF.bin")
    write_key(key, t["tokens"][:n], t["hidden"][:n], t["logits_full"][:n])
    model = synth.cached_gguf(name)
    dump = str(tmp_path / "dump.bin")
    gpu, out_gpu = run_check(exe_gpu, model, key, {"IMI_DUMP": dump})
    cpu, out_cpu = run_check(exe_cpu, model, key)
    record_property("check_engine", out_gpu.strip().splitlines()[-3:])
    record_property("check_imi", out_cpu.strip().splitlines()[-3:])
    assert gpu[0] == cpu[0] == n
    assert gpu[5] == cpu[5], f"same next word: engine {gpu[5]}, imi {cpu[5]}"
    for k, what in ((1, "hidden mean"), (2, "hidden max"), (3, "score mean"), (4, "score max")):
        assert gpu[k] - cpu[k] <= 1e-3, f"{what}: engine {gpu[k]:.4g}, imi {cpu[k]:.4g}"
    # IMI_DUMP: the engine's own answers, position by position, against the oracle with the engine's exponential
    toks, H, L = read_key(dump)
    o = oracle.Oracle(model, n_ctx=64, exp="cr")
    for i, tk in enumerate(toks):
        o.step(int(tk))
        assert same_bits(H[i], o.hidden) and same_bits(L[i], o.logits), f"dumped answer {i}"


def test_imi_brain_drop_in(tmp_path, tiny_path):
    exe = str(tmp_path / "dropin_brain")
    lib = os.path.join(ROOT, "nunchi_b200")
    r = subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror",
                        "-I", os.path.join(ROOT, "include", "drop_in"), "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "dropin_brain.cpp"), "-o", exe, "-L", lib, "-limi_cuda",
                        "-Wl,-rpath," + lib], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    toks = synth.random_ids(12, 1003, 51)
    out = str(tmp_path / "brain.bin")
    r = subprocess.run([exe, tiny_path, out, *map(str, toks)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    s = synth.TINY
    assert f'"blocks": {s.n_layer}, "pattern": {s.n_layer}, "embd_rows": {s.n_vocab}, "n_embd": {s.n_embd}' in r.stdout
    got_t, H, L = read_key(out)
    assert list(got_t) == [int(x) for x in toks]
    o = oracle.Oracle(tiny_path, n_ctx=64, exp="cr")
    for i, tk in enumerate(toks):
        o.step(int(tk))
        assert same_bits(H[i], o.hidden) and same_bits(L[i], o.logits), f"position {i}"
