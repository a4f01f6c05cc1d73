"""Failure paths on the GPU (B200), made without faulting or hanging the device:

* a bounded device wait that runs out: a kernel waits on an mbarrier nothing completes (a flag nothing sets) with a
  short limit, gives up, reports IMI_E_TIMEOUT through the error flag and returns; the context stays usable;
* files the engine must refuse on the host before any kernel runs: a truncated GGUF (IMI_E_FILE), a table of a type
  the kernels do not read (IMI_E_FORMAT; imi's load fails the same way on a non-Q6_K word table, seoul.cpp:95-97);
* device allocation refused under a memory budget (IMI_CUDA_MAX_DEVICE_BYTES): load and new conversations fail with
  IMI_E_NOMEM and the engine keeps working with what it holds."""
import os
import subprocess
import sys
import time

import numpy as np
import pytest

import nunchi_b200 as nb
from nunchi_b200 import synth

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bounded_wait_gives_up_and_context_stays_usable():
    L = nb.lib()
    t0 = time.perf_counter()
    st = L.imi_cuda_check_wait_timeout(0, 50.0)
    dt = time.perf_counter() - t0
    assert st == 7, L.imi_cuda_error().decode()            # IMI_E_TIMEOUT
    assert "gave up" in L.imi_cuda_error().decode()
    assert dt < 10.0
    x = np.linspace(-2, 2, 256).astype(np.float32)         # the device still runs kernels afterwards
    q, d, s = nb.q8_cut(x)
    assert q.max() == 127 and q.min() == -127


def test_truncated_gguf_is_a_file_error(tmp_path, tiny_path):
    data = open(tiny_path, "rb").read()
    for cut in (100, len(data) // 2, len(data) - 7):
        p = tmp_path / f"cut{cut}.gguf"
        p.write_bytes(data[:cut])
        with pytest.raises(nb.ImiError) as ei:
            nb.Engine(str(p), n_ctx=16)
        assert ei.value.status == 2, str(ei.value)           # IMI_E_FILE
    with pytest.raises(nb.ImiError) as ei:
        nb.Engine(str(tmp_path / "missing.gguf"), n_ctx=16)
    assert ei.value.status == 2


def test_table_of_an_unread_type_is_a_format_error(tmp_path):
    s = synth.TINY
    f32 = np.zeros((s.n_embd, s.n_ff), np.float32)          # ffn_down as plain floats: not a 4-bit table
    p = synth.write_gguf(str(tmp_path / "f32down.gguf"), s, 0,
                         override={"blk.0.ffn_down.weight": (synth.GGML_F32, (s.n_ff, s.n_embd), f32)})
    with pytest.raises(nb.ImiError) as ei:
        nb.Engine(p, n_ctx=16)
    assert ei.value.status == 3 and "blk.0.ffn_down.weight" in str(ei.value)   # IMI_E_FORMAT


def test_device_memory_budget(tiny_path):
    """Run in a child process: the budget is read at load from the environment."""
    code = f"""
import os, sys
sys.path.insert(0, {ROOT!r})
import nunchi_b200 as nb
try:
    nb.Engine({tiny_path!r}, n_ctx=64)
    sys.exit("loaded within a 1 MB budget")
except nb.ImiError as ex:
    assert ex.status == 6 and "IMI_CUDA_MAX_DEVICE_BYTES" in str(ex), ex
os.environ["IMI_CUDA_MAX_DEVICE_BYTES"] = str(64 << 20)
e = nb.Engine({tiny_path!r}, n_ctx=64)
states = []
try:
    for _ in range(100000):
        states.append(e.new_state())
    sys.exit("no state was refused")
except nb.ImiError as ex:
    assert ex.status == 6, ex
assert len(states) >= 1
states[0].step(1)                    # the engine keeps working with what it holds
assert states[0].pos == 1
del states[-1]
states.append(e.new_state())         # freeing one makes room for one
print("ok", len(states))
"""
    env = dict(os.environ, IMI_CUDA_MAX_DEVICE_BYTES=str(1 << 20))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
