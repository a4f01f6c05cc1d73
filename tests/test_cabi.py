"""The drop-in boundary on CPU: the engine library loads, exports exactly what include/imi_cuda.h declares, and
refuses work cleanly where there is no GPU (no CPU fallback). No compute call runs here."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import nunchi_b200 as nb
from nunchi_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "imi_cuda.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(imi_cuda_[a-z0-9_]+)\s*\(", src)))


def has_gpu():
    try:
        return subprocess.run(["nvidia-smi", "-L"], capture_output=True, timeout=20).returncode == 0
    except Exception:
        return False


def test_library_exports_every_declared_symbol():
    lib = nb.lib()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"{n} declared in imi_cuda.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", nb.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (imi_cuda_[a-z0-9_]+)", out)))
    assert exported == names, "the library exports symbols the header does not declare (or the reverse)"


def test_cpp_wrapper_header_compiles():
    src = "#include \"imi_seoul_cuda.h\"\nint main() { imi_seoul b; return b.n_embd; }\n"
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.join(ROOT, "include"), "-x", "c++", "-"],
                       input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_no_device_is_an_error_not_a_fallback(tiny_path):
    with pytest.raises(nb.ImiError) as ei:
        nb.Engine(tiny_path)
    assert ei.value.status == 8                      # IMI_E_NODEV
    with pytest.raises(nb.ImiError):
        nb.q8_cut(np.zeros(64, np.float32))
    assert nb.lib().imi_cuda_error()


def test_argument_errors_before_any_device_work():
    L = nb.lib()
    h = C.c_void_p()
    assert L.imi_cuda_load(b"/nonexistent.gguf", 0, 64, 1, None) == 1      # IMI_E_ARG: out is null
    assert L.imi_cuda_get_info(None, None) == 1
    assert L.imi_cuda_step(None, 0, None, 1) == 1
    assert L.imi_cuda_step2(None, 0, None, 1, None, 0, None, 1) == 1
    assert L.imi_cuda_step_multi(None, 0, None, None, None) == 1
    assert L.imi_cuda_step_batch(None, None, None, 0, 0, None) == 1
    assert L.imi_cuda_greedy(None, 0, None, 0, None) == 1
    assert L.imi_cuda_state_pos(None) == -1
    assert L.imi_cuda_launches_per_step(None, 1, 1) == 0
    assert L.imi_cuda_q4_matvec(0, None, 8, 256, None, None, None, 1, None, None) == 1
    assert L.imi_cuda_q4_matvec(0, b"x", 8, 100, b"x", b"x", b"x", 1, b"x", None) == 1   # width not / 256
    del h


def test_synthetic_model_reads_with_the_gguf_package(tiny_path):
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(tiny_path)
    names = {t.name for t in r.tensors}
    s = synth.TINY
    assert "token_embd.weight" in names and "output_norm.weight" in names
    for il in range(s.n_layer):
        key = "attn_q.weight" if s.is_attn(il) else "shortconv.in_proj.weight"
        assert f"blk.{il}.{key}" in names
    f = r.fields["lfm3.block_count"]
    assert int(f.parts[f.data[0]][0]) == s.n_layer


def test_synthetic_model_is_deterministic(tmp_path):
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    synth.write_gguf(str(a), synth.TINY, seed=0)
    synth.write_gguf(str(b), synth.TINY, seed=0)
    assert a.read_bytes() == b.read_bytes()
    synth.write_gguf(str(b), synth.TINY, seed=1)
    assert a.read_bytes() != b.read_bytes()
