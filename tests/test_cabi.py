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


def test_model_file_keys_and_tensors(tiny_path):
    """The model file beside the brain (imi_file, imi/model.h:17-36): keys, arrays and tensor headers of the GGUF through
    the library's reader, no device needed."""
    L = nb.lib()
    L.imi_cuda_file_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    for f in ("imi_cuda_file_find_key", "imi_cuda_file_n_keys"):
        getattr(L, f).restype = C.c_int64
    L.imi_cuda_file_find_key.argtypes = [C.c_void_p, C.c_char_p]
    L.imi_cuda_file_key_type.argtypes = [C.c_void_p, C.c_int64]
    L.imi_cuda_file_key_data.argtypes = [C.c_void_p, C.c_int64]
    L.imi_cuda_file_key_data.restype = C.c_void_p
    L.imi_cuda_file_key_str.argtypes = [C.c_void_p, C.c_int64]
    L.imi_cuda_file_key_str.restype = C.c_char_p
    L.imi_cuda_file_arr_n.argtypes = [C.c_void_p, C.c_int64]
    L.imi_cuda_file_arr_n.restype = C.c_uint64
    L.imi_cuda_file_arr_data.argtypes = [C.c_void_p, C.c_int64]
    L.imi_cuda_file_arr_data.restype = C.c_void_p
    L.imi_cuda_file_tensor.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int64),
                                       C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    L.imi_cuda_file_close.argtypes = [C.c_void_p]
    h = C.c_void_p()
    assert L.imi_cuda_file_open(b"/nonexistent.gguf", C.byref(h)) == 2     # IMI_E_FILE
    assert L.imi_cuda_file_open(tiny_path.encode(), C.byref(h)) == 0
    s = synth.TINY
    k = L.imi_cuda_file_find_key(h, b"lfm3.block_count")
    assert k >= 0 and L.imi_cuda_file_key_type(h, k) == 4
    assert C.cast(L.imi_cuda_file_key_data(h, k), C.POINTER(C.c_uint32))[0] == s.n_layer
    assert L.imi_cuda_file_key_str(h, L.imi_cuda_file_find_key(h, b"general.architecture")) == b"lfm3"
    k = L.imi_cuda_file_find_key(h, b"lfm3.attention.sliding_window_pattern")
    assert L.imi_cuda_file_arr_n(h, k) == s.n_layer
    pat = C.cast(L.imi_cuda_file_arr_data(h, k), C.POINTER(C.c_uint8))
    assert [pat[i] for i in range(s.n_layer)] == [int(il in s.swa_layers) for il in range(s.n_layer)]
    assert L.imi_cuda_file_find_key(h, b"no.such.key") == -1
    ty, ne, d, nbytes = C.c_int(), (C.c_int64 * 4)(), C.c_void_p(), C.c_size_t()
    assert L.imi_cuda_file_tensor(h, b"token_embd.weight", C.byref(ty), ne, C.byref(d), C.byref(nbytes)) == 0
    assert ty.value == 2 and list(ne)[:2] == [s.n_embd, s.n_vocab] and nbytes.value == s.n_vocab * s.n_embd // 32 * 18
    assert L.imi_cuda_file_tensor(h, b"missing.weight", None, None, None, None) == -1
    L.imi_cuda_file_close(h)


def test_drop_in_headers_compile():
    """The reference's headers' names on the engine (include/drop_in: seoul.h, brain.h, model.h), no ggml needed."""
    src = ('#include "seoul.h"\n#include "brain.h"\n#include "model.h"\n'
           'int main() { imi_seoul s; imi_brain b; imi_file f; (void) f.key_i("x", 0);\n'
           '  return s.n_embd + b.n_vocab + (int) s.t_tables + (int) s.t_sync + (int) s.t_attn; }\n')
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-I",
                        os.path.join(ROOT, "include", "drop_in"), "-I", os.path.join(ROOT, "include"), "-x", "c++",
                        "-"], input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    exe = os.path.join(ROOT, "oracle", "_ref", "seoul_check_cuda")
    if os.path.exists(exe):   # the reference's check tool, unmodified, linked to the engine: runs without a device
        r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
        assert r.returncode == 1 and "usage: imi-seoul-check" in r.stderr
