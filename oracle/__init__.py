"""The oracle: CPU checkers for the decode path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline import this package; the engine never does.

* `Oracle`   - the C restatement of imi's brain step (imi_oracle.c -> liboracle.so), float order identical to imi's
               AVX2 code.
* `Reference`- the reference's own imi/core/seoul.cpp + tables.cpp compiled unmodified against a small ggml/gguf
               shim (oracle/_ref/libimi_ref.so; built where the reference tree exists, then shipped with the repo
               snapshot).
Both expose the imi_seoul surface used by the tests: load / reset / step / step2 / step_batch / hidden / logits.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_fp = C.POINTER(C.c_float)


def _lib(name: str):
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
    return C.CDLL(path)


def _arr(x, dtype):
    return None if x is None else np.ascontiguousarray(x, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Oracle:
    """imi's step restated in C (liboracle.so). exp="cr": the build whose exponential is correctly rounded
    (liboracle_cr.so) in place of the C library's expf, the only operation in which the engine may differ from imi."""

    _libs = {}

    @classmethod
    def lib(cls, exp: str = "libc"):
        if exp not in cls._libs:
            L = _lib({"libc": "liboracle.so", "cr": "liboracle_cr.so"}[exp])
            L.or_load.restype = C.c_void_p
            L.or_load.argtypes = [C.c_char_p, C.c_int, C.c_int]
            L.or_error.restype = C.c_char_p
            L.or_free.argtypes = [C.c_void_p]
            L.or_info.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
            L.or_state_new.restype = C.c_void_p
            L.or_state_new.argtypes = [C.c_void_p]
            L.or_state_free.argtypes = [C.c_void_p]
            L.or_state_reset.argtypes = [C.c_void_p, C.c_void_p]
            L.or_state_pos.argtypes = [C.c_void_p]
            for f in ("or_hidden", "or_logits", "or_conv_state"):
                getattr(L, f).restype = _fp
            L.or_hidden.argtypes = [C.c_void_p]
            L.or_logits.argtypes = [C.c_void_p]
            L.or_conv_state.argtypes = [C.c_void_p, C.c_int]
            for f in ("or_k_cache", "or_v_cache"):
                getattr(L, f).restype = C.POINTER(C.c_uint16)
                getattr(L, f).argtypes = [C.c_void_p, C.c_int]
            L.or_state_import.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            L.or_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_int]
            L.or_step_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
            L.or_rms_scale.restype = C.c_float
            L.or_rms_scale.argtypes = [C.c_void_p, C.c_int, C.c_float]
            L.or_cut.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            L.or_block_dots.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
            L.or_q4_matvec.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_void_p, C.c_int]
            L.or_f2h.restype = C.c_uint16
            L.or_f2h.argtypes = [C.c_float]
            L.or_h2f.restype = C.c_float
            L.or_h2f.argtypes = [C.c_uint16]
            L.or_rope_angles.argtypes = [C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p]
            cls._libs[exp] = L
        return cls._libs[exp]

    def __init__(self, path: str, n_ctx: int = 512, threads: int = 0, exp: str = "libc"):
        self.L = L = self.lib(exp)
        self.h = L.or_load(path.encode(), n_ctx, threads or os.cpu_count() or 1)
        if not self.h:
            raise RuntimeError(f"oracle load failed: {L.or_error().decode()}")
        info = (C.c_int * 10)()
        L.or_info(self.h, info)
        (self.n_embd, self.n_vocab, self.n_ctx, self.n_layer, self.n_head, self.n_head_kv, self.head_dim, self.n_ff,
         self.d_conv, self.n_attn) = list(info)
        self.state = self.new_state()

    def new_state(self):
        return OracleState(self)

    def __del__(self):
        try:
            self.state = None
            self.L.or_free(self.h)
        except Exception:
            pass

    # the brain's own conversation (imi_seoul keeps one as its own)
    def reset(self):
        self.state.reset()

    @property
    def pos(self):
        return self.state.pos

    def step(self, token: int = -1, embd=None, want_logits: bool = True) -> int:
        return self.state.step(token, embd, want_logits)

    def step_batch(self, tokens=None, embd=None, want_logits=True, hidden_all=False):
        return self.state.step_batch(tokens, embd, want_logits, hidden_all)

    def step2(self, token_a, embd_a, logits_a, b: "OracleState", token_b, embd_b, logits_b):
        """imi's riding step: each conversation gets exactly the numbers its own step() gives (seoul.cpp:222-224)."""
        if self.state.pos >= self.n_ctx or b.pos >= self.n_ctx:
            return 1
        self.state.step(token_a, embd_a, logits_a)
        b.step(token_b, embd_b, logits_b)
        return 0

    @property
    def hidden(self):
        return self.state.hidden

    @property
    def logits(self):
        return self.state.logits


class OracleState:
    def __init__(self, m: Oracle):
        self.m, self.L = m, m.L
        self.h = self.L.or_state_new(m.h)

    def __del__(self):
        try:
            self.L.or_state_free(self.h)
        except Exception:
            pass

    def reset(self):
        self.L.or_state_reset(self.m.h, self.h)

    @property
    def pos(self):
        return self.L.or_state_pos(self.h)

    def step(self, token=-1, embd=None, want_logits=True):
        e = _arr(embd, np.float32)
        return self.L.or_step(self.m.h, self.h, int(token), _ptr(e), int(bool(want_logits)))

    def step_batch(self, tokens=None, embd=None, want_logits=True, hidden_all=False):
        t, e = _arr(tokens, np.int32), _arr(embd, np.float32)
        n = len(t) if t is not None else e.shape[0]
        ha = np.zeros((n, self.m.n_embd), np.float32) if hidden_all else None
        rc = self.L.or_step_batch(self.m.h, self.h, _ptr(t), _ptr(e), n, int(bool(want_logits)), _ptr(ha))
        if rc:
            raise RuntimeError("context full")
        return ha

    @property
    def hidden(self):
        return np.ctypeslib.as_array(self.L.or_hidden(self.h), (self.m.n_embd,)).copy()

    @property
    def logits(self):
        return np.ctypeslib.as_array(self.L.or_logits(self.h), (self.m.n_vocab,)).copy()

    def k_cache(self, ai):
        kvd = self.m.n_head_kv * self.m.head_dim
        return np.ctypeslib.as_array(self.L.or_k_cache(self.h, ai), (self.m.n_ctx, kvd)).copy()

    def v_cache(self, ai):
        kvd = self.m.n_head_kv * self.m.head_dim
        return np.ctypeslib.as_array(self.L.or_v_cache(self.h, ai), (self.m.n_ctx, kvd)).copy()

    def conv_state(self, il):
        return np.ctypeslib.as_array(self.L.or_conv_state(self.h, il), (self.m.d_conv, self.m.n_embd)).copy()

    def import_memory(self, pos, k, v, conv):
        """Start from another implementation's memory: position, K/V caches [n_attn][pos][kvd] (fp16 bits) and conv
        memory [n_conv][d_conv][n_embd] (oldest tap first), e.g. the engine's checkpoint (nunchi_b200 State.unpack)."""
        k, v = np.ascontiguousarray(k, np.uint16), np.ascontiguousarray(v, np.uint16)
        conv = np.ascontiguousarray(conv, np.float32)
        if self.L.or_state_import(self.m.h, self.h, int(pos), _ptr(k), _ptr(v), _ptr(conv)):
            raise ValueError("position beyond the oracle's n_ctx")


# ---- kernel-level pieces (module functions over the C restatement) ----

def cut(x):
    """imi_q8::from: int8 codes, fp32 scale and scale*sum per 32 values."""
    L = Oracle.lib()
    x = _arr(x, np.float32)
    n = x.size
    q, d, s = np.zeros(n, np.int8), np.zeros(n // 32, np.float32), np.zeros(n // 32, np.float32)
    L.or_cut(_ptr(x), n, _ptr(q), _ptr(d), _ptr(s))
    return q, d, s


def rms_scale(x, eps=1e-5):
    x = _arr(x, np.float32)
    return float(Oracle.lib().or_rms_scale(_ptr(x), x.size, eps))


def block_dots(q4: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    out = np.zeros((rows, cols // 32), np.int32)
    q4, xq = _arr(q4, np.uint8), _arr(xq, np.int8)
    Oracle.lib().or_block_dots(_ptr(q4), rows, cols, _ptr(xq), _ptr(out))
    return out


def q4_matvec(q4, rows, cols, xq, xd, xs, threads=0) -> np.ndarray:
    """imi_q4_group per row for ncol = len(xq) // cols inputs: out[ncol][rows]."""
    q4, xq, xd, xs = _arr(q4, np.uint8), _arr(xq, np.int8), _arr(xd, np.float32), _arr(xs, np.float32)
    ncol = xq.size // cols
    out = np.zeros((ncol, rows), np.float32)
    Oracle.lib().or_q4_matvec(_ptr(q4), rows, cols, _ptr(xq), _ptr(xd), _ptr(xs), ncol, _ptr(out),
                              threads or os.cpu_count() or 1)
    return out


def f2h(x: float) -> int:
    return int(Oracle.lib().or_f2h(float(x)))


def rope_angles(pos: int, n: int, base: float, freq_factor=None):
    ff = _arr(freq_factor, np.float32)
    cs, sn = np.zeros(n // 2, np.float32), np.zeros(n // 2, np.float32)
    Oracle.lib().or_rope_angles(pos, n, base, _ptr(ff), _ptr(cs), _ptr(sn))
    return cs, sn


# ---- the Q6_K word table of the product's own files (imi_q8k / imi_q6k_row / imi_q6k_dequant_row) ----

def _q6k_lib(L, prefix):
    f = getattr(L, prefix + "q6k_row")
    if not getattr(f, "_typed", False):
        if prefix == "or_":
            L.or_q8k_from.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            L.or_q6k_row.restype = C.c_float
            L.or_q6k_row.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
            L.or_q6k_dequant_row.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        else:
            L.oref_q8k_from.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            L.oref_q6k_row.restype = C.c_float
            L.oref_q6k_row.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
            L.oref_q6k_dequant_row.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        f._typed = True
    return L


def q8k_from(x, reference: bool = False):
    """imi_q8k::from: int8 codes, an fp32 scale per 256 values and the code sum of every 16 (restatement, or the
    reference's own function with reference=True)."""
    x = _arr(x, np.float32)
    n = x.size
    q, d, bs = np.zeros(n, np.int8), np.zeros(n // 256, np.float32), np.zeros(n // 16, np.int16)
    if reference:
        _q6k_lib(Reference.lib(), "oref_").oref_q8k_from(_ptr(x), n, _ptr(q), _ptr(d), _ptr(bs))
    else:
        _q6k_lib(Oracle.lib(), "or_").or_q8k_from(_ptr(x), n, _ptr(q), _ptr(d), _ptr(bs))
    return q, d, bs


def q6k_rows(rows_q6k, x, reference: bool = False) -> np.ndarray:
    """The word scores of Q6_K rows ([rows][cols/256 * 210] bytes) for the input x (cut by imi_q8k::from inside), in
    imi's AVX2 order (tables.cpp:235-278): the restatement, or the reference's own imi_q6k_row."""
    rows_q6k, x = _arr(rows_q6k, np.uint8), _arr(x, np.float32)
    nbk = x.size // 256
    out = np.zeros(rows_q6k.shape[0], np.float32)
    if reference:
        L = _q6k_lib(Reference.lib(), "oref_")
        for r in range(rows_q6k.shape[0]):
            out[r] = L.oref_q6k_row(_ptr(rows_q6k[r]), _ptr(x), nbk)
    else:
        L = _q6k_lib(Oracle.lib(), "or_")
        q, d, bs = q8k_from(x)
        for r in range(rows_q6k.shape[0]):
            out[r] = L.or_q6k_row(_ptr(rows_q6k[r]), _ptr(q), _ptr(d), _ptr(bs), nbk)
    return out


def q6k_dequant_row(row, nblocks: int, reference: bool = False) -> np.ndarray:
    """A Q6_K row as floats (the word lookup, tables.cpp:216-233)."""
    row = _arr(row, np.uint8)
    y = np.zeros(256 * nblocks, np.float32)
    if reference:
        _q6k_lib(Reference.lib(), "oref_").oref_q6k_dequant_row(_ptr(row), _ptr(y), nblocks)
    else:
        _q6k_lib(Oracle.lib(), "or_").or_q6k_dequant_row(_ptr(row), _ptr(y), nblocks)
    return y


# ---- the reference's own code ----

def reference_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libimi_ref.so"))


class Reference:
    """imi_seoul from the reference's seoul.cpp + tables.cpp (oracle/_ref/libimi_ref.so)."""

    _L = None
    _LIB = "libimi_ref.so"

    @classmethod
    def lib(cls):
        if cls._L is None:
            L = _lib(os.path.join("_ref", cls._LIB))
            L.oref_load.restype = C.c_void_p
            L.oref_load.argtypes = [C.c_char_p, C.c_int, C.c_int]
            L.oref_free.argtypes = [C.c_void_p]
            L.oref_reset.argtypes = [C.c_void_p]
            L.oref_pos.argtypes = [C.c_void_p]
            L.oref_info.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
            L.oref_step.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]
            L.oref_step_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]
            for f in ("oref_hidden", "oref_logits", "oref_state_hidden", "oref_state_logits"):
                getattr(L, f).restype = _fp
                getattr(L, f).argtypes = [C.c_void_p]
            L.oref_state_new.restype = C.c_void_p
            L.oref_state_new.argtypes = [C.c_void_p]
            L.oref_state_free.argtypes = [C.c_void_p]
            L.oref_swap.argtypes = [C.c_void_p, C.c_void_p]
            L.oref_state_pos.argtypes = [C.c_void_p]
            L.oref_step2.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                     C.c_int]
            L.oref_bench_tables.restype = C.c_double
            L.oref_bench_tables.argtypes = [C.c_void_p, C.c_int, C.c_int]
            L.oref_cut.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            L.oref_q4_matvec.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p]
            cls._L = L
        return cls._L

    def __init__(self, path: str, n_ctx: int = 512, threads: int = 0):
        L = self.lib()
        self.h = L.oref_load(path.encode(), threads or os.cpu_count() or 1, n_ctx)
        if not self.h:
            raise RuntimeError("reference load failed")
        info = (C.c_int * 10)()
        L.oref_info(self.h, info)
        (self.n_embd, self.n_vocab, self.n_ctx, self.n_layer, self.n_head, self.n_head_kv, self.head_dim, self.n_ff,
         self.d_conv, self.n_threads) = list(info)

    def __del__(self):
        try:
            self.lib().oref_free(self.h)
        except Exception:
            pass


    def reset(self):
        self.lib().oref_reset(self.h)

    @property
    def pos(self):
        return self.lib().oref_pos(self.h)

    def step(self, token=-1, embd=None, want_logits=True):
        e = _arr(embd, np.float32)
        self.lib().oref_step(self.h, int(token), _ptr(e), int(bool(want_logits)))

    def step_batch(self, tokens=None, embd=None, want_logits=True, hidden_all=False):
        t, e = _arr(tokens, np.int32), _arr(embd, np.float32)
        n = len(t) if t is not None else e.shape[0]
        ha = np.zeros((n, self.n_embd), np.float32) if hidden_all else None
        self.lib().oref_step_batch(self.h, _ptr(t), _ptr(e), n, int(bool(want_logits)), _ptr(ha))
        return ha

    def new_state(self):
        return RefState(self)

    def swap_state(self, s: "RefState"):
        self.lib().oref_swap(self.h, s.h)

    def step2(self, token_a, embd_a, logits_a, b: "RefState", token_b, embd_b, logits_b):
        ea, eb = _arr(embd_a, np.float32), _arr(embd_b, np.float32)
        self.lib().oref_step2(self.h, int(token_a), _ptr(ea), int(bool(logits_a)), b.h, int(token_b), _ptr(eb),
                              int(bool(logits_b)))

    @property
    def hidden(self):
        return np.ctypeslib.as_array(self.lib().oref_hidden(self.h), (self.n_embd,)).copy()

    @property
    def logits(self):
        return np.ctypeslib.as_array(self.lib().oref_logits(self.h), (self.n_vocab,)).copy()

    def bench_tables(self, ncol=1, reps=5) -> float:
        return float(self.lib().oref_bench_tables(self.h, ncol, reps))


class RefState:
    def __init__(self, r: Reference):
        self.r, self.L = r, r.lib()
        self.h = self.L.oref_state_new(r.h)

    def __del__(self):
        try:
            self.L.oref_state_free(self.h)
        except Exception:
            pass

    @property
    def pos(self):
        return self.L.oref_state_pos(self.h)

    @property
    def hidden(self):
        return np.ctypeslib.as_array(self.L.oref_state_hidden(self.h), (self.r.n_embd,)).copy()

    @property
    def logits(self):
        return np.ctypeslib.as_array(self.L.oref_state_logits(self.h), (self.r.n_vocab,)).copy()


def ref_cut(x):
    L = Reference.lib()
    x = _arr(x, np.float32)
    n = x.size
    q, d, s = np.zeros(n, np.int8), np.zeros(n // 32, np.float32), np.zeros(n // 32, np.float32)
    L.oref_cut(_ptr(x), n, _ptr(q), _ptr(d), _ptr(s))
    return q, d, s


def ref_q4_matvec(q4, rows, cols, x) -> np.ndarray:
    """The reference's imi_q4_group / group2 / group_batch over float inputs x[ncol][cols] -> out[ncol][rows]."""
    x = _arr(x, np.float32).reshape(-1, cols)
    out = np.zeros((x.shape[0], rows), np.float32)
    q4 = _arr(q4, np.uint8)
    if Reference.lib().oref_q4_matvec(_ptr(q4), rows, cols, _ptr(x), x.shape[0], _ptr(out)) != 0:
        raise ValueError("shape not supported by the reference kernel")
    return out


def reference_q6k_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libimi_ref_q6k.so"))


class ReferenceQ6K(Reference):
    """The reference's imi_seoul with its own Q6_K word table (no word-table renames: oracle/_ref/libimi_ref_q6k.so),
    for files whose token_embd is Q6_K, as the product's are."""

    _L = None
    _LIB = "libimi_ref_q6k.so"
