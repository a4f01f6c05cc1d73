"""nunchi_b200: a B200 decode engine for imi's brain token loop (the Seoul / LFM3 hybrid backbone).

Python binding over the C-ABI of include/imi_cuda.h (libimi_cuda.so, built in-tree by nunchi_b200.build). The
classes mirror imi's C++ interface (imi/core/seoul.h): `Seoul` has load / reset / step / step2 / step_batch /
new_state / swap_state and the hidden / logits outputs. There is no CPU path: without the built library or a CUDA
device every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libimi_cuda.so")

STATUS = {0: "ok", 1: "bad argument", 2: "file", 3: "format", 4: "context full", 5: "cuda", 6: "out of memory",
          7: "device wait timed out", 8: "no device"}


class ImiError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class ContextFull(ImiError):
    pass


class Info(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_embd", "n_vocab", "n_ctx", "n_layer", "n_attn", "n_head", "n_head_kv",
                                        "head_dim", "n_ff", "d_conv", "n_swa", "max_batch")] + \
               [("weight_bytes", C.c_size_t), ("state_bytes", C.c_size_t), ("cols_per_read", C.c_int)]


_L = None
_vp, _fp, _ip = C.c_void_p, C.c_void_p, C.c_void_p


def lib():
    """The engine library (raises if it is not built: run `python -m nunchi_b200.build`)."""
    global _L
    if _L is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m nunchi_b200.build`")
        L = C.CDLL(LIB_PATH)
        L.imi_cuda_error.restype = C.c_char_p
        L.imi_cuda_load.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
        L.imi_cuda_free.argtypes = [_vp]
        L.imi_cuda_free.restype = None
        L.imi_cuda_get_info.argtypes = [_vp, C.POINTER(Info)]
        L.imi_cuda_state_new.argtypes = [_vp, C.POINTER(_vp)]
        L.imi_cuda_state_free.argtypes = [_vp]
        L.imi_cuda_state_free.restype = None
        L.imi_cuda_state_reset.argtypes = [_vp]
        L.imi_cuda_state_pos.argtypes = [_vp]
        L.imi_cuda_step.argtypes = [_vp, C.c_int32, _fp, C.c_int]
        L.imi_cuda_step2.argtypes = [_vp, C.c_int32, _fp, C.c_int, _vp, C.c_int32, _fp, C.c_int]
        L.imi_cuda_step_multi.argtypes = [_vp, C.c_int, _ip, _fp, _ip]
        L.imi_cuda_step_batch.argtypes = [_vp, _ip, _fp, C.c_int, C.c_int, _fp]
        L.imi_cuda_greedy.argtypes = [_vp, C.c_int, _ip, C.c_int, _ip]
        L.imi_cuda_get_hidden.argtypes = [_vp, _fp]
        L.imi_cuda_get_logits.argtypes = [_vp, _fp]
        L.imi_cuda_get_argmax.argtypes = [_vp, C.POINTER(C.c_int32), C.POINTER(C.c_float)]
        L.imi_cuda_stream.restype = _vp
        L.imi_cuda_stream.argtypes = [_vp]
        L.imi_cuda_launches_per_step.argtypes = [_vp, C.c_int, C.c_int]
        L.imi_cuda_launches_per_batch.argtypes = [_vp, C.c_int, C.c_int]
        L.imi_cuda_bench_tables.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_size_t)]
        L.imi_cuda_trace_table.argtypes = [_vp, C.c_int, C.c_int, C.c_int, _vp, C.POINTER(C.c_int)]
        L.imi_cuda_state_save.argtypes = [_vp, _vp, C.c_size_t, C.POINTER(C.c_size_t)]
        L.imi_cuda_state_load.argtypes = [_vp, _vp, C.c_size_t]
        L.imi_cuda_trace_step.argtypes = [_vp, C.c_int32, C.c_int, _vp, C.c_int, _vp, _vp, C.POINTER(C.c_int)]
        L.imi_cuda_q8_cut.argtypes = [C.c_int, _fp, C.c_int, _vp, _fp, _fp]
        L.imi_cuda_q6k_scores.argtypes = [C.c_int, _vp, C.c_int, C.c_int, _fp, _fp, _vp, _fp, _vp]
        L.imi_cuda_q4_matvec.argtypes = [C.c_int, _vp, C.c_int, C.c_int, _vp, _fp, _fp, C.c_int, _fp, _ip]
        L.imi_cuda_q4_matvec_static.argtypes = [C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, _vp, C.c_int, _vp, _vp]
        L.imi_cuda_check_wait_timeout.argtypes = [C.c_int, C.c_double]
        L.imi_cuda_q4_matmul.argtypes = [C.c_int, _vp, C.c_int, C.c_int, _vp, _fp, _fp, C.c_int, _fp]
        L.imi_cuda_bench_matvec.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_float),
                                            C.POINTER(C.c_size_t)]
        _L = L
    return _L


def _check(st: int):
    if st != 0:
        msg = lib().imi_cuda_error().decode(errors="replace")
        raise (ContextFull if st == 4 else ImiError)(st, msg)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(x):
    return None if x is None else np.ascontiguousarray(x, dtype=np.float32)


class Engine:
    """One GGUF model resident on one GPU (imi_seoul::load, seoul.cpp:93-186)."""

    def __init__(self, path: str, device: int = 0, n_ctx: int = 512, max_batch: int = 8):
        h = _vp()
        _check(lib().imi_cuda_load(os.fspath(path).encode(), device, n_ctx, max_batch, C.byref(h)))
        self.h = h
        info = Info()
        _check(lib().imi_cuda_get_info(self.h, C.byref(info)))
        self.info = info
        for n, _ in Info._fields_:
            setattr(self, n, getattr(info, n))

    def close(self):
        if getattr(self, "h", None):
            lib().imi_cuda_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_state(self) -> "State":
        return State(self)

    @property
    def stream(self) -> int:
        """cudaStream_t of every launch of this engine (as an integer handle)."""
        return int(lib().imi_cuda_stream(self.h) or 0)

    def launches_per_step(self, n: int = 1, want_logits: bool = True) -> int:
        return lib().imi_cuda_launches_per_step(self.h, n, int(bool(want_logits)))

    def launches_per_batch(self, n: int, want_logits: bool = True) -> int:
        return lib().imi_cuda_launches_per_batch(self.h, n, int(bool(want_logits)))

    def prefill_launches(self, n_vecs: int, chunk: int, n_ids: int) -> int:
        """launches of configs[2]'s reads: the vectors in chunks of `chunk`, then the ids with the word scores"""
        k = sum(self.launches_per_batch(min(chunk, n_vecs - a), False) for a in range(0, n_vecs, chunk))
        return k + self.launches_per_batch(n_ids, True)

    def bench_tables(self, ncol: int = 1, reps: int = 20):
        """imi_seoul::bench_tables: all layer tables back to back; (mean ms per pass, table bytes per pass)."""
        ms, b = C.c_float(), C.c_size_t()
        _check(lib().imi_cuda_bench_tables(self.h, ncol, reps, C.byref(ms), C.byref(b)))
        return float(ms.value), int(b.value)


def trace_table(engine: "Engine", layer: int, which: int, ncol: int = 1) -> np.ndarray:
    """Diagnostics: per-CTA phase timestamps (ns) of one table read (imi_cuda_trace_table)."""
    buf = np.zeros((1024, 16), np.uint64)
    g = C.c_int()
    _check(lib().imi_cuda_trace_table(engine.h, layer, which, ncol, _ptr(buf), C.byref(g)))
    return buf[: g.value]


def trace_step(state: "State", token: int, want_logits: bool = True, max_launches: int = 256):
    """Diagnostics: per-launch per-CTA phase timestamps (ns) of one decode step (imi_cuda_trace_step)."""
    nsm = 148
    out = np.zeros((max_launches, nsm, 16), np.uint64)
    kinds, grids = np.zeros(max_launches, np.int32), np.zeros(max_launches, np.int32)
    n = C.c_int()
    _check(lib().imi_cuda_trace_step(state.h, int(token), int(bool(want_logits)), _ptr(out), max_launches, _ptr(kinds),
                                     _ptr(grids), C.byref(n)))
    return out[: n.value], kinds[: n.value], grids[: n.value]


class State:
    """One conversation on the device (imi_seoul_state, seoul.h:21-26)."""

    def __init__(self, engine: Engine):
        self.engine = engine
        h = _vp()
        _check(lib().imi_cuda_state_new(engine.h, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None) and self.engine.h:
            lib().imi_cuda_state_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _check(lib().imi_cuda_state_reset(self.h))

    @property
    def pos(self) -> int:
        return lib().imi_cuda_state_pos(self.h)

    def step(self, token: int = -1, embd=None, want_logits: bool = True):
        e = _f32(embd)
        _check(lib().imi_cuda_step(self.h, int(token), _ptr(e), int(bool(want_logits))))

    def step_batch(self, tokens=None, embd=None, want_logits: bool = True, hidden_all: bool = False):
        t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        e = _f32(embd)
        n = len(t) if t is not None else e.shape[0]
        ha = np.zeros((n, self.engine.n_embd), np.float32) if hidden_all else None
        _check(lib().imi_cuda_step_batch(self.h, _ptr(t), _ptr(e), n, int(bool(want_logits)), _ptr(ha)))
        return ha

    @property
    def hidden(self) -> np.ndarray:
        out = np.zeros(self.engine.n_embd, np.float32)
        _check(lib().imi_cuda_get_hidden(self.h, _ptr(out)))
        return out

    @property
    def logits(self) -> np.ndarray:
        out = np.zeros(self.engine.n_vocab, np.float32)
        _check(lib().imi_cuda_get_logits(self.h, _ptr(out)))
        return out

    def save(self) -> bytes:
        """Checkpoint of this conversation (imi_cuda_state_save: position, K/V, conv memory, outputs)."""
        n = C.c_size_t()
        _check(lib().imi_cuda_state_save(self.h, None, 0, C.byref(n)))
        buf = np.zeros(n.value, np.uint8)
        _check(lib().imi_cuda_state_save(self.h, _ptr(buf), n.value, C.byref(n)))
        return buf.tobytes()

    def load(self, image: bytes):
        buf = np.frombuffer(image, np.uint8).copy()
        _check(lib().imi_cuda_state_load(self.h, _ptr(buf), buf.size))

    def unpack(self, image: bytes = None) -> dict:
        """The checkpoint's fields as arrays (pos, k, v [n_attn][pos][kvd] fp16 bits, conv [n_conv][d_conv][E])."""
        b = image if image is not None else self.save()
        h = np.frombuffer(b[:44], np.int32)
        pos, na, _, kvd, nconv, dconv, E, V = (int(x) for x in h[2:10])
        o = 44
        def take(n, dt, shape):
            nonlocal o
            a = np.frombuffer(b[o:o + n * np.dtype(dt).itemsize], dt).reshape(shape)
            o += n * np.dtype(dt).itemsize
            return a
        k = take(na * pos * kvd, np.uint16, (na, pos, kvd))
        v = take(na * pos * kvd, np.uint16, (na, pos, kvd))
        conv = take(nconv * dconv * E, np.float32, (nconv, dconv, E))
        hid = take(E, np.float32, (E,))
        return {"pos": pos, "k": k, "v": v, "conv": conv, "hidden": hid, "next_pick": int(h[10])}

    def argmax(self):
        i, v = C.c_int32(), C.c_float()
        _check(lib().imi_cuda_get_argmax(self.h, C.byref(i), C.byref(v)))
        return int(i.value), float(v.value)


def _handles(states):
    arr = (_vp * len(states))(*[s.h for s in states])
    return arr


def step2(a: State, token_a, embd_a, logits_a, b: State, token_b, embd_b, logits_b):
    """imi_seoul::step2 (seoul.cpp:208-220): two conversations, one table read each step, numbers as alone."""
    ea, eb = _f32(embd_a), _f32(embd_b)
    _check(lib().imi_cuda_step2(a.h, int(token_a), _ptr(ea), int(bool(logits_a)), b.h, int(token_b), _ptr(eb),
                                int(bool(logits_b))))


def step_multi(states, tokens=None, embd=None, want_logits=None):
    n = len(states)
    t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
    e = _f32(embd)
    w = None if want_logits is None else np.ascontiguousarray(want_logits, dtype=np.int32)
    _check(lib().imi_cuda_step_multi(_handles(states), n, _ptr(t), _ptr(e), _ptr(w)))


def greedy(states, steps: int, tokens=None) -> np.ndarray:
    """`steps` greedy positions per conversation on the device; returns ids[steps][n]."""
    n = len(states)
    t = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
    ids = np.zeros((steps, n), np.int32)
    _check(lib().imi_cuda_greedy(_handles(states), n, _ptr(t), steps, _ptr(ids)))
    return ids


def q8_cut(x, device: int = 0):
    """The device 8-bit cut (imi_q8::from): codes, scales, scale * code sums per 32 values."""
    x = _f32(x).ravel()
    n = x.size
    q, d, s = np.zeros(n, np.int8), np.zeros(n // 32, np.float32), np.zeros(n // 32, np.float32)
    _check(lib().imi_cuda_q8_cut(device, _ptr(x), n, _ptr(q), _ptr(d), _ptr(s)))
    return q, d, s


def q6k_scores(q6k, x, device: int = 0):
    """Word scores of Q6_K rows ([rows][cols/256 * 210] bytes) for the float input x on the device (imi_q8k::from +
    imi_q6k_row): (scores[rows], (codes, scales, code sums of the input cut))."""
    q6k = np.ascontiguousarray(q6k, dtype=np.uint8)
    x = _f32(x).ravel()
    rows, cols = q6k.shape[0], x.size
    out = np.zeros(rows, np.float32)
    q, d, bs = np.zeros(cols, np.int8), np.zeros(cols // 256, np.float32), np.zeros(cols // 16, np.int16)
    _check(lib().imi_cuda_q6k_scores(device, _ptr(q6k), rows, cols, _ptr(x), _ptr(out), _ptr(q), _ptr(d), _ptr(bs)))
    return out, (q, d, bs)


def q4_matvec(q4, rows: int, cols: int, xq, xd, xs, dots: bool = False, device: int = 0):
    """A GGUF Q4_0 table times 8-bit inputs on the device: out[ncol][rows] (and integer block dots for one input)."""
    q4 = np.ascontiguousarray(q4, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    xd, xs = _f32(xd), _f32(xs)
    ncol = xq.size // cols
    out = np.zeros((ncol, rows), np.float32)
    dd = np.zeros((rows, cols // 32), np.int32) if dots else None
    _check(lib().imi_cuda_q4_matvec(device, _ptr(q4), rows, cols, _ptr(xq), _ptr(xd), _ptr(xs), ncol, _ptr(out),
                                    _ptr(dd)))
    return (out, dd) if dots else out


def q4_matmul(q4, rows: int, cols: int, xq, xd, xs, device: int = 0):
    """The same as q4_matvec for many inputs on the tensor cores (imi_cuda_q4_matmul): out[ncol][rows]."""
    q4 = np.ascontiguousarray(q4, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    xd, xs = _f32(xd), _f32(xs)
    ncol = xq.size // cols
    out = np.zeros((ncol, rows), np.float32)
    _check(lib().imi_cuda_q4_matmul(device, _ptr(q4), rows, cols, _ptr(xq), _ptr(xd), _ptr(xs), ncol, _ptr(out)))
    return out


def bench_matvec(rows: int, cols: int, ncol: int, reps: int = 20, device: int = 0):
    """The isolated table read timed on the device (imi_cuda_bench_matvec): (mean ms per read, algorithmic bytes)."""
    ms, b = C.c_float(), C.c_size_t()
    _check(lib().imi_cuda_bench_matvec(device, rows, cols, ncol, reps, C.byref(ms), C.byref(b)))
    return float(ms.value), int(b.value)


class Seoul:
    """imi_seoul's surface (seoul.h:28-72) on the engine: the brain with its own conversation."""

    def __init__(self, path: str, ctx_len: int = 512, device: int = 0, max_batch: int = 8):
        self.engine = Engine(path, device, ctx_len, max_batch)
        self.n_embd, self.n_vocab, self.n_ctx = self.engine.n_embd, self.engine.n_vocab, self.engine.n_ctx
        self.state = self.engine.new_state()

    def reset(self):
        self.state.reset()

    @property
    def pos(self):
        return self.state.pos

    def step(self, token=-1, embd=None, want_logits=True):
        self.state.step(token, embd, want_logits)

    def step_batch(self, tokens=None, embd=None, want_logits=True, hidden_all=False):
        return self.state.step_batch(tokens, embd, want_logits, hidden_all)

    def new_state(self) -> State:
        return self.engine.new_state()

    def swap_state(self, s: State):
        """Trade the brain's conversation for s (no copying, seoul.cpp:203-206)."""
        self.state.h, s.h = s.h, self.state.h

    def step2(self, token_a, embd_a, logits_a, b: State, token_b, embd_b, logits_b):
        step2(self.state, token_a, embd_a, logits_a, b, token_b, embd_b, logits_b)

    @property
    def hidden(self):
        return self.state.hidden

    @property
    def logits(self):
        return self.state.logits
