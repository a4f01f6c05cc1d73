"""The table read that allocates nothing (imi_cuda_q4_matvec_static) against the allocating entry point
(imi_cuda_q4_matvec) and against the oracle (imi_q4_group's per-row result restated in C) on the same inputs,
through the C-ABI on device buffers. Two calls in a row with different shapes share the one static scratch; each
must match. The kernels keep imi's accumulation order, so the results agree bit for bit; the float tolerance below
is the stated bound should that ever not hold (rel 1e-6).

This file is collected last on purpose: it must pass after the other tests have used the device, and alone."""
import ctypes as C

import numpy as np
import pytest

import nunchi_b200 as nb
import oracle
from nunchi_b200 import synth

pytestmark = pytest.mark.gpu

STATIC_TABLE_BYTES = 16 * 1024 * 1024   # IMI_CUDA_STATIC_TABLE_BYTES in include/imi_cuda.h
RTOL = 1e-6


def _case(rows, cols, ncol, seed):
    rng = np.random.default_rng(seed)
    q4 = synth._q4_0(rng, rows, cols).reshape(-1)
    x = rng.standard_normal((ncol, cols)).astype(np.float32)
    cuts = [oracle.cut(v) for v in x]
    cq, cd, cs = (np.concatenate([c[k] for c in cuts]) for k in range(3))
    return q4, cq, cd, cs


def _static(torch, q4, rows, cols, cq, cd, cs, stream):
    dev = torch.device("cuda:0")
    t_q4 = torch.from_numpy(q4).to(dev)
    t_q = torch.from_numpy(cq).to(dev)
    t_d = torch.from_numpy(cd).to(dev)
    t_s = torch.from_numpy(cs).to(dev)
    ncol = cq.size // cols
    t_out = torch.full((ncol, rows), float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    st = nb.lib().imi_cuda_q4_matvec_static(0, C.c_void_p(t_q4.data_ptr()), rows, cols, C.c_void_p(t_q.data_ptr()),
                                            C.c_void_p(t_d.data_ptr()), C.c_void_p(t_s.data_ptr()), ncol,
                                            C.c_void_p(t_out.data_ptr()), C.c_void_p(stream.cuda_stream))
    return st, t_out.cpu().numpy()


def test_static_matches_allocating_entry_two_calls_in_a_row():
    torch = pytest.importorskip("torch")
    stream = torch.cuda.Stream()
    # the second call is smaller than the first, so stale table bytes of the first would show if they were read
    for rows, cols, ncol, seed in [(2048, 2048, 2, 11), (300, 8192, 1, 12)]:
        q4, cq, cd, cs = _case(rows, cols, ncol, seed)
        want = nb.q4_matvec(q4, rows, cols, cq, cd, cs)
        truth = np.asarray(oracle.q4_matvec(q4, rows, cols, cq, cd, cs), np.float32).reshape(want.shape)
        st, got = _static(torch, q4, rows, cols, cq, cd, cs, stream)
        assert st == 0, nb.lib().imi_cuda_error().decode()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=0)
        np.testing.assert_allclose(got, truth, rtol=RTOL, atol=0)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert np.array_equal(got.view(np.uint32), truth.view(np.uint32))


def test_static_largest_table_and_refusal_beyond_it():
    torch = pytest.importorskip("torch")
    stream = torch.cuda.Stream()
    cols = 2048
    rows = STATIC_TABLE_BYTES // (cols // 32 * 18)          # the largest table of this width that fits
    q4, cq, cd, cs = _case(rows, cols, 1, 13)
    want = nb.q4_matvec(q4, rows, cols, cq, cd, cs)
    st, got = _static(torch, q4, rows, cols, cq, cd, cs, stream)
    assert st == 0, nb.lib().imi_cuda_error().decode()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=0)
    truth = np.asarray(oracle.q4_matvec(q4, rows, cols, cq, cd, cs), np.float32).reshape(got.shape)
    np.testing.assert_allclose(got, truth, rtol=RTOL, atol=0)
    # one more row passes the limit: refused before any device work, with the limit in the message
    st, _ = _static(torch, np.zeros((rows + 1) * (cols // 32) * 18, np.uint8), rows + 1, cols,
                    np.zeros(cols, np.int8), np.zeros(cols // 32, np.float32), np.zeros(cols // 32, np.float32), stream)
    assert st == 1                                           # IMI_E_ARG
    assert str(STATIC_TABLE_BYTES) in nb.lib().imi_cuda_error().decode()


def test_static_refuses_host_buffers():
    torch = pytest.importorskip("torch")
    q4, cq, cd, cs = _case(64, 256, 1, 14)
    out = np.zeros(64, np.float32)
    st = nb.lib().imi_cuda_q4_matvec_static(0, q4.ctypes.data, 64, 256, cq.ctypes.data, cd.ctypes.data,
                                            cs.ctypes.data, 1, out.ctypes.data, None)
    assert st == 1                                           # IMI_E_ARG: host memory is not device memory
    assert "device memory" in nb.lib().imi_cuda_error().decode()
    assert torch.cuda.is_available()
