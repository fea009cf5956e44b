"""The allocation-free norm-backward entry point, called through its exported C symbol.

``ht_norm_backward_noalloc`` serves callers that cannot allocate device memory, such as runtimes
that plan every buffer in a fixed pool up front or hosts that forbid ``cudaMalloc`` after start-up:
its scratch partial sums live in a fixed device array inside the library instead of a buffer the
caller allocates.  These tests compare it with the regular entry point (``norm_backward`` into
caller-allocated partial rows, then ``sum_rows``) on two calls in a row, so contents left in the
shared array by the first call would show up as an error in the second.  The file name makes
pytest collect it after every other test file.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

_ARGTYPES = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
             ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _entry_points():
    import hybrid_training.ops as ops

    ext = ops.extension()  # fails loudly when the native module is missing
    fn = ctypes.CDLL(str(ops.extension_path())).ht_norm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = _ARGTYPES
    return ext, fn


def _check_against_regular_path(ext, fn, rows: int, d: int, rms: bool) -> None:
    dev = torch.device("cuda")
    res = torch.randn(rows, d, device=dev)
    delta = torch.randn(rows, d, device=dev).bfloat16()
    w = 1 + 0.1 * torch.randn(d, device=dev)
    b = None if rms else 0.1 * torch.randn(d, device=dev)
    r = torch.empty(rows, d, device=dev)
    y = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
    mean = torch.empty(rows, device=dev)
    rstd = torch.empty(rows, device=dev)
    ext.norm_forward(res, delta, w, b, r, y, mean, rstd, 1e-5, rms)
    dy = torch.randn(rows, d, device=dev).bfloat16()
    dr = torch.randn(rows, d, device=dev)

    # Regular entry point: caller-allocated partial rows reduced by sum_rows.
    blocks = ext.norm_backward_blocks(rows)
    part_w = torch.empty(blocks, d, device=dev)
    part_b = None if rms else torch.empty(blocks, d, device=dev)
    dres_ref = torch.empty(rows, d, device=dev)
    ddelta_ref = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
    ext.norm_backward(dy, dr, r, w, mean, rstd, dres_ref, ddelta_ref, part_w, part_b, rms)
    dw_ref = torch.empty(d, device=dev)
    ext.sum_rows(part_w, dw_ref, 0.0)
    db_ref = None
    if not rms:
        db_ref = torch.empty(d, device=dev)
        ext.sum_rows(part_b, db_ref, 0.0)

    # Allocation-free entry point; outputs start as NaN so an unwritten element fails the check.
    dres = torch.full((rows, d), float("nan"), device=dev)
    ddelta = torch.full((rows, d), float("nan"), device=dev, dtype=torch.bfloat16)
    dw = torch.full((d,), float("nan"), device=dev)
    db = torch.full((d,), float("nan"), device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(dy.data_ptr(), 1, dr.data_ptr(), r.data_ptr(), w.data_ptr(), 0, mean.data_ptr(), rstd.data_ptr(),
            dres.data_ptr(), ddelta.data_ptr(), 1, dw.data_ptr(), db.data_ptr(), rows, d, int(rms), stream)
    assert rc == 0, f"ht_norm_backward_noalloc returned {rc}"
    torch.cuda.synchronize()
    assert _rel(dres, dres_ref) < 1e-5, _rel(dres, dres_ref)
    assert _rel(ddelta, ddelta_ref) < 1e-2, _rel(ddelta, ddelta_ref)
    assert _rel(dw, dw_ref) < 1e-5, _rel(dw, dw_ref)
    if not rms:
        assert _rel(db, db_ref) < 1e-5, _rel(db, db_ref)


def test_noalloc_norm_backward_matches_regular_entry_point_twice() -> None:
    ext, fn = _entry_points()
    torch.manual_seed(0)
    # The first call on the device also looks up the shared array's address.
    _check_against_regular_path(ext, fn, rows=333, d=768, rms=False)
    # The second call reuses the array with fewer blocks and a wider row.
    _check_against_regular_path(ext, fn, rows=50, d=2048, rms=True)


def test_noalloc_rejects_hidden_size_above_limit() -> None:
    _, fn = _entry_points()
    one = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    rc = fn(None, 1, None, one, one, 0, one, one, one, None, 1, one, one, 4, 8193, 1, None)
    assert rc == 2
