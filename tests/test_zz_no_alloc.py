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
import re
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

_HEADER = Path(__file__).resolve().parents[1] / "hybrid_training" / "ops" / "csrc" / "norm_noalloc.h"
_CTYPES = {"int": ctypes.c_int, "cudaStream_t": ctypes.c_void_p}


def _argtypes_from_header() -> list:
    """ctypes argument list parsed from the C declaration, so the signature has a single source."""
    text = _HEADER.read_text()
    m = re.search(r"int\s+ht_norm_backward_noalloc\s*\(([^)]*)\)\s*;", text)
    assert m is not None, "declaration of ht_norm_backward_noalloc not found in norm_noalloc.h"
    out = []
    for arg in m.group(1).split(","):
        decl = " ".join(arg.split())
        typ = decl.rsplit(" ", 1)[0]
        out.append(ctypes.c_void_p if "*" in decl else _CTYPES[typ.replace("const ", "")])
    return out


def _max_cols_from_header() -> int:
    return int(re.search(r"#define\s+HT_NORM_NOALLOC_MAX_COLS\s+(\d+)", _HEADER.read_text()).group(1))


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


def _entry_points():
    import hybrid_training.ops as ops

    ext = ops.extension()  # fails loudly when the native module is missing
    fn = ctypes.CDLL(str(ops.extension_path())).ht_norm_backward_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = _argtypes_from_header()
    return ext, fn


def _torch_reference(dy, dr, r, w, mean, rstd, rms: bool):
    """fp32 PyTorch statement of the same backward (independent of both native entry points)."""
    dy = dy.float()
    mu = torch.zeros_like(mean) if rms else mean
    xhat = (r - mu[:, None]) * rstd[:, None]
    g = dy * w[None, :]
    d = r.shape[1]
    mg = torch.zeros_like(rstd) if rms else g.sum(1) / d
    mgx = (g * xhat).sum(1) / d
    dres = rstd[:, None] * (g - mg[:, None] - xhat * mgx[:, None]) + dr
    return dres, (dy * xhat).sum(0), dy.sum(0)


def _check_against_regular_path(ext, fn, rows: int, d: int, rms: bool, garbage_mean: bool = False) -> None:
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
    # RMSNorm ignores the mean; a buffer of garbage there must not change the result.
    mean_arg = torch.randn(rows, device=dev) * 100 if (rms and garbage_mean) else mean

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
    rc = fn(dy.data_ptr(), 1, dr.data_ptr(), r.data_ptr(), w.data_ptr(), 0, mean_arg.data_ptr(), rstd.data_ptr(),
            dres.data_ptr(), ddelta.data_ptr(), 1, dw.data_ptr(), db.data_ptr(), rows, d, int(rms), stream)
    assert rc == 0, f"ht_norm_backward_noalloc returned {rc}"
    torch.cuda.synchronize()
    assert _rel(dres, dres_ref) < 1e-5, _rel(dres, dres_ref)
    assert _rel(ddelta, ddelta_ref) < 1e-2, _rel(ddelta, ddelta_ref)
    assert _rel(dw, dw_ref) < 1e-5, _rel(dw, dw_ref)
    if not rms:
        assert _rel(db, db_ref) < 1e-5, _rel(db, db_ref)
    t_dres, t_dw, t_db = _torch_reference(dy, dr, r, w, mean, rstd, rms)
    assert _rel(dres, t_dres) < 1e-4, _rel(dres, t_dres)
    assert _rel(dw, t_dw) < 1e-4, _rel(dw, t_dw)
    if not rms:
        assert _rel(db, t_db) < 1e-4, _rel(db, t_db)


def test_noalloc_norm_backward_matches_regular_entry_point_twice() -> None:
    ext, fn = _entry_points()
    torch.manual_seed(0)
    # The first call on the device also looks up the shared array's address.
    _check_against_regular_path(ext, fn, rows=333, d=768, rms=False)
    # The second call reuses the array with fewer blocks and a wider row.
    _check_against_regular_path(ext, fn, rows=50, d=2048, rms=True)


def test_noalloc_norm_backward_widest_and_ragged_hidden_sizes() -> None:
    ext, fn = _entry_points()
    torch.manual_seed(1)
    d_max = _max_cols_from_header()
    # The widest accepted row launches 1024 threads per block, twice in a row.
    _check_against_regular_path(ext, fn, rows=300, d=d_max, rms=False)
    _check_against_regular_path(ext, fn, rows=77, d=d_max, rms=True)
    # A hidden size that is not a multiple of the 8 columns per thread; RMSNorm with a garbage mean.
    _check_against_regular_path(ext, fn, rows=129, d=1001, rms=True, garbage_mean=True)
    _check_against_regular_path(ext, fn, rows=129, d=1001, rms=False)


def test_noalloc_rejects_hidden_size_above_limit() -> None:
    _, fn = _entry_points()
    one = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    rc = fn(None, 1, None, one, one, 0, one, one, one, None, 1, one, one, 4, _max_cols_from_header() + 1, 1, None)
    assert rc == 2
