"""The bounds-checked build (``-DHT_BOUNDS_CHECK``) of the element-wise, norm and optimizer kernels.

Every guarded index of these kernels is compared with the extent of the buffer it addresses; a
violation would be recorded in the module's error word instead of performed.  The checked kernels
run on the same kind of inputs as the regular tests, ragged sizes included, and must give the
regular build's results with the word still zero.  This is how the kernels are checked where
compute-sanitizer is not available.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _mods():
    import hybrid_training.ops as ops

    return ops.extension(), ops.checked_extension()


@pytest.mark.parametrize("rows,d", [(37, 768), (129, 100), (8, 8192), (300, 1001)])
def test_checked_norm_kernels_match_and_stay_in_bounds(rows: int, d: int) -> None:
    ext, chk = _mods()
    chk.bounds_reset()
    dev = torch.device("cuda")
    res = torch.randn(rows, d, device=dev)
    delta = torch.randn(rows, d, device=dev).bfloat16()
    w = 1 + 0.1 * torch.randn(d, device=dev)
    b = 0.1 * torch.randn(d, device=dev)
    outs = []
    for mod in (ext, chk):
        r = torch.empty(rows, d, device=dev)
        y = torch.empty(rows, d, device=dev, dtype=torch.bfloat16)
        mean, rstd = torch.empty(rows, device=dev), torch.empty(rows, device=dev)
        mod.norm_forward(res, delta, w, b, r, y, mean, rstd, 1e-5, False)
        dy = torch.ones(rows, d, device=dev).bfloat16()
        blocks = mod.norm_backward_blocks(rows)
        pw, pb = torch.empty(blocks, d, device=dev), torch.empty(blocks, d, device=dev)
        dres = torch.empty(rows, d, device=dev)
        mod.norm_backward(dy, None, r, w, mean, rstd, dres, None, pw, pb, False)
        dw, db = torch.zeros(d, device=dev), torch.zeros(d, device=dev)
        mod.sum_rows_pair(pw, dw, 0.0, pb, db, 0.0)
        outs.append((r, y, dres, dw, db))
    for a, c in zip(*outs):
        assert torch.equal(a, c)
    assert chk.bounds_status() == [0, 0, 0, 0]


def test_checked_elementwise_and_optimizer_kernels_match_and_stay_in_bounds() -> None:
    ext, chk = _mods()
    chk.bounds_reset()
    dev = torch.device("cuda")
    g = torch.randn(333, 64, device=dev).bfloat16()
    pre = torch.randn(333, 64, device=dev).bfloat16()
    h = torch.randn(5, 7, 2 * 72, device=dev).bfloat16()
    gs = torch.randn(5, 7, 72, device=dev).bfloat16()
    ids = torch.randint(0, 90, (3, 17), device=dev, dtype=torch.int32)
    table = torch.randn(40, 24, device=dev)
    pos = torch.randn(32, 24, device=dev)
    egrad = torch.randn(3, 17, 24, device=dev)
    x = torch.randn(1000, 257, device=dev)
    qkv = torch.randn(2, 16, 4 * 64, device=dev).bfloat16()
    ang = torch.arange(16, device=dev)[:, None] * torch.arange(32, device=dev)[None] * 0.01
    n = 4 * 2501
    p0, gr, m0 = (torch.randn(n, device=dev) for _ in range(3))
    v0 = torch.rand(n, device=dev) * 0.1  # second moments are non-negative
    hyper = torch.tensor([1e-2, 2.0, 1.0, 0.0], device=dev)
    results = []
    for mod in (ext, chk):
        out = torch.empty_like(g)
        mod.gelu_backward(g, pre, out)
        sw = torch.empty(5, 7, 72, device=dev, dtype=torch.bfloat16)
        mod.swiglu_forward(h, sw)
        dh = torch.empty_like(h)
        mod.swiglu_backward(h, gs, dh)
        emb = torch.empty(3, 17, 24, device=dev)
        mod.embedding_forward(ids, table, pos, emb, 50)  # rows 50..89 live here
        dtab = torch.zeros_like(table)
        mod.embedding_backward(ids, egrad, dtab, 50)
        cs = torch.zeros(257, device=dev)
        mod.column_sum(x, cs, 0.0)
        rot = qkv.clone()
        mod.rope_(rot, ang.cos(), ang.sin(), 3, 64, False)
        p, m, v = p0.clone(), m0.clone(), v0.clone()
        mod.adamw_flat(p, gr, m, v, None, hyper, 0.9, 0.95, 1e-8, 0.1, True)
        results.append((out, sw, dh, emb, cs, rot, p, m, v, dtab))
    for a, c in zip(results[0][:-1], results[1][:-1]):
        assert torch.equal(a, c)
    assert torch.allclose(results[0][-1], results[1][-1], atol=1e-6)  # atomics: the order of duplicate rows varies
    assert chk.bounds_status() == [0, 0, 0, 0]
