"""Numerics of every native sm_100a kernel against a plain fp32 PyTorch statement of the same op.

Shapes include ragged sizes (not multiples of the tile) to exercise TMA
out-of-bounds fill and the epilogue masks.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ops():
    import hybrid_training.ops as ops

    ops.extension()  # fail loudly if the native module is missing
    return ops


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("m,n,k", [(256, 512, 192), (200, 300, 100), (1, 33, 64), (1000, 257, 770)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_matches_fp32(m: int, n: int, k: int, a_mn: bool, b_mn: bool) -> None:
    ops = _ops()
    dev = torch.device("cuda")
    a = torch.randn((k, m) if a_mn else (m, k), device=dev).bfloat16()
    b = torch.randn((k, n) if b_mn else (n, k), device=dev).bfloat16()
    if (a.stride(0) * 2) % 16 or (b.stride(0) * 2) % 16:
        pytest.skip("TMA needs 16-byte aligned operand rows")
    d = ops.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn, out_dtype=torch.float32)
    ref, _ = ops.reference_gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn)
    assert _rel(d, ref) < 1e-5, _rel(d, ref)


@pytest.mark.parametrize("m,n,k,a_mn,b_mn,epi", [
    (1024, 768, 256, False, False, "plain"), (300, 520, 192, False, False, "gelu"), (8192, 2304, 768, False, False, "plain"),
    (777, 512, 320, False, True, "gelu_bwd"), (640, 1024, 448, False, True, "plain"), (3072, 768, 8192, True, True, "wgrad"),
    (2304, 768, 1000, True, True, "wgrad_fast"), (600, 256, 4096, True, True, "wgrad")])
def test_gemm_cta_pair_matches_single_cta_and_fp32(m: int, n: int, k: int, a_mn: bool, b_mn: bool, epi: str) -> None:
    """256-row tiles on CTA pairs (tcgen05.mma.cta_group::2) against the single-CTA kernel and fp32 torch,
    for the forward, data-gradient and weight-gradient layouts and their epilogues (split-K included)."""
    ops = _ops()
    ext = ops.extension()
    dev = torch.device("cuda")
    torch.manual_seed(1)
    a = torch.randn((k, m) if a_mn else (m, k), device=dev).bfloat16()
    b = (torch.randn((k, n) if b_mn else (n, k), device=dev) * 0.05).bfloat16()
    bias = torch.randn(n, device=dev) if epi == "gelu" else None
    pre = torch.randn(m, n, device=dev).bfloat16() if epi == "gelu_bwd" else None
    c0 = torch.randn(m, n, device=dev)
    outs = []
    try:
        ops.set_deterministic_reductions(epi != "wgrad_fast")
        for mode in (0, 1):
            ext.set_gemm_pair(mode)
            if epi == "gelu":
                aux = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                y = ops.gemm(a, b, bias=bias, aux=aux, epilogue=ops.EPI_GELU)
                outs.append((y, aux))
            elif epi == "gelu_bwd":
                outs.append((ops.gemm(a, b, b_mn_major=True, aux=pre, epilogue=ops.EPI_GELU_BWD), None))
            elif epi.startswith("wgrad"):
                d = c0.clone()
                ops.gemm(a, b, out=d, a_mn_major=True, b_mn_major=True, beta=1.0)
                outs.append((d, None))
            else:
                outs.append((ops.gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn), None))
        torch.cuda.synchronize()
    finally:
        ext.set_gemm_pair(0)
        ops.set_deterministic_reductions(True)
    if epi == "gelu":
        ref, ref_pre = ops.reference_gemm(a, b, bias=bias, epilogue=ops.EPI_GELU)
    elif epi == "gelu_bwd":
        ref, ref_pre = ops.reference_gemm(a, b, b_mn_major=True, aux=pre, epilogue=ops.EPI_GELU_BWD)
    elif epi.startswith("wgrad"):
        ref, ref_pre = ops.reference_gemm(a, b, a_mn_major=True, b_mn_major=True, c=c0, beta=1.0)
    else:
        ref, ref_pre = ops.reference_gemm(a, b, a_mn_major=a_mn, b_mn_major=b_mn)
    tol = 1e-5 if epi.startswith("wgrad") else 1e-2
    for y, aux in outs:
        assert _rel(y, ref) < tol, (epi, _rel(y, ref))
        if aux is not None:
            assert _rel(aux, ref_pre) < 1e-2
    if epi != "wgrad_fast":  # same tile sums in the same order: equal bits
        assert torch.equal(outs[0][0], outs[1][0]) or _rel(outs[0][0], outs[1][0]) < 1e-6


def test_gemm_epilogues() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    m, n, k = 384, 520, 256
    a = torch.randn(m, k, device=dev).bfloat16()
    b = (torch.randn(n, k, device=dev) * 0.05).bfloat16()
    bias = torch.randn(n, device=dev)
    pre = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    y = ops.gemm(a, b, bias=bias, aux=pre, epilogue=ops.EPI_GELU)
    ref, ref_pre = ops.reference_gemm(a, b, bias=bias, epilogue=ops.EPI_GELU)
    assert _rel(y, ref) < 1e-2 and _rel(pre, ref_pre) < 1e-2
    g = torch.randn(m, n, device=dev).bfloat16()
    w = torch.randn(n, n, device=dev).bfloat16()
    dx = ops.gemm(g, w, b_mn_major=True, aux=pre, epilogue=ops.EPI_GELU_BWD)
    ref_dx, _ = ops.reference_gemm(g, w, b_mn_major=True, aux=pre, epilogue=ops.EPI_GELU_BWD)
    assert _rel(dx, ref_dx) < 1e-2
    # fp32 accumulation with beta and a device-side alpha
    c = torch.randn(n, k, device=dev)
    alpha = torch.tensor([0.5], device=dev)
    out = c.clone()
    ops.gemm(g, a, out=out, a_mn_major=True, b_mn_major=True, beta=1.0, alpha=alpha)
    ref_acc, _ = ops.reference_gemm(g, a, a_mn_major=True, b_mn_major=True, c=c, beta=1.0, alpha=alpha)
    assert _rel(out, ref_acc) < 1e-5


@pytest.mark.parametrize("m,n,k", [(8192, 768, 256), (2048, 3072, 128), (4096, 768, 192), (8192, 2304, 64)])
def test_gemm_tile_widths_on_model_shapes(m: int, n: int, k: int) -> None:
    """N = 768 / 3072 outputs run 128 x 192 tiles (fewer idle SMs in the last wave), N = 2304 runs 128 x 256:
    plain, GELU and GELU' epilogues, B K-major (forward) and MN-major (data gradient), against fp32 PyTorch."""
    ops = _ops()
    dev = torch.device("cuda")
    a = torch.randn(m, k, device=dev).bfloat16()
    w = (torch.randn(n, k, device=dev) * 0.05).bfloat16()
    bias = torch.randn(n, device=dev)
    ref = a.float() @ w.float().t() + bias
    y = ops.gemm(a, w, bias=bias)
    assert _rel(y, ref) < 1e-2
    pre = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    h = ops.gemm(a, w, bias=bias, aux=pre, epilogue=ops.EPI_GELU)
    assert _rel(pre, ref) < 1e-2
    assert _rel(h, torch.nn.functional.gelu(ref, approximate="tanh")) < 1e-2
    wt = (torch.randn(k, n, device=dev) * 0.05).bfloat16()  # [K, N] read MN-major
    ref_mn = a.float() @ wt.float()
    assert _rel(ops.gemm(a, wt, b_mn_major=True), ref_mn) < 1e-2
    dpre = torch.randn(m, n, device=dev).bfloat16()
    dx = ops.gemm(a, wt, b_mn_major=True, aux=dpre, epilogue=ops.EPI_GELU_BWD)
    x = dpre.float()
    t = torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
    dgelu = 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
    assert _rel(dx, ref_mn * dgelu) < 2e-2


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_split_k_weight_gradient_shapes(out_dtype: torch.dtype) -> None:
    """Few output tiles and a long K: the K loop is split and the partials are summed in order."""
    ops = _ops()
    dev = torch.device("cuda")
    k, m, n = 4096, 296, 200
    g = torch.randn(k, m, device=dev).bfloat16()
    x = torch.randn(k, n, device=dev).bfloat16()
    alpha = torch.tensor([0.25], device=dev)
    c = torch.randn(m, n, device=dev).to(out_dtype)
    out = c.clone()
    ops.gemm(g, x, out=out, a_mn_major=True, b_mn_major=True, beta=1.0 if out_dtype == torch.float32 else 0.0, alpha=alpha)
    ref, _ = ops.reference_gemm(g, x, a_mn_major=True, b_mn_major=True, c=c if out_dtype == torch.float32 else None,
                                beta=1.0 if out_dtype == torch.float32 else 0.0, alpha=alpha)
    assert _rel(out, ref) < (1e-5 if out_dtype == torch.float32 else 1e-2), _rel(out, ref)
    again = c.clone()
    ops.gemm(g, x, out=again, a_mn_major=True, b_mn_major=True, beta=1.0 if out_dtype == torch.float32 else 0.0, alpha=alpha)
    assert torch.equal(again, out), "split-K result must be deterministic"


@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_gemm_split_k_reduce_add_into_the_output(beta: float) -> None:
    """With reproducibility off, split-K partial tiles are TMA reduce-added straight into an fp32 output."""
    ops = _ops()
    dev = torch.device("cuda")
    k, m, n = 4096, 296, 200
    g = torch.randn(k, m, device=dev).bfloat16()
    x = torch.randn(k, n, device=dev).bfloat16()
    store = torch.randn(m, 256, device=dev)  # padded rows: the output is a strided view
    c = store[:, :n].clone()
    pad = store[:, n:].clone()
    out = store[:, :n]
    try:
        ops.set_deterministic_reductions(False)
        ops.gemm(g, x, out=out, a_mn_major=True, b_mn_major=True, beta=beta)
    finally:
        ops.set_deterministic_reductions(True)
    ref = g.float().t() @ x.float() + (c if beta else 0.0)
    assert _rel(out, ref) < 1e-5, _rel(out, ref)
    assert torch.equal(store[:, n:], pad)  # the zero-fill and the reduce-adds stay inside the view


def test_gelu_mlp_matches_fp32() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    x = torch.randn(3, 100, 256, device=dev).bfloat16().requires_grad_(True)
    w1 = (torch.randn(512, 256, device=dev) * 0.05).requires_grad_(True)
    b1 = (torch.randn(512, device=dev) * 0.1).requires_grad_(True)
    w2 = (torch.randn(256, 512, device=dev) * 0.05).requires_grad_(True)
    b2 = (torch.randn(256, device=dev) * 0.1).requires_grad_(True)
    y = ops.gelu_mlp(x, w1, b1, w2, b2)
    ref_in = [t.detach().float().cpu().requires_grad_(True) for t in (x, w1, b1, w2, b2)]
    xr, w1r, b1r, w2r, b2r = ref_in
    h = F.gelu(xr @ w1r.bfloat16().float().t() + b1r, approximate="tanh")
    ref = h @ w2r.bfloat16().float().t() + b2r
    assert _rel(y, ref) < 2e-2, _rel(y, ref)
    g = torch.randn_like(ref)
    y.backward(g.to(dev).bfloat16())
    ref.backward(g.bfloat16().float())
    for got, want in zip((x, w1, b1, w2, b2), ref_in):
        assert _rel(got.grad, want.grad) < 3e-2, _rel(got.grad, want.grad)


@pytest.mark.parametrize("rows,k,f,bias", [(300, 256, 256, True), (1024, 512, 384, False), (77, 64, 128, True)])
def test_swiglu_mlp_matches_fp32(rows: int, k: int, f: int, bias: bool) -> None:
    """SwiGLU inside fc1's epilogue and its gradient inside fc2's data-gradient epilogue, against fp32 torch."""
    ops = _ops()
    dev = torch.device("cuda")
    x = torch.randn(rows, k, device=dev).bfloat16().requires_grad_(True)
    w1 = (torch.randn(2 * f, k, device=dev) * 0.08).requires_grad_(True)
    b1 = (torch.randn(2 * f, device=dev) * 0.1).requires_grad_(True) if bias else None
    w2 = (torch.randn(k, f, device=dev) * 0.08).requires_grad_(True)
    b2 = (torch.randn(k, device=dev) * 0.1).requires_grad_(True) if bias else None
    params = [t for t in (x, w1, b1, w2, b2) if t is not None]
    y = ops.swiglu_mlp(x, w1, b1, w2, b2)
    ref_in = [t.detach().float().cpu().requires_grad_(True) for t in params]
    xr, w1r, w2r = ref_in[0], ref_in[1], ref_in[3 if bias else 2]
    b1r, b2r = (ref_in[2], ref_in[4]) if bias else (None, None)
    h = xr @ w1r.bfloat16().float().t() + (b1r if bias else 0.0)
    gate, up = h[:, :f], h[:, f:]
    ref = (F.silu(gate) * up) @ w2r.bfloat16().float().t() + (b2r if bias else 0.0)
    assert _rel(y, ref) < 2e-2, _rel(y, ref)
    # the saved pre-activations are exactly the fused GEMM's h
    hh, a = ops.swiglu_gemm(x.detach(), w1.detach().bfloat16(), None if b1 is None else b1.detach())
    assert _rel(hh, h.detach()) < 1e-2 and _rel(a, F.silu(gate) * up) < 2e-2
    g = torch.randn_like(ref)
    y.backward(g.to(dev).bfloat16())
    ref.backward(g.bfloat16().float())
    for got, want in zip(params, ref_in):
        assert _rel(got.grad, want.grad) < 3e-2, _rel(got.grad, want.grad)


@pytest.mark.parametrize("d,hkv,causal,fast", [(64, 4, True, False), (64, 4, True, True), (128, 2, True, False),
                                               (64, 4, False, True)])
def test_attention_query_windows_compose_the_full_attention(d: int, hkv: int, causal: bool, fast: bool) -> None:
    """Query windows (one context-parallel rank each) reproduce the full kernel: outputs of the window
    rows, dQ of the window rows, and dK / dV summed over the windows, against an fp32 torch oracle."""
    from hybrid_training.ops.attention import attention_window_backward, attention_window_forward, reference_attention

    torch.manual_seed(0)
    dev = torch.device("cuda")
    b, s, h = 2, 512, 8
    w = (h + 2 * hkv) * d
    qkv = (torch.randn(b, s, w, device=dev) * 0.5).bfloat16()
    dout = torch.randn(b, s, h * d, device=dev).bfloat16()
    ref_in = qkv.float().cpu().requires_grad_(True)
    ref = reference_attention(ref_in, h, hkv, d, causal=causal)
    ref.float().backward(dout.float().cpu())
    out = torch.zeros(b, s, h * d)
    dq = torch.zeros(b, s, h * d)
    dkv = torch.zeros(b, s, w - h * d)
    ops = _ops()
    ops.set_deterministic_reductions(not fast)  # fast: the fused D = 64 backward kernel
    try:
        for begin, length in ((0, 128), (128, 256), (384, 128)):
            o_full, lse = attention_window_forward(qkv, h, hkv, d, begin, length, causal)
            assert torch.count_nonzero(o_full[:, :begin]) == 0 and torch.count_nonzero(o_full[:, begin + length:]) == 0
            out[:, begin:begin + length] = o_full[:, begin:begin + length].float().cpu()
            g = attention_window_backward(qkv, o_full, lse, dout[:, begin:begin + length], h, hkv, d, begin, length, causal)
            dq[:, begin:begin + length] = g[:, begin:begin + length, : h * d].float().cpu()
            dkv += g[..., h * d:].float().cpu()
    finally:
        ops.set_deterministic_reductions(True)
    assert _rel(out, ref) < 2e-2, _rel(out, ref)
    assert _rel(dq, ref_in.grad[..., : h * d]) < 3e-2
    assert _rel(dkv, ref_in.grad[..., h * d:]) < 3e-2


def test_column_sum_and_sum_rows() -> None:
    ops = _ops()
    ext = ops.extension()
    dev = torch.device("cuda")
    for rows, cols, dt in ((8192, 768, torch.bfloat16), (1000, 3000, torch.bfloat16), (777, 130, torch.float32), (5, 7, torch.bfloat16)):
        x = torch.randn(rows, cols, device=dev).to(dt)
        out = torch.randn(cols, device=dev)
        base = out.clone()
        ext.column_sum(x, out, 1.0)
        ref = x.float().sum(0) + base
        assert _rel(out, ref) < 1e-5, (rows, cols, _rel(out, ref))
        ext.column_sum(x, out, 0.0)
        assert _rel(out, x.float().sum(0)) < 1e-5


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_split_k_long_reduction_with_many_tiles(out_dtype: torch.dtype) -> None:
    """80 output tiles (more than half the SMs) and K = 8192: split three ways so the last wave fills."""
    ops = _ops()
    dev = torch.device("cuda")
    m, n, k = 1280, 2048, 8192
    a = torch.randn(m, k, device=dev).bfloat16()
    b = torch.randn(n, k, device=dev).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=out_dtype)
    ops.gemm(a, b, out=out)
    ref = a.float() @ b.float().t()
    err = float((out.float() - ref).abs().max()) / float(ref.abs().max())
    assert err < (1e-5 if out_dtype == torch.float32 else 1e-2), err


def test_gemm_unaligned_output_rows_use_the_scalar_store_path() -> None:
    """Output rows whose stride is not a multiple of 16 bytes cannot use TMA or vector stores."""
    ops = _ops()
    dev = torch.device("cuda")
    a = torch.randn(300, 64, device=dev).bfloat16()
    b = torch.randn(333, 64, device=dev).bfloat16()
    for dtype in (torch.bfloat16, torch.float32):
        store = torch.full((300, 333), 7.0, device=dev, dtype=dtype)  # row stride 666 / 1332 bytes
        ops.gemm(a, b, out=store)
        ref = a.float() @ b.float().t()
        assert _rel(store, ref) < 1e-2, dtype
        acc = torch.ones(300, 333, device=dev)
        ops.gemm(a, b, out=acc, beta=1.0)  # accumulate into an fp32 output
        assert _rel(acc, ref + 1.0) < 1e-2


def test_gemm_padded_output_rows() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    a = torch.randn(64, 128, device=dev).bfloat16()
    b = torch.randn(1003, 128, device=dev).bfloat16()
    store = torch.zeros(64, 1024, device=dev, dtype=torch.bfloat16)
    ops.gemm(a, b, out=store[:, :1003])
    ref, _ = ops.reference_gemm(a, b)
    assert _rel(store[:, :1003], ref) < 1e-2
    assert float(store[:, 1003:].abs().max()) == 0.0


def _torch_add_norm(res: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, eps: float,
                    rms: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 PyTorch statement of the fused op: r = res + delta, y = LayerNorm(r) or RMSNorm(r)."""
    r = res + delta.float()
    if rms:
        y = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps) * w
    else:
        y = torch.nn.functional.layer_norm(r, (r.shape[-1],), w, b, eps)
    return r, y


@pytest.mark.parametrize("rms", [False, True])
@pytest.mark.parametrize("d", [768, 100, 2048, 8192])
def test_add_norm_forward_backward(rms: bool, d: int) -> None:
    ops = _ops()
    dev = torch.device("cuda")
    rows = 37
    res = torch.randn(rows, d, device=dev, requires_grad=True)
    delta = torch.randn(rows, d, device=dev).bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(d, device=dev)).requires_grad_(True)
    b = None if rms else (0.1 * torch.randn(d, device=dev)).requires_grad_(True)
    r, y = ops.add_norm(res, delta, w, b, eps=1e-5, rms=rms, out_dtype=torch.bfloat16)
    res_c, delta_c = res.detach().double().cpu().requires_grad_(True), delta.detach().double().cpu().requires_grad_(True)
    w_c = w.detach().double().cpu().requires_grad_(True)
    b_c = None if b is None else b.detach().double().cpu().requires_grad_(True)
    r_ref, y_ref = _torch_add_norm(res_c, delta_c, w_c, b_c, 1e-5, rms)
    assert _rel(r, r_ref) < 1e-6 and _rel(y, y_ref) < 1e-2
    gy = torch.randn(rows, d, dtype=torch.float64)
    gr = torch.randn(rows, d, dtype=torch.float64)
    torch.autograd.backward([r, y], [gr.float().to(dev), gy.to(dev).bfloat16()])
    torch.autograd.backward([r_ref, y_ref], [gr, gy.bfloat16().double()])
    assert _rel(res.grad, res_c.grad) < 1e-2
    assert _rel(delta.grad, delta_c.grad) < 2e-2
    assert _rel(w.grad, w_c.grad) < 1e-2
    if b is not None:
        assert _rel(b.grad, b_c.grad) < 1e-2


@pytest.mark.parametrize("d,h,hkv,s,causal", [(64, 4, 4, 128, True), (64, 4, 2, 100, True), (128, 4, 1, 192, True),
                                               (128, 2, 2, 64, True), (64, 2, 1, 700, True), (64, 2, 2, 300, False),
                                               (128, 2, 1, 260, False)])
def test_attention_forward_backward(d: int, h: int, hkv: int, s: int, causal: bool) -> None:
    ops = _ops()
    dev = torch.device("cuda")
    bsz = 2
    qkv = (torch.randn(bsz, s, (h + 2 * hkv) * d, device=dev) * 0.5).bfloat16().requires_grad_(True)
    out = ops.attention(qkv, h, hkv, d, causal=causal)
    ref_in = qkv.detach().float().cpu().requires_grad_(True)
    ref = ops.reference_attention(ref_in, h, hkv, d, causal=causal)
    assert _rel(out, ref) < 2e-2, _rel(out, ref)
    g = torch.randn_like(ref)
    out.backward(g.to(dev).bfloat16())
    ref.backward(g.bfloat16().float())
    assert _rel(qkv.grad, ref_in.grad) < 3e-2, _rel(qkv.grad, ref_in.grad)


@pytest.mark.parametrize("h,hkv,s,causal", [(4, 4, 128, True), (4, 2, 100, True), (2, 1, 700, True), (2, 2, 300, False),
                                             (12, 12, 1024, True), (3, 3, 260, False)])
def test_attention_backward_fused_kernel(h: int, hkv: int, s: int, causal: bool) -> None:
    """D = 64 backward as one kernel (dQ summed by reduce-adds) against fp32 PyTorch and the two-kernel path."""
    ops = _ops()
    dev = torch.device("cuda")
    d, bsz = 64, 2
    qkv0 = (torch.randn(bsz, s, (h + 2 * hkv) * d, device=dev) * 0.5).bfloat16()
    g = torch.randn(bsz, s, h * d, device=dev).bfloat16()
    grads = {}
    for deterministic in (True, False):
        qkv = qkv0.clone().requires_grad_(True)
        try:
            ops.set_deterministic_reductions(deterministic)
            out = ops.attention(qkv, h, hkv, d, causal=causal)
            out.backward(g)
        finally:
            ops.set_deterministic_reductions(True)
        grads[deterministic] = qkv.grad.float()
    ref_in = qkv0.float().cpu().requires_grad_(True)
    ref = ops.reference_attention(ref_in, h, hkv, d, causal=causal)
    ref.backward(g.float().cpu())
    q_cols, kv_cols = h * d, hkv * d
    for name, sl in (("dq", slice(0, q_cols)), ("dk", slice(q_cols, q_cols + kv_cols)), ("dv", slice(q_cols + kv_cols, None))):
        fused, ordered, want = grads[False][..., sl], grads[True][..., sl], ref_in.grad[..., sl]
        assert _rel(fused, want) < 3e-2, (name, _rel(fused, want))
        assert _rel(fused, ordered) < 2e-2, (name, _rel(fused, ordered))


def test_attention_lse_and_error_word() -> None:
    """The forward's log-sum-exp (used by the backward) and the kernel's timeout word."""
    ops = _ops()
    ext = ops.extension()
    dev = torch.device("cuda")
    b, s, h, hkv, d = 2, 384, 4, 2, 64
    qkv = (torch.randn(b, s, (h + 2 * hkv) * d, device=dev) * 0.5).bfloat16()
    out = torch.empty(b, s, h * d, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(b, h, s, device=dev)
    ext.attention_forward(qkv, out, lse, h, hkv, d, True, 1.0 / math.sqrt(d))
    q = qkv[..., : h * d].float().view(b, s, h, d).transpose(1, 2)
    k = qkv[..., h * d:(h + hkv) * d].float().view(b, s, hkv, d).transpose(1, 2).repeat_interleave(h // hkv, dim=1)
    scores = (q @ k.transpose(-1, -2)) / math.sqrt(d)
    scores = scores.masked_fill(torch.triu(torch.ones(s, s, dtype=torch.bool, device=dev), 1), float("-inf"))
    ref = torch.logsumexp(scores, dim=-1)
    assert float((lse - ref).abs().max()) < 1e-2
    assert int(ext.attention_error_word(qkv).abs().sum()) == 0


def test_head_cross_entropy_matches_torch() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    rows, d, v = 300, 128, 1003
    h = torch.randn(rows, d, device=dev).bfloat16().requires_grad_(True)
    w = (torch.randn(v, d, device=dev) * 0.05).requires_grad_(True)
    t = torch.randint(0, v, (rows,), device=dev)
    loss = ops.lm_head_cross_entropy(h, w, t)
    hr, wr = h.detach().float().cpu().requires_grad_(True), w.detach().cpu().requires_grad_(True)
    ref = F.cross_entropy(hr @ wr.bfloat16().float().t(), t.cpu())
    assert abs(float(loss) - float(ref)) < 2e-2
    (loss * 2.0).backward()
    (ref * 2.0).backward()
    assert _rel(h.grad, hr.grad) < 3e-2 and _rel(w.grad, wr.grad) < 3e-2


def test_adamw_flat_matches_reference() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    n = 4096 + 64
    p, g = torch.randn(n, device=dev), torch.randn(n, device=dev)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    copy = torch.empty(n, device=dev, dtype=torch.bfloat16)
    pr, mr, vr = p.cpu().clone(), m.cpu().clone(), v.cpu().clone()
    for step in (1, 2, 3):
        hyper = torch.tensor([1e-2, float(step), 0.5, 0.0], device=dev)
        ops.adamw_flat(p, g, m, v, copy, hyper, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
        ops.reference_adamw(pr, g.cpu(), mr, vr, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=step,
                            grad_scale=0.5)
    assert torch.allclose(p.cpu(), pr, atol=1e-5) and torch.allclose(copy.float().cpu(), pr, atol=1e-2)


def test_embedding_swiglu_rope() -> None:
    ops = _ops()
    dev = torch.device("cuda")
    ids = torch.randint(0, 50, (3, 17), device=dev)
    table = torch.randn(40, 24, device=dev, requires_grad=True)
    pos = torch.randn(32, 24, device=dev, requires_grad=True)
    out = ops.embedding(ids, table, pos, vocab_start=10)
    # fp32 PyTorch statement: rows [10, 50) of the vocabulary live here, others contribute zero.
    local = ids.cpu() - 10
    owned = (local >= 0) & (local < 40)
    t_c, p_c = table.detach().cpu(), pos.detach().cpu()
    ref = torch.where(owned[..., None], t_c[local.clamp(0, 39)], torch.zeros(())) + p_c[:17][None]
    assert torch.allclose(out.cpu(), ref, atol=1e-6)
    g = torch.randn(3, 17, 24)
    out.backward(g.to(dev))
    table_grad = torch.zeros(40, 24).index_add_(0, local[owned], g[owned])
    pos_grad = torch.zeros(32, 24)
    pos_grad[:17] = g.sum(0)
    assert torch.allclose(table.grad.cpu(), table_grad, atol=1e-5)
    assert torch.allclose(pos.grad.cpu(), pos_grad, atol=1e-5)
    h = torch.randn(5, 7, 64, device=dev).bfloat16().requires_grad_(True)
    y = ops.swiglu(h)
    hr = h.detach().float().cpu().requires_grad_(True)
    gate, up = hr[..., :32], hr[..., 32:]
    yr = torch.nn.functional.silu(gate) * up
    assert _rel(y, yr) < 1e-2
    y.float().sum().backward()
    yr.sum().backward()
    assert _rel(h.grad, hr.grad) < 2e-2
    cos, sin = ops.rope_tables(16, 64, 10000.0, dev)
    qkv = torch.randn(2, 16, (2 + 2) * 64, device=dev).bfloat16()
    rot = ops.apply_rope(qkv, cos, sin, 2, 1, 64)
    # Rotate-half RoPE written out: angle(position t, pair i) = t * theta^(-2i / D).
    inv = 10000.0 ** (-torch.arange(0, 64, 2, dtype=torch.float64) / 64)
    ang = torch.arange(16, dtype=torch.float64)[:, None] * inv[None]
    c, s_ = torch.cat([ang.cos(), ang.cos()], -1), torch.cat([ang.sin(), ang.sin()], -1)
    x = qkv.double().cpu().reshape(2, 16, 4, 64)
    qk = x[:, :, :3]
    rotated = torch.cat([-qk[..., 32:], qk[..., :32]], -1)
    rot_ref = torch.cat([qk * c[None, :, None] + rotated * s_[None, :, None], x[:, :, 3:]], 2).reshape(2, 16, 256)
    assert _rel(rot, rot_ref) < 1e-2
    assert torch.equal(rot[..., 192:], qkv[..., 192:])  # values untouched


def test_fma_pipe_exp2_is_within_its_error_bound() -> None:
    """The polynomial 2^x that shares the softmax exponentials with the MUFU unit, against exp2f."""
    ops = _ops()
    ext = ops.extension()
    dev = torch.device("cuda")
    x = torch.cat([torch.linspace(-126.0, 0.0, 1 << 20, device=dev), -torch.rand(1 << 20, device=dev) * 40,
                   torch.tensor([0.0, -0.5, -0.49999997, -1.0, -125.5, -126.0, -200.0, float("-inf")], device=dev)])
    poly, mufu = torch.empty_like(x), torch.empty_like(x)
    ext.exp2_poly_eval(x, poly, mufu)
    exact = torch.exp2(x.double())
    normal = exact > 2.0 ** -125
    rel = ((poly.double() - exact).abs() / exact)[normal]
    assert float(rel.max()) < 1.1e-4, float(rel.max())  # the fitted bound is 1.0e-4
    assert float(((mufu.double() - exact).abs() / exact)[normal].max()) < 1e-5
    assert float(poly[~normal].abs().max()) < 2.0 ** -124  # clamped inputs underflow towards zero
    assert torch.isfinite(poly).all() and (poly >= 0).all()
