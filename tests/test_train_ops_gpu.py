"""The training-side operators (freeml_b200/csrc/train_ops.cu, the backward
pass, loss and optimiser step of Model::Run(input, target)) against plain
PyTorch fp32 restatements of the reference functions they follow."""
import ctypes

import numpy as np
import pytest
import torch

from freeml_b200 import _lib

pytestmark = pytest.mark.gpu


def p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.fixture(autouse=True)
def _dev():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)


def test_matmul_left_batched_strided():
    """Mul<Left> / MatMul_Strided<Left>: out = L^T R per plane, row strides."""
    B, K, M, N, lda, ldb = 3, 37, 70, 45, 80, 50
    a = torch.randn(B, K, lda, device="cuda")
    b = torch.randn(B, K, ldb, device="cuda")
    out = torch.full((B, M, N + 3), 7.0, device="cuda")
    _lib.call("fml_matmul_left", p(out), p(a), p(b), M, N, K, lda, ldb, N + 3, B, K * lda, K * ldb, M * (N + 3), None)
    ref = torch.einsum("bkm,bkn->bmn", a[:, :, :M].double(), b[:, :, :N].double()).float()
    torch.testing.assert_close(out[:, :, :N], ref, rtol=1e-5, atol=1e-4)
    assert (out[:, :, N:] == 7.0).all()


def test_gelu_derivative():
    x = torch.randn(10007, device="cuda") * 3
    out = torch.empty_like(x)
    _lib.call("fml_gelu_derivative", p(out), p(x), x.numel(), None)
    xd = x.double()
    ref = 0.5 * (1 + torch.erf(xd / np.sqrt(2))) + xd * torch.exp(-0.5 * xd * xd) / np.sqrt(2 * np.pi)
    torch.testing.assert_close(out.double(), ref, rtol=1e-5, atol=1e-6)


def test_softmax_backward():
    rows, cols = 77, 130
    y = torch.softmax(torch.randn(rows, cols, device="cuda"), dim=1)
    g = torch.randn(rows, cols, device="cuda")
    out = torch.empty_like(y)
    _lib.call("fml_softmax_backward", p(out), p(y), p(g), rows, cols, None)
    ref = y * (g - (g * y).sum(dim=1, keepdim=True))
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)


def test_scatter_add_rows_accumulates():
    V, T, width = 50, 300, 96
    out = torch.randn(V, width, device="cuda")
    src = torch.randn(T, width, device="cuda")
    idx = torch.randint(0, V, (T,), device="cuda")
    ref = out.clone().index_add_(0, idx, src)
    _lib.call("fml_scatter_add_rows", p(out), p(src), p(idx.float()), T, width, V, 1, 1, None)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("with_xhat", [True, False])
def test_layernorm_backward(with_xhat):
    rows, cols = 64, 200
    x = torch.randn(rows, cols, device="cuda", dtype=torch.float64) * 2 + 0.5
    gamma = (1 + 0.1 * torch.randn(cols, device="cuda", dtype=torch.float64))
    dy = torch.randn(rows, cols, device="cuda", dtype=torch.float64)
    xr = x.clone().requires_grad_(True)
    gr = gamma.clone().requires_grad_(True)
    y = torch.nn.functional.layer_norm(xr, (cols,), weight=gr, bias=None, eps=1e-5)
    y.backward(dy)
    xf, gf, dyf = x.float(), gamma.float(), dy.float()
    mean = xf.mean(dim=1, keepdim=True)
    xhat = (xf - mean) / torch.sqrt(((xf - mean) ** 2).mean(dim=1, keepdim=True) + 1e-5)
    dx = torch.empty_like(xf)
    dgamma = torch.empty(cols, device="cuda")
    dbeta = torch.empty(cols, device="cuda")
    ws = torch.empty(2 * rows, device="cuda")
    _lib.call("fml_layernorm_backward", p(dx), p(dyf), p(xf), p(gf), p(dgamma), p(dbeta),
              p(xhat) if with_xhat else None, rows, cols, 1e-5, p(ws), None)
    torch.testing.assert_close(dx.double(), xr.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dgamma.double(), gr.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dbeta.double(), dy.sum(dim=0), rtol=1e-4, atol=1e-4)


def test_adamw_update():
    n = 5000
    param = torch.randn(n, device="cuda") * 0.02
    grad = torch.randn(n, device="cuda") * 1e-2
    mt = torch.randn(n, device="cuda") * 1e-3
    vt = torch.rand(n, device="cuda") * 1e-4
    lr, b1, b2, eps, wd, t = 1e-3, 0.9, 0.999, 1e-8, 0.01, 3
    # the hyperparameters as the kernel (and the reference, all in T = float)
    # sees them: 1 - beta is formed in fp32
    f = lambda x: float(np.float32(x))  # noqa: E731
    b1f, b2f = f(b1), f(b2)
    ib1, ib2 = f(np.float32(1) - np.float32(b1)), f(np.float32(1) - np.float32(b2))
    b1p, b2p = f(b1 ** t), f(b2 ** t)
    P, G, Mt, Vt = (x.double() for x in (param, grad, mt, vt))
    m = b1f * Mt + ib1 * G
    v = b2f * Vt + ib2 * G * G
    ref = P + f(lr) * (m / f(1 - b1p)) / (torch.sqrt(v / f(1 - b2p)) + f(eps)) - f(lr) * f(wd) * P
    _lib.call("fml_adamw_update", p(param), p(grad), p(mt), p(vt), n, lr, b1, b2, b1p, b2p, eps, wd, None)
    torch.testing.assert_close(param.double(), ref, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(mt.double(), m, rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(vt.double(), v, rtol=1e-5, atol=1e-11)


@pytest.mark.parametrize("ids", [1, 0])
def test_cross_entropy_with_logits(ids):
    """Gradient (onehot - softmax) [/ valid rows] and loss (mean over valid id
    rows, or sum over dense-target rows), with an ignored row (-1)."""
    steps, planes, vocab = 33, 2, 301
    logits = torch.randn(planes, steps, vocab, device="cuda") * 3
    tid = torch.randint(0, vocab, (planes, steps), device="cuda")
    if ids:
        tid[1, 5] = -1
        target = tid.float()
    else:
        target = torch.nn.functional.one_hot(tid, vocab).float()
    grad = torch.empty_like(logits)
    ws = torch.empty(planes * steps + 1, device="cuda")
    loss = ctypes.c_float(0.0)
    _lib.call("fml_xent_with_logits", p(grad), ctypes.byref(loss), p(target), p(logits), vocab, steps, planes, planes,
              ids, p(ws), None)
    lg = logits.double().reshape(-1, vocab)
    t = tid.reshape(-1)
    prob = torch.softmax(lg, dim=1)
    valid = t != -1
    onehot = torch.nn.functional.one_hot(t.clamp(min=0), vocab).double() * valid[:, None]
    if ids:
        ref_grad = (onehot - prob) / valid.sum() * valid[:, None]
        ref_loss = torch.nn.functional.cross_entropy(lg[valid], t[valid], reduction="mean")
    else:
        ref_grad = onehot - prob
        ref_loss = torch.nn.functional.cross_entropy(lg, t, reduction="sum")
    torch.testing.assert_close(grad.reshape(-1, vocab).double(), ref_grad, rtol=1e-4, atol=1e-6)
    assert abs(loss.value - ref_loss.item()) <= 1e-4 * abs(ref_loss.item()) + 1e-5


def test_merge_qkv():
    heads, tokens, hd = 4, 37, 32
    q, k, v = (torch.randn(heads, tokens, hd, device="cuda") for _ in range(3))
    packed = torch.empty(tokens, 3 * heads * hd, device="cuda")
    _lib.call("fml_merge_qkv", p(packed), p(q), p(k), p(v), hd, tokens, heads, None)
    ref = torch.cat([x.permute(1, 0, 2).reshape(tokens, heads * hd) for x in (q, k, v)], dim=1)
    assert torch.equal(packed, ref)
