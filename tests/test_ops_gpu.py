"""Per-operator parity: the sm_100a kernels behind the C ABI against the
reference's own outputs (golden fixtures from FreeML's MatrixCPU path) and
the C oracle on seeded random shapes.

fp32 bound: |gpu - ref| <= 1e-5 + 1e-5 |ref| for the elementwise/row ops
(only reduction order differs), 1e-4 relative-to-scale for contractions."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _lib_loaded():
    from freeml_b200 import _lib
    _lib.load()


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(got, ref, rtol=1e-5, atol=1e-5):
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol)


def gemm_close(got, ref, A, B):
    # contraction bound scaled by sum |a||b| (order-independent error bound)
    scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-5 * scale + 1e-6)


def test_golden_ops(golden):
    from freeml_b200 import matrix_ops as F
    _, _, o = golden
    A, B, Bt, g, beta = o["A"], o["B"], o["Bt"], o["gamma"], o["beta"]
    M, K = A.shape
    out = torch.empty(M, B.shape[1], device="cuda")
    F.Mul(out, cu(A), cu(B), F.NONE)
    gemm_close(host(out), o["mul_none"], A, B)
    out = torch.empty(M, Bt.shape[0], device="cuda")
    F.Mul(out, cu(A), cu(Bt), F.RIGHT)
    gemm_close(host(out), o["mul_right"], A, Bt.T)
    y = torch.empty(M, K, device="cuda")
    F.LayerNormOp(y, cu(A), cu(g))
    close(host(y), o["layernorm"], 2e-5, 2e-5)
    F.LayerNormOp(y, cu(A), cu(g), cu(beta))
    close(host(y), o["layernorm_beta"], 2e-5, 2e-5)
    F.Softmax(y, cu(A))
    close(host(y), o["softmax"])
    F.GeluMat(y, cu(A))
    close(host(y), o["gelu"], 1e-6, 1e-6)
    F.Add(y, cu(A), cu(A[::-1]))
    np.testing.assert_array_equal(host(y), o["add"])
    S = o["S"]
    s = torch.empty_like(cu(S))
    F.ScaleAdd(s, cu(S), cu(o["scale"]), cu(o["mask"]))
    np.testing.assert_array_equal(host(s), o["scale_add"])  # one fma per element, like the reference
    gr = torch.empty(o["idx"].size, o["table"].shape[1], device="cuda")
    F.GatherRows(gr, cu(o["table"]), cu(o["idx"]))
    np.testing.assert_array_equal(host(gr), o["gather_rows"])
    pk = o["packed"]
    q, k, v = (torch.empty(pk.shape[0], 32, device="cuda") for _ in range(3))
    F.SplitQKV(q, k, v, cu(pk))
    for t, name in ((q, "split_q"), (k, "split_k"), (v, "split_v")):
        np.testing.assert_array_equal(host(t), o[name])


def test_golden_strided_attention_pieces(golden):
    from freeml_b200 import matrix_ops as F
    _, _, o = golden
    Q, K, P = o["attn_Q"], o["attn_K"], o["attn_P"]
    T, d = Q.shape
    hd, h = 16, 1
    S = torch.zeros(T, T, device="cuda")
    # scores = Q_h K_h^T: head views at column offset h*hd with row stride d
    F.MatMul_Strided(S, cu(Q), cu(K), T, T, hd, d, d, T, F.RIGHT, off_a=h * hd, off_b=h * hd)
    gemm_close(host(S), o["strided_right_h1"], Q[:, h * hd:(h + 1) * hd], K[:, h * hd:(h + 1) * hd].T)
    Y = torch.zeros(T, d, device="cuda")
    F.MatMul_Strided(Y, cu(P), cu(K), T, hd, T, T, d, d, F.NONE, off_b=h * hd, off_c=h * hd)
    ref = o["strided_none_h1"]
    got = host(Y)
    np.testing.assert_array_equal(got[:, :h * hd], 0)
    gemm_close(got[:, h * hd:(h + 1) * hd], ref[:, h * hd:(h + 1) * hd], P, K[:, h * hd:(h + 1) * hd])


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (128, 512, 128), (130, 96, 260), (512, 1536, 512),
                                   (1, 512, 512), (8, 1024, 4096), (64, 4096, 1024), (33, 12, 2048), (5, 260, 100)])
@pytest.mark.parametrize("mode", [0, 1])
def test_matmul_vs_oracle(M, N, K, mode):
    """Tiled GEMM, and at <= 64 rows the small-batch kernels (split-K for
    Mul<None>, the decode GEMV for Mul<Right>), against the oracle."""
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(M * 7 + N * 3 + K + mode)
    A = rs.randn(M, K).astype(np.float32)
    B = (0.02 * rs.randn(*((N, K) if mode else (K, N)))).astype(np.float32)
    out = torch.empty(M, N, device="cuda")
    F.Mul(out, cu(A), cu(B), mode)
    ref = O.op_mul(A, B, mode)
    gemm_close(host(out), ref, A, B.T if mode else B)


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 33), (64, 512), (3, 4096), (17, 128), (9, 640), (5, 2048)])
def test_row_ops_vs_oracle(rows, cols):
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(rows + cols)
    x = (3 * rs.randn(rows, cols)).astype(np.float32)
    g = (1 + 0.1 * rs.randn(cols)).astype(np.float32)
    y = torch.empty(rows, cols, device="cuda")
    F.LayerNormOp(y, cu(x), cu(g))
    close(host(y), O.op_layernorm(x, g), 3e-5, 3e-5)
    F.Softmax(y, cu(x))
    close(host(y), O.op_softmax(x), 1e-5, 1e-6)
    F.GeluMat(y, cu(x))
    close(host(y), O.op_gelu(x), 1e-6, 1e-6)


def test_softmax_masked_rows():
    from freeml_b200 import matrix_ops as F
    x = np.array([[0.0, -np.inf, 0.0, -np.inf], [5.0, -np.inf, -np.inf, -np.inf]], np.float32)
    y = torch.empty(2, 4, device="cuda")
    F.Softmax(y, cu(x))
    np.testing.assert_array_equal(host(y), O.op_softmax(x))


def test_gather_rows_out_of_range_is_zero():
    from freeml_b200 import matrix_ops as F
    table = np.arange(12, dtype=np.float32).reshape(3, 4)
    idx = np.array([2, 7, 0], np.float32)
    out = torch.full((3, 4), 5.0, device="cuda")
    F.GatherRows(out, cu(table), cu(idx))
    np.testing.assert_array_equal(host(out), np.stack([table[2], np.zeros(4, np.float32), table[0]]))


def test_elementwise_and_fill():
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(0)
    a, b = rs.randn(1001).astype(np.float32), rs.randn(1001).astype(np.float32)
    y = torch.empty(1001, device="cuda")
    F.Add(y, cu(a), cu(b))
    np.testing.assert_array_equal(host(y), a + b)
    F.PerElementMul(y, cu(a), cu(b))
    np.testing.assert_array_equal(host(y), a * b)
    F.Scale(y, cu(a), 0.5)
    np.testing.assert_array_equal(host(y), a * np.float32(0.5))
    F.Fill(y, 3.0)
    assert np.all(host(y) == 3.0)
    F.Clear(y)
    assert np.all(host(y) == 0.0)
    m = rs.randn(6, 5).astype(np.float32)
    bias = rs.randn(5).astype(np.float32)
    z = torch.empty(6, 5, device="cuda")
    F.BroadcastAdd(z, cu(m), cu(bias))
    np.testing.assert_array_equal(host(z), m + bias)


def _attention_case(B, H, hd, C, lens, seed):
    rs = np.random.RandomState(seed)
    q = rs.randn(B, H * hd).astype(np.float32)
    kc = rs.randn(B, H, C, hd).astype(np.float32)
    vc = rs.randn(B, H, C, hd).astype(np.float32)
    return q, kc, vc, np.asarray(lens, np.int32)


def _attention_oracle(q, kc, vc, lens, scale):
    B, H, C, hd = kc.shape
    out = np.zeros((B, H * hd), np.float32)
    for b in range(B):
        n = int(lens[b])
        if n == 0:
            continue
        out[b] = O.attention_decode_ref(q[b].reshape(H, hd), kc[b, :, :n], vc[b, :, :n], scale).ravel()
    return out


@pytest.mark.parametrize("B,H,hd,C,lens", [
    (1, 8, 64, 128, [128]),    # config 2: 8 heads x hd 64, KV length 128
    (1, 8, 64, 512, [512]),    # ... 512
    (1, 8, 64, 2048, [2048]),  # ... 2048
    (3, 4, 32, 100, [1, 37, 100]),
    (2, 2, 128, 300, [300, 65]),
    (4, 8, 64, 512, [0, 1, 511, 512]),
])
def test_attention_decode_vs_oracle(B, H, hd, C, lens):
    from freeml_b200 import matrix_ops as F
    q, kc, vc, ln = _attention_case(B, H, hd, C, lens, B * 100 + C)
    scale = float(1.0 / np.sqrt(np.float32(hd)))
    out = torch.empty(B, H * hd, device="cuda")
    F.attention_decode(out, cu(q), cu(kc), cu(vc), torch.from_numpy(ln).cuda(), scale)
    ref = _attention_oracle(q, kc, vc, ln, np.float32(scale))
    close(host(out), ref, 2e-5, 2e-5)


@pytest.mark.parametrize("splits", [2, 3, 5, 8])
def test_attention_cluster_merge_matches_global_merge(monkeypatch, splits):
    """2..8 key splits run as one thread-block cluster per (row, head) and
    merge through distributed shared memory; the result is bit-identical to
    the global-partials merge (same arithmetic, same order) and matches the
    oracle, including empty rows and splits past a short row's keys."""
    from freeml_b200 import matrix_ops as F
    B, H, hd, C, lens = 4, 8, 64, 512, [0, 1, 300, 512]
    q, kc, vc, ln = _attention_case(B, H, hd, C, lens, 77)
    scale = float(1.0 / np.sqrt(np.float32(hd)))
    monkeypatch.setenv("FML_ATTN_SPLITS", str(splits))
    outs = []
    for cluster in ("1", "0"):
        monkeypatch.setenv("FML_ATTN_CLUSTER", cluster)
        out = torch.empty(B, H * hd, device="cuda")
        F.attention_decode(out, cu(q), cu(kc), cu(vc), torch.from_numpy(ln).cuda(), scale)
        outs.append(host(out))
    np.testing.assert_array_equal(outs[0], outs[1])
    close(outs[0], _attention_oracle(q, kc, vc, ln, np.float32(scale)), 2e-5, 2e-5)


def test_attention_decode_rejects_small_workspace():
    from freeml_b200 import FmlError
    from freeml_b200 import matrix_ops as F
    q, kc, vc, ln = _attention_case(1, 8, 64, 128, [128], 0)
    out = torch.empty(1, 512, device="cuda")
    with pytest.raises(FmlError):
        F.attention_decode(out, cu(q), cu(kc), cu(vc), torch.from_numpy(ln).cuda(), 0.125,
                           workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))


def _prefill_case(B, H, hd, C, P, seed, poison=False):
    rs = np.random.RandomState(seed)
    q = rs.randn(B * P, H * hd).astype(np.float32)
    kc = rs.randn(B, H, C, hd).astype(np.float32)
    vc = rs.randn(B, H, C, hd).astype(np.float32)
    if poison:  # cache rows past the prompt are never read into a result
        kc[:, :, P:] = np.nan
        vc[:, :, P:] = np.nan
    return q, kc, vc


def _prefill_oracle(q, kc, vc, P, scale):
    B, H, C, hd = kc.shape
    out = np.empty((B * P, H * hd), np.float32)
    for b in range(B):
        qb = q[b * P:(b + 1) * P].reshape(P, H, hd).transpose(1, 0, 2)
        ob = O.attention_prefill_ref(np.ascontiguousarray(qb), kc[b, :, :P], vc[b, :, :P], scale)
        out[b * P:(b + 1) * P] = ob.transpose(1, 0, 2).reshape(P, H * hd)
    return out


# tolerances against the fp32 oracle: outputs are convex combinations of
# unit-variance values, scores are sums of hd unit-variance products
PREFILL_TOL = {"fp32": 2e-5, "tf32x3": 1e-4, "tf32": 3e-2}


@pytest.mark.parametrize("B,H,hd,C,P", [
    (1, 2, 64, 300, 300),     # one partial 128-query tile after two full ones
    (2, 3, 32, 200, 130),
    (1, 2, 128, 260, 257),    # hd 128: 32-key tiles
    (3, 1, 64, 64, 1),        # one-row prompts
    (1, 4, 64, 512, 512),     # config 2's head shape
    (2, 2, 64, 1024, 777),
    (2, 2, 64, 256, 200),     # second query tile of a CTA ends past the prompt
    (1, 1, 64, 2048, 1536),   # config 4's prompt length
])
@pytest.mark.parametrize("mode", ["tf32x3", "fp32", "tf32"])
def test_attention_prefill_vs_oracle(B, H, hd, C, P, mode):
    """Prefill attention (fml_attention_prefill) in each math mode against the
    oracle's op-by-op restatement; in the TF32 modes the tcgen05 kernel,
    128-query tiles with prompts that end mid-tile.  Cache rows past the
    prompt hold NaN: they must not reach any output."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    q, kc, vc = _prefill_case(B, H, hd, C, P, B * 1000 + P + hd, poison=True)
    scale = float(1.0 / np.sqrt(np.float32(hd)))
    out = torch.full((B * P, H * hd), 7.0, device="cuda")
    m = {"fp32": _lib.FML_MATH_FP32, "tf32x3": _lib.FML_MATH_TF32X3, "tf32": _lib.FML_MATH_TF32}[mode]
    F.attention_prefill(out, cu(q), cu(kc), cu(vc), P, scale, m)
    got = host(out)
    ref = _prefill_oracle(q, kc, vc, P, np.float32(scale))
    assert np.isfinite(got).all()
    tol = PREFILL_TOL[mode]
    np.testing.assert_allclose(got, ref, rtol=tol, atol=tol)
    if mode == "tf32":
        assert np.abs(got - ref).max() > 1e-6  # it really is the reduced-precision path
    n = ctypes_u64()
    _lib.call("fml_device_error_count", ctypes.byref(n))
    assert n.value == 0


@pytest.mark.parametrize("mode", ["tf32x3", "tf32"])
def test_attention_prefill_one_tile_kernel_at_hd64(monkeypatch, mode):
    """At head dim 64 the TF32 modes run the two-tile warp-specialised
    kernel; FML_PREFILL_ATTN_SIMPLE=1 selects the one-tile kernel (the one
    head dims 32 and 128 use).  Both match the oracle."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    B, H, hd, C, P = 2, 2, 64, 640, 600
    q, kc, vc = _prefill_case(B, H, hd, C, P, 11, poison=True)
    scale = float(1.0 / np.sqrt(np.float32(hd)))
    m = {"tf32x3": _lib.FML_MATH_TF32X3, "tf32": _lib.FML_MATH_TF32}[mode]
    ref = _prefill_oracle(q, kc, vc, P, np.float32(scale))
    for simple in ("1", "0"):
        monkeypatch.setenv("FML_PREFILL_ATTN_SIMPLE", simple)
        out = torch.full((B * P, H * hd), 7.0, device="cuda")
        F.attention_prefill(out, cu(q), cu(kc), cu(vc), P, scale, m)
        np.testing.assert_allclose(host(out), ref, rtol=PREFILL_TOL[mode], atol=PREFILL_TOL[mode])


def test_attention_prefill_modes_agree_on_engine_shape():
    """Config 3's attention shape (12 heads x hd 64, 256-row prompts, 4
    sequences): the TF32x3 tensor-core kernel and the fp32 CUDA-core kernel
    agree to fp32 level."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    B, H, hd, C, P = 4, 12, 64, 1024, 256
    q, kc, vc = _prefill_case(B, H, hd, C, P, 5)
    scale = float(1.0 / np.sqrt(np.float32(hd)))
    outs = []
    for m in (_lib.FML_MATH_TF32X3, _lib.FML_MATH_FP32):
        out = torch.empty(B * P, H * hd, device="cuda")
        F.attention_prefill(out, cu(q), cu(kc), cu(vc), P, scale, m)
        outs.append(host(out))
    np.testing.assert_allclose(outs[0], outs[1], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (130, 96, 260), (512, 1536, 512), (4096, 512, 2048), (7, 300, 64),
                                   # decode sizes (<= 64 rows; the GEMV serves them in every math mode)
                                   (1, 1536, 512), (32, 2048, 512), (17, 132, 128)])
def test_matmul_tensor_core_tf32x3_vs_oracle(M, N, K):
    """Mul<Right> on tcgen05 (TF32x3): fp32-level accuracy."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(M + N + K)
    A = rs.randn(M, K).astype(np.float32)
    B = (0.02 * rs.randn(N, K)).astype(np.float32)
    out = torch.empty(M, N, device="cuda")
    prev = _lib.load().fml_get_math_mode()
    _lib.call("fml_set_math_mode", _lib.FML_MATH_TF32X3)
    try:
        F.Mul(out, cu(A), cu(B), F.RIGHT)
        got = host(out)
    finally:
        _lib.call("fml_set_math_mode", prev)
    ref = O.op_mul(A, B, 1)
    gemm_close(got, ref, A, B.T)
    n = ctypes_u64()
    _lib.call("fml_device_error_count", ctypes.byref(n))
    assert n.value == 0


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (130, 96, 260)])
def test_matmul_tensor_core_tf32_vs_oracle(M, N, K):
    """Mul<Right> on tcgen05, one TF32 product: within TF32 rounding
    (2^-10 relative per product, bounded by 2e-3 of sum |a||b|)."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(M * N + K)
    A = rs.randn(M, K).astype(np.float32)
    B = (0.02 * rs.randn(N, K)).astype(np.float32)
    out = torch.empty(M, N, device="cuda")
    prev = _lib.load().fml_get_math_mode()
    _lib.call("fml_set_math_mode", _lib.FML_MATH_TF32)
    try:
        F.Mul(out, cu(A), cu(B), F.RIGHT)
        got = host(out)
    finally:
        _lib.call("fml_set_math_mode", prev)
    ref = O.op_mul(A, B, 1)
    scale = np.abs(A).astype(np.float64) @ np.abs(B.T).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 2e-3 * scale + 1e-6)
    assert np.abs(got - ref).max() > 0  # it really is the reduced-precision path


def ctypes_u64():
    import ctypes
    return ctypes.c_uint64()


@pytest.fixture(params=["tf32x3", "fp32"])
def math_mode(request):
    """Run a contraction test in the TF32x3 tensor-core mode (the default)
    and in the fp32 CUDA-core mode, restoring the previous mode after."""
    from freeml_b200 import _lib
    prev = _lib.load().fml_get_math_mode()
    _lib.call("fml_set_math_mode", {"tf32x3": _lib.FML_MATH_TF32X3, "fp32": _lib.FML_MATH_FP32}[request.param])
    yield request.param
    _lib.call("fml_set_math_mode", prev)


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (128, 384, 128), (130, 96, 260), (512, 2048, 512),
                                   (512, 512, 2048), (200, 36, 64), (65, 1000, 96)])
def test_mul_none_vs_oracle(M, N, K, math_mode):
    """Mul<None> (Dense.h:207: x [M x K] . W [K x N], W in its stored
    row-major layout) above 64 rows: on tcgen05 in TF32x3 the weight tile is
    read N-major straight from that layout; partial 128-column tiles and a K
    that is not a multiple of the 32-wide stage included."""
    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(M * 5 + N + K)
    A = rs.randn(M, K).astype(np.float32)
    B = (0.02 * rs.randn(K, N)).astype(np.float32)
    out = torch.empty(M, N, device="cuda")
    before = _lib.launch_count()
    F.Mul(out, cu(A), cu(B), F.NONE)
    assert _lib.launch_count() > before
    gemm_close(host(out), O.op_mul(A, B, 0), A, B)
    n = ctypes_u64()
    _lib.call("fml_device_error_count", ctypes.byref(n))
    assert n.value == 0


@pytest.mark.parametrize("T,d,H", [(128, 128, 4), (512, 512, 8), (96, 64, 2)])
def test_attention_strided_pieces_vs_oracle(T, d, H, math_mode):
    """The per-head contractions of CausalSelfAttentionLayer.h:445-497 as the
    drop-in issues them (MatMul_Strided over head views with row stride d):
    scores S = Q_h K_h^T and Y_h = P V_h written into column block h of Y;
    tcgen05 above 64 rows in TF32x3."""
    from freeml_b200 import matrix_ops as F
    rs = np.random.RandomState(T + d + H)
    hd = d // H
    Q, Kc, V = (rs.randn(T, d).astype(np.float32) for _ in range(3))
    P = np.abs(rs.randn(T, T)).astype(np.float32)
    P /= P.sum(axis=1, keepdims=True)
    Y = torch.zeros(T, d, device="cuda")
    for h in (0, H - 1):
        S = torch.zeros(T, T, device="cuda")
        F.MatMul_Strided(S, cu(Q), cu(Kc), T, T, hd, d, d, T, F.RIGHT, off_a=h * hd, off_b=h * hd)
        qh, kh, vh = Q[:, h * hd:(h + 1) * hd], Kc[:, h * hd:(h + 1) * hd], V[:, h * hd:(h + 1) * hd]
        gemm_close(host(S), qh.astype(np.float64) @ kh.T.astype(np.float64), qh, kh.T)
        F.MatMul_Strided(Y, cu(P), cu(V), T, hd, T, T, d, d, F.NONE, off_b=h * hd, off_c=h * hd)
        got = host(Y)[:, h * hd:(h + 1) * hd]
        gemm_close(got, P.astype(np.float64) @ vh.astype(np.float64), P, vh)
    if H > 2:
        np.testing.assert_array_equal(host(Y)[:, hd:(H - 1) * hd], 0)  # other heads' columns untouched
