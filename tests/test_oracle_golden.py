"""Pins the C oracle (oracle/freeml_oracle.c) against golden vectors that the
unmodified FreeML MatrixCPU path produced (tests/golden/make_golden.py).

The bar is bit-exactness: the oracle keeps the reference's fp32 evaluation
order, so every weight, logit and token must match to the last bit."""
import hashlib

import numpy as np
import pytest

from oracle import oracle as O


def _shape(m):
    return O.LMShape(V=m["V"], C=m["C"], d=m["d"], H=m["H"], L=m["L"])


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", ["cfg1", "odd"])
def test_weights_bit_exact(golden, name):
    meta, _, _ = golden
    m = meta["greedy"][name]
    w = O.init_weights(_shape(m), m["wseed"])
    assert w.size == m["weights_count"]
    assert _sha(w) == m["weights_sha256"]


def test_config3_weights_bit_exact(golden):
    meta, _, _ = golden
    m = meta["weights_sha256"]["cfg3"]
    w = O.init_weights(_shape(m), m["wseed"])
    assert w.size == m["count"]
    assert [float(x) for x in w[:8]] == m["first8"]
    assert _sha(w) == m["sha256"]


@pytest.mark.parametrize("name", ["cfg1", "odd"])
def test_prompt_recipe(golden, name):
    meta, g, _ = golden
    m = meta["greedy"][name]
    p = O.prompt_tokens(m["pseed"], m["V"], m["plen"])
    np.testing.assert_array_equal(p, g[f"{name}_prompt"])
    np.testing.assert_array_equal(p, np.random.RandomState(m["pseed"]).randint(0, m["V"], m["plen"]))


@pytest.mark.parametrize("name", ["cfg1", "odd"])
def test_greedy_loop_bit_exact(golden, name):
    meta, g, _ = golden
    m = meta["greedy"][name]
    s = _shape(m)
    w = O.init_weights(s, m["wseed"])
    toks, logits = O.greedy(s, w, g[f"{name}_prompt"], m["new"])
    np.testing.assert_array_equal(toks, g[f"{name}_tokens"])
    np.testing.assert_array_equal(logits, g[f"{name}_logits"])


@pytest.mark.parametrize("name", ["cfg1", "odd"])
def test_full_window_forward_bit_exact(golden, name):
    """One forward over the zero-padded C window (what Model::Run computes);
    the oracle's shorter window gives the same causal rows."""
    meta, g, _ = golden
    m = meta["greedy"][name]
    s = _shape(m)
    w = O.init_weights(s, m["wseed"])
    window = np.zeros(s.C, np.uint32)
    window[: m["plen"] + m["new"]] = g[f"{name}_tokens"]
    full = O.forward(s, w, window)
    np.testing.assert_array_equal(full, g[f"{name}_window_logits"])
    n = m["plen"] + m["new"] - 3
    part = O.forward(s, w, window[:n])
    np.testing.assert_array_equal(part, g[f"{name}_window_logits"][:n])


def test_ops_bit_exact(golden):
    _, _, o = golden
    A, B, Bt, gam, beta = o["A"], o["B"], o["Bt"], o["gamma"], o["beta"]
    np.testing.assert_array_equal(O.op_mul(A, B, 0), o["mul_none"])
    np.testing.assert_array_equal(O.op_mul(A, Bt, 1), o["mul_right"])
    np.testing.assert_array_equal(O.op_mul(o["small"], o["small_B"], 0), o["mul_none_small"])
    np.testing.assert_array_equal(O.op_layernorm(A, gam), o["layernorm"])
    np.testing.assert_array_equal(O.op_layernorm(A, gam, beta), o["layernorm_beta"])
    np.testing.assert_array_equal(O.op_softmax(A), o["softmax"])
    np.testing.assert_array_equal(O.op_gelu(A), o["gelu"])
    np.testing.assert_array_equal(O.op_add(A, A[::-1].copy()), o["add"])
    np.testing.assert_array_equal(O.op_scale_add(o["S"], float(o["scale"][0]), o["mask"]), o["scale_add"])
    np.testing.assert_array_equal(O.op_gather_rows(o["table"], o["idx"]), o["gather_rows"])


def test_strided_attention_pieces(golden):
    _, _, o = golden
    Q, K, P = o["attn_Q"], o["attn_K"], o["attn_P"]
    hd, h = 16, 1
    qh, kh = Q[:, h * hd:(h + 1) * hd], K[:, h * hd:(h + 1) * hd]
    np.testing.assert_array_equal(O.op_mul(qh, kh, 1), o["strided_right_h1"])
    y = np.zeros_like(Q)
    y[:, h * hd:(h + 1) * hd] = O.op_mul(P, kh, 0)
    np.testing.assert_array_equal(y, o["strided_none_h1"])


def test_split_qkv(golden):
    _, _, o = golden
    pk = o["packed"]
    np.testing.assert_array_equal(pk[:, :32], o["split_q"])
    np.testing.assert_array_equal(pk[:, 32:64], o["split_k"])
    np.testing.assert_array_equal(pk[:, 64:], o["split_v"])


def test_argmax_tie_rule():
    row = np.array([0.0, 3.0, 1.0, 3.0], np.float32)
    assert O.argmax_first(row) == 1
    assert O.argmax_first(np.zeros(7, np.float32)) == 0


def test_known_answers():
    # LayerNorm of a constant row is 0; softmax of a one-hot-dominant row; Gelu(0) = 0
    np.testing.assert_array_equal(O.op_layernorm(np.full((2, 8), 3.0, np.float32), np.ones(8, np.float32)),
                                  np.zeros((2, 8), np.float32))
    p = O.op_softmax(np.array([[0.0, -np.inf, 0.0, -np.inf]], np.float32))
    np.testing.assert_array_equal(p, np.array([[0.5, 0.0, 0.5, 0.0]], np.float32))
    assert O.op_gelu(np.zeros(3, np.float32)).tolist() == [0.0, 0.0, 0.0]
