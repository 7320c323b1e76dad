"""Pins the PyTorch fp32 restatement (tests/torch_ref.py) against the
reference's golden greedy-loop logits, so that it can stand in for the C
oracle at config-5 size on the GPU."""
import numpy as np
import torch

from oracle import oracle as O
from tests import torch_ref


def test_torch_reference_matches_golden_logits(golden):
    meta, g, _ = golden
    for name in ("cfg1", "odd"):
        m = meta["greedy"][name]
        s = O.LMShape(m["V"], m["C"], m["d"], m["H"], m["L"])
        w = torch.from_numpy(O.init_weights(s, m["wseed"]))
        toks = g[f"{name}_tokens"]
        P, N = m["plen"], m["new"]
        ref = g[f"{name}_logits"]  # rows P-1 .. P+N-2
        got = torch_ref.forward(w, s.V, s.C, s.d, s.H, s.L, toks[: P + N - 1].astype(np.int64), P - 1, N).numpy()
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_torch_reference_matches_reference_build_at_config3_shape():
    """The restatement against FreeML itself (oracle/_ref/ref_nanollm: the
    unmodified reference headers compiled here, Model::Run on MatrixCPU) at
    BASELINE config 3's full shape -- d 512, 8 layers, 8 heads, V 4096 and a
    512-token window, every row -- on the reference's own seed-3 weights, so
    that the GPU parity tests may use it for config 3 and 4 sequences the C
    oracle is too slow to check one by one."""
    import pytest
    if not O.ref_available():
        pytest.skip("the reference harness (oracle/_ref) is not built on this machine")
    s = O.LMShape(4096, 512, 512, 8, 8)
    window = O.prompt_tokens(4, s.V, s.C)
    ref = O.ref_forward(s, 3, window)  # [512 x 4096], every row of one Model::Run
    w = torch.from_numpy(O.init_weights(s, 3))
    with torch.no_grad():
        got = torch_ref.forward(w, s.V, s.C, s.d, s.H, s.L, window.astype(np.int64), 0, s.C).numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4)
    # and the greedy choice of every row wherever the reference's top-2 gap is clear
    top2 = np.sort(ref, axis=1)[:, -2:]
    clear = top2[:, 1] - top2[:, 0] > 2e-3
    assert clear.sum() > 400
    np.testing.assert_array_equal(got.argmax(axis=1)[clear], ref.argmax(axis=1)[clear])
