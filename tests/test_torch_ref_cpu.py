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
