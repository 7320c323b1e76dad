"""The allocation-free attention entry point, fml_attention_decode_noalloc.

It exists for callers that may not allocate device memory -- for example a
host runtime that owns the GPU's memory through its own pool and forbids
libraries to call cudaMalloc.  Instead of a caller workspace it uses a fixed
array inside the library.  These checks call it through the C ABI and compare
it with fml_attention_decode (caller workspace) on consecutive calls, so a
second call that finds the previous call's partials and counters in the
shared array must still give the right answer.  This file is collected last
so that a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-5  # the attention parity bound used by tests/test_ops_gpu.py


def _case(B, H, hd, C, lens, seed):
    rs = np.random.RandomState(seed)
    dev = torch.device("cuda", 0)
    q = torch.from_numpy(rs.randn(B, H * hd).astype(np.float32)).to(dev)
    kc = torch.from_numpy(rs.randn(B, H, C, hd).astype(np.float32)).to(dev)
    vc = torch.from_numpy(rs.randn(B, H, C, hd).astype(np.float32)).to(dev)
    ln = torch.from_numpy(np.asarray(lens, np.int32)).to(dev)
    return q, kc, vc, ln


def _with_workspace(q, kc, vc, ln, scale):
    from freeml_b200 import _lib
    B, H, C, hd = kc.shape
    need = int(_lib.load().fml_attention_workspace_bytes(B, H, hd, C))
    ws = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty(B, H * hd, device=q.device)
    _lib.call("fml_attention_decode", out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ln.data_ptr(),
              B, H, hd, C, ctypes.c_float(scale), ws.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
    return out


def _no_alloc(q, kc, vc, ln, scale):
    from freeml_b200 import _lib
    B, H, C, hd = kc.shape
    out = torch.full((B, H * hd), float("nan"), device=q.device)
    _lib.call("fml_attention_decode_noalloc", out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              ln.data_ptr(), B, H, hd, C, ctypes.c_float(scale), torch.cuda.current_stream().cuda_stream)
    return out


# How the key-range splits are merged.  By default up to 8 splits form one
# thread-block cluster and merge on chip, which touches only the counters in
# the fixed array; with clusters off, or with 16 splits, every split writes
# its partials into the array and the last one to finish merges them, so a
# second call runs over the first call's partials and counters.
MERGES = {
    "cluster": {},
    "global": {"FML_ATTN_CLUSTER": "0"},
    "global-16-splits": {"FML_ATTN_SPLITS": "16"},
}


@pytest.mark.parametrize("merge", sorted(MERGES))
@pytest.mark.parametrize("B,H,hd,C,lens", [
    (1, 8, 64, 2048, [2048]),           # a single sequence: many splits of the key range
    (4, 8, 64, 512, [0, 1, 300, 512]),  # ragged lengths, including an empty one
])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(B, H, hd, C, lens, merge, monkeypatch):
    for k, v in MERGES[merge].items():
        monkeypatch.setenv(k, v)  # read by the library at every call
    torch.cuda.set_device(0)
    scale = float(1.0 / np.sqrt(hd))
    first = _case(B, H, hd, C, lens, seed=C + B)
    second = _case(B, H, hd, C, lens[::-1], seed=C + B + 1)
    for q, kc, vc, ln in (first, second):
        ref = _with_workspace(q, kc, vc, ln, scale)
        got = _no_alloc(q, kc, vc, ln, scale)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=TOL, atol=TOL)


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch():
    from freeml_b200 import FmlError, _lib
    torch.cuda.set_device(0)
    t = torch.zeros(16, device="cuda")
    p = t.data_ptr()
    # 2048 sequences x 32 heads x head_dim 128 needs ~34 MB of split partials
    with pytest.raises(FmlError) as e:
        _lib.call("fml_attention_decode_noalloc", p, p, p, p, p, 2048, 32, 128, 4096, ctypes.c_float(0.1),
                  torch.cuda.current_stream().cuda_stream)
    assert e.value.status == 4
    assert "fixed" in str(e.value)
