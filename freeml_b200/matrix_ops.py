"""FreeML's generic operator names over torch CUDA tensors, dispatched to the
sm_100a kernels of libfreeml_cuda.so.

Each function keeps the reference's name and argument order
(MatrixLibrary/MatrixBase_Functions.h, MatrixLibrary/MatrixBase_Mul.h), with
torch tensors standing in for MatrixCUDA<float> storage: fp32, contiguous,
row-major [rows x cols] (FreeML's Dims3D{x = cols, y = rows}).  Shape errors
raise FmlError (FML_ERR_INVALID) where the reference would assert.
"""
from __future__ import annotations

import torch

from ._lib import FmlError, call

NONE, RIGHT = 0, 1  # TransposeMode::None / TransposeMode::Right (MatrixBase_Mul.h:27)


def _p(t: torch.Tensor | None):
    if t is None:
        return None
    if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise FmlError(1, "matrix_ops", "expected a contiguous float32 CUDA tensor")
    return t.data_ptr()


def _s():
    return torch.cuda.current_stream().cuda_stream


def _check(cond: bool, msg: str):
    if not cond:
        raise FmlError(1, "matrix_ops", msg)


def GatherRows(out, src, indices):
    """MatrixBase_Functions.h:203-242; indices hold float row ids."""
    _check(out.shape[-1] == src.shape[-1] and indices.numel() == out.numel() // out.shape[-1], "GatherRows shapes")
    call("fml_gather_rows", _p(out), _p(src), _p(indices), indices.numel(), src.shape[-1], src.numel() // src.shape[-1], _s())


def Add(out, L, R):
    _check(out.numel() == L.numel() == R.numel(), "Add shapes")
    call("fml_add", _p(out), _p(L), _p(R), R.numel(), _s())


def BroadcastAdd(out, L, R):
    call("fml_broadcast_add", _p(out), _p(L), _p(R), L.numel(), L.shape[-1], _s())


def PerElementMul(out, L, R):
    call("fml_mul_elementwise", _p(out), _p(L), _p(R), R.numel(), _s())


def Scale(out, inp, val):
    if isinstance(val, torch.Tensor):
        call("fml_scale", _p(out), _p(inp), 0.0, _p(val), inp.numel(), _s())
    else:
        call("fml_scale", _p(out), _p(inp), float(val), None, inp.numel(), _s())


def ScaleAdd(out, inp, scale, add):
    """out = in * scale[0] + add (MatrixBase_Functions.h:1056-1070)."""
    _check(out.numel() == inp.numel() == add.numel(), "ScaleAdd shapes")
    call("fml_scale_add", _p(out), _p(inp), _p(scale), _p(add), inp.numel(), _s())


def Fill(out, val):
    if isinstance(val, torch.Tensor):
        call("fml_fill", _p(out), 0.0, _p(val), out.numel(), _s())
    else:
        call("fml_fill", _p(out), float(val), None, out.numel(), _s())


def Clear(out):
    Fill(out, 0.0)


def Copy(out, inp):
    _check(out.numel() == inp.numel(), "Copy shapes")
    call("fml_copy", _p(out), _p(inp), inp.numel(), _s())


def LayerNormOp(out, inp, gamma, beta=None, xHat=None, eps=1e-5):
    cols = inp.shape[-1]
    call("fml_layernorm", _p(out), _p(inp), _p(gamma), _p(beta), _p(xHat), inp.numel() // cols, cols, eps, _s())


def GeluMat(out, inp):
    call("fml_gelu", _p(out), _p(inp), inp.numel(), _s())


def Softmax(out, inp):
    cols = inp.shape[-1]
    call("fml_softmax", _p(out), _p(inp), inp.numel() // cols, cols, _s())


def SplitQKV(q, k, v, packed):
    d = q.shape[-1]
    call("fml_split_qkv", _p(q), _p(k), _p(v), _p(packed), q.numel() // d, d, _s())


def Mul(out, L, R, mode: int = NONE):
    """Mul<None|Right> (MatrixBase_Mul.h:591-615)."""
    M, K = L.shape
    N = R.shape[0] if mode == RIGHT else R.shape[1]
    _check((R.shape[1] if mode == RIGHT else R.shape[0]) == K and tuple(out.shape) == (M, N), "Mul shapes")
    call("fml_matmul", _p(out), _p(L), _p(R), M, N, K, int(mode == RIGHT), _s())


def MatMul_Strided(out, L, R, M, N, K, lda, ldb, ldc, mode: int = NONE, batch=1, plane_a=0, plane_b=0, plane_c=0,
                   off_a=0, off_b=0, off_c=0):
    """MatMul_Strided<None|Right> (MatrixBase_Mul.h:617-722) on element views
    starting at the given offsets (the reference's SetData(ptr, offset))."""
    es = 4
    call("fml_matmul_strided", out.data_ptr() + off_c * es, L.data_ptr() + off_a * es, R.data_ptr() + off_b * es,
         M, N, K, lda, ldb, ldc, int(mode == RIGHT), batch, plane_a, plane_b, plane_c, _s())


def attention_decode_workspace_bytes(batch: int, heads: int, head_dim: int, context: int) -> int:
    from ._lib import load
    return int(load().fml_attention_workspace_bytes(batch, heads, head_dim, context))


def attention_prefill(out, q, kcache, vcache, prompt_len, scale, mode=None):
    """Causal attention over whole prompts (fml_attention_prefill).
    q/out: [B*P, H*hd] (row b*P + t); kcache/vcache: [B, H, C, hd] with rows
    0..P-1 filled.  mode: FML_MATH_* (default: the library's math mode)."""
    from ._lib import load
    B, H, C, hd = kcache.shape
    P = int(prompt_len)
    _check(q.shape == (B * P, H * hd) and out.shape == q.shape and vcache.shape == kcache.shape,
           "attention_prefill shapes")
    if mode is None:
        mode = int(load().fml_get_math_mode())
    call("fml_attention_prefill", _p(out), _p(q), _p(kcache), _p(vcache), B, H, hd, C, P, float(scale), int(mode),
         _s())


def attention_decode(out, q, kcache, vcache, lens, scale, workspace=None):
    """Causal attention of the newest row per sequence over a KV cache
    (fml_attention_decode).  q/out: [B, H*hd]; kcache/vcache: [B, H, C, hd];
    lens: int32 [B] (keys 0..lens[b]-1)."""
    B, H, C, hd = kcache.shape
    need = attention_decode_workspace_bytes(B, H, hd, C)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=q.device)
    _check(lens.dtype == torch.int32 and lens.is_cuda, "lens must be a CUDA int32 tensor")
    call("fml_attention_decode", _p(out), _p(q), _p(kcache), _p(vcache), lens.data_ptr(), B, H, hd, C, float(scale),
         workspace.data_ptr(), workspace.numel(), _s())
