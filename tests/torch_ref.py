"""PyTorch fp32 restatement of the NanoLLM forward, for parity checks at
sizes the C oracle cannot run (config 5: 6.6e9 parameters).  Test
infrastructure only.

It follows the same reference code as oracle/freeml_oracle.c
(oracle_forward): Embedding gathers + AddLayer (Embedding.h:161-170,
AddLayer.h:149); per TransformerBlock (TransformerBlock.h:355-401)
LayerNormOp without beta (LayerNorm.h:148-165, biased variance, eps 1e-5),
QKV Dense with W [d x 3d], causal attention with scores * 1/sqrt(hd) and a
-inf upper triangle (CausalSelfAttentionLayer.h:424-499), proj Dense applied
as Y W^T (W stored out x in), residual Add, LayerNorm, fc Dense W [d x 4d],
exact-erf GELU (Gelu.h), mlp Dense W [4d x d], residual Add; final LayerNorm
and the lm_head tied to the token table (NanoLLM.cpp:315-348).  Parameters
use the packed order of oracle_init_weights / fml_lm_bind_packed.  Pinned by
tests/test_torch_ref_cpu.py against the reference's golden logits."""
import math

import torch


def _layernorm(x, g):
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + 1e-5) * g


def forward(params: torch.Tensor, V: int, C: int, d: int, H: int, L: int, tokens, row0: int, nrows: int,
            bf16_from_row=None):
    """Logits rows [row0, row0 + nrows) of a forward over `tokens` (T <= C).

    bf16_from_row = r: rows >= r multiply by the Dense weights and the tied
    lm_head rounded to bf16 (nearest even) -- what the decode engine's
    bf16-weight mode computes for the rows it generates after an fp32
    prefill of rows < r (a row's K/V come from its own QKV, so the rule is
    exact per row)."""
    p = params.to(torch.float32)
    dev = p.device
    tokens = torch.as_tensor(tokens, dtype=torch.long, device=dev)
    T = tokens.numel()
    hd = d // H
    off = 0

    def take(n, *shape):
        nonlocal off
        t = p[off:off + n].view(*shape)
        off += n
        return t

    tok = take(V * d, V, d)
    pos = take(C * d, C, d)
    x = tok[tokens] + pos[:T]
    r0 = T if bf16_from_row is None else bf16_from_row

    def lin(inp, w):
        out = inp @ w
        if r0 < inp.shape[0]:
            out[r0:] = inp[r0:] @ w.to(torch.bfloat16).to(torch.float32)
        return out

    causal = torch.triu(torch.ones(T, T, dtype=torch.bool, device=dev), diagonal=1)
    for _ in range(L):
        g0 = take(d, d)
        wqkv = take(3 * d * d, d, 3 * d)
        wprj = take(d * d, d, d)
        g1 = take(d, d)
        wfc = take(4 * d * d, d, 4 * d)
        wmlp = take(4 * d * d, 4 * d, d)
        qkv = lin(_layernorm(x, g0), wqkv)
        q, k, v = (t.view(T, H, hd).transpose(0, 1) for t in qkv.split(d, dim=1))
        s = (q @ k.transpose(-1, -2)) * (1.0 / math.sqrt(hd))
        s = s.masked_fill(causal, float("-inf"))
        y = (torch.softmax(s, dim=-1) @ v).transpose(0, 1).reshape(T, d)
        buf = x + lin(y, wprj.t())
        h = torch.nn.functional.gelu(lin(_layernorm(buf, g1), wfc))
        x = buf + lin(h, wmlp)
    gf = take(d, d)
    xf = _layernorm(x[row0:row0 + nrows], gf)
    if r0 >= row0 + nrows:
        return xf @ tok.t()
    out = xf @ tok.t()
    lo = max(r0 - row0, 0)
    out[lo:] = xf[lo:] @ tok.t().to(torch.bfloat16).to(torch.float32)
    return out
