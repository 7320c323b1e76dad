"""TEST INFRASTRUCTURE -- ctypes front-end of the C oracle (freeml_oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's ``cpu_baseline`` leg may
import this module, and only as the checker.  The product never imports it.

It also knows how to run the reference harness ``oracle/_ref/ref_nanollm``
(FreeML's own ``MatrixCPU`` path, built by ``oracle/Makefile``) when present.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import tempfile
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_BIN = os.path.join(HERE, "_ref", "ref_nanollm")


class OracleCfg(ctypes.Structure):
    _fields_ = [("V", ctypes.c_uint32), ("C", ctypes.c_uint32), ("d", ctypes.c_uint32),
                ("H", ctypes.c_uint32), ("L", ctypes.c_uint32)]


@dataclass(frozen=True)
class LMShape:
    """A NanoLLM shape: vocab V, context C, width d, heads H, layers L."""
    V: int
    C: int
    d: int
    H: int
    L: int

    def c(self) -> OracleCfg:
        return OracleCfg(self.V, self.C, self.d, self.H, self.L)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        fp = ctypes.POINTER(ctypes.c_float)
        up = ctypes.POINTER(ctypes.c_uint32)
        cp = ctypes.POINTER(OracleCfg)
        L.oracle_weight_count.argtypes = [cp]
        L.oracle_weight_count.restype = ctypes.c_uint64
        L.oracle_init_weights.argtypes = [cp, ctypes.c_uint32, fp]
        L.oracle_prompt_tokens.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, up]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_forward.argtypes = [cp, fp, up, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, fp]
        L.oracle_greedy.argtypes = [cp, fp, up, ctypes.c_uint32, ctypes.c_uint32, up, fp]
        L.oracle_argmax.argtypes = [fp, ctypes.c_uint32]
        L.oracle_argmax.restype = ctypes.c_uint32
        L.oracle_gather_rows.argtypes = [fp, fp, fp, ctypes.c_uint32, ctypes.c_uint32]
        L.oracle_add.argtypes = [fp, fp, fp, ctypes.c_uint64]
        L.oracle_layernorm.argtypes = [fp, fp, fp, fp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_float]
        L.oracle_gelu.argtypes = [fp, fp, ctypes.c_uint64]
        L.oracle_softmax.argtypes = [fp, fp, ctypes.c_uint32, ctypes.c_uint32]
        L.oracle_scale_add.argtypes = [fp, fp, ctypes.c_float, fp, ctypes.c_uint64]
        L.oracle_mul.argtypes = [fp, fp, fp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int]
        L.oracle_matmul_strided.argtypes = [fp, fp, fp] + [ctypes.c_uint32] * 6 + [ctypes.c_int]
        L.oracle_split_qkv.argtypes = [fp, fp, fp, fp, ctypes.c_uint32, ctypes.c_uint32]
        L.oracle_set_threads(int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)))
        _lib = L
    return _lib


def build() -> None:
    """Compile the C restatement (and the reference harness when the FreeML tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _up(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def prompt_tokens(seed: int, V: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().oracle_prompt_tokens(seed, V, n, _up(out))
    return out


def weight_count(s: LMShape) -> int:
    c = s.c()
    return int(lib().oracle_weight_count(ctypes.byref(c)))


def init_weights(s: LMShape, seed: int) -> np.ndarray:
    w = np.empty(weight_count(s), np.float32)
    c = s.c()
    rc = lib().oracle_init_weights(ctypes.byref(c), seed, _fp(w))
    assert rc == 0
    return w


def forward(s: LMShape, w: np.ndarray, tokens: np.ndarray, row0: int = 0, nrows: int | None = None) -> np.ndarray:
    """Logits rows [row0, row0+nrows) of one forward over ``tokens`` (T <= C)."""
    tokens = np.ascontiguousarray(tokens, np.uint32)
    T = tokens.size
    nrows = T - row0 if nrows is None else nrows
    out = np.empty((nrows, s.V), np.float32)
    c = s.c()
    rc = lib().oracle_forward(ctypes.byref(c), _fp(w), _up(tokens), T, row0, nrows, _fp(out))
    assert rc == 0, rc
    return out


def greedy(s: LMShape, w: np.ndarray, prompt: np.ndarray, nnew: int):
    prompt = np.ascontiguousarray(prompt, np.uint32)
    toks = np.empty(prompt.size + nnew, np.uint32)
    logits = np.empty((nnew, s.V), np.float32)
    c = s.c()
    rc = lib().oracle_greedy(ctypes.byref(c), _fp(w), _up(prompt), prompt.size, nnew, _up(toks), _fp(logits))
    assert rc == 0, rc
    return toks, logits


def argmax_first(row: np.ndarray) -> int:
    """First index of the maximum (the reference's strict '>' tie rule)."""
    row = np.ascontiguousarray(row, np.float32)
    return int(lib().oracle_argmax(_fp(row), row.size))


# ---- single operators (fp32 numpy in, numpy out) ----------------------------

def op_layernorm(x, gamma, beta=None, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    out = np.empty_like(x)
    b = None if beta is None else _fp(np.ascontiguousarray(beta, np.float32))
    lib().oracle_layernorm(_fp(out), _fp(x), _fp(np.ascontiguousarray(gamma, np.float32)), b, rows, cols, eps)
    return out


def op_gelu(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().oracle_gelu(_fp(out), _fp(x), x.size)
    return out


def op_softmax(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().oracle_softmax(_fp(out), _fp(x), x.shape[0], x.shape[1])
    return out


def op_mul(L, R, mode: int):
    """mode 0: L @ R (R is K x N); mode 1: L @ R.T (R is N x K)."""
    L = np.ascontiguousarray(L, np.float32)
    R = np.ascontiguousarray(R, np.float32)
    M, K = L.shape
    N = R.shape[0] if mode else R.shape[1]
    out = np.empty((M, N), np.float32)
    lib().oracle_mul(_fp(out), _fp(L), _fp(R), M, N, K, mode)
    return out


def op_scale_add(x, scale, add):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().oracle_scale_add(_fp(out), _fp(x), scale, _fp(np.ascontiguousarray(add, np.float32)), x.size)
    return out


def op_add(a, b):
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty_like(a)
    lib().oracle_add(_fp(out), _fp(a), _fp(np.ascontiguousarray(b, np.float32)), a.size)
    return out


def op_gather_rows(src, idx):
    src = np.ascontiguousarray(src, np.float32)
    idx = np.ascontiguousarray(idx, np.float32)
    out = np.empty((idx.size, src.shape[1]), np.float32)
    lib().oracle_gather_rows(_fp(out), _fp(src), _fp(idx), idx.size, src.shape[1])
    return out


def attention_decode_ref(q, k, v, scale):
    """Single-query attention restated from the reference ops (Q K^T via
    MatMul_Strided<Right>, ScaleAdd with a zero mask, Softmax, P V via
    MatMul_Strided<None>), per head.  q: [H, hd]; k, v: [H, n, hd]."""
    H, hd = q.shape
    out = np.empty((H, hd), np.float32)
    for h in range(H):
        s = op_mul(q[h:h + 1], k[h], 1)
        s = op_scale_add(s, scale, np.zeros_like(s))
        p = op_softmax(s)
        out[h] = op_mul(p, v[h], 0)[0]
    return out


def attention_prefill_ref(q, k, v, scale):
    """Whole-prompt causal attention restated from the reference ops
    (CausalSelfAttentionLayer.h:445-497: Q K^T via MatMul_Strided<Right>,
    ScaleAdd with the 0/-inf lower-triangular mask, Softmax, P V via
    MatMul_Strided<None>), per head.  q, k, v: [H, P, hd] -> [H, P, hd]."""
    H, P, hd = q.shape
    mask = np.where(np.tril(np.ones((P, P), bool)), 0.0, -np.inf).astype(np.float32)
    out = np.empty((H, P, hd), np.float32)
    for h in range(H):
        s = op_scale_add(op_mul(q[h], k[h], 1), scale, mask)
        out[h] = op_mul(op_softmax(s), v[h], 0)
    return out


# ---- the reference harness (FreeML's own MatrixCPU path) --------------------

def ref_available() -> bool:
    return os.path.exists(REF_BIN)


def _shape_args(s: LMShape, wseed: int):
    return ["--vocab", str(s.V), "--ctx", str(s.C), "--d", str(s.d), "--heads", str(s.H),
            "--layers", str(s.L), "--wseed", str(wseed)]


def ref_weights(s: LMShape, wseed: int) -> np.ndarray:
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "w.bin")
        subprocess.run([REF_BIN, "weights", *_shape_args(s, wseed), "--out", out], check=True)
        return np.fromfile(out, np.float32)


def ref_greedy(s: LMShape, wseed: int, prompt: np.ndarray, nnew: int):
    with tempfile.TemporaryDirectory() as td:
        pf, tf, lf = (os.path.join(td, n) for n in ("p.bin", "t.bin", "l.bin"))
        np.ascontiguousarray(prompt, np.uint32).tofile(pf)
        subprocess.run([REF_BIN, "greedy", *_shape_args(s, wseed), "--prompt", pf, "--plen", str(prompt.size),
                        "--new", str(nnew), "--out-tokens", tf, "--out-logits", lf], check=True)
        return np.fromfile(tf, np.uint32), np.fromfile(lf, np.float32).reshape(nnew, s.V)


def ref_save(s: LMShape, wseed: int, directory: str, name: str) -> str:
    """FreeML's own Model::Save of the built model (ModelLibrary/Model.h:91-159)
    into directory/name; returns that path."""
    subprocess.run([REF_BIN, "save", *_shape_args(s, wseed), "--dir", directory, "--name", name], check=True,
                   capture_output=True)
    return os.path.join(directory, name)


REF_VOCAB_BIN = os.path.join(HERE, "_ref", "ref_vocab")


def ref_vocab(corpus: bytes, text: bytes, ids: np.ndarray) -> dict:
    """NanoLLM's own BuildVocab / encode / decode / DecodeMatrixTokens
    (Examples/NanoLLM/NanoLLM.cpp:95-206) on the given inputs."""
    with tempfile.TemporaryDirectory() as td:
        paths = [os.path.join(td, n) for n in ("corpus.bin", "text.bin", "ids.bin")]
        for p, data in zip(paths, (corpus, text, np.ascontiguousarray(ids, np.uint32).tobytes())):
            with open(p, "wb") as f:
                f.write(data)
        subprocess.run([REF_VOCAB_BIN, *paths, td], check=True, capture_output=True)
        rd = lambda n: open(os.path.join(td, n), "rb").read()  # noqa: E731
        return {"unique": rd("unique.bin"), "corpus_ids": np.frombuffer(rd("corpus_ids.bin"), np.uint32).copy(),
                "encode": np.frombuffer(rd("encode.bin"), np.uint32).copy(), "decode": rd("decode.bin"),
                "decode_tokens": rd("decode_tokens.bin")}


def ref_train(s: LMShape, wseed: int, pseed: int, iters: int, lr: float = 1e-4):
    """NanoLLM training iterations on FreeML's CPU path (Model::Run(window,
    target): forward, cross-entropy, backward, AdamW) over the seeded token
    stream; returns (losses [iters] float64, parameters after the last step)."""
    with tempfile.TemporaryDirectory() as td:
        lf, wf = os.path.join(td, "l.bin"), os.path.join(td, "w.bin")
        subprocess.run([REF_BIN, "train", *_shape_args(s, wseed), "--iters", str(iters), "--pseed", str(pseed),
                        "--lr", repr(float(lr)), "--out-losses", lf, "--out", wf], check=True, capture_output=True)
        return np.fromfile(lf, np.float64), np.fromfile(wf, np.float32)


def ref_forward(s: LMShape, wseed: int, window: np.ndarray) -> np.ndarray:
    with tempfile.TemporaryDirectory() as td:
        wf, lf = os.path.join(td, "w.bin"), os.path.join(td, "l.bin")
        np.ascontiguousarray(window, np.uint32).tofile(wf)
        subprocess.run([REF_BIN, "forward", *_shape_args(s, wseed), "--window", wf, "--out-logits", lf], check=True)
        return np.fromfile(lf, np.float32).reshape(s.C, s.V)


def ref_time(s: LMShape, wseed: int, forwards: int, warmup: int, pseed: int = 1) -> dict:
    import json
    p = subprocess.run([REF_BIN, "time", *_shape_args(s, wseed), "--forwards", str(forwards),
                        "--warmup", str(warmup), "--pseed", str(pseed)],
                       check=True, capture_output=True, text=True)
    return json.loads(p.stdout.strip().splitlines()[-1])


def ref_op(op: str, dims: list, inputs: list, **kw) -> np.ndarray:
    """Run one generic FreeML operator; dims[0] is the output (x, y, z)."""
    with tempfile.TemporaryDirectory() as td:
        fi, fo = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
        np.concatenate([np.ascontiguousarray(a, np.float32).ravel() for a in inputs]).tofile(fi)
        cmd = [REF_BIN, "op", "--op", op, "--dims", ":".join(",".join(map(str, d)) for d in dims),
               "--in", fi, "--out", fo]
        for k, v in kw.items():
            cmd += ["--" + k, str(v)]
        subprocess.run(cmd, check=True)
        return np.fromfile(fo, np.float32)
