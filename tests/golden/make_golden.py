"""Regenerate the golden fixtures in this directory from FreeML's own CPU path.

Run (in a container that has the FreeML tree and the built harness):

    make -C oracle all
    python tests/golden/make_golden.py              # every fixture
    python tests/golden/make_golden.py checkpoint   # only ckpt_tiny.tgz
    python tests/golden/make_golden.py vocab        # only vocab.npz
    python tests/golden/make_golden.py train        # only train_tiny.npz

Every number below comes from ``oracle/_ref/ref_nanollm`` -- the unmodified
reference ``Model<float, MatrixCPU<float>>`` and its generic operators -- never
from the oracle restatement or the CUDA code.  The fixtures are small (a few
hundred KB) so that the CPU test suite can pin the oracle without the
reference tree.
"""
import hashlib
import json
import os
import sys
import tarfile
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

# (name, shape, weight seed, prompt seed, prompt length, decode steps)
GREEDY_CASES = [
    ("cfg1", O.LMShape(V=256, C=128, d=128, H=4, L=4), 0, 1, 16, 112),
    ("odd", O.LMShape(V=97, C=48, d=64, H=2, L=2), 11, 12, 8, 40),       # non-power-of-two vocab
]
# a checkpoint written by FreeML's Model::Save, committed as a tarball
# (name, shape, weight seed, prompt seed, prompt length, decode steps)
CHECKPOINT_CASE = ("ckpt_tiny", O.LMShape(V=61, C=16, d=32, H=1, L=2), 11, 5, 4, 12)  # head dim 32
# weight-init hashes only (the tensors are too big to commit)
HASH_CASES = [
    ("cfg3", O.LMShape(V=4096, C=512, d=512, H=8, L=8), 3),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_checkpoint() -> dict:
    """The tiny model saved by FreeML's Model::Save, as ckpt_tiny.tgz, plus its
    reference greedy tokens."""
    name, s, wseed, pseed, plen, nnew = CHECKPOINT_CASE
    with tempfile.TemporaryDirectory() as td:
        path = O.ref_save(s, wseed, td, "nanollm_tiny")
        with tarfile.open(os.path.join(HERE, f"{name}.tgz"), "w:gz") as tar:
            tar.add(path, arcname="nanollm_tiny")
    prompt = np.random.RandomState(pseed).randint(0, s.V, plen).astype(np.uint32)
    toks, _ = O.ref_greedy(s, wseed, prompt, nnew)
    print(name, "checkpoint tokens", toks)
    w = O.ref_weights(s, wseed)
    return {name: {"V": s.V, "C": s.C, "d": s.d, "H": s.H, "L": s.L, "wseed": wseed,
                                 "pseed": pseed, "plen": plen, "new": nnew, "dir": "nanollm_tiny",
                                 "weights_sha256": sha(w), "weights_count": int(w.size),
                                 "tokens": [int(t) for t in toks]}}


# NanoLLM training iterations on the reference CPU path (losses and the
# parameters after the last AdamW step), committed as train_tiny.npz
TRAIN_CASE = ("train_tiny", O.LMShape(V=61, C=16, d=32, H=1, L=2), 11, 5, 3)


def make_train() -> None:
    name, s, wseed, pseed, iters = TRAIN_CASE
    losses, w = O.ref_train(s, wseed, pseed, iters)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), losses=losses, weights=w,
                        shape=np.array([s.V, s.C, s.d, s.H, s.L, wseed, pseed, iters], np.int64))
    print(name, "losses", losses)


def make_vocab() -> None:
    """NanoLLM's vocabulary code on a synthetic byte corpus (bytes on both
    sides of 0x80, some absent), a text with absent bytes and ids past the
    vocabulary, as vocab.npz."""
    rs = np.random.RandomState(21)
    alphabet = np.concatenate([np.arange(9, 14), np.arange(32, 127), np.arange(0xC0, 0xE0)]).astype(np.uint8)
    present = rs.choice(alphabet, 90, replace=False)
    corpus = rs.choice(present, 4000).astype(np.uint8).tobytes()
    text = rs.choice(alphabet, 300).astype(np.uint8).tobytes()
    ids = rs.randint(0, 100, 200).astype(np.uint32)
    r = O.ref_vocab(corpus, text, ids)
    np.savez_compressed(os.path.join(HERE, "vocab.npz"), corpus=np.frombuffer(corpus, np.uint8),
                        text=np.frombuffer(text, np.uint8), ids=ids,
                        unique=np.frombuffer(r["unique"], np.uint8), corpus_ids=r["corpus_ids"],
                        encode=r["encode"], decode=np.frombuffer(r["decode"], np.uint8),
                        decode_tokens=np.frombuffer(r["decode_tokens"], np.uint8))
    print("vocab", len(r["unique"]), "symbols")


def main():
    assert O.ref_available(), "build oracle/_ref/ref_nanollm first (make -C oracle all)"
    meta = {"greedy": {}, "weights_sha256": {}}
    arrays = {}
    for name, s, wseed, pseed, plen, nnew in GREEDY_CASES:
        prompt = np.random.RandomState(pseed).randint(0, s.V, plen).astype(np.uint32)
        toks, logits = O.ref_greedy(s, wseed, prompt, nnew)
        w = O.ref_weights(s, wseed)
        window = np.zeros(s.C, np.uint32)
        window[:toks.size] = toks
        full = O.ref_forward(s, wseed, window)
        arrays[f"{name}_prompt"] = prompt
        arrays[f"{name}_tokens"] = toks
        arrays[f"{name}_logits"] = logits
        arrays[f"{name}_window_logits"] = full
        meta["greedy"][name] = {"V": s.V, "C": s.C, "d": s.d, "H": s.H, "L": s.L, "wseed": wseed,
                                "pseed": pseed, "plen": plen, "new": nnew,
                                "weights_sha256": sha(w), "weights_count": int(w.size)}
        print(name, "tokens", toks[:8], "...")
    meta["checkpoint"] = make_checkpoint()
    make_vocab()
    make_train()
    for name, s, wseed in HASH_CASES:
        w = O.ref_weights(s, wseed)
        meta["weights_sha256"][name] = {"V": s.V, "C": s.C, "d": s.d, "H": s.H, "L": s.L, "wseed": wseed,
                                        "sha256": sha(w), "count": int(w.size),
                                        "first8": [float(x) for x in w[:8]]}
        print(name, "weights", w.size)

    # single operators on seeded inputs
    rs = np.random.RandomState(2)
    M, K, N = 40, 96, 72
    A = rs.randn(M, K).astype(np.float32)
    B = (0.02 * rs.randn(K, N)).astype(np.float32)
    Bt = (0.02 * rs.randn(N, K)).astype(np.float32)
    g = (1 + 0.1 * rs.randn(K)).astype(np.float32)
    beta = (0.1 * rs.randn(K)).astype(np.float32)
    ops = {"A": A, "B": B, "Bt": Bt, "gamma": g, "beta": beta}
    ops["mul_none"] = O.ref_op("mul_none", [(N, M, 1), (K, M, 1), (N, K, 1)], [A, B]).reshape(M, N)
    ops["mul_right"] = O.ref_op("mul_right", [(N, M, 1), (K, M, 1), (K, N, 1)], [A, Bt]).reshape(M, N)
    small = A[:8, :16].copy()
    ops["small"] = small
    ops["small_B"] = B[:16, :8].copy()
    ops["mul_none_small"] = O.ref_op("mul_none", [(8, 8, 1), (16, 8, 1), (8, 16, 1)], [small, ops["small_B"]]).reshape(8, 8)
    ops["layernorm"] = O.ref_op("layernorm", [(K, M, 1), (K, M, 1), (K, 1, 1)], [A, g]).reshape(M, K)
    ops["layernorm_beta"] = O.ref_op("layernorm_beta", [(K, M, 1), (K, M, 1), (K, 1, 1), (K, 1, 1)], [A, g, beta]).reshape(M, K)
    ops["softmax"] = O.ref_op("softmax", [(K, M, 1), (K, M, 1)], [A]).reshape(M, K)
    ops["gelu"] = O.ref_op("gelu", [(K, M, 1), (K, M, 1)], [A]).reshape(M, K)
    ops["add"] = O.ref_op("add", [(K, M, 1), (K, M, 1), (K, M, 1)], [A, A[::-1].copy()]).reshape(M, K)
    mask = np.where(np.tril(np.ones((M, M))) > 0, 0.0, -np.inf).astype(np.float32)
    S = rs.randn(M, M).astype(np.float32)
    ops["S"] = S
    ops["mask"] = mask
    ops["scale"] = np.array([1.0 / np.sqrt(np.float32(32))], np.float32)
    ops["scale_add"] = O.ref_op("scale_add", [(M, M, 1), (M, M, 1), (1, 1, 1), (M, M, 1)], [S, ops["scale"], mask]).reshape(M, M)
    table = rs.randn(50, K).astype(np.float32)
    idx = rs.randint(0, 50, M).astype(np.float32)
    ops["table"], ops["idx"] = table, idx
    ops["gather_rows"] = O.ref_op("gather_rows", [(K, M, 1), (K, 50, 1), (1, M, 1)], [table, idx]).reshape(M, K)
    # attention core pieces as CausalSelfAttentionLayer uses them: head h of
    # width hd at column offset h*hd, row stride d
    T, d, hd, h = 24, 64, 16, 1
    Q = rs.randn(T, d).astype(np.float32)
    Kk = rs.randn(T, d).astype(np.float32)
    P = rs.rand(T, T).astype(np.float32)
    ops["attn_Q"], ops["attn_K"], ops["attn_P"] = Q, Kk, P
    ops["strided_right_h1"] = O.ref_op("matmul_strided_right", [(T, T, 1), (d, T, 1), (d, T, 1)], [Q, Kk],
                                       hd=hd, off=h * hd).reshape(T, T)
    ops["strided_none_h1"] = O.ref_op("matmul_strided_none", [(d, T, 1), (T, T, 1), (d, T, 1)], [P, Kk],
                                      hd=hd, off=h * hd).reshape(T, d)
    packed = rs.randn(M, 3 * 32).astype(np.float32)
    ops["packed"] = packed
    zeros = np.zeros((M, 32), np.float32)
    qkv = O.ref_op("split_qkv", [(32, M, 1), (32, M, 1), (32, M, 1), (96, M, 1)], [zeros, zeros, packed])
    ops["split_q"], ops["split_k"], ops["split_v"] = (qkv[i * M * 32:(i + 1) * M * 32].reshape(M, 32) for i in range(3))

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    if sys.argv[1:] == ["train"]:  # refresh only train_tiny.npz
        assert O.ref_available(), "build oracle/_ref first (make -C oracle all)"
        make_train()
    elif sys.argv[1:] == ["vocab"]:  # refresh only vocab.npz
        assert os.path.exists(O.REF_VOCAB_BIN), "build oracle/_ref first (make -C oracle all)"
        make_vocab()
    elif sys.argv[1:] == ["checkpoint"]:  # refresh only the checkpoint fixture
        assert O.ref_available(), "build oracle/_ref/ref_nanollm first (make -C oracle all)"
        path = os.path.join(HERE, "golden.json")
        with open(path) as f:
            meta = json.load(f)
        meta["checkpoint"] = make_checkpoint()
        with open(path, "w") as f:
            json.dump(meta, f, indent=1, sort_keys=True)
    else:
        main()
