"""FreeML checkpoints (the directory Model::Save writes, ModelLibrary/Model.h:
91-159) read by the library's host-side reader: shapes, the packed
parameters against the reference's own weights, and rejection of what the
engine cannot run.  CPU only; the fixture ckpt_tiny.tgz was written by the
unmodified reference (tests/golden/make_golden.py)."""
import hashlib
import os
import re
import shutil
import tarfile

import numpy as np
import pytest

from freeml_b200 import FmlError
from freeml_b200 import lm as LM
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture()
def ckpt(tmp_path, golden):
    meta = golden[0]["checkpoint"]["ckpt_tiny"]
    with tarfile.open(os.path.join(HERE, "golden", "ckpt_tiny.tgz")) as tar:
        tar.extractall(tmp_path, filter="data")
    return str(tmp_path / meta["dir"]), meta


def _layer_file(path, layer_name):
    """The .blob_layer file whose root record names `layer_name`."""
    for f in os.listdir(path):
        if f.endswith(".blob_layer"):
            txt = open(os.path.join(path, f)).read()
            if re.search(rf"^NAME Layer_Name\nDATA {re.escape(layer_name)}\n", txt, re.M):
                return os.path.join(path, f)
    raise AssertionError(layer_name)


def _matrix_file(layer_path, key):
    txt = open(layer_path).read()
    m = re.search(rf"^NAME {re.escape(key)}\nDATA (\S+)\nTYPE MATRIX", txt, re.M)
    return os.path.join(os.path.dirname(layer_path), m.group(1))


def test_checkpoint_shape(ckpt):
    path, meta = ckpt
    s = LM.checkpoint_shape(path)
    assert (s.vocab, s.context, s.d_model, s.n_head, s.n_layer) == (meta["V"], meta["C"], meta["d"], meta["H"],
                                                                    meta["L"])


def test_checkpoint_params_are_the_reference_weights(ckpt):
    """Bit-identical to the reference model's parameters (their sha256) and to
    the oracle's restatement of the reference initialisation."""
    path, meta = ckpt
    w = LM.checkpoint_params(path)
    assert w.size == meta["weights_count"]
    assert hashlib.sha256(w.tobytes()).hexdigest() == meta["weights_sha256"]
    ref = O.init_weights(O.LMShape(meta["V"], meta["C"], meta["d"], meta["H"], meta["L"]), meta["wseed"])
    np.testing.assert_array_equal(w.view(np.uint32), ref.view(np.uint32))


def test_missing_directory_is_rejected(tmp_path):
    with pytest.raises(FmlError, match="model.guide"):
        LM.checkpoint_shape(str(tmp_path / "nothing"))


def test_wrong_buffer_size_is_rejected(ckpt):
    from freeml_b200._lib import call
    path, meta = ckpt
    buf = np.empty(meta["weights_count"] - 1, np.float32)
    with pytest.raises(FmlError, match="parameter"):
        call("fml_checkpoint_pack", path.encode(), buf.ctypes.data, buf.size)


def test_untied_lm_head_is_rejected(ckpt):
    path, _ = ckpt
    hdr = _matrix_file(_layer_file(path, "lm_head"), "Dense_Weights")
    txt = open(hdr).read()
    open(hdr, "w").write(re.sub(r"^GUID \S+", "GUID 12345", txt, flags=re.M))
    with pytest.raises(FmlError, match="not tied"):
        LM.checkpoint_params(path)


def test_bias_is_rejected(ckpt):
    """The engine models use_bias = false (NanoLLM.cpp:57): a Dense bias
    matrix in the checkpoint is refused, not dropped."""
    path, _ = ckpt
    head = _layer_file(path, "lm_head")
    w = _matrix_file(head, "Dense_Weights")
    with open(head, "a") as f:
        f.write(f"NAME Dense_Bias\nDATA {os.path.basename(w)}\nTYPE MATRIX\n;\n")
    with pytest.raises(FmlError, match="bias"):
        LM.checkpoint_params(path)


def test_truncated_payload_is_rejected(ckpt):
    path, _ = ckpt
    hdr = _matrix_file(_layer_file(path, "embedding_pos"), "Embedding_Weights")
    data = re.search(r"^DATA (\S+)", open(hdr).read(), re.M).group(1)
    p = os.path.join(path, data)
    raw = open(p, "rb").read()
    open(p, "wb").write(raw[:-4])
    with pytest.raises(FmlError, match="bytes"):
        LM.checkpoint_params(path)


def test_shape_mismatch_is_rejected(ckpt, tmp_path):
    """A layer whose stored dims disagree with the others (here: the fc
    weight of block 1 relabelled) is refused."""
    path, _ = ckpt
    blk = _layer_file(path, "block_1")
    fc = re.search(r"^NAME DenseFCData\nDATA (\S+)", open(blk).read(), re.M).group(1)
    hdr = _matrix_file(os.path.join(path, fc), "Dense_Weights")
    txt = open(hdr).read()
    open(hdr, "w").write(re.sub(r"^DIMX (\d+)", lambda m: f"DIMX {int(m.group(1)) // 2}", txt, flags=re.M))
    with pytest.raises(FmlError, match="expected"):
        LM.checkpoint_params(path)
    shutil.rmtree(path)
