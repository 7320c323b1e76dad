"""NanoLM: the KV-cached, batched greedy token loop of FreeML's NanoLLM graph on
B200 (fml_lm_* in include/freeml_cuda.h).

Weights are taken in the reference's canonical order (token table, position
table, per layer {ln0 gamma, W_qkv, W_attn_proj, ln1 gamma, W_fc, W_mlp_proj},
ln_f gamma) and storage layouts (Dense_Weights as InitDenseBlob allocates them,
LayerLibrary/Dense.h:34-36).  Prompts and tokens are uint32 ids.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import FML_LM_NCLASS, PROFILE_CLASSES, LMConfig, call, load


@dataclass(frozen=True)
class NanoLLMShape:
    vocab: int
    context: int
    d_model: int
    n_head: int
    n_layer: int

    def param_count(self) -> int:
        d = self.d_model
        return self.vocab * d + self.context * d + self.n_layer * (2 * d + 12 * d * d) + d


# BASELINE.json configurations (the workload shapes)
CONFIGS = {
    1: dict(shape=NanoLLMShape(256, 128, 128, 4, 4), wseed=0, batch=1, prompt=16, pseed=1, new=112),
    3: dict(shape=NanoLLMShape(4096, 512, 512, 8, 8), wseed=3, batch=32, prompt=128, pseed=4, new=384),
    4: dict(shape=NanoLLMShape(32000, 2048, 1024, 16, 12), wseed=5, batch=64, prompt=1536, pseed=6, new=64),
    5: dict(shape=NanoLLMShape(32000, 4096, 4096, 32, 32), wseed=7, batch=8, prompt=1024, pseed=8, new=256),
}


def prompt_tokens(seed: int, vocab: int, batch: int, length: int) -> np.ndarray:
    """The workload's prompts: numpy's legacy RandomState(seed).randint(0, V),
    drawn sequence-major -- the same stream as std::mt19937(seed) with masked
    rejection."""
    return np.random.RandomState(seed).randint(0, vocab, size=(batch, length)).astype(np.uint32)


class NanoLM:
    def __init__(self, shape: NanoLLMShape, max_batch: int, device: int = 0):
        load()
        self.shape = shape
        self.max_batch = max_batch
        self.device = device
        self._cfg = LMConfig(shape.vocab, shape.context, shape.d_model, shape.n_head, shape.n_layer, max_batch)
        h = ctypes.c_void_p()
        torch.cuda.set_device(device)
        call("fml_lm_create", ctypes.byref(self._cfg), device, ctypes.byref(h))
        self._h = h
        self.batch = 0
        dev = torch.device("cuda", device)
        self._next = torch.zeros(max_batch, dtype=torch.int32, device=dev)
        self._logits = None

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            call("fml_lm_destroy", self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _stream():
        return torch.cuda.current_stream().cuda_stream

    def bind(self, params) -> None:
        """params: canonical packed parameters (numpy on host or torch on device)."""
        n = self.shape.param_count()
        if isinstance(params, np.ndarray):
            params = np.ascontiguousarray(params, np.float32)
            assert params.size == n, (params.size, n)
            call("fml_lm_bind_packed", self._h, params.ctypes.data, 1, self._stream())
        else:
            assert params.is_cuda and params.dtype == torch.float32 and params.numel() == n
            call("fml_lm_bind_packed", self._h, params.contiguous().data_ptr(), 0, self._stream())

    def load_checkpoint(self, path: str) -> None:
        """Bind the weights of a FreeML checkpoint directory (Model::Save of a
        NanoLLM model) -- fml_lm_load_checkpoint; the shapes must match."""
        call("fml_lm_load_checkpoint", self._h, str(path).encode(), self._stream())

    def prefill(self, prompts) -> None:
        """prompts: [B, P] uint32 (numpy or CUDA int32 tensor)."""
        if isinstance(prompts, np.ndarray):
            prompts = torch.from_numpy(np.ascontiguousarray(prompts, np.uint32).view(np.int32)).to(
                torch.device("cuda", self.device))
        B, P = prompts.shape
        call("fml_lm_prefill", self._h, prompts.contiguous().data_ptr(), B, P, self._stream())
        self.batch = B

    def step(self, want_logits: bool = False):
        """One greedy step on device; returns (next tokens [B] int32 tensor, logits or None)."""
        logits_ptr = None
        if want_logits:
            if self._logits is None:
                self._logits = torch.empty(self.max_batch, self.vocab_slice()[1], dtype=torch.float32,
                                           device=torch.device("cuda", self.device))
            logits_ptr = self._logits.data_ptr()
        call("fml_lm_step", self._h, self._next.data_ptr(), logits_ptr, self._stream())
        return self._next[: self.batch], (self._logits[: self.batch] if want_logits else None)

    def steps(self, n: int) -> None:
        """n greedy steps on device (multi-step graphs); the last tokens stay
        pending (pending_tokens())."""
        call("fml_lm_steps", self._h, n, self._stream())

    def vocab_slice(self):
        """(first row, rows) of the vocabulary this engine's logits cover:
        all of it, or the rank's share under tensor parallelism."""
        rank, world = getattr(self, "tp", (0, 1))
        vl = -(-self.shape.vocab // world)
        v0 = rank * vl
        return v0, min(vl, self.shape.vocab - v0)

    def step_host(self, tokens_in: np.ndarray, tokens_out: np.ndarray) -> None:
        """The host-buffer step: tokens_in -> device, step, next tokens -> tokens_out."""
        assert tokens_in.dtype == np.uint32 and tokens_out.dtype == np.uint32
        call("fml_lm_step_host", self._h, tokens_in.ctypes.data, tokens_out.ctypes.data, self._stream())

    def generate_host(self, tokens_in: np.ndarray, steps: int) -> np.ndarray:
        """`steps` host-buffer steps in one call: step 0 consumes tokens_in
        ([batch] uint32, host), each later step the tokens the previous one
        brought back to the host; returns the next tokens of every step
        ([steps, batch] uint32)."""
        assert tokens_in.dtype == np.uint32 and tokens_in.shape == (self.batch,)
        tokens_in = np.ascontiguousarray(tokens_in)
        out = np.empty((steps, self.batch), np.uint32)
        call("fml_lm_generate_host", self._h, steps, tokens_in.ctypes.data, out.ctypes.data, self._stream())
        return out

    def generate(self, prompts: np.ndarray, n_new: int, want_logits: bool = False, logit_rows=None):
        """Greedy decode: returns tokens [B, P + n_new] (uint32) and, if asked,
        the logits of every generated position [n_new - 1, B, V] (the prefill's
        last-row logits are not returned; step k's logits are row P + k).
        `logit_rows` keeps only those sequences' logits ([n_new - 1, len, V])."""
        B, P = prompts.shape
        self.prefill(prompts)
        toks = [torch.from_numpy(np.ascontiguousarray(prompts, np.uint32).view(np.int32)).cuda(self.device)]
        pending = self.pending_tokens()
        outs, logits = [pending.clone().view(B, 1)], []
        sel = None if logit_rows is None else torch.as_tensor(list(logit_rows), device=pending.device)
        for k in range(n_new - 1):
            nxt, lg = self.step(want_logits)
            outs.append(nxt.clone().view(B, 1))
            if want_logits:
                logits.append(lg.clone() if sel is None else lg.index_select(0, sel))
        torch.cuda.synchronize()
        seq = torch.cat(toks + outs, dim=1).cpu().numpy().view(np.uint32)
        return seq, (torch.stack(logits).cpu().numpy() if want_logits else None)

    def pending_tokens(self):
        """The token each sequence consumes next (after prefill: the argmax of
        its last prompt row), as a CUDA int32 tensor [B]."""
        buf = torch.empty(self.batch, dtype=torch.int32, device=torch.device("cuda", self.device))
        call("fml_lm_pending", self._h, buf.data_ptr(), self._stream())
        return buf

    def set_tensor_parallel(self, rank: int, world: int, nccl_id: bytes) -> None:
        """Join a tensor-parallel group of `world` engines (one per GPU and
        process); `nccl_id` comes from nccl_unique_id() on one rank.  Call
        before bind()."""
        buf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        call("fml_lm_set_tensor_parallel", self._h, int(rank), int(world), buf)
        self.tp = (int(rank), int(world))

    def tp_ipc_handles(self) -> bytes:
        """This rank's 128 bytes of CUDA IPC handles for the fused all-reduce."""
        buf = ctypes.create_string_buffer(128)
        call("fml_lm_tp_ipc_handles", self._h, buf)
        return buf.raw

    def tp_connect(self, handles_by_rank) -> None:
        """Open every rank's buffers (the handles of all ranks, rank order);
        the decode step then all-reduces inside its projection kernels."""
        blob = b"".join(bytes(h) for h in handles_by_rank)
        buf = ctypes.create_string_buffer(blob, len(blob))
        call("fml_lm_tp_connect", self._h, buf)

    def stamped_pass(self, run, steps: int):
        """Run `run()` (which must enqueue `steps` engine steps through the
        recorded graph) with in-graph completion stamps, and return
        (stamps [steps, kernels] in ns as int64, classes [kernels]): the time
        each kernel of the step finished, as the timed graph runs it.  Stamps
        are turned off again afterwards."""
        stride = ctypes.c_uint32()
        buf = torch.zeros(max(1, steps) * (3 + 7 * self.shape.n_layer), dtype=torch.int64,
                          device=torch.device("cuda", self.device))
        call("fml_lm_set_stamps", self._h, buf.data_ptr(), buf.numel(), ctypes.byref(stride))
        try:
            run()
            torch.cuda.synchronize(self.device)
            nk = ctypes.c_uint32()
            cls = (ctypes.c_int * stride.value)()
            call("fml_lm_stamp_classes", self._h, ctypes.cast(cls, ctypes.c_void_p), stride.value, ctypes.byref(nk))
        finally:
            call("fml_lm_set_stamps", self._h, None, 0, None)
        st = buf.view(-1, stride.value)[:steps, :nk.value].cpu().numpy()
        return st, [PROFILE_CLASSES[c] for c in list(cls)[:nk.value]]

    def set_prefill_math(self, mode: int) -> None:
        """FML_MATH_TF32X3 (default, tensor cores), FML_MATH_TF32 or FML_MATH_FP32."""
        call("fml_lm_set_prefill_math", self._h, int(mode))

    def set_weight_format(self, fmt: str) -> None:
        """'fp32' (default) or 'bf16': the storage of the weights the decode
        step streams (fml_lm_set_weight_format)."""
        call("fml_lm_set_weight_format", self._h, {"fp32": 0, "bf16": 1}[fmt])

    def set_graph(self, on: bool) -> None:
        call("fml_lm_set_graph", self._h, int(on))

    def position(self, b: int = 0) -> int:
        v = ctypes.c_uint32()
        call("fml_lm_get_position", self._h, b, ctypes.byref(v))
        return v.value

    def rewind(self, pos: int, pending) -> None:
        """Rewind every active sequence to `pos` with the given pending tokens
        (numpy uint32 on the host, or a CUDA int32 tensor: stream-ordered)."""
        if isinstance(pending, np.ndarray):
            pending = np.ascontiguousarray(pending, np.uint32)
            call("fml_lm_rewind", self._h, pos, pending.ctypes.data, 1, self._stream())
        else:
            call("fml_lm_rewind", self._h, pos, pending.contiguous().data_ptr(), 0, self._stream())

    def step_bytes(self) -> int:
        return int(load().fml_lm_step_bytes(self._h))

    def attention_bytes(self) -> int:
        return int(load().fml_lm_attention_bytes(self._h))

    def set_profiling(self, on: bool) -> None:
        call("fml_lm_set_profiling", self._h, int(on))

    def profile(self) -> dict:
        ms = (ctypes.c_double * FML_LM_NCLASS)()
        n = (ctypes.c_uint64 * FML_LM_NCLASS)()
        call("fml_lm_get_profile", self._h, ctypes.cast(ms, ctypes.c_void_p), ctypes.cast(n, ctypes.c_void_p),
             FML_LM_NCLASS)
        return {PROFILE_CLASSES[i]: (float(ms[i]), int(n[i])) for i in range(FML_LM_NCLASS)}


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL id for set_tensor_parallel (make it on one rank
    and share it with the others)."""
    buf = ctypes.create_string_buffer(128)
    call("fml_nccl_unique_id", buf)
    return buf.raw


def checkpoint_shape(path: str) -> NanoLLMShape:
    """(V, C, d, H, L) of a FreeML NanoLLM checkpoint directory, read from its
    stored shapes (fml_checkpoint_config; host only)."""
    cfg = LMConfig()
    call("fml_checkpoint_config", str(path).encode(), ctypes.byref(cfg))
    return NanoLLMShape(cfg.vocab, cfg.context, cfg.d_model, cfg.n_head, cfg.n_layer)


def checkpoint_params(path: str) -> np.ndarray:
    """Every parameter of a FreeML NanoLLM checkpoint in the canonical packed
    order (fml_checkpoint_pack; host only)."""
    shape = checkpoint_shape(path)
    out = np.empty(shape.param_count(), np.float32)
    call("fml_checkpoint_pack", str(path).encode(), out.ctypes.data, out.size)
    return out


def random_params(shape: NanoLLMShape, seed: int, device: int = 0) -> torch.Tensor:
    """Seeded random-init parameters of the NanoLLM architecture, generated on
    the GPU in the canonical order: N(0, 0.02) tables and Dense weights
    (Dense.h:75-80, Embedding.h:51-56), attention/MLP output projections
    scaled by 1/sqrt(2L) (TransformerBlock.h:247-256, :317-323), LayerNorm
    gammas 1.  Same distribution as the reference's init, not its exact draws
    (those come from std::mt19937 on the host)."""
    g = torch.Generator(device=torch.device("cuda", device))
    g.manual_seed(seed)
    d, L = shape.d_model, shape.n_layer
    out = torch.empty(shape.param_count(), dtype=torch.float32, device=torch.device("cuda", device))
    out.normal_(0.0, 0.02, generator=g)
    rs = 1.0 / float(np.sqrt(2.0 * L))
    off = shape.vocab * d + shape.context * d
    for _ in range(L):
        out[off:off + d] = 1.0
        off += d + 3 * d * d
        out[off:off + d * d] *= rs
        off += d * d
        out[off:off + d] = 1.0
        off += d + 4 * d * d
        out[off:off + 4 * d * d] *= rs
        off += 4 * d * d
    out[off:off + d] = 1.0
    return out
