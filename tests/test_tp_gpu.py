"""Tensor parallelism on two GPUs (BASELINE config 5's scheme), run as two
processes, one engine and one GPU each, sharing an NCCL id.  Both ranks must
produce the same token streams, and their vocabulary slices of the logits,
put together, must match the reference teacher-forced (config-3 weights from
the reference's initialisation, checked by the C oracle).  NVLS is off, as
for every multi-process GPU test here."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-3
SHAPE = (4096, 512, 512, 8, 8)  # config 3: V C d H L
NSEQ, N = 4, 24


def _rank(rank, world, q_id, q_out, fused, q_h):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        from freeml_b200.lm import CONFIGS, NanoLLMShape, NanoLM, nccl_unique_id, prompt_tokens
        if rank == 0:
            nid = nccl_unique_id()
            for _ in range(world - 1):
                q_id.put(nid)
        else:
            nid = q_id.get(timeout=120)
        c = CONFIGS[3]
        s = O.LMShape(*SHAPE)
        w = O.init_weights(s, c["wseed"])
        prompts = prompt_tokens(c["pseed"], s.V, c["batch"], c["prompt"])[:NSEQ]
        lm = NanoLM(NanoLLMShape(*SHAPE), NSEQ, device=rank)
        lm.set_tensor_parallel(rank, world, nid)
        if fused:
            # every rank's IPC handles, in rank order, to every rank
            mine = lm.tp_ipc_handles()
            for _ in range(world - 1):
                q_h[1 - rank].put((rank, mine))
            got = {rank: mine}
            while len(got) < world:
                r, hnd = q_h[rank].get(timeout=120)
                got[r] = hnd
            lm.tp_connect([got[r] for r in range(world)])
        lm.bind(w)
        toks, logits = lm.generate(prompts, N, want_logits=True)
        # the same steps again as multi-step graphs (fml_lm_steps, with the
        # all-reduces captured inside): the last pending token must match
        lm.rewind(c["prompt"], np.ascontiguousarray(toks[:, c["prompt"]], np.uint32))
        lm.steps(N - 1)
        again = lm.pending_tokens().cpu().numpy().view(np.uint32)[:NSEQ]
        assert np.array_equal(again, toks[:, c["prompt"] + N - 1]), "multi-step graphs gave another stream"
        v0, vl = lm.vocab_slice()
        import ctypes
        from freeml_b200 import _lib
        errs = ctypes.c_uint64(0)
        _lib.call("fml_device_error_count", ctypes.byref(errs))
        lm.close()
        q_out.put((rank, toks, logits, v0, vl) if errs.value == 0 else (rank, None, f"{errs.value} device errors", 0, 0))
    except Exception as e:  # reported to the parent
        q_out.put((rank, None, repr(e), 0, 0))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [False, True], ids=["nccl", "fused_allreduce"])
def test_tensor_parallel_two_gpus_matches_reference(fused):
    """NCCL all-reduce, and the all-reduce fused into the projection GEMVs
    over NVLink peer memory."""
    world = 2
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    q_h = [ctx.Queue() for _ in range(world)]
    procs = [ctx.Process(target=_rank, args=(r, world, q_id, q_out, fused, q_h)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, toks, logits, v0, vl = q_out.get(timeout=600)
            assert toks is not None, f"rank {r}: {logits}"
            res[r] = (toks, logits, v0, vl)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    np.testing.assert_array_equal(res[0][0], res[1][0])
    toks = res[0][0]
    full = np.zeros((N - 1, NSEQ, SHAPE[0]), np.float32)
    for r in range(world):
        _, lg, v0, vl = res[r]
        full[:, :, v0:v0 + vl] = lg[:, :, :vl]
    s = O.LMShape(*SHAPE)
    w = O.init_weights(s, 3)
    P = 128
    for b in (0, NSEQ - 1):
        ref = O.forward(s, w, toks[b, : P + N - 1], row0=P - 1, nrows=N)
        got_tok = toks[b, P:]
        for t in range(N):
            row = ref[t]
            top2 = np.sort(row)[-2:]
            if top2[1] - top2[0] > 2e-3:
                assert O.argmax_first(row) == got_tok[t], f"sequence {b}: divergence at step {t}"
        np.testing.assert_allclose(full[:, b, :], ref[1:], rtol=RTOL, atol=ATOL)
