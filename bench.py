"""Decode throughput of FreeML's NanoLLM token loop on B200.

Workload: BASELINE config 3 -- vocab 4096, context 512, d_model 512, 8 heads,
8 layers, 4x GELU MLP; 32 independent sequences, 128-token prompts, greedy
decode of 384 tokens.  Sequences are sharded 32/N across N GPUs (one process
per GPU, no collective on the data path): total work is fixed, so the scaling
is strong.

One bench step = one full greedy decode pass of this rank's sequences: rewind
every sequence to the end of its prompt (the prefill is done once, untimed),
then 383 engine steps (tokens 2..384; the first comes from the prefill).  The
metric counts the tokens those engine steps produce.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (1/2/4/8 B200) & % HBM roofline; vs FreeML MatrixCPU host"
UNIT = "tokens/s"
CONFIG = 3
FALLBACK_HBM_GBS = 6650.0


# ---- algorithmic work (the roofline numerators), fp32 throughout ----------

def weight_bytes(d: int, L: int, vocab: int, tpw: int = 1) -> int:
    """Weight bytes one rank reads per engine step: per layer QKV 3d x d/tpw,
    projection d/tpw x d, fc d x 4d/tpw, mlp 4d/tpw x d; the tied embedding's
    vocabulary slice as the logits head; the LayerNorm gammas (2L + 1) x d."""
    dl, fl, vl = d // tpw, 4 * d // tpw, -(-vocab // tpw)
    return 4 * (L * (4 * d * dl + 2 * d * fl) + vl * d + (2 * L + 1) * d)


def weight_bytes_bf16(d: int, L: int, vocab: int, tpw: int = 1) -> int:
    """weight_bytes with the decode GEMVs' matrices and the lm_head rows at
    2 bytes (the bf16-weight mode); the LayerNorm gammas stay fp32."""
    dl, fl, vl = d // tpw, 4 * d // tpw, -(-vocab // tpw)
    return 2 * (L * (4 * d * dl + 2 * d * fl) + vl * d) + 4 * (2 * L + 1) * d


def decode_pass_bytes(d: int, L: int, vocab: int, B: int, P: int, steps: int, tpw: int = 1) -> int:
    """Bytes of one decode pass of B sequences from key length P: every step
    reads the weights once, each sequence's cached K and V rows (p + 1 keys of
    d/tpw per layer), writes its new K/V row, and reads and writes its
    residual row."""
    dl = d // tpw
    return sum(weight_bytes(d, L, vocab, tpw) + B * 4 * (2 * dl * L * (p + 1) + 2 * dl * L + 2 * d)
               for p in range(P, P + steps))


def attention_pass_bytes(d: int, L: int, B: int, P: int, steps: int, tpw: int = 1) -> int:
    """Bytes the decode attention kernels move over one pass: the K and V
    rows of p + 1 keys per sequence and layer, and the q and output rows."""
    dl = d // tpw
    return sum(4 * L * B * (2 * dl * (p + 1) + 2 * dl) for p in range(P, P + steps))


def prefill_flops(d: int, L: int, vocab: int, B: int, P: int) -> int:
    """FLOPs of one prefill of B prompts of P tokens: 2 x 12 d^2 per token
    and layer for the four contractions, causal attention at half of
    4 P^2 d per sequence and layer, and the last row's logits."""
    return L * (24 * B * P * d * d + 2 * B * P * P * d) + 2 * B * vocab * d


def kernel_times_from_stamps(stamps, classes):
    """Per-class time inside the step graph from completion stamps
    [steps, kernels] (ns): a kernel's time is its completion minus the
    previous kernel's (the first kernel of step s: minus step s-1's last).
    Step 0 has no previous step in the pass and is left out."""
    by, n, total = {}, {}, 0
    steps, nk = stamps.shape
    for st in range(1, steps):
        prev = int(stamps[st - 1, nk - 1])
        for i in range(nk):
            t = int(stamps[st, i])
            by[classes[i]] = by.get(classes[i], 0) + (t - prev)
            n[classes[i]] = n.get(classes[i], 0) + 1
            prev = t
        total += int(stamps[st, nk - 1]) - int(stamps[st - 1, nk - 1])
    return {"by_class_ns": by, "launches": n, "total_ns": total, "steps": max(steps - 1, 0)}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", action="store_true",
                    help="with N > 1 GPUs: tensor parallelism over all ranks (each runs every sequence) "
                         "instead of sequence sharding (BASELINE config 5's scheme)")
    ap.add_argument("--tp-nccl", action="store_true",
                    help="with --tp: NCCL all-reduce calls instead of the one-shot all-reduce over NVLink peer "
                         "memory")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=3,
                    help="BASELINE config (3 is the headline metric's; 4 and 5 add a timed prefill; 2 is the "
                         "per-operator microbench through the C ABI)")
    ap.add_argument("--profile-only", action="store_true", help="a few passes for ncu (no JSON)")
    ap.add_argument("--profile-phase", choices=["decode", "prefill"], default="decode",
                    help="with --profile-only: 3 decode steps at mid-decode, or one prefill")
    return ap.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def decode_contraction_path(d: int, vocab: int, b_local: int, tp: bool) -> str:
    """Where the engine runs one rank's decode contractions (default math
    mode TF32x3, fp32 weights; vocab = the rank's vocabulary rows): the
    rule of lm_engine.cu's
    decode_on_tensor_cores (one rank, d a multiple of 1024 up to 4096, at
    least 32 rows) and lm_head_on_tensor_cores (at least 32 rows and 148
    column tiles of 128 in the vocabulary)."""
    dense = not tp and d % 1024 == 0 and d <= 4096 and b_local >= 32
    head = b_local >= 32 and -(-vocab // 128) >= 148
    where = "tcgen05 (TF32x3, K split + reduction)" if dense else "the CUDA cores (fp32 GEMVs)"
    head_where = "tcgen05 (TF32x3)" if head else "a CUDA-core GEMV with fused argmax"
    return f"decode contractions on {where}, logits head on {head_where}"


def workload_config(n_gpus, b_local, tp=False):
    from freeml_b200.lm import CONFIGS
    c = CONFIGS[CONFIG]
    s = c["shape"]
    return {"workload": f"BASELINE config {CONFIG}: NanoLLM V{s.vocab} C{s.context} d{s.d_model} H{s.n_head} "
                        f"L{s.n_layer}, {c['batch']} sequences, prompt {c['prompt']}, greedy decode {c['new']}",
            "vocab": s.vocab, "context": s.context, "d_model": s.d_model, "n_head": s.n_head, "n_layer": s.n_layer,
            "sequences": c["batch"], "sequences_per_gpu": b_local, "prompt": c["prompt"], "decode_tokens": c["new"],
            "step": f"one greedy decode pass ({c['new'] - 1} engine steps) of every sequence",
            "l2": "per engine step the working set (all weights + the K/V rows read) exceeds the 126 MB L2",
            "parallelism": (f"tp{n_gpus} (heads / fc columns / vocabulary split, all-reduce after each "
                            f"row-parallel projection)") if tp else f"dp{n_gpus} (sequence sharding, no collective)"}


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi samples (200 ms) of one GPU while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def ncu_traffic(name):
    """dram bytes (read + write) per launch of the dominant kernel, from the
    committed ncu summary (profiles/<name>_traffic.json) taken at the bench's
    average key length."""
    p = os.path.join(ROOT, "profiles", f"{name}_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return None


# ------------------------------------------------------------ reference arm --

def cpu_reference_time(forwards: int, warmup: int):
    """FreeML's own MatrixCPU Model::Run on config 3's window (T = 512), the
    reference harness built from the FreeML tree (oracle/_ref).  Falls back to
    the C oracle restatement when the harness was not built."""
    from freeml_b200.lm import CONFIGS
    from oracle import oracle as O
    c = CONFIGS[CONFIG]
    s = c["shape"]
    sh = O.LMShape(s.vocab, s.context, s.d_model, s.n_head, s.n_layer)
    if O.ref_available():
        r = O.ref_time(sh, c["wseed"], forwards, warmup, pseed=c["pseed"])
        return {"seconds_per_forward": r["seconds_per_forward"], "threads": r["threads"], "kind": "reference",
                "forwards": forwards}
    ncpu = os.cpu_count() or 1
    O.set_threads(ncpu)
    w = O.init_weights(sh, c["wseed"])
    toks = O.prompt_tokens(c["pseed"], s.vocab, s.context)
    for _ in range(warmup):
        O.forward(sh, w, toks, row0=s.context - 1, nrows=1)
    t0 = time.perf_counter()
    for _ in range(forwards):
        O.forward(sh, w, toks, row0=s.context - 1, nrows=1)
    dt = (time.perf_counter() - t0) / forwards
    return {"seconds_per_forward": dt, "threads": ncpu, "kind": "port", "forwards": forwards}


def run_reference(args, ws, rank):
    if rank != 0:
        return 0
    # a reference step = one full-window Model::Run (one token for one
    # sequence); cap the count so that the run stays within a few minutes
    est = 6.0
    k = max(1, min(args.steps, int(240 / est)))
    w = max(0, min(args.warmup, 2))
    r = cpu_reference_time(k, w)
    tps = 1.0 / r["seconds_per_forward"]
    b = workload_config(1, 32)
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": ws, "steps": k,
            "warmup": w, "ms_per_step": r["seconds_per_forward"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded weights/prompts)",
            "config": b,
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": r["threads"], "kind": r["kind"],
                             "sample": f"{k} full-window (T=512) forwards of one sequence after {w} warm-up; the "
                                       "reference recomputes the whole window per generated token, batch 1, so "
                                       "tokens/s = 1 / seconds per forward"},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.steps != k:
        line["note"] = f"steps capped at {k} (each reference step is a ~{est:.0f} s CPU forward)"
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------ config 2 --

def run_microbench(args, rank):
    """single operators through the C ABI (the calls the
    MatrixCUDA drop-in makes), seed 2, inputs N(0,1), weights N(0,0.02).
    Each call is timed alone with CUDA events, L2 flushed (a 256 MB write)
    before every timed call; median of the timed calls."""
    import torch

    from freeml_b200 import _lib
    from freeml_b200 import matrix_ops as ops
    if rank != 0:
        return 0
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(2)
    dev = torch.device("cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    peak, peak_kind = hbm_peak()
    reps = max(args.steps, 5)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        ts = []
        for _ in range(reps):
            flush.fill_(1.0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=g, device=dev) * std

    rows = []
    launches0 = _lib.launch_count()
    for (fin, fout) in [(512, 512), (1024, 4096), (4096, 1024), (4096, 4096)]:
        for batch in (1, 8, 64):
            x, w = randn(batch, fin), randn(fin, fout, std=0.02)
            y = torch.empty(batch, fout, device=dev)
            ms = timed(lambda: ops.Mul(y, x, w))
            nbytes = 4 * (fin * fout + batch * (fin + fout))
            rows.append({"op": "Dense y = x.W (Mul<None>)", "in": fin, "out": fout, "batch": batch, "us": ms * 1e3,
                         "bytes": nbytes, "GBps": nbytes / ms / 1e6, "frac_hbm": nbytes / ms / 1e6 / peak,
                         "gflops": 2 * batch * fin * fout / ms / 1e6})
    for width in (512, 4096):
        nrows = 4096
        x, gm = randn(nrows, width), torch.ones(width, device=dev)
        y = torch.empty_like(x)
        ms = timed(lambda: ops.LayerNormOp(y, x, gm))
        nbytes = 8 * nrows * width
        rows.append({"op": "LayerNormOp", "rows": nrows, "width": width, "us": ms * 1e3, "bytes": nbytes,
                     "GBps": nbytes / ms / 1e6, "frac_hbm": nbytes / ms / 1e6 / peak})
    x = randn(1 << 20)
    y = torch.empty_like(x)
    ms = timed(lambda: ops.GeluMat(y, x))
    rows.append({"op": "GeluMat", "elements": 1 << 20, "us": ms * 1e3, "bytes": 8 << 20,
                 "GBps": (8 << 20) / ms / 1e6, "frac_hbm": (8 << 20) / ms / 1e6 / peak})
    H, hd = 8, 64
    for kv in (128, 512, 2048):
        q = randn(1, H * hd)
        kc, vc = randn(1, H, kv, hd), randn(1, H, kv, hd)
        lens = torch.full((1,), kv, dtype=torch.int32, device=dev)
        out = torch.empty(1, H * hd, device=dev)
        ws_bytes = ops.attention_decode_workspace_bytes(1, H, hd, kv)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        ms = timed(lambda: ops.attention_decode(out, q, kc, vc, lens, 1.0 / hd ** 0.5, ws))
        nbytes = 4 * (2 * kv * H * hd + 2 * H * hd)
        rows.append({"op": "attention decode step (1 query, causal, split-KV)", "heads": H, "head_dim": hd,
                     "kv_len": kv, "us": ms * 1e3, "bytes": nbytes, "GBps": nbytes / ms / 1e6,
                     "frac_hbm": nbytes / ms / 1e6 / peak})
    launches = _lib.launch_count() - launches0
    line = {"metric": "per-operator time and HBM fraction (BASELINE config 2)", "value": None, "unit": "us",
            "n_gpus": 1, "steps": reps, "warmup": max(args.warmup, 3), "ms_per_step": None,
            "higher_is_better": False, "scaling": "replicas only", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seed 2, inputs N(0,1), weights N(0,0.02)",
            "config": {"workload": "BASELINE config 2 per-op microbench", "l2": "flushed before every timed call",
                       "ln_rows": 4096},
            "gpu_launches": int(launches), "peak_hbm_gbs": peak, "peak_source": peak_kind, "ops": rows}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ ours --

def main():
    global CONFIG
    args = parse()
    CONFIG = args.config
    ws, rank, local = dist_env()
    pg = None
    if ws > 1:
        import datetime

        import torch.distributed as dist
        backend = "gloo" if args.impl == "reference" else "nccl"
        if backend == "nccl":
            import torch
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
        pg = dist
    if args.impl == "reference":
        rc = run_reference(args, ws, rank)
        if pg is not None:
            pg.destroy_process_group()
        return rc
    if CONFIG == 2:
        rc = run_microbench(args, rank)
        if pg is not None:
            pg.destroy_process_group()
        return rc

    import numpy as np
    import torch

    from freeml_b200 import _lib
    from freeml_b200.lm import CONFIGS, NanoLM, prompt_tokens, random_params
    from freeml_b200.shard import max_over_ranks, shard_bounds

    torch.cuda.set_device(local)
    c = CONFIGS[CONFIG]
    s = c["shape"]
    B_total, P, NEW = c["batch"], c["prompt"], c["new"]
    if B_total % ws:
        raise SystemExit(f"{B_total} sequences do not shard evenly over {ws} GPUs")
    tp = args.tp and ws > 1
    b_lo, b_hi = (0, B_total) if tp else shard_bounds(B_total, ws, rank)
    B = b_hi - b_lo
    dp = 1 if tp else ws  # ranks whose tokens add up
    steps_per_pass = NEW - 1

    params = random_params(s, c["wseed"], local)
    prompts = prompt_tokens(c["pseed"], s.vocab, B_total, P)[b_lo:b_hi]
    lm = NanoLM(s, B, device=local)
    if tp:
        from freeml_b200.lm import nccl_unique_id
        nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            nid.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        pg.broadcast(nid, src=0)
        lm.set_tensor_parallel(rank, ws, bytes(nid.cpu().numpy().tobytes()))
        if not args.tp_nccl:
            mine = torch.frombuffer(bytearray(lm.tp_ipc_handles()), dtype=torch.uint8).cuda()
            allh = [torch.empty_like(mine) for _ in range(ws)]
            pg.all_gather(allh, mine)
            lm.tp_connect([h.cpu().numpy().tobytes() for h in allh])
    lm.bind(params)
    del params
    lm.prefill(prompts)
    first = lm.pending_tokens().clone()
    torch.cuda.synchronize()

    def one_pass():
        lm.rewind(P, first)
        lm.steps(steps_per_pass)  # graphs of several engine steps each

    def barrier():
        if pg is not None:
            pg.barrier()

    for _ in range(max(args.warmup, 0)):
        one_pass()
    torch.cuda.synchronize()

    # ---- timed prefills of this rank's prompts (tensor-core contractions);
    # each leaves the same KV rows and first tokens behind ----
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_prefill = 3  # back-to-back prefills of the same prompts, averaged
    pe0.record()
    for _ in range(n_prefill):
        lm.prefill(prompts)
    pe1.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(pe0.elapsed_time(pe1) / n_prefill, pg, "cuda")
    dm, Lm = s.d_model, s.n_layer
    prefill_flop = dp * prefill_flops(dm, Lm, s.vocab, B, P)

    if args.profile_only and args.profile_phase == "prefill":
        # for ncu (--profile-from-start off): one more prefill of the same
        # prompts (tensor-core contractions, 4096 rows) between Start/Stop
        torch.cuda.cudart().cudaProfilerStart()
        lm.prefill(prompts)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        lm.close()
        return 0

    if args.profile_only:
        # for ncu (--profile-from-start off): bring every sequence to the
        # middle of its decode (average key length), then profile 3 engine
        # steps between cudaProfilerStart/Stop
        lm.rewind(P, first)
        for _ in range(steps_per_pass // 2):
            lm.step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(3):
            lm.step()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        lm.close()
        return 0

    # ---- timed region: K passes, CUDA events on the launching stream ----
    stream = torch.cuda.current_stream()
    sampler = ClockSampler(physical_gpu(local))
    launches0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.3)  # let nvidia-smi take its first sample
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        one_pass()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    launches = _lib.launch_count() - launches0
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), pg, "cuda")
    tokens = dp * B * steps_per_pass * args.steps
    value = tokens / (ms_max / 1e3)

    # ---- e2e: the same passes through the host-buffer step (H2D + D2H) ----
    first_host = first.cpu().numpy().view(np.uint32).copy()
    e2e_passes = max(1, min(args.steps, 5))
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_passes):
        lm.rewind(P, first)
        lm.generate_host(first_host, steps_per_pass)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, "cuda")
    e2e_value = dp * B * steps_per_pass * e2e_passes / e2e_s

    # ---- the same decode passes with bf16 weights (fml_lm_set_weight_format):
    # a separate figure with its own byte count, not the fp32 headline ----
    d, L = s.d_model, s.n_layer
    tpw = ws if tp else 1
    bf_passes = max(1, min(args.steps, 5))
    lm.set_weight_format("bf16")
    one_pass()  # makes the bf16 copy and records the graphs
    barrier()
    torch.cuda.synchronize()
    bf0, bf1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    bf0.record(stream)
    for _ in range(bf_passes):
        one_pass()
    bf1.record(stream)
    torch.cuda.synchronize()
    bf_ms = max_over_ranks(bf0.elapsed_time(bf1), pg, "cuda") / bf_passes
    lm.set_weight_format("fp32")
    bf_bytes = decode_pass_bytes(d, L, s.vocab, B, P, steps_per_pass, tpw) - steps_per_pass * (
        weight_bytes(d, L, s.vocab, tpw) - weight_bytes_bf16(d, L, s.vocab, tpw))

    # ---- per-kernel times inside the replayed step graph (the timed code
    # path, with programmatic dependent launch): one more pass with
    # completion stamps, every kernel's CTAs stamping the global timer ----
    peak, peak_kind = hbm_peak()
    dl = d // tpw  # this rank's share of the weights and heads
    step_bytes = decode_pass_bytes(d, L, s.vocab, B, P, steps_per_pass, tpw)
    pass_ms = ms_max / args.steps
    stamps, classes = lm.stamped_pass(one_pass, steps_per_pass)
    kt = kernel_times_from_stamps(stamps, classes)
    # the attention launches of steps 1.. (step 0 follows the rewind kernel,
    # not a finished step, so it has no start to measure from)
    att_bytes = sum(4 * L * B * (2 * dl * (p + 1) + 2 * dl) for p in range(P + 1, P + steps_per_pass))
    att_s, att_n = kt["by_class_ns"].get("attention", 0) / 1e9, kt["launches"].get("attention", 0)
    achieved = att_bytes / att_s / 1e9 if att_s > 0 else None
    k_name = "attention_kernel (split-KV decode attention)"
    traffic = ncu_traffic("attention") if CONFIG == 3 else None

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": pass_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic: seeded N(0,0.02) weights of the config-{CONFIG} architecture, seeded uniform prompts",
            "config": dict(workload_config(ws, B, tp),
                           allreduce=("NCCL" if args.tp_nccl else "one-shot kernel over NVLink peer memory "
                                      "(decode; prefill: NCCL)") if tp else None,
                           engine="per-operation kernels (CUDA graphs of 16 engine steps, programmatic "
                                  "dependent launch between all kernels); "
                                  + decode_contraction_path(s.d_model, -(-s.vocab // (ws if tp else 1)), B, tp)
                                  + "; prefill contractions on tcgen05 (TF32x3)"),
            "gpu_launches": int(launches),
            "clocks": clocks,
            "roofline": {"bound": "hbm", "kernel": k_name,
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": (achieved / peak) if achieved else None, "peak_source": peak_kind,
                         "traffic": (traffic or {}).get("bytes_per_launch_at_bench_avg"),
                         "algorithmic_bytes_per_launch": att_bytes / max(att_n, 1),
                         "avg_launch_us": att_s / max(att_n, 1) * 1e6,
                         "share_of_step_time": kt["by_class_ns"].get("attention", 0) / kt["total_ns"]
                         if kt["total_ns"] else None,
                         "timing": "in the replayed step graph: each launch's time = its last CTA's completion "
                                   "stamp minus the previous kernel's (global timer), over steps 1..382 of one "
                                   "extra pass"},
            "step_roofline": {"algorithmic_bytes_per_pass": step_bytes,
                              "achieved_GBps": step_bytes / (pass_ms / 1e3) / 1e9,
                              "frac": step_bytes / (pass_ms / 1e3) / 1e9 / peak},
            "kernel_us_per_step": {k: v / 1e3 / max(kt["steps"], 1) for k, v in kt["by_class_ns"].items()},
            "stamped_step_us": kt["total_ns"] / 1e3 / max(kt["steps"], 1),
            "prefill": {"ms": prefill_ms, "prefills_timed": n_prefill, "tokens_per_s": dp * B * P / (prefill_ms / 1e3),
                        "algorithmic_tflop": prefill_flop / 1e12,
                        "tflops": prefill_flop / (prefill_ms / 1e3) / 1e12,
                        "math": "TF32x3 on tcgen05 (three kind::tf32 MMAs per product, fp32 accumulate in TMEM)",
                        "frac_of_tf32x3_peak": prefill_flop / (prefill_ms / 1e3) / 1e12 / (tensor_peak() / 2 / 3),
                        "peak_note": "tf32 dense = half the measured bf16 peak, / 3 for the three-pass split"},
            "bf16_weights": {"tokens_per_s": dp * B * steps_per_pass / (bf_ms / 1e3), "ms_per_pass": bf_ms,
                             "algorithmic_bytes_per_pass": bf_bytes,
                             "step_frac": bf_bytes / (bf_ms / 1e3) / 1e9 / peak,
                             "note": "decode GEMVs stream bf16 copies of the weights (fp32 accumulate); prefill, "
                                     "embedding, gammas and K/V cache fp32; a separate mode with a looser logits "
                                     "bound, not the fp32 headline"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 4 * B * dp * steps_per_pass,
                    "d2h_bytes_per_step": 4 * B * dp * steps_per_pass,
                    "path": "fml_lm_generate_host (host token buffers: every engine step copies its tokens "
                            "H2D from pinned memory, runs, copies the next tokens D2H and synchronises)"}}

    if rank == 0 and ws == 1 and not args.no_cpu_baseline and CONFIG == 3:
        try:
            r = cpu_reference_time(2, 1)
            line["cpu_baseline"] = {"value": 1.0 / r["seconds_per_forward"], "unit": UNIT, "cores": r["threads"],
                                    "kind": r["kind"],
                                    "sample": "2 full-window (T=512) forwards of one config-3 sequence after 1 "
                                              "warm-up; the reference recomputes the window per generated token "
                                              "(batch 1), so tokens/s = 1 / seconds per forward"}
        except Exception as e:  # the CPU baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": None, "kind": None,
                                    "sample": f"unavailable: {e}"}
    lm.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
