"""The roofline numerators bench.py reports (algorithmic bytes and FLOPs of
the decode step, the attention kernel and the prefill), checked on the CPU
against the figures the path's arithmetic gives by hand, so that a
roofline fraction always divides the work the path must do."""
import bench


# (d, L, vocab): BASELINE configs 3, 4 and 5
CFG3, CFG4, CFG5 = (512, 8, 4096), (1024, 12, 32000), (4096, 32, 32000)


def test_weight_bytes_per_step():
    # 12 d^2 per layer (QKV 3, proj 1, fc 4, mlp 4), the tied embedding once,
    # (2L + 1) LayerNorm gammas, fp32
    for (d, L, V), mb in ((CFG3, 109.1), (CFG4, 735.2), (CFG5, 26295.2)):
        want = 4 * (12 * d * d * L + V * d + (2 * L + 1) * d)
        assert bench.weight_bytes(d, L, V) == want
        assert abs(want / 1e6 - mb) < 0.1


def test_bf16_weight_bytes_per_step():
    # the bf16-weight mode streams the 12 d^2 per layer and the lm_head rows
    # at 2 bytes; the gammas stay fp32
    for d, L, V in (CFG3, CFG4, CFG5):
        want = 2 * (12 * d * d * L + V * d) + 4 * (2 * L + 1) * d
        assert bench.weight_bytes_bf16(d, L, V) == want
        assert abs(bench.weight_bytes_bf16(d, L, V) / bench.weight_bytes(d, L, V) - 0.5) < 1e-3


def test_tensor_parallel_weight_share():
    d, L, V = CFG5
    full = bench.weight_bytes(d, L, V)
    half = bench.weight_bytes(d, L, V, tpw=2)
    # every contraction and the vocabulary split in two; gammas replicated
    assert half == 4 * (6 * d * d * L + V // 2 * d + (2 * L + 1) * d)
    assert abs(half / full - 0.5) < 1e-3


def test_decode_pass_bytes_config3_average():
    d, L, V = CFG3
    B, P, steps = 32, 128, 383
    total = bench.decode_pass_bytes(d, L, V, B, P, steps)
    # 0.445 GB per engine step on average: 109 MB of weights and ~10.5 MB of
    # K/V per sequence at the mean key length
    assert abs(total / steps / 1e9 - 0.445) < 0.003
    # the step's bytes = weights + the attention kernel's bytes + each
    # sequence's residual row read and written
    attn = bench.attention_pass_bytes(d, L, B, P, steps)
    assert total == steps * bench.weight_bytes(d, L, V) + attn + steps * B * 4 * 2 * d


def test_attention_bytes_per_launch_config3():
    d, L, _ = CFG3
    B, P, steps = 32, 128, 383
    per_launch = bench.attention_pass_bytes(d, L, B, P, steps) / (steps * L)
    # K and V of 320 keys on average (32 sequences x 512 floats), plus q / out
    assert abs(per_launch / 1e6 - 42.07) < 0.01


def test_prefill_flops():
    for (d, L, V), B, P, tflop in ((CFG3, 32, 128, 0.21), (CFG4, 64, 1536, 33.4), (CFG5, 8, 1024, 107.8)):
        f = bench.prefill_flops(d, L, V, B, P)
        assert f == L * (24 * B * P * d * d + 2 * B * P * P * d) + 2 * B * V * d
        assert abs(f / 1e12 - tflop) / tflop < 0.01


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` times the reference's own CPU path on the
    host (one step here) and prints one JSON line with the same metric, unit
    and direction as the GPU arm, marked as the reference."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert (d["metric"], d["unit"], d["higher_is_better"]) == (bench.METRIC, bench.UNIT, True)
    assert d["value"] > 0 and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_kernel_times_from_stamps():
    """In-graph kernel times: each kernel's completion minus the previous
    kernel's; the first kernel of a step is measured from the previous
    step's last; step 0 (no previous step in the pass) is left out; the
    per-class times add up to the stamped step time."""
    import numpy as np
    classes = ["embed", "qkv", "attention", "finalize"]
    # two steps of 4 kernels, completion times in ns
    stamps = np.array([[100, 110, 150, 160],
                       [170, 185, 235, 240]], dtype=np.int64)
    kt = bench.kernel_times_from_stamps(stamps, classes)
    assert kt["steps"] == 1
    assert kt["by_class_ns"] == {"embed": 10, "qkv": 15, "attention": 50, "finalize": 5}
    assert kt["launches"] == {"embed": 1, "qkv": 1, "attention": 1, "finalize": 1}
    assert kt["total_ns"] == 80 == sum(kt["by_class_ns"].values())


def test_decode_contraction_path_follows_the_engine_rule():
    """The bench line names where the decode contractions ran: tensor cores
    from 32 rows with d a multiple of 1024 on one rank (config 4 at one and
    two GPUs), CUDA-core GEMVs otherwise (config 3, config 4 at 16 rows per
    GPU, config 5 with or without tensor parallelism); the logits head on
    tensor cores from 32 rows and 148 column tiles of the rank's vocabulary."""
    p = bench.decode_contraction_path
    assert p(512, 4096, 32, False).startswith("decode contractions on the CUDA cores")
    assert "logits head on a CUDA-core GEMV" in p(512, 4096, 32, False)  # 32 column tiles
    assert p(1024, 32000, 64, False) == ("decode contractions on tcgen05 (TF32x3, K split + reduction), "
                                         "logits head on tcgen05 (TF32x3)")
    assert p(1024, 32000, 32, False).startswith("decode contractions on tcgen05")
    assert p(1024, 32000, 16, False).startswith("decode contractions on the CUDA cores")
    assert "logits head on a CUDA-core GEMV" in p(1024, 32000, 16, False)
    assert p(4096, 32000, 8, False).startswith("decode contractions on the CUDA cores")
    assert p(4096, 16000, 8, True).startswith("decode contractions on the CUDA cores")
