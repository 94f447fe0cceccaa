"""CPU checks of bench.py's own rules: the multi-GPU gather mode and the
algorithmic byte count of a decode launch (the roofline's numerator)."""
import numpy as np

import bench


def test_gather_mode_follows_the_bytes_each_rank_receives():
    qwen = bench.WORKLOADS["qwen2.5-7b-decode-b16"]          # 3.2 MB of outputs per rank
    llama70 = bench.WORKLOADS["llama3-70b-1kvhead-b256"]     # 42 MB per rank
    assert bench.choose_gather(qwen, 2) == "overlap"
    assert bench.choose_gather(qwen, 4) == "serial"
    assert bench.choose_gather(qwen, 8) == "serial"
    assert bench.choose_gather(llama70, 2) == "serial"
    assert bench.choose_gather(llama70, 8) == "serial"
    # workloads without a decode batch (prefill, GEMM, page kernels) never gather
    assert bench.choose_gather(bench.WORKLOADS["fp8-gemm-8192"], 8) == "overlap"


def test_algorithmic_bytes_of_one_sequence():
    # one Qwen-shaped sequence of 17 tokens (two pages) in bf16: KV read
    # 17 x 2 x 4 x 256, append write 2 x 4 x 256, new rows 2 x 4 x 256,
    # q and o 2 x 28 x 256, block table 2 x 4 x 4
    w = dict(bench.WORKLOADS["qwen2.5-7b-decode-b16"])
    got = bench.algorithmic_bytes_per_launch(w, np.array([17]))
    assert got == 17 * 2 * 4 * 256 + 2 * 4 * 256 + 2 * 4 * 256 + 2 * 28 * 256 + 2 * 4 * 4
    # FP8 pages: one byte per element plus a 4-byte scale per row
    f = dict(w, kv="fp8")
    got8 = bench.algorithmic_bytes_per_launch(f, np.array([17]))
    assert got8 == 17 * 2 * 4 * 132 + 2 * 4 * 132 + 2 * 4 * 256 + 2 * 28 * 256 + 2 * 4 * 4
