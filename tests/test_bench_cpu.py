"""Host-side checks of bench.py's helpers (CPU, no GPU).

RefGpuDequant restates the reference's per-forward weight decode as the
libtorch ops it issues (R/nf4_ltx23.R:77-115 with the byte table of
R/jit_ltx23.R:270-281; R/fp8_ltx23.R:79-80) so that bench.py can time the
reference's GPU algorithm beside the engine.  On the CPU it must produce the
oracle's bf16 weights bit for bit, including across its 4 MiB chunking.
"""
import torch

import bench
from oracle import torch_ref as T


def test_reference_gpu_decode_restatement_matches_the_oracle():
    torch.manual_seed(0)
    w = torch.randn(300, 640) * 0.02
    dq = bench.RefGpuDequant(torch.device("cpu"))
    p, a = T.ltx23_nf4_quantize(w)
    for chunk in (dq.CHUNK_BYTES, 4096, 96):  # one chunk, several, a ragged last one
        dq.CHUNK_BYTES = chunk
        got = dq.nf4(p, a, 300, 640)
        ref = T.ltx23_nf4_dequantize(p, a, (300, 640))
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    w8, s = T.fp8_quantize(w)
    got8 = dq.fp8(w8.view(torch.uint8), float(s))
    ref8 = torch.empty(300, 640, dtype=torch.bfloat16)
    T.fp8_linear_forward(torch.zeros(1, 640, dtype=torch.bfloat16), w8, s, w_buffer=ref8)
    assert torch.equal(got8.view(torch.int16), ref8.view(torch.int16))


def test_nf4_levels_match_the_oracle_table():
    assert bench.NF4_LEVELS == T.NF4_TABLE


def test_reference_arm_line_matches_the_gpu_arm_config_and_uses_every_core(capsys):
    import json
    import os
    import types

    torch.set_num_threads(1)  # what torchrun's OMP_NUM_THREADS=1 leaves behind
    args = types.SimpleNamespace(workload="nf4", warmup=0, steps=1, gpus=2)
    bench.run_reference_arm(args, world=2, rank=0)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["config"] == bench.headline_config("nf4", 2)
    assert {"M", "N", "K", "format"} <= set(line["config"])
    assert line["row_slice"] == bench.REF_ROW_SLICE
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    # the other ranks print nothing
    bench.run_reference_arm(args, world=2, rank=1)
    assert capsys.readouterr().out == ""


def test_profile_traffic_is_keyed_to_the_plan():
    plan = {"twophase": True, "pair": True, "bm": 256}
    traffic, src = bench.profile_traffic("nf4", plan)
    assert traffic is not None and traffic > 0 and "same plan" in src
    traffic, src = bench.profile_traffic("nf4", dict(plan, bm=192))
    assert traffic is None and "another plan" in src
