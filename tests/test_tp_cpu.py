"""Host-side tests of the column-parallel linear (no GPU): the sharding of the
reference's flat NF4 / fp8 buffers over out_features is row-local and exact,
and world-size-2 gloo ranks that each compute only their shard reassemble the
full reference output bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diffuser_b200 import tp
from oracle import numpy_ref as R
from tests.gpu_util import seeded_bf16, seeded_f32, to_bits


def test_shard_rows_partition_the_weight():
    for world in (1, 2, 4, 8):
        spans = [tp.shard_rows(12288, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == 12288
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        tp.shard_rows(100, 3, 0)
    with pytest.raises(ValueError):
        tp.shard_rows(128, 2, 2)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_nf4_shard_equals_quantized_rows(world):
    # NF4 blocks never straddle a weight row: quantizing the full W and taking
    # rank r's byte ranges equals quantizing rank r's rows alone.
    n, k = 64 * world, 192
    w = seeded_f32((n, k), 7, 0.02).numpy()
    packed, absmax = R.nf4_quantize(w)
    for r in range(world):
        p, a = tp.shard_nf4(packed, absmax, n, k, world, r)
        n0, n1 = tp.shard_rows(n, world, r)
        p2, a2 = R.nf4_quantize(w[n0:n1])
        assert np.array_equal(p, p2) and np.array_equal(a, a2)


def test_shard_size_checks():
    packed = np.zeros(64 * 128 // 2, np.uint8)
    absmax = np.ones(64 * 128 // 64, np.float32)
    with pytest.raises(ValueError):
        tp.shard_nf4(packed, absmax, 64, 100, 2, 0)
    with pytest.raises(ValueError):
        tp.shard_nf4(packed[:-2], absmax, 64, 128, 2, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, fmt, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k = 9, 256, 192
        x = to_bits(seeded_bf16((m, k), 3))
        w = seeded_f32((n, k), 4, 0.02).numpy()
        bias = to_bits(seeded_bf16((n,), 5, 0.5))
        n0, n1 = tp.shard_rows(n, world, rank)
        if fmt == "nf4":
            packed, absmax = R.nf4_quantize(w)
            p, a = tp.shard_nf4(packed, absmax, n, k, world, rank)
            block = R.nf4_linear_bf16(x, np.ascontiguousarray(p), np.ascontiguousarray(a), n1 - n0, k,
                                      bias[n0:n1])
            full = R.nf4_linear_bf16(x, packed, absmax, n, k, bias)
        else:
            w8, scale = R.fp8_quantize(w)
            block = R.fp8_linear_bf16(x, np.ascontiguousarray(tp.shard_fp8(w8, world, rank)), scale,
                                      n1 - n0, k, bias[n0:n1])
            full = R.fp8_linear_bf16(x, w8, scale, n, k, bias)
        # all-gather the [M, N/world] blocks and restore [M, N]
        t = torch.from_numpy(block.astype(np.int32))
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        y = torch.cat(parts, dim=1).numpy().astype(np.uint16)
        np.save(os.path.join(out_dir, f"ok_{rank}.npy"), np.array([np.array_equal(y, full)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt", ["nf4", "fp8"])
def test_gloo_world2_shards_reassemble_the_reference_output(tmp_path, fmt):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), fmt, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        assert bool(np.load(tmp_path / f"ok_{r}.npy")[0])
