"""Column-parallel fused linear on 2..8 GPUs of one node (skipped with fewer
than two): each rank's kernel writes its [M, N/world] block into every rank's
y -- through CUDA-IPC peer pointers, or with one multimem store per 16 bytes
through an NVLink multicast mapping of symmetric-memory y buffers -- and a
bounded flag barrier completes the call.  The assembled y must equal, bit for
bit, the single-GPU fused linear on the full weight (split-K off on both
sides), and the NCCL all-gather path.  The failure test stays on the IPC path
(no multicast object exists while a rank is made to miss a call)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(7, 256, 256), (300, 1024, 512), (1000, 2048, 1024), (2304, 3072, 1536)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, multicast=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    nccl = dist.new_group(backend="nccl", timeout=datetime.timedelta(seconds=60))
    from diffuser_b200 import ops, tp
    results = []
    try:
        grp = tp.TpGroup(max_tokens=2304, max_out_features=3072, pg=nccl if multicast else None,
                         multicast=multicast)
    except RuntimeError as e:
        if "multicast" not in str(e):
            raise
        np.save(os.path.join(out_dir, f"tp_{rank}.npy"),
                np.array([("no_multicast", 0, 0, 0, True, True, 0.0)], dtype=object), allow_pickle=True)
        dist.destroy_process_group(nccl)
        dist.destroy_process_group()
        return
    try:
        for fmt in ("nf4", "fp8"):
            for (m, n, k) in SHAPES:
                g = torch.Generator(device="cuda").manual_seed(m + n + k)
                w = torch.randn(n, k, generator=g, device="cuda") * 0.02
                x = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
                bias = (torch.randn(n, generator=g, device="cuda") * 0.5).to(torch.bfloat16)
                ops.set_tile_override(0, 1)  # the column-parallel path never splits K
                try:
                    if fmt == "nf4":
                        p, a = ops.ltx23_nf4_quantize(w)
                        ref = ops.nf4_linear(x, p, a, n, bias)
                        mod = tp.ColumnParallelNf4Linear(k, n, grp, bias=True).cuda()
                        mod.set_nf4_weight(p, a)
                    else:
                        w8, s = ops.fp8_quantize(w)
                        ref = ops.fp8_linear(x, w8, float(s.item()), bias)
                        mod = tp.ColumnParallelFp8Linear(k, n, grp, bias=True).cuda()
                        mod.set_fp8_weight(w8, float(s.item()))
                finally:
                    ops.set_tile_override(0, 0)
                mod.set_bias(bias)
                torch.cuda.synchronize()
                dist.barrier()
                same = []
                for _ in range(3):  # several epochs, both output buffers
                    y = mod(x)
                    torch.cuda.synchronize()
                    same.append(bool(torch.equal(y, ref)))
                ops.set_tile_override(0, 1)  # same no-split plan for the local shard
                try:
                    y2 = mod.forward_nccl(x, pg=nccl)
                    torch.cuda.synchronize()
                finally:
                    ops.set_tile_override(0, 0)
                rel = ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
                results.append((fmt, m, n, k, all(same), bool(torch.equal(y2, ref)), rel))
        results.append(("device_error", ops.device_error(), 0, 0, True, True, 0.0))
    finally:
        grp.close()
        dist.destroy_process_group(nccl)
        dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"tp_{rank}.npy"), np.array(results, dtype=object), allow_pickle=True)


@pytest.mark.parametrize("multicast", [False, True], ids=["peer_stores", "multimem"])
def test_column_parallel_matches_single_gpu(tmp_path, multicast):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), multicast), nprocs=world,
                       join=True, start_method="spawn")
    table = {r: [tuple(row) for row in np.load(tmp_path / f"tp_{r}.npy", allow_pickle=True)]
             for r in range(world)}
    if any(row[0] == "no_multicast" for rows in table.values() for row in rows):
        pytest.skip("NVLink multicast is not available on these GPUs")
    for r, rows in table.items():
        for fmt, m, n, k, fused_equal, nccl_equal, rel in rows:
            if fmt == "device_error":
                assert m == 0, table
                continue
            assert fused_equal and nccl_equal, table


def _timeout_rank(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    from diffuser_b200 import ops, tp
    grp = tp.TpGroup(max_tokens=64, max_out_features=256)
    code = -1
    try:
        w = torch.randn(256, 128, device="cuda") * 0.02
        w8, s = ops.fp8_quantize(w)
        mod = tp.ColumnParallelFp8Linear(128, 256, grp, bias=False).cuda()
        mod.set_fp8_weight(w8, float(s.item()))
        x = torch.randn(16, 128, device="cuda").to(torch.bfloat16)
        ops.device_error()  # clear
        dist.barrier()
        if rank == 0:
            # the peers skip this call: their flags never reach this epoch, so
            # the bounded wait runs out and records a timeout (no fault, no hang)
            mod(x)
            torch.cuda.synchronize()
        code = ops.device_error()
        dist.barrier()
    finally:
        grp.close()
        dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"timeout_{rank}.npy"), np.array([code]))


def test_column_parallel_wait_times_out_when_a_rank_is_missing(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    from diffuser_b200 import _lib
    mp.start_processes(_timeout_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    assert int(np.load(tmp_path / "timeout_0.npy")[0]) == _lib.DQ_ERR_TIMEOUT
    for r in range(1, world):
        assert int(np.load(tmp_path / f"timeout_{r}.npy")[0]) == 0
