"""Column-parallel (tensor-parallel over out_features) quantized linears.

The reference runs each quantized linear on one GPU (R/nf4_ltx23.R:235-246,
R/fp8_ltx23.R:70-83).  Here the weight rows are split across the `world`
GPUs of one node: rank r owns rows [r*N/world, (r+1)*N/world).  NF4 blocks of
64 never straddle a weight row, so a rank's share of the reference's packed
buffer is the contiguous byte range [n0*K/2, n1*K/2) and of absmax the range
[n0*K/64, n1*K/64); fp8 shards are row slices sharing the scalar scale.

`forward` runs the fused dequant-GEMM on the local shard and its epilogue
stores every output tile straight into every rank's y [M, N] over NVLink
(peer pointers from CUDA IPC), then raises a per-rank flag; a bounded device
wait completes the call.  With `TpGroup(..., multicast=True)` the y buffers
are symmetric memory bound to an NVLink multicast object and each epilogue
store is a single `multimem.st` that the NVSwitch writes into every rank's y:
a rank's NVLink egress is its own block once instead of once per peer.  There
is no library collective on this path; `forward_nccl` is the conventional
alternative (local GEMM, NCCL all-gather, column permute) kept for comparison.

Every rank must call the same modules in the same order with the same token
count.  The returned y is a view of a shared buffer that is double-buffered:
it stays valid until the second-next call of any module of the same group.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, ops

NF4_BLOCK = 64


# ------------------------------------------------------------------ shards
def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [n0, n1) of an N-row weight owned by `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n % world != 0:
        raise ValueError(f"out_features {n} is not divisible by the {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_nf4(packed, absmax, n: int, k: int, world: int, rank: int):
    """This rank's byte ranges of the reference's flat NF4 buffers
    (`weight_nf4` uint8 [N*K/2], `weight_absmax` f32 [N*K/64])."""
    if k % NF4_BLOCK != 0:
        raise ValueError("in_features must be a multiple of 64 for NF4")
    n0, n1 = shard_rows(n, world, rank)
    flat_p = packed.reshape(-1)
    flat_a = absmax.reshape(-1)
    if flat_p.shape[0] != n * k // 2 or flat_a.shape[0] != n * k // NF4_BLOCK:
        raise ValueError("packed / absmax sizes do not match (N, K)")
    return (flat_p[n0 * k // 2:n1 * k // 2], flat_a[n0 * k // NF4_BLOCK:n1 * k // NF4_BLOCK])


def shard_fp8(w8, world: int, rank: int):
    """This rank's rows of an e4m3 weight [N, K]."""
    n0, n1 = shard_rows(w8.shape[0], world, rank)
    return w8[n0:n1]


def shard_bias(bias, n: int, world: int, rank: int):
    if bias is None:
        return None
    n0, n1 = shard_rows(n, world, rank)
    return bias[n0:n1]


# ------------------------------------------------------------ shared buffers
class _CudaView:
    """A raw device allocation presented to torch (zero copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def _check(name, rc):
    _lib.check(name, rc)


class TpGroup:
    """Buffers shared by the `world` ranks of one column-parallel group.

    Per rank: two output buffers of `max_tokens x max_out_features` bf16 (used
    alternately), a uint32[world] flag array and a uint32 completion counter,
    allocated by the library and mapped into every other rank's process with
    CUDA IPC.  `pg` is any torch.distributed process group spanning the ranks
    (gloo is enough: it only carries the 64-byte IPC handles once).
    """

    def __init__(self, max_tokens: int, max_out_features: int, pg=None, device=None,
                 multicast: bool = False):
        import torch.distributed as dist
        self.pg = pg
        self.rank = dist.get_rank(pg)
        self.world = dist.get_world_size(pg)
        if self.world > 8:
            raise ValueError("column-parallel groups span at most 8 GPUs")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.max_tokens = int(max_tokens)
        self.max_n = int(max_out_features)
        self.epoch = 0
        lib = _lib.lib()
        ybytes = self.max_tokens * self.max_n * 2
        self._own = []
        self._symm = None
        self._mc = None
        with torch.cuda.device(self.device):
            if multicast:
                ys = self._symmetric_y(ybytes)
                shared = (256,)  # flags (the counter below is never shared)
            else:
                shared = (ybytes, ybytes, 256)  # y0, y1, flags
            for nbytes in shared + (256,):  # ..., counter
                p = ctypes.c_void_p()
                _check("dq_tp_buffer_alloc", lib.dq_tp_buffer_alloc(nbytes, ctypes.byref(p)))
                self._own.append(p.value)
            handles = []
            for p in self._own[:len(shared)]:
                h = ctypes.create_string_buffer(_lib.DQ_IPC_HANDLE_BYTES)
                _check("dq_ipc_handle", lib.dq_ipc_handle(ctypes.c_void_p(p), h))
                handles.append(h.raw)
            gathered = [None] * self.world
            dist.all_gather_object(gathered, handles, group=pg)
            self._opened = []
            ptrs = [[None] * self.world for _ in range(len(shared))]
            for q in range(self.world):
                for j in range(len(shared)):
                    if q == self.rank:
                        ptrs[j][q] = self._own[j]
                    else:
                        p = ctypes.c_void_p()
                        _check("dq_ipc_open", lib.dq_ipc_open(gathered[q][j], ctypes.byref(p)))
                        self._opened.append(p.value)
                        ptrs[j][q] = p.value
        if multicast:
            ptrs = ys + ptrs
        arr = ctypes.c_void_p * self.world
        self._y_ranks = [arr(*ptrs[0]), arr(*ptrs[1])]
        self._flag_ranks = arr(*ptrs[2])
        self._counter = ctypes.c_void_p(self._own[-1])
        self._closed = False

    @property
    def multicast(self) -> bool:
        return self._mc is not None

    def _symmetric_y(self, ybytes: int):
        """The two y buffers as one symmetric-memory allocation bound to an
        NVLink multicast object.  Returns the per-rank pointer lists of both
        halves and keeps the multicast address of each half."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        group = self.pg if self.pg is not None else dist.group.WORLD
        try:  # older releases need the group registered first
            symm.enable_symm_mem_for_group(group.group_name)
        except Exception:  # noqa: BLE001 - newer ones need nothing
            pass
        buf = symm.empty(2 * ybytes // 2, dtype=torch.bfloat16, device=self.device)
        hdl = symm.rendezvous(buf, group)
        base = buf.data_ptr()
        peers = list(hdl.buffer_ptrs)
        if not hdl.multicast_ptr or peers[self.rank] != base:
            raise RuntimeError("NVLink multicast is not available for this group")
        self._symm = (buf, hdl)
        self._mc = [hdl.multicast_ptr, hdl.multicast_ptr + ybytes]
        return [[p for p in peers], [p + ybytes for p in peers]]

    def next_call(self):
        """Advance to the next call: (epoch, y-rank pointer array, own y ptr,
        multicast address of the y buffer or None)."""
        self.epoch += 1
        buf = self.epoch & 1
        own = self._y_ranks[buf][self.rank]
        return self.epoch, self._y_ranks[buf], own, None if self._mc is None else self._mc[buf]

    def output_view(self, ptr: int, m: int, n: int) -> torch.Tensor:
        t = torch.as_tensor(_CudaView(ptr, (m, n), "<u2"), device=self.device)
        return t.view(torch.bfloat16)

    def close(self):
        """Unmap peers and free this rank's buffers (collective: every rank
        calls it after its last use)."""
        if self._closed:
            return
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pg)
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.dq_ipc_close(ctypes.c_void_p(p))
            dist.barrier(group=self.pg)
            for p in self._own:
                lib.dq_tp_buffer_free(ctypes.c_void_p(p))
        self._symm = None
        self._mc = None
        self._closed = True


# ------------------------------------------------------------------ modules
class _ColumnParallelBase(torch.nn.Module):
    def __init__(self, in_features: int, out_features: int, group: TpGroup, bias: bool):
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.group = group
        self.n0, self.n1 = shard_rows(self.out_features, group.world, group.rank)
        if self.out_features > group.max_n:
            raise ValueError("out_features exceeds the group's buffer width")
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(self.n1 - self.n0, dtype=torch.bfloat16),
                                           requires_grad=False)
        else:
            self.register_parameter("bias", None)

    def set_bias(self, full_bias: torch.Tensor):
        with torch.no_grad():
            self.bias.copy_(full_bias.reshape(-1)[self.n0:self.n1])

    def _prep(self, x):
        if not x.is_cuda:
            raise RuntimeError("the column-parallel linear has no CPU path")
        if x.dtype != torch.bfloat16:
            raise TypeError("activations must be bfloat16")
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        m = x2.shape[0]
        if m > self.group.max_tokens:
            raise ValueError(f"{m} tokens exceed the group's buffer ({self.group.max_tokens})")
        return x2, m

    def _launch(self, fn, x2, m, weight_args, fmt):
        """One column-parallel call through the workspace-taking entry point:
        from 1024 tokens each rank runs the two-phase plan (its shard decoded
        once into the workspace inside the GEMM launch)."""
        g = self.group
        epoch, y_ranks, own, mc = g.next_call()
        n = self.out_features
        # the shared buffer is [max_tokens, max_n]; this call uses its first m*n
        stream = ctypes.c_void_p(torch.cuda.current_stream(x2.device).cuda_stream)
        ws_bytes = max(ops.workspace_size(m, self.n1 - self.n0, self.in_features, fmt), 256)
        ws = ops.workspace(x2.device, ws_bytes)
        b = self.bias
        head = (ctypes.c_void_p(x2.data_ptr()), m, self.in_features, *weight_args,
                None if b is None else ctypes.c_void_p(b.data_ptr()), n, g.rank, g.world, y_ranks)
        tail = (g._flag_ranks, g._counter, epoch, ctypes.c_void_p(ws.data_ptr()), ws_bytes, stream)
        rc = fn(*head, *tail) if mc is None else fn(*head, ctypes.c_void_p(mc), *tail)
        _check(fn.__name__ if hasattr(fn, "__name__") else "dq_tp_linear", rc)
        return g.output_view(own, m, n)

    def forward(self, x):
        x2, m = self._prep(x)
        y = self._forward_fused(x2, m)
        return y.reshape(*x.shape[:-1], self.out_features)

    def forward_nccl(self, x, pg=None):
        """Local fused GEMM, NCCL all-gather of the [M, N/world] blocks over
        process group `pg` (NCCL), then the permute to [M, N] (the
        library-collective baseline)."""
        import torch.distributed as dist
        x2, m = self._prep(x)
        y_local = self._forward_local(x2)
        blocks = torch.empty((self.group.world, m, self.n1 - self.n0), dtype=torch.bfloat16,
                             device=x2.device)
        dist.all_gather_into_tensor(blocks, y_local, group=pg)
        y = blocks.permute(1, 0, 2).reshape(m, self.out_features)
        return y.reshape(*x.shape[:-1], self.out_features)


class ColumnParallelNf4Linear(_ColumnParallelBase):
    """`ltx23_nf4_linear` (R/nf4_ltx23.R:211-247) split over out_features."""

    def __init__(self, in_features, out_features, group: TpGroup, bias=True):
        super().__init__(in_features, out_features, group, bias)
        n_local = self.n1 - self.n0
        self.register_buffer("weight_nf4", torch.zeros(n_local * self.in_features // 2,
                                                       dtype=torch.uint8))
        self.register_buffer("weight_absmax", torch.ones(n_local * self.in_features // NF4_BLOCK,
                                                         dtype=torch.float32))

    def set_nf4_weight(self, packed_full, absmax_full):
        """Keep this rank's share of the full packed / absmax buffers."""
        p, a = shard_nf4(packed_full, absmax_full, self.out_features, self.in_features,
                         self.group.world, self.group.rank)
        with torch.no_grad():
            self.weight_nf4.copy_(p)
            self.weight_absmax.copy_(a)

    def _forward_fused(self, x2, m):
        lib = _lib.lib()
        fn = lib.dq_tp_linear_nf4_mc_ws if self.group.multicast else lib.dq_tp_linear_nf4_ws
        return self._launch(fn, x2, m,
                            (ctypes.c_void_p(self.weight_nf4.data_ptr()),
                             ctypes.c_void_p(self.weight_absmax.data_ptr())), _lib.DQ_FMT_NF4)

    def _forward_local(self, x2):
        return ops.nf4_linear(x2, self.weight_nf4, self.weight_absmax, self.n1 - self.n0, self.bias)


class ColumnParallelFp8Linear(_ColumnParallelBase):
    """`ltx23_fp8_linear` (R/fp8_ltx23.R:49-84) split over out_features."""

    def __init__(self, in_features, out_features, group: TpGroup, bias=True):
        super().__init__(in_features, out_features, group, bias)
        self.register_buffer("weight_fp8", torch.zeros(self.n1 - self.n0, self.in_features,
                                                       dtype=torch.uint8))
        self.scale = 1.0

    def set_fp8_weight(self, w8_full, scale):
        with torch.no_grad():
            self.weight_fp8.copy_(shard_fp8(w8_full, self.group.world, self.group.rank)
                                  .view(torch.uint8))
        self.scale = float(scale)

    def _forward_fused(self, x2, m):
        lib = _lib.lib()
        fn = lib.dq_tp_linear_fp8_mc_ws if self.group.multicast else lib.dq_tp_linear_fp8_ws
        return self._launch(fn, x2, m,
                            (ctypes.c_void_p(self.weight_fp8.data_ptr()), ctypes.c_float(self.scale)),
                            _lib.DQ_FMT_FP8)

    def _forward_local(self, x2):
        return ops.fp8_linear(x2, self.weight_fp8.view(torch.float8_e4m3fn), self.scale, self.bias)

