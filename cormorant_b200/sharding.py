"""Batch sharding across GPUs of one node (one process per GPU, torch.distributed).

Every Cormorant kernel call is independent per batch item (per image, per
batched-GEMM slice; VectorOP per element range), so ranks take contiguous
shards and run with no communication.  Only when a caller needs the outputs
together are they gathered: to every rank (``gather_batches``, an all-gather)
or to one rank (``gather_to_root``: every other rank sends its shard and the
root receives each into its offset of the full output, one grouped set of
point-to-point transfers), over NCCL (NVLink / NVSwitch) on GPUs or gloo on CPU.
"""
from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of `total` items; shares differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    lo = total * rank // world
    hi = total * (rank + 1) // world
    return lo, hi - lo


def _bytes(t):
    # neither NCCL nor gloo has an int16 type; the gathers only move bytes
    import torch
    return t.reshape(-1).view(torch.uint8)


def _check_local(local, total, per_item, rank, world):
    lo, cnt = shard_range(total, rank, world)
    if local.numel() != cnt * per_item:
        raise ValueError(f"rank {rank}: expected {cnt * per_item} words, got {local.numel()}")
    return lo, cnt


def gather_batches(local, total: int, per_item: int, group=None, out=None):
    """All-gather rank shards of a [count * per_item] tensor into the full [total * per_item] tensor.

    Equal shards (total divisible by the world size) are gathered straight into `out`
    (allocated if not given) by one all-gather; unequal ones are padded to the largest
    shard for the collective and trimmed.  Returns the full tensor on every rank.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    _check_local(local, total, per_item, rank, world)
    if out is None:
        out = torch.empty(total * per_item, dtype=local.dtype, device=local.device)
    elif out.numel() != total * per_item or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous tensor of {total * per_item} words")
    if total % world == 0:
        dist.all_gather_into_tensor(_bytes(out), _bytes(local.contiguous()), group=group)
        return out
    counts = [shard_range(total, r, world)[1] for r in range(world)]
    cmax = max(counts)
    padded = torch.zeros(cmax * per_item, dtype=local.dtype, device=local.device)
    padded[: local.numel()] = local.reshape(-1)
    parts = [torch.empty(cmax * per_item * local.element_size(), dtype=torch.uint8, device=local.device)
             for _ in range(world)]
    dist.all_gather(parts, _bytes(padded), group=group)
    flat = out.reshape(-1)
    for r, (p, c) in enumerate(zip(parts, counts)):
        lo = shard_range(total, r, world)[0]
        flat[lo * per_item:(lo + c) * per_item] = p.view(local.dtype)[: c * per_item]
    return out


def gather_to_root(local, total: int, per_item: int, root: int = 0, group=None, out=None):
    """Gather rank shards into the full output on `root` only.

    Every other rank sends its shard; the root posts one receive per rank straight
    into that rank's offset of `out` (allocated on the root if not given) and copies
    its own shard in place.  Returns the full tensor on the root and None elsewhere.
    Shards may be unequal.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    _check_local(local, total, per_item, rank, world)
    if not 0 <= root < world:
        raise ValueError(f"bad root {root} of {world}")
    ops = []
    if rank == root:
        if out is None:
            out = torch.empty(total * per_item, dtype=local.dtype, device=local.device)
        elif out.numel() != total * per_item or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous tensor of {total * per_item} words")
        flat = out.reshape(-1)
        lo, cnt = shard_range(total, rank, world)
        flat[lo * per_item:(lo + cnt) * per_item] = local.reshape(-1)
        for r in range(world):
            lo_r, cnt_r = shard_range(total, r, world)
            if r != root and cnt_r:
                peer = r if group is None else dist.get_global_rank(group, r)
                ops.append(dist.P2POp(dist.irecv, _bytes(flat[lo_r * per_item:(lo_r + cnt_r) * per_item]), peer, group))
    elif local.numel():
        peer = root if group is None else dist.get_global_rank(group, root)
        ops.append(dist.P2POp(dist.isend, _bytes(local.contiguous()), peer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return out if rank == root else None


class RootOutputs:
    """Full-size output buffers held by the root rank, written by every rank's kernels.

    The gather fused into the producing kernels: the root allocates each output in full
    and exports it (cm_ipc_export); every other rank maps it (cm_ipc_open) and passes
    `address(i, first_item)` -- the mapped buffer advanced to its shard -- as the output
    of its MatMul / VectorOP / Pooling calls.  The kernels' ordinary stores then put each
    output word straight into the root GPU's memory over NVLink while the kernel runs: no
    collective, no copy after the kernels.  `sizes` are the outputs' word counts (every
    item of every rank); `tensors` holds them on the root (None elsewhere).  The data are
    complete on the root once every rank has synchronized its kernels (then a barrier).
    Call close() on every rank before the process group goes away.
    """

    def __init__(self, sizes, root: int = 0, group=None):
        import ctypes as C
        import torch
        import torch.distributed as dist
        from ._lib import check, lib
        self.rank = dist.get_rank(group)
        self.root, self.group = root, group
        L = lib()
        self.tensors, handles = None, None
        if self.rank == root:
            self.tensors = [torch.empty(max(int(w), 1), dtype=torch.int16, device="cuda") for w in sizes]
            handles = []
            for t in self.tensors:
                h = (C.c_ubyte * 80)()
                check(L.cm_ipc_export(C.c_void_p(t.data_ptr()), h))
                handles.append(bytes(h))
        box = [handles]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, root) if group is not None else root,
                                   group=group)
        self._opened = []
        if self.rank == root:
            self.ptrs = [t.data_ptr() for t in self.tensors]
        else:
            self.ptrs = []
            for hb in box[0]:
                h = (C.c_ubyte * 80).from_buffer_copy(hb)
                p = C.c_void_p()
                check(L.cm_ipc_open(h, C.byref(p)))
                self._opened.append(p.value)
                self.ptrs.append(p.value)

    def address(self, i: int, word_offset: int) -> int:
        """Device address (valid in this process) of word `word_offset` of output i."""
        return int(self.ptrs[i]) + 2 * int(word_offset)

    def close(self) -> None:
        """Unmap on the importing ranks, then a barrier, so the root frees its buffers only
        after every mapping is gone."""
        import torch.distributed as dist
        from ._lib import check, lib
        for p in self._opened:
            check(lib().cm_ipc_close(p))
        self._opened, self.ptrs = [], []
        dist.barrier(group=self.group)
        self.tensors = None
