"""Host-side multi-GPU logic on CPU: shard ranges and the output gather, as
world_size-2 (and 3) gloo process groups on 127.0.0.1."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cormorant_b200.sharding import gather_batches, gather_to_root, shard_range


@pytest.mark.parametrize("total", [0, 1, 7, 8, 64, 256, 1 << 28])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_ranges_partition(total, world):
    start = 0
    for r in range(world):
        lo, cnt = shard_range(total, r, world)
        assert lo == start and cnt >= 0
        start += cnt
    assert start == total
    counts = [shard_range(total, r, world)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _worker(rank, world, port, total, per_item, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["GLOO_SOCKET_IFNAME"] = "lo"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        lo, cnt = shard_range(total, rank, world)
        # each "batch item" b holds words b*1000 + j (what a per-item kernel would write)
        local = torch.tensor([b * 1000 + j for b in range(lo, lo + cnt) for j in range(per_item)], dtype=torch.int16)
        want = torch.tensor([b * 1000 + j for b in range(total) for j in range(per_item)], dtype=torch.int16)
        ok = True
        full = gather_batches(local, total, per_item)
        ok &= bool(torch.equal(full, want))
        # into a caller's buffer (poisoned first: every word must be written)
        out = torch.full((total * per_item,), -23131, dtype=torch.int16)
        ok &= gather_batches(local, total, per_item, out=out) is out and bool(torch.equal(out, want))
        # to one rank only: the root gets everything, the others None
        for root in range(world):
            out = torch.full((total * per_item,), -23131, dtype=torch.int16) if rank == root else None
            got = gather_to_root(local, total, per_item, root=root, out=out)
            if rank == root:
                ok &= got is out and bool(torch.equal(got, want))
            else:
                ok &= got is None
        q.put((rank, ok))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 8), (2, 7), (3, 8), (4, 8)])
def test_gathers_gloo(world, total):
    """All-gather (equal and unequal shards) and the gather to a root rank, on gloo ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 500) + world * 7 + total
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, 5, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] for r in res), res


def test_gather_checks_shard_size():
    """A shard of the wrong length is refused before any communication."""
    from cormorant_b200.sharding import _check_local
    with pytest.raises(ValueError):
        _check_local(torch.zeros(6, dtype=torch.int16), 8, 2, 0, 2)
