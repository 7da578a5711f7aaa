"""The fused gather on 2 GPUs (skipped with fewer): every rank's MatMul, VectorOP and
Pooling kernels write their batch shard straight into rank 0's full-size output buffers
(sharding.RootOutputs, CUDA IPC over NVLink), and rank 0's buffers must equal the oracle
word for word; the copy-engine push (cm_copy_async into the mapped buffer) and the NCCL
gathers (to rank 0, to every rank) are checked the same way.

Run as spawned child processes, one per GPU, NCCL on 127.0.0.1 with NVLS off and a short
process-group timeout; the parent waits with a limit and reports each rank's verdict."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{rank}"))
        import cormorant_b200 as cm
        import oracle
        from cormorant_b200 import sharding
        cm.init(str(rank))
        port_ = oracle.port() if rank == 0 else None
        rng = np.random.default_rng(11)                 # same data on every rank
        verdicts = []
        # MatMul: batch 5 over 2 ranks (3 + 2 items), tensor-core and CUDA-core sizes
        for (n, k, m, B) in ((300, 257, 140, 5), (7, 13, 9, 5)):
            a = rng.integers(-1024, 1024, B * n * k).astype(np.int16)
            b = rng.integers(-1024, 1024, B * k * m).astype(np.int16)
            lo, cnt = sharding.shard_range(B, rank, WORLD)
            ta = torch.from_numpy(a[lo * n * k:(lo + cnt) * n * k].copy()).cuda()
            tb = torch.from_numpy(b[lo * k * m:(lo + cnt) * k * m].copy()).cuda()
            local = torch.full((cnt * n * m,), -23131, dtype=torch.int16, device="cuda")
            ro = sharding.RootOutputs([B * n * m])
            if rank == 0:
                ro.tensors[0].fill_(-23131)
            dist.barrier()
            cm.MatmulKernel(ta, tb, ro.address(0, lo * n * m), n, k, m, cnt)
            cm.MatmulKernel(ta, tb, local, n, k, m, cnt)
            torch.cuda.synchronize()
            dist.barrier()
            full_root = sharding.gather_to_root(local, B, n * m)
            full_all = sharding.gather_batches(local, B, n * m)
            if rank == 0:
                want = port_.matmul(a, b, n, k, m, B)
                verdicts.append(("matmul fused", np.array_equal(ro.tensors[0].cpu().numpy(), want)))
                ro.tensors[0].fill_(-23131)
            dist.barrier()
            # the copy-engine push: every rank copies its local shard into the root's buffer
            import ctypes as C
            from cormorant_b200._lib import check, lib
            s = torch.cuda.Stream()
            check(lib().cm_copy_async(C.c_void_p(ro.address(0, lo * n * m)), C.c_void_p(local.data_ptr()),
                                      cnt * n * m * 2, C.c_void_p(s.cuda_stream)))
            s.synchronize()
            dist.barrier()
            if rank == 0:
                verdicts.append(("matmul copy push", np.array_equal(ro.tensors[0].cpu().numpy(), want)))
                verdicts.append(("matmul to_root", np.array_equal(full_root.cpu().numpy(), want)))
            verdicts.append(("matmul all_gather", port_ is None or np.array_equal(full_all.cpu().numpy(), want)))
            ro.close()
        # VectorOP over contiguous element slices; Pooling over images
        N = 1 << 20
        x = rng.integers(-32768, 32768, N).astype(np.int16)
        y = rng.integers(1, 32768, N).astype(np.int16)
        lo, cnt = sharding.shard_range(N, rank, WORLD)
        imgs = rng.integers(-2048, 2048, 4 * 8 * 30 * 30).astype(np.int16)
        ilo, icnt = sharding.shard_range(4, rank, WORLD)
        per_in, per_out = 8 * 30 * 30, 8 * 15 * 15
        ro = sharding.RootOutputs([N, 4 * per_out])
        tx = torch.from_numpy(x[lo:lo + cnt].copy()).cuda()
        ty = torch.from_numpy(y[lo:lo + cnt].copy()).cuda()
        cm.VectorOPKernel(tx, ty, ro.address(0, lo), cnt, 3)            # DIV
        timg = torch.from_numpy(imgs[ilo * per_in:(ilo + icnt) * per_in].copy()).cuda()
        geo = (icnt, 8, 30, 30, 15, 15, 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 0)   # AVG 3x3 s2 p1
        cm.PoolingKernel(timg, ro.address(1, ilo * per_out), *geo)
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            verdicts.append(("vectorop fused", np.array_equal(ro.tensors[0].cpu().numpy(), port_.vectorop(x, y, N, 3))))
            wantp = port_.pool(imgs, 4, 8, 30, 30, 15, 15, 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 0)
            verdicts.append(("pool fused", np.array_equal(ro.tensors[1].cpu().numpy(), wantp)))
        ro.close()
        q.put((rank, verdicts, None))
    except Exception as e:                              # report instead of leaving the parent waiting
        q.put((rank, [], repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_fused_gather_two_gpus():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in procs:
            res.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, verdicts, err in res:
        assert err is None, f"rank {rank}: {err}"
        bad = [name for name, ok in verdicts if not ok]
        assert not bad, f"rank {rank}: {bad}"
    assert any(v for _, v, _ in res)
