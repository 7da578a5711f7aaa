#!/usr/bin/env python
"""Benchmark of the Cormorant Q8.8 kernels on B200 -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config matmul|vectorop|pool|resnet|lenet]

Default workload (the metric's configuration): the
batched MatMul sweep, raw int16 uniform [-1024, 1024):
    B=64 x {256^3, 1024^3, 4096^3}  +  B=8 x (8192x4096)(4096x11008).
One step = one pass over the sweep.  metric = Q8.8 GOPS = 2*n*k*m*batch / time
(the reference bench's definition, inference-scheduler/bench_src/bench_matmul.c).
--config vectorop: the 2^28-element sweep of the six ops, GB/s = ports*size*2B / time.
--config pool: the seven pooling variants on [256,64,112,112], GB/s = (x+y bytes) / time.
--config resnet / lenet: the ResNet-18-shaped network at batch 256 and LeNet-5 at batch 1,
images/s; the call list (folded epilogues, plane images, conv weights prepared once) is
captured as one CUDA graph and replayed per step (--no-graph, --no-prepared, --no-planes,
--unfused select the slower forms).

Multi-GPU (torchrun, one rank per GPU): every workload is sharded by batch
(VectorOP by contiguous element range); no collective runs in the timed
region; the total work is fixed, so scaling is "strong".  Time = max over ranks.
The line adds "gather": one NCCL all-gather of a step's outputs to every rank, timed
after the timed region.

--impl reference times the reference's own CPU implementation (the unmodified
reference kernels compiled against oracle/'s shim, oracle/_ref; else the C
restatement) on this host's cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

MATMUL_SWEEP = [(256, 256, 256, 64), (1024, 1024, 1024, 64), (4096, 4096, 4096, 64), (8192, 4096, 11008, 8)]
VOP_N = 1 << 28
VOP_OPS = [0, 1, 2, 3, 4, 5]
POOL_SHAPE = (256, 64, 112, 112)
# name, ph, pw, sh, sw, pt, pl, dh, dw, type, lp, cip, out_h, out_w
POOL_SWEEP = [
    ("max3x3s2p1d1", 3, 3, 2, 2, 1, 1, 1, 1, 0, 2, 0, 56, 56),
    ("max3x3s2p1d2", 3, 3, 2, 2, 1, 1, 2, 2, 0, 2, 0, 55, 55),
    ("avg3x3s2p1cip0", 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 0, 56, 56),
    ("avg3x3s2p1cip1", 3, 3, 2, 2, 1, 1, 1, 1, 1, 2, 1, 56, 56),
    ("lp2_2x2s2", 2, 2, 2, 2, 0, 0, 1, 1, 2, 2, 0, 56, 56),
    ("globalmax", 112, 112, 1, 1, 0, 0, 1, 1, 0, 2, 0, 1, 1),
    ("globalavg", 112, 112, 1, 1, 0, 0, 1, 1, 1, 2, 0, 1, 1),
]


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch recorded from an ncu capture (profiles/*.md, 'traffic_bytes_per_launch[<name>] = N')."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"traffic_bytes_per_launch\[{re.escape(name)}\]\s*=\s*([0-9.eE+]+)", f.read_text())
        if m:
            return float(m.group(1))
    return None


def fill(view, rng, lo: int, hi: int) -> None:
    """Fill a host array with a repeated 1 Mi-word random block (timing data only)."""
    import numpy as np
    base = rng.integers(lo, hi, size=1 << 20, dtype=np.int16)
    n = view.size
    for off in range(0, n, base.size):
        view[off:off + base.size] = base[:min(base.size, n - off)]


def gpu_indices(world: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in vis.split(",") if v.strip()]
    if ids and all(v.isdigit() for v in ids):
        return [int(v) for v in ids[:world]]
    return list(range(world))


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    lo = total * rank // world
    hi = total * (rank + 1) // world
    return lo, hi - lo


# --------------------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ",".join(map(str, gpu_indices))],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        loaded = [s for s, p in zip(sm, power) if p > 250.0] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# --------------------------------------------------------------------------------------
# workloads (GPU side)
# --------------------------------------------------------------------------------------
class MatmulSweep:
    name = "matmul"
    metric = "Q8.8 GOPS (batched MatMul sweep)"
    unit = "GOPS"
    dominant = "gemm_q88"

    sweep = MATMUL_SWEEP

    def __init__(self, rank, world):
        self.rank, self.world = rank, world
        self.shapes = []   # (n, k, m, batch_local)
        for (n, k, m, b) in self.sweep:
            _, cnt = shard(b, rank, world)
            self.shapes.append((n, k, m, cnt))
        self.units_total = sum(2.0 * n * k * m * b for (n, k, m, b) in self.sweep)   # Q8.8 ops, all ranks
        self.units_local = sum(2.0 * n * k * m * b for (n, k, m, b) in self.shapes)
        # algorithmic int8 tensor ops: 4 s8 MMAs per Q8.8 multiply-add
        self.dom_units_local = 4.0 * self.units_local

    def config(self, world):
        if self.sweep is not MATMUL_SWEEP:
            return {"workload": "matmul single shape " + ",".join(map(str, self.sweep[0])) + " (n,k,m,batch)",
                    "inputs": "raw int16 uniform [-1024,1024)", "parallelism": f"batch-sharded over {world} GPU(s)"}
        return {"workload": "matmul_sweep (BASELINE configs[1])",
                "shapes": "B=64 x {256,1024,4096}^3 + B=8 x 8192x4096x11008 (n x k x m)",
                "inputs": "raw int16 uniform [-1024,1024), seeded per rank",
                "parallelism": f"batch-sharded over {world} GPU(s), no collective in the timed region",
                "l2": "inputs larger than L2 (9.6 GB per step; each shape evicts the previous)"}

    def setup(self):
        import torch
        self.bufs = []
        g = torch.Generator(device="cuda").manual_seed(1234 + self.rank)
        for (n, k, m, b) in self.shapes:
            if b == 0:
                self.bufs.append(None)
                continue
            a = torch.randint(-1024, 1024, (b * n * k,), dtype=torch.int16, device="cuda", generator=g)
            bb = torch.randint(-1024, 1024, (b * k * m,), dtype=torch.int16, device="cuda", generator=g)
            c = torch.empty(b * n * m, dtype=torch.int16, device="cuda")
            self.bufs.append((a, bb, c))

    def step(self, cm, stream):
        for (n, k, m, b), t in zip(self.shapes, self.bufs):
            if t is None:
                continue
            cm.MatmulKernel(t[0], t[1], t[2], n, k, m, b, stream=stream)

    def gather_outputs(self):
        """(local output shard, items over all ranks, words per item) of each output of a step."""
        import torch
        out = []
        for (n, k, m, b), (_, _, _, B), t in zip(self.shapes, self.sweep, self.bufs):
            c = t[2] if t is not None else torch.empty(0, dtype=torch.int16, device="cuda")
            out.append((c, B, n * m))
        return out

    def per_part(self, cm, stream, iters):
        """Per-shape device times of the GEMM and split kernels (a separate profiled pass)."""
        out = []
        L = cm.lib()
        import ctypes as C
        import torch
        for (n, k, m, b), t in zip(self.shapes, self.bufs):
            if t is None:
                continue
            L.cm_profile_begin()
            for _ in range(iters):
                cm.MatmulKernel(t[0], t[1], t[2], n, k, m, b, stream=stream)
            torch.cuda.synchronize()
            L.cm_profile_end()
            res = {}
            for kind in ("gemm_q88", "split"):
                ms, cnt = C.c_double(), C.c_uint64()
                L.cm_profile_read(kind.encode(), C.byref(ms), C.byref(cnt))
                res[kind] = ms.value / iters
            ops = 2.0 * n * k * m * b
            out.append({"shape": f"{b}x{n}x{k}x{m}", "gemm_ms": round(res["gemm_q88"], 4),
                        "split_ms": round(res["split"], 4),
                        "gemm_int8_tops": round(4 * ops / (res["gemm_q88"] * 1e-3) / 1e12, 1),
                        "q88_gops_with_split": round(ops / ((res["gemm_q88"] + res["split"]) * 1e-3) / 1e9, 1)})
        return out

    def release(self):
        self.bufs = []

    # ---- end to end through the reference-facing API (cm_buf_* + run_matmul) ----
    def e2e_setup(self):
        from cormorant_b200.runtime import InferenceBuf
        import numpy as np
        self.e2e = []
        rng = np.random.default_rng(99 + self.rank)
        self.h2d = self.d2h = 0
        for (n, k, m, b) in self.shapes:
            if b == 0:
                continue
            A = InferenceBuf.alloc(b * n * k)
            B = InferenceBuf.alloc(b * k * m)
            Cb = InferenceBuf.alloc(b * n * m)
            fill(A.ptr(), rng, -1024, 1024)
            fill(B.ptr(), rng, -1024, 1024)
            self.e2e.append((n, k, m, b, A, B, Cb))
            self.h2d += 2 * (b * n * k + b * k * m)
            self.d2h += 2 * b * n * m

    def e2e_step(self):
        from cormorant_b200.runtime import run_matmul
        for (n, k, m, b, A, B, Cb) in self.e2e:
            A.sync_to_device()
            B.sync_to_device()
            run_matmul(A, B, Cb, n, k, m, b, n * k, k * m, n * m)
            Cb.sync_from_device()

    def e2e_release(self):
        for t in self.e2e:
            for buf in t[4:]:
                buf.free()
        self.e2e = []


class VectorOPSweep:
    name = "vectorop"
    metric = "VectorOP GB/s (six ops on 2^28 elements)"
    unit = "GB/s"
    dominant = "vectorop"

    def __init__(self, rank, world):
        self.rank, self.world = rank, world
        self.lo, self.n = shard(VOP_N, rank, world)
        ports = lambda op: 3 if op < 4 else 2   # noqa: E731  (bench_vectorop.c byte formula)
        self.units_total = sum(ports(op) * VOP_N * 2.0 for op in VOP_OPS) / 1e9          # GB per step
        self.units_local = sum(ports(op) * self.n * 2.0 for op in VOP_OPS) / 1e9
        self.dom_units_local = self.units_local * 1e9                                  # bytes

    def config(self, world):
        return {"workload": "vectorop_sweep (BASELINE configs[2])", "ops": "ADD,SUB,MUL,DIV,RELU,RELU6",
                "elements": VOP_N, "inputs": "raw int16 uniform full range; DIV zeros -> 1",
                "parallelism": f"contiguous element slices over {world} GPU(s)",
                "l2": "inputs larger than L2 (1.5 GB per op)"}

    def setup(self):
        import torch
        g = torch.Generator(device="cuda").manual_seed(77 + self.rank)
        self.a = torch.randint(-32768, 32768, (self.n,), dtype=torch.int32, device="cuda", generator=g).to(torch.int16)
        self.b = torch.randint(-32768, 32768, (self.n,), dtype=torch.int32, device="cuda", generator=g).to(torch.int16)
        self.b[self.b == 0] = 1
        self.c = torch.empty_like(self.a)

    def step(self, cm, stream):
        for op in VOP_OPS:
            cm.VectorOPKernel(self.a, self.b, self.c, self.n, op, stream=stream)

    def gather_outputs(self):
        return [(self.c, VOP_N, 1) for _ in VOP_OPS]

    def per_part(self, cm, stream, iters):
        import ctypes as C
        import torch
        L = cm.lib()
        out = []
        for op in VOP_OPS:
            L.cm_profile_begin()
            for _ in range(iters):
                cm.VectorOPKernel(self.a, self.b, self.c, self.n, op, stream=stream)
            torch.cuda.synchronize()
            L.cm_profile_end()
            ms, cnt = C.c_double(), C.c_uint64()
            L.cm_profile_read(b"vectorop", C.byref(ms), C.byref(cnt))
            t = ms.value / iters
            byts = (3 if op < 4 else 2) * self.n * 2.0
            out.append({"op": op, "ms": round(t, 4), "gbs": round(byts / (t * 1e-3) / 1e9, 1)})
        return out

    def release(self):
        self.a = self.b = self.c = None

    def e2e_setup(self):
        from cormorant_b200.runtime import InferenceBuf
        import numpy as np
        rng = np.random.default_rng(5 + self.rank)
        self.A, self.B, self.C = (InferenceBuf.alloc(self.n) for _ in range(3))
        fill(self.A.ptr(), rng, -32768, 32768)
        fill(self.B.ptr(), rng, 1, 32768)
        self.h2d = sum((2 if op < 4 else 1) * self.n * 2 for op in VOP_OPS)
        self.d2h = len(VOP_OPS) * self.n * 2

    def e2e_step(self):
        from cormorant_b200.runtime import run_op
        for op in VOP_OPS:
            self.A.sync_to_device()
            if op < 4:
                self.B.sync_to_device()
            run_op(self.A, self.B if op < 4 else None, self.C, self.n, op, 1, 0, 0)
            self.C.sync_from_device()

    def e2e_release(self):
        for b in (self.A, self.B, self.C):
            b.free()


class PoolSweep:
    name = "pool"
    metric = "Pooling GB/s (seven variants on [256,64,112,112])"
    unit = "GB/s"
    dominant = "pool"

    def __init__(self, rank, world):
        N, C, H, W = POOL_SHAPE
        self.rank, self.world = rank, world
        _, self.nb = shard(N, rank, world)
        xb = lambda nb: nb * C * H * W * 2.0   # noqa: E731
        yb = lambda nb, c: nb * C * c[12] * c[13] * 2.0   # noqa: E731
        self.units_total = sum(xb(N) + yb(N, c) for c in POOL_SWEEP) / 1e9
        self.units_local = sum(xb(self.nb) + yb(self.nb, c) for c in POOL_SWEEP) / 1e9
        self.dom_units_local = self.units_local * 1e9

    def config(self, world):
        return {"workload": "pool_sweep (BASELINE configs[4])", "input": "[256,64,112,112] raw uniform [-2048,2048)",
                "variants": [c[0] for c in POOL_SWEEP], "parallelism": f"batch-sharded over {world} GPU(s)",
                "l2": "inputs larger than L2 (411 MB)"}

    def setup(self):
        import torch
        N, C, H, W = POOL_SHAPE
        g = torch.Generator(device="cuda").manual_seed(55 + self.rank)
        self.x = torch.randint(-2048, 2048, (self.nb * C * H * W,), dtype=torch.int16, device="cuda", generator=g)
        self.y = torch.empty(self.nb * C * 56 * 56, dtype=torch.int16, device="cuda")

    def _one(self, cm, c, stream):
        N, C, H, W = POOL_SHAPE
        _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip, oh, ow = c
        cm.PoolingKernel(self.x, self.y, self.nb, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip,
                         stream=stream)

    def step(self, cm, stream):
        for c in POOL_SWEEP:
            self._one(cm, c, stream)

    def gather_outputs(self):
        N, C, H, W = POOL_SHAPE
        return [(self.y[: self.nb * C * c[-2] * c[-1]], N, C * c[-2] * c[-1]) for c in POOL_SWEEP]

    def per_part(self, cm, stream, iters):
        import ctypes as C_
        import torch
        N, C, H, W = POOL_SHAPE
        L = cm.lib()
        out = []
        for c in POOL_SWEEP:
            L.cm_profile_begin()
            for _ in range(iters):
                self._one(cm, c, stream)
            torch.cuda.synchronize()
            L.cm_profile_end()
            ms, cnt = C_.c_double(), C_.c_uint64()
            L.cm_profile_read(b"pool", C_.byref(ms), C_.byref(cnt))
            t = ms.value / iters
            byts = self.nb * C * (H * W + c[12] * c[13]) * 2.0
            out.append({"variant": c[0], "ms": round(t, 4), "gbs": round(byts / (t * 1e-3) / 1e9, 1)})
        return out

    def release(self):
        self.x = self.y = None

    def e2e_setup(self):
        from cormorant_b200.runtime import InferenceBuf
        import numpy as np
        N, C, H, W = POOL_SHAPE
        rng = np.random.default_rng(8 + self.rank)
        self.X = InferenceBuf.alloc(self.nb * C * H * W)
        self.Y = InferenceBuf.alloc(self.nb * C * 56 * 56)
        fill(self.X.ptr(), rng, -2048, 2048)
        self.h2d = len(POOL_SWEEP) * self.nb * C * H * W * 2
        self.d2h = sum(self.nb * C * c[12] * c[13] * 2 for c in POOL_SWEEP)

    def e2e_step(self):
        from cormorant_b200.runtime import InferenceBuf, run_pool
        N, C, H, W = POOL_SHAPE
        for c in POOL_SWEEP:
            _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip, oh, ow = c
            self.X.sync_to_device()
            run_pool(self.X, self.Y, self.nb, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip)
            InferenceBuf.init_view(self.Y, 0, self.nb * C * oh * ow).sync_from_device()

    def e2e_release(self):
        self.X.free()
        self.Y.free()


class NetworkBench:
    """LeNet-5 (config 0, batch 1, CUDA-graph replay) or ResNet-18-shaped (config 3, batch 256)."""
    unit = "images/s"
    dominant = "gemm_q88"

    def __init__(self, rank, world, which):
        from cormorant_b200 import networks
        self.which, self.rank, self.world = which, rank, world
        if which == "lenet":
            self.batch_total, self.local = 1 * world, 1          # replicas: one batch-1 stream per GPU
            self.net = networks.lenet5(batch=1)
            self.metric = "LeNet-5 images/s (batch 1 per GPU, CUDA-graph replay)"
        else:
            _, self.local = shard(256, rank, world)
            self.batch_total = 256
            self.net = networks.resnet18(batch=max(self.local, 1))
            self.metric = "ResNet-18-shaped images/s (batch 256)"
        self.fused = not UNFUSED
        if self.fused:                                           # Conv->Relu (/ Conv->Add->Relu) folded
            self.net = networks.fuse(self.net, residual=FUSE_RESIDUAL)
        self.planes = self.fused and PLANES and which != "lenet"
        if self.planes:                                          # conv outputs produced as the next convs' operand
            self.net = networks.chain(self.net)
        self.units_total = float(self.batch_total)
        self.units_local = float(self.local)
        self.dom_units_local = 8.0 * self.net.macs_per_image * self.local   # int8 ops (4 MMAs x 2 per MAC)

    def config(self, world):
        calls = ("reference call list, Conv->Relu" + (" and Conv->Add->Relu" if FUSE_RESIDUAL else "")
                 + " and Gemm(MatMul->Add)->Relu chains folded into cm_conv_fused / cm_matmul_fused"
                 + ("; conv outputs read by convs written as plane images (cm_conv_planes)" if self.planes else "")
                 if self.fused else "reference call list, one C-ABI call per node")
        if self.which == "lenet":
            return {"workload": "lenet5 (BASELINE configs[0])", "batch": 1, "input": "1x1x28x28 uniform [0,1)",
                    "parallelism": f"replicas only: one batch-1 stream per GPU ({world})", "calls": calls,
                    "launches": ("whole call list run as one kernel launch (cm_calls), captured as a CUDA graph"
                                 if ONE_LAUNCH else "whole call list captured once as a CUDA graph and replayed")}
        return {"workload": "resnet18-shaped (BASELINE configs[3])", "batch": 256,
                "input": "256x3x224x224 uniform [0,1)", "macs_per_image": self.net.macs_per_image, "calls": calls,
                "parallelism": f"batch-sharded over {world} GPU(s)", "l2": "inputs larger than L2 (77 MB input, 1.1 GB activations)",
                "launches": ("whole call list captured once as a CUDA graph and replayed" if GRAPH
                             else "one launch per kernel from the host")}

    def setup(self):
        import torch
        from cormorant_b200 import networks
        self.x = networks.make_input(self.net)
        self.bufs = networks.gpu_buffers(self.net, self.x)
        # the network's conv weights prepared once (constants of the call list)
        self.wcache = networks.prepare_weights(self.net, self.bufs) if PREPARED and self.local > 0 else {}
        self.graph = None
        if GRAPH and self.local > 0:
            self.graph, self.launches_per_step = self._capture(self.bufs)

    def _backend(self, stream):
        from cormorant_b200 import networks
        return networks.GpuBackend(stream, one_launch=ONE_LAUNCH, weights=self.wcache)

    def _capture(self, bufs):
        """The whole call list captured once as a CUDA graph (its scratch allocations become
        graph memory nodes); returns (graph, kernel launches per replay)."""
        import torch
        import cormorant_b200 as cm
        from cormorant_b200 import networks
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):            # warm: module loading and attribute setup happen outside capture
                networks.execute(self.net, self._backend(s), bufs)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        l0 = cm.launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            networks.execute(self.net, self._backend(torch.cuda.current_stream()), bufs)
        n = cm.launch_count() - l0
        torch.cuda.synchronize()
        return g, n

    def gather_outputs(self):
        """ResNet: the logits of every image; LeNet runs replicas (nothing to gather)."""
        if self.which == "lenet":
            return []
        out = self.bufs[self.net.resolve(self.net.output)]
        return [(out[: self.local * 1000], self.batch_total, 1000)]

    def profile_dominant(self, cm, stream, iters):
        """Device time (ms) and launch count of the GEMM kernel over `iters` eager passes, from
        CUDA events around each launch (a graph replay carries no per-launch events)."""
        import ctypes as C
        import torch
        from cormorant_b200 import networks
        L = cm.lib()
        torch.cuda.synchronize()
        L.cm_profile_begin()
        for _ in range(iters):
            networks.execute(self.net, self._backend(stream), self.bufs)
        torch.cuda.synchronize()
        L.cm_profile_end()
        ms, cnt = C.c_double(), C.c_uint64()
        L.cm_profile_read(self.dominant.encode(), C.byref(ms), C.byref(cnt))
        return ms.value, cnt.value

    def step(self, cm, stream):
        from cormorant_b200 import networks
        if self.graph is not None:
            self.graph.replay()
        elif self.local > 0:
            networks.execute(self.net, self._backend(stream), self.bufs)

    def per_part(self, cm, stream, iters):
        import ctypes as C
        import torch
        from cormorant_b200 import networks
        L = cm.lib()
        L.cm_profile_begin()
        for _ in range(iters):
            networks.execute(self.net, self._backend(stream), self.bufs)
        torch.cuda.synchronize()
        L.cm_profile_end()
        out = {}
        for kind in ("gemm_q88", "split", "pool", "vectorop", "conv_aux"):
            ms, cnt = C.c_double(), C.c_uint64()
            L.cm_profile_read(kind.encode(), C.byref(ms), C.byref(cnt))
            out[kind + "_ms"] = round(ms.value / iters, 4)
        return [out]

    def release(self):
        self.bufs = None
        self.graph = None
        self.wcache = {}

    def e2e_setup(self):
        import torch
        from cormorant_b200 import networks
        self.bufs = networks.gpu_buffers(self.net)
        self.wcache = networks.prepare_weights(self.net, self.bufs) if PREPARED else {}
        self.hx = torch.from_numpy(self.x.copy()).pin_memory()
        out_words = self.net.buffers[self.net.resolve(self.net.output)]
        self.hy = torch.empty(out_words, dtype=torch.int16).pin_memory()
        self.h2d = self.hx.numel() * 2
        self.d2h = out_words * 2
        self.e2e_graph = None
        self.e2e_path = ("pinned host input -> device copy -> the call list through the C ABI (ConvKernel, VectorOPKernel, "
                         "PoolingKernel, MatmulKernel) -> logits copied to pinned host")
        self.copy_stream = None
        if self.which != "lenet":
            # two device input buffers: step i+1's input crosses PCIe on a copy stream while
            # step i computes; a copy waits until the forward that last read its buffer is done
            self.copy_stream = torch.cuda.Stream()
            self.xbufs = [self.bufs[self.net.input], torch.empty_like(self.bufs[self.net.input])]
            self.copied = [torch.cuda.Event(), torch.cuda.Event()]
            self.consumed = [None, None]
            self.e2e_i = 0
            self.e2e_path += "; the next step's input copy overlaps this step's compute (copy stream, two input buffers)"
            self.e2e_graphs = None
            if GRAPH:
                # one graph of the call list per input buffer; the copies stay outside the graphs
                self.e2e_graphs = []
                for b in range(2):
                    self.bufs[self.net.input] = self.xbufs[b]
                    self.e2e_graphs.append(self._capture(self.bufs)[0])
                self.e2e_path += "; the call list replayed as a CUDA graph (one per input buffer)"
        if self.which == "lenet":
            self.e2e_path += "; captured once as a CUDA graph and replayed per image"
            # batch 1 is host-launch-bound: the whole step (pinned H2D copy, the call
            # list, D2H copy of the logits) is captured once and replayed per image
            for _ in range(3):
                self._e2e_body()
            torch.cuda.synchronize()
            self.e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.e2e_graph):
                self._e2e_body()
            torch.cuda.synchronize()

    def _e2e_body(self):
        import torch
        from cormorant_b200 import networks
        self.bufs[self.net.input].copy_(self.hx, non_blocking=True)
        networks.execute(self.net, self._backend(torch.cuda.current_stream()), self.bufs)
        self.hy.copy_(self.bufs[self.net.resolve(self.net.output)], non_blocking=True)

    def e2e_step(self):
        if self.e2e_graph is not None:
            self.e2e_graph.replay()
        elif self.copy_stream is not None:
            self._e2e_pipelined()
        else:
            self._e2e_body()

    def e2e_start(self, start_event):
        """Timed region starts: the first input copy is issued inside it."""
        if self.copy_stream is not None:
            self.copy_stream.wait_event(start_event)
            self._issue_copy(self.e2e_i)

    def _issue_copy(self, i):
        import torch
        b = i % 2
        with torch.cuda.stream(self.copy_stream):
            if self.consumed[b] is not None:
                self.copy_stream.wait_event(self.consumed[b])
            self.xbufs[b].copy_(self.hx, non_blocking=True)
            self.copied[b].record(self.copy_stream)

    def _e2e_pipelined(self):
        import torch
        from cormorant_b200 import networks
        i = self.e2e_i
        b = i % 2
        self._issue_copy(i + 1)                              # the next step's input, overlapped
        cur = torch.cuda.current_stream()
        cur.wait_event(self.copied[b])
        self.bufs[self.net.input] = self.xbufs[b]
        if self.e2e_graphs is not None:
            self.e2e_graphs[b].replay()
        else:
            networks.execute(self.net, self._backend(cur), self.bufs)
        ev = torch.cuda.Event()
        ev.record(cur)
        self.consumed[b] = ev
        self.hy.copy_(self.bufs[self.net.resolve(self.net.output)], non_blocking=True)
        self.e2e_i = i + 1

    def e2e_release(self):
        self.e2e_graph = None
        self.e2e_graphs = None
        self.bufs = None
        self.wcache = {}


UNFUSED = False      # --unfused: networks run node by node
FUSE_RESIDUAL = True   # --no-fuse-residual: fold Conv->Relu only
PLANES = True          # --no-planes: every conv splits its own input
ONE_LAUNCH = False     # --one-launch: lenet's whole call list as one cm_calls launch (slower on B200)
GRAPH = True           # --no-graph: the network configs launch every kernel from the host each step
PREPARED = True        # --no-prepared: every conv call prepares its weight planes again

WORKLOADS = {"matmul": MatmulSweep, "vectorop": VectorOPSweep, "pool": PoolSweep,
             "lenet": lambda r, w: NetworkBench(r, w, "lenet"), "resnet": lambda r, w: NetworkBench(r, w, "resnet")}


# --------------------------------------------------------------------------------------
# CPU side: the reference implementation (or the restatement) on a bounded sample
# --------------------------------------------------------------------------------------
def _cpu_worker(args):
    """Runs in a spawned process: one slice of the sample; returns (units, seconds, kind)."""
    config, wid, nworkers = args
    sys.path.insert(0, str(ROOT))
    import numpy as np
    import oracle
    kind = "reference" if oracle.have_ref() else "port"
    chk = oracle.ref() if kind == "reference" else oracle.port()
    if kind == "port":
        chk.set_threads(1)
    rng = np.random.default_rng(1000 + wid)
    units = 0.0
    if config == "matmul":
        rows = 4
        jobs = []
        for (n, k, m, b) in MATMUL_SWEEP:
            a = rng.integers(-1024, 1024, size=rows * k, dtype=np.int16)
            bm = rng.integers(-1024, 1024, size=k * m, dtype=np.int16)
            jobs.append((a, bm, rows, k, m))
        t0 = time.perf_counter()
        for (a, bm, r, k, m) in jobs:
            chk.matmul(a, bm, r, k, m, 1)
            units += 2.0 * r * k * m
        dt = time.perf_counter() - t0
    elif config == "vectorop":
        n = 1 << 20
        a = rng.integers(-32768, 32768, size=n, dtype=np.int16)
        b = rng.integers(-32768, 32768, size=n, dtype=np.int16)
        b[b == 0] = 1
        t0 = time.perf_counter()
        for op in VOP_OPS:
            chk.vectorop(a, b, n, op)
            units += (3 if op < 4 else 2) * n * 2.0 / 1e9
        dt = time.perf_counter() - t0
    elif config in ("lenet", "resnet"):
        from cormorant_b200 import networks     # the call list only (pure Python, no GPU)
        net = networks.lenet5(batch=1) if config == "lenet" else networks.resnet18(batch=1)
        x = networks.make_input(net)
        bufs = {name: np.zeros(max(w, 1), np.int16) for name, w in net.buffers.items()}
        bufs.update({name: np.asarray(a, np.int16) for name, a in net.consts.items()})
        bufs[net.input][:] = x
        R = lambda name: None if name is None else bufs[net.resolve(name)]  # noqa: E731
        dt = 0.0
        for node in net.nodes:
            nk = node[0]
            t0 = time.perf_counter()
            scale = 1.0
            if nk == "conv":
                _, xn, wn, bn, yn, a = node
                a = list(a)
                m = a[4]
                if config == "resnet" and m > 8:
                    # the reference's output-channel tile (TILE_M = 8); time scaled by m / 8
                    per = a[1] * a[7] * a[8]
                    w8, b8 = R(wn)[: 8 * per], (R(bn)[:8] if bn else None)
                    a[4] = 8
                    chk.conv(R(xn), w8, b8, *a)
                    scale = m / 8.0
                else:
                    R(yn)[:] = chk.conv(R(xn), R(wn), R(bn), *a)[: R(yn).size]
            elif nk == "vectorop":
                _, an, bn, cn, a = node
                R(cn)[:] = chk.vectorop(R(an), R(bn), *a, c=R(cn).copy())[: R(cn).size]
            elif nk == "pool":
                _, xn, yn, a = node
                R(yn)[:] = chk.pool(R(xn), *a)[: R(yn).size]
            else:
                _, an, bn, cn, a = node
                R(cn)[:] = chk.matmul(R(an), R(bn), *a)[: R(cn).size]
            dt += (time.perf_counter() - t0) * scale
        units = 1.0
    else:
        N, C, H, W = POOL_SHAPE
        nb, cs = 1, 8
        x = rng.integers(-2048, 2048, size=nb * cs * H * W, dtype=np.int16)
        t0 = time.perf_counter()
        for c in POOL_SWEEP:
            _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip, oh, ow = c
            chk.pool(x, nb, cs, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip)
            units += nb * cs * (H * W + oh * ow) * 2.0 / 1e9
        dt = time.perf_counter() - t0
    return units, dt, kind


SAMPLE_TEXT = {
    "matmul": "4 output rows of one batch item per sweep shape per worker process (reference MatmulKernel with n=4)",
    "vectorop": "2^20 elements per op per worker process",
    "pool": "one image x 8 channels of [.,64,112,112] per variant per worker process",
    "lenet": "one whole LeNet-5 inference (batch 1) per worker process",
    "resnet": ("one ResNet-18 image per worker process; each conv layer computes 8 of its output channels "
               "(the reference's TILE_M) and its time is scaled by out_ch / 8; pools and vector ops run in full"),
}


def cpu_sample(config: str, workers: int, pool=None):
    """One bounded sample on `workers` processes; returns (value, unit-consistent, kind)."""
    import multiprocessing as mp
    own = pool is None
    if own:
        pool = mp.get_context("spawn").Pool(workers)
    t0 = time.perf_counter()
    res = pool.map(_cpu_worker, [(config, w, workers) for w in range(workers)])
    wall = time.perf_counter() - t0
    if own:
        pool.close()
        pool.join()
    units = sum(r[0] for r in res)
    kind = res[0][2]
    if config == "resnet":
        # scaled per-image estimates: the workers run in parallel, each at 1/dt images per second
        rate = sum(r[0] / r[1] for r in res)
        return rate, 1.0, kind
    return units, wall, kind


def cpu_units_to_value(config, units, seconds):
    if config == "matmul":
        return units / seconds / 1e9       # GOPS
    return units / seconds                 # GB/s (units already in GB) or images/s


def int8_peak() -> int:
    """Library int8 reference point: torch._int_mm (cuBLASLt, s8 x s8 -> s32) at 8192^3."""
    import torch
    n = 8192
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
    for _ in range(5):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best, tot, it = 1e9, 0.0, 0
    t_end = time.time() + 4.0
    while time.time() < t_end:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        best, tot, it = min(best, ms), tot + ms, it + 1
    ops = 2.0 * n ** 3
    print(json.dumps({"int8_mm_tops_burst": ops / (best * 1e-3) / 1e12, "int8_mm_tops_sustained": ops / (tot / it * 1e-3) / 1e12,
                      "iters": it, "how": "torch._int_mm 8192^3 s8xs8->s32, best and mean over 4 s"}))
    return 0


# --------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="matmul")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-workers", type=int, default=0)
    ap.add_argument("--per-part", action="store_true", help="add a per-shape/per-variant device-time breakdown")
    ap.add_argument("--no-fuse-residual", action="store_true",
                    help="lenet/resnet: fold Conv->Relu only (keep the residual Add / Relu passes)")
    ap.add_argument("--unfused", action="store_true",
                    help="lenet/resnet: run the reference call list node by node (no Conv->Relu/Add folding)")
    ap.add_argument("--one-launch", action="store_true",
                    help="lenet: the whole call list in one single-CTA launch (cm_calls) instead of one launch per call")
    ap.add_argument("--no-prepared", action="store_true",
                    help="network configs: prepare the conv weight planes in every call instead of once")
    ap.add_argument("--no-graph", action="store_true",
                    help="network configs: launch every kernel from the host instead of replaying a CUDA graph")
    ap.add_argument("--no-planes", action="store_true",
                    help="resnet: no plane images between convs (each conv splits its NCHW input)")
    ap.add_argument("--shape", default="", help="matmul only: one n,k,m,batch case instead of the sweep")
    ap.add_argument("--int8-peak", action="store_true", help="measure cuBLASLt int8 GEMM (torch._int_mm) and exit")
    args = ap.parse_args()
    global UNFUSED, FUSE_RESIDUAL, PLANES, ONE_LAUNCH, GRAPH, PREPARED
    UNFUSED = args.unfused
    GRAPH = not args.no_graph
    PREPARED = not args.no_prepared
    FUSE_RESIDUAL = not args.no_fuse_residual
    PLANES = not args.no_planes
    ONE_LAUNCH = args.one_launch
    if args.int8_peak:
        return int8_peak()
    if args.shape:
        MatmulSweep.sweep = [tuple(int(v) for v in args.shape.split(","))]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    W = max(args.warmup, 3)
    K = max(args.steps, 1)
    workers = args.cpu_workers or min(os.cpu_count() or 1, 64)

    if args.impl == "reference":
        if rank != 0:
            return 0
        wl = WORKLOADS[args.config](0, 1)
        import multiprocessing as mp
        pool = mp.get_context("spawn").Pool(workers)
        for _ in range(W):
            cpu_sample(args.config, workers, pool)
        vals, kind = [], "port"
        t_all = 0.0
        for _ in range(K):
            u, s, kind = cpu_sample(args.config, workers, pool)
            vals.append(cpu_units_to_value(args.config, u, s))
            t_all += s
        pool.close()
        pool.join()
        v = statistics.median(vals)
        line = {"impl": "reference", "metric": wl.metric, "value": v, "unit": wl.unit, "n_gpus": args.gpus,
                "steps": K, "warmup": W, "ms_per_step": t_all / K * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "ap_fixed<16,8> C-simulation on host cores",
                "data": "synthetic", "config": wl.config(1),
                "cpu_baseline": {"value": v, "unit": wl.unit, "cores": workers, "kind": kind,
                                 "sample": SAMPLE_TEXT[args.config]},
                "e2e": {"value": v, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    import cormorant_b200 as cm
    cm.init(str(local))
    L = cm.lib()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # The CPU baseline pool is spawned before heavy GPU work (rank 0, N = 1 only).
    cpu_line = None
    want_cpu = (rank == 0 and world == 1 and not args.no_cpu_baseline)
    cpool = None
    if want_cpu:
        import multiprocessing as mp
        cpool = mp.get_context("spawn").Pool(workers)

    wl = WORKLOADS[args.config](rank, world)
    wl.setup()
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    for _ in range(W):
        wl.step(cm, stream)
    torch.cuda.synchronize()
    barrier()

    sampler = ClockSampler(gpu_indices(world)) if rank == 0 else None
    time.sleep(0.3 if sampler else 0.0)
    barrier()
    torch.cuda.synchronize()
    lc0 = L.cm_launch_count()
    L.cm_profile_begin()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(K):
        wl.step(cm, stream)
    end.record(stream)
    torch.cuda.synchronize()
    L.cm_profile_end()
    barrier()
    clocks = sampler.stop() if sampler else None
    launches = L.cm_launch_count() - lc0
    elapsed_ms = start.elapsed_time(end)
    import ctypes as C
    dms, dcnt = C.c_double(), C.c_uint64()
    L.cm_profile_read(wl.dominant.encode(), C.byref(dms), C.byref(dcnt))
    dom_note = ""
    if getattr(wl, "graph", None) is not None and wl.dominant == "gemm_q88":
        # graph replays carry no per-launch events: the GEMM's launch durations come from K
        # eager passes right after the timed region
        dms.value, dcnt.value = wl.profile_dominant(cm, stream, K)
        dom_note = ("; GEMM launch durations from CUDA events around each launch over K eager passes right "
                    "after the timed region (which replays a CUDA graph)")
    dom_ms = max_over_ranks(dms.value)
    elapsed_ms = max_over_ranks(elapsed_ms)
    ms_per_step = elapsed_ms / K
    value = wl.units_total / (ms_per_step * 1e-3)
    if args.config == "matmul":
        value /= 1e9
    if getattr(wl, "graph", None) is not None:
        launches = wl.launches_per_step * K        # graph replays launch the captured kernels
    launches_total = int(sum_over_ranks(float(launches)))

    peaks = load_peaks()
    # achieved on the dominant kernel (rank 0): algorithmic units of all its launches / their device time
    if args.config == "lenet":
        roof = {"bound": "launch", "achieved": None, "peak": None, "unit": None, "frac": None, "traffic": None,
                "kernel": "whole network, CUDA graph",
                "note": "0.83 MOPs per image: latency-bound; no roofline fraction (too small)"}
    elif wl.dominant == "gemm_q88":
        achieved = (wl.dom_units_local * K) / (dms.value * 1e-3) / 1e12 if dms.value > 0 else 0.0
        # burst figure for a timed region of about a second or less, sustained beyond
        which = "bf16_sustained" if elapsed_ms > 1500.0 else "bf16"
        peak = 2.0 * peaks[which]
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(f"gemm_q88:{args.config}"),
                "kernel": "gemm_q88_kernel",
                "note": (f"int8 tensor ops (4 s8 MMAs per Q8.8 MAC, x2 ops per MAC) per second on rank 0; peak = "
                         f"2 x {peaks['source']} bf16 {'sustained' if which == 'bf16_sustained' else 'burst'} "
                         f"{peaks[which]} TF/s (dense int8 rate is twice bf16 on B200); traffic = DRAM bytes of "
                         + ("one 4096^3 x 64 launch" if args.config == "matmul" else "one layer-1 3x3 conv GEMM launch")
                         + " (ncu, profiles/)" + dom_note)}
    else:
        achieved = (wl.dom_units_local * K) / (dms.value * 1e-3) / 1e9 if dms.value > 0 else 0.0
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(wl.dominant),
                "kernel": wl.dominant, "note": f"algorithmic bytes / kernel time on rank 0; of {peaks['source']}"}

    # N > 1: the outputs stay sharded in `value`; end to end, a caller that wants every
    # output on every GPU adds one NCCL all-gather of them per step (NVLink / NVSwitch)
    gather = None
    gspec = wl.gather_outputs() if (world > 1 and hasattr(wl, "gather_outputs")) else []
    if gspec:
        from cormorant_b200 import sharding
        gather_bytes = 0
        for t, total, per_item in gspec:                # warm the collectives once
            sharding.gather_batches(t, total, per_item)
        torch.cuda.synchronize()
        barrier()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gs.record(stream)
        for t, total, per_item in gspec:
            full = sharding.gather_batches(t, total, per_item)
            gather_bytes += full.numel() * 2
            del full
        ge.record(stream)
        torch.cuda.synchronize()
        g_ms = max_over_ranks(gs.elapsed_time(ge))
        gv = wl.units_total / ((ms_per_step + g_ms) * 1e-3)
        if args.config == "matmul":
            gv /= 1e9
        gather = {"ms_per_step": g_ms, "bytes_per_step": gather_bytes, "value_with_gather": gv, "unit": wl.unit,
                  "note": "every output of one step all-gathered to every rank (NCCL all_gather over NVLink / "
                          "NVSwitch, max over ranks); value_with_gather = units / (ms_per_step + gather ms); "
                          "gathering to every GPU is bound by each GPU's NVLink ingress, so it does not scale "
                          "with N"}
        torch.cuda.empty_cache()
    per_part = wl.per_part(cm, stream, max(2, min(K, 5))) if (args.per_part and rank == 0) else None
    wl.release()
    torch.cuda.empty_cache()

    e2e = None
    if not args.no_e2e:
        wl.e2e_setup()
        wl.e2e_step()                      # warm-up pass
        torch.cuda.synchronize()
        barrier()
        e_steps = K if args.config in ("lenet", "resnet") else max(1, min(K, 3))
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        if hasattr(wl, "e2e_start"):
            wl.e2e_start(es)
        for _ in range(e_steps):
            wl.e2e_step()
        ee.record()
        torch.cuda.synchronize()
        e_ms = max_over_ranks(es.elapsed_time(ee) / e_steps)
        ev = wl.units_total / (e_ms * 1e-3)
        if args.config == "matmul":
            ev /= 1e9
        e2e = {"value": ev, "unit": wl.unit, "ms_per_step": e_ms,
               "h2d_bytes_per_step": int(sum_over_ranks(float(wl.h2d))),
               "d2h_bytes_per_step": int(sum_over_ranks(float(wl.d2h))),
               "path": getattr(wl, "e2e_path", "cm_buf_sync_to_device -> run_* (cm_* C ABI) -> cm_buf_sync_from_device, "
                                                "pinned host mirrors")}
        wl.e2e_release()

    if want_cpu:
        cpu_sample(args.config, workers, cpool)     # warm
        u, s, kind = cpu_sample(args.config, workers, cpool)
        cpool.close()
        cpool.join()
        cpu_line = {"value": cpu_units_to_value(args.config, u, s), "unit": wl.unit, "cores": workers, "kind": kind,
                    "sample": SAMPLE_TEXT[args.config] + f"; {s:.1f} s wall on {workers} processes"}

    if rank == 0:
        line = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": K, "warmup": W,
                "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "q8.8 int16 (ap_fixed<16,8>); s8 tcgen05 MMA, s32 accumulate"
                if wl.dominant == "gemm_q88" else "q8.8 int16 (ap_fixed<16,8>), int32 / IEEE f32 epilogue",
                "data": "synthetic (seeded)", "config": wl.config(world), "roofline": roof,
                "cpu_baseline": cpu_line, "e2e": e2e, "gpu_launches": launches_total, "clocks": clocks}
        if gather is not None:
            line["gather"] = gather
        if per_part is not None:
            line["per_part"] = per_part
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
