#!/usr/bin/env python
"""Benchmark of the Cormorant Q8.8 kernels on B200 -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config all|matmul|vectorop|pool|resnet|lenet]

Default (--config all): every BASELINE config is measured; the line's own keys are the
headline workload, BASELINE.json configs[1] (the metric's configuration): the batched
MatMul sweep, raw int16 uniform [-1024, 1024),
    B=64 x {256^3, 1024^3, 4096^3}  +  B=8 x (8192x4096)(4096x11008),
one step = one pass over the sweep, metric = Q8.8 GOPS = 2*n*k*m*batch / time (the
reference bench's definition, inference-scheduler/bench_src/bench_matmul.c:82-101).
"configs" holds one record per config, each measured the same way (value, ms_per_step,
roofline of its dominant kernel, e2e through the reference-facing API, cpu_baseline,
clocks, per-part breakdown):
  matmul    the headline again;
  lenet     LeNet-5 batch 1, images/s (one step = one inference, CUDA-graph replay);
  vectorop  the 2^28-element sweep of the six ops, GB/s = ports*size*2B / time
            (bench_vectorop.c:92-95);
  pool      the seven pooling variants on [256,64,112,112], GB/s = (x+y bytes) / time
            (bench_pool.c:223-224);
  resnet    the ResNet-18-shaped network at batch 256, images/s; the call list (folded
            epilogues, plane images, conv weights prepared once) captured as one CUDA graph
            and replayed per step (--no-graph, --no-prepared, --no-planes, --unfused select
            the slower forms).
Sub-configs whose step is short time K x STEP_MULT steps so that each timed region lasts a
few hundred ms.  GEMM configs measure the int8 tensor pipe's ceiling (cm_int8_mma_rate) and
cuBLASLt's int8 rate just before their timed region: the roofline's peak.

Multi-GPU (torchrun, one rank per GPU): every workload is sharded by batch
(VectorOP by contiguous element range); no collective runs in the timed
region; the total work is fixed, so scaling is "strong".  Time = max over ranks.
Each record adds "gather": one step's outputs gathered to rank 0 (grouped NCCL
send/recv into offsets) and all-gathered to every rank, each timed on the device.

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
    strides = None          # --shape n,k,m,batch,a_bs,b_bs,c_bs: explicit batch strides (row-strided form)

    def _st(self, n, k, m):
        return self.strides if self.strides is not None else (n * k, k * m, n * m)

    def _words(self, n, k, m, b):
        a_bs, b_bs, c_bs = self._st(n, k, m)
        return (b - 1) * a_bs + n * k, (b - 1) * b_bs + k * m, (b - 1) * c_bs + n * m

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
            return {"workload": "matmul single shape " + ",".join(map(str, self.sweep[0])) + " (n,k,m,batch)"
                    + ("" if self.strides is None else " strides " + ",".join(map(str, self.strides))
                       + " (a_bs,b_bs,c_bs)"),
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
            wa, wb, wc = self._words(n, k, m, b)
            a = torch.randint(-1024, 1024, (wa,), dtype=torch.int16, device="cuda", generator=g)
            bb = torch.randint(-1024, 1024, (wb,), dtype=torch.int16, device="cuda", generator=g)
            c = torch.empty(wc, dtype=torch.int16, device="cuda")
            self.bufs.append((a, bb, c))

    def step(self, cm, stream):
        for (n, k, m, b), t in zip(self.shapes, self.bufs):
            if t is None:
                continue
            cm.MatmulKernel(t[0], t[1], t[2], n, k, m, b, *self._st(n, k, m), stream=stream)

    def step_into(self, cm, stream, outs, before=None, after=None):
        """The step with output i written at device address outs[i]; before(i) / after(i)
        run around output i's kernels."""
        for i, ((n, k, m, b), t, o) in enumerate(zip(self.shapes, self.bufs, outs)):
            if t is None:
                continue
            if before:
                before(i)
            cm.MatmulKernel(t[0], t[1], o, n, k, m, b, *self._st(n, k, m), stream=stream)
            if after:
                after(i)

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
                cm.MatmulKernel(t[0], t[1], t[2], n, k, m, b, *self._st(n, k, m), stream=stream)
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
    e2e_path = ("per batch chunk of a shape: views of the shape's A, B and C buffers (cm_buf_init_view) -> "
                "cm_buf_sync_to_device_async(A, B) -> run_matmul (cm_matmul_async) -> cm_buf_sync_from_device_async(C), "
                "pinned host mirrors; uploads, kernels and downloads on three streams (runtime.CopyOverlap), chunks "
                "of at most ~270 MB of upload in Johnson order for the upload -> download flow (chunks whose upload "
                "is smaller than their download first, by increasing upload, then the rest by decreasing download), "
                "so the download stream starts after the first chunk instead of after the largest shape")

    E2E_CHUNK_BYTES = 270 << 20          # upload bytes per chunk, at most (one batch item at least)

    def e2e_setup(self):
        from cormorant_b200.runtime import CopyOverlap, InferenceBuf
        import numpy as np
        self.e2e = []          # owner buffers per shape
        self.e2e_calls = []    # (n, k, m, items, a_bs, b_bs, c_bs, A view, B view, C view)
        rng = np.random.default_rng(99 + self.rank)
        self.h2d = self.d2h = 0
        jobs = []
        for (n, k, m, b) in self.shapes:
            if b == 0:
                continue
            wa, wb, wc = self._words(n, k, m, b)
            A = InferenceBuf.alloc(wa)
            B = InferenceBuf.alloc(wb)
            Cb = InferenceBuf.alloc(wc)
            fill(A.ptr(), rng, -1024, 1024)
            fill(B.ptr(), rng, -1024, 1024)
            self.e2e.append((A, B, Cb))
            self.h2d += 2 * (wa + wb)
            self.d2h += 2 * wc
            a_bs, b_bs, c_bs = self._st(n, k, m)
            # batch chunks as views; explicit strides (which may overlap items) run whole
            per_up = 2 * (a_bs + b_bs)
            items = b if self.strides is not None else max(1, min(b, self.E2E_CHUNK_BYTES // per_up))
            for i0 in range(0, b, items):
                c = min(items, b - i0)
                views = (InferenceBuf.init_view(A, i0 * a_bs, (c - 1) * a_bs + n * k),
                         InferenceBuf.init_view(B, i0 * b_bs, (c - 1) * b_bs + k * m),
                         InferenceBuf.init_view(Cb, i0 * c_bs, (c - 1) * c_bs + n * m))
                up = 2 * (views[0].count() + views[1].count())
                down = 2 * views[2].count()
                jobs.append((up, down, (n, k, m, c, a_bs, b_bs, c_bs) + views))
        first = sorted((j for j in jobs if j[0] < j[1]), key=lambda j: j[0])
        rest = sorted((j for j in jobs if j[0] >= j[1]), key=lambda j: -j[1])
        self.e2e_calls = [j[2] for j in first + rest]
        self.pipe = CopyOverlap()

    def e2e_start(self, start_event):
        self.pipe.start(start_event)

    def e2e_step(self):
        from cormorant_b200.runtime import run_matmul
        for (n, k, m, c, a_bs, b_bs, c_bs, A, B, Cb) in self.e2e_calls:
            self.pipe.call([A, B], [Cb], lambda s, n=n, k=k, m=m, c=c, st=(a_bs, b_bs, c_bs), A=A, B=B, Cb=Cb:
                           run_matmul(A, B, Cb, n, k, m, c, *st, stream=s))

    def e2e_finish(self):
        self.pipe.join()

    def e2e_release(self):
        self.e2e_calls = []
        for t in self.e2e:
            for buf in t:
                buf.free()
        self.e2e = []
        self.pipe = None


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

    def step_into(self, cm, stream, outs, before=None, after=None):
        for i, (op, o) in enumerate(zip(VOP_OPS, outs)):
            if before:
                before(i)
            cm.VectorOPKernel(self.a, self.b, o, self.n, op, stream=stream)
            if after:
                after(i)

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

    e2e_path = ("per op: cm_buf_sync_to_device_async(a[, b]) -> run_op (cm_vectorop_async) -> "
                "cm_buf_sync_from_device_async(c), pinned host mirrors; consecutive ops use two buffer sets so one "
                "op's copies overlap the next op's kernel (runtime.CopyOverlap)")

    def e2e_setup(self):
        from cormorant_b200.runtime import CopyOverlap, InferenceBuf
        import numpy as np
        rng = np.random.default_rng(5 + self.rank)
        self.sets = []
        for _ in range(2):
            A, B, C = (InferenceBuf.alloc(self.n) for _ in range(3))
            fill(A.ptr(), rng, -32768, 32768)
            fill(B.ptr(), rng, 1, 32768)
            self.sets.append((A, B, C))
        self.h2d = sum((2 if op < 4 else 1) * self.n * 2 for op in VOP_OPS)
        self.d2h = len(VOP_OPS) * self.n * 2
        self.pipe = CopyOverlap()

    def e2e_start(self, start_event):
        self.pipe.start(start_event)

    def e2e_step(self):
        from cormorant_b200.runtime import run_op
        for i, op in enumerate(VOP_OPS):
            A, B, C = self.sets[i % 2]
            ins = [A, B] if op < 4 else [A]
            self.pipe.call(ins, [C], lambda s, op=op, A=A, B=B, C=C:
                           run_op(A, B if op < 4 else None, C, self.n, op, 1, 0, 0, stream=s))

    def e2e_finish(self):
        self.pipe.join()

    def e2e_release(self):
        for t in self.sets:
            for b in t:
                b.free()
        self.sets = []
        self.pipe = None


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

    def _one(self, cm, c, stream, y=None):
        N, C, H, W = POOL_SHAPE
        _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip, oh, ow = c
        cm.PoolingKernel(self.x, self.y if y is None else y, self.nb, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh,
                         dw, t, lp, cip, stream=stream)

    def step_into(self, cm, stream, outs, before=None, after=None):
        for i, (c, o) in enumerate(zip(POOL_SWEEP, outs)):
            if before:
                before(i)
            self._one(cm, c, stream, o)
            if after:
                after(i)

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

    e2e_path = ("per variant: cm_buf_sync_to_device_async(x) -> run_pool (cm_pool_async) -> "
                "cm_buf_sync_from_device_async(y), pinned host mirrors; consecutive variants use two buffer pairs so "
                "one variant's copies overlap the next variant's kernel (runtime.CopyOverlap)")

    def e2e_setup(self):
        from cormorant_b200.runtime import CopyOverlap, InferenceBuf
        import numpy as np
        N, C, H, W = POOL_SHAPE
        rng = np.random.default_rng(8 + self.rank)
        self.X = [InferenceBuf.alloc(self.nb * C * H * W) for _ in range(2)]
        self.Y = [InferenceBuf.alloc(self.nb * C * 56 * 56) for _ in range(2)]
        for x in self.X:
            fill(x.ptr(), rng, -2048, 2048)
        # one output view per (variant, buffer): the variant's output words only
        self.Yv = [[InferenceBuf.init_view(y, 0, self.nb * C * c[12] * c[13]) for y in self.Y] for c in POOL_SWEEP]
        self.h2d = len(POOL_SWEEP) * self.nb * C * H * W * 2
        self.d2h = sum(self.nb * C * c[12] * c[13] * 2 for c in POOL_SWEEP)
        self.pipe = CopyOverlap()

    def e2e_start(self, start_event):
        self.pipe.start(start_event)

    def e2e_step(self):
        from cormorant_b200.runtime import run_pool
        N, C, H, W = POOL_SHAPE
        for i, c in enumerate(POOL_SWEEP):
            _, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip, oh, ow = c
            X, Yv = self.X[i % 2], self.Yv[i][i % 2]
            self.pipe.call([X], [Yv], lambda s, X=X, Yv=Yv, c=c:
                           run_pool(X, Yv, self.nb, C, H, W, c[12], c[13], c[1], c[2], c[3], c[4], c[5], c[6], c[7],
                                    c[8], c[9], c[10], c[11], stream=s))

    def e2e_finish(self):
        self.pipe.join()

    def e2e_release(self):
        self.Yv = []
        for b in self.X + self.Y:
            b.free()
        self.X = self.Y = []
        self.pipe = None


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
            # one cm_calls launch (--one-launch) takes the plain conv and pool calls
            self.net = networks.fuse(self.net, residual=FUSE_RESIDUAL, conv_pool_macs=0 if ONE_LAUNCH else 1 << 22)
        self.planes = self.fused and PLANES and which != "lenet"
        if self.planes:                                          # conv outputs produced as the next convs' operand
            self.net = networks.chain(self.net)
        self.units_total = float(self.batch_total)
        self.units_local = float(self.local)
        self.dom_units_local = 8.0 * self.net.macs_per_image * self.local   # int8 ops (4 MMAs x 2 per MAC)

    def config(self, world):
        calls = ("reference call list, Conv->Relu" + (" and Conv->Add->Relu" if FUSE_RESIDUAL else "")
                 + " and Gemm(MatMul->Add)->Relu chains folded into cm_conv_fused / cm_matmul_fused"
                 + ("; launch-bound Conv->Relu->MaxPool chains as one cm_conv_pool" if not ONE_LAUNCH else "")
                 + ("; conv outputs read by convs written as plane images (cm_conv_planes), channels-last outputs "
                    "into the stem's max pool and the final global pool" if self.planes else "")
                 if self.fused else "reference call list, one C-ABI call per node")
        if self.which == "lenet":
            return {"workload": "lenet5 (BASELINE configs[0])", "batch": 1, "input": "1x1x28x28 uniform [0,1)",
                    "parallelism": f"replicas only: one batch-1 stream per GPU ({world})", "calls": calls,
                    "launches": ("whole call list run as one kernel launch (cm_calls), captured as a CUDA graph"
                                 if ONE_LAUNCH else "whole call list captured once as a CUDA graph and replayed")
                    + (f"; {self.SEQ_IMAGES} consecutive batch-1 inferences (each its whole call list, in order on"
                       " one stream) per graph replay, so one host launch serves 8 images" if GRAPH else "")}
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
        self.graph_seq = None
        self.pending = 0
        if GRAPH and self.local > 0:
            self.graph, self.launches_per_step = self._capture(self.bufs)
            if self.which == "lenet":
                # batch-1 inferences take ~20 us each: one host graph launch per image would
                # make the rate depend on how fast the host submits, so SEQ_IMAGES consecutive
                # inferences (each its whole call list, in order on one stream) form one graph
                self.graph_seq, _ = self._capture(self.bufs, reps=self.SEQ_IMAGES)

    def _backend(self, stream):
        from cormorant_b200 import networks
        return networks.GpuBackend(stream, one_launch=ONE_LAUNCH, weights=self.wcache)

    SEQ_IMAGES = 8      # LeNet: consecutive inferences per replay of the device-timed graph

    def _capture(self, bufs, reps=1):
        """The whole call list captured once as a CUDA graph (its scratch allocations become
        graph memory nodes), `reps` times in a row; returns (graph, kernel launches per pass)."""
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
            for _ in range(reps):
                networks.execute(self.net, self._backend(torch.cuda.current_stream()), bufs)
        n = (cm.launch_count() - l0) // reps
        torch.cuda.synchronize()
        return g, n

    def step_into(self, cm, stream, outs, before=None, after=None):
        """The call list with the network output at outs[0], replayed as its own CUDA graph."""
        if getattr(self, "_into", None) is None or self._into[0] != outs[0]:
            bufs = dict(self.bufs)
            bufs[self.net.resolve(self.net.output)] = int(outs[0])
            self._into = (outs[0], self._capture(bufs)[0])
        if before:
            before(0)
        self._into[1].replay()
        if after:
            after(0)

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
        if self.graph_seq is not None:
            self.pending += 1
            if self.pending == self.SEQ_IMAGES:
                self.graph_seq.replay()
                self.pending = 0
        elif self.graph is not None:
            self.graph.replay()
        elif self.local > 0:
            networks.execute(self.net, self._backend(stream), self.bufs)

    def step_flush(self, cm, stream):
        """Steps not yet run by a multi-image replay run one by one."""
        for _ in range(self.pending):
            self.graph.replay()
        self.pending = 0

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
        if self.which != "lenet":
            try:
                out["layers"] = self.per_layer(stream)
            except Exception as e:          # a breakdown, never a reason to lose the record
                out["layers"] = {"error": f"{type(e).__name__}: {e}"}
        return [out]

    def per_layer(self, stream, passes: int = 3):
        """Per-call roofline of a network's call list: CUDA events around every call of the
        call list in eager passes (median over `passes`; each call's time includes the host
        work of issuing it, which dominates launch-bound calls); conv / MatMul calls against the int8
        pipe's ceiling at the timed region's clock (`self.roof_peak`, int8 TOPS), pools and
        VectorOP against the measured HBM copy rate (`self.hbm_gbs`)."""
        import torch
        from cormorant_b200 import networks
        be = self._backend(stream)
        calls = []
        for name in ("conv", "conv_fused", "conv_planes", "matmul", "matmul_fused", "pool", "pool_planes",
                     "pool_nhwc_planes", "pool_nhwc", "planes_fill", "vectorop"):
            if not hasattr(be, name):
                continue

            def wrap(*a, _o=getattr(be, name), _n=name, **k):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                _o(*a, **k)
                e1.record(stream)
                calls.append((_n, a, e0, e1))
            setattr(be, name, wrap)
        times = []
        for _ in range(passes):
            calls.clear()
            networks.execute(self.net, be, self.bufs)
            torch.cuda.synchronize()
            times.append([c[2].elapsed_time(c[3]) for c in calls])
        rows = []
        for i, (name, a, _, _) in enumerate(calls):
            ms = sorted(t[i] for t in times)[len(times) // 2]
            rec = {"call": i, "kind": name, "us": round(ms * 1e3, 1)}
            if name.startswith("conv"):
                geo = a[6:23] if name == "conv_planes" else a[4:21]
                b, ci, _, _, co, oh, ow, kh, kw = geo[:9]
                dw = geo[16]
                macs = b * co * oh * ow * kh * kw * (1 if dw else ci)
                rec["shape"] = f"{kh}x{kw}/{geo[9]} {ci}->{co} {oh}x{ow}"
                rec["int8_tops"] = round(8.0 * macs / (ms * 1e-3) / 1e12, 1)
                if getattr(self, "roof_peak", None):
                    rec["frac"] = round(rec["int8_tops"] / self.roof_peak, 3)
            elif name.startswith("matmul"):
                n, k, m, bt = a[3:7]
                rec["shape"] = f"{n}x{k}x{m} b{bt}"
                rec["int8_tops"] = round(8.0 * n * k * m * bt / (ms * 1e-3) / 1e12, 1)
                if getattr(self, "roof_peak", None):
                    rec["frac"] = round(rec["int8_tops"] / self.roof_peak, 3)
            elif name.startswith("pool"):
                args = a[2:]
                b, c, ih, iw, oh, ow = args[:6]
                nbytes = 2 * b * c * (ih * iw + oh * ow)
                rec["shape"] = f"{args[6]}x{args[7]}/{args[8]} {c}ch {ih}x{iw}->{oh}x{ow}"
                rec["gbs"] = round(nbytes / (ms * 1e-3) / 1e9, 1)
                if getattr(self, "hbm_gbs", None):
                    rec["frac"] = round(rec["gbs"] / self.hbm_gbs, 3)
            rows.append(rec)
        return rows

    def release(self):
        self.bufs = None
        self.graph = None
        self.graph_seq = None
        self._into = None
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
            self.copy_times = []
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
            # batch 1 is host-launch-bound: the whole step (pinned H2D copy, the call list,
            # D2H copy of the logits) is captured once as a CUDA graph (also the remainder
            # path), and E2E_IMAGES consecutive steps are captured as one pipelined graph
            for _ in range(3):
                self._e2e_body()
            torch.cuda.synchronize()
            self.want_y = self.hy.clone()                     # the logits of a plain step
            self.e2e_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.e2e_graph):
                self._e2e_body()
            torch.cuda.synchronize()
            self._capture_pipelined_lenet()
            self.e2e_path += (f"; {self.E2E_IMAGES} consecutive batch-1 inferences captured as one CUDA graph and replayed:"
                              " each image's call list runs alone on the compute stream, image i+1's input copy"
                              " (copy stream) overlaps image i's call list and image i's logits copy (a third"
                              " stream) overlaps image i+1's; input and output buffers double-buffered, events"
                              " order every reuse")

    def _e2e_body(self):
        import torch
        from cormorant_b200 import networks
        self.bufs[self.net.input].copy_(self.hx, non_blocking=True)
        networks.execute(self.net, self._backend(torch.cuda.current_stream()), self.bufs)
        self.hy.copy_(self.bufs[self.net.resolve(self.net.output)], non_blocking=True)

    E2E_IMAGES = 8      # consecutive batch-1 inferences per pipelined LeNet graph

    def _capture_pipelined_lenet(self):
        """E2E_IMAGES steps as one graph: per image an upload on the copy stream into input
        buffer b = i % 2, the call list on the capture stream (reading x_b, writing y_b), and
        the logits download on the download stream; image i+2's upload waits for image i's
        call list (x_b free), image i+2's call list for image i's download (y_b free)."""
        import torch
        from cormorant_b200 import networks
        K = self.E2E_IMAGES
        xin, yout = self.net.input, self.net.resolve(self.net.output)
        xb = [self.bufs[xin], torch.empty_like(self.bufs[xin])]
        yb = [self.bufs[yout], torch.empty_like(self.bufs[yout])]
        self.hxs = [self.hx.clone().pin_memory() for _ in range(K)]
        self.hys = [torch.empty_like(self.hy).pin_memory() for _ in range(K)]
        up, down = torch.cuda.Stream(), torch.cuda.Stream()

        def body():
            main = torch.cuda.current_stream()
            up.wait_stream(main)
            down.wait_stream(main)
            used, drained = [None, None], [None, None]
            for i in range(K):
                b = i % 2
                with torch.cuda.stream(up):
                    if used[b] is not None:
                        up.wait_event(used[b])
                    xb[b].copy_(self.hxs[i], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(up)
                main.wait_event(ready)
                if drained[b] is not None:
                    main.wait_event(drained[b])
                bufs = dict(self.bufs)
                bufs[xin], bufs[yout] = xb[b], yb[b]
                networks.execute(self.net, self._backend(main), bufs)
                done = torch.cuda.Event()
                done.record(main)
                used[b] = done
                with torch.cuda.stream(down):
                    down.wait_event(done)
                    self.hys[i].copy_(yb[b], non_blocking=True)
                    fin = torch.cuda.Event()
                    fin.record(down)
                drained[b] = fin
            main.wait_stream(up)
            main.wait_stream(down)

        for _ in range(2):
            body()
        torch.cuda.synchronize()
        self.e2e_pipe_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.e2e_pipe_graph):
            body()
        torch.cuda.synchronize()
        self.e2e_pending = 0

    def e2e_step(self):
        if getattr(self, "e2e_pipe_graph", None) is not None:
            self.e2e_pending += 1
            if self.e2e_pending == self.E2E_IMAGES:
                self.e2e_pipe_graph.replay()
                self.e2e_pending = 0
        elif self.e2e_graph is not None:
            self.e2e_graph.replay()
        elif self.copy_stream is not None:
            self._e2e_pipelined()
        else:
            self._e2e_body()

    def e2e_finish(self):
        """Steps not yet run by a pipelined replay run one by one."""
        if getattr(self, "e2e_pipe_graph", None) is not None:
            for _ in range(self.e2e_pending):
                self.e2e_graph.replay()
            self.e2e_pending = 0

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
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(self.copy_stream)
            self.xbufs[b].copy_(self.hx, non_blocking=True)
            t1.record(self.copy_stream)
            self.copied[b].record(self.copy_stream)
            self.copy_times.append((t0, t1))

    def e2e_extra(self):
        """The input copies' own device time (host -> device over PCIe): how much of a step
        the copy takes when the host is busy or idle.  LeNet: whether every image's logits
        copied back by the pipelined graph equal those of a plain step."""
        if getattr(self, "e2e_pipe_graph", None) is not None:
            import torch
            torch.cuda.synchronize()
            return {"outputs_match": all(bool(torch.equal(h, self.want_y)) for h in self.hys + [self.hy])}
        if not getattr(self, "copy_times", None):
            return {}
        ms = [a.elapsed_time(b) for a, b in self.copy_times[1:]] or [0.0]
        med = sorted(ms)[len(ms) // 2]
        return {"h2d_copy_ms_median": round(med, 4), "h2d_copy_ms_max": round(max(ms), 4),
                "h2d_gbs_median": round(self.hx.numel() * 2 / (med * 1e-3) / 1e9, 1) if med > 0 else None}

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
        self.e2e_pipe_graph = None
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
        reps = 50 if config == "lenet" else 1       # a LeNet-5 inference is ~1 ms of CPU
        for node in [nd for _ in range(reps) for nd in net.nodes]:
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
        units = float(reps)
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
    "lenet": "50 whole LeNet-5 inferences (batch 1) per worker process, kernel time summed per worker",
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
    if config in ("resnet", "lenet"):
        # per-worker rates (kernel time only, summed over the call list; ResNet's conv times are
        # scaled estimates): the workers run in parallel, each at units/dt images per second
        rate = sum(r[0] / r[1] for r in res)
        return rate, 1.0, kind
    return units, wall, kind


def cpu_units_to_value(config, units, seconds):
    if config == "matmul":
        return units / seconds / 1e9       # GOPS
    return units / seconds                 # GB/s (units already in GB) or images/s


def int8_ceiling(cm, seconds: float = 0.4) -> dict:
    """The int8 tensor-pipe ceiling of this GPU, measured now (before a GEMM config's timed region):
    the GEMM's own MMA stream with its operands resident in shared memory (cm_int8_mma_rate, CTA
    pairs and single CTAs: no memory traffic, so nothing but the pipe bounds it), and cuBLASLt's
    int8 GEMM (torch._int_mm 8192^3, s8 x s8 -> s32) as a library reference point."""
    import ctypes as C
    import torch
    from cormorant_b200 import _lib
    L = cm.lib()
    out = {}
    for pairs, key in ((1, "mma_pairs_tops"), (0, "mma_single_tops")):
        tops, ms, mhz = C.c_double(), C.c_double(), C.c_double()
        _lib.check(L.cm_int8_mma_rate(pairs, 16384, C.byref(tops), C.byref(ms), C.byref(mhz)))
        out[key] = round(tops.value, 1)
        out[key.replace("_tops", "_sm_mhz")] = round(mhz.value, 1)
    n = 8192
    a = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best, t_end = 1e9, time.time() + seconds
    while time.time() < t_end:
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        torch._int_mm(a, b)
        e_.record()
        torch.cuda.synchronize()
        best = min(best, s_.elapsed_time(e_))
    out["cublaslt_int8_tops"] = round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1)
    best = "mma_pairs" if out["mma_pairs_tops"] >= out["mma_single_tops"] else "mma_single"
    out["ceiling_tops"] = out[best + "_tops"]
    out["ceiling_sm_mhz"] = out[best + "_sm_mhz"]     # the SM clock the ceiling was measured at
    del a, b
    torch.cuda.empty_cache()
    return out


def int8_peak() -> int:
    """--int8-peak: print the int8 ceiling measurements and exit."""
    import torch
    import cormorant_b200 as cm
    torch.cuda.set_device(0)
    cm.init("0")
    print(json.dumps({**int8_ceiling(cm, seconds=4.0),
                      "how": "cm_int8_mma_rate (the GEMM's MMAs on resident operands; pairs = cta_group::2) and "
                             "torch._int_mm 8192^3 s8xs8->s32 (best over 4 s)"}))
    return 0


# Sub-configs of the default run time more steps than K where one step is short, so that
# each timed region lasts a few hundred ms (enough nvidia-smi clock samples).
STEP_MULT = {"matmul": 1, "resnet": 5, "vectorop": 10, "pool": 20, "lenet": 500}
ALL_CONFIGS = ["matmul", "lenet", "vectorop", "pool", "resnet"]


class Env:
    """Per-process plumbing shared by the configs of one run."""

    def __init__(self, args, world, rank, local, cm, cpool, workers):
        import torch
        self.args, self.world, self.rank, self.local = args, world, rank, local
        self.cm, self.L = cm, cm.lib()
        self.cpool, self.workers = cpool, workers
        self.peaks = load_peaks()
        self.stream = torch.cuda.current_stream()
        self.cpu_warm = False

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def reduce(self, x: float, op: str) -> float:
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return float(t.item())


def measure(name: str, env: Env, K: int, W: int, detail: bool) -> dict | None:
    """One config on every rank: setup, W warm-up steps, K timed steps (barrier + synchronize on both
    sides, CUDA events, max over ranks), the dominant kernel's roofline, the output gathers (N > 1),
    the per-part breakdown, the end-to-end run through the reference-facing API and the CPU baseline
    (rank 0 at N = 1).  Returns rank 0's record (None on other ranks)."""
    import ctypes as C
    import torch
    cm, L, world, rank, stream = env.cm, env.L, env.world, env.rank, env.stream
    wl = WORKLOADS[name](rank, world)
    wl.setup()
    torch.cuda.synchronize()
    for _ in range(W):
        wl.step(cm, stream)
    if hasattr(wl, "step_flush"):
        wl.step_flush(cm, stream)
    torch.cuda.synchronize()
    env.barrier()

    ceiling = int8_ceiling(cm) if wl.dominant == "gemm_q88" and name != "lenet" else None
    env.barrier()
    sampler = ClockSampler(gpu_indices(world)) if rank == 0 else None
    time.sleep(0.3 if sampler else 0.0)
    env.barrier()
    torch.cuda.synchronize()
    lc0 = L.cm_launch_count()
    L.cm_profile_begin()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(K):
        wl.step(cm, stream)
    if hasattr(wl, "step_flush"):
        wl.step_flush(cm, stream)
    end.record(stream)
    torch.cuda.synchronize()
    L.cm_profile_end()
    env.barrier()
    clocks = sampler.stop() if sampler else None
    launches = L.cm_launch_count() - lc0
    elapsed_ms = start.elapsed_time(end)
    dms, dcnt = C.c_double(), C.c_uint64()
    L.cm_profile_read(wl.dominant.encode(), C.byref(dms), C.byref(dcnt))
    dom_note = ""
    if getattr(wl, "graph", None) is not None and wl.dominant == "gemm_q88" and name != "lenet":
        # graph replays carry no per-launch events: the GEMM's launch durations come from K
        # eager passes right after the timed region
        dms.value, dcnt.value = wl.profile_dominant(cm, stream, K)
        dom_note = ("; GEMM launch durations from CUDA events around each launch over K eager passes right "
                    "after the timed region (which replays a CUDA graph)")
    # the SM clock the GEMM launches themselves ran at (cycle counter / global timer of each
    # launch's first CTA), over the same launches as the durations
    gemm_mhz = C.c_double(0.0)
    if wl.dominant == "gemm_q88" and L.cm_profile_gemm_clock(C.byref(gemm_mhz)) != 0:
        gemm_mhz.value = 0.0
    elapsed_ms = env.reduce(elapsed_ms, "max")
    ms_per_step = elapsed_ms / K
    scale = 1e9 if name == "matmul" else 1.0
    value = wl.units_total / (ms_per_step * 1e-3) / scale
    if getattr(wl, "graph", None) is not None:
        launches = wl.launches_per_step * K        # graph replays launch the captured kernels
    launches_total = int(env.reduce(float(launches), "sum"))

    peaks = env.peaks
    if name == "lenet":
        roof = {"bound": "launch", "achieved": None, "peak": None, "unit": None, "frac": None, "traffic": None,
                "kernel": "whole network, CUDA graph",
                "note": "0.83 MOPs per image: latency-bound; no roofline fraction (too small)"}
    elif wl.dominant == "gemm_q88":
        achieved = (wl.dom_units_local * K) / (dms.value * 1e-3) / 1e12 if dms.value > 0 else 0.0
        which = "bf16_sustained" if elapsed_ms > 1500.0 else "bf16"
        proxy = 2.0 * peaks[which]
        burst = ceiling["ceiling_tops"]
        # The ceiling is a burst measurement taken just before the timed region, at the SM
        # clock the probe reports; the GEMM runs for seconds, under the power cap, at the
        # clock the sampler saw.  The pipe's rate per clock is fixed, so the ceiling at the
        # GEMM's clock is the burst figure x run clock / probe clock: frac is the fraction
        # of the pipe's per-clock capacity, whatever the power cap does to the clock.
        sampled_mhz = (clocks or {}).get("sm_mhz")
        run_mhz = round(gemm_mhz.value, 1) if gemm_mhz.value > 0 else sampled_mhz
        probe_mhz = ceiling.get("ceiling_sm_mhz")
        scale_ = run_mhz / probe_mhz if run_mhz and probe_mhz else 1.0
        peak = round(burst * scale_, 1)
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(f"gemm_q88:{name}"),
                "kernel": "gemm_q88_kernel",
                "peak_burst": burst, "frac_of_burst": round(achieved / burst, 4),
                "peak_clock_scale": {"run_sm_mhz": run_mhz, "ceiling_sm_mhz": probe_mhz, "scale": round(scale_, 4),
                                     "gemm_sm_mhz": round(gemm_mhz.value, 1) if gemm_mhz.value > 0 else None,
                                     "sampled_sm_mhz": sampled_mhz},
                "int8_ceiling": ceiling,
                "int8_measured_tops": ceiling["cublaslt_int8_tops"],
                "frac_of_cublaslt_int8": round(achieved / ceiling["cublaslt_int8_tops"], 4),
                "proxy_2x_bf16": round(proxy, 1), "frac_of_proxy": round(achieved / proxy, 4),
                "note": ("achieved = int8 tensor ops (4 s8 MMAs per Q8.8 multiply-add, 2 ops each) of the GEMM "
                         "launches / their CUDA-event time on rank 0; peak_burst = the int8 tensor pipe's ceiling "
                         "measured in this run just before the timed region (cm_int8_mma_rate: the GEMM's MMA "
                         "stream on shared-memory-resident operands, best of CTA pairs and single CTAs, at the SM "
                         "clock it reports); peak = that ceiling at the SM clock the GEMM launches ran at (their "
                         "own cycle counter over the global timer; the sampled median when absent): burst x run "
                         "clock / probe clock, the pipe's per-clock capacity at the clock the power cap left; also "
                         f"against cuBLASLt's int8 GEMM (a library rate, not a ceiling) and 2 x the {peaks['source']} "
                         f"bf16 {'sustained' if which == 'bf16_sustained' else 'burst'} rate {peaks[which]} TF/s; "
                         "traffic = DRAM bytes of "
                         + ("one 4096^3 x 64 launch" if name == "matmul" else "one layer-1 3x3 conv GEMM launch")
                         + " (ncu, profiles/)" + dom_note)}
    else:
        achieved = (wl.dom_units_local * K) / (dms.value * 1e-3) / 1e9 if dms.value > 0 else 0.0
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(wl.dominant),
                "kernel": wl.dominant,
                "note": f"algorithmic bytes / kernel CUDA-event time on rank 0; peak = {peaks['source']} HBM copy rate"}

    gather = measure_gathers(wl, env, ms_per_step, scale, K) if world > 1 else None
    wl.roof_peak = roof.get("peak") if roof.get("unit") == "TFLOP/s" else None
    wl.hbm_gbs = peaks["hbm_gbs"]
    per_part = wl.per_part(cm, stream, max(2, min(K, 5))) if (detail and rank == 0) else None
    wl.release()
    torch.cuda.empty_cache()

    e2e = None
    if not env.args.no_e2e:
        wl.e2e_setup()
        # warm-up passes: ResNet alternates two input buffers, each with its own CUDA graph,
        # and a graph's first replay uploads it; both are replayed once before the timing
        for _ in range(2 if name == "resnet" else 1):
            wl.e2e_step()
        if hasattr(wl, "e2e_finish"):
            wl.e2e_finish()
        torch.cuda.synchronize()
        env.barrier()
        e_steps = K if name in ("lenet", "resnet") else max(1, min(K, 3))
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        if hasattr(wl, "e2e_start"):
            wl.e2e_start(es)
        for _ in range(e_steps):
            wl.e2e_step()
        if hasattr(wl, "e2e_finish"):
            wl.e2e_finish()
        ee.record()
        torch.cuda.synchronize()
        e_ms = env.reduce(es.elapsed_time(ee) / e_steps, "max")
        e2e = {"value": wl.units_total / (e_ms * 1e-3) / scale, "unit": wl.unit, "ms_per_step": e_ms,
               "steps": e_steps,
               "h2d_bytes_per_step": int(env.reduce(float(wl.h2d), "sum")),
               "d2h_bytes_per_step": int(env.reduce(float(wl.d2h), "sum")),
               "path": getattr(wl, "e2e_path", "cm_buf_sync_to_device -> run_* (cm_* C ABI) -> "
                                                "cm_buf_sync_from_device, pinned host mirrors")}
        if hasattr(wl, "e2e_extra"):
            e2e.update(wl.e2e_extra())
        wl.e2e_release()
        torch.cuda.empty_cache()

    cpu_line = None
    if env.cpool is not None:
        if not env.cpu_warm:
            cpu_sample(name, env.workers, env.cpool)     # warm: the workers load the reference kernels
            env.cpu_warm = True
        u, sec, kind = cpu_sample(name, env.workers, env.cpool)
        cpu_line = {"value": cpu_units_to_value(name, u, sec), "unit": wl.unit, "cores": env.workers, "kind": kind,
                    "sample": SAMPLE_TEXT[name] + f"; {sec:.1f} s wall on {env.workers} processes"}
    if rank != 0:
        return None
    rec = {"metric": wl.metric, "value": value, "unit": wl.unit, "n_gpus": world, "steps": K, "warmup": W,
           "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "q8.8 int16 (ap_fixed<16,8>); s8 tcgen05 MMA, s32 accumulate"
           if wl.dominant == "gemm_q88" and name != "lenet" else "q8.8 int16 (ap_fixed<16,8>), int32 / IEEE f32 epilogue",
           "data": "synthetic (seeded)", "config": wl.config(world), "roofline": roof,
           "cpu_baseline": cpu_line, "e2e": e2e, "gpu_launches": launches_total, "clocks": clocks}
    if gather is not None:
        rec["gather"] = gather
    if per_part is not None:
        rec["per_part"] = per_part
    return rec


def measure_gathers(wl, env: Env, ms_per_step: float, scale: float, K: int) -> dict | None:
    """N > 1: the outputs stay sharded in `value`.  A caller that wants them together on one GPU
    (or every GPU) gets them three ways, each timed on the device (max over ranks):
      fused_to_root  every rank's kernels write their output shard straight into rank 0's buffers
                     (sharding.RootOutputs: CUDA-IPC-mapped, plain stores over NVLink while the
                     kernels run); K whole steps timed, gather included;
      to_root        after the step, every rank sends its shards and rank 0 receives each into its
                     offset (grouped NCCL send/recv);
      all_gather     after the step, every output to every rank (NCCL all_gather_into_tensor).
      copy_to_root   the other ranks compute each output into their own memory and push it to
                     rank 0 with one copy-engine cudaMemcpyAsync (cm_copy_async, NVLink) on a copy
                     stream while the next output computes; K whole steps timed.
    The fused and copy forms' root output is checked word for word against the NCCL gather of
    the same step's last output."""
    import torch
    from cormorant_b200 import sharding
    spec = wl.gather_outputs() if hasattr(wl, "gather_outputs") else []
    if not spec:
        return None
    world, rank, stream = env.world, env.rank, env.stream
    full_bytes = sum(total * per_item * 2 for _, total, per_item in spec)
    # bytes that cross NVLink into the receiving GPU: every shard but its own
    ingress = sum((total - sharding.shard_range(total, 0, world)[1]) * per_item * 2 for _, total, per_item in spec)
    res = {"unit": wl.unit, "bytes_per_step": full_bytes, "ingress_bytes_per_gpu": ingress}
    last_nccl = None
    for kind in ("to_root", "all_gather"):
        outs = []
        for t, total, per_item in spec:
            if kind == "to_root":
                outs.append(torch.empty(total * per_item, dtype=torch.int16, device="cuda") if rank == 0 else None)
            else:
                outs.append(torch.empty(total * per_item, dtype=torch.int16, device="cuda"))

        def run():
            for (t, total, per_item), o in zip(spec, outs):
                if kind == "to_root":
                    sharding.gather_to_root(t, total, per_item, root=0, out=o)
                else:
                    sharding.gather_batches(t, total, per_item, out=o)
        run()                                           # warm the communicators
        torch.cuda.synchronize()
        env.barrier()
        gs, ge = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        gs.record(stream)
        run()
        ge.record(stream)
        torch.cuda.synchronize()
        g_ms = env.reduce(gs.elapsed_time(ge), "max")
        res[kind] = {"ms_per_step": g_ms, "ingress_gbs": round(ingress / (g_ms * 1e-3) / 1e9, 1) if g_ms > 0 else None,
                     "value_with_gather": wl.units_total / ((ms_per_step + g_ms) * 1e-3) / scale}
        if kind == "to_root" and rank == 0:
            last_nccl = outs[-1]
        del outs
        env.barrier()
    if hasattr(wl, "step_into"):
        ro = sharding.RootOutputs([total * per_item for _, total, per_item in spec])
        addrs = [ro.address(i, sharding.shard_range(total, rank, world)[0] * per_item)
                 for i, (_, total, per_item) in enumerate(spec)]
        for _ in range(2):                              # warm (a network captures its graph)
            wl.step_into(env.cm, stream, addrs)
        torch.cuda.synchronize()
        env.barrier()
        fs, fe = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        fs.record(stream)
        for _ in range(K):
            wl.step_into(env.cm, stream, addrs)
        fe.record(stream)
        torch.cuda.synchronize()
        env.barrier()
        f_ms = env.reduce(fs.elapsed_time(fe), "max") / K
        same = None
        if rank == 0:
            same = bool(torch.equal(ro.tensors[-1], last_nccl))
        res["fused_to_root"] = {"ms_per_step": f_ms,
                                "ingress_gbs": round(ingress / (f_ms * 1e-3) / 1e9, 1) if f_ms > 0 else None,
                                "value_with_gather": wl.units_total / (f_ms * 1e-3) / scale,
                                "steps": K, "matches_nccl_gather": same}
        # copy engines: the other ranks compute output i into their own memory, then push it to
        # rank 0 with one cudaMemcpyAsync on a copy stream while output i+1 computes
        import ctypes as C
        L = env.L
        locs = None
        if rank == 0:
            outs = addrs
        else:
            locs = [torch.empty(max(sharding.shard_range(total, rank, world)[1] * per_item, 1), dtype=torch.int16,
                                device="cuda") for _, total, per_item in spec]
            outs = [t.data_ptr() for t in locs]
        cstream = torch.cuda.Stream()
        copied = [None] * len(spec)

        def before(i):
            if copied[i] is not None:
                stream.wait_event(copied[i])      # last step's push of this buffer is done

        def after(i):
            if rank == 0:
                return
            _, total, per_item = spec[i]
            ev = torch.cuda.Event()
            ev.record(stream)
            cstream.wait_event(ev)
            nbytes = sharding.shard_range(total, rank, world)[1] * per_item * 2
            L.cm_copy_async(C.c_void_p(addrs[i]), C.c_void_p(outs[i]), nbytes, C.c_void_p(cstream.cuda_stream))
            done = torch.cuda.Event()
            done.record(cstream)
            copied[i] = done
        for _ in range(2):
            wl.step_into(env.cm, stream, outs, before, after)
        stream.wait_stream(cstream)
        torch.cuda.synchronize()
        env.barrier()
        cs_, ce_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cs_.record(stream)
        cstream.wait_event(cs_)
        for _ in range(K):
            wl.step_into(env.cm, stream, outs, before, after)
        stream.wait_stream(cstream)
        ce_.record(stream)
        torch.cuda.synchronize()
        env.barrier()
        c_ms = env.reduce(cs_.elapsed_time(ce_), "max") / K
        same = bool(torch.equal(ro.tensors[-1], last_nccl)) if rank == 0 else None
        res["copy_to_root"] = {"ms_per_step": c_ms,
                               "ingress_gbs": round(ingress / (c_ms * 1e-3) / 1e9, 1) if c_ms > 0 else None,
                               "value_with_gather": wl.units_total / (c_ms * 1e-3) / scale,
                               "steps": K, "matches_nccl_gather": same}
        outs = locs = None
        ro.close()
    del last_nccl
    torch.cuda.empty_cache()
    env.barrier()
    res["note"] = ("value_with_gather = units / time of a step whose outputs end up on rank 0 (fused_to_root: the "
                   "kernels write there directly; copy_to_root: copy-engine pushes overlapped with the next output's "
                   "kernels; both K steps timed; to_root / all_gather: ms_per_step + the NCCL "
                   "collective's ms); ingress_gbs = bytes arriving at one GPU / that time; the receiving GPU's "
                   "NVLink ingress bounds every form")
    return res


# --------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["all"] + sorted(WORKLOADS), default="all",
                    help="all (default): the MatMul sweep as the headline line plus every BASELINE config in "
                         "'configs'; or one config alone")
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
    ap.add_argument("--shape", default="", help="matmul only: one n,k,m,batch[,a_bs,b_bs,c_bs] case instead "
                                                "of the sweep")
    ap.add_argument("--int8-peak", action="store_true", help="measure the int8 ceilings (MMA stream, cuBLASLt) and exit")
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
        v = tuple(int(x) for x in args.shape.split(","))
        if len(v) not in (4, 7):
            ap.error("--shape takes n,k,m,batch or n,k,m,batch,a_bs,b_bs,c_bs")
        MatmulSweep.sweep = [v[:4]]
        MatmulSweep.strides = v[4:] if len(v) == 7 else None
        if args.config == "all":
            args.config = "matmul"
    names = ALL_CONFIGS if args.config == "all" else [args.config]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    W = max(args.warmup, 3)
    K = max(args.steps, 1)
    workers = args.cpu_workers or min(os.cpu_count() or 1, 64)

    if args.impl == "reference":
        if rank != 0:
            return 0
        import multiprocessing as mp
        pool = mp.get_context("spawn").Pool(workers)
        recs = {}
        for i, name in enumerate(names):
            wl = WORKLOADS[name](0, 1)
            # the headline config takes W + K samples; the others 1 + 3 (a ResNet sample is ~10 s of CPU)
            w_, k_ = (W, K) if i == 0 else (1, 3)
            for _ in range(w_):
                cpu_sample(name, workers, pool)
            vals, kind, t_all = [], "port", 0.0
            for _ in range(k_):
                u, sec, kind = cpu_sample(name, workers, pool)
                vals.append(cpu_units_to_value(name, u, sec))
                t_all += sec
            v = statistics.median(vals)
            recs[name] = {"impl": "reference", "metric": wl.metric, "value": v, "unit": wl.unit, "n_gpus": args.gpus,
                          "steps": k_, "warmup": w_, "ms_per_step": t_all / k_ * 1e3, "higher_is_better": True,
                          "scaling": "strong", "vs_baseline": None,
                          "dtype": "ap_fixed<16,8> C-simulation on host cores",
                          "data": "synthetic", "config": wl.config(1),
                          "cpu_baseline": {"value": v, "unit": wl.unit, "cores": workers, "kind": kind,
                                           "sample": SAMPLE_TEXT[name]},
                          "e2e": {"value": v, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        pool.close()
        pool.join()
        line = dict(recs[names[0]])
        if len(names) > 1:
            line["configs"] = recs
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

    # The CPU baseline pool is spawned before heavy GPU work (rank 0, N = 1 only).
    cpool = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import multiprocessing as mp
        cpool = mp.get_context("spawn").Pool(workers)
    env = Env(args, world, rank, local, cm, cpool, workers)
    recs = {}
    for i, name in enumerate(names):
        mult = 1 if i == 0 or len(names) == 1 else STEP_MULT[name]
        if name == "lenet" and len(names) == 1:
            mult = STEP_MULT["lenet"]
        recs[name] = measure(name, env, K * mult, W, detail=args.per_part or len(names) > 1)
        env.barrier()
    if cpool is not None:
        cpool.close()
        cpool.join()
    if rank == 0:
        line = dict(recs[names[0]])
        if len(names) > 1:
            line["configs"] = {n: recs[n] for n in names}
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
