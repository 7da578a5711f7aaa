"""Regenerate the golden vectors in this directory from the REFERENCE kernels.

    python tests/golden/make_golden.py

Needs oracle/_ref (the unmodified reference kernels, kernels/*/kernel/*.cpp,
compiled against oracle/ap_fixed.h -- see oracle/Makefile), i.e. the
reference tree; the committed .npz files are what the CPU tests read.

Cases follow the reference's own C-simulation tests:
  vectorop: the 30 saturation/boundary KATs (TestSimulation.cpp:192-248), the
            two broadcast tests (:274-339), random full-range data per op and size
            (:358-379 sizes), extra broadcast layouts;
  matmul:   the shape / batch / broadcast / saturation matrix of TestMatmulSim.cpp:276-367;
  conv:     the 20 cases of TestConvSim.cpp:284-628 (including both saturation KATs);
  pool:     the 25 cases of TestPoolingSim.cpp:161-229 with that test's own
            deterministic input formula (:103-106), plus full-range variants.
Random data comes from numpy PCG64 with fixed seeds (the reference's
std::default_random_engine / mt19937 streams are not reproduced).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import oracle  # noqa: E402

LSB = 256


def q(v: float) -> int:
    """Data_t(double): floor to the 2^-8 grid (AP_TRN), then wrap to 16 bits (AP_WRAP)."""
    r = int(np.floor(v * LSB))
    return ((r + 32768) % 65536) - 32768


class Book:
    def __init__(self):
        self.arrays: dict[str, np.ndarray] = {}
        self.meta: list[dict] = []

    def add(self, kind: str, name: str, params: dict, inputs: dict[str, np.ndarray], out: np.ndarray):
        i = len(self.meta)
        for k, v in inputs.items():
            self.arrays[f"c{i}_{k}"] = np.asarray(v, np.int16)
        self.arrays[f"c{i}_out"] = np.asarray(out, np.int16)
        self.meta.append({"kind": kind, "name": name, "params": params, "inputs": list(inputs)})

    def save(self, path: Path):
        np.savez_compressed(path, meta=np.frombuffer(json.dumps(self.meta).encode(), np.uint8), **self.arrays)


def rnd(rng, n, lo=-32768, hi=32768):
    return rng.integers(lo, hi, size=int(n)).astype(np.int16)


SAT_KATS = [  # (op, a, b) -- TestSimulation.cpp:192-248
    (0, 100.0, 100.0), (0, 64.0, 64.0), (0, 127.99609375, 0.00390625), (0, -100.0, -100.0),
    (0, -128.0, -0.00390625), (0, 64.0, 63.99609375), (0, -64.0, -64.0),
    (1, 100.0, -100.0), (1, 127.99609375, -0.00390625), (1, -100.0, 100.0), (1, -128.0, 0.00390625),
    (2, 16.0, 16.0), (2, 12.0, 12.0), (2, -16.0, -16.0), (2, -16.0, 16.0), (2, 11.0, 11.0),
    (4, -0.00390625, 0.0), (4, -1.0, 0.0), (4, 0.0, 0.0), (4, 0.00390625, 0.0), (4, 3.5, 0.0),
    (5, -1.0, 0.0), (5, -0.00390625, 0.0), (5, 0.0, 0.0), (5, 0.00390625, 0.0), (5, 3.0, 0.0),
    (5, 5.99609375, 0.0), (5, 6.0, 0.0), (5, 6.00390625, 0.0), (5, 8.0, 0.0), (5, 20.0, 0.0),
]


def make_vectorop(R) -> Book:
    bk = Book()
    for op, av, bv in SAT_KATS:
        a = np.full(8, q(av), np.int16)
        b = np.full(8, q(bv), np.int16)
        p = dict(size=8, op=op, outer=1, a_inc=0, b_inc=0)
        bk.add("vectorop", f"kat op{op} {av} {bv}", p, {"a": a, "b": b}, R.vectorop(a, b, 8, op))
    # broadcast tests, TestSimulation.cpp:286-334
    a = np.array([q(v) for v in range(1, 9)], np.int16)
    b = np.full(4, q(1), np.int16)
    bk.add("vectorop", "a_advances", dict(size=4, op=0, outer=2, a_inc=4, b_inc=0), {"a": a, "b": b},
           R.vectorop(a, b, 4, 0, 2, 4, 0))
    a = np.full(4, q(2), np.int16)
    b = np.array([q(v) for v in range(1, 13)], np.int16)
    bk.add("vectorop", "b_advances", dict(size=4, op=2, outer=3, a_inc=0, b_inc=4), {"a": a, "b": b},
           R.vectorop(a, b, 4, 2, 3, 0, 4))
    rng = np.random.default_rng(42)
    for op in range(8):
        for size in (1, 8, 64, 256, 1024):
            a, b = rnd(rng, size), rnd(rng, size)
            if op == 3:
                b[rng.random(size) < 0.05] = 0
            p = dict(size=size, op=op, outer=1, a_inc=0, b_inc=0)
            bk.add("vectorop", f"random op{op} n{size}", p, {"a": a, "b": b}, R.vectorop(a, b, size, op))
    for (outer, size, ai, bi) in [(3, 5, 9, 0), (4, 7, 3, 2), (3, 16, 0, 0), (6, 24, 32, 8), (4, 1000, 1000, 0)]:
        for op in (0, 2, 3, 5):
            a = rnd(rng, (outer - 1) * ai + size)
            b = rnd(rng, (outer - 1) * bi + size)
            c0 = np.full((outer - 1) * (ai + bi) + size, -23131, np.int16)
            p = dict(size=size, op=op, outer=outer, a_inc=ai, b_inc=bi)
            bk.add("vectorop", f"bcast op{op} {outer}x{size} ({ai},{bi})", p, {"a": a, "b": b, "c0": c0},
                   R.vectorop(a, b, size, op, outer, ai, bi, c=c0.copy()))
    return bk


def make_matmul(R) -> Book:
    bk = Book()
    TN, TK, TM = 4, 256, 16
    shapes = [(1, 1, 1), (TN, TK, TM), (2 * TN, TK, TM), (TN, 2 * TK, TM), (TN, TK, 2 * TM), (TN + 2, TK, TM),
              (TN, TK + 5, TM), (TN, TK, TM + 3), (TN + 2, TK + 5, TM + 3), (7, 13, 5), (TN + 1, 1, TM + 1),
              (1, TK, TM), (TN, TK, 1), (3 * TN, 2 * TK + 7, 2 * TM + 1)]
    rng = np.random.default_rng(43)
    for dist in ("unit", "full"):
        for (n, k, m) in shapes:
            lo, hi = (-256, 257) if dist == "unit" else (-32768, 32768)
            a, b = rnd(rng, n * k, lo, hi), rnd(rng, k * m, lo, hi)
            p = dict(n=n, k=k, m=m, batch=1, a_bs=n * k, b_bs=k * m, c_bs=n * m)
            bk.add("matmul", f"{dist} {n}x{k}x{m}", p, {"a": a, "b": b}, R.matmul(a, b, n, k, m))
    BN, BK, BM = TN + 1, TK // 4, TM + 3
    for (batch, a_bs, b_bs) in [(3, BN * BK, BK * BM), (4, 0, BK * BM), (4, BN * BK, 0), (6, BN * BK, BK * BM)]:
        a = rnd(rng, BN * BK if a_bs == 0 else batch * a_bs, -256, 257)
        b = rnd(rng, BK * BM if b_bs == 0 else batch * b_bs, -256, 257)
        p = dict(n=BN, k=BK, m=BM, batch=batch, a_bs=a_bs, b_bs=b_bs, c_bs=BN * BM)
        bk.add("matmul", f"batch{batch} a_bs{a_bs} b_bs{b_bs}", p, {"a": a, "b": b},
               R.matmul(a, b, BN, BK, BM, batch, a_bs, b_bs, BN * BM))
    for bv in (100.0, -100.0):   # TestMatmulSim.cpp:364-367
        a = np.full(TN * 3, q(100.0), np.int16)
        b = np.full(3 * TM, q(bv), np.int16)
        p = dict(n=TN, k=3, m=TM, batch=1, a_bs=TN * 3, b_bs=3 * TM, c_bs=TN * TM)
        bk.add("matmul", f"saturation b={bv}", p, {"a": a, "b": b}, R.matmul(a, b, TN, 3, TM))
    return bk


def osz(n, k, s, d, p0, p1):
    return (n + p0 + p1 - (d * (k - 1) + 1)) // s + 1


def make_conv(R) -> Book:
    bk = Book()
    TM, TIC = 8, 16
    # (N, C, H, W, M, kh, kw, sh, sw, dh, dw, pt, pl, pb, pr, bias, dw)  TestConvSim.cpp:284-585
    cases = [
        (1, 1, 5, 5, 1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0), (1, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
        (1, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0), (1, 1, 6, 6, 1, 3, 3, 2, 2, 1, 1, 0, 0, 0, 0, 0, 0),
        (1, 1, 5, 5, 2, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0), (2, 1, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0),
        (1, TIC + 5, 5, 5, 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 0), (1, 1, 5, 5, TM + 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
        (1, 1, 9, 9, 1, 3, 3, 1, 1, 2, 2, 0, 0, 0, 0, 0, 0), (1, 1, 7, 7, 1, 5, 5, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0),
        (1, 2 * TIC + 3, 14, 14, 2 * TM + 1, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 0),
        (1, 1, 6, 8, 2, 3, 5, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0), (1, 1, 7, 7, 1, 3, 3, 2, 2, 1, 1, 1, 1, 0, 0, 0, 0),
        (1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, 0, 0, 0, 0, 0, 1), (1, 4, 8, 8, 4, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1),
        (1, TM + 3, 6, 6, TM + 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0, 1), (1, 4, 9, 9, 4, 3, 3, 1, 1, 2, 2, 0, 0, 0, 0, 0, 1),
        (1, 8, 8, 8, 8, 3, 3, 2, 2, 1, 1, 1, 1, 1, 1, 0, 1),
    ]
    rng = np.random.default_rng(44)
    for dist in ("unit", "full"):
        for cs in cases:
            N, C, H, W, M, kh, kw, sh, sw, dh, dw, pt, pl, pb, pr, hb, dwm = cs
            oh, ow = osz(H, kh, sh, dh, pt, pb), osz(W, kw, sw, dw, pl, pr)
            lo, hi = (-256, 257) if dist == "unit" else (-32768, 32768)
            x = rnd(rng, N * C * H * W, lo, hi)
            w = rnd(rng, M * (1 if dwm else C) * kh * kw, lo // 2, hi // 2)
            b = rnd(rng, M, lo, hi)
            p = dict(batch=N, in_ch=C, in_h=H, in_w=W, out_ch=M, out_h=oh, out_w=ow, kh=kh, kw=kw, stride_h=sh,
                     stride_w=sw, dil_h=dh, dil_w=dw, pad_top=pt, pad_left=pl, has_bias=hb, is_depthwise=dwm)
            y = R.conv(x, w, b, N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw, pt, pl, hb, dwm)
            bk.add("conv", f"{dist} {cs}", p, {"x": x, "w": w, "bias": b}, y)
    for (wv, bv) in ((256, 32767), (-256, -32768)):   # TestConvSim.cpp:594-628
        x = np.full(9, 32767, np.int16)
        w = np.array([wv], np.int16)
        b = np.array([bv], np.int16)
        p = dict(batch=1, in_ch=1, in_h=3, in_w=3, out_ch=1, out_h=3, out_w=3, kh=1, kw=1, stride_h=1, stride_w=1,
                 dil_h=1, dil_w=1, pad_top=0, pad_left=0, has_bias=1, is_depthwise=0)
        bk.add("conv", f"saturation w={wv}", p, {"x": x, "w": w, "bias": b},
               R.conv(x, w, b, 1, 1, 3, 3, 1, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0, 1, 0))
    return bk


POOL_CASES = [  # TestPoolingSim.cpp:165-227: N,C,H,W, oh,ow, ph,pw, sh,sw, pt,pl, dh,dw, type, lp, cip
    (1, 4, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0), (1, 4, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0, 0),
    (1, 8, 6, 10, 3, 5, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0), (3, 4, 6, 6, 3, 3, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0),
    (1, 16, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0), (1, 4, 8, 8, 6, 6, 2, 2, 1, 1, 0, 0, 2, 2, 0, 0, 0),
    (1, 8, 4, 4, 1, 1, 4, 4, 1, 1, 0, 0, 1, 1, 0, 0, 0), (2, 12, 6, 6, 1, 1, 6, 6, 1, 1, 0, 0, 1, 1, 0, 0, 0),
    (1, 4, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 1, 0, 0), (1, 4, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 4, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 0), (1, 12, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 1, 0, 0),
    (1, 8, 4, 4, 1, 1, 4, 4, 1, 1, 0, 0, 1, 1, 1, 0, 0), (2, 16, 6, 6, 1, 1, 6, 6, 1, 1, 0, 0, 1, 1, 1, 0, 0),
    (1, 4, 6, 10, 3, 5, 2, 2, 2, 2, 0, 0, 1, 1, 1, 0, 0), (1, 4, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 2, 1, 0),
    (1, 4, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 2, 2, 0), (1, 4, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 2, 1, 0),
    (1, 4, 8, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 2, 2, 0), (1, 8, 4, 4, 1, 1, 4, 4, 1, 1, 0, 0, 1, 1, 2, 1, 0),
    (1, 8, 4, 4, 1, 1, 4, 4, 1, 1, 0, 0, 1, 1, 2, 2, 0), (2, 16, 6, 6, 1, 1, 6, 6, 1, 1, 0, 0, 1, 1, 2, 2, 0),
    (1, 4, 5, 5, 1, 1, 5, 5, 1, 1, 0, 0, 1, 1, 0, 0, 0), (1, 2, 2, 2, 2, 2, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0, 0),
    (1, 32, 8, 8, 4, 4, 2, 2, 2, 2, 0, 0, 1, 1, 0, 0, 0),
]


def pool_test_input(n: int) -> np.ndarray:
    """TestPoolingSim.cpp:103-106: v = ((42*1103515245 + i*12345) mod 2^32 >> 16) % 81;
    x = Data_t((v - 40) * 0.1f)  (float32 product, then floor to 2^-8)."""
    i = np.arange(n, dtype=np.uint64)
    u = (np.uint64(42 * 1103515245) + i * np.uint64(12345)) & np.uint64(0xFFFFFFFF)
    v = ((u >> np.uint64(16)) % np.uint64(81)).astype(np.int64)
    f = (v - 40).astype(np.float32) * np.float32(0.1)
    return np.floor(f.astype(np.float64) * 256.0).astype(np.int16)


def make_pool(R) -> Book:
    bk = Book()
    rng = np.random.default_rng(45)
    for dist in ("reftest", "full"):
        for cs in POOL_CASES:
            N, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip = cs
            x = pool_test_input(N * C * H * W) if dist == "reftest" else rnd(rng, N * C * H * W)
            p = dict(batch=N, channels=C, in_h=H, in_w=W, out_h=oh, out_w=ow, pool_h=ph, pool_w=pw, stride_h=sh,
                     stride_w=sw, pad_top=pt, pad_left=pl, dil_h=dh, dil_w=dw, pool_type=t, lp_order=lp,
                     count_include_pad=cip)
            bk.add("pool", f"{dist} {cs}", p, {"x": x}, R.pool(x, N, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw,
                                                               t, lp, cip))
    return bk


def main():
    R = oracle.ref()
    for name, fn in (("vectorop", make_vectorop), ("matmul", make_matmul), ("conv", make_conv), ("pool", make_pool)):
        bk = fn(R)
        bk.save(HERE / f"{name}.npz")
        print(f"{name}: {len(bk.meta)} cases")


if __name__ == "__main__":
    main()
