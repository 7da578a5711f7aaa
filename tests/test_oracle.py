"""CPU tests of the parity checker itself (no GPU).

1. The C restatement (oracle/cm_oracle.c) reproduces every committed golden
   vector (tests/golden/*.npz, generated from the reference kernels by
   tests/golden/make_golden.py).
2. The golden KATs hold the values the reference's own tests expect
   (TestSimulation.cpp:192-248, TestMatmulSim.cpp:364-367, TestConvSim.cpp:594-628).
3. When the reference tree was available at build time (oracle/_ref): the
   reference's own C-simulation tests pass against the fixed-point shim, and
   the restatement agrees with the reference kernels on seeded random calls.
4. The numpy float64 MatMul restatement (oracle/fast.py) agrees with the C one.
"""
import json
import subprocess
import zlib
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import fast
from tests._util import assert_same, rand16

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    return z, meta


def run_port(port, kind, p, arr):
    if kind == "vectorop":
        c0 = arr.get("c0")
        return port.vectorop(arr["a"], arr["b"], p["size"], p["op"], p["outer"], p["a_inc"], p["b_inc"],
                             c=None if c0 is None else c0.copy())
    if kind == "matmul":
        return port.matmul(arr["a"], arr["b"], p["n"], p["k"], p["m"], p["batch"], p["a_bs"], p["b_bs"], p["c_bs"])
    if kind == "conv":
        return port.conv(arr["x"], arr["w"], arr["bias"], p["batch"], p["in_ch"], p["in_h"], p["in_w"], p["out_ch"],
                         p["out_h"], p["out_w"], p["kh"], p["kw"], p["stride_h"], p["stride_w"], p["dil_h"],
                         p["dil_w"], p["pad_top"], p["pad_left"], p["has_bias"], p["is_depthwise"])
    return port.pool(arr["x"], p["batch"], p["channels"], p["in_h"], p["in_w"], p["out_h"], p["out_w"], p["pool_h"],
                     p["pool_w"], p["stride_h"], p["stride_w"], p["pad_top"], p["pad_left"], p["dil_h"], p["dil_w"],
                     p["pool_type"], p["lp_order"], p["count_include_pad"])


@pytest.mark.parametrize("name", ["vectorop", "matmul", "conv", "pool"])
def test_port_matches_golden(port, name):
    z, meta = load(name)
    assert len(meta) >= 30
    for i, m in enumerate(meta):
        arr = {k: z[f"c{i}_{k}"] for k in m["inputs"]}
        got = run_port(port, m["kind"], m["params"], arr)
        assert_same(got, z[f"c{i}_out"], f"{name} case {i} ({m['name']})")


def sat(v):
    return max(-32768, min(32767, v))


def kat_expect(op, a, b):
    """Documented op semantics on raw words (VectorOP.cpp:8-35)."""
    if op == 0:
        return sat(a + b)
    if op == 1:
        return sat(a - b)
    if op == 2:
        return sat((a * b) >> 8)
    if op == 4:
        return max(a, 0)
    return min(max(a, 0), 0x600)


def test_golden_kats_hold_reference_expectations():
    z, meta = load("vectorop")
    n = 0
    for i, m in enumerate(meta):
        if m["name"].startswith("kat"):
            a, b, out = int(z[f"c{i}_a"][0]), int(z[f"c{i}_b"][0]), z[f"c{i}_out"]
            assert (out == kat_expect(m["params"]["op"], a, b)).all(), m["name"]
            n += 1
    assert n == 31
    z, meta = load("matmul")
    sats = [(m, z[f"c{i}_out"]) for i, m in enumerate(meta) if m["name"].startswith("saturation")]
    assert len(sats) == 2
    assert (sats[0][1] == 32767).all() and (sats[1][1] == -32768).all()
    z, meta = load("conv")
    sats = [z[f"c{i}_out"] for i, m in enumerate(meta) if m["name"].startswith("saturation")]
    assert (sats[0] == 32767).all() and (sats[1] == -32768).all()


def test_division_semantics(port):
    """DIV: b == 0 -> 0; otherwise (a << 8) / b truncated toward zero (dtype.py:110-124), saturated."""
    rng = np.random.default_rng(3)
    for _ in range(20000):
        a, b = int(rng.integers(-32768, 32768)), int(rng.integers(-32768, 32768))
        want = 0 if b == 0 else sat(int(np.trunc((a * 256) / b)) if abs(a * 256) < 2**52 else 0)
        if b != 0:
            q = abs(a * 256) // abs(b)
            want = sat(q if (a * 256 >= 0) == (b > 0) else -q)
        assert port.scalar(3, a, b) == want, (a, b)


need_ref = pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (needs the reference tree)")


@need_ref
@pytest.mark.parametrize("binary", ["TestSimulation", "TestMatmulSim", "TestConvSim", "TestPoolingSim"])
def test_reference_csim_suite_passes_on_shim(binary):
    exe = Path(oracle.ORACLE_DIR) / "_ref" / binary
    if not exe.exists():
        pytest.skip("reference test binaries not built")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def _seed(*xs):
    return zlib.crc32(repr(xs).encode())


@need_ref
@pytest.mark.parametrize("trial", range(6))
def test_port_vs_reference_fuzz(port, trial):
    R = oracle.ref()
    rng = np.random.default_rng(_seed("fuzz", trial))
    # vectorop
    for _ in range(10):
        op = int(rng.integers(0, 8))
        outer = int(rng.integers(1, 5))
        size = int(rng.integers(1, 300))
        ai, bi = int(rng.integers(0, 2 * size)), int(rng.integers(0, 2 * size))
        a, b = rand16(rng, (outer - 1) * ai + size), rand16(rng, (outer - 1) * bi + size)
        c0 = rand16(rng, (outer - 1) * (ai + bi) + size)
        assert_same(port.vectorop(a, b, size, op, outer, ai, bi, c=c0.copy()),
                    R.vectorop(a, b, size, op, outer, ai, bi, c=c0.copy()), "vectorop fuzz")
    # matmul
    for _ in range(4):
        n, k, m, batch = (int(rng.integers(1, 40)), int(rng.integers(1, 300)), int(rng.integers(1, 40)),
                          int(rng.integers(1, 4)))
        a, b = rand16(rng, batch * n * k), rand16(rng, batch * k * m)
        assert_same(port.matmul(a, b, n, k, m, batch), R.matmul(a, b, n, k, m, batch), "matmul fuzz")
    # conv
    for _ in range(4):
        N, C, H, W, M = (int(rng.integers(1, 3)), int(rng.integers(1, 20)), int(rng.integers(3, 12)),
                         int(rng.integers(3, 12)), int(rng.integers(1, 12)))
        kh, kw = int(rng.integers(1, 5)), int(rng.integers(1, 5))
        sh, sw, dh, dw = (int(rng.integers(1, 3)) for _ in range(4))
        pt, pl = int(rng.integers(0, 3)), int(rng.integers(0, 3))
        dwm = int(rng.random() < 0.25)
        if dwm:
            M = C
        oh = (H + 2 * pt - dh * (kh - 1) - 1) // sh + 1
        ow = (W + 2 * pl - dw * (kw - 1) - 1) // sw + 1
        if oh < 1 or ow < 1:
            continue
        x, w, bias = rand16(rng, N * C * H * W), rand16(rng, M * (1 if dwm else C) * kh * kw), rand16(rng, M)
        args = (N, C, H, W, M, oh, ow, kh, kw, sh, sw, dh, dw, pt, pl, 1, dwm)
        assert_same(port.conv(x, w, bias, *args), R.conv(x, w, bias, *args), "conv fuzz")
    # pool
    for _ in range(6):
        N, C, H, W = int(rng.integers(1, 3)), int(rng.integers(1, 12)), int(rng.integers(1, 14)), int(rng.integers(1, 14))
        ph, pw = int(rng.integers(1, min(H, 7) + 1)), int(rng.integers(1, min(W, 7) + 1))
        sh, sw, dh, dw = (int(rng.integers(1, 3)) for _ in range(4))
        pt, pl = int(rng.integers(0, ph)), int(rng.integers(0, pw))
        oh = (H + 2 * pt - dh * (ph - 1) - 1) // sh + 1
        ow = (W + 2 * pl - dw * (pw - 1) - 1) // sw + 1
        if oh < 1 or ow < 1:
            continue
        t, lp, cip = int(rng.integers(0, 4)), int(rng.integers(0, 3)), int(rng.integers(0, 2))
        x = rand16(rng, N * C * H * W)
        args = (N, C, H, W, oh, ow, ph, pw, sh, sw, pt, pl, dh, dw, t, lp, cip)
        assert_same(port.pool(x, *args), R.pool(x, *args), f"pool fuzz {args}")


def test_fast_matmul_matches_port(port):
    rng = np.random.default_rng(8)
    for (n, k, m) in [(17, 300, 9), (5, 4096, 7), (64, 64, 64)]:
        a, b = rand16(rng, n * k), rand16(rng, k * m)
        assert_same(fast.matmul_2d(a.reshape(n, k), b.reshape(k, m)), port.matmul(a, b, n, k, m), "fast")


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built")
@pytest.mark.parametrize("c_bs", [0, 7, 15000, 29999])
def test_overlapping_batch_outputs_follow_batch_order(port, c_bs):
    """c_batch_stride < n*m: output slices of different batch steps overlap and the
    reference's batch loop lets later steps win; the threaded restatement must keep that
    order (sizes large enough that the work is split across threads)."""
    n, k, m, batch = 200, 300, 150, 3
    rng = np.random.default_rng(c_bs)
    a = rng.integers(-32768, 32768, batch * n * k).astype(np.int16)
    b = rng.integers(-32768, 32768, batch * k * m).astype(np.int16)
    init = np.full((batch - 1) * c_bs + n * m, -23131, np.int16)
    got = port.matmul(a, b, n, k, m, batch, n * k, k * m, c_bs, c=init.copy())
    want = oracle.ref().matmul(a, b, n, k, m, batch, n * k, k * m, c_bs, c=init.copy())
    assert np.array_equal(got, want)
