"""The generated C project (cormorant_b200.codegen): the reference scheduler's
inference.h / inference.c / test_inference.c layout with libcormorant_cuda.so as the
backend.  CPU tests check the buffer plan, the emitted API and files, and that the
project compiles with -Werror and links; GPU tests compile and run it and compare the
network output for the reference's ramp input with the oracle, word for word (the
reference's own generated GT check, inference-scheduler/src/codegen/_test.py)."""
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

from cormorant_b200 import codegen, networks
from tests.test_networks import OracleBackend, cpu_buffers

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "cormorant_b200" / "libcormorant_cuda.so"
INCLUDE = ROOT / "include"

NETS = {
    "lenet5": lambda: networks.lenet5(),
    "lenet5_b3": lambda: networks.lenet5(batch=3),
    "resnet18_b2": lambda: networks.resnet18(batch=2),
}


MODES = ["plain", "fused", "planes", "prepared"]


def _net(name, mode):
    net = NETS[name]()
    if mode == "plain":
        return net
    net = networks.fuse(net)
    return networks.chain(net) if mode in ("planes", "prepared") else net


def _nchw_outputs(net):
    outs = set()
    for n in net.nodes:
        if n[0] in ("planes", "poolp", "poolnp"):
            continue
        if n[0] == "conv":
            if n[4] is not None:
                outs.add(net.resolve(n[4]))
        else:
            outs.add(net.resolve(codegen._output(n)))
    return outs


def _expected(net, port):
    bufs = cpu_buffers(net, codegen.ramp_input(net))
    networks.execute(net, OracleBackend(port), bufs)
    return bufs[net.resolve(net.output)].copy()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", list(NETS))
def test_layout_never_overlaps_live_tensors(name, mode):
    """Two intermediates that are live at the same node never share a word of the pool."""
    net = _net(name, mode)
    L = codegen.plan_layout(net)
    io = {net.resolve(net.input), net.resolve(net.output)}
    inter = _nchw_outputs(net) - io
    assert set(L.acts) == inter
    items = list(L.acts.items())
    for name_a, (oa, wa) in items:
        assert oa % codegen.ALIGN_WORDS == 0 and oa + wa <= L.act_words
        fa, la = L.live[name_a]
        for name_b, (ob, wb) in items:
            if name_a >= name_b:
                continue
            fb, lb = L.live[name_b]
            if fa <= lb and fb <= la:           # live ranges meet
                assert oa + wa <= ob or ob + wb <= oa, (name_a, name_b)
    # weights: back to back, aligned, disjoint
    spans = sorted(L.weights.values())
    for (o1, w1), (o2, _) in zip(spans, spans[1:]):
        assert o1 % codegen.ALIGN_WORDS == 0 and o1 + w1 <= o2
    assert L.act_words <= sum(codegen._align(net.buffers[n]) for n in L.acts)


def test_layout_reuses_memory_on_resnet():
    net = networks.fuse(networks.resnet18(batch=2))
    L = codegen.plan_layout(net)
    total = sum(net.buffers[n] for n in L.acts)
    assert L.act_words < total / 2


def test_emitted_api_and_weight_files(tmp_path):
    net = networks.fuse(networks.lenet5())
    out = net.resolve(net.output)
    exp = np.arange(10, dtype=np.int16)
    files = codegen.emit_project(net, tmp_path, expected=exp)
    h = (tmp_path / "include/inference.h").read_text()
    for sym in ("typedef int16_t Data_t;", "INFERENCE_BYTES_PER_ELEM  2u", "inference_buf_alloc(unsigned n_elem)",
                "inference_buf_init_view(", "inference_buf_sync_to_device(", "inference_buf_fill_float(",
                "INFERENCE_BUF_POOL_SIZE_BYTES", "int  inference_init(const char *vectoropkernel_instance,",
                "const char *matmulkernel_instance", "const char *convkernel_instance",
                "const char *poolingkernel_instance", "void inference_deinit(void);",
                f"int inference_run(inference_buf_t *in_x, inference_buf_t *out_{out});",
                "#define INFERENCE_X_SIZE  784u", f"#define INFERENCE_{out.upper()}_SIZE  10u"):
        assert sym in h, sym
    src = (tmp_path / "src/inference.c").read_text()
    assert src.count("cm_conv_pool_async(") == 2              # Conv+Relu+MaxPool twice, one launch each
    assert src.count("cm_matmul_fused_async(") == 3 and src.count("cm_pool_async(") == 0   # Gemm(+Relu) x 3
    assert "cm_vectorop_async(" not in src
    assert src.count("CHECK(cm_synchronize(NULL));") == 1
    # weights above the threshold go to .dat files (raw little-endian words), the rest inline
    for name, arr in net.consts.items():
        dat = tmp_path / "weights" / f"{name}.dat"
        if arr.size > codegen.LARGE_WEIGHT_THRESHOLD:
            assert dat.read_bytes() == np.asarray(arr, "<i2").tobytes()
            assert f'_load_weight(&w_{name}, "{name}")' in src
        else:
            assert not dat.exists() and f"static const Data_t {name}_init[{arr.size}]" in src
    assert "test/test_inference.c" in files and "expected" not in " ".join(files)


def test_large_expected_goes_to_dat(tmp_path):
    net = networks.fuse(networks.resnet18(batch=5))
    exp = np.arange(5000, dtype=np.int16)
    codegen.emit_project(net, tmp_path, expected=exp)
    out = net.resolve(net.output)
    assert (tmp_path / "expected" / f"{out}.dat").read_bytes() == exp.astype("<i2").tobytes()
    t = (tmp_path / "test/test_inference.c").read_text()
    assert f'_load_expected(&exp_heap, "{out}"' in t
    with pytest.raises(ValueError):
        codegen.emit_project(net, tmp_path / "bad", expected=exp[:10])


def test_ramp_input_matches_reference_fill():
    net = networks.lenet5(batch=100)                       # 78400 words: wraps past 0xFFFF
    r = codegen.ramp_input(net)
    assert r.dtype == np.int16 and r.size == 78400
    assert r[0] == 0 and r[255] == 255 and r[32768] == -32768 and r[65535] == -1 and r[65536] == 0


@pytest.mark.skipif(not LIB.exists(), reason="libcormorant_cuda.so not built")
@pytest.mark.parametrize("mode", MODES)
def test_project_compiles_and_fails_cleanly_without_gpu(tmp_path, mode):
    """gcc -Wall -Wextra -Werror over the generated sources, linked against the library;
    with no GPU visible inference_init reports the failure and the test binary exits 1."""
    net = _net("resnet18_b2", mode)
    codegen.emit_project(net, tmp_path, expected=np.zeros(2000, np.int16), prepared=mode == "prepared")
    exe = codegen.compile_project(tmp_path, INCLUDE, LIB)
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible: the run itself is covered by the gpu tests")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    assert "inference_init" in r.stderr and "cm_init" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", list(NETS))
def test_generated_project_bit_exact_on_gpu(tmp_path, port, name, mode):
    net = _net(name, mode)
    exp = _expected(net, port)
    codegen.emit_project(net, tmp_path, expected=exp, prepared=mode == "prepared")
    exe = codegen.compile_project(tmp_path, INCLUDE, LIB)
    r = subprocess.run([str(exe), "20"], capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "test_inference PASSED" in r.stdout and "timing: 20 runs" in r.stdout


@pytest.mark.gpu
def test_generated_project_reports_missing_weights_and_mismatch(tmp_path, port):
    net = networks.fuse(networks.lenet5())
    exp = _expected(net, port)
    exp_bad = exp.copy()
    exp_bad[3] ^= 1
    codegen.emit_project(net, tmp_path, expected=exp_bad)
    exe = codegen.compile_project(tmp_path, INCLUDE, LIB)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "test_inference FAILED (1 mismatches)" in r.stdout
    out = net.resolve(net.output)
    assert f"GT MISMATCH {out}[3]" in r.stderr
    big = next(n for n, a in net.consts.items() if a.size > codegen.LARGE_WEIGHT_THRESHOLD)
    os.remove(tmp_path / "weights" / f"{big}.dat")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "cannot open weight file" in r.stderr


def test_chained_project_uses_plane_images(tmp_path):
    """The stem writes channels-last for the max pool, which writes the layer-1 convs'
    plane image (cm_pool_nhwc_planes_async): no split pass remains."""
    net = _net("resnet18_b2", "planes")
    codegen.emit_project(net, tmp_path, expected=np.zeros(2000, np.int16))
    src = (tmp_path / "src/inference.c").read_text()
    assert src.count("cm_planes_create(") == len(net.planes) == src.count("cm_planes_destroy(")
    assert src.count("cm_conv_planes_async(") == 20 and src.count("cm_planes_fill_async(") == 0
    assert src.count("cm_pool_nhwc_planes_async(") == 1
    assert src.count("cm_pool_nhwc_async(") == 1                     # the global pool after the last block
    if LIB.exists():
        codegen.compile_project(tmp_path, INCLUDE, LIB)


@pytest.mark.skipif(not LIB.exists(), reason="libcormorant_cuda.so not built")
def test_plane_pool_project_compiles(tmp_path):
    net = networks.chain(networks.fuse(networks.resnet18(batch=2)), pool_planes=True, pool_nhwc=False)
    codegen.emit_project(net, tmp_path, expected=np.zeros(2000, np.int16))
    assert (tmp_path / "src/inference.c").read_text().count("cm_pool_planes_async(") == 1
    codegen.compile_project(tmp_path, INCLUDE, LIB)


def test_prepared_project_builds_weights_once(tmp_path):
    """prepared=True: inference_init creates one cm_conv_weights_t per conv and one
    cm_matmul_weights_t for the classifier Gemm (after the weight pool reaches the device),
    inference_run calls cm_conv_prepared_async / cm_matmul_prepared_async for them,
    inference_deinit destroys them."""
    net = _net("resnet18_b2", "prepared")
    codegen.emit_project(net, tmp_path, expected=np.zeros(2000, np.int16), prepared=True)
    src = (tmp_path / "src/inference.c").read_text()
    nconv = sum(1 for n in net.nodes if n[0] == "conv")
    assert src.count("cm_conv_weights_create(") == nconv == src.count("cm_conv_prepared_async(")
    assert src.count("cm_conv_weights_destroy(") == nconv
    assert "cm_conv_planes_async(" not in src and "cm_conv_fused_async(" not in src
    assert src.index("cm_buf_sync_to_device(g_wpool)") < src.index("cm_conv_weights_create(")
    # the classifier Gemm's B: prepared once as well
    assert src.count("cm_matmul_weights_create(") == 1 == src.count("cm_matmul_prepared_async(")
    assert src.count("cm_matmul_weights_destroy(") == 1
    assert "cm_matmul_fused_async(" not in src
    assert src.index("cm_buf_sync_to_device(g_wpool)") < src.index("cm_matmul_weights_create(")


# ---- the reference scheduler's own files (tests/golden/make_calllists.py) ----------
REFPROJ = ROOT / "tests" / "golden" / "refproj_lenet5"


@pytest.mark.parametrize("batch", [1, 3])
def test_weight_files_equal_the_reference_scheduler(tmp_path, batch):
    """weights/*.dat of the generated project are byte for byte the files the reference
    scheduler writes for the same network (CodeGenerator.generate_weight_dat)."""
    codegen.emit_project(networks.lenet5(batch), tmp_path)
    ref = sorted((REFPROJ / "weights").glob("*.dat"))
    ours = sorted((tmp_path / "weights").glob("*.dat"))
    assert ref and [p.name for p in ours] == [p.name for p in ref]
    for a, b in zip(ours, ref):
        assert a.read_bytes() == b.read_bytes(), a.name


@pytest.mark.parametrize("batch", [1, 3])
def test_reference_expected_output_equals_the_oracle(port, batch):
    """The expected words of the reference's generated test (its fixed-point simulator on
    the ramp input, alignment gaps as zeros) equal the oracle's run of the derived call list."""
    net = networks.lenet5(batch)
    want = np.load(REFPROJ / f"expected_lenet5_b{batch}.npy")
    got = _expected(net, port)
    assert np.array_equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["plain", "fused"])
@pytest.mark.parametrize("batch", [1, 3])
def test_reference_files_run_unchanged_on_gpu(tmp_path, batch, mode):
    """The reference scheduler's weights/*.dat and its expected output words drive the
    generated CUDA project unchanged: our weight files are replaced by the reference's and
    the test binary compares the network output with the reference's expected words."""
    net = networks.lenet5(batch)
    if mode == "fused":
        net = networks.fuse(net)
    want = np.load(REFPROJ / f"expected_lenet5_b{batch}.npy")
    codegen.emit_project(net, tmp_path, expected=want)
    for f in (REFPROJ / "weights").glob("*.dat"):
        (tmp_path / "weights" / f.name).write_bytes(f.read_bytes())
    exe = codegen.compile_project(tmp_path, INCLUDE, LIB)
    r = subprocess.run([str(exe), "3"], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "test_inference PASSED" in r.stdout


def _net_from_reference_list(name):
    """A Net whose calls, buffer sizes and constant layouts are the reference scheduler's own
    (calllists.json), with the graph's constant words placed in those layouts; nothing comes
    from scheduler.derive."""
    import json
    from cormorant_b200.networks import Net
    from cormorant_b200.scheduler import Layout, _const_words, infer_shapes
    from tests.golden.scheduler_graphs import GRAPHS
    ref = json.loads((ROOT / "tests" / "golden" / "calllists.json").read_text())["graphs"][name]
    g = GRAPHS[name]()
    infer_shapes(g)
    net = Net(name + "+reference-list", int(g.tensors[ref["input"]].shape[0]), ref["input"], ref["output"])
    net.aliases = dict(ref["aliases"])
    for t, lay in ref["layouts"].items():
        if t in net.aliases:
            continue
        if t in g.tensors and g.tensors[t].is_const:
            net.consts[t] = _const_words(g.tensors[t], Layout(*lay))
        else:
            net.buffers[t] = lay[1]
    kinds = {"vectorop": 3, "matmul": 3, "matmul_at": 3, "conv": 4, "pool": 2}
    for kind, names, args in ref["calls"]:
        net.nodes.append((kind, *names[:kinds[kind]], tuple(args)))
    return net


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["lenet5_b3", "matmul_gapped", "matmul_outer", "broadcast_aligned"])
def test_project_from_the_reference_node_list_on_gpu(tmp_path, port, name):
    """The reference scheduler's own call list (not scheduler.derive's) emitted as a CUDA
    project, compiled and run: output equal to the oracle's run of the same list."""
    net = _net_from_reference_list(name)
    exp = _expected(net, port)
    codegen.emit_project(net, tmp_path, expected=exp)
    exe = codegen.compile_project(tmp_path, INCLUDE, LIB)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, cwd=tmp_path)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "test_inference PASSED" in r.stdout
