"""cormorant_b200.scheduler against the reference scheduler's own derivation.

tests/golden/calllists.json holds, for every graph of tests/golden/scheduler_graphs.py,
the calls the reference's unmodified scheduler code emits (inference-scheduler/src:
OnnxGraph, the node classes' emit_call, CodeGenerator's layouts), parsed into
(kernel, buffers, scalars), and the buffer allocations; written by
tests/golden/make_calllists.py.  Every call and every allocation must be equal, and
graphs the reference refuses must be refused here too.  The two BASELINE networks
(LeNet-5 at batch 1 and 3, the ResNet-18 shape at batch 2) are among the graphs, so the
call lists the bench, the GPU tests and the code generator run are the reference's.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from cormorant_b200 import networks, scheduler
from tests.golden.scheduler_graphs import ERROR_GRAPHS, GRAPHS

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "calllists.json").read_text())


def _as_calls(net):
    out = []
    for node in net.nodes:
        kind = node[0]
        if kind == "conv":
            names, args = list(node[1:5]), node[5]
        elif kind == "pool":
            names, args = list(node[1:3]), node[3]
        else:
            names, args = list(node[1:4]), node[4]
        out.append([kind, names, [int(v) for v in args]])
    return out


def test_every_graph_has_a_fixture():
    assert set(GOLDEN["graphs"]) == set(GRAPHS)
    assert set(GOLDEN["errors"]) == set(ERROR_GRAPHS)


@pytest.mark.parametrize("name", sorted(GRAPHS))
def test_calls_equal_the_reference_scheduler(name):
    want = GOLDEN["graphs"][name]
    net = scheduler.derive(GRAPHS[name]())
    got = _as_calls(net)
    assert len(got) == len(want["calls"])
    for i, (g, w) in enumerate(zip(got, want["calls"])):
        assert g == w, f"{name} call {i}: {g} != reference {w}"
    assert net.aliases == want["aliases"]
    assert net.input == want["input"] and net.output == want["output"]


@pytest.mark.parametrize("name", sorted(GRAPHS))
def test_allocations_equal_the_reference_layouts(name):
    want = GOLDEN["graphs"][name]["allocs"]
    net = scheduler.derive(GRAPHS[name]())
    got = {k: L.alloc for k, L in net.layouts.items()}
    assert got == want
    layouts = GOLDEN["graphs"][name]["layouts"]
    assert {k: [L.numel, L.alloc, L.n_chunks, L.chunk, L.stride] for k, L in net.layouts.items()} == layouts
    # buffers and constants are sized by those allocations
    for k, words in net.buffers.items():
        assert words == want[k]
    for k, arr in net.consts.items():
        assert arr.size == max(want[k], 1)


@pytest.mark.parametrize("name", sorted(ERROR_GRAPHS))
def test_refused_graphs_are_refused(name):
    with pytest.raises(scheduler.SchedulerError):
        scheduler.derive(ERROR_GRAPHS[name]())


def test_networks_are_the_derived_lists():
    """networks.lenet5 / resnet18 are scheduler.derive of their graphs (the bench's lists)."""
    for net, name in ((networks.lenet5(1), "lenet5_b1"), (networks.lenet5(3), "lenet5_b3"),
                      (networks.resnet18(2), "resnet18_b2")):
        assert _as_calls(net) == GOLDEN["graphs"][name]["calls"]


def test_strided_constants_hold_zero_gaps():
    """A constant raised to a strided layout keeps its data in the chunks, zeros in the gaps
    (the reference's strided ROM arrays, tensor.py emit_weight_decl_strided)."""
    g = GRAPHS["broadcast"]()
    net = scheduler.derive(g)
    name = next(op.inputs[1] for op in g.ops if op.op_type == "Mul")   # the [2, 5, 6] co-input
    L = net.layouts[name]
    assert L.n_chunks == 10 and L.stride == 8 and L.chunk == 6
    words = net.consts[name].reshape(10, 8)
    assert (words[:, 6:] == 0).all()
    assert np.array_equal(words[:, :6].reshape(-1), g.tensors[name].data)


def test_gemm_bias_fuses_in_every_derived_form():
    """The Gemm decomposition's MatMul -> Add(bias) [-> Relu] folds into one fused MatMul in
    the forms the scheduler emits: a whole-tensor Add at one row, the bias row broadcast
    over n rows, and the row-strided form over gapped rows."""
    for batch in (1, 3):
        f = networks.fuse(networks.lenet5(batch), conv_pool_macs=0)
        assert [n[0] for n in f.nodes] == ["conv", "pool", "conv", "pool", "matmul", "matmul", "matmul"]
        assert [n[5] for n in f.nodes[4:]] == [3, 3, 2]
    f = networks.fuse(networks.lenet5(3), conv_pool_macs=0)
    assert f.nodes[5][4] == (1, 120, 84, 3, 120, 0, 88)    # row-strided, rows 88 words apart
