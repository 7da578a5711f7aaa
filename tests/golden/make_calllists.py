"""Golden call lists from the reference's own inference scheduler (test infrastructure).

    python tests/golden/make_calllists.py [--reference <path of the reference tree>]

Needs the reference tree (the location comes from --reference, else CM_REFERENCE_TREE,
else BASELINE.json's reference_path); the fixtures it writes are what the tests read,
here and on machines without the reference.

Every graph of scheduler_graphs.py is handed to the reference scheduler's unmodified
code (inference-scheduler/src: OnnxGraph, the node classes, CodeGenerator) as an
in-memory model.  The `onnx` package is not installed here, so a stand-in module is
put in its place: onnx.load returns the model objects built below, checker.check_model
accepts them, shape_inference.infer_shapes returns them as they are (their value_info
already carries every intermediate shape, computed by cormorant_b200.scheduler's
shape rules), and helper / numpy_helper build and read the same plain objects.  For
every scheduled node the text of the reference's emit_call(layouts) is parsed into
(kernel, buffer names, scalar arguments), with the broadcast CHUNK / CHUNK_STRIDE
macros given the values generate_header() defines for them; buffer allocations and layouts
(numel, alloc, n_chunks, chunk, stride) are CodeGenerator's.  Graphs the reference refuses record its SchedulerError.

For LeNet-5 (batch 1 and 3) the reference's weights/<name>.dat files of the weights
above its 4096-word threshold (generate_weight_dat) and the expected output words of
its generated test for the ramp input (_simulate + _expected_storage, alignment gaps
included) are written to refproj_lenet5/.

Outputs: tests/golden/calllists.json, tests/golden/refproj_lenet5/.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from cormorant_b200.scheduler import infer_shapes  # noqa: E402
from tests.golden.scheduler_graphs import ERROR_GRAPHS, GRAPHS  # noqa: E402

FLOAT, INT64 = 1, 7


# ---- plain stand-ins for the ONNX protobuf objects the reference reads ----------
class _Dim:
    def __init__(self, v):
        self.dim_value = int(v)

    def HasField(self, f):
        return f == "dim_value"


class _Obj:
    def __init__(self, **kw):
        self.__dict__.update(kw)

    def HasField(self, f):
        return getattr(self, f, None) is not None


def _vi(name, elem_type, shape):
    return _Obj(name=name, type=_Obj(tensor_type=_Obj(elem_type=elem_type,
                                                      shape=_Obj(dim=[_Dim(d) for d in shape]))))


def _attr(name, v):
    a = _Obj(name=name, i=0, f=0.0, ints=[], s=b"")
    if isinstance(v, str):
        a.s = v.encode()
    elif isinstance(v, float):
        a.f = v
    elif isinstance(v, (list, tuple)):
        a.ints = [int(x) for x in v]
    else:
        a.i = int(v)
    return a


def _node(op_type, inputs, outputs, name="", attrs=None):
    return _Obj(op_type=op_type, input=list(inputs), output=list(outputs), name=name,
                attribute=[_attr(k, v) for k, v in (attrs or {}).items()])


_MODELS: dict = {}


def _stub_onnx():
    onnx = types.ModuleType("onnx")
    onnx.NodeProto = onnx.ModelProto = onnx.TypeProto = onnx.ValueInfoProto = _Obj
    onnx.TensorProto = types.SimpleNamespace(FLOAT=1, UINT8=2, INT8=3, UINT16=4, INT16=5, INT32=6, INT64=7,
                                             BOOL=9, FLOAT16=10, DOUBLE=11, UINT32=12, UINT64=13)
    onnx.load = lambda path: _MODELS[str(path)]
    onnx.checker = types.SimpleNamespace(check_model=lambda m: None)
    onnx.shape_inference = types.SimpleNamespace(infer_shapes=lambda m: m)
    helper = types.ModuleType("onnx.helper")
    helper.make_node = lambda op, inputs, outputs, name="", **kw: _node(op, inputs, outputs, name, kw)
    helper.make_tensor_value_info = lambda name, et, shape: _vi(name, et, shape)
    helper.make_graph = lambda nodes, name, inputs, outputs, initializer=(), value_info=(): _Obj(
        node=list(nodes), name=name, input=list(inputs), output=list(outputs), initializer=list(initializer),
        value_info=list(value_info))
    helper.make_model = lambda graph, opset_imports=(), **kw: _Obj(graph=graph, opset_import=list(opset_imports),
                                                                   ir_version=8)
    nph = types.ModuleType("onnx.numpy_helper")
    nph.to_array = lambda init: init.array
    onnx.helper, onnx.numpy_helper = helper, nph
    sys.modules.update({"onnx": onnx, "onnx.helper": helper, "onnx.numpy_helper": nph,
                        "onnx.shape_inference": onnx.shape_inference, "onnx.checker": onnx.checker})


def _model(g):
    """The scheduler.Graph as the reference's ONNX model objects: constants become float
    initializers (raw / 256; int64 shape tensors as they are), every operator output that
    is not the graph output gets a value_info entry with its inferred shape."""
    infer_shapes(g)
    T = g.tensors
    consts = [t for t in T.values() if t.is_const]
    inits = []
    for t in consts:
        if t.data.dtype == np.int64:
            inits.append(_Obj(name=t.name, data_type=INT64, array=t.data.reshape(t.shape)))
        else:
            inits.append(_Obj(name=t.name, data_type=FLOAT,
                              array=(t.data.astype(np.float32) / 256.0).reshape(t.shape)))
    produced = [o for op in g.ops for o in op.outputs]
    vis = [_vi(n, FLOAT, T[n].shape) for n in produced if n not in g.outputs]
    nodes = [_node(op.op_type, op.inputs, op.outputs, op.name, op.attrs) for op in g.ops]
    graph = _Obj(node=nodes, name=g.name, input=[_vi(n, FLOAT, T[n].shape) for n in g.inputs],
                 output=[_vi(n, FLOAT, T[n].shape) for n in g.outputs], initializer=inits, value_info=vis)
    return _Obj(graph=graph, opset_import=[], ir_version=8)


# ---- the reference's emitted calls, parsed ------------------------------------
_CALL = re.compile(r"(run_\w+)\((.*?)\);", re.S)
_LOOP = re.compile(r"for \(unsigned _i = 0u; _i < (\d+)u; _i\+\+\)")


def _calls_of(gen, src_pkg):
    nodes_mod = src_pkg.nodes
    op_codes = {v: k for k, v in nodes_mod.OP_NAMES.items()}
    c2onnx, macros = {}, {}
    graph = gen._graph
    for sn in graph.nodes:
        for t in sn.inputs + [sn.output]:
            c2onnx[t.c_name] = t.onnx_name
        if sn.outer_count > 1 and not isinstance(sn, (nodes_mod.MatmulNode, nodes_mod.ReshapeNode)):
            c_up = sn.output.c_name.upper()
            macros[f"INFERENCE_{c_up}_CHUNK"] = sn.chunk_size
            macros[f"INFERENCE_{c_up}_CHUNK_STRIDE"] = sn.aligned_chunk_size

    def value(tok, i):
        tok = tok.strip()
        if tok == "NULL":
            return None
        if tok in c2onnx:
            return c2onnx[tok]
        if tok in macros:
            return macros[tok]
        if tok in op_codes:
            return op_codes[tok]
        m = re.fullmatch(r"_i \* (\d+)u", tok)
        if m:
            return i * int(m.group(1))
        m = re.fullmatch(r"(\d+)u?", tok)
        if m:
            return int(m.group(1))
        raise ValueError(f"cannot read argument {tok!r}")

    out = []
    for sn in graph.nodes:
        text = sn.emit_call(gen._layouts)
        if not text.strip():
            continue
        loop = _LOOP.search(text)
        reps = int(loop.group(1)) if loop else 1
        for i in range(reps):
            for fn, body in _CALL.findall(text):
                v = [value(t, i) for t in body.split(",")]
                if fn == "run_op":
                    out.append(["vectorop", v[:3], v[3:]])
                elif fn == "run_matmul":
                    out.append(["matmul", v[:3], v[3:]])
                elif fn == "run_matmul_at":
                    out.append(["matmul_at", [v[0], v[2], v[4]], [v[1], v[3], v[5]] + v[6:]])
                elif fn == "run_conv":
                    out.append(["conv", v[:4], v[4:]])
                elif fn == "run_pool":
                    out.append(["pool", v[:2], v[2:]])
                else:
                    raise ValueError(fn)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args()
    ref = args.reference or os.environ.get("CM_REFERENCE_TREE")
    if not ref:
        ref = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
    sched = Path(ref) / "inference-scheduler"
    if not (sched / "src" / "nodes.py").is_file():
        sys.exit(f"reference scheduler not found under {sched}")
    _stub_onnx()
    sys.path.insert(0, str(sched))
    import src                       # the reference scheduler package (inference-scheduler/src)
    import src.codegen
    import src.graph
    import src.nodes  # noqa: F401

    result = {"generator": "tests/golden/make_calllists.py", "graphs": {}, "errors": {}}
    tmp = Path(tempfile.mkdtemp())
    refproj = HERE / "refproj_lenet5"
    for name, build in list(GRAPHS.items()) + list(ERROR_GRAPHS.items()):
        path = tmp / f"{name}.onnx"
        path.write_bytes(b"")
        _MODELS[str(path)] = _model(build())
        try:
            og = src.graph.OnnxGraph(str(path))
            gen = src.codegen.CodeGenerator(og, str(path))
        except src.nodes.SchedulerError as e:
            result["errors"][name] = str(e).splitlines()[0]
            print(f"{name}: refused: {str(e).splitlines()[0]}")
            continue
        if name in ERROR_GRAPHS:
            raise SystemExit(f"{name}: the reference accepted a graph listed as refused")
        aliases = {sn.output.onnx_name: sn.inputs[0].onnx_name for sn in og.nodes
                   if isinstance(sn, src.nodes.ReshapeNode)}
        rec = {"calls": _calls_of(gen, src),
               "allocs": {k: v.alloc for k, v in gen._layouts.items()},
               "layouts": {k: [v.numel, v.alloc, v.n_chunks, v.chunk, v.stride] for k, v in gen._layouts.items()},
               "aliases": aliases,
               "input": og.input_tensors[0].onnx_name, "output": og.output_tensors[0].onnx_name}
        result["graphs"][name] = rec
        print(f"{name}: {len(rec['calls'])} calls")
        if name.startswith("lenet5"):
            # the reference's weight files and its generated test's expected words
            wdir = refproj / "weights"
            wdir.mkdir(parents=True, exist_ok=True)
            for t in gen.large_weight_tensors:
                (wdir / f"{t.c_name}.dat").write_bytes(gen.generate_weight_dat(t))
            out_t = og.output_tensors[0]
            words = gen._expected_storage(out_t.onnx_name, gen._simulate()[out_t.onnx_name])
            np.save(refproj / f"expected_{name}.npy", np.asarray(words).view(np.int16))
    (HERE / "calllists.json").write_text(json.dumps(result, indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "calllists.json")


if __name__ == "__main__":
    main()
