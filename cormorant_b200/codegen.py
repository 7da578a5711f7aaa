"""CUDA backend of the inference-scheduler code generator.

The reference's scheduler turns an ONNX graph into a small C project: include/inference.h
(the inference_buf_* / inference_init / inference_run API), src/inference.c (one buffer
pool, weight arrays, run_op / run_matmul / run_conv / run_pool helpers that program the
FPGA kernels over AXI-Lite and poll IsDone), CMakeLists.txt, weights/<name>.dat and
test/test_inference.c with a bit-exact ground-truth check
(inference-scheduler/src/codegen/_header.py, _source.py, _buf_impl.py, _cmake.py, _test.py).

`emit_project` writes the same project for a kernel-call list (`networks.Net`) with
libcormorant_cuda.so as the backend:

* inference.h keeps the reference API: Data_t, INFERENCE_BYTES_PER_ELEM, the
  INFERENCE_<NAME>_SIZE macros, INFERENCE_BUF_POOL_SIZE_BYTES, inference_buf_* (thin
  inline wrappers of cm_buf_*: a device allocation plus a pinned host mirror, "phys"
  becoming the device address), one INFERENCE_<KERNEL>_INSTANCE macro and one
  inference_init() parameter per kernel the network uses (_header.py:280-318), then
  inference_deinit() and inference_run(inputs..., outputs...) (_header.py:320-352).
  inference_run returns 0 or a CM_E* status instead of void; callers that ignore it
  compile unchanged.
* inference.c: every run_* helper becomes one cm_*_async call on the legacy default
  stream (the reference's Start + busy-wait pairs, _source.py:175-420, become a queue of
  launches with ONE cm_synchronize at the end of inference_run).  Conv -> Relu and
  Conv -> Add(-> Relu) chains of a fused call list become cm_conv_fused_async.
* Buffers: weights live in one owner buffer, synced to the device once by
  inference_init; intermediates live in a second owner buffer laid out by liveness
  (address-ordered first fit: a tensor takes the lowest free range that no tensor live at
  the same time holds).  The caller's input and output buffers are handed to the kernels
  directly, as the reference's output-alias redirect does (_source.py:735-770).
* Weights of more than LARGE_WEIGHT_THRESHOLD words are read at init from
  INFERENCE_WEIGHTS_DIR "/weights/<name>.dat" (raw little-endian words,
  _source.py:426-470); smaller ones are static arrays in inference.c
  (inference-scheduler/src/tensor.py:35 sets the threshold).
* test/test_inference.c fills each input with the reference's ramp
  (word i = i & 0xFFFF, dtype.py:307-310), runs, and compares every output word with the
  expected words (embedded up to LARGE_EXPECTED_THRESHOLD words, else read from
  expected/<name>.dat, _test.py:63-135, _simulate.py:190), printing
  "test_inference PASSED" / "FAILED".  An optional first argument N times N further
  inference_run calls (host clock, inputs and outputs crossing PCIe each call).

The expected words are an argument: this module computes nothing itself.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .networks import Net, _inputs, output_of as _output

LARGE_WEIGHT_THRESHOLD = 4096          # inference-scheduler/src/tensor.py:35
LARGE_EXPECTED_THRESHOLD = 4096        # inference-scheduler/src/codegen/_simulate.py:190
ALIGN_WORDS = 128                      # 256-byte slots: whole 32-byte sectors, 16-byte TMA bases

KERNELS = (                            # (node kind, kernel name, init parameter)
    ("vectorop", "VectorOPKernel", "vectoropkernel_instance"),
    ("matmul", "MatmulKernel", "matmulkernel_instance"),
    ("conv", "ConvKernel", "convkernel_instance"),
    ("pool", "PoolingKernel", "poolingkernel_instance"),
)
_OP_NAMES = {0: "ADD", 1: "SUB", 2: "MUL", 3: "DIV", 4: "RELU", 5: "RELU6"}


def _align(n: int) -> int:
    return (n + ALIGN_WORDS - 1) // ALIGN_WORDS * ALIGN_WORDS


@dataclass
class Layout:
    """Where every buffer of a network lives in the generated program."""
    weights: dict          # name -> (offset, words) in the weight pool
    weight_words: int
    acts: dict             # resolved intermediate name -> (offset, words) in the activation pool
    act_words: int
    live: dict             # resolved intermediate name -> (first node, last node)


def plan_layout(net: Net) -> Layout:
    """Weights back to back; intermediates packed by liveness with address-ordered first fit."""
    R = net.resolve
    weights, off = {}, 0
    for name, arr in net.consts.items():
        weights[name] = (off, int(np.asarray(arr).size))
        off += _align(max(int(np.asarray(arr).size), 1))
    weight_words = off

    io = {R(net.input), R(net.output)}
    live: dict = {}
    for i, node in enumerate(net.nodes):
        y = R(_output(node))
        if node[0] == "conv" and node[4] is not None:
            y = R(node[4])                   # the NCHW output (a plane image output is separate)
        if y not in io and y not in net.consts and y not in net.planes:
            first, last = live.get(y, (i, i))
            live[y] = (min(first, i), max(last, i))
        for name in _inputs(node):
            r = R(name)
            if r in live:
                live[r] = (live[r][0], max(live[r][1], i))

    acts: dict = {}
    held: list = []                          # [(offset, words, last node)] sorted by offset
    top = 0
    for i, node in enumerate(net.nodes):
        y = R(_output(node))
        if node[0] == "conv" and node[4] is not None:
            y = R(node[4])
        if y in live and y not in acts and live[y][0] == i:
            words = _align(max(net.buffers[y], 1))
            pos, placed = 0, None
            for o, w, _ in held:
                if o - pos >= words:
                    placed = pos
                    break
                pos = max(pos, o + w)
            if placed is None:
                placed = pos
            acts[y] = (placed, net.buffers[y])
            held.append((placed, words, live[y][1]))
            held.sort()
            top = max(top, placed + words)
        held = [h for h in held if h[2] > i]
    return Layout(weights, weight_words, acts, top, live)


def _c_words(arr: np.ndarray, indent: str = "    ", per_line: int = 12) -> str:
    words = [f"0x{int(v) & 0xFFFF:04X}" for v in np.asarray(arr, np.int16).reshape(-1)]
    lines = [indent + ", ".join(words[i:i + per_line]) for i in range(0, len(words), per_line)]
    return ",\n".join(lines)


def _dat_bytes(arr: np.ndarray) -> bytes:
    return np.ascontiguousarray(np.asarray(arr, np.int16).reshape(-1)).astype("<i2").tobytes()


_LOAD_WEIGHT = r"""/* Read weights/<name>.dat (raw little-endian words) into the view's host mirror. */
static int _load_weight(inference_buf_t *buf, const char *name)
{
    char path[1024];
    FILE *f;
    size_t got;
    snprintf(path, sizeof path, INFERENCE_WEIGHTS_DIR "/weights/%s.dat", name);
    f = fopen(path, "rb");
    if (!f) {
        fprintf(stderr, "inference_init: cannot open weight file '%s'\n", path);
        return 1;
    }
    got = fread(inference_buf_ptr(buf), INFERENCE_BYTES_PER_ELEM, inference_buf_count(buf), f);
    fclose(f);
    if (got != inference_buf_count(buf)) {
        fprintf(stderr, "inference_init: '%s': got %zu words, expected %u\n", path, got,
                inference_buf_count(buf));
        return 1;
    }
    return 0;
}

"""


class _Emitter:
    def __init__(self, net: Net, lib_path: str | None, prepared: bool = False):
        self.net = net
        # prepared: every conv's weight planes and every Gemm's B planes built once by
        # inference_init (cm_conv_weights_create, cm_matmul_weights_create) and the calls made
        # through cm_conv_prepared_async / cm_matmul_prepared_async
        self.prepared = prepared
        self._conv_index: dict = {}
        self._mm_index: dict = {}
        self.R = net.resolve
        self.layout = plan_layout(net)
        # one init parameter per kernel of the unfused call list, as the reference's
        # generated header has, so the signature does not change with fusion
        kinds = set(net.source_kinds) or {n[0] for n in net.nodes}
        self.kernels = [k for k in KERNELS if k[0] in kinds]
        self.lib_path = lib_path
        self.in_c, self.out_c = self.R(net.input), self.R(net.output)

    # ---- buffer expressions --------------------------------------------------
    @staticmethod
    def _pvar(name: str) -> str:
        return "p_" + "".join(ch if ch.isalnum() or ch == "_" else "_" for ch in name)

    def _planes(self, name: str | None) -> str:
        return "NULL" if name is None else self._pvar(name)

    def _buf(self, name: str | None) -> str:
        if name is None:
            return "NULL"
        r = self.R(name)
        if r == self.in_c:
            return "in_" + r
        if r == self.out_c:
            return "out_" + r
        if r in self.net.consts:
            return "&w_" + r
        return "&t_" + r

    def _dev(self, name: str | None, const: bool = True) -> str:
        if name is None:
            return "NULL"
        return f"{'IN' if const else 'OUT'}({self._buf(name)})"

    # ---- inference.h ---------------------------------------------------------
    def header(self) -> str:
        net, L = self.net, self.layout
        pool_bytes = (L.weight_words + L.act_words) * 2
        pool_bytes = (pool_bytes + 4095) // 4096 * 4096
        in_words, out_words = net.buffers[self.in_c], net.buffers[self.out_c]
        inst = "\n".join(
            f"#ifndef INFERENCE_{k.upper()}_INSTANCE\n#  define INFERENCE_{k.upper()}_INSTANCE  \"0\"\n#endif"
            for _, k, _ in self.kernels)
        params = ",\n                    ".join(f"const char *{p}" for _, _, p in self.kernels)
        return f"""/*
 * inference.h -- generated for network '{net.name}' (batch {net.batch}).
 * Backend: libcormorant_cuda.so (B200, sm_100a); buffers are device allocations with a
 * pinned host mirror.
 */
#pragma once

#ifdef __cplusplus
extern "C" {{
#endif

#include <stdint.h>
#include "cormorant_cuda.h"

/* ---- Data type: ap_fixed<16,8>, raw int16 words, value = raw / 256.0 ---- */
typedef int16_t Data_t;
#define INFERENCE_BYTES_PER_ELEM  2u

/* ---- Array size constants ---- */
#define INFERENCE_{self.in_c.upper()}_SIZE  {in_words}u
#define INFERENCE_{self.out_c.upper()}_SIZE  {out_words}u

/* ---- Device buffer pool: weights ({L.weight_words} words) + intermediates ({L.act_words} words) ---- */
#define INFERENCE_BUF_POOL_SIZE_BYTES  {pool_bytes}u

/* ---- Buffer API: inference_buf_* over cm_buf_* ----
 * An owner is a device allocation plus a pinned host mirror of the same size; a view
 * aliases a slice of an owner.  inference_buf_ptr() is the host mirror,
 * inference_buf_phys() the device address the kernels use.  inference_run() syncs
 * its inputs to the device and its outputs back. */
typedef cm_buf_t inference_buf_t;
static inline inference_buf_t *inference_buf_alloc(unsigned n_elem) {{ return cm_buf_alloc(n_elem); }}
static inline void inference_buf_retain(inference_buf_t *buf) {{ cm_buf_retain(buf); }}
static inline void inference_buf_release(inference_buf_t *buf) {{ cm_buf_release(buf); }}
static inline void inference_buf_free(inference_buf_t *buf) {{ cm_buf_free(buf); }}
static inline Data_t *inference_buf_ptr(inference_buf_t *buf) {{ return cm_buf_ptr(buf); }}
static inline uint64_t inference_buf_phys(const inference_buf_t *buf) {{ return cm_buf_dev(buf); }}
static inline unsigned inference_buf_count(const inference_buf_t *buf) {{ return cm_buf_count(buf); }}
static inline void inference_buf_init_view(inference_buf_t *view, inference_buf_t *base,
                                           unsigned offset_elems, unsigned count_elems)
{{ cm_buf_init_view(view, base, offset_elems, count_elems); }}
static inline void inference_buf_sync_to_device(inference_buf_t *buf) {{ (void)cm_buf_sync_to_device(buf); }}
static inline void inference_buf_sync_from_device(inference_buf_t *buf) {{ (void)cm_buf_sync_from_device(buf); }}
/* Each value cast to Data_t with C's conversion, as the reference does. */
static inline void inference_buf_fill_float(inference_buf_t *buf, const float *src, unsigned n)
{{ Data_t *d = cm_buf_ptr(buf); unsigned i; for (i = 0; i < n; i++) d[i] = (Data_t)src[i]; }}
static inline void inference_buf_read_float(const inference_buf_t *buf, float *dst, unsigned n)
{{ const Data_t *s = (const Data_t *)buf->virt; unsigned i; for (i = 0; i < n; i++) dst[i] = (float)s[i]; }}

/* ---- Kernel instances: the CUDA device ordinal (every kernel runs on the same GPU) ---- */
{inst}

/*
 * inference_init() -- select the GPU, allocate the pools, load the weights.
 * Every instance names the same device ordinal (NULL = same as the first).
 * Returns 0 on success, non-zero on failure.
 */
int  inference_init({params});

/* inference_deinit() -- release the pools and the library. */
void inference_deinit(void);

/*
 * inference_run() -- execute the whole graph.
 *   {('in_' + self.in_c):<22} [in]   inference_buf_t*  ({in_words} elem)
 *   {('out_' + self.out_c):<22} [out]  inference_buf_t*  ({out_words} elem)
 * Returns 0 (CM_OK) or a negative CM_E* status.
 */
int inference_run(inference_buf_t *in_{self.in_c}, inference_buf_t *out_{self.out_c});

#ifdef __cplusplus
}}
#endif
"""

    # ---- inference.c ---------------------------------------------------------
    def _call(self, i: int, node) -> str:
        kind = node[0]
        if kind == "convpool":
            _, x, wn, bn, y, args, epi, resid, pargs = node
            a = ", ".join(f"{int(v)}u" for v in args)
            pa = ", ".join(f"{int(v)}u" for v in pargs)
            what = "Conv" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "") + "+MaxPool"
            return (f"    /* {i}: {what} -> {self.R(y)} (one launch) */\n"
                    f"    CHECK(cm_conv_pool_async({self._dev(x)}, {self._dev(wn)}, {self._dev(bn)}, {self._dev(y, False)},\n"
                    f"        {a}, {int(epi)}u, {self._dev(resid)},\n        {pa}, NULL));")
        if kind == "conv" and self.prepared:
            x, y, resid, xp, yp, rp = node[1], node[4], None, None, None, None
            epi = 0
            if len(node) > 6:
                epi, resid = node[6], node[7]
            if len(node) > 8:
                xp, yp, rp = node[8], node[9], node[10]
            what = "Conv" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "")
            dst = " and ".join(v for v in (self.R(y) if y else None, yp) if v)
            return (f"    /* {i}: {what} -> {dst} (weights prepared by inference_init) */\n"
                    f"    CHECK(cm_conv_prepared_async(g_cw[{self._conv_index[i]}], {self._dev(x)}, {self._planes(xp)}, "
                    f"{self._dev(y, False)}, {self._planes(yp)},\n        {int(epi)}u, {self._dev(resid)}, "
                    f"{self._planes(rp)}, NULL));")
        if kind == "conv" and len(node) > 8:
            _, x, wn, bn, y, args, epi, resid, xp, yp, rp = node
            a = ", ".join(f"{int(v)}u" for v in args)
            what = "Conv" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "")
            dst = " and ".join(v for v in (self.R(y) if y else None, yp) if v)
            return (f"    /* {i}: {what} -> {dst} */\n"
                    f"    CHECK(cm_conv_planes_async({self._dev(x)}, {self._planes(xp)}, {self._dev(wn)}, {self._dev(bn)}, "
                    f"{self._dev(y, False)}, {self._planes(yp)},\n        {a}, {int(epi)}u, {self._dev(resid)}, "
                    f"{self._planes(rp)}, NULL));")
        if kind == "poolp":
            _, xp, yp, args = node
            a = ", ".join(f"{int(v)}u" for v in args)
            return (f"    /* {i}: Pool {xp} -> {yp} (plane images) */\n"
                    f"    CHECK(cm_pool_planes_async({self._planes(xp)}, {self._planes(yp)},\n        {a}, NULL));")
        if kind == "poolnp":
            _, x, yp, args = node
            a = ", ".join(f"{int(v)}u" for v in args[:15])
            return (f"    /* {i}: Pool {self.R(x)} (channels-last) -> {yp} (plane image) */\n"
                    f"    CHECK(cm_pool_nhwc_planes_async({self._dev(x)}, {self._planes(yp)},\n        {a}, NULL));")
        if kind == "poolng":
            _, x, y, args = node
            a = ", ".join(f"{int(v)}u" for v in args)
            return (f"    /* {i}: global Pool {self.R(x)} (channels-last) -> {self.R(y)} */\n"
                    f"    CHECK(cm_pool_nhwc_async({self._dev(x)}, {self._dev(y, False)},\n        {a}, NULL));")
        if kind == "planes":
            _, x, pn = node
            return (f"    /* {i}: {self.R(x)} -> plane image {pn} */\n"
                    f"    CHECK(cm_planes_fill_async({self._planes(pn)}, {self._dev(x)}, NULL));")
        if kind == "conv":
            _, x, wn, bn, y, args = node[:6]
            epi, resid = (node[6], node[7]) if len(node) > 6 else (0, None)
            a = ", ".join(f"{int(v)}u" for v in args)
            what = "Conv" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "")
            if epi:
                return (f"    /* {i}: {what} -> {self.R(y)} */\n"
                        f"    CHECK(cm_conv_fused_async({self._dev(x)}, {self._dev(wn)}, {self._dev(bn)}, "
                        f"{self._dev(y, False)},\n        {a}, {int(epi)}u, {self._dev(resid)}, NULL));")
            return (f"    /* {i}: {what} -> {self.R(y)} */\n"
                    f"    CHECK(cm_conv_async({self._dev(x)}, {self._dev(wn)}, {self._dev(bn)}, "
                    f"{self._dev(y, False)},\n        {a}, NULL));")
        if kind == "vectorop":
            _, a_, b_, c_, args = node
            a = ", ".join(f"{int(v)}u" for v in args)
            return (f"    /* {i}: VectorOP {_OP_NAMES.get(int(args[1]), args[1])} -> {self.R(c_)} */\n"
                    f"    CHECK(cm_vectorop_async({self._dev(a_)}, {self._dev(b_)}, {self._dev(c_, False)}, "
                    f"{a}, NULL));")
        if kind == "matmul" and i in self._mm_index:
            a_, c_, args = node[1], node[3], node[4]
            epi, bias = (node[5], node[6]) if len(node) > 5 else (0, None)
            n, _, _, batch, a_bs, _, c_bs = (int(v) for v in args)
            what = "MatMul" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "")
            return (f"    /* {i}: {what} -> {self.R(c_)} (B prepared by inference_init) */\n"
                    f"    CHECK(cm_matmul_prepared_async(g_mw[{self._mm_index[i]}], {self._dev(a_)}, {self._dev(c_, False)}, "
                    f"{n}u, {batch}u, {a_bs}u, {c_bs}u, {int(epi)}u, {self._dev(bias)}, NULL));")
        if kind == "matmul" and len(node) > 5:
            _, a_, b_, c_, args, epi, bias = node
            a = ", ".join(f"{int(v)}u" for v in args)
            what = "MatMul" + ("+Add" if epi & 2 else "") + ("+Relu" if epi & 1 else "")
            return (f"    /* {i}: {what} -> {self.R(c_)} */\n"
                    f"    CHECK(cm_matmul_fused_async({self._dev(a_)}, {self._dev(b_)}, {self._dev(c_, False)}, "
                    f"{a}, {int(epi)}u, {self._dev(bias)}, NULL));")
        if kind == "matmul":
            _, a_, b_, c_, args = node
            a = ", ".join(f"{int(v)}u" for v in args)
            return (f"    /* {i}: MatMul -> {self.R(c_)} */\n"
                    f"    CHECK(cm_matmul_async({self._dev(a_)}, {self._dev(b_)}, {self._dev(c_, False)}, "
                    f"{a}, NULL));")
        if kind == "matmul_at":
            # run_matmul_at (_source.py:261-299): element offsets added to the three bases
            _, a_, b_, c_, args = node
            ao, bo, co = (int(v) for v in args[:3])
            a = ", ".join(f"{int(v)}u" for v in args[3:])
            return (f"    /* {i}: MatMul at +{ao}, +{bo}, +{co} -> {self.R(c_)} */\n"
                    f"    CHECK(cm_matmul_async({self._dev(a_)} + {ao}u, {self._dev(b_)} + {bo}u, "
                    f"{self._dev(c_, False)} + {co}u, {a}, NULL));")
        if kind == "pool":
            _, x, y, args = node
            a = ", ".join(f"{int(v)}u" for v in args)
            return (f"    /* {i}: Pool -> {self.R(y)} */\n"
                    f"    CHECK(cm_pool_async({self._dev(x)}, {self._dev(y, False)},\n        {a}, NULL));")
        raise ValueError(kind)

    def source(self) -> str:
        net, L = self.net, self.layout
        small = [n for n, (_, w) in L.weights.items() if w <= LARGE_WEIGHT_THRESHOLD]
        large = [n for n, (_, w) in L.weights.items() if w > LARGE_WEIGHT_THRESHOLD]
        arrays = "\n".join(
            f"static const Data_t {n}_init[{L.weights[n][1]}] = {{\n{_c_words(net.consts[n])}\n}};"
            for n in small)
        views = "\n".join([f"static inference_buf_t w_{n};" for n in L.weights] +
                          [f"static inference_buf_t t_{n};" for n in L.acts])
        wviews = "\n".join(f"    inference_buf_init_view(&w_{n}, g_wpool, {o}u, {w}u);"
                           for n, (o, w) in L.weights.items())
        aviews = "\n".join(f"    inference_buf_init_view(&t_{n}, g_apool, {o}u, {w}u);"
                           for n, (o, w) in L.acts.items())
        fills = "\n".join(
            [f"    memcpy(inference_buf_ptr(&w_{n}), {n}_init, sizeof {n}_init);" for n in small] +
            [f"    if (_load_weight(&w_{n}, \"{n}\")) goto fail;" for n in large])
        params = ", ".join(f"const char *{p}" for _, _, p in self.kernels)
        first = self.kernels[0][2]
        same = "\n".join(
            f"    if ({p} && strcmp({p}, {first}) != 0) {{\n"
            f"        fprintf(stderr, \"inference_init: {k} instance '%s' differs from '%s'\\n\", {p}, {first});\n"
            f"        return 1;\n    }}"
            for _, k, p in self.kernels[1:])
        convs = [i for i, n in enumerate(net.nodes) if n[0] == "conv"] if self.prepared else []
        self._conv_index = {i: j for j, i in enumerate(convs)}
        # MatMuls whose B is a network constant shared by the batch steps (a Gemm's weights)
        mms = [i for i, n in enumerate(net.nodes)
               if self.prepared and n[0] == "matmul" and net.resolve(n[2]) in net.consts
               and (int(n[4][3]) == 1 or int(n[4][5]) == 0)]
        self._mm_index = {i: j for j, i in enumerate(mms)}
        calls = "\n".join(self._call(i, n) for i, n in enumerate(net.nodes))
        cwdecl = (f"/* ---- conv weights prepared once (cm_conv_weights_create) ---- */\n"
                  f"static cm_conv_weights_t *g_cw[{len(convs)}];\n") if convs else ""
        cwcreate = "\n".join(
            f"    if (cm_conv_weights_create({self._dev(net.nodes[i][2])}, {self._dev(net.nodes[i][3])},\n"
            f"            {', '.join(f'{int(v)}u' for v in net.nodes[i][5])}, &g_cw[{j}]) != CM_OK) {{\n"
            f"        fprintf(stderr, \"inference_init: preparing conv {i}: %s\\n\", cm_last_error());\n"
            f"        goto fail;\n    }}"
            for j, i in enumerate(convs))
        cwdestroy = "\n".join(f"    cm_conv_weights_destroy(g_cw[{j}]);\n    g_cw[{j}] = NULL;" for j in range(len(convs)))
        if mms:
            cwdecl += (f"/* ---- Gemm B operands prepared once (cm_matmul_weights_create) ---- */\n"
                       f"static cm_matmul_weights_t *g_mw[{len(mms)}];\n")
            cwcreate += "\n" + "\n".join(
                f"    if (cm_matmul_weights_create({self._dev(net.nodes[i][2])}, {int(net.nodes[i][4][1])}u, "
                f"{int(net.nodes[i][4][2])}u, &g_mw[{j}]) != CM_OK) {{\n"
                f"        fprintf(stderr, \"inference_init: preparing MatMul {i}: %s\\n\", cm_last_error());\n"
                f"        goto fail;\n    }}"
                for j, i in enumerate(mms))
            cwdestroy += "\n" + "\n".join(f"    cm_matmul_weights_destroy(g_mw[{j}]);\n    g_mw[{j}] = NULL;"
                                            for j in range(len(mms)))
        pdecl = "\n".join(f"static cm_planes_t *{self._pvar(n)} = NULL;   /* {b}x{c}x{h}x{w}, frame {fr} */"
                          for n, (b, c, h, w, fr) in net.planes.items())
        pcreate = "\n".join(
            f"    {self._pvar(n)} = cm_planes_create({b}u, {c}u, {h}u, {w}u, {fr[0]}u, {fr[1]}u, {fr[2]}u, {fr[3]}u);\n"
            f"    if (!{self._pvar(n)}) goto fail;"
            for n, (b, c, h, w, fr) in net.planes.items())
        pdestroy = "\n".join(f"    cm_planes_destroy({self._pvar(n)});\n    {self._pvar(n)} = NULL;" for n in net.planes)
        loader = _LOAD_WEIGHT if large else ""
        return f"""/*
 * inference.c -- generated for network '{net.name}' (batch {net.batch}, {len(net.nodes)} kernel calls).
 * Every kernel call is queued on the legacy default CUDA stream; inference_run()
 * synchronizes once, after the last one.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "inference.h"

#ifndef INFERENCE_WEIGHTS_DIR
#  define INFERENCE_WEIGHTS_DIR  "."
#endif

#define IN(b)   ((const int16_t *)(uintptr_t)inference_buf_phys(b))
#define OUT(b)  ((int16_t *)(uintptr_t)inference_buf_phys(b))
#define CHECK(call) do {{ int _rc = (call); if (_rc != CM_OK) return _rc; }} while (0)

/* ---- weights of at most {LARGE_WEIGHT_THRESHOLD} words ---- */
{arrays}

/* ---- pools and views ---- */
static inference_buf_t *g_wpool = NULL;   /* {L.weight_words} words */
static inference_buf_t *g_apool = NULL;   /* {L.act_words} words */
{views}
/* ---- plane images: conv outputs kept in the next convs' operand form (cm_conv_planes) ---- */
{pdecl}
{cwdecl}
{loader}int inference_init({params})
{{
{same}
    if (cm_init({first}) != CM_OK) {{
        fprintf(stderr, "inference_init: cm_init(\\"%s\\"): %s\\n", {first} ? {first} : "(null)",
                cm_last_error());
        return 1;
    }}
    g_wpool = inference_buf_alloc({max(L.weight_words, 1)}u);
    g_apool = inference_buf_alloc({max(L.act_words, 1)}u);
    if (!g_wpool || !g_apool) {{
        fprintf(stderr, "inference_init: pool allocation failed: %s\\n", cm_last_error());
        goto fail;
    }}
{wviews}
{aviews}
{fills}
{pcreate}
    if (cm_buf_sync_to_device(g_wpool) != CM_OK) goto fail;
{cwcreate}
    return 0;
fail:
    inference_deinit();
    return 1;
}}

void inference_deinit(void)
{{
{cwdestroy}
{pdestroy}
    if (g_apool) inference_buf_release(g_apool);
    if (g_wpool) inference_buf_release(g_wpool);
    g_apool = g_wpool = NULL;
    cm_release();
}}

int inference_run(inference_buf_t *in_{self.in_c}, inference_buf_t *out_{self.out_c})
{{
    if (!g_wpool) return CM_ENOINIT;
    CHECK(cm_buf_sync_to_device(in_{self.in_c}));
{calls}
    CHECK(cm_synchronize(NULL));
    return cm_buf_sync_from_device(out_{self.out_c});
}}
"""

    # ---- test/test_inference.c -------------------------------------------------
    def test(self, expected: np.ndarray) -> str:
        out = self.out_c
        n = int(np.asarray(expected).size)
        if n <= LARGE_EXPECTED_THRESHOLD:
            exp_decl = f"static const Data_t expected_{out}_data[{n}] = {{\n{_c_words(expected)}\n}};"
            exp_load = f"    expected_{out} = expected_{out}_data;"
        else:
            exp_decl = ""
            exp_load = (f"    if (_load_expected(&exp_heap, \"{out}\", INFERENCE_{out.upper()}_SIZE)) "
                        "{ rc = 1; goto cleanup; }\n"
                        f"    expected_{out} = exp_heap;")
        inst = ", ".join(f"INFERENCE_{k.upper()}_INSTANCE" for _, k, _ in self.kernels)
        return f"""/*
 * test_inference.c -- generated for network '{self.net.name}': ramp input, one run,
 * every output word compared with the expected words.  Usage: test_inference [N]
 * (N > 0 also times N further inference_run calls).
 */
#include <stdio.h>
#include <stdlib.h>
#include <time.h>
#include "inference.h"

#ifndef INFERENCE_EXPECTED_DIR
#  define INFERENCE_EXPECTED_DIR  "."
#endif

{exp_decl}

static int _load_expected(Data_t **dst, const char *name, unsigned count)
{{
    char path[1024];
    FILE *f;
    size_t got;
    snprintf(path, sizeof path, INFERENCE_EXPECTED_DIR "/expected/%s.dat", name);
    f = fopen(path, "rb");
    if (!f) {{ fprintf(stderr, "GT: cannot open expected file '%s'\\n", path); return 1; }}
    *dst = (Data_t *)malloc((size_t)count * sizeof(Data_t));
    if (!*dst) {{ fclose(f); return 1; }}
    got = fread(*dst, sizeof(Data_t), count, f);
    fclose(f);
    if (got != count) {{ fprintf(stderr, "GT: '%s': got %zu expected %u\\n", path, got, count); return 1; }}
    return 0;
}}

int main(int argc, char **argv)
{{
    int rc = 0, iters = argc > 1 ? atoi(argv[1]) : 0;
    unsigned i, mismatches = 0;
    inference_buf_t *{self.in_c} = NULL, *{out} = NULL;
    const Data_t *expected_{out} = NULL;
    Data_t *exp_heap = NULL;
    (void)_load_expected;

    if (inference_init({inst}) != 0) {{
        fprintf(stderr, "inference_init failed\\n");
        return 1;
    }}
    {self.in_c} = inference_buf_alloc(INFERENCE_{self.in_c.upper()}_SIZE);
    {out} = inference_buf_alloc(INFERENCE_{out.upper()}_SIZE);
    if (!{self.in_c} || !{out}) {{ fprintf(stderr, "inference_buf_alloc failed\\n"); rc = 1; goto cleanup; }}
    {{
        Data_t *p = inference_buf_ptr({self.in_c});
        for (i = 0u; i < INFERENCE_{self.in_c.upper()}_SIZE; i++)
            p[i] = (Data_t)(i & 0xFFFFu);   /* i / 256.0 */
    }}
    rc = inference_run({self.in_c}, {out});
    if (rc != 0) {{ fprintf(stderr, "inference_run: %s\\n", cm_strerror(rc)); rc = 1; goto cleanup; }}
{exp_load}
    {{
        const Data_t *p = inference_buf_ptr({out});
        unsigned lim = INFERENCE_{out.upper()}_SIZE < 8u ? INFERENCE_{out.upper()}_SIZE : 8u;
        printf("Output '{out}' (%u elem, first %u):\\n", INFERENCE_{out.upper()}_SIZE, lim);
        for (i = 0u; i < lim; i++) printf("  [%u] (%.4f)\\n", i, p[i] / 256.0);
        for (i = 0u; i < INFERENCE_{out.upper()}_SIZE; i++) {{
            if (p[i] != expected_{out}[i]) {{
                if (mismatches < 10u)
                    fprintf(stderr, "GT MISMATCH {out}[%u]: got %.4f expected %.4f\\n", i,
                            p[i] / 256.0, expected_{out}[i] / 256.0);
                mismatches++;
            }}
        }}
    }}
    if (mismatches) {{
        printf("test_inference FAILED (%u mismatches)\\n", mismatches);
        rc = 1;
        goto cleanup;
    }}
    printf("test_inference PASSED\\n");
    if (iters > 0) {{
        struct timespec t0, t1;
        double ms;
        clock_gettime(CLOCK_MONOTONIC, &t0);
        for (i = 0; i < (unsigned)iters && rc == 0; i++) rc = inference_run({self.in_c}, {out});
        clock_gettime(CLOCK_MONOTONIC, &t1);
        ms = (t1.tv_sec - t0.tv_sec) * 1e3 + (t1.tv_nsec - t0.tv_nsec) / 1e6;
        printf("timing: %d runs, %.4f ms/run\\n", iters, ms / iters);
        if (rc) rc = 1;
    }}
cleanup:
    if ({self.in_c}) inference_buf_release({self.in_c});
    if ({out}) inference_buf_release({out});
    free(exp_heap);
    inference_deinit();
    return rc;
}}
"""

    def cmake(self) -> str:
        lib = self.lib_path or "${CORMORANT_LIB}"
        return f"""cmake_minimum_required(VERSION 3.16)
project(inference_{self.net.name.replace('+', '_')} C)
# libcormorant_cuda.so and include/cormorant_cuda.h of the cormorant_b200 package
set(CORMORANT_LIB "{lib}" CACHE FILEPATH "libcormorant_cuda.so")
set(CORMORANT_INCLUDE "" CACHE PATH "directory holding cormorant_cuda.h")
set(INFERENCE_WEIGHTS_DIR "${{CMAKE_CURRENT_SOURCE_DIR}}" CACHE PATH "directory holding weights/")
add_library(inference STATIC src/inference.c)
target_include_directories(inference PUBLIC include ${{CORMORANT_INCLUDE}})
target_compile_definitions(inference PRIVATE INFERENCE_WEIGHTS_DIR="${{INFERENCE_WEIGHTS_DIR}}")
target_link_libraries(inference PUBLIC ${{CORMORANT_LIB}})
add_executable(test_inference test/test_inference.c)
target_compile_definitions(test_inference PRIVATE INFERENCE_EXPECTED_DIR="${{CMAKE_CURRENT_SOURCE_DIR}}")
target_link_libraries(test_inference PRIVATE inference)
"""


def emit_project(net: Net, out_dir, expected: np.ndarray | None = None, lib_path: str | None = None,
                 prepared: bool = False) -> dict:
    """Write the generated project for `net` under out_dir and return {relative path: bytes written}.

    expected: the network output for the ramp input (word i = i & 0xFFFF), as int16; when
    given, test/test_inference.c and (above LARGE_EXPECTED_THRESHOLD words)
    expected/<output>.dat are written.  prepared: inference_init builds every conv's weight
    planes once (cm_conv_weights_create) and inference_run calls cm_conv_prepared_async."""
    em = _Emitter(net, lib_path, prepared)
    out = Path(out_dir)
    files = {"include/inference.h": em.header().encode(), "src/inference.c": em.source().encode(),
             "CMakeLists.txt": em.cmake().encode()}
    for name, (_, words) in em.layout.weights.items():
        if words > LARGE_WEIGHT_THRESHOLD:
            files[f"weights/{name}.dat"] = _dat_bytes(net.consts[name])
    if expected is not None:
        expected = np.asarray(expected, np.int16).reshape(-1)
        if expected.size != net.buffers[em.out_c]:
            raise ValueError(f"expected has {expected.size} words, output has {net.buffers[em.out_c]}")
        files["test/test_inference.c"] = em.test(expected).encode()
        if expected.size > LARGE_EXPECTED_THRESHOLD:
            files[f"expected/{em.out_c}.dat"] = _dat_bytes(expected)
    for rel, data in files.items():
        p = out / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(data)
    return {rel: len(data) for rel, data in files.items()}


def ramp_input(net: Net) -> np.ndarray:
    """The generated test's input: word i = i & 0xFFFF (the reference's ramp fill)."""
    n = net.buffers[net.resolve(net.input)]
    return (np.arange(n, dtype=np.int64) & 0xFFFF).astype(np.uint16).view(np.int16)


def compile_project(out_dir, include_dir, lib_path, cc: str | None = None) -> Path:
    """Compile src/inference.c + test/test_inference.c into out_dir/test_inference with gcc,
    linked against libcormorant_cuda.so (rpath set to its folder)."""
    import subprocess
    out = Path(out_dir)
    lib = Path(lib_path).resolve()
    exe = out / "test_inference"
    cmd = [cc or os.environ.get("CC", "gcc"), "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror",
           "-D_POSIX_C_SOURCE=200809L",
           f"-DINFERENCE_WEIGHTS_DIR=\"{out.resolve()}\"", f"-DINFERENCE_EXPECTED_DIR=\"{out.resolve()}\"",
           "-I", str(out / "include"), "-I", str(include_dir),
           str(out / "src/inference.c"), str(out / "test/test_inference.c"),
           "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe
