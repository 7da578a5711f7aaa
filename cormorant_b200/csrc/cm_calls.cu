// cm_calls.cu -- a list of small kernel calls in ONE launch (no reference counterpart).
//
// A batch-1 network (the LeNet-5 configuration: 0.4 M multiply-accumulates, 7 calls
// after folding) is bound by launch latency: each call is a few microseconds of
// launch and drain for well under a microsecond of work.  cm_calls_async runs the
// whole list as one CTA of 1024 threads that executes the calls in order, with a
// block barrier between them (the barrier orders each call's global stores before
// the next call's loads).  Each call computes exactly what its own entry point
// computes, from the same arithmetic as the CUDA-core kernels:
//   conv     int32 wrap sum of x*w over the in-image taps, + bias << 8, one floor /
//            saturate narrowing (ConvKernel.cpp:160-230), then the fused epilogue
//   MatMul   int32 wrap dot product, one narrowing (MatmulKernel.cpp:204-218), then
//            the fused bias-row add / ReLU
//   MaxPool  max over the in-image taps; a window with none gives -32768 (kAccMin,
//            PoolingKernel.cpp:193-197, 212-213)
//   VectorOP ADD / SUB saturating, MUL (a*b) >> 8 saturated, RELU, RELU6, copy
//            (VectorOP.cpp:108-140)
// Calls outside that set or above the size limits are refused (CM_EUNSUPPORTED) and
// run through their own entry points instead.
#include <cuda_runtime.h>

#include "cm_common.cuh"

namespace cm {
namespace {

constexpr uint32_t kCallThreads = 1024;
constexpr uint64_t kMaxCallMacs = 1ull << 22;     // per call
constexpr uint32_t kStageBytes = 200u * 1024u;    // shared memory for one call's operands
constexpr uint32_t kStageWords = kStageBytes / 2;
constexpr uint64_t kMaxCallOutputs = 1ull << 20;  // per call

struct CallArgs {
    uint32_t kind, epi;
    const int16_t* in0;
    const int16_t* in1;
    const int16_t* in2;
    const int16_t* resid;
    int16_t* out;
    uint32_t a[17];
};

struct CallList {
    uint32_t count;
    CallArgs c[CM_CALLS_MAX];
};

__device__ __forceinline__ int16_t epilogue_conv(int16_t v, uint32_t epi, const int16_t* resid, uint64_t i) {
    int32_t r = v;
    if (epi & 2u) r = sat16(r + (int32_t)resid[i]);
    if (epi & 1u) r = max(r, 0);
    return (int16_t)r;
}

// Operands are staged in shared memory first (kStageWords int16 words per call, checked
// on the host): the serial per-output loops then read shared memory instead of waiting on
// global loads, which is what bounds one CTA.
__device__ void stage(int16_t* dst, const int16_t* src, uint32_t n) {
    if ((((uintptr_t)src | (uintptr_t)dst) & 15u) == 0) {
        const uint32_t n8 = n / 8;
        for (uint32_t i = threadIdx.x; i < n8; i += blockDim.x) ((uint4*)dst)[i] = __ldg((const uint4*)src + i);
        for (uint32_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
    } else {
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldg(src + i);
    }
}

__device__ __forceinline__ uint32_t up8(uint32_t n) { return (n + 7u) & ~7u; }

__device__ void run_conv(const CallArgs& c, int16_t* sm) {
    const uint32_t N = c.a[0], C = c.a[1], H = c.a[2], W = c.a[3], M = c.a[4], OH = c.a[5], OW = c.a[6];
    const uint32_t kh = c.a[7], kw = c.a[8], sh = c.a[9], sw = c.a[10], dh = c.a[11], dw = c.a[12];
    const uint32_t pt = c.a[13], pl = c.a[14], has_bias = c.a[15], dwise = c.a[16];
    const uint32_t nx = N * C * H * W, nw = M * (dwise ? 1u : C) * kh * kw;
    int16_t* xs = sm;
    int16_t* ws = sm + up8(nx);
    stage(xs, c.in0, nx);
    stage(ws, c.in1, nw);
    __syncthreads();
    const uint32_t total = N * M * OH * OW;
    for (uint32_t t = threadIdx.x; t < total; t += blockDim.x) {
        const uint32_t ow = t % OW, r0 = t / OW, oh = r0 % OH, r1 = r0 / OH, m = r1 % M, n = r1 / M;
        uint32_t acc = 0;
        const uint32_t c_lo = dwise ? m : 0u, c_hi = dwise ? m + 1 : C;
        for (uint32_t ci = c_lo; ci < c_hi; ++ci) {
            const int16_t* xc = xs + (n * C + ci) * H * W;
            const int16_t* wc = ws + (m * (dwise ? 1u : C) + (dwise ? 0u : ci)) * kh * kw;
            for (uint32_t r = 0; r < kh; ++r) {
                const int32_t ih = (int32_t)(oh * sh + r * dh) - (int32_t)pt;
                if (ih < 0 || ih >= (int32_t)H) continue;
                for (uint32_t s = 0; s < kw; ++s) {
                    const int32_t iw = (int32_t)(ow * sw + s * dw) - (int32_t)pl;
                    if (iw < 0 || iw >= (int32_t)W) continue;
                    acc += (uint32_t)((int32_t)xc[(uint32_t)ih * W + (uint32_t)iw] * (int32_t)wc[r * kw + s]);
                }
            }
        }
        if (has_bias) acc += (uint32_t)((int32_t)__ldg(c.in2 + m) * 256);
        c.out[t] = epilogue_conv(narrow_acc(acc), c.epi, c.resid, t);
    }
}

// MatMul: a block of 1024 threads = output columns j x K splits; the K split partial
// sums (int32 wrap, so order-free) meet in shared memory.
__device__ void run_matmul(const CallArgs& c, int16_t* sm) {
    const uint32_t n = c.a[0], k = c.a[1], m = c.a[2], batch = c.a[3], a_bs = c.a[4], b_bs = c.a[5], c_bs = c.a[6];
    const uint32_t nm = n * m, total = batch * nm;
    const uint32_t na = batch > 1 && a_bs ? (batch - 1) * a_bs + n * k : n * k;
    const uint32_t nb = batch > 1 && b_bs ? (batch - 1) * b_bs + k * m : k * m;
    int16_t* as = sm;
    int16_t* bs = sm + up8(na);
    uint32_t* part = (uint32_t*)(bs + up8(nb));              // [kSplit][outputs in flight]
    stage(as, c.in0, na);
    stage(bs, c.in1, nb);
    __syncthreads();
    uint32_t split = 1;                                      // K split: fill the block, at most 32 ways
    while (split < 32 && split * 2 * min(total, blockDim.x) <= blockDim.x * 2 && split * 2 <= k) split *= 2;
    const uint32_t per_round = blockDim.x / split;
    for (uint32_t base = 0; base < total; base += per_round) {
        const uint32_t o = threadIdx.x % per_round, sidx = threadIdx.x / per_round;
        const uint32_t t = base + o;
        uint32_t acc = 0;
        if (t < total) {
            const uint32_t z = t / nm, rem = t - z * nm, i = rem / m, j = rem - i * m;
            const int16_t* ar = as + z * (batch > 1 ? a_bs : 0u) + i * k;
            const int16_t* bc = bs + z * (batch > 1 ? b_bs : 0u) + j;
            for (uint32_t q = sidx; q < k; q += split) acc += (uint32_t)((int32_t)ar[q] * (int32_t)bc[q * m]);
        }
        part[sidx * per_round + o] = acc;
        __syncthreads();
        if (sidx == 0 && t < total) {
            for (uint32_t q = 1; q < split; ++q) acc += part[q * per_round + o];
            const uint32_t z = t / nm, rem = t - z * nm, i = rem / m, j = rem - i * m;
            int32_t v = narrow_acc(acc);
            if (c.epi & 2u) v = sat16(v + (int32_t)__ldg(c.in2 + j));
            if (c.epi & 1u) v = max(v, 0);
            c.out[(uint64_t)z * c_bs + (uint64_t)i * m + j] = (int16_t)v;
        }
        __syncthreads();
    }
}

__device__ void run_maxpool(const CallArgs& c, int16_t* sm) {
    const uint32_t N = c.a[0], C = c.a[1], H = c.a[2], W = c.a[3], OH = c.a[4], OW = c.a[5];
    const uint32_t ph = c.a[6], pw = c.a[7], sh = c.a[8], sw = c.a[9], pt = c.a[10], pl = c.a[11], dh = c.a[12],
                   dw = c.a[13];
    stage(sm, c.in0, N * C * H * W);
    __syncthreads();
    const uint32_t total = N * C * OH * OW;
    for (uint32_t t = threadIdx.x; t < total; t += blockDim.x) {
        const uint32_t ow = t % OW, r0 = t / OW, oh = r0 % OH, plane = r0 / OH;
        const int16_t* xc = sm + plane * H * W;
        int32_t v = -32768;
        for (uint32_t r = 0; r < ph; ++r) {
            const int32_t ih = (int32_t)(oh * sh + r * dh) - (int32_t)pt;
            if (ih < 0 || ih >= (int32_t)H) continue;
            for (uint32_t s = 0; s < pw; ++s) {
                const int32_t iw = (int32_t)(ow * sw + s * dw) - (int32_t)pl;
                if (iw < 0 || iw >= (int32_t)W) continue;
                v = max(v, (int32_t)xc[(uint32_t)ih * W + (uint32_t)iw]);
            }
        }
        c.out[t] = (int16_t)v;
    }
}

__device__ void run_vectorop(const CallArgs& c) {
    const uint32_t size = c.a[0], op = c.a[1], outer = c.a[2], a_inc = c.a[3], b_inc = c.a[4];
    const uint32_t total = size * outer;
    for (uint32_t t = threadIdx.x; t < total; t += blockDim.x) {
        const uint32_t o = t / size, i = t - o * size;
        const int32_t a = c.in0[(uint64_t)o * a_inc + i];
        const int32_t b = (op <= CM_OP_MUL) ? (int32_t)c.in1[(uint64_t)o * b_inc + i] : 0;
        int32_t v;
        if (op == CM_OP_ADD) v = sat16(a + b);
        else if (op == CM_OP_SUB) v = sat16(a - b);
        else if (op == CM_OP_MUL) v = sat16((a * b) >> 8);
        else if (op == CM_OP_RELU) v = max(a, 0);
        else if (op == CM_OP_RELU6) v = min(max(a, 0), 0x600);
        else v = a;
        c.out[(uint64_t)o * (a_inc + b_inc) + i] = (int16_t)v;
    }
}

__global__ void __launch_bounds__(kCallThreads, 1) calls_kernel(const __grid_constant__ CallList L) {
    griddep_wait();
    extern __shared__ __align__(16) int16_t stage_smem[];
    for (uint32_t k = 0; k < L.count; ++k) {
        const CallArgs& c = L.c[k];
        if (c.kind == CM_CALL_CONV) run_conv(c, stage_smem);
        else if (c.kind == CM_CALL_MATMUL) run_matmul(c, stage_smem);
        else if (c.kind == CM_CALL_POOL) run_maxpool(c, stage_smem);
        else run_vectorop(c);
        __syncthreads();
    }
}

// Empty string when call c can run inside the one-launch kernel, else why not.
const char* call_refusal(const cm_call_t& c) {
    const unsigned* a = c.args;
    if (!c.out) return "null output";
    switch (c.kind) {
    case CM_CALL_CONV: {
        const uint64_t outs = (uint64_t)a[0] * a[4] * a[5] * a[6];
        const uint64_t per = (uint64_t)(a[16] ? 1u : a[1]) * a[7] * a[8];
        if (!c.in0 || !c.in1 || (a[15] && !c.in2) || ((c.epilogue & 2u) && !c.resid)) return "null conv operand";
        if (c.epilogue > 3u) return "conv epilogue";
        if (a[16] && a[4] > a[1]) return "depthwise out_ch > in_ch";
        if (outs > kMaxCallOutputs || outs * per > kMaxCallMacs) return "conv too large";
        const uint64_t nx = (uint64_t)a[0] * a[1] * a[2] * a[3], nw = (uint64_t)a[4] * per;
        if (((nx + 7) & ~7ull) + nw > kStageWords) return "conv operands exceed shared memory";
        return "";
    }
    case CM_CALL_MATMUL: {
        const uint64_t outs = (uint64_t)a[3] * a[0] * a[2];
        if (!c.in0 || !c.in1 || ((c.epilogue & 2u) && !c.in2)) return "null matmul operand";
        if (c.epilogue > 3u) return "matmul epilogue";
        if (a[3] > 1 && (uint64_t)a[6] < (uint64_t)a[0] * a[2]) return "overlapping matmul outputs";
        if (outs > kMaxCallOutputs || outs * a[1] > kMaxCallMacs) return "matmul too large";
        const uint64_t na = a[3] > 1 && a[4] ? (uint64_t)(a[3] - 1) * a[4] + (uint64_t)a[0] * a[1] : (uint64_t)a[0] * a[1];
        const uint64_t nb = a[3] > 1 && a[5] ? (uint64_t)(a[3] - 1) * a[5] + (uint64_t)a[1] * a[2] : (uint64_t)a[1] * a[2];
        if (((na + 7) & ~7ull) + ((nb + 7) & ~7ull) + 2 * kCallThreads > kStageWords)
            return "matmul operands exceed shared memory";
        return "";
    }
    case CM_CALL_POOL: {
        const uint64_t outs = (uint64_t)a[0] * a[1] * a[4] * a[5];
        if (!c.in0) return "null pool input";
        if (a[14] != CM_POOL_MAX) return "pool type (MAX only)";
        if (outs > kMaxCallOutputs || (uint64_t)a[6] * a[7] > 1024) return "pool too large";
        if ((uint64_t)a[0] * a[1] * a[2] * a[3] > kStageWords) return "pool input exceeds shared memory";
        return "";
    }
    case CM_CALL_VECTOROP: {
        const uint64_t outs = (uint64_t)a[0] * a[2];
        if (!c.in0 || (a[1] <= CM_OP_MUL && !c.in1)) return "null vectorop operand";
        if (a[1] == CM_OP_DIV) return "vectorop DIV";
        if (a[2] > 1 && (uint64_t)a[3] + a[4] < a[0]) return "overlapping vectorop rows";
        if (outs > kMaxCallOutputs) return "vectorop too large";
        return "";
    }
    default:
        return "unknown call kind";
    }
}

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_calls_supported(const cm_call_t* calls, unsigned count) {
    if (!calls || count == 0 || count > CM_CALLS_MAX) return 0;
    for (unsigned i = 0; i < count; ++i)
        if (call_refusal(calls[i])[0]) return 0;
    return 1;
}

extern "C" int cm_calls_async(const cm_call_t* calls, unsigned count, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (count == 0) return CM_OK;
    if (!calls) return set_error(CM_EINVAL, "cm_calls: null call list");
    if (count > CM_CALLS_MAX) return set_error(CM_EUNSUPPORTED, "cm_calls: %u calls (at most %u)", count, CM_CALLS_MAX);
    CallList L{};
    L.count = count;
    for (unsigned i = 0; i < count; ++i) {
        const char* why = call_refusal(calls[i]);
        if (why[0]) return set_error(CM_EUNSUPPORTED, "cm_calls: call %u: %s", i, why);
        CallArgs& d = L.c[i];
        d.kind = calls[i].kind;
        d.epi = calls[i].epilogue;
        d.in0 = calls[i].in0; d.in1 = calls[i].in1; d.in2 = calls[i].in2; d.resid = calls[i].resid;
        d.out = calls[i].out;
        for (int k = 0; k < 17; ++k) d.a[k] = calls[i].args[k];
    }
    cudaStream_t s = (cudaStream_t)stream;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(calls_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStageBytes);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(calls)");
        attr = true;
    }
    {
        ProfScope ps_(PK_CONV_AUX, s);
        launch_k(calls_kernel, 1, kCallThreads, kStageBytes, s, L);
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_calls");
}

extern "C" int cm_calls(const cm_call_t* calls, unsigned count) {
    int rc = cm_calls_async(calls, count, nullptr);
    return rc ? rc : finish_sync(nullptr);
}
