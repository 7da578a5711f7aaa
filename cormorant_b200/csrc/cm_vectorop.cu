// cm_vectorop.cu -- VectorOPKernel on B200 (reference: kernels/vectorop/kernel/VectorOP.cpp).
//
// Element-wise Q8.8 ops, HBM-bound.  Layout: three flat int16 arrays; with
// broadcasting, element (o, i) reads a[o*a_inc+i], b[o*b_inc+i] and writes
// c[o*(a_inc+b_inc)+i] (VectorOP.cpp:179).
//
//  * vec path: 128-bit streaming loads/stores (8 words each), four vectors in
//    flight per thread, grid = a multiple of the SM count, grid-stride loop.
//    Used when rows of the (outer x size) view do not overlap in c and every
//    row start is 16-byte aligned.
//  * general path: one thread per output word, output-driven, so that when
//    rows overlap in c the write of the largest o wins -- the order of the
//    reference's sequential store loop (VectorOP.cpp:117-134).
//
// Op semantics (VectorOP.cpp:8-35, reference scheduler model dtype.py:110-124):
//   ADD/SUB  sat16(a +- b)            MUL  sat16(floor(a*b / 256))
//   DIV      b == 0 -> 0, else sat16(trunc_toward_zero(a*256 / b))
//   RELU     max(a, 0)                RELU6 min(max(a, 0), 0x0600)
//   other op codes copy a (the switch default, VectorOP.cpp:108).
#include "cm_common.cuh"

namespace cm {
namespace {

enum { K_ADD = 0, K_SUB, K_MUL, K_DIV, K_RELU, K_RELU6, K_COPY };

// Exact conversions for 0 <= x <= 2^23 by the classic bias trick: the integer
// is placed in the mantissa of 2^23 (bit pattern 0x4B000000 + x), and 2^23 is
// subtracted in float -- two full-rate ops instead of a quarter-rate convert.
__device__ __forceinline__ float u23_to_f(uint32_t x) {
    return __fsub_rn(__uint_as_float(0x4B000000u + x), 8388608.0f);
}
// Nearest integer (ties to even) of 0 <= f < 2^23, by the same bias.
__device__ __forceinline__ uint32_t f_to_u23_rn(float f) {
    return __float_as_uint(__fadd_rn(f, 8388608.0f)) - 0x4B000000u;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// trunc((a * 256) / b) for b != 0, exact, as far as int16 saturation can tell.
// un = |a*256| <= 2^23 and ud = |b| in [1, 2^15] are exact in float.  rcp.approx
// has a relative error below 2^-23 and the product adds at most 2^-24, so for a
// true quotient Q = un/ud < 2^21 the estimate qf is within 0.38 of Q and its
// nearest integer is floor(Q) or floor(Q)+1; one remainder test removes the
// excess (reciprocal estimate plus integer correction, Hacker's Delight ch. 10).
// For Q >= 2^21 every candidate saturates to the same int16 as the exact value.
__device__ __forceinline__ int32_t div_q88(int32_t a, int32_t b) {
    const int32_t n = a * 256;
    const uint32_t un = (uint32_t)(n < 0 ? -n : n);
    const uint32_t ud = (uint32_t)(b < 0 ? -b : b);
    const float qf = __fmul_rn(u23_to_f(un), rcp_approx(u23_to_f(ud)));
    uint32_t q = f_to_u23_rn(qf);
    if ((int32_t)(un - q * ud) < 0) q -= 1;     // true remainder is in (-ud, ud): exact mod 2^32
    return ((n ^ b) < 0) ? -(int32_t)q : (int32_t)q;
}

template <int OP>
__device__ __forceinline__ int16_t op1(int16_t a, int16_t b) {
    if (OP == K_ADD) return sat16((int32_t)a + (int32_t)b);
    if (OP == K_SUB) return sat16((int32_t)a - (int32_t)b);
    if (OP == K_MUL) return sat16(((int32_t)a * (int32_t)b) >> 8);
    if (OP == K_DIV) return b == 0 ? (int16_t)0 : sat16(div_q88(a, b));
    if (OP == K_RELU) return a < 0 ? (int16_t)0 : a;
    if (OP == K_RELU6) return a < 0 ? (int16_t)0 : (a > 0x600 ? (int16_t)0x600 : a);
    return a;
}

// One 32-bit word = two int16 lanes.
template <int OP>
__device__ __forceinline__ uint32_t op2(uint32_t a, uint32_t b) {
    if (OP == K_ADD) return __vaddss2(a, b);            // per-halfword saturating add
    if (OP == K_SUB) return __vsubss2(a, b);            // per-halfword saturating subtract
    if (OP == K_RELU) return __vmaxs2(a, 0u);
    if (OP == K_RELU6) return __vmins2(__vmaxs2(a, 0u), 0x06000600u);
    if (OP == K_COPY) return a;
    const int16_t lo = op1<OP>((int16_t)(a & 0xFFFF), (int16_t)(b & 0xFFFF));
    const int16_t hi = op1<OP>((int16_t)(a >> 16), (int16_t)(b >> 16));
    return (uint32_t)(uint16_t)lo | ((uint32_t)(uint16_t)hi << 16);
}

template <int OP>
__device__ __forceinline__ uint4 op8(uint4 a, uint4 b) {
    return make_uint4(op2<OP>(a.x, b.x), op2<OP>(a.y, b.y), op2<OP>(a.z, b.z), op2<OP>(a.w, b.w));
}

constexpr int UNROLL = 4;

// Vector path.  Work item t indexes 8-word vectors of the (outer x nv) view.
// TWO_D: row o = t / nv with row strides (in vectors) a_inc, b_inc, c_inc.
template <int OP, bool TWO_D>
__global__ void __launch_bounds__(256) vop_vec_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b,
                                                      uint4* __restrict__ c, uint64_t total, FastDiv nv,
                                                      uint64_t a_inc, uint64_t b_inc, uint64_t c_inc) {
    griddep_wait();
    constexpr bool UNARY = (OP >= K_RELU);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t0 < total; t0 += stride * UNROLL) {
        uint4 va[UNROLL], vb[UNROLL];
        uint64_t ci[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const uint64_t t = t0 + (uint64_t)u * stride;
            if (t < total) {
                uint64_t ai = t, bi = t;
                ci[u] = t;
                if (TWO_D) {
                    const uint32_t o = nv.div((uint32_t)t);
                    const uint64_t j = t - (uint64_t)o * nv.d;
                    ai = o * a_inc + j;
                    bi = o * b_inc + j;
                    ci[u] = o * c_inc + j;
                }
                va[u] = __ldcs(a + ai);
                if (!UNARY) vb[u] = __ldcs(b + bi);
                else vb[u] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const uint64_t t = t0 + (uint64_t)u * stride;
            if (t < total) __stcs(c + ci[u], op8<OP>(va[u], vb[u]));
        }
    }
}

// General path: c[j] gets the value of the last (largest) o that writes it.
template <int OP>
__global__ void __launch_bounds__(256) vop_general_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b,
                                                          int16_t* __restrict__ c, uint64_t c_len, uint32_t size,
                                                          uint32_t outer, uint64_t a_inc, uint64_t b_inc, uint64_t c_inc) {
    griddep_wait();
    constexpr bool UNARY = (OP >= K_RELU);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < c_len; j += stride) {
        uint64_t o = outer - 1;
        if (c_inc != 0) {
            const uint64_t q = j / c_inc;
            if (q < o) o = q;
        }
        const uint64_t i = j - o * c_inc;
        if (i >= size) continue;   // a gap between rows: never written
        const int16_t av = a[o * a_inc + i];
        const int16_t bv = UNARY ? (int16_t)0 : b[o * b_inc + i];
        c[j] = op1<OP>(av, bv);
    }
}

struct VopCall {
    const int16_t* a; const int16_t* b; int16_t* c;
    uint32_t size, outer; uint64_t a_inc, b_inc, c_inc;
};

template <int OP>
int launch_general(const Context* cx, const VopCall& v, cudaStream_t s) {
    const uint64_t c_len = (uint64_t)(v.outer - 1) * v.c_inc + v.size;
    const unsigned grid = grid_for(cx, c_len, 256, 16);
    {
        ProfScope ps_(PK_VECTOROP, s);
        launch_k(vop_general_kernel<OP>, grid, 256, 0, s, v.a, v.b, v.c, c_len, v.size, v.outer, v.a_inc, v.b_inc, v.c_inc);
    }
    count_launch();
    return CM_OK;
}

template <int OP>
int launch_vec(const Context* cx, const int16_t* a, const int16_t* b, int16_t* c, uint64_t rows, uint64_t nv,
               uint64_t a_inc_v, uint64_t b_inc_v, uint64_t c_inc_v, cudaStream_t s) {
    const uint64_t total = rows * nv;
    if (total == 0) return CM_OK;
    const unsigned grid = grid_for(cx, (total + UNROLL - 1) / UNROLL, 256, 8);
    if (rows == 1) {
        {
            ProfScope ps_(PK_VECTOROP, s);
            launch_k(vop_vec_kernel<OP, false>, grid, 256, 0, s, (const uint4*)a, (const uint4*)b, (uint4*)c, total, FastDiv(1), 0, 0, 0);
        }
    } else {
        {
            ProfScope ps_(PK_VECTOROP, s);
            launch_k(vop_vec_kernel<OP, true>, grid, 256, 0, s, (const uint4*)a, (const uint4*)b, (uint4*)c, total,
                                                          FastDiv((uint32_t)nv), a_inc_v, b_inc_v, c_inc_v);
        }
    }
    count_launch();
    return CM_OK;
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

template <int OP>
int run(const Context* cx, const VopCall& v, cudaStream_t s) {
    constexpr bool UNARY = (OP >= K_RELU);
    const bool overlap = v.outer > 1 && v.c_inc < v.size;
    if (!overlap) {
        if (v.outer == 1) {
            // Flat: vectors over the common 16-byte-aligned middle, words at the edges.
            const uintptr_t mis = (uintptr_t)v.a & 15u;
            const bool same = ((uintptr_t)v.c & 15u) == mis && (UNARY || ((uintptr_t)v.b & 15u) == mis) && (mis & 1u) == 0;
            if (same) {
                const uint64_t head = mis ? (16 - mis) / 2 : 0;
                if (head >= v.size) return launch_general<OP>(cx, v, s);
                const uint64_t nv = (v.size - head) / 8;
                const uint64_t tail = (v.size - head) - nv * 8;
                if (head) {
                    VopCall h = v; h.size = (uint32_t)head;
                    launch_general<OP>(cx, h, s);
                }
                launch_vec<OP>(cx, v.a + head, UNARY ? nullptr : v.b + head, v.c + head, 1, nv, 0, 0, 0, s);
                if (tail) {
                    const uint64_t off = head + nv * 8;
                    VopCall t = v; t.a += off; if (!UNARY) t.b += off; t.c += off; t.size = (uint32_t)tail;
                    launch_general<OP>(cx, t, s);
                }
                return CM_OK;
            }
        } else if (v.size % 8 == 0 && v.a_inc % 8 == 0 && v.b_inc % 8 == 0 && al16(v.a) && al16(v.c) &&
                   (UNARY || al16(v.b)) && (uint64_t)v.outer * (v.size / 8) < (1ull << 32)) {
            return launch_vec<OP>(cx, v.a, v.b, v.c, v.outer, v.size / 8, v.a_inc / 8, UNARY ? 0 : v.b_inc / 8,
                                  v.c_inc / 8, s);
        }
    }
    return launch_general<OP>(cx, v, s);
}

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_vectorop_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned size, unsigned op,
                                 unsigned outer, unsigned a_inc, unsigned b_inc, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (size == 0 || outer == 0) return CM_OK;
    const bool unary = op >= CM_OP_RELU;
    if (!a || !c || (!unary && !b)) return set_error(CM_EINVAL, "cm_vectorop: null buffer");
    VopCall v{a, unary ? nullptr : b, c, size, outer, a_inc, b_inc, (uint64_t)a_inc + (uint64_t)b_inc};
    cudaStream_t s = (cudaStream_t)stream;
    switch (op) {
        case CM_OP_ADD: rc = run<K_ADD>(cx, v, s); break;
        case CM_OP_SUB: rc = run<K_SUB>(cx, v, s); break;
        case CM_OP_MUL: rc = run<K_MUL>(cx, v, s); break;
        case CM_OP_DIV: rc = run<K_DIV>(cx, v, s); break;
        case CM_OP_RELU: rc = run<K_RELU>(cx, v, s); break;
        case CM_OP_RELU6: rc = run<K_RELU6>(cx, v, s); break;
        default: rc = run<K_COPY>(cx, v, s); break;
    }
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_vectorop launch");
}

extern "C" int cm_vectorop(const int16_t* a, const int16_t* b, int16_t* c, unsigned size, unsigned op,
                           unsigned outer, unsigned a_inc, unsigned b_inc) {
    int rc = cm_vectorop_async(a, b, c, size, op, outer, a_inc, b_inc, nullptr);
    return rc ? rc : finish_sync(nullptr);
}
