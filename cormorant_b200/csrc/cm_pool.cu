// cm_pool.cu -- PoolingKernel on B200 (reference: kernels/pool/kernel/PoolingKernel.cpp).
//
// NCHW, one (n, c) plane at a time, HBM-bound.
//  * window kernel: one CTA per (plane, band of output rows).  The input rows
//    the band touches are one contiguous range of the plane; they are staged
//    in shared memory with 128-bit loads, then every thread computes output
//    pixels from shared memory and writes them coalesced along the row.
//  * global kernel (GlobalMax/Avg/LpPool, i.e. pool = in, pad 0): one warp per
//    plane, 128-bit loads, warp-shuffle reduction.
//
// Arithmetic (PoolingKernel.cpp:122-267), accumulator = ap_fixed<32,16> raw (int32, wraps):
//   MAX : max of x<<8 over taps, padded taps = -128.0, start = -32768.0
//   AVG : sum of x<<8 over valid taps; result = AccData_t(float(acc) * (1.0f/denom)),
//         denom = count_include_pad ? pool_h*pool_w : valid taps (0 -> factor 0)
//   LP1 : sum |x|<<8                LP2 (lp_order != 1): AccData_t(sqrtf(float(acc)))
//   then saturate_cast: floor by 8 bits, clamp to int16.
// float(acc) rounds to nearest-even; AccData_t(float) floors to 2^-16 and
// wraps to 32 bits; NaN (LP2 of a wrapped negative sum) converts to 0.
#include <algorithm>

#include "cm_common.cuh"

namespace cm {
namespace {

enum { P_MAX = 0, P_AVG = 1, P_LP1 = 2, P_LP2 = 3 };

// AccData_t(float f) on the raw Q16.16 word.
__device__ __forceinline__ uint32_t acc_from_float(float f) {
    if (isnan(f)) return 0u;
    return (uint32_t)(unsigned long long)__float2ll_rd(__fmul_rn(f, 65536.0f));  // exact scale, floor
}

// float(AccData_t acc) -- round to nearest even, then the exact 2^-16 scale.
__device__ __forceinline__ float acc_to_float(uint32_t acc) {
    return __fmul_rn(__int2float_rn((int32_t)acc), 0x1p-16f);
}

template <int TYPE>
__device__ __forceinline__ int16_t finalize(uint32_t acc, uint32_t denom) {
    if (TYPE == P_AVG) {
        const float inv = denom > 0u ? __fdiv_rn(1.0f, __uint2float_rn(denom)) : 0.0f;
        acc = acc_from_float(__fmul_rn(acc_to_float(acc), inv));
    } else if (TYPE == P_LP2) {
        acc = acc_from_float(__fsqrt_rn(acc_to_float(acc)));
    }
    return narrow_acc(acc);
}

struct PoolP {
    uint32_t in_h, in_w, out_h, out_w, ph, pw, sh, sw, pt, pl, dh, dw, cip;
    uint32_t band_rows, n_bands;
    FastDiv fd_ow;
};

template <int TYPE>
__device__ __forceinline__ void tap(uint32_t& acc, int32_t v) {
    if (TYPE == P_MAX) {
        const int32_t t = v * 256;
        if (t > (int32_t)acc) acc = (uint32_t)t;
    } else if (TYPE == P_AVG) {
        acc += (uint32_t)(v * 256);
    } else if (TYPE == P_LP1) {
        acc += (uint32_t)((v < 0 ? -v : v) * 256);
    } else {
        acc += (uint32_t)(v * v);
    }
}

// Computes one output pixel; `src(ih, iw)` reads a valid input tap.
template <int TYPE, class Src>
__device__ __forceinline__ int16_t pool_pixel(const PoolP& p, uint32_t oh, uint32_t ow, Src src) {
    uint32_t acc = (TYPE == P_MAX) ? 0x80000000u : 0u;
    uint32_t valid = 0;
    for (uint32_t r = 0; r < p.ph; ++r) {
        const int64_t ih = (int64_t)oh * p.sh + (int64_t)r * p.dh - (int64_t)p.pt;
        const bool row_ok = ih >= 0 && ih < (int64_t)p.in_h;
        for (uint32_t s = 0; s < p.pw; ++s) {
            const int64_t iw = (int64_t)ow * p.sw + (int64_t)s * p.dw - (int64_t)p.pl;
            if (row_ok && iw >= 0 && iw < (int64_t)p.in_w) {
                ++valid;
                tap<TYPE>(acc, src(ih, iw));
            } else if (TYPE == P_MAX) {
                tap<TYPE>(acc, -32768);   // padded tap holds -128.0 for MAX; 0 adds nothing otherwise
            }
        }
    }
    return finalize<TYPE>(acc, p.cip ? p.ph * p.pw : valid);
}

template <int TYPE>
__global__ void __launch_bounds__(256) pool_window_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y, PoolP p) {
    extern __shared__ __align__(16) int16_t smem[];
    const uint64_t blk = blockIdx.x;
    const uint64_t plane = blk / p.n_bands;
    const uint32_t band = (uint32_t)(blk - plane * p.n_bands);
    const uint32_t oh0 = band * p.band_rows;
    const uint32_t oh1 = min(p.out_h, oh0 + p.band_rows);
    const int64_t ih_lo = (int64_t)oh0 * p.sh - (int64_t)p.pt;
    const int64_t ih_hi = (int64_t)(oh1 - 1) * p.sh + (int64_t)(p.ph ? p.ph - 1 : 0) * p.dh - (int64_t)p.pt;
    const int64_t r_lo = ih_lo > 0 ? ih_lo : 0;
    const int64_t r_hi = ih_hi < (int64_t)p.in_h - 1 ? ih_hi : (int64_t)p.in_h - 1;
    const uint64_t count = (r_hi >= r_lo && p.ph) ? (uint64_t)(r_hi - r_lo + 1) * p.in_w : 0;

    // Stage the contiguous input range; shared and global addresses share
    // their offset mod 16 so the middle moves as 128-bit words.
    const int16_t* src = x + plane * (uint64_t)p.in_h * p.in_w + (uint64_t)r_lo * p.in_w;
    const uint32_t mis = (uint32_t)(((uintptr_t)src & 15u) >> 1);
    int16_t* tile = smem + mis;
    if (((uintptr_t)src & 1u) == 0) {
        const uint64_t head = mis ? ((uint64_t)(8 - mis) < count ? (uint64_t)(8 - mis) : count) : 0;
        const uint64_t nvec = (count - head) / 8;
        for (uint64_t i = threadIdx.x; i < head; i += blockDim.x) tile[i] = src[i];
        const uint4* s4 = (const uint4*)(src + head);
        uint4* d4 = (uint4*)(tile + head);
        for (uint64_t i = threadIdx.x; i < nvec; i += blockDim.x) d4[i] = __ldcs(s4 + i);
        for (uint64_t i = head + nvec * 8 + threadIdx.x; i < count; i += blockDim.x) tile[i] = src[i];
    } else {
        for (uint64_t i = threadIdx.x; i < count; i += blockDim.x) tile[i] = src[i];
    }
    __syncthreads();

    const uint32_t n_out = (oh1 - oh0) * p.out_w;
    int16_t* yp = y + plane * (uint64_t)p.out_h * p.out_w;
    const uint32_t in_w = p.in_w;
    for (uint32_t idx = threadIdx.x; idx < n_out; idx += blockDim.x) {
        const uint32_t q = p.fd_ow.div(idx);
        const uint32_t oh = oh0 + q, ow = idx - q * p.out_w;
        yp[(uint64_t)oh * p.out_w + ow] = pool_pixel<TYPE>(
            p, oh, ow, [&](int64_t ih, int64_t iw) { return (int32_t)tile[(uint64_t)(ih - r_lo) * in_w + iw]; });
    }
}

// Fallback when one output row's input rows do not fit in shared memory.
template <int TYPE>
__global__ void __launch_bounds__(256) pool_direct_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                          PoolP p, uint64_t total) {
    const uint64_t ohw = (uint64_t)p.out_h * p.out_w;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t plane = t / ohw;
        const uint64_t r = t - plane * ohw;
        const uint32_t oh = (uint32_t)(r / p.out_w), ow = (uint32_t)(r % p.out_w);
        const int16_t* xp = x + plane * (uint64_t)p.in_h * p.in_w;
        const uint32_t in_w = p.in_w;
        y[t] = pool_pixel<TYPE>(p, oh, ow, [&](int64_t ih, int64_t iw) { return (int32_t)__ldg(xp + (uint64_t)ih * in_w + iw); });
    }
}

template <int TYPE>
__device__ __forceinline__ void reduce_word(uint32_t& acc, int32_t v) {
    if (TYPE == P_MAX) acc = (uint32_t)max((int32_t)acc, v);
    else if (TYPE == P_AVG) acc += (uint32_t)v;
    else if (TYPE == P_LP1) acc += (uint32_t)(v < 0 ? -v : v);
    else acc += (uint32_t)(v * v);
}

// Global pools: warp per plane.  Sums are formed on raw words and scaled by
// 2^8 afterwards (the same value mod 2^32); MAX keeps the largest word.
template <int TYPE>
__global__ void __launch_bounds__(256) pool_global_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                          uint64_t planes, uint32_t hw) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t plane = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; plane < planes; plane += warps) {
        const int16_t* xp = x + plane * hw;
        uint32_t acc = (TYPE == P_MAX) ? 0xFFFF8000u : 0u;   // MAX starts at the smallest word
        if (((uintptr_t)xp & 15u) == 0) {
            const uint32_t nvec = hw / 8;
            const uint4* x4 = (const uint4*)xp;
            for (uint32_t i = lane; i < nvec; i += 32) {
                const uint4 v = __ldcs(x4 + i);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    reduce_word<TYPE>(acc, (int32_t)(int16_t)(w[j] & 0xFFFF));
                    reduce_word<TYPE>(acc, (int32_t)(int16_t)(w[j] >> 16));
                }
            }
            for (uint32_t i = nvec * 8 + lane; i < hw; i += 32) reduce_word<TYPE>(acc, xp[i]);
        } else {
            for (uint32_t i = lane; i < hw; i += 32) reduce_word<TYPE>(acc, xp[i]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, acc, o);
            if (TYPE == P_MAX) acc = (uint32_t)max((int32_t)acc, (int32_t)other);
            else acc += other;
        }
        if (lane == 0) {
            uint32_t a;
            if (TYPE == P_MAX) a = hw ? (uint32_t)((int32_t)acc * 256) : 0x80000000u;
            else if (TYPE == P_LP2) a = acc;
            else a = acc * 256u;
            y[plane] = finalize<TYPE>(a, hw);
        }
    }
}

constexpr size_t kSmemBudget = 48 * 1024;

template <int TYPE>
int launch(const Context* cx, const int16_t* x, int16_t* y, uint64_t planes, const PoolP& p0, bool global,
           cudaStream_t s) {
    if (global) {
        const unsigned grid = grid_for(cx, planes * 32, 256, 8);
        {
            ProfScope ps_(PK_POOL, s);
            pool_global_kernel<TYPE><<<grid, 256, 0, s>>>(x, y, planes, p0.in_h * p0.in_w);
        }
        count_launch();
        return CM_OK;
    }
    PoolP p = p0;
    const uint64_t win_rows = (uint64_t)(p.ph ? p.ph - 1 : 0) * p.dh + 1;
    const uint64_t max_rows = (kSmemBudget - 16) / 2 / (p.in_w ? p.in_w : 1);
    if (win_rows <= max_rows && p.in_w > 0) {
        uint64_t band = p.out_h;
        if (p.sh > 0) band = std::min<uint64_t>(band, (max_rows - win_rows) / p.sh + 1);
        if (band == 0) band = 1;
        p.band_rows = (uint32_t)band;
        p.n_bands = (uint32_t)((p.out_h + band - 1) / band);
        p.fd_ow = FastDiv(p.out_w);
        const uint64_t rows_needed = std::min<uint64_t>((uint64_t)(band - 1) * p.sh + win_rows, p.in_h ? p.in_h : 1);
        const size_t smem = (size_t)rows_needed * p.in_w * 2 + 16;
        const uint64_t blocks = planes * p.n_bands;
        if (blocks >= (1ull << 31)) return set_error(CM_EUNSUPPORTED, "cm_pool: too many planes");
        {
            ProfScope ps_(PK_POOL, s);
            pool_window_kernel<TYPE><<<(unsigned)blocks, 256, smem, s>>>(x, y, p);
        }
    } else {
        const uint64_t total = planes * p.out_h * p.out_w;
        {
            ProfScope ps_(PK_POOL, s);
            pool_direct_kernel<TYPE><<<grid_for(cx, total, 256, 8), 256, 0, s>>>(x, y, p, total);
        }
    }
    count_launch();
    return CM_OK;
}

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_pool_async(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                             unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                             unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                             unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                             unsigned count_include_pad, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    const uint64_t planes = (uint64_t)batch * channels;
    if (planes == 0 || out_h == 0 || out_w == 0) return CM_OK;
    if (!y || (!x && (uint64_t)in_h * in_w > 0)) return set_error(CM_EINVAL, "cm_pool: null buffer");
    if ((uint64_t)out_h * out_w >= (1ull << 32)) return set_error(CM_EUNSUPPORTED, "cm_pool: output plane too large");
    PoolP p{};
    p.in_h = in_h; p.in_w = in_w; p.out_h = out_h; p.out_w = out_w; p.ph = pool_h; p.pw = pool_w;
    p.sh = stride_h; p.sw = stride_w; p.pt = pad_top; p.pl = pad_left; p.dh = dil_h; p.dw = dil_w;
    p.cip = count_include_pad ? 1u : 0u;
    const bool global = pad_top == 0 && pad_left == 0 && pool_h == in_h && pool_w == in_w && out_h == 1 &&
                        out_w == 1 && (dil_h == 1 || pool_h <= 1) && (dil_w == 1 || pool_w <= 1) &&
                        (uint64_t)in_h * in_w > 0 && (uint64_t)in_h * in_w < (1ull << 31);
    cudaStream_t s = (cudaStream_t)stream;
    if (pool_type == CM_POOL_MAX) rc = launch<P_MAX>(cx, x, y, planes, p, global, s);
    else if (pool_type == CM_POOL_AVG) rc = launch<P_AVG>(cx, x, y, planes, p, global, s);
    else if (lp_order == 1u) rc = launch<P_LP1>(cx, x, y, planes, p, global, s);
    else rc = launch<P_LP2>(cx, x, y, planes, p, global, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_pool launch");
}

extern "C" int cm_pool(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                       unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                       unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left, unsigned dil_h,
                       unsigned dil_w, unsigned pool_type, unsigned lp_order, unsigned count_include_pad) {
    int rc = cm_pool_async(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
                           pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad, nullptr);
    return rc ? rc : finish_sync(nullptr);
}
