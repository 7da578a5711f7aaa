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

#include "cm_async.cuh"

namespace cm {
namespace {

enum { P_MAX = 0, P_AVG = 1, P_LP1 = 2, P_LP2 = 3 };

// AccData_t(float f) on the raw Q16.16 word.
__device__ __forceinline__ uint32_t acc_from_float(float f) {
    if (isnan(f)) return 0u;
    const float t = __fmul_rn(f, 65536.0f);          // exact scale; |t| <= 2^31 here
    if (t >= 2147483648.0f) return 0x80000000u;       // +2^31 wraps to -2^31 (AP_WRAP)
    return (uint32_t)__float2int_rd(t);               // floor
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
    uint32_t band_rows, n_bands, pitch, off0, buf_elems, row_groups, strips;
    FastDiv fd_ow, fd_vpr, fd_strips;
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

// Window kernel (persistent, double-buffered).  Work item = (plane, band of
// output rows).  A band's input rows [ih_lo, ih_lo + rows) and columns
// [-pad_left, ...) are staged in shared memory as a padded tile whose
// out-of-range cells hold the window identity (-128.0 for MAX, 0 otherwise), so
// taps need no bounds checks.  Column iw lives at tile column off0 + iw with
// off0 a multiple of 8, so 16-byte-aligned input rows are copied with 16-byte
// cp.async; each CTA fetches its next item into the second buffer while it
// computes the current one.  PH..DW > 0 fix the window geometry at compile time
// (fully unrolled taps with immediate offsets); 0 means "from p".
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int TYPE, int PH, int PW, int SH, int SW, int DH, int DW, int PL>
__global__ void __launch_bounds__(256) pool_stream_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                          PoolP p, uint64_t items, uint32_t aligned) {
    griddep_wait();
    extern __shared__ __align__(16) int16_t smem[];
    __shared__ float inv_tab[65];
    const uint32_t ph = PH ? PH : p.ph, pw = PW ? PW : p.pw;
    const uint32_t sh = SH ? SH : p.sh, sw = SW ? SW : p.sw;
    const uint32_t dh = DH ? DH : p.dh, dw = DW ? DW : p.dw;
    const uint32_t pitch = p.pitch, off0 = p.off0, in_w = p.in_w;
    const int16_t pad = (TYPE == P_MAX) ? (int16_t)-32768 : (int16_t)0;
    if (TYPE == P_AVG && threadIdx.x < 65) inv_tab[threadIdx.x] = threadIdx.x ? __fdiv_rn(1.0f, (float)threadIdx.x) : 0.0f;

    // Stage item `it` into `tile`: identity margins with plain stores, input rows
    // with cp.async (committed as one group) or plain copies when misaligned.
    auto issue = [&](uint64_t it, uint32_t tb) {   // tb: element offset of the tile buffer in smem
        const uint64_t plane = it / p.n_bands;
        const uint32_t band = (uint32_t)(it - plane * p.n_bands);
        const uint32_t oh0 = band * p.band_rows, oh1 = min(p.out_h, oh0 + p.band_rows);
        const int32_t ih_lo = (int32_t)(oh0 * sh) - (int32_t)p.pt;
        const uint32_t rows = (oh1 - 1 - oh0) * sh + (ph - 1) * dh + 1;
        const int32_t t_lo = max(0, -ih_lo);
        const int32_t t_hi = max(t_lo, min((int32_t)rows, (int32_t)p.in_h - ih_lo));
        const uint32_t lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
        for (uint32_t tr = threadIdx.x >> 5; tr < rows; tr += nwarps) {
            const uint32_t trow = tb + tr * pitch;
            if ((int32_t)tr < t_lo || (int32_t)tr >= t_hi) {
                for (uint32_t c = lane; c < pitch; c += 32) smem[trow + c] = pad;
            } else {
                for (uint32_t c = lane; c < off0; c += 32) smem[trow + c] = pad;
                for (uint32_t c = off0 + in_w + lane; c < pitch; c += 32) smem[trow + c] = pad;
            }
        }
        const int16_t* src = x + plane * (uint64_t)p.in_h * in_w + (uint64_t)(ih_lo + t_lo) * in_w;
        const uint32_t nrow = (uint32_t)(t_hi - t_lo);
        if (aligned) {
            const uint32_t vpr = in_w / 8, total = nrow * vpr;
            for (uint32_t i = threadIdx.x; i < total; i += blockDim.x) {
                const uint32_t r = p.fd_vpr.div(i), c8 = i - r * vpr;
                cp_async16(&smem[tb + (t_lo + r) * pitch + off0 + 8 * c8], src + 8 * (uint64_t)i);
            }
        } else {
            for (uint32_t i = threadIdx.x; i < nrow * in_w; i += blockDim.x) {
                const uint32_t r = i / in_w, c = i - r * in_w;
                smem[tb + (t_lo + r) * pitch + off0 + c] = src[i];
            }
        }
        cp_async_commit();
    };

    // Compute item `it` from tile buffer `tb`.  Thread t owns output column ow of
    // row group g (t = g*out_w + ow) and walks that group's consecutive output
    // rows, so per output there are only the taps and two pointer increments.
    auto compute = [&](uint64_t it, uint32_t tb) {
        const uint64_t plane = it / p.n_bands;
        const uint32_t band = (uint32_t)(it - plane * p.n_bands);
        const uint32_t oh0 = band * p.band_rows, oh1 = min(p.out_h, oh0 + p.band_rows);
        const uint32_t nr = oh1 - oh0, G = p.row_groups;
        const uint32_t rpg = (nr + G - 1) / G;
        const uint32_t rowstep = dh * pitch, advance = sh * pitch;
        for (uint32_t t = threadIdx.x; t < G * p.out_w; t += blockDim.x) {
            const uint32_t g = p.fd_ow.div(t), ow = t - g * p.out_w;
            const uint32_t r0 = g * rpg, r1 = min(nr, r0 + rpg);
            if (r0 >= r1) continue;
            uint32_t base = tb + r0 * advance + off0 - p.pl + ow * sw;
            int16_t* yo = y + plane * (uint64_t)p.out_h * p.out_w + (uint64_t)(oh0 + r0) * p.out_w + ow;
            uint32_t vc = pw;       // AVG without padding in the divisor: valid columns of this ow
            if (TYPE == P_AVG && !p.cip) {
                vc = 0;
                for (uint32_t c = 0; c < pw; ++c) {
                    const int32_t iw = (int32_t)(ow * sw + c * dw) - (int32_t)p.pl;
                    vc += (iw >= 0 && iw < (int32_t)in_w);
                }
            }
            // Window reduction of output row q (tile offset b); compile-time windows
            // gather all taps first and reduce them as a tree to keep chains short.
            auto reduce = [&](uint32_t b) -> uint32_t {
                if constexpr (PH > 0 && PW > 0) {
                    int32_t v[(PH * PW > 0) ? PH * PW : 1];
#pragma unroll
                    for (uint32_t r = 0; r < (uint32_t)PH; ++r)
#pragma unroll
                        for (uint32_t c = 0; c < (uint32_t)PW; ++c) v[r * PW + c] = smem[b + r * rowstep + c * dw];
#pragma unroll
                    for (uint32_t i = 0; i < PH * PW; ++i) {
                        if (TYPE == P_LP1) v[i] = v[i] < 0 ? -v[i] : v[i];
                        else if (TYPE == P_LP2) v[i] = v[i] * v[i];
                    }
#pragma unroll
                    for (uint32_t w = 1; w < PH * PW; w *= 2)
#pragma unroll
                        for (uint32_t i = 0; i + w < PH * PW; i += 2 * w)
                            v[i] = (TYPE == P_MAX) ? max(v[i], v[i + w]) : (int32_t)((uint32_t)v[i] + (uint32_t)v[i + w]);
                    return (TYPE == P_MAX) ? (uint32_t)(v[0] * 256) : (TYPE == P_LP2 ? (uint32_t)v[0] : (uint32_t)v[0] * 256u);
                } else {
                    int32_t m = -32768;
                    uint32_t sum = 0;
                    for (uint32_t r = 0; r < ph; ++r) {
                        const uint32_t row = b + r * rowstep;
                        for (uint32_t c = 0; c < pw; ++c) {
                            const int32_t x1 = smem[row + c * dw];
                            if (TYPE == P_MAX) m = max(m, x1);
                            else if (TYPE == P_AVG) sum += (uint32_t)x1;
                            else if (TYPE == P_LP1) sum += (uint32_t)(x1 < 0 ? -x1 : x1);
                            else sum += (uint32_t)(x1 * x1);
                        }
                    }
                    return (TYPE == P_MAX) ? (uint32_t)(m * 256) : (TYPE == P_LP2 ? sum : sum * 256u);
                }
            };
            auto emit = [&](uint32_t acc, uint32_t q) -> int16_t {
                if (TYPE == P_AVG) {
                    uint32_t denom = ph * pw;
                    if (!p.cip) {
                        uint32_t vr = 0;
                        const int32_t ihq = (int32_t)((oh0 + q) * sh) - (int32_t)p.pt;
#pragma unroll
                        for (uint32_t r = 0; r < (PH ? (uint32_t)PH : ph); ++r) {
                            const int32_t ih = ihq + (int32_t)(r * dh);
                            vr += (ih >= 0 && ih < (int32_t)p.in_h);
                        }
                        denom = vr * vc;
                    }
                    const float inv = denom <= 64u ? inv_tab[denom] : __fdiv_rn(1.0f, __uint2float_rn(denom));
                    return narrow_acc(acc_from_float(__fmul_rn(acc_to_float(acc), inv)));
                }
                return finalize<TYPE>(acc, 0);
            };
            uint32_t q = r0;
            for (; q + 2 <= r1; q += 2, base += 2 * advance, yo += 2 * p.out_w) {
                const uint32_t a0 = reduce(base), a1 = reduce(base + advance);
                yo[0] = emit(a0, q);
                yo[p.out_w] = emit(a1, q + 1);
            }
            if (q < r1) *yo = emit(reduce(base), q);
        }
    };

    // Strip compute for compile-time geometry (PL >= 0): thread = V = 8/SW
    // consecutive outputs of one row group.  Their taps lie in NC aligned 16-byte
    // chunks per tap row, loaded whole; taps are picked from registers at
    // compile-time positions, so each output costs ~NC*PH/V shared loads.
    constexpr bool VEC = PL >= 0 && PH > 0 && PW > 0 && SW > 0 && DW > 0 && (8 % (SW > 0 ? SW : 1)) == 0;
    constexpr int V = VEC ? 8 / SW : 1;
    constexpr int E = PL <= 0 ? 0 : ((PL + 7) / 8) * 8 - PL;   // tile column of output 0's first tap, mod 8
    constexpr int NC = VEC ? (E + (V - 1) * SW + (PW - 1) * DW + 8) / 8 : 1;
    auto compute_vec = [&](uint64_t it, uint32_t tb) {
        const uint64_t plane = it / p.n_bands;
        const uint32_t band = (uint32_t)(it - plane * p.n_bands);
        const uint32_t oh0 = band * p.band_rows, oh1 = min(p.out_h, oh0 + p.band_rows);
        const uint32_t nr = oh1 - oh0, G = p.row_groups, nstrips = p.strips;
        const uint32_t rpg = (nr + G - 1) / G;
        const uint32_t rowstep = DH * pitch, advance = SH * pitch;
        for (uint32_t t = threadIdx.x; t < G * nstrips; t += blockDim.x) {
            const uint32_t g = p.fd_strips.div(t), j = t - g * nstrips;
            const uint32_t r0 = g * rpg, r1 = min(nr, r0 + rpg);
            if (r0 >= r1) continue;
            const uint32_t ow0 = j * V;
            uint32_t base = tb + r0 * advance + 8 * j;   // chunk holding tile column E + 8j: 16-byte aligned
            int16_t* yo = y + plane * (uint64_t)p.out_h * p.out_w + (uint64_t)(oh0 + r0) * p.out_w + ow0;
            const uint32_t nv = min((uint32_t)V, p.out_w - ow0);
            uint32_t vc[V];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                vc[v] = PW;
                if (TYPE == P_AVG && !p.cip) {
                    vc[v] = 0;
#pragma unroll
                    for (int c = 0; c < PW; ++c) {
                        const int32_t iw = (int32_t)((ow0 + v) * SW + c * DW) - PL;
                        vc[v] += (iw >= 0 && iw < (int32_t)in_w);
                    }
                }
            }
            for (uint32_t q = r0; q < r1; ++q, base += advance, yo += p.out_w) {
                int32_t acc[V];
#pragma unroll
                for (int v = 0; v < V; ++v) acc[v] = (TYPE == P_MAX) ? -32768 : 0;
#pragma unroll
                for (int r = 0; r < PH; ++r) {
                    uint32_t w[NC * 4];
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        const uint4 u = *(const uint4*)&smem[base + r * rowstep + 8 * c];
                        w[4 * c] = u.x; w[4 * c + 1] = u.y; w[4 * c + 2] = u.z; w[4 * c + 3] = u.w;
                    }
#pragma unroll
                    for (int v = 0; v < V; ++v)
#pragma unroll
                        for (int c = 0; c < PW; ++c) {
                            const int idx = E + v * SW + c * DW;
                            const int32_t x1 = (int32_t)(int16_t)((w[idx >> 1] >> (16 * (idx & 1))) & 0xFFFFu);
                            if (TYPE == P_MAX) acc[v] = max(acc[v], x1);
                            else if (TYPE == P_AVG) acc[v] += x1;
                            else if (TYPE == P_LP1) acc[v] += (x1 < 0 ? -x1 : x1);
                            else acc[v] = (int32_t)((uint32_t)acc[v] + (uint32_t)(x1 * x1));
                        }
                }
                uint32_t vr = PH;
                if (TYPE == P_AVG && !p.cip) {
                    vr = 0;
                    const int32_t ihq = (int32_t)((oh0 + q) * SH) - (int32_t)p.pt;
#pragma unroll
                    for (int r = 0; r < PH; ++r) {
                        const int32_t ih = ihq + r * DH;
                        vr += (ih >= 0 && ih < (int32_t)p.in_h);
                    }
                }
                int16_t out[V];
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    uint32_t a;
                    if (TYPE == P_MAX) a = (uint32_t)(acc[v] * 256);
                    else if (TYPE == P_LP2) a = (uint32_t)acc[v];
                    else a = (uint32_t)acc[v] * 256u;
                    if (TYPE == P_AVG) {
                        const uint32_t denom = p.cip ? PH * PW : vr * vc[v];
                        const float inv = inv_tab[denom];
                        out[v] = narrow_acc(acc_from_float(__fmul_rn(acc_to_float(a), inv)));
                    } else {
                        out[v] = finalize<TYPE>(a, 0);
                    }
                }
                if (nv == (uint32_t)V && V == 4 && ((uintptr_t)yo & 7u) == 0) {
                    *(uint2*)yo = make_uint2((uint32_t)(uint16_t)out[0] | ((uint32_t)(uint16_t)out[1 % V] << 16),
                                             (uint32_t)(uint16_t)out[2 % V] | ((uint32_t)(uint16_t)out[3 % V] << 16));
                } else {
#pragma unroll
                    for (int v = 0; v < V; ++v)
                        if ((uint32_t)v < nv) yo[v] = out[v];
                }
            }
        }
    };

    uint32_t cur = 0, other = p.buf_elems;
    uint64_t it = blockIdx.x;
    if (it < items) issue(it, cur);
    for (; it < items; it += gridDim.x) {
        const uint64_t nxt = it + gridDim.x;
        if (nxt < items) issue(nxt, other);
        else cp_async_commit();            // empty group keeps the wait count uniform
        cp_async_wait1();                  // item `it` has landed
        __syncthreads();
        if (VEC) compute_vec(it, cur);
        else compute(it, cur);
        __syncthreads();                   // the buffer may be refilled next
        const uint32_t t = cur; cur = other; other = t;
    }
}

// Row-streaming kernel for compile-time geometries (no shared memory).
// Thread = (plane, strip j of V = 8/SW consecutive outputs).  Each input row the
// strip needs is read once: one coalesced 16-byte load of input columns
// [8j, 8j+8), plus PL columns on the left and HR on the right taken from the
// neighbouring lanes' loads by warp shuffle (a direct 2-byte load at warp
// edges; the window identity outside the plane).  The row's horizontal window
// reductions for the V outputs go into a register ring over the progression of
// tap rows (spaced DH); consecutive output rows advance it by SH/DH rows, so a
// row shared by two output rows is reduced once.
template <int TYPE, int PH, int PW, int SH, int SW, int DH, int DW, int PT, int PL>
__global__ void __launch_bounds__(256) pool_rows_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                        PoolP p, uint64_t total) {
    griddep_wait();
    constexpr int V = 8 / SW;
    constexpr int SPAN = (V - 1) * SW + (PW - 1) * DW + 1;   // input columns under the strip
    constexpr int HR = SPAN - PL - 8 > 0 ? SPAN - PL - 8 : 0;
    constexpr int ADV = SH / DH;                             // new tap rows per output row
    static_assert(SH % DH == 0 && PL <= 8 && HR <= 8 && V * SW == 8, "geometry");
    __shared__ float inv_tab[PH * PW + 1];
    if (TYPE == P_AVG && threadIdx.x <= PH * PW) inv_tab[threadIdx.x] = threadIdx.x ? __fdiv_rn(1.0f, (float)threadIdx.x) : 0.0f;
    __syncthreads();

    const int32_t pad = (TYPE == P_MAX) ? -32768 : 0;
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool live = t < total;
    const uint64_t tt = live ? t : total - 1;                // inactive lanes mirror a real strip
    const uint32_t nstrips = p.strips;
    const uint64_t plane = tt / nstrips;
    const uint32_t j = (uint32_t)(tt - plane * nstrips);
    const uint32_t in_w = p.in_w, in_h = p.in_h;
    const int16_t* xp = x + plane * (uint64_t)in_h * in_w + 8 * j;
    const bool first = j == 0, last = j == nstrips - 1;

    // Input row ih of this strip: one 16-byte load (zeros outside the plane).
    auto lrow = [&](int32_t ih) -> uint4 {
        uint4 c = make_uint4(0, 0, 0, 0);
        if (ih >= 0 && ih < (int32_t)in_h) c = __ldcs((const uint4*)(xp + (uint64_t)ih * in_w));
        return c;
    };
    // Horizontal reductions of input row ih (loaded as c) for this strip's V outputs.
    auto hrow = [&](int32_t ih, uint4 c, int32_t (&h)[V]) {
        const bool ok = ih >= 0 && ih < (int32_t)in_h;
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        int32_t e[SPAN];
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (PL + k < SPAN) e[PL + k] = ok ? (int32_t)(int16_t)(w[k >> 1] >> (16 * (k & 1))) : pad;
        if (PL > 0) {
            const uint32_t nb = __shfl_up_sync(0xFFFFFFFFu, c.w, 1);           // left neighbour's columns 6, 7
            const uint32_t nb2 = __shfl_up_sync(0xFFFFFFFFu, c.z, 1);          // columns 4, 5
#pragma unroll
            for (int k = 0; k < PL; ++k) {
                const int col = 8 - PL + k;                                    // column in the left chunk
                int32_t v = pad;
                if (ok && !first) {
                    if (lane > 0) v = (int32_t)(int16_t)((col >= 6 ? nb : nb2) >> (16 * (col & 1)));
                    else v = xp[(int64_t)ih * in_w - 8 + col];
                }
                e[k] = v;
            }
        }
        if (HR > 0) {
            const uint32_t nb = __shfl_down_sync(0xFFFFFFFFu, c.x, 1);         // right neighbour's columns 0, 1
            const uint32_t nb2 = __shfl_down_sync(0xFFFFFFFFu, c.y, 1);        // columns 2, 3
#pragma unroll
            for (int k = 0; k < HR; ++k) {
                int32_t v = pad;
                if (ok && !last) {
                    if (lane < 31) v = (int32_t)(int16_t)((k >= 2 ? nb2 : nb) >> (16 * (k & 1)));
                    else v = xp[(int64_t)ih * in_w + 8 + k];
                }
                e[PL + 8 + k] = v;
            }
        }
#pragma unroll
        for (int v = 0; v < V; ++v) {
            int32_t a = (TYPE == P_MAX) ? -32768 : 0;
#pragma unroll
            for (int c2 = 0; c2 < PW; ++c2) {
                const int32_t x1 = e[v * SW + c2 * DW];
                if (TYPE == P_MAX) a = max(a, x1);
                else if (TYPE == P_AVG) a += x1;
                else if (TYPE == P_LP1) a += (x1 < 0 ? -x1 : x1);
                else a = (int32_t)((uint32_t)a + (uint32_t)(x1 * x1));
            }
            h[v] = a;
        }
    };

    uint32_t vc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        vc[v] = PW;
        if (TYPE == P_AVG && !p.cip) {
            vc[v] = 0;
#pragma unroll
            for (int c2 = 0; c2 < PW; ++c2) {
                const int32_t iw = (int32_t)((8 * j / SW + v) * SW + c2 * DW) - PL;
                vc[v] += (iw >= 0 && iw < (int32_t)in_w);
            }
        }
    }
    const uint32_t ow0 = j * V;
    const uint32_t nv = ow0 < p.out_w ? min((uint32_t)V, p.out_w - ow0) : 0u;
    int16_t* yo = y + plane * (uint64_t)p.out_h * p.out_w + ow0;

    // Rows entering the ring at output row oh: tap rows r = PH-ADV .. PH-1.
    constexpr int NEW = ADV < PH ? ADV : PH;
    auto new_row = [&](uint32_t oh, int i) -> int32_t { return (int32_t)(oh * SH) - PT + (PH - NEW + i) * DH; };
    int32_t ring[PH][V];
#pragma unroll
    for (int r = 0; r < PH; ++r) hrow(-PT + r * DH, lrow(-PT + r * DH), ring[r]);
    uint4 ahead[NEW];                                        // loads for the next output row, in flight
#pragma unroll
    for (int i = 0; i < NEW; ++i) ahead[i] = lrow(new_row(1, i));
    for (uint32_t oh = 0; oh < p.out_h; ++oh) {
        if (oh > 0) {
            uint4 cur[NEW];
#pragma unroll
            for (int i = 0; i < NEW; ++i) cur[i] = ahead[i];
#pragma unroll
            for (int i = 0; i < NEW; ++i) ahead[i] = lrow(oh + 1 < p.out_h ? new_row(oh + 1, i) : -1);
#pragma unroll
            for (int r = 0; r + ADV < PH; ++r)
#pragma unroll
                for (int v = 0; v < V; ++v) ring[r][v] = ring[r + ADV][v];
#pragma unroll
            for (int i = 0; i < NEW; ++i) hrow(new_row(oh, i), cur[i], ring[PH - NEW + i]);
        }
        uint32_t vr = PH;
        if (TYPE == P_AVG && !p.cip) {
            vr = 0;
#pragma unroll
            for (int r = 0; r < PH; ++r) {
                const int32_t ih = (int32_t)(oh * SH) - PT + r * DH;
                vr += (ih >= 0 && ih < (int32_t)in_h);
            }
        }
        int16_t out[V];
#pragma unroll
        for (int v = 0; v < V; ++v) {
            int32_t a = ring[0][v];
#pragma unroll
            for (int r = 1; r < PH; ++r) {
                if (TYPE == P_MAX) a = max(a, ring[r][v]);
                else a = (int32_t)((uint32_t)a + (uint32_t)ring[r][v]);
            }
            uint32_t acc;
            if (TYPE == P_MAX) acc = (uint32_t)(a * 256);
            else if (TYPE == P_LP2) acc = (uint32_t)a;
            else acc = (uint32_t)a * 256u;
            if (TYPE == P_AVG) {
                const uint32_t denom = p.cip ? PH * PW : vr * vc[v];
                out[v] = narrow_acc(acc_from_float(__fmul_rn(acc_to_float(acc), inv_tab[denom])));
            } else {
                out[v] = finalize<TYPE>(acc, 0);
            }
        }
        if (live) {
            int16_t* dst = yo + (uint64_t)oh * p.out_w;
            if (nv == (uint32_t)V && V == 4 && ((uintptr_t)dst & 7u) == 0) {
                *(uint2*)dst = make_uint2((uint32_t)(uint16_t)out[0] | ((uint32_t)(uint16_t)out[1 % V] << 16),
                                          (uint32_t)(uint16_t)out[2 % V] | ((uint32_t)(uint16_t)out[3 % V] << 16));
            } else {
#pragma unroll
                for (int v = 0; v < V; ++v)
                    if ((uint32_t)v < nv) dst[v] = out[v];
            }
        }
    }
}

// Whole-plane kernel for compile-time geometries whose input plane fits in
// shared memory (at most kPlaneMax bytes, rows of a multiple of 8 columns).
// Persistent CTAs walk the planes.  Warp 0 is the producer: each plane arrives
// as ONE bulk copy on the TMA engine (a long sequential DRAM stream) into one
// of kPlaneBufs buffers, issued as soon as every consumer thread has released
// that buffer (full / empty mbarriers, no CTA-wide barrier).  A buffer holds
// the plane between rows of window-identity cells (PT above, the rows the last
// output row reaches below), written once per CTA, so only the strips at the
// plane's left and right edges check their halo columns.  The other threads
// are (band of output rows, strip j of V = 8/SW outputs): per input row one
// 16-byte shared-memory read of columns [8j, 8j+8) plus PL / HR halo columns and
// the horizontal window reductions, kept in a ring over the PH tap rows so that
// a row shared by consecutive output rows of the band is reduced once.
constexpr uint32_t kPlaneMax = 28 * 1024;
constexpr uint32_t kPlaneBufs = 2;

template <int TYPE, int PH, int PW, int SH, int SW, int DH, int DW, int PT, int PL>
__global__ void __launch_bounds__(512) pool_plane_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y, PoolP p,
                                                         uint64_t planes, uint32_t buf_bytes, uint32_t rows_bot,
                                                         int* status, uint64_t timeout_ns) {
    griddep_wait();
    constexpr int V = 8 / SW;
    constexpr int SPAN = (V - 1) * SW + (PW - 1) * DW + 1;   // input columns under the strip
    constexpr int HR = SPAN - PL - 8 > 0 ? SPAN - PL - 8 : 0;
    constexpr int ADV = SH / DH;                             // new tap rows per output row
    constexpr int NEW = ADV < PH ? ADV : PH;
    static_assert(PL <= 8 && HR <= 8 && V * SW == 8 && SH % DH == 0, "geometry");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ uint64_t full_b[kPlaneBufs], empty_b[kPlaneBufs];
    __shared__ float inv_tab[PH * PW + 1];
    __shared__ int abort_flag;
    const int32_t pad = (TYPE == P_MAX) ? -32768 : 0;
    const uint32_t in_w = p.in_w, in_h = p.in_h;
    const uint32_t plane_elems = in_h * in_w, plane_bytes = plane_elems * 2;
    const uint64_t out_elems = (uint64_t)p.out_h * p.out_w;
    const uint32_t consumers = blockDim.x - 32;
    // window identity in the frame rows of every buffer
    for (uint32_t b = 0; b < kPlaneBufs; ++b) {
        int16_t* bp = (int16_t*)(smem_raw + b * buf_bytes);
        for (uint32_t i = threadIdx.x; i < (PT + rows_bot) * in_w; i += blockDim.x)
            bp[i < PT * in_w ? i : plane_elems + i] = (int16_t)pad;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        for (uint32_t b = 0; b < kPlaneBufs; ++b) {
            mbar_init(smem_u32(&full_b[b]), 1);
            mbar_init(smem_u32(&empty_b[b]), consumers);
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (TYPE == P_AVG && threadIdx.x <= PH * PW) inv_tab[threadIdx.x] = threadIdx.x ? __fdiv_rn(1.0f, (float)threadIdx.x) : 0.0f;
    __syncthreads();
    const WaitCtl wc{&abort_flag, status, timeout_ns};

    if (threadIdx.x < 32) {
        const uint32_t lane = threadIdx.x;
        uint32_t k = 0;
        if (lane == 0) {
            for (uint64_t plane = blockIdx.x; plane < planes; plane += gridDim.x, ++k) {
                const uint32_t b = k % kPlaneBufs;
                if (k >= kPlaneBufs && !mbar_wait(smem_u32(&empty_b[b]), ((k / kPlaneBufs) - 1) & 1u, wc)) break;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                const uint32_t bar = smem_u32(&full_b[b]);
                mbar_expect_tx(bar, plane_bytes);
                bulk_g2s(smem_u32(smem_raw + b * buf_bytes) + PT * in_w * 2, x + plane * plane_elems, plane_bytes, bar);
            }
        }
        if (lane == 0) {
            if (abort_flag) {
                // let the copies still in flight land before the CTA's shared memory is released
                volatile int never = 0;
                const WaitCtl drain{&never, status, timeout_ns};
                for (uint32_t q = k > kPlaneBufs ? k - kPlaneBufs : 0u; q < k; ++q)
                    mbar_wait(smem_u32(&full_b[q % kPlaneBufs]), (q / kPlaneBufs) & 1u, drain);
            }
        }
        return;
    }

    // consumer thread = (band bnd of p.band_rows output rows, strip j)
    const uint32_t ct = threadIdx.x - 32;
    const uint32_t nstrips = p.strips;
    const uint32_t j = ct % nstrips, bnd = ct / nstrips;
    const uint32_t oh0 = bnd * p.band_rows, oh1 = min(p.out_h, oh0 + p.band_rows);
    const bool first = j == 0, last = j == nstrips - 1;
    const uint32_t ow0 = j * V;
    const uint32_t nv = ow0 < p.out_w ? min((uint32_t)V, p.out_w - ow0) : 0u;
    uint32_t vc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
        vc[v] = PW;
        if (TYPE == P_AVG && !p.cip) {
            vc[v] = 0;
#pragma unroll
            for (int c2 = 0; c2 < PW; ++c2) {
                const int32_t iw = (int32_t)((ow0 + v) * SW + c2 * DW) - PL;
                vc[v] += (iw >= 0 && iw < (int32_t)in_w);
            }
        }
    }

    // AVG: this strip's reciprocals for rows whose PH taps are all inside the plane (all
    // but the first and last output rows), kept in registers
    float inv_in[V];
#pragma unroll
    for (int v = 0; v < V; ++v) inv_in[v] = TYPE == P_AVG ? inv_tab[p.cip ? PH * PW : PH * vc[v]] : 0.0f;
    // output rows whose PH taps all lie inside the plane: oh_in0 <= oh <= oh_in1
    constexpr int32_t oh_in0 = (PT + SH - 1) / SH;
    const int32_t last_ok = (int32_t)p.in_h - 1 + PT - (PH - 1) * DH;
    const int32_t oh_in1 = last_ok < 0 ? -1 : last_ok / SH;

    uint32_t k = 0;
    for (uint64_t plane = blockIdx.x; plane < planes; plane += gridDim.x, ++k) {
        const uint32_t b = k % kPlaneBufs;
        if (!mbar_wait(smem_u32(&full_b[b]), (k / kPlaneBufs) & 1u, wc)) break;
        // element (ih, iw) of the plane; rows -PT.. and in_h.. hold the identity
        const int16_t* sp = (const int16_t*)(smem_raw + b * buf_bytes) + PT * in_w;
        int16_t* yp = y + plane * out_elems;
        // Horizontal reductions of input row ih for this strip's V outputs.
        auto hrow = [&](int32_t ih, int32_t (&h)[V]) {
            const int16_t* row = sp + ih * (int32_t)in_w + 8 * j;
            int32_t e[SPAN];
            const uint4 c = *(const uint4*)row;
            const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (PL + q < SPAN) e[PL + q] = (int32_t)(int16_t)(w[q >> 1] >> (16 * (q & 1)));
#pragma unroll
            for (int q = 0; q < PL; ++q) e[q] = first ? pad : (int32_t)row[q - PL];
#pragma unroll
            for (int q = 0; q < HR; ++q) e[PL + 8 + q] = last ? pad : (int32_t)row[8 + q];
#pragma unroll
            for (int v = 0; v < V; ++v) {
                int32_t a = (TYPE == P_MAX) ? -32768 : 0;
#pragma unroll
                for (int c2 = 0; c2 < PW; ++c2) {
                    const int32_t x1 = e[v * SW + c2 * DW];
                    if (TYPE == P_MAX) a = max(a, x1);
                    else if (TYPE == P_AVG) a += x1;
                    else if (TYPE == P_LP1) a += (x1 < 0 ? -x1 : x1);
                    else a = (int32_t)((uint32_t)a + (uint32_t)(x1 * x1));
                }
                h[v] = a;
            }
        };
        if (oh0 < oh1) {
            int32_t ring[PH][V];
#pragma unroll
            for (int r = 0; r < PH; ++r) hrow((int32_t)(oh0 * SH) - PT + r * DH, ring[r]);
            for (uint32_t oh = oh0; oh < oh1; ++oh) {
                if (oh > oh0) {
#pragma unroll
                    for (int r = 0; r + ADV < PH; ++r)
#pragma unroll
                        for (int v = 0; v < V; ++v) ring[r][v] = ring[r + ADV][v];
#pragma unroll
                    for (int i = 0; i < NEW; ++i) hrow((int32_t)(oh * SH) - PT + (PH - NEW + i) * DH, ring[PH - NEW + i]);
                }
                const bool inner = (int32_t)oh >= oh_in0 && (int32_t)oh <= oh_in1;
                uint32_t vr = PH;
                if (TYPE == P_AVG && !p.cip && !inner) {
                    vr = 0;
#pragma unroll
                    for (int r = 0; r < PH; ++r) {
                        const int32_t ih = (int32_t)(oh * SH) - PT + r * DH;
                        vr += (ih >= 0 && ih < (int32_t)in_h);
                    }
                }
                // Results before the int16 narrowing.  With at most 3 x 3 taps the Q16.16
                // accumulator (the word sum a times 2^8) cannot wrap, and the reference's
                // power-of-two scales are exact, so (PoolingKernel.cpp:168-172, 253-263):
                //   AVG  floor(rn(float(acc) * 2^-16 * inv) at 2^-16) >> 8 = floor(rn(a * inv)),
                //        inv = rn(1 / denom)
                //   LP2  floor(sqrt_rn(rn(acc)) * 2^8) >> 8 = floor(sqrt_rn(rn(acc))) with acc the
                //        wrapped sum of squares (negative -> NaN -> 0); the root's value is at
                //        most 181, so the Q16.16 word never wraps and the narrowing saturates
                //   LP1  the sum of |x|, MAX the largest word
                // then one saturating pack per pair of outputs.
                int32_t res[V];
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    int32_t a = ring[0][v];
#pragma unroll
                    for (int r = 1; r < PH; ++r) {
                        if (TYPE == P_MAX) a = max(a, ring[r][v]);
                        else a = (int32_t)((uint32_t)a + (uint32_t)ring[r][v]);
                    }
                    if (TYPE == P_AVG) {
                        const float inv = (p.cip || inner || vr == (uint32_t)PH) ? inv_in[v] : inv_tab[vr * vc[v]];
                        res[v] = __float2int_rd(__fmul_rn(__int2float_rn(a), inv));
                    } else if (TYPE == P_LP2) {
                        res[v] = __float2int_rz(__fsqrt_rn(__int2float_rn(a)));   // NaN -> 0
                    } else {
                        res[v] = a;
                    }
                }
                int16_t* dst = yp + (uint64_t)oh * p.out_w + ow0;
                if (nv == (uint32_t)V && V == 4 && ((uintptr_t)dst & 7u) == 0) {
                    uint32_t lo, hi;
                    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(lo) : "r"(res[1 % V]), "r"(res[0]));
                    asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(hi) : "r"(res[3 % V]), "r"(res[2 % V]));
                    *(uint2*)dst = make_uint2(lo, hi);
                } else {
#pragma unroll
                    for (int v = 0; v < V; ++v)
                        if ((uint32_t)v < nv) dst[v] = sat16(res[v]);
                }
            }
        }
        mbar_arrive(smem_u32(&empty_b[b]));   // this thread is done with the buffer
    }
}

// Fallback when one output row's input rows do not fit in shared memory.
template <int TYPE>
__global__ void __launch_bounds__(256) pool_direct_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                          PoolP p, uint64_t total) {
    griddep_wait();
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
// Global pools of small planes (hw <= 512, e.g. the 7x7 maps before a classifier): a warp
// per plane would leave most lanes idle and chain its few loads; instead a block stages
// `ppb` consecutive planes (one contiguous run) in shared memory with coalesced 4-byte
// loads and thread t reduces plane t.  Same sums (mod 2^32) and maxima as the warp kernel.
template <int TYPE>
__global__ void __launch_bounds__(256) pool_global_small_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                                uint64_t planes, uint32_t hw) {
    griddep_wait();
    extern __shared__ __align__(16) int16_t sbuf[];     // blockDim.x planes x hw words
    const uint32_t ppb = blockDim.x, tid = threadIdx.x;
    for (uint64_t p0 = (uint64_t)blockIdx.x * ppb; p0 < planes; p0 += (uint64_t)gridDim.x * ppb) {
        const uint32_t np = planes - p0 < ppb ? (uint32_t)(planes - p0) : ppb;
        const uint32_t words = np * hw;
        const int16_t* src = x + p0 * hw;
        if (((uintptr_t)src & 3u) == 0) {
            const uint32_t* s4 = (const uint32_t*)src;
            for (uint32_t i = tid; i < words / 2; i += ppb) ((uint32_t*)sbuf)[i] = __ldcs(s4 + i);
            if ((words & 1u) && tid == 0) sbuf[words - 1] = src[words - 1];
        } else {
            for (uint32_t i = tid; i < words; i += ppb) sbuf[i] = __ldcs(src + i);
        }
        __syncthreads();
        if (tid < np) {
            uint32_t acc = (TYPE == P_MAX) ? 0xFFFF8000u : 0u;
            const int16_t* v = sbuf + tid * hw;
            for (uint32_t k = 0; k < hw; ++k) reduce_word<TYPE>(acc, v[k]);
            uint32_t a;
            if (TYPE == P_MAX) a = (uint32_t)((int32_t)acc * 256);
            else if (TYPE == P_LP2) a = acc;
            else a = acc * 256u;
            y[p0 + tid] = finalize<TYPE>(a, hw);
        }
        __syncthreads();
    }
}

template <int TYPE>
__global__ void __launch_bounds__(256) pool_global_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                          uint64_t planes, uint32_t hw) {
    griddep_wait();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t plane = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; plane < planes; plane += warps) {
        const int16_t* xp = x + plane * hw;
        uint32_t acc = (TYPE == P_MAX) ? 0xFFFF8000u : 0u;   // MAX starts at the smallest word
        if (((uintptr_t)xp & 15u) == 0) {
            const uint32_t nvec = hw / 8;
            const uint4* x4 = (const uint4*)xp;
            for (uint32_t i0 = lane; i0 < nvec; i0 += 4 * 32) {
                uint4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i0 + 32 * u < nvec) v[u] = __ldcs(x4 + i0 + 32 * u);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (i0 + 32 * u >= nvec) break;
                    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        reduce_word<TYPE>(acc, (int32_t)(int16_t)(w[j] & 0xFFFF));
                        reduce_word<TYPE>(acc, (int32_t)(int16_t)(w[j] >> 16));
                    }
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

// Global pools of a channels-last tensor x [images][hw][C] (C a multiple of 8, x 16-byte
// aligned): four adjacent threads take one (image, 8 consecutive channels) item, each the
// pixels p = its lane mod 4, 4 + that, ... with one 16-byte load of 8 words per pixel (up to
// 4 pixels' loads issued together); the four partial reductions meet by shuffles (sums mod
// 2^32 and maxima are order-free), and the item's first thread applies the NCHW kernels'
// finalize and stores the 8 results with one 16-byte store into y [image][C] (a global
// pool's output is the same in both layouts).
template <int TYPE>
__global__ void __launch_bounds__(256) pool_global_nhwc_kernel(const int16_t* __restrict__ x, int16_t* __restrict__ y,
                                                               uint64_t groups, uint32_t C, uint32_t hw) {
    griddep_wait();
    const uint32_t G = C / 8;
    const uint32_t sl = threadIdx.x & 3u;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x / 4;
    // whole warps iterate together (the shuffles below need every lane of an item)
    const uint64_t rounds = (groups + stride - 1) / stride;
    uint64_t t = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 4;
    for (uint64_t r = 0; r < rounds; ++r, t += stride) {
        const bool live = t < groups;
        const uint64_t n = live ? t / G : 0;
        const uint32_t c0 = live ? (uint32_t)(t - n * G) * 8u : 0u;
        const uint4* src = (const uint4*)(x + n * hw * C + c0);
        const uint32_t step = C / 8;                       // one pixel, in 16-byte units
        uint32_t acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = (TYPE == P_MAX) ? 0xFFFF8000u : 0u;
        for (uint32_t p0 = sl; live && p0 < hw; p0 += 16) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (p0 + 4 * u < hw) v[u] = __ldcs(src + (uint64_t)(p0 + 4 * u) * step);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (p0 + 4 * u >= hw) break;
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    reduce_word<TYPE>(acc[2 * j], (int32_t)(int16_t)(w[j] & 0xFFFF));
                    reduce_word<TYPE>(acc[2 * j + 1], (int32_t)(int16_t)(w[j] >> 16));
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, acc[k], o);
                if (TYPE == P_MAX) acc[k] = (uint32_t)max((int32_t)acc[k], (int32_t)other);
                else acc[k] += other;
            }
        }
        if (live && sl == 0) {
            uint32_t out[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t a0, a1;
                if (TYPE == P_MAX) { a0 = (uint32_t)((int32_t)acc[2 * j] * 256); a1 = (uint32_t)((int32_t)acc[2 * j + 1] * 256); }
                else if (TYPE == P_LP2) { a0 = acc[2 * j]; a1 = acc[2 * j + 1]; }
                else { a0 = acc[2 * j] * 256u; a1 = acc[2 * j + 1] * 256u; }
                out[j] = (uint32_t)(uint16_t)finalize<TYPE>(a0, hw) | ((uint32_t)(uint16_t)finalize<TYPE>(a1, hw) << 16);
            }
            *(uint4*)(y + n * C + c0) = make_uint4(out[0], out[1], out[2], out[3]);
        }
    }
}

// Per tile buffer (two per CTA): small enough for 8 resident CTAs per SM.
constexpr size_t kSmemBudget = 16 * 1024;

template <int TYPE>
int launch(const Context* cx, const int16_t* x, int16_t* y, uint64_t planes, const PoolP& p0, bool global,
           cudaStream_t s) {
    if (global) {
        const uint64_t hw = (uint64_t)p0.in_h * p0.in_w;
        if (hw > 0 && hw <= 512) {
            // planes per block: a power of two in [32, 256] with at most 32 KB staged
            uint32_t ppb = 256;
            while (ppb > 32 && (uint64_t)ppb * hw * 2 > 32768) ppb /= 2;
            const unsigned grid = grid_for(cx, planes, ppb, 2048 / ppb);
            {
                ProfScope ps_(PK_POOL, s);
                launch_k(pool_global_small_kernel<TYPE>, grid, ppb, (size_t)ppb * hw * 2, s, x, y, planes, (uint32_t)hw);
            }
            count_launch();
            return CM_OK;
        }
        const unsigned grid = grid_for(cx, planes * 32, 256, 8);
        {
            ProfScope ps_(PK_POOL, s);
            launch_k(pool_global_kernel<TYPE>, grid, 256, 0, s, x, y, planes, p0.in_h * p0.in_w);
        }
        count_launch();
        return CM_OK;
    }
    PoolP p = p0;
    // Padded-tile kernel when one output row's window rows fit the budget and all
    // tile offsets fit comfortably in 32 bits.
    const uint64_t win_rows = (uint64_t)(p.ph ? p.ph - 1 : 0) * p.dh + 1;
    const uint64_t off0 = ((uint64_t)p.pl + 7) & ~7ull;
    const uint64_t span = off0 - p.pl + (uint64_t)(p.out_w - 1) * p.sw + (uint64_t)(p.pw ? p.pw - 1 : 0) * p.dw + 1;
    uint64_t pitch = (std::max<uint64_t>(off0 + p.in_w, span) + 7) & ~7ull;
    // Compile-time geometries with a strip kernel: (ph, pw, sh, sw, dh, dw, pad_left).
    int spec = -1;
    const uint32_t specs[3][7] = {{3, 3, 2, 2, 1, 1, 1}, {3, 3, 2, 2, 2, 2, 1}, {2, 2, 2, 2, 1, 1, 0}};
    for (int i = 0; i < 3; ++i)
        if (p.ph == specs[i][0] && p.pw == specs[i][1] && p.sh == specs[i][2] && p.sw == specs[i][3] &&
            p.dh == specs[i][4] && p.dw == specs[i][5] && p.pl == specs[i][6])
            spec = i;
    if (spec >= 0) {
        // strips of V = 8/sw outputs read NC aligned 16-byte chunks per tap row
        const uint64_t V = 8 / p.sw, E = off0 - p.pl;
        const uint64_t NC = (E + (V - 1) * p.sw + (p.pw - 1) * p.dw + 8) / 8;
        const uint64_t nstrips = (p.out_w + V - 1) / V;
        const uint64_t need = 8 * (nstrips - 1) + 8 * NC;   // strip j reads tile columns [8j, 8j + 8 NC)
        pitch = std::max<uint64_t>(pitch, (need + 7) & ~7ull);
        p.strips = (uint32_t)nstrips;
        p.fd_strips = FastDiv(p.strips);
    }
    const bool small = p.in_h < (1u << 24) && p.in_w < (1u << 24) && p.out_h < (1u << 24) && p.pt < (1u << 24) &&
                       (uint64_t)p.sh * p.out_h < (1ull << 30) && win_rows < (1ull << 24) && pitch < (1u << 20);
    // Whole-plane kernel: compile-time geometry, the plane fits a shared-memory
    // buffer, 16-byte-aligned planes and rows, one 8-column chunk per strip.
    const uint64_t plane_bytes = (uint64_t)p.in_h * p.in_w * 2;
    if (spec >= 0 && (p.in_w & 7u) == 0 && ((uintptr_t)x & 15u) == 0 && p.in_w == 8 * p.strips && p.pt == p.pl &&
        plane_bytes > 0 && plane_bytes <= kPlaneMax && p.out_h < (1u << 16) && p.strips <= 240 &&
        (uint64_t)(p.out_h - 1) * p.sh < p.in_h + 64) {
        // consumer threads = strips x bands of `band_rows` output rows (>= 2 rows a band
        // for the row reuse), at most 480 of them next to the producer warp
        uint32_t rows = 2;
        while (p.strips * ((p.out_h + rows - 1) / rows) > 480) ++rows;
        p.band_rows = rows;
        const uint32_t threads = 32 + p.strips * ((p.out_h + rows - 1) / rows);
        // buffer: the plane framed by PT rows above, the rows the last output row reaches
        // below the plane, and 8 columns each side
        const int64_t max_ih = (int64_t)(p.out_h - 1) * p.sh - p.pt + (int64_t)(p.ph - 1) * p.dh;
        const uint32_t rows_bot = (uint32_t)std::max<int64_t>(0, max_ih - ((int64_t)p.in_h - 1));
        const uint32_t buf_bytes = (uint32_t)(((uint64_t)(p.pt + p.in_h + rows_bot) * p.in_w * 2 + 127) & ~127ull);
        const size_t smem = kPlaneBufs * (size_t)buf_bytes;
        {
            ProfScope ps_(PK_POOL, s);
#define CM_PLANE_LAUNCH(PH_, PW_, SH_, SW_, DH_, DW_, PT_, PL_)                                          \
    do {                                                                                                 \
        auto k_ = pool_plane_kernel<TYPE, PH_, PW_, SH_, SW_, DH_, DW_, PT_, PL_>;                      \
        cudaFuncSetAttribute(k_, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);               \
        int per_sm = 1;                                                                                  \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_, (int)threads, smem);                 \
        const uint64_t grid = std::min<uint64_t>(planes, (uint64_t)cx->sm_count * std::max(per_sm, 1)); \
        launch_k(k_, (unsigned)grid, threads, smem, s, x, y, p, planes, buf_bytes, rows_bot, cx->status, cx->timeout_ns); \
    } while (0)
            if (spec == 0)
                CM_PLANE_LAUNCH(3, 3, 2, 2, 1, 1, 1, 1);
            else if (spec == 1)
                CM_PLANE_LAUNCH(3, 3, 2, 2, 2, 2, 1, 1);
            else
                CM_PLANE_LAUNCH(2, 2, 2, 2, 1, 1, 0, 0);
#undef CM_PLANE_LAUNCH
        }
        count_launch();
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "pool plane kernel");
    }
    // Row-streaming kernel: compile-time geometry, 16-byte-aligned rows, and exactly
    // one 8-column input chunk per strip of V outputs.
    if (spec >= 0 && (p.in_w & 7u) == 0 && ((uintptr_t)x & 15u) == 0 && p.in_w == 8 * p.strips &&
        p.pt == p.pl && p.in_h < (1u << 24) && p.out_h < (1u << 24) && planes * p.strips < (1ull << 40)) {
        const uint64_t total = planes * p.strips;
        const uint64_t blocks = (total + 255) / 256;
        {
            ProfScope ps_(PK_POOL, s);
            if (spec == 0)
                launch_k(pool_rows_kernel<TYPE, 3, 3, 2, 2, 1, 1, 1, 1>, (unsigned)blocks, 256, 0, s, x, y, p, total);
            else if (spec == 1)
                launch_k(pool_rows_kernel<TYPE, 3, 3, 2, 2, 2, 2, 1, 1>, (unsigned)blocks, 256, 0, s, x, y, p, total);
            else
                launch_k(pool_rows_kernel<TYPE, 2, 2, 2, 2, 1, 1, 0, 0>, (unsigned)blocks, 256, 0, s, x, y, p, total);
        }
        count_launch();
        return CM_OK;
    }
    if (p.ph > 0 && p.pw > 0 && small && win_rows * pitch * 2 <= kSmemBudget) {
        // Two tile buffers per CTA (double buffering); each at most kSmemBudget / 2 ... kSmemBudget.
        uint64_t band = p.out_h;
        const uint64_t max_rows = kSmemBudget / (pitch * 2);
        if (p.sh > 0) band = std::min<uint64_t>(band, (max_rows - win_rows) / p.sh + 1);
        if (band == 0) band = 1;
        p.band_rows = (uint32_t)band;
        p.n_bands = (uint32_t)((p.out_h + band - 1) / band);
        p.pitch = (uint32_t)pitch;
        p.off0 = (uint32_t)off0;
        p.fd_ow = FastDiv(p.out_w);
        p.fd_vpr = FastDiv(std::max<uint32_t>(p.in_w / 8, 1u));
        p.row_groups = spec >= 0 ? std::max<uint32_t>(1u, 256u / p.strips) : std::max<uint32_t>(1u, 256u / p.out_w);
        const uint64_t buf_rows = (band - 1) * p.sh + win_rows;
        p.buf_elems = (uint32_t)(buf_rows * pitch);
        const size_t smem = (size_t)2 * p.buf_elems * 2;
        const uint64_t items = planes * p.n_bands;
        const uint32_t aligned = ((p.in_w & 7u) == 0 && ((uintptr_t)x & 15u) == 0) ? 1u : 0u;
        // resident CTAs per SM from the shared-memory footprint, at most 8 (2048 threads)
        const uint64_t per_sm = std::max<uint64_t>(1, std::min<uint64_t>(8, (220u * 1024u) / (smem + 1024)));
        const uint64_t grid = std::min<uint64_t>(items, (uint64_t)cx->sm_count * per_sm);
        {
            ProfScope ps_(PK_POOL, s);
#define CM_POOL_LAUNCH(PH_, PW_, SH_, SW_, DH_, DW_, PL_)                                                \
    do {                                                                                                 \
        auto k_ = pool_stream_kernel<TYPE, PH_, PW_, SH_, SW_, DH_, DW_, PL_>;                          \
        cudaFuncSetAttribute(k_, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);               \
        launch_k(k_, (unsigned)grid, 256, smem, s, x, y, p, items, aligned);                                  \
    } while (0)
            if (spec == 0)
                CM_POOL_LAUNCH(3, 3, 2, 2, 1, 1, 1);
            else if (spec == 1)
                CM_POOL_LAUNCH(3, 3, 2, 2, 2, 2, 1);
            else if (spec == 2)
                CM_POOL_LAUNCH(2, 2, 2, 2, 1, 1, 0);
            else
                CM_POOL_LAUNCH(0, 0, 0, 0, 0, 0, -1);
#undef CM_POOL_LAUNCH
        }
    } else {
        const uint64_t total = planes * p.out_h * p.out_w;
        {
            ProfScope ps_(PK_POOL, s);
            launch_k(pool_direct_kernel<TYPE>, grid_for(cx, total, 256, 8), 256, 0, s, x, y, p, total);
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

extern "C" int cm_pool_nhwc_async(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                                  unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                                  unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                                  unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                                  unsigned count_include_pad, cm_stream_t stream) {
    (void)stride_h; (void)stride_w; (void)count_include_pad;
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    const uint64_t hw = (uint64_t)in_h * in_w;
    if ((uint64_t)batch * channels == 0) return CM_OK;
    if (!x || !y) return set_error(CM_EINVAL, "cm_pool_nhwc: null buffer");
    const bool global = pad_top == 0 && pad_left == 0 && pool_h == in_h && pool_w == in_w && out_h == 1 && out_w == 1 &&
                        (dil_h == 1 || pool_h <= 1) && (dil_w == 1 || pool_w <= 1) && hw > 0 && hw < (1ull << 31);
    if (!global) return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc: global pools only (the window covers the whole plane)");
    if (channels % 8u != 0 || ((uintptr_t)x & 15u) != 0 || ((uintptr_t)y & 15u) != 0)
        return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc: channels a multiple of 8 and 16-byte aligned buffers");
    const uint64_t groups = (uint64_t)batch * (channels / 8u);
    cudaStream_t s = (cudaStream_t)stream;
    const unsigned grid = grid_for(cx, groups * 4, 256, 8);
    {
        ProfScope ps_(PK_POOL, s);
        if (pool_type == CM_POOL_MAX) launch_k(pool_global_nhwc_kernel<P_MAX>, grid, 256, 0, s, x, y, groups, channels, (uint32_t)hw);
        else if (pool_type == CM_POOL_AVG) launch_k(pool_global_nhwc_kernel<P_AVG>, grid, 256, 0, s, x, y, groups, channels, (uint32_t)hw);
        else if (lp_order == 1u) launch_k(pool_global_nhwc_kernel<P_LP1>, grid, 256, 0, s, x, y, groups, channels, (uint32_t)hw);
        else launch_k(pool_global_nhwc_kernel<P_LP2>, grid, 256, 0, s, x, y, groups, channels, (uint32_t)hw);
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_pool_nhwc launch");
}

extern "C" int cm_pool_nhwc(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                            unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                            unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left, unsigned dil_h,
                            unsigned dil_w, unsigned pool_type, unsigned lp_order, unsigned count_include_pad) {
    int rc = cm_pool_nhwc_async(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
                                pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_pool(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                       unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                       unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left, unsigned dil_h,
                       unsigned dil_w, unsigned pool_type, unsigned lp_order, unsigned count_include_pad) {
    int rc = cm_pool_async(x, y, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w,
                           pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad, nullptr);
    return rc ? rc : finish_sync(nullptr);
}
