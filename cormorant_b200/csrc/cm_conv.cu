// cm_conv.cu -- ConvKernel on B200 (reference: kernels/conv/kernel/ConvKernel.cpp).
//
// Standard conv (group = 1) runs on the tcgen05 Q8.8 GEMM core (cm_gemm.cu),
// in one of two forms.
//
// Implicit GEMM (the usual case: dilation_w == 1, strides <= 8, channel
// padding cheap): rows = output pixels (n, oh, ow), columns = output channels,
// K = taps in (r, s, c) order.  One pre-pass writes the input as channels-last
// hi/lo planes with the spatial zero padding materialised (out-of-range taps
// read 0, ConvKernel.cpp:184-202) and per-pixel channel sums; the GEMM's TMA
// producer then loads each A tile straight from those planes (no im2col
// buffer).  The row terms are kh x kw box sums of the channel sums; the column
// terms carry bias << 8 (ConvKernel.cpp:160-169).  The epilogue writes
// y[n][m][p] (NCHW) with column stride P.
//
// Explicit im2col (everything else, e.g. the 3-channel stem): rows = output
// pixels of a chunk of images, columns = output channels, K in the weight
// layout's (c, r, s) order; the im2col pre-pass gathers each row's taps into
// K-major planes.  Images are processed in chunks so that either form's
// scratch stays bounded.  Outputs of at most 64 channels use the GEMM's
// 64-column tiles (packed weight planes).
//
// Depthwise conv (is_depthwise = 1, ConvKernel.cpp:251-319) is a per-channel
// kh x kw stencil: CUDA cores, one thread per output pixel, int32 wrap sum.
#include <algorithm>
#include <new>

#include "cm_gemm.cuh"

namespace cm {
namespace {

struct DwArgs {
    uint32_t C, H, W, M, out_h, out_w, kh, kw, sh, sw, dh, dw, pt, pl, has_bias;
};

__global__ void __launch_bounds__(256) conv_depthwise_kernel(const int16_t* __restrict__ x, const int16_t* __restrict__ w,
                                                             const int16_t* __restrict__ bias, int16_t* __restrict__ y,
                                                             DwArgs a, uint64_t total) {
    griddep_wait();
    const uint64_t ohw = (uint64_t)a.out_h * a.out_w;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t plane = t / ohw;            // n * M + m
        const uint64_t p = t - plane * ohw;
        const uint64_t n = plane / a.M, m = plane - n * a.M;
        const uint32_t oh = (uint32_t)(p / a.out_w), ow = (uint32_t)(p - (uint64_t)oh * a.out_w);
        uint32_t acc = a.has_bias ? (uint32_t)((int32_t)bias[m] * 256) : 0u;
        // input channel = output channel m (ConvKernel.cpp:262-266)
        const int16_t* xp = x + (n * a.C + m) * (uint64_t)a.H * a.W;
        const int16_t* wp = w + m * (uint64_t)a.kh * a.kw;
        for (uint32_t r = 0; r < a.kh; ++r) {
            const int64_t ih = (int64_t)oh * a.sh + (int64_t)r * a.dh - (int64_t)a.pt;
            if (ih < 0 || ih >= (int64_t)a.H) continue;
            for (uint32_t s = 0; s < a.kw; ++s) {
                const int64_t iw = (int64_t)ow * a.sw + (int64_t)s * a.dw - (int64_t)a.pl;
                if (iw < 0 || iw >= (int64_t)a.W) continue;
                acc += (uint32_t)((int32_t)__ldg(xp + (uint64_t)ih * a.W + iw) * (int32_t)__ldg(wp + r * a.kw + s));
            }
        }
        y[t] = narrow_acc(acc);
    }
}

// Fused elementwise epilogue (cm_conv_fused): bit 1 adds the residual word at the
// same index with saturation (VectorOP ADD), then bit 0 applies ReLU (VectorOP
// RELU; VectorOP.cpp:8-35, :106-111).
__device__ __forceinline__ int16_t epilogue_word(int16_t v, uint32_t epi, const int16_t* resid, uint64_t i) {
    int32_t r = v;
    if (epi & 2u) r = sat16(r + (int32_t)resid[i]);
    if (epi & 1u) r = max(r, 0);
    return (int16_t)r;
}

__global__ void __launch_bounds__(256) conv_epilogue_kernel(int16_t* __restrict__ y, const int16_t* __restrict__ resid,
                                                            uint64_t total, uint32_t epi) {
    griddep_wait();
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x)
        y[t] = epilogue_word(y[t], epi, resid, t);
}

// Launch-bound sizes: standard conv with G consecutive lanes per output word
// (G a power of two <= 32) taking the kernel rows (c, r) = lane, lane + G, ...;
// the int32 wrap sums meet by shuffle, bias << 8 is added, one narrowing
// follows (ConvKernel.cpp:160-230).
// q = a / b, r = a - q*b, in 32-bit arithmetic when both fit (a 64-bit division is a long
// instruction sequence on the latency path of these small kernels).
__device__ __forceinline__ void divmod64(uint64_t a, uint64_t b, uint64_t& q, uint64_t& r) {
    if (((a | b) >> 32) == 0) {
        const uint32_t q32 = (uint32_t)a / (uint32_t)b;
        q = q32;
        r = (uint32_t)a - q32 * (uint32_t)b;
    } else {
        q = a / b;
        r = a - q * b;
    }
}

// One kernel row of a direct conv tap sum: sum over s < kw of x[iw0 + s*dw] * w[s] (taps
// outside the input row add nothing).  Up to 8 taps issue all their loads before the first
// multiply, so a row costs one memory round trip instead of one per tap.
__device__ __forceinline__ uint32_t row_dot(const int16_t* __restrict__ xr, const int16_t* __restrict__ wr, int64_t iw0,
                                            const DwArgs& a) {
    uint32_t acc = 0;
    if (a.kw <= 8) {
        int32_t xv[8], wv[8];
#pragma unroll
        for (uint32_t s = 0; s < 8; ++s) {
            const int64_t iw = iw0 + (int64_t)s * a.dw;
            const bool ok = s < a.kw && iw >= 0 && iw < (int64_t)a.W;
            xv[s] = ok ? (int32_t)__ldg(xr + iw) : 0;
            wv[s] = s < a.kw ? (int32_t)__ldg(wr + s) : 0;
        }
#pragma unroll
        for (uint32_t s = 0; s < 8; ++s) acc += (uint32_t)(xv[s] * wv[s]);
    } else {
        for (uint32_t s = 0; s < a.kw; ++s) {
            const int64_t iw = iw0 + (int64_t)s * a.dw;
            if (iw < 0 || iw >= (int64_t)a.W) continue;
            acc += (uint32_t)((int32_t)__ldg(xr + iw) * (int32_t)__ldg(wr + s));
        }
    }
    return acc;
}

__global__ void __launch_bounds__(256) conv_direct_kernel(const int16_t* __restrict__ x, const int16_t* __restrict__ w,
                                                          const int16_t* __restrict__ bias, int16_t* __restrict__ y,
                                                          DwArgs a, uint64_t total, uint32_t G, uint32_t epi,
                                                          const int16_t* __restrict__ resid) {
    griddep_wait();
    const uint64_t ohw = (uint64_t)a.out_h * a.out_w;
    const uint32_t khw = a.kh * a.kw, rows = a.C * a.kh;
    const uint32_t g = threadIdx.x & (G - 1);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x / G;
    for (uint64_t t0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / G; t0 < (total + stride - 1) / stride * stride;
         t0 += stride) {
        const bool live = t0 < total;
        const uint64_t t = live ? t0 : 0;
        uint64_t plane, p, n, m, oh64, ow64;
        divmod64(t, ohw, plane, p);                // plane = n * M + m
        divmod64(plane, a.M, n, m);
        divmod64(p, a.out_w, oh64, ow64);
        const uint32_t oh = (uint32_t)oh64, ow = (uint32_t)ow64;
        uint32_t acc = 0;
        for (uint32_t kr = g; live && kr < rows; kr += G) {
            const uint32_t c = kr / a.kh, r = kr - c * a.kh;
            const int64_t ih = (int64_t)oh * a.sh + (int64_t)r * a.dh - (int64_t)a.pt;
            if (ih < 0 || ih >= (int64_t)a.H) continue;
            const int16_t* xr = x + ((n * a.C + c) * (uint64_t)a.H + (uint64_t)ih) * a.W;
            const int16_t* wr = w + (m * a.C + c) * (uint64_t)khw + (uint64_t)r * a.kw;
            acc += row_dot(xr, wr, (int64_t)ow * a.sw - (int64_t)a.pl, a);
        }
        for (uint32_t o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
        if (live && g == 0) {
            if (a.has_bias) acc += (uint32_t)((int32_t)bias[m] * 256);
            y[t] = epilogue_word(narrow_acc(acc), epi, resid, t);
        }
    }
}

// ConvKernel (+ its fused epilogue) followed by a MAX PoolingKernel on the conv's output, in
// one CUDA-core launch for launch-bound sizes.  A pooled output word takes G x T lanes: T tap
// slots (pool taps slot, slot + T, ...) of G lanes each; the G lanes of a slot split the conv
// pixel's reduction (rows (c, r) as in conv_direct_kernel) and meet by shuffles, the slot's
// first lane narrows the sum and applies the epilogue (resid at the conv output's index), and
// the slots' maxima meet by shuffles.  Taps outside the conv output contribute the pool's
// -128.0 padding, which is also where the maximum starts.  The conv output is never written.
// Every lane runs the same loop counts (the shuffles need the whole warp).
struct PoolGeo {
    uint32_t out_h, out_w, ph, pw, sh, sw, pt, pl, dh, dw;
};

__global__ void __launch_bounds__(256) conv_pool_direct_kernel(const int16_t* __restrict__ x, const int16_t* __restrict__ w,
                                                               const int16_t* __restrict__ bias, int16_t* __restrict__ y,
                                                               DwArgs a, PoolGeo q, uint64_t total, uint32_t G,
                                                               uint32_t T, uint32_t epi, const int16_t* __restrict__ resid) {
    griddep_wait();
    const uint64_t qhw = (uint64_t)q.out_h * q.out_w, chw = (uint64_t)a.out_h * a.out_w;
    const uint32_t khw = a.kh * a.kw, rows = a.C * a.kh, taps = q.ph * q.pw;
    const uint32_t L = G * T, li = threadIdx.x & (L - 1), g = li & (G - 1), slot = li / G;
    const uint32_t tap_rounds = (taps + T - 1) / T;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x / L;
    for (uint64_t t0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / L; t0 < (total + stride - 1) / stride * stride;
         t0 += stride) {
        const bool live = t0 < total;
        const uint64_t t = live ? t0 : 0;
        uint64_t plane, p, n, m, qh64, qw64;
        divmod64(t, qhw, plane, p);                // plane = n * M + m
        divmod64(plane, a.M, n, m);
        divmod64(p, q.out_w, qh64, qw64);
        const uint32_t qh = (uint32_t)qh64, qw = (uint32_t)qw64;
        int32_t best = -32768;
        for (uint32_t rd = 0; rd < tap_rounds; ++rd) {
            const uint32_t tap = slot + rd * T;
            const uint32_t pr = tap / q.pw, pc = tap - pr * q.pw;
            const int64_t oh = (int64_t)qh * q.sh + (int64_t)pr * q.dh - (int64_t)q.pt;
            const int64_t ow = (int64_t)qw * q.sw + (int64_t)pc * q.dw - (int64_t)q.pl;
            const bool in = live && tap < taps && oh >= 0 && oh < (int64_t)a.out_h && ow >= 0 && ow < (int64_t)a.out_w;
            uint32_t acc = 0;
            for (uint32_t kr = g; in && kr < rows; kr += G) {
                const uint32_t c = kr / a.kh, r = kr - c * a.kh;
                const int64_t ih = oh * a.sh + (int64_t)r * a.dh - (int64_t)a.pt;
                if (ih < 0 || ih >= (int64_t)a.H) continue;
                const int16_t* xr = x + ((n * a.C + c) * (uint64_t)a.H + (uint64_t)ih) * a.W;
                const int16_t* wr = w + (m * a.C + c) * (uint64_t)khw + (uint64_t)r * a.kw;
                acc += row_dot(xr, wr, ow * a.sw - (int64_t)a.pl, a);
            }
            for (uint32_t o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
            if (in && g == 0) {
                if (a.has_bias) acc += (uint32_t)((int32_t)bias[m] * 256);
                const uint64_t ci = plane * chw + (uint64_t)oh * a.out_w + (uint64_t)ow;
                best = max(best, (int32_t)epilogue_word(narrow_acc(acc), epi, resid, ci));
            }
        }
        for (uint32_t o = G; o < L; o <<= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
        if (live && li == 0) y[t] = (int16_t)best;
    }
}

// Empty reduction (in_ch * kh * kw == 0): every output is bias (or 0).
__global__ void conv_bias_fill_kernel(const int16_t* __restrict__ bias, int16_t* __restrict__ y, uint32_t M,
                                      uint64_t ohw, uint64_t total, uint32_t has_bias) {
    griddep_wait();
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t m = (t / ohw) % M;
        y[t] = has_bias ? bias[m] : (int16_t)0;
    }
}

constexpr uint64_t kIm2colBudget = 4ull << 30;  // bytes of im2col planes per chunk
constexpr uint64_t kNhwcBudget = 4ull << 30;    // bytes of channels-last planes per chunk

// ---- implicit GEMM pre-passes ------------------------------------------------

struct NhwcGeom {
    uint32_t C, H, W, Cp, Hp, Wp, pt, pl, nimg;
};

// x [nimg][C][H][W] -> planes [2][nimg][Hp][Wp][Cp] (hi, lo'), the spatial padding
// and the channels c >= C written as x = 0; S[n][hp][wp] = sum_{c<C} (x - 128).
// Block = 256 consecutive padded pixels of one image, all channels in tiles of
// 32: each tile is read channel by channel (thread = pixel, so a warp reads 32
// neighbouring pixels of one channel and the block 512 bytes of each channel
// row), transposed through shared memory, and written as two 16-byte runs of
// 16 channels per plane; the thread keeps its pixel's channel sum.
constexpr uint32_t kNhwcPix = 256, kNhwcCh = 32;

__global__ void __launch_bounds__(256) conv_nhwc_split_kernel(const int16_t* __restrict__ x, NhwcGeom g,
                                                              int8_t* __restrict__ planes, int32_t* __restrict__ S) {
    griddep_wait();
    __shared__ int16_t tile[kNhwcCh][kNhwcPix + 2];
    const uint32_t n = blockIdx.y;
    const uint32_t HWp = g.Hp * g.Wp;
    const uint32_t q = threadIdx.x;
    const uint32_t qp = blockIdx.x * kNhwcPix + q;
    const uint64_t HW = (uint64_t)g.H * g.W;
    int64_t src = -1;
    if (qp < HWp) {
        const uint32_t hp = qp / g.Wp, wp = qp - hp * g.Wp;
        const int32_t ih = (int32_t)hp - (int32_t)g.pt, iw = (int32_t)wp - (int32_t)g.pl;
        if (ih >= 0 && ih < (int32_t)g.H && iw >= 0 && iw < (int32_t)g.W)
            src = (int64_t)(((uint64_t)n * g.C * g.H + (uint32_t)ih) * g.W + (uint32_t)iw);
    }
    const uint64_t plane = (uint64_t)g.nimg * HWp * g.Cp;
    int8_t* dst = planes + ((uint64_t)n * HWp + qp) * g.Cp;
    int32_t sum = 0;
    for (uint32_t c0 = 0; c0 < g.Cp; c0 += kNhwcCh) {
        __syncthreads();
#pragma unroll
        for (uint32_t c = 0; c < kNhwcCh; ++c) {
            int16_t v = 0;
            if (src >= 0 && c0 + c < g.C) v = __ldg(x + (uint64_t)src + (uint64_t)(c0 + c) * HW);
            tile[c][q] = v;
        }
        __syncthreads();
        if (qp < HWp) {
#pragma unroll
            for (uint32_t h = 0; h < kNhwcCh; h += 16) {
                if (c0 + h >= g.Cp) break;
                uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
#pragma unroll
                for (uint32_t j = 0; j < 16; ++j) {
                    const int16_t v = tile[h + j][q];
                    hw[j / 4] |= (uint32_t)(uint8_t)(v >> 8) << (8 * (j % 4));
                    lw[j / 4] |= (((uint32_t)v & 255u) ^ 0x80u) << (8 * (j % 4));
                    if (c0 + h + j < g.C) sum += (int32_t)v - 128;
                }
                *(uint4*)(dst + c0 + h) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *(uint4*)(dst + plane + c0 + h) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
        }
    }
    if (qp < HWp) S[(uint64_t)n * HWp + qp] = sum;
}

// Whole-image variant for small maps whose H*W is not a multiple of 4 (7x7, 9x9 ...):
// block = one image.  Its C*H*W words are one contiguous run, read into shared memory
// with 4-byte loads (2-byte when the run is not 4-byte aligned); then item (padded
// pixel, 16 channels) -- consecutive threads take consecutive 16-channel groups, so
// the 16-byte hi / lo stores of a pixel are contiguous -- converts its 16 words, and
// the channel sums meet by shared-memory atomics.  Every padded pixel is written
// (the frame as x = 0), so no border pass follows.
constexpr uint32_t kImgSplitThreads = 512;
constexpr uint32_t kImgSplitSmem = 100u * 1024u;

__global__ void __launch_bounds__(kImgSplitThreads) conv_nhwc_split_img_kernel(const int16_t* __restrict__ x, NhwcGeom g,
                                                                               int8_t* __restrict__ planes,
                                                                               int32_t* __restrict__ S) {
    griddep_wait();
    extern __shared__ __align__(16) uint8_t img_smem[];
    const uint32_t HW = g.H * g.W, words = g.C * HW;
    int16_t* img = (int16_t*)img_smem;
    int32_t* ssum = (int32_t*)(img_smem + (((uint64_t)words * 2 + 15) & ~15ull));
    const uint32_t n = blockIdx.x;
    const uint32_t HWp = g.Hp * g.Wp;
    const int16_t* xi = x + (uint64_t)n * words;
    if ((((uintptr_t)xi) & 3u) == 0) {
        const uint32_t* x4 = (const uint32_t*)xi;
        uint32_t* i4 = (uint32_t*)img;
        for (uint32_t i = threadIdx.x; i < words / 2; i += blockDim.x) i4[i] = __ldg(x4 + i);
        if ((words & 1u) && threadIdx.x == 0) img[words - 1] = __ldg(xi + words - 1);
    } else {
        for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) img[i] = __ldg(xi + i);
    }
    for (uint32_t p = threadIdx.x; p < HWp; p += blockDim.x) ssum[p] = 0;
    __syncthreads();
    const uint64_t plane = (uint64_t)g.nimg * HWp * g.Cp;
    const uint32_t groups = g.Cp / 16, items = HWp * groups;
    for (uint32_t it = threadIdx.x; it < items; it += blockDim.x) {
        const uint32_t p = it / groups, grp = it - p * groups;
        const uint32_t hp = p / g.Wp, wp = p - hp * g.Wp;
        const int32_t ih = (int32_t)hp - (int32_t)g.pt, iw = (int32_t)wp - (int32_t)g.pl;
        const bool inside = ih >= 0 && ih < (int32_t)g.H && iw >= 0 && iw < (int32_t)g.W;
        const uint32_t pix = inside ? (uint32_t)ih * g.W + (uint32_t)iw : 0u;
        uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
        int32_t sum = 0;
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
            const uint32_t c = grp * 16 + j;
            const int16_t v = (inside && c < g.C) ? img[c * HW + pix] : (int16_t)0;
            hw[j / 4] |= (uint32_t)(uint8_t)(v >> 8) << (8 * (j % 4));
            lw[j / 4] |= (((uint32_t)v & 255u) ^ 0x80u) << (8 * (j % 4));
            if (c < g.C) sum += (int32_t)v - 128;
        }
        int8_t* dst = planes + ((uint64_t)n * HWp + p) * g.Cp + grp * 16;
        *(uint4*)dst = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *(uint4*)(dst + plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        atomicAdd(&ssum[p], sum);
    }
    __syncthreads();
    for (uint32_t p = threadIdx.x; p < HWp; p += blockDim.x) S[(uint64_t)n * HWp + p] = ssum[p];
}

// Four-pixel variant (H*W a multiple of 4, 8-byte aligned input): block = 256
// consecutive input pixels of one image (64 quads), channels in tiles of 32.
// Load: thread = (quad, channel), one 8-byte read of 4 pixels of a channel row.
// Convert: thread = (quad, 8 channels), eight 8-byte shared reads, byte
// permutes into 8-byte hi/lo runs per pixel written at the pixel's padded
// position.  The padding frame is written by conv_nhwc_border_kernel.
__global__ void __launch_bounds__(256) conv_nhwc_split4_kernel(const int16_t* __restrict__ x, NhwcGeom g,
                                                               int8_t* __restrict__ planes, int32_t* __restrict__ S) {
    griddep_wait();
    __shared__ uint2 tile[kNhwcCh][64 + 1];                 // [channel][quad], 4 words per entry
    const uint32_t n = blockIdx.y;
    const uint32_t HW = g.H * g.W, nq = HW / 4;
    const uint32_t q0 = blockIdx.x * 64;
    const uint32_t HWp = g.Hp * g.Wp;
    const uint64_t plane = (uint64_t)g.nimg * HWp * g.Cp;
    const uint2* xq = (const uint2*)(x + (uint64_t)n * g.C * HW);
    // load role
    const uint32_t lq = threadIdx.x & 63u, lc = threadIdx.x >> 6;
    // convert role: quad cq, channels 8*cg .. 8*cg + 7 of the tile
    const uint32_t cq = threadIdx.x >> 2, cg = threadIdx.x & 3u;
    const bool qlive = q0 + cq < nq;
    // padded position of each pixel; input pixels no tap reads (beyond Hp / Wp) are skipped
    uint64_t dst[4];
    bool keep[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t p = 4 * (q0 + cq) + j;
        const uint32_t h = p / g.W, w = p - h * g.W;
        keep[j] = qlive && h + g.pt < g.Hp && w + g.pl < g.Wp;
        dst[j] = (((uint64_t)n * g.Hp + h + g.pt) * g.Wp + w + g.pl) * g.Cp;
    }
    int32_t sum[4] = {0, 0, 0, 0};
    for (uint32_t c0 = 0; c0 < g.Cp; c0 += kNhwcCh) {
        __syncthreads();
#pragma unroll
        for (uint32_t i = 0; i < kNhwcCh / 4; ++i) {
            const uint32_t c = lc + 4 * i;
            uint2 v = make_uint2(0, 0);
            if (q0 + lq < nq && c0 + c < g.C) v = __ldg(xq + (uint64_t)(c0 + c) * nq + q0 + lq);
            tile[c][lq] = v;
        }
        __syncthreads();
        if (qlive && c0 + 8 * cg < g.Cp) {
            uint2 v[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) v[c] = tile[8 * cg + c][cq];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c0 + 8 * cg + c < g.C) {
                    sum[0] += (int32_t)(int16_t)(v[c].x & 0xFFFFu);
                    sum[1] += (int32_t)(int16_t)(v[c].x >> 16);
                    sum[2] += (int32_t)(int16_t)(v[c].y & 0xFFFFu);
                    sum[3] += (int32_t)(int16_t)(v[c].y >> 16);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // word holding pixel j of channel c: v[c].x (j < 2) or v[c].y; halfword j & 1
                const uint32_t hs = (j & 1) ? 3u : 1u, ls = (j & 1) ? 2u : 0u;   // byte of the hi / lo half
                uint32_t hw[2], lw[2];
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const uint32_t a0 = j < 2 ? v[4 * h2].x : v[4 * h2].y, a1 = j < 2 ? v[4 * h2 + 1].x : v[4 * h2 + 1].y;
                    const uint32_t a2 = j < 2 ? v[4 * h2 + 2].x : v[4 * h2 + 2].y, a3 = j < 2 ? v[4 * h2 + 3].x : v[4 * h2 + 3].y;
                    const uint32_t h01 = __byte_perm(a0, a1, hs | ((hs + 4) << 4)), h23 = __byte_perm(a2, a3, hs | ((hs + 4) << 4));
                    const uint32_t l01 = __byte_perm(a0, a1, ls | ((ls + 4) << 4)), l23 = __byte_perm(a2, a3, ls | ((ls + 4) << 4));
                    hw[h2] = __byte_perm(h01, h23, 0x5410);
                    lw[h2] = __byte_perm(l01, l23, 0x5410) ^ 0x80808080u;
                }
                if (keep[j]) {
                    const uint64_t o = dst[j] + c0 + 8 * cg;
                    *(uint2*)(planes + o) = make_uint2(hw[0], hw[1]);
                    *(uint2*)(planes + plane + o) = make_uint2(lw[0], lw[1]);
                }
            }
        }
    }
    // the four channel groups of a quad meet by shuffle; padded channels (x = 0) add nothing
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sum[j] += __shfl_xor_sync(0xFFFFFFFFu, sum[j], 1);
        sum[j] += __shfl_xor_sync(0xFFFFFFFFu, sum[j], 2);
    }
    if (cg == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (keep[j]) S[dst[j] / g.Cp] = (int32_t)((uint32_t)sum[j] - 128u * g.C);
    }
}

// Padding frame of the channels-last planes: every padded pixel outside the
// input gets x = 0 in all channels (h = 0, l' = -128) and S = -128 * C.  Grid y =
// image; the frame is enumerated directly: pt rows on top, the rows below the
// input, then the left / right margins of the input rows.
__global__ void __launch_bounds__(256) conv_nhwc_border_kernel(NhwcGeom g, int8_t* __restrict__ planes,
                                                               int32_t* __restrict__ S) {
    griddep_wait();
    const uint32_t n = blockIdx.y;
    const uint32_t HWp = g.Hp * g.Wp;
    const uint64_t plane = (uint64_t)g.nimg * HWp * g.Cp;
    const uint32_t cq = g.Cp / 16;
    const uint32_t rows_in = min(g.H, g.Hp > g.pt ? g.Hp - g.pt : 0u);            // input rows inside the window
    const uint32_t top = min(g.pt, g.Hp) * g.Wp;
    const uint32_t bot = (g.Hp > g.pt + rows_in ? g.Hp - g.pt - rows_in : 0u) * g.Wp;
    const uint32_t L = min(g.pl, g.Wp), R = g.Wp > g.pl + g.W ? g.Wp - g.pl - g.W : 0u;
    const uint64_t nb = (uint64_t)top + bot + (uint64_t)rows_in * (L + R);
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nb * cq; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t e = (uint32_t)(t / cq), run = (uint32_t)(t - (uint64_t)e * cq);
        uint32_t hp, wp;
        if (e < top) {
            hp = e / g.Wp; wp = e - hp * g.Wp;
        } else if (e < top + bot) {
            const uint32_t f = e - top;
            hp = g.pt + rows_in + f / g.Wp; wp = f % g.Wp;
        } else {
            const uint32_t f = e - top - bot, row = f / (L + R), col = f - row * (L + R);
            hp = g.pt + row; wp = col < L ? col : g.pl + g.W + (col - L);
        }
        const uint64_t pix = (uint64_t)n * HWp + (uint64_t)hp * g.Wp + wp;
        const uint64_t o = pix * g.Cp + 16 * run;
        *(uint4*)(planes + o) = make_uint4(0, 0, 0, 0);
        *(uint4*)(planes + plane + o) = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        if (run == 0) S[pix] = (int32_t)(0u - 128u * g.C);
    }
}

// S of a plane image before its producer adds the channel sums: 0 at the image's
// pixels, -128*C on the frame (x = 0 in every channel).  Grid-stride over the
// n*Hp*Wp words (multiply-high divisions by Wp and Hp).
__global__ void __launch_bounds__(256) planes_reset_S_kernel(int32_t* __restrict__ S, uint64_t total, FastDiv fwp,
                                                             FastDiv fhp, uint32_t H, uint32_t W, uint32_t pt,
                                                             uint32_t pl, int32_t frame) {
    griddep_wait();
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        // rows of one image chunk stay below 2^31 words (checked by the caller)
        const uint32_t row = fwp.div((uint32_t)t), w = (uint32_t)t - row * fwp.d;
        const uint32_t h = row - fhp.div(row) * fhp.d;
        const bool inside = h >= pt && h < pt + H && w >= pl && w < pl + W;
        S[t] = inside ? 0 : frame;
    }
}

// MaxPool from plane image to plane image: thread = output pixel, all its channels in
// 16-channel groups.  Each in-image tap contributes one 16-byte hi run and one lo' run,
// rebuilt into word pairs and reduced with __vmaxs2; taps outside the image are the
// pool's padding, which never wins (it holds -32768, PoolingKernel's kAccMin), so a
// window with no tap inside gives -32768.  The output pixel's channels are written as
// hi / lo' runs (channels past C as x = 0) and its channel sum to S directly.
struct PoolPlanesGeo {
    uint32_t in_h, in_w, out_h, out_w, ph, pw, sh, sw, pt, pl, dh, dw, C, Cp;
    uint32_t xHp, xWp, xpt, xpl, yHp, yWp, ypt, ypl;
    uint64_t x_plane, y_plane;
};

__global__ void __launch_bounds__(256) pool_max_planes_kernel(const int8_t* __restrict__ xin, int8_t* __restrict__ yout,
                                                              int32_t* __restrict__ yS, PoolPlanesGeo g, uint64_t total,
                                                              FastDiv fd_ow, FastDiv fd_oh) {
    griddep_wait();
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        // t < 2^32 (checked by the caller)
        const uint32_t row = fd_ow.div((uint32_t)t), ow = (uint32_t)t - row * fd_ow.d;
        const uint32_t n = fd_oh.div(row), oh = row - n * fd_oh.d;
        const int32_t ih0 = (int32_t)(oh * g.sh) - (int32_t)g.pt, iw0 = (int32_t)(ow * g.sw) - (int32_t)g.pl;
        const uint64_t ypix = ((uint64_t)n * g.yHp + oh + g.ypt) * g.yWp + ow + g.ypl;
        int32_t sum = 0;
        for (uint32_t c0 = 0; c0 < g.Cp; c0 += 16) {
            uint32_t acc[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = 0x80008000u;
            for (uint32_t r = 0; r < g.ph; ++r) {
                const int32_t ih = ih0 + (int32_t)(r * g.dh);
                if (ih < 0 || ih >= (int32_t)g.in_h) continue;
                for (uint32_t q = 0; q < g.pw; ++q) {
                    const int32_t iw = iw0 + (int32_t)(q * g.dw);
                    if (iw < 0 || iw >= (int32_t)g.in_w) continue;
                    const uint64_t xpix = ((uint64_t)n * g.xHp + (uint32_t)ih + g.xpt) * g.xWp + (uint32_t)iw + g.xpl;
                    const int8_t* src = xin + xpix * g.Cp + c0;
                    const uint4 hv = __ldg((const uint4*)src), lv = __ldg((const uint4*)(src + g.x_plane));
                    const uint32_t h4[4] = {hv.x, hv.y, hv.z, hv.w};
                    const uint32_t l4[4] = {lv.x ^ 0x80808080u, lv.y ^ 0x80808080u, lv.z ^ 0x80808080u, lv.w ^ 0x80808080u};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[2 * k] = __vmaxs2(acc[2 * k], __byte_perm(l4[k], h4[k], 0x5140));
                        acc[2 * k + 1] = __vmaxs2(acc[2 * k + 1], __byte_perm(l4[k], h4[k], 0x7362));
                    }
                }
            }
            const uint32_t live = c0 < g.C ? min(16u, g.C - c0) : 0u;
            uint32_t hw[4], lw[4];
            int32_t shi = 0, slo = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                uint32_t a = acc[2 * k], b = acc[2 * k + 1];
                if (4u * k + 0 >= live) a &= 0xFFFF0000u;
                if (4u * k + 1 >= live) a &= 0x0000FFFFu;
                if (4u * k + 2 >= live) b &= 0xFFFF0000u;
                if (4u * k + 3 >= live) b &= 0x0000FFFFu;
                hw[k] = __byte_perm(a, b, 0x7531);
                lw[k] = __byte_perm(a, b, 0x6420) ^ 0x80808080u;
                shi = __dp4a((int)hw[k], 0x01010101, shi);
                slo = __dp4a((int)lw[k], 0x01010101, slo);
            }
            sum += 256 * shi + slo + 128 * (int32_t)(16u - live);
            int8_t* dst = yout + ypix * g.Cp + c0;
            *(uint4*)dst = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *(uint4*)(dst + g.y_plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        yS[ypix] = sum;
    }
}

// MAX pool from a channels-last int16 tensor x [n][in_h][in_w][C] (C a multiple of 16) to
// plane image y: thread = (output pixel, 16-channel group), the G = Cp / 16 groups of a
// pixel on consecutive lanes.  Per tap two 16-byte loads of 16 words, a halfword-pair max
// (identity -32768: a window with no tap in the image gives it, as the NCHW pool does),
// then the hi / lo' split and the group's channel sum, the pixel's sum combined over its
// groups by shuffles and stored once (no atomics).  Channels past C hold x = 0.
__global__ void __launch_bounds__(256, 4) pool_max_nhwc_planes_kernel(const int16_t* __restrict__ x,
                                                                   int8_t* __restrict__ yout, int32_t* __restrict__ yS,
                                                                   PoolPlanesGeo g, uint64_t total, uint32_t g_log,
                                                                   FastDiv fd_ow, FastDiv fd_oh) {
    griddep_wait();
    const uint32_t G = 1u << g_log;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    // whole warps iterate together (the shuffles below need every lane of a pixel's groups)
    for (uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t0 < (total + stride - 1) / stride * stride;
         t0 += stride) {
        const bool live_t = t0 < total;
        const uint64_t t = live_t ? t0 : 0;          // t < 2^32 (checked by the caller)
        const uint32_t pix = (uint32_t)t >> g_log, grp = (uint32_t)t & (G - 1u);
        const uint32_t row = fd_ow.div(pix), ow = pix - row * fd_ow.d;
        const uint32_t n = fd_oh.div(row), oh = row - n * fd_oh.d;
        const uint32_t c0 = grp * 16u;
        const int32_t ih0 = (int32_t)(oh * g.sh) - (int32_t)g.pt, iw0 = (int32_t)(ow * g.sw) - (int32_t)g.pl;
        uint32_t acc[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = 0x80008000u;
        const bool real = c0 < g.C;
        if (live_t && real && g.ph == 3 && g.pw == 3) {
            // 3 x 3 windows (ResNet's stem pool): the taps' loads issued together, then the max
            uint4 v[9][2];
#pragma unroll
            for (uint32_t r = 0; r < 3; ++r) {
                const int32_t ih = ih0 + (int32_t)(r * g.dh);
                const bool rin = ih >= 0 && ih < (int32_t)g.in_h;
#pragma unroll
                for (uint32_t q = 0; q < 3; ++q) {
                    const int32_t iw = iw0 + (int32_t)(q * g.dw);
                    v[3 * r + q][0] = v[3 * r + q][1] = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
                    if (rin && iw >= 0 && iw < (int32_t)g.in_w) {
                        const uint4* src = (const uint4*)(x + (((uint64_t)n * g.in_h + (uint32_t)ih) * g.in_w + (uint32_t)iw) * g.C + c0);
                        v[3 * r + q][0] = __ldg(src);
                        v[3 * r + q][1] = __ldg(src + 1);
                    }
                }
            }
#pragma unroll
            for (uint32_t k = 0; k < 9; ++k) {
                acc[0] = __vmaxs2(acc[0], v[k][0].x); acc[1] = __vmaxs2(acc[1], v[k][0].y);
                acc[2] = __vmaxs2(acc[2], v[k][0].z); acc[3] = __vmaxs2(acc[3], v[k][0].w);
                acc[4] = __vmaxs2(acc[4], v[k][1].x); acc[5] = __vmaxs2(acc[5], v[k][1].y);
                acc[6] = __vmaxs2(acc[6], v[k][1].z); acc[7] = __vmaxs2(acc[7], v[k][1].w);
            }
        } else if (live_t && real) {
            for (uint32_t r = 0; r < g.ph; ++r) {
                const int32_t ih = ih0 + (int32_t)(r * g.dh);
                if (ih < 0 || ih >= (int32_t)g.in_h) continue;
                for (uint32_t q = 0; q < g.pw; ++q) {
                    const int32_t iw = iw0 + (int32_t)(q * g.dw);
                    if (iw < 0 || iw >= (int32_t)g.in_w) continue;
                    const uint4* src = (const uint4*)(x + (((uint64_t)n * g.in_h + (uint32_t)ih) * g.in_w + (uint32_t)iw) * g.C + c0);
                    const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
                    acc[0] = __vmaxs2(acc[0], v0.x); acc[1] = __vmaxs2(acc[1], v0.y);
                    acc[2] = __vmaxs2(acc[2], v0.z); acc[3] = __vmaxs2(acc[3], v0.w);
                    acc[4] = __vmaxs2(acc[4], v1.x); acc[5] = __vmaxs2(acc[5], v1.y);
                    acc[6] = __vmaxs2(acc[6], v1.z); acc[7] = __vmaxs2(acc[7], v1.w);
                }
            }
        }
        uint32_t hw[4], lw[4];
        int32_t shi = 0, slo = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t a = real ? acc[2 * k] : 0u, b = real ? acc[2 * k + 1] : 0u;   // x = 0 past C
            hw[k] = __byte_perm(a, b, 0x7531);
            lw[k] = __byte_perm(a, b, 0x6420) ^ 0x80808080u;
            shi = __dp4a((int)hw[k], 0x01010101, shi);
            slo = __dp4a((int)lw[k], 0x01010101, slo);
        }
        // x - 128 = 256*hi + lo' summed over the group's channels; padding channels hold x = 0
        // and are not part of the sum (their lo' bytes count -128 each: add it back)
        int32_t sum = 256 * shi + slo + (real ? 0 : 128 * 16);
        for (uint32_t o = G >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        if (live_t) {
            const uint64_t ypix = ((uint64_t)n * g.yHp + oh + g.ypt) * g.yWp + ow + g.ypl;
            int8_t* dst = yout + ypix * g.Cp + c0;
            *(uint4*)dst = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *(uint4*)(dst + g.y_plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            if (grp == 0) yS[ypix] = sum;
        }
    }
}

// rowterm of output pixel (n, oh, ow) = 128 * sum over its kh x kw taps of S.
// The channel sums of a conv's OUTPUT plane image cleared (0 inside the image, the frame's
// value on the frame) by the launch that computes the conv's row terms from its INPUT
// image, instead of a launch of its own: images [0, nimg) of S [nimg][Hp][Wp].
struct SumsReset {
    int32_t* S = nullptr;
    uint32_t nimg = 0, Hp = 0, Wp = 0, H = 0, W = 0, pt = 0, pl = 0;
    int32_t frame = 0;
};

__device__ __forceinline__ void sums_reset_image(const SumsReset& z, uint32_t n, uint32_t first_row, uint32_t row_step,
                                                 uint32_t first_col, uint32_t col_step) {
    int32_t* S = z.S + (uint64_t)n * z.Hp * z.Wp;
    for (uint32_t h = first_row; h < z.Hp; h += row_step) {
        const bool row_in = h >= z.pt && h < z.pt + z.H;
        for (uint32_t w = first_col; w < z.Wp; w += col_step)
            S[(uint64_t)h * z.Wp + w] = row_in && w >= z.pl && w < z.pl + z.W ? 0 : z.frame;
    }
}

__global__ void __launch_bounds__(256) conv_rowterm_kernel(const int32_t* __restrict__ S, uint32_t Hp, uint32_t Wp,
                                                           uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw,
                                                           uint32_t sh, uint32_t sw, uint32_t dh, uint64_t total,
                                                           int32_t* __restrict__ rowterm, SumsReset z, FastDiv fdP,
                                                           FastDiv fdW) {
    griddep_wait();
    // blocks past the row-term grid clear the output image's sums, one image at a time
    if (z.S && blockIdx.x >= gridDim.x - z.nimg) {
        sums_reset_image(z, blockIdx.x - (gridDim.x - z.nimg), threadIdx.x / 32, blockDim.x / 32, threadIdx.x % 32, 32);
        return;
    }
    const uint64_t nthreads = (uint64_t)(gridDim.x - (z.S ? z.nimg : 0)) * blockDim.x;
    const uint64_t P = (uint64_t)out_h * out_w;
    const bool small = total < (1ull << 32);
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += nthreads) {
        // multiply-high divisions when the index fits 32 bits (a 64-bit division costs more
        // than the rest of this thread's work)
        uint64_t n, p;
        uint32_t oh, ow;
        if (small) {
            const uint32_t n32 = fdP.div((uint32_t)t), p32 = (uint32_t)t - n32 * (uint32_t)P;
            oh = fdW.div(p32);
            ow = p32 - oh * out_w;
            n = n32; p = p32;
        } else {
            n = t / P; p = t - n * P;
            oh = (uint32_t)(p / out_w); ow = (uint32_t)(p - (uint64_t)oh * out_w);
        }
        const int32_t* b = S + ((uint64_t)n * Hp + (uint64_t)oh * sh) * Wp + (uint64_t)ow * sw;
        uint32_t sum = 0;
        if (kh <= 3 && kw <= 3) {
            // up to 3 x 3 taps: the loads issued together, then summed
            uint32_t v[9];
#pragma unroll
            for (uint32_t r = 0; r < 3; ++r)
#pragma unroll
                for (uint32_t q = 0; q < 3; ++q)
                    v[3 * r + q] = r < kh && q < kw ? (uint32_t)__ldg(b + (uint64_t)r * dh * Wp + q) : 0u;
#pragma unroll
            for (uint32_t k = 0; k < 9; ++k) sum += v[k];
        } else {
            for (uint32_t r = 0; r < kh; ++r)
                for (uint32_t q = 0; q < kw; ++q) sum += (uint32_t)__ldg(b + (uint64_t)r * dh * Wp + q);
        }
        rowterm[t] = (int32_t)(sum * 128u);
    }
}

// Separable form for rows of at least 16 outputs: warp = output row oh of image n
// (4 rows per block, grid (ceil(out_h / 4), images)).  Its lanes sum the kh input rows
// of S column by column into the warp's slice of shared memory (coalesced loads), then
// each output adds kw column sums: about kh*Wp/out_w + kw reads per output instead of
// kh*kw, no divisions, and no block-wide barrier.
constexpr uint32_t kRowtermThreads = 128;

__global__ void __launch_bounds__(kRowtermThreads) conv_rowterm_rows_kernel(const int32_t* __restrict__ S, uint32_t Hp,
                                                                          uint32_t Wp, uint32_t out_h, uint32_t out_w,
                                                                          uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw,
                                                                          uint32_t dh, int32_t* __restrict__ rowterm,
                                                                          SumsReset z) {
    griddep_wait();
    extern __shared__ uint32_t colsum_all[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // the last block column clears image blockIdx.y of the output image's sums
    if (z.S && blockIdx.x == gridDim.x - 1) {
        sums_reset_image(z, blockIdx.y, warp, kRowtermThreads / 32, lane, 32);
        return;
    }
    const uint32_t oh = blockIdx.x * (kRowtermThreads / 32) + warp, n = blockIdx.y;
    if (oh >= out_h) return;
    const uint32_t need = (out_w - 1) * sw + kw;
    uint32_t* colsum = colsum_all + warp * need;
    const int32_t* b = S + ((uint64_t)n * Hp + (uint64_t)oh * sh) * Wp;
    for (uint32_t c = lane; c < need; c += 32) {
        uint32_t v = 0;
        for (uint32_t r = 0; r < kh; ++r) v += (uint32_t)__ldg(b + (uint64_t)r * dh * Wp + c);
        colsum[c] = v;
    }
    __syncwarp();
    int32_t* out = rowterm + ((uint64_t)n * out_h + oh) * out_w;
    for (uint32_t ow = lane; ow < out_w; ow += 32) {
        uint32_t sum = 0;
        for (uint32_t q = 0; q < kw; ++q) sum += colsum[ow * sw + q];
        out[ow] = (int32_t)(sum * 128u);
    }
}

// Row terms of nb images (S: [nb][Hp][Wp], rt: [nb][out_h][out_w]).
// z.S != null: the same launch clears the output image's sums for these nb images (z.nimg = nb).
void rowterm_launch(const Context* cx, const int32_t* S, uint32_t Hp, uint32_t Wp, uint32_t out_h, uint32_t out_w,
                    uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw, uint32_t dh, uint32_t nb, int32_t* rt,
                    cudaStream_t s, SumsReset z = SumsReset{}) {
    const uint64_t need_bytes = ((uint64_t)(out_w - 1) * sw + kw) * 4 * (kRowtermThreads / 32);
    // up to 3 x 3 taps the per-output kernel issues all of an output's loads at once; the
    // separable form pays off for larger windows
    if (out_w >= 16 && need_bytes <= 48u * 1024u && (kh > 3 || kw > 3)) {
        for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
            const uint32_t bz = std::min(65535u, nb - b0);
            SumsReset zb = z;
            if (zb.S) { zb.S += (uint64_t)b0 * zb.Hp * zb.Wp; zb.nimg = bz; }
            launch_k(conv_rowterm_rows_kernel, dim3((out_h + 3) / 4 + (zb.S ? 1u : 0u), bz), kRowtermThreads, (size_t)need_bytes, s, 
                S + (uint64_t)b0 * Hp * Wp, Hp, Wp, out_h, out_w, kh, kw, sh, sw, dh, rt + (uint64_t)b0 * out_h * out_w, zb);
            count_launch();
        }
    } else {
        const uint64_t tot = (uint64_t)nb * out_h * out_w;
        if (z.S) z.nimg = nb;
        launch_k(conv_rowterm_kernel, grid_for(cx, tot, 256, 8) + (z.S ? nb : 0u), 256, 0, s, S, Hp, Wp, out_h, out_w, kh, kw, sh,
                                                                                        sw, dh, tot, rt, z,
                 FastDiv((uint32_t)std::min<uint64_t>((uint64_t)out_h * out_w, 0xFFFFFFFFull)), FastDiv(out_w));
        count_launch();
    }
}

// weights [M][C][kh][kw] -> N-major planes: tap k = (c, r, s) of output channel m
// goes to row k' = r*KR_pad + s*Cp + c, element (p, k', m) at
// planes[p*plane + k'*pitch + m] -- [2][Kt][M_pad] (pitch M_pad, plane Kt*M_pad)
// or packed [Kt][64 hi | 64 lo] (pitch 128, plane 64) for M <= 64.  The rows
// that hold no tap stay as zeroed beforehand (h = l' = 0 adds nothing).
// colterm[m] += 128 * sum_k (w - 128), plus 16384 * K + (bias << 8) from the
// first tile (mod 2^32; colterm zeroed beforehand).  Block = 32 channels x 128
// taps: rows of w read along k, transposed through shared memory, written as
// 16-byte runs of 16 channels.  With kh = kw = 1, C = Cp = KR_pad = K the rows
// keep the natural order.
__global__ void __launch_bounds__(256) conv_weights_kernel(const int16_t* __restrict__ w, const int16_t* __restrict__ bias,
                                                           uint32_t M, uint32_t C, uint32_t kh, uint32_t kw, uint32_t Cp,
                                                           uint32_t KR_pad, uint32_t pitch, uint64_t plane,
                                                           int8_t* __restrict__ planes, int32_t* __restrict__ colterm) {
    griddep_wait();
    __shared__ int16_t tile[32][130];
    const uint32_t khw = kh * kw, K = C * khw;
    const uint32_t k0 = blockIdx.x * 128, m0 = blockIdx.y * 32;
    const uint32_t t = threadIdx.x;
    {
        const uint32_t ml = t / 8, kq = (t % 8) * 16, m = m0 + ml;
        int32_t sum = 0;
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
            const uint32_t k = k0 + kq + j;
            int16_t v = 0;
            if (m < M && k < K) {
                v = __ldg(w + (uint64_t)m * K + k);
                sum += (int32_t)v - 128;
            }
            tile[ml][kq + j] = v;
        }
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
        sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 4);
        if ((t % 8) == 0 && m < M) {
            uint32_t add = (uint32_t)sum * 128u;
            if (blockIdx.x == 0) {
                add += K * 16384u;
                if (bias) add += (uint32_t)((int32_t)bias[m] * 256);
            }
            atomicAdd((unsigned int*)(colterm + m), add);
        }
    }
    __syncthreads();
    const uint32_t kl = t / 2, half = t % 2, k = k0 + kl;
    // a run of 16 channels that starts below M ends within the row (M_pad, or 64 packed)
    if (planes && k < K && m0 + 16 * half < M) {
        const uint32_t c = k / khw, rs = k - c * khw;
        const uint32_t r = rs / kw, sx = rs - r * kw;
        const uint64_t o = ((uint64_t)r * KR_pad + (uint64_t)sx * Cp + c) * pitch + m0 + 16 * half;
        uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
            const int16_t v = tile[16 * half + j][kl];
            hw[j / 4] |= (uint32_t)(uint8_t)(v >> 8) << (8 * (j % 4));
            lw[j / 4] |= (uint32_t)(uint8_t)((v & 255) - 128) << (8 * (j % 4));
        }
        *(uint4*)(planes + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *(uint4*)(planes + plane + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
}

// Weight planes + column terms for a conv GEMM (see conv_weights_kernel).
int conv_weights(const Context* cx, const int16_t* weight, const int16_t* bias, uint32_t M, uint32_t C, uint32_t kh,
                 uint32_t kw, uint32_t Cp, uint32_t KR_pad, uint32_t pitch, uint64_t plane, uint64_t plane_bytes,
                 int8_t* planes, int32_t* colterm, cudaStream_t s) {
    cudaError_t e = planes ? cudaMemsetAsync(planes, 0, plane_bytes, s) : cudaSuccess;
    if (e == cudaSuccess) e = cudaMemsetAsync(colterm, 0, (size_t)M * sizeof(int32_t), s);
    if (e != cudaSuccess) return cuda_error(e, "memset conv weights");
    const uint32_t K = C * kh * kw;
    const dim3 grid((K + 127) / 128, (M + 31) / 32);
    {
        ProfScope ps_(PK_SPLIT, s);
        launch_k(conv_weights_kernel, grid, 256, 0, s, weight, bias, M, C, kh, kw, Cp, KR_pad, pitch, plane, planes, colterm);
    }
    count_launch();
    return CM_OK;
}

// im2col -> K-major planes [2][rows][K_pad], row = n*P + p (output pixel p of image
// n), column k = (c, r, s) in the weight layout's order; out-of-range taps read
// 0 (ConvKernel.cpp:184-202).  rowterm[row] = 128 * sum_k (x - 128).
// Block = 128 rows, thread = one row: for each slice of up to 160 columns the
// thread gathers its taps (a warp reads one tap of 32 neighbouring pixels),
// packs them into 16-byte runs in shared memory, and the block then copies the
// slice out as consecutive 16-byte runs (whole rows when K_pad <= 160).
constexpr uint32_t kIcRows = 128, kIcSlice = 160, kIcPitch = kIcSlice + 16;

__global__ void __launch_bounds__(kIcRows) im2col_rows_kernel(const int16_t* __restrict__ x, ConvGeom g, uint32_t P,
                                                              uint64_t rows, uint32_t K, uint32_t K_pad,
                                                              int8_t* __restrict__ planes, int32_t* __restrict__ rowterm) {
    griddep_wait();
    __shared__ __align__(16) int8_t stage[2][kIcRows * kIcPitch];
    const uint64_t plane = rows * K_pad;
    const uint64_t r0 = (uint64_t)blockIdx.x * kIcRows;
    const uint64_t t = r0 + threadIdx.x;
    const bool live = t < rows;
    const uint32_t n = live ? (uint32_t)(t / P) : 0u;
    const uint32_t p = live ? (uint32_t)(t - (uint64_t)n * P) : 0u;
    const uint32_t oh = p / g.out_w, ow = p - oh * g.out_w;
    const int32_t ihb = (int32_t)(oh * g.sh) - (int32_t)g.pt;
    const int32_t iwb = (int32_t)(ow * g.sw) - (int32_t)g.pl;
    const int16_t* xn = x + (uint64_t)n * g.C * g.H * g.W;
    const uint32_t nrows = rows - r0 < kIcRows ? (uint32_t)(rows - r0) : kIcRows;
    uint32_t c = 0, r = 0, sx = 0;
    int32_t sum = 0;
    for (uint32_t s0 = 0; s0 < K_pad; s0 += kIcSlice) {
        const uint32_t sw = min(kIcSlice, K_pad - s0);      // multiple of 16
        for (uint32_t k0 = s0; k0 < s0 + sw; k0 += 16) {
            uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
#pragma unroll
            for (uint32_t j = 0; j < 16; ++j) {
                int16_t v = 0;
                if (live && k0 + j < K) {
                    const int32_t ih = ihb + (int32_t)(r * g.dh), iw = iwb + (int32_t)(sx * g.dw);
                    if (ih >= 0 && ih < (int32_t)g.H && iw >= 0 && iw < (int32_t)g.W)
                        v = __ldg(xn + ((uint64_t)c * g.H + (uint32_t)ih) * g.W + (uint32_t)iw);
                    sum += (int32_t)v - 128;
                    if (++sx == g.kw) {
                        sx = 0;
                        if (++r == g.kh) { r = 0; ++c; }
                    }
                }
                hw[j / 4] |= (uint32_t)(uint8_t)(v >> 8) << (8 * (j % 4));
                lw[j / 4] |= (((uint32_t)v & 255u) ^ 0x80u) << (8 * (j % 4));
            }
            const uint32_t o = threadIdx.x * kIcPitch + (k0 - s0);
            *(uint4*)(stage[0] + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *(uint4*)(stage[1] + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        __syncthreads();
        const uint32_t cpr = sw / 16, nchunks = nrows * cpr;
        for (uint32_t i = threadIdx.x; i < nchunks; i += kIcRows) {
            const uint32_t rr = i / cpr, cc = i - rr * cpr;
            const uint64_t go = (r0 + rr) * K_pad + s0 + 16 * cc;
            const uint32_t so = rr * kIcPitch + 16 * cc;
            *(uint4*)(planes + go) = *(const uint4*)(stage[0] + so);
            *(uint4*)(planes + plane + go) = *(const uint4*)(stage[1] + so);
        }
        __syncthreads();
    }
    if (live) rowterm[t] = (int32_t)((uint32_t)sum * 128u);
}

// im2col from a shared-memory window: block = up to 128 consecutive output
// pixels of one output row (thread = pixel).  The block first stages the input
// window those pixels read -- C channels x kh tap rows x the columns they span,
// zero outside the image, followed by a run of zeros that the K padding points
// at -- with loads coalesced along the row; then each thread walks its taps
// through a per-slice offset table (one broadcast read and one window read per
// tap, no bounds checks), packs pairs of words into hi/lo bytes with byte
// permutes, and the K-major rows are written through the same staging as
// im2col_rows_kernel.
constexpr uint32_t kWinMax = 96 * 1024;   // window bytes

__global__ void __launch_bounds__(kIcRows) im2col_win_kernel(const int16_t* __restrict__ x, ConvGeom g, uint32_t P,
                                                             uint64_t rows, uint32_t K, uint32_t K_pad, uint32_t WC,
                                                             FastDiv fd_wc, FastDiv fd_kh, int8_t* __restrict__ planes,
                                                             int32_t* __restrict__ rowterm) {
    griddep_wait();
    extern __shared__ __align__(16) uint8_t smem_dyn[];
    int8_t* stage0 = (int8_t*)smem_dyn;
    int8_t* stage1 = stage0 + kIcRows * kIcPitch;
    uint32_t* tab = (uint32_t*)(stage1 + kIcRows * kIcPitch);         // kIcSlice entries
    int16_t* win = (int16_t*)(tab + kIcSlice);                         // [C][kh][WC], then zeros
    const uint32_t ow0 = blockIdx.x * kIcRows, oh = blockIdx.y, n = blockIdx.z;
    const uint32_t npix = min(kIcRows, g.out_w - ow0);
    const uint32_t khw = g.kh * g.kw;
    const uint32_t wrows = g.C * g.kh, wcells = wrows * WC, zeros = (kIcRows - 1) * g.sw + 1;
    // stage the window: tap row r of channel c is input row oh*sh - pt + r*dh,
    // window column q is input column ow0*sw - pl + q; 8 loads in flight per thread
    {
        const int32_t ih0 = (int32_t)(oh * g.sh) - (int32_t)g.pt, iw0 = (int32_t)(ow0 * g.sw) - (int32_t)g.pl;
        const int16_t* xn = x + (uint64_t)n * g.C * g.H * g.W;
        for (uint32_t i0 = 0; i0 < wcells; i0 += 8 * kIcRows) {
            int16_t v[8];
#pragma unroll
            for (uint32_t m = 0; m < 8; ++m) {
                const uint32_t i = i0 + m * kIcRows + threadIdx.x;
                v[m] = 0;
                if (i < wcells) {
                    const uint32_t wr = fd_wc.div(i), q = i - wr * WC;
                    const uint32_t c = fd_kh.div(wr), r = wr - c * g.kh;
                    const int32_t ih = ih0 + (int32_t)(r * g.dh), iw = iw0 + (int32_t)q;
                    if (ih >= 0 && ih < (int32_t)g.H && iw >= 0 && iw < (int32_t)g.W)
                        v[m] = __ldg(xn + ((uint64_t)c * g.H + (uint32_t)ih) * g.W + (uint32_t)iw);
                }
            }
#pragma unroll
            for (uint32_t m = 0; m < 8; ++m) {
                const uint32_t i = i0 + m * kIcRows + threadIdx.x;
                if (i < wcells) win[i] = v[m];
            }
        }
        for (uint32_t i = threadIdx.x; i < zeros; i += kIcRows) win[wcells + i] = 0;
    }
    const uint32_t t = threadIdx.x;
    const bool live = t < npix;
    const int16_t* wp = win + (live ? t : 0u) * g.sw;
    const uint64_t row0 = (uint64_t)n * P + (uint64_t)oh * g.out_w + ow0;   // first K-major row of the block
    const uint64_t plane = rows * K_pad;
    uint32_t sum = 0;                                  // sum of the taps' words (padding reads 0)
    for (uint32_t s0 = 0; s0 < K_pad; s0 += kIcSlice) {
        const uint32_t sw = min(kIcSlice, K_pad - s0);
        __syncthreads();   // window staged / previous slice copied out
        for (uint32_t i = threadIdx.x; i < sw; i += kIcRows) {
            const uint32_t k = s0 + i;
            uint32_t off = wcells;                            // K padding: the zero run
            if (k < K) {
                const uint32_t c = k / khw, rs = k - c * khw;
                const uint32_t r = rs / g.kw, sx = rs - r * g.kw;
                off = (c * g.kh + r) * WC + sx * g.dw;
            }
            tab[i] = off;
        }
        __syncthreads();
        for (uint32_t k0 = 0; k0 < sw; k0 += 16) {
            uint32_t u[8];
#pragma unroll
            for (uint32_t jj = 0; jj < 8; ++jj) {
                const int16_t v0 = wp[tab[k0 + 2 * jj]], v1 = wp[tab[k0 + 2 * jj + 1]];
                sum += (uint32_t)(int32_t)v0 + (uint32_t)(int32_t)v1;
                u[jj] = (uint32_t)(uint16_t)v0 | ((uint32_t)(uint16_t)v1 << 16);
            }
            uint32_t hw[4], lw[4];
#pragma unroll
            for (uint32_t q = 0; q < 4; ++q) {
                hw[q] = __byte_perm(u[2 * q], u[2 * q + 1], 0x7531);
                lw[q] = __byte_perm(u[2 * q], u[2 * q + 1], 0x6420) ^ 0x80808080u;
            }
            const uint32_t o = t * kIcPitch + k0;
            *(uint4*)(stage0 + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *(uint4*)(stage1 + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        __syncthreads();
        const uint32_t cpr = sw / 16, nchunks = npix * cpr;
        for (uint32_t i = threadIdx.x; i < nchunks; i += kIcRows) {
            const uint32_t rr = i / cpr, cc = i - rr * cpr;
            const uint64_t go = (row0 + rr) * K_pad + s0 + 16 * cc;
            const uint32_t so = rr * kIcPitch + 16 * cc;
            *(uint4*)(planes + go) = *(const uint4*)(stage0 + so);
            *(uint4*)(planes + plane + go) = *(const uint4*)(stage1 + so);
        }
    }
    // rowterm = 128 * sum_k (x - 128) over the K real taps
    if (live) rowterm[row0 + t] = (int32_t)((sum - 128u * K) * 128u);
}

uint32_t pow2_ceil(uint32_t v) {
    uint32_t p = 1;
    while (p < v && p < (1u << 30)) p <<= 1;
    return p;
}

uint32_t log2u(uint32_t p) {
    uint32_t l = 0;
    while ((1u << l) < p) ++l;
    return l;
}

struct ImplicitPlan {
    uint32_t Cp, Hp, Wp, KR, KR_pad, Kt, bw, bh, bn;
};

// The implicit GEMM applies when each kernel row's taps are one contiguous run
// of the channels-last input (dilation_w == 1), the traversal strides fit TMA
// (<= 8), and the channel padding (C up to Cp, kw*Cp up to 32) costs at most
// half again the real reduction length in MMA steps.
bool plan_implicit(uint32_t C, uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw,
                   uint32_t dh, uint32_t dw, ImplicitPlan* ip) {
    if (dw != 1 || sh == 0 || sw == 0 || sh > 8 || sw > 8 || kh == 0 || kw == 0 || C == 0) return false;
    const uint64_t Cp = (C + 15ull) & ~15ull;
    if (Cp > 8192) return false;
    const uint64_t KR = (uint64_t)kw * Cp, KR_pad = (KR + 127) & ~127ull, Kt = KR_pad * kh;
    const uint64_t Kreal = (uint64_t)C * kh * kw;
    // MMA work: every kernel row runs ceil(KR/32) 32-deep steps (the zero tail of
    // each row's last block is skipped); allow at most half again the real taps
    const uint64_t steps = (uint64_t)kh * ((KR + 31) / 32) * 32;
    if (2 * steps > 3 * Kreal || Kt > (1ull << 30)) return false;
    const uint64_t Hp = (uint64_t)(out_h - 1) * sh + (uint64_t)(kh - 1) * dh + 1;
    const uint64_t Wp = (uint64_t)(out_w - 1) * sw + (kw - 1) + 1;
    if (Hp * Wp >= (1ull << 31)) return false;
    uint32_t bw = std::min<uint32_t>(pow2_ceil(out_w), 128);
    while (bw * sw > 256) bw >>= 1;
    uint32_t bh = std::min<uint32_t>(pow2_ceil(out_h), 128 / bw);
    while (bh * sh > 256) bh >>= 1;
    ip->Cp = (uint32_t)Cp; ip->Hp = (uint32_t)Hp; ip->Wp = (uint32_t)Wp;
    ip->KR = (uint32_t)KR; ip->KR_pad = (uint32_t)KR_pad; ip->Kt = (uint32_t)Kt;
    ip->bw = bw; ip->bh = bh; ip->bn = 128 / (bw * bh);
    return true;
}

// Tile shape (bw x bh x bn = 128 output pixels: columns, rows, images; powers of two) with
// the fewest padded pixels over nimg images -- 16 x 8 for a 112-wide map, 8 x 8 x 2
// images for 56, 1 x 1 x 128 images for 7 x 7 -- instead of bw = the width rounded up (a
// 14 x 14 map in 16 x 8 tiles computes 31 % padding).  A tile's time goes by its K blocks
// whatever its shape.  Ties go to the wider tile (coalesced output runs), then to the
// taller one (fewer images: neighbouring rows share input rows in L2); a conv writing
// NCHW words counts tiles narrower than 8 columns (scattered 2-byte stores) a quarter
// dearer.  TMA box extents: bw*sw, bh*sh <= 256.
void pick_tiles(uint32_t out_h, uint32_t out_w, uint32_t sh, uint32_t sw, uint64_t nimg, bool nchw_out,
                uint32_t* bw_out, uint32_t* bh_out, uint32_t* bn_out) {
    double best = -1.0;
    for (uint32_t bw = 1; bw <= 128; bw *= 2) {
        if (bw * sw > 256) break;
        for (uint32_t bh = 1; bw * bh <= 128; bh *= 2) {
            if (bh * sh > 256) break;
            const uint32_t bn = 128 / (bw * bh);
            double cost = (double)((out_w + bw - 1) / bw * bw) * (double)((out_h + bh - 1) / bh * bh) *
                          (double)((nimg + bn - 1) / bn * bn);
            if (nchw_out && bw < 8 && bw < out_w) cost *= 1.25;
            if (best < 0 || cost < best || (cost == best && (bw > *bw_out || (bw == *bw_out && bh > *bh_out)))) {
                best = cost; *bw_out = bw; *bh_out = bh; *bn_out = bn;
            }
        }
    }
}

// ---- space-to-depth form of strided convolutions with few input channels -----
// A conv with stride s in both directions equals a stride-1 conv over the input
// regrouped into s x s blocks: virtual pixel (h', w') holds channels (th, tw, c) =
// x[c][s*h' + th - pt][s*w' + tw - pl] (zero outside the image), and the virtual
// kernel is ceil(kh/s) x ceil(kw/s) with tap (r', u', th, tw, c) = w[c][s*r' + th][s*u' + tw]
// (zero where that index is past the original kernel).  For the 3-channel 7x7 stride-2
// stem this is 12 channels and a 4x4 kernel: the implicit GEMM applies (no im2col
// buffer).  The virtual taps past the original kernel have zero weights, so the row
// terms are the box sums over the ORIGINAL taps (conv_rowterm_kernel over per-pixel
// channel sums of the padded original image) and the column terms come from the
// original weights.

//
// Row stacking (T = 2): virtual pixel (h', w') also carries the channels of virtual
// pixel (h' + 1, w'), channels (t, th, tw, c), so one kernel row of the stacked image
// spans two virtual kernel rows -- a stride-1 conv with kernel rows 2 apart (dilation 2)
// and ceil(kh2 / 2) of them.  For the stem that is 24 channels (32 with padding) x 4
// taps = one full 128-byte K block per stacked row: 2 K blocks per tile instead of 4
// half-empty ones, the same MMA steps.  A tile's time there goes by its K blocks (each
// a round of TMA boxes), not by their bytes.

struct S2dPlan {
    uint32_t s, C2, kh2, kw2, Hpo, Wpo;
    uint32_t T = 1, kh3 = 0;   // row stacking; kh3 = stacked kernel rows (dilation T)
    ImplicitPlan ip;
};

bool plan_s2d(uint32_t C, uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw,
              uint32_t dh, uint32_t dw, S2dPlan* sp, uint32_t T = 1) {
    if (sh != sw || sh < 2 || sh > 4 || dh != 1 || dw != 1 || C == 0 || kh == 0 || kw == 0) return false;
    const uint32_t s = sh, C2 = s * s * C;
    if (C2 > 64) return false;
    const uint32_t kh2 = (kh + s - 1) / s, kw2 = (kw + s - 1) / s;
    ImplicitPlan ip;
    if (T == 2) {
        if (2 * C2 > 64 || kh2 < 2) return false;
        const uint32_t kh3 = (kh2 + 1) / 2;
        const uint64_t Cp = (2ull * C2 + 15ull) & ~15ull, KR = (uint64_t)kw2 * Cp, KR_pad = (KR + 127) & ~127ull;
        const uint64_t Hp = (uint64_t)out_h + kh2 - 1, Wp = (uint64_t)out_w + kw2 - 1;
        if (Hp * Wp >= (1ull << 31)) return false;
        uint32_t bw = std::min<uint32_t>(pow2_ceil(out_w), 128);
        uint32_t bh = std::min<uint32_t>(pow2_ceil(out_h), 128 / bw);
        ip.Cp = (uint32_t)Cp; ip.Hp = (uint32_t)Hp; ip.Wp = (uint32_t)Wp;
        ip.KR = (uint32_t)KR; ip.KR_pad = (uint32_t)KR_pad; ip.Kt = (uint32_t)(KR_pad * kh3);
        ip.bw = bw; ip.bh = bh; ip.bn = 128 / (bw * bh);
        const uint64_t steps = (uint64_t)kh3 * ((KR + 31) / 32) * 32;
        if (steps > 2ull * C * kh * kw) return false;
        sp->s = s; sp->C2 = C2; sp->kh2 = kh2; sp->kw2 = kw2;
        sp->Hpo = ip.Hp * s; sp->Wpo = ip.Wp * s;
        sp->T = 2; sp->kh3 = kh3;
        sp->ip = ip;
        return true;
    }
    if (!plan_implicit(C2, out_h, out_w, kh2, kw2, 1, 1, 1, 1, &ip)) {
        // plan_implicit's waste rule counts the virtual taps as real; re-plan without it
        const uint64_t Cp = (C2 + 15ull) & ~15ull, KR = (uint64_t)kw2 * Cp, KR_pad = (KR + 127) & ~127ull;
        const uint64_t Hp = (uint64_t)out_h + kh2 - 1, Wp = (uint64_t)out_w + kw2 - 1;
        if (Hp * Wp >= (1ull << 31)) return false;
        uint32_t bw = std::min<uint32_t>(pow2_ceil(out_w), 128);
        uint32_t bh = std::min<uint32_t>(pow2_ceil(out_h), 128 / bw);
        ip.Cp = (uint32_t)Cp; ip.Hp = (uint32_t)Hp; ip.Wp = (uint32_t)Wp;
        ip.KR = (uint32_t)KR; ip.KR_pad = (uint32_t)KR_pad; ip.Kt = (uint32_t)(KR_pad * kh2);
        ip.bw = bw; ip.bh = bh; ip.bn = 128 / (bw * bh);
    }
    // MMA steps against the original taps: allow up to 2x (the im2col it replaces costs more)
    const uint64_t steps = (uint64_t)kh2 * ((ip.KR + 31) / 32) * 32;
    if (steps > 2ull * C * kh * kw) return false;
    sp->s = s; sp->C2 = C2; sp->kh2 = kh2; sp->kw2 = kw2;
    sp->Hpo = ip.Hp * s; sp->Wpo = ip.Wp * s;
    sp->T = 1; sp->kh3 = kh2;
    sp->ip = ip;
    return true;
}

struct S2dGeom {
    uint32_t C, H, W, s, C2, Cp, Hs, Ws, pt, pl, Hpo, Wpo, nimg;
};

// x [nimg][C][H][W] -> virtual planes [2][nimg][Hs][Ws][Cp]; channels >= C2 hold x = 0.
// So[n][hp][wp] = sum_c (x - 128) over the ORIGINAL padded image (x = 0 outside).
// Thread = one virtual pixel: each of its s*s*C words is read once (for the planes and
// the channel sums), Cp/16 16-byte runs per plane.  s*s*C <= 64.
// S_, C_ > 0 fix s and C at compile time (the channel index of every word is then a
// constant and the packing stays in registers); 0 takes them from g.
template <int S_, int C_>
__global__ void __launch_bounds__(256) conv_s2d_split_kernel(const int16_t* __restrict__ x, S2dGeom g, uint64_t total,
                                                             int8_t* __restrict__ planes, int32_t* __restrict__ So) {
    griddep_wait();
    constexpr uint32_t CPC = S_ > 0 ? ((uint32_t)(S_ * S_ * C_) + 15u) / 16u * 16u : 0u;
    const uint32_t S = S_ > 0 ? (uint32_t)S_ : g.s, CC = C_ > 0 ? (uint32_t)C_ : g.C;
    const uint32_t Cp = CPC ? CPC : g.Cp;
    const uint64_t plane = (uint64_t)g.nimg * g.Hs * g.Ws * g.Cp;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t n = t / ((uint64_t)g.Hs * g.Ws);
        const uint32_t rem = (uint32_t)(t - n * g.Hs * g.Ws);
        const uint32_t hv = rem / g.Ws, wv = rem - hv * g.Ws;
        const int16_t* xn = x + n * g.C * g.H * g.W;
        int8_t* dst = planes + t * g.Cp;
        uint32_t hw[16], lw[16];                         // up to 64 channels per plane
#pragma unroll
        for (int q = 0; q < 16; ++q) { hw[q] = 0; lw[q] = 0x80808080u; }
        uint32_t c2 = 0;
#pragma unroll
        for (uint32_t th = 0; th < S; ++th)
#pragma unroll
            for (uint32_t tw = 0; tw < S; ++tw) {
                const int32_t ih = (int32_t)(S * hv + th) - (int32_t)g.pt, iw = (int32_t)(S * wv + tw) - (int32_t)g.pl;
                const bool in = ih >= 0 && ih < (int32_t)g.H && iw >= 0 && iw < (int32_t)g.W;
                const int16_t* xp = xn + (in ? (uint64_t)ih * g.W + (uint32_t)iw : 0);
                int32_t sum = 0;
#pragma unroll
                for (uint32_t c = 0; c < CC; ++c, ++c2) {
                    const int16_t v = in ? __ldg(xp + (uint64_t)c * g.H * g.W) : (int16_t)0;
                    sum += (int32_t)v - 128;
                    const uint32_t q = c2 >> 2, sh = 8 * (c2 & 3);
                    hw[q] |= (uint32_t)(uint8_t)(v >> 8) << sh;
                    lw[q] = (lw[q] & ~(0xFFu << sh)) | ((((uint32_t)v & 255u) ^ 0x80u) << sh);
                }
                So[(n * g.Hpo + S * hv + th) * g.Wpo + S * wv + tw] = sum;
            }
#pragma unroll
        for (uint32_t c0 = 0; c0 < Cp; c0 += 16) {
            const uint32_t q = c0 / 4;
            *(uint4*)(dst + c0) = make_uint4(hw[q], hw[q + 1], hw[q + 2], hw[q + 3]);
            *(uint4*)(dst + plane + c0) = make_uint4(lw[q], lw[q + 1], lw[q + 2], lw[q + 3]);
        }
    }
}

// Row form of the same conversion for fixed S_, C_: block = RB_ consecutive virtual rows
// hv0 .. hv0 + RB_ - 1 of one image (grid (ceil(Hs / RB_), images)).  The input rows they
// cover, (RB_ - 1) * S_ + T_ * S_ per channel, are staged in shared memory once with
// coalesced loads (16-byte loads when rows are 16-byte aligned; rows outside the image as
// zeros), so rows shared by consecutive virtual rows are read once; then each thread
// converts virtual pixels (hv, wv): shared-memory reads, So written as one S_-word run per
// original row.  The staged rows fit in kS2dRowSmem.
constexpr uint32_t kS2dRowThreads = 128;
constexpr uint32_t kS2dRowSmem = 32u * 1024u;

// input rows per channel a band of rb virtual rows stages
__host__ __device__ constexpr uint32_t s2d_band_rows(uint32_t s, uint32_t t, uint32_t rb) { return (rb - 1) * s + t * s; }

// Row terms of the original conv computed by the split itself (S2dRt::rt != null, KH_ > 0:
// the original kernel height; stride S_, dilation 1): output row oh = hv of the band reads
// padded rows S_*oh .. S_*oh + KH_ - 1, so the band stages S_*(RB_ - 1) + KH_ rows when that
// is more than the split needs, and So is not written.
struct S2dRt {
    int32_t* rt;                   // [nimg][out_h][out_w], as rowterm_launch writes it
    uint32_t out_h, out_w, kw;
};

__host__ __device__ constexpr uint32_t s2d_stage_rows(uint32_t s, uint32_t t, uint32_t rb, uint32_t kh) {
    return s2d_band_rows(s, t, rb) > (rb - 1) * s + kh ? s2d_band_rows(s, t, rb) : (rb - 1) * s + kh;
}

// T_ = 2: a virtual pixel also carries virtual row hv + 1 and writes its channels after
// those of row hv (row stacking); So is written for row hv only.
template <int S_, int C_, int T_ = 1, int RB_ = 1, int KH_ = 0>
__global__ void __launch_bounds__(kS2dRowThreads) conv_s2d_rows_kernel(const int16_t* __restrict__ x, S2dGeom g,
                                                                        int8_t* __restrict__ planes,
                                                                        int32_t* __restrict__ So, S2dRt rtp) {
    griddep_wait();
    static_assert(S_ >= 2 && T_ * S_ * S_ * C_ <= 64, "space-to-depth channels");
    constexpr uint32_t C2 = (uint32_t)(S_ * S_ * C_), CPC = (T_ * C2 + 15u) / 16u * 16u;
    constexpr uint32_t RPC = s2d_stage_rows(S_, T_, RB_, KH_);   // staged input rows per channel
    const bool fused_rt = KH_ > 0 && rtp.rt != nullptr;
    extern __shared__ __align__(16) int16_t rowbuf[];      // [RPC][C_][W], then (fused_rt) [RB_][Wpo] int32
    const uint32_t hv0 = blockIdx.x * RB_, n = blockIdx.y;
    const uint32_t W = g.W;
    const int16_t* xn = x + (uint64_t)n * C_ * g.H * W;
    const bool quads = (W & 7u) == 0 && (((uintptr_t)x) & 15u) == 0;
    const bool pairs = (W & 1u) == 0 && (((uintptr_t)x) & 3u) == 0;
    if (quads) {
        // every 16-byte piece of every staged row is one item: each thread issues up to
        // kBatch loads before its first shared-memory store, so the block's rows arrive in
        // one memory round trip instead of one per row
        constexpr uint32_t kBatch = 8;
        const uint32_t per_row = W / 8, items = RPC * (uint32_t)C_ * per_row;
        for (uint32_t base = 0; base < items; base += kBatch * blockDim.x) {
            uint4 v[kBatch];
#pragma unroll
            for (uint32_t k = 0; k < kBatch; ++k) {
                const uint32_t idx = base + k * blockDim.x + threadIdx.x;
                v[k] = make_uint4(0, 0, 0, 0);
                if (idx < items) {
                    const uint32_t r = idx / per_row, i = idx - r * per_row;
                    const uint32_t lr = r / C_, c = r % C_;
                    const int32_t ih = (int32_t)(S_ * hv0 + lr) - (int32_t)g.pt;
                    if (ih >= 0 && ih < (int32_t)g.H)
                        v[k] = __ldg((const uint4*)(xn + ((uint64_t)c * g.H + (uint32_t)ih) * W) + i);
                }
            }
#pragma unroll
            for (uint32_t k = 0; k < kBatch; ++k) {
                const uint32_t idx = base + k * blockDim.x + threadIdx.x;
                if (idx < items) ((uint4*)rowbuf)[idx] = v[k];
            }
        }
    }
    for (uint32_t r = 0; !quads && r < RPC * (uint32_t)C_; ++r) {
        const uint32_t lr = r / C_, c = r % C_;            // local row lr: input row S_*hv0 + lr - pt
        const int32_t ih = (int32_t)(S_ * hv0 + lr) - (int32_t)g.pt;
        int16_t* dst = rowbuf + r * W;
        if (ih >= 0 && ih < (int32_t)g.H) {
            const int16_t* src = xn + ((uint64_t)c * g.H + (uint32_t)ih) * W;
            if (pairs) {
                for (uint32_t i = threadIdx.x; i < W / 2; i += blockDim.x)
                    ((uint32_t*)dst)[i] = __ldg((const uint32_t*)src + i);
            } else {
                for (uint32_t i = threadIdx.x; i < W; i += blockDim.x) dst[i] = __ldg(src + i);
            }
        } else {
            for (uint32_t i = threadIdx.x; i < W; i += blockDim.x) dst[i] = 0;
        }
    }
    __syncthreads();
    const uint64_t plane = (uint64_t)g.nimg * g.Hs * g.Ws * g.Cp;
    const uint32_t rows = min((uint32_t)RB_, g.Hs - hv0);
    for (uint32_t item = threadIdx.x; item < rows * g.Ws; item += blockDim.x) {
        const uint32_t i = item / g.Ws, wv = item - i * g.Ws;
        const uint32_t hv = hv0 + i;
        // the virtual pixel's words in channel order c2 = (th*S_ + tw)*C_ + c (x = 0 outside
        // the image and past T_*C2), gathered first, then split four at a time with byte
        // permutes: hi = the words' high bytes, lo' = their low bytes ^ 0x80
        uint32_t v[CPC];
#pragma unroll
        for (uint32_t c2 = T_ * C2; c2 < CPC; ++c2) v[c2] = 0;
#pragma unroll
        for (uint32_t th = 0; th < (uint32_t)(T_ * S_); ++th) {   // th >= S_: stacked row hv + 1
            const int16_t* lrow = rowbuf + (S_ * i + th) * C_ * W;
#pragma unroll
            for (uint32_t tw = 0; tw < (uint32_t)S_; ++tw) {
                const int32_t iw = (int32_t)(S_ * wv + tw) - (int32_t)g.pl;
                const bool in = iw >= 0 && iw < (int32_t)W;
#pragma unroll
                for (uint32_t c = 0; c < (uint32_t)C_; ++c)
                    v[(th * S_ + tw) * C_ + c] = in ? (uint32_t)(uint16_t)lrow[c * W + (uint32_t)iw] : 0u;
            }
            if (th < (uint32_t)S_ && !fused_rt) {
                int32_t sums[S_];
#pragma unroll
                for (uint32_t tw = 0; tw < (uint32_t)S_; ++tw) {
                    int32_t sum = -128 * C_;
#pragma unroll
                    for (uint32_t c = 0; c < (uint32_t)C_; ++c) sum += (int32_t)(int16_t)v[(th * S_ + tw) * C_ + c];
                    sums[tw] = sum;
                }
                int32_t* so = So + ((uint64_t)n * g.Hpo + S_ * hv + th) * g.Wpo + S_ * wv;
                if constexpr (S_ == 2) {
                    *(int2*)so = make_int2(sums[0], sums[1]);
                } else {
#pragma unroll
                    for (uint32_t tw = 0; tw < (uint32_t)S_; ++tw) so[tw] = sums[tw];
                }
            }
        }
        uint32_t hw[CPC / 4], lw[CPC / 4];
#pragma unroll
        for (uint32_t q = 0; q < CPC / 4; ++q) {
            const uint32_t p01 = v[4 * q] | (v[4 * q + 1] << 16), p23 = v[4 * q + 2] | (v[4 * q + 3] << 16);
            hw[q] = __byte_perm(p01, p23, 0x7531);
            lw[q] = __byte_perm(p01, p23, 0x6420) ^ 0x80808080u;
        }
        int8_t* dst = planes + (((uint64_t)n * g.Hs + hv) * g.Ws + wv) * g.Cp;
#pragma unroll
        for (uint32_t c0 = 0; c0 < CPC; c0 += 16) {
            const uint32_t q = c0 / 4;
            *(uint4*)(dst + c0) = make_uint4(hw[q], hw[q + 1], hw[q + 2], hw[q + 3]);
            *(uint4*)(dst + plane + c0) = make_uint4(lw[q], lw[q + 1], lw[q + 2], lw[q + 3]);
        }
    }
    if constexpr (KH_ > 0) {
        if (fused_rt) {
            // V[i][col] = sum over kernel rows r and channels c of (x - 128) at padded row
            // S_*(hv0 + i) + r, padded column col (x = 0 outside the image); then
            // rt = 128 * sum over q < kw of V[i][S_*ow + q] -- the box sums of So
            int32_t* V = (int32_t*)(((uintptr_t)(rowbuf + RPC * (uint32_t)C_ * W) + 15u) & ~(uintptr_t)15u);
            const uint32_t Wpo = g.Wpo;
            for (uint32_t item = threadIdx.x; item < (uint32_t)RB_ * Wpo; item += blockDim.x) {
                const uint32_t i = item / Wpo, col = item - i * Wpo;
                const int32_t iw = (int32_t)col - (int32_t)g.pl;
                int32_t v = -128 * KH_ * C_;
                if (iw >= 0 && iw < (int32_t)W) {
#pragma unroll
                    for (uint32_t r = 0; r < (uint32_t)KH_; ++r)
#pragma unroll
                        for (uint32_t c = 0; c < (uint32_t)C_; ++c) v += rowbuf[((S_ * i + r) * C_ + c) * W + (uint32_t)iw];
                }
                V[item] = v;
            }
            __syncthreads();
            const uint32_t rows_out = hv0 < rtp.out_h ? min((uint32_t)RB_, rtp.out_h - hv0) : 0u;
            for (uint32_t item = threadIdx.x; item < rows_out * rtp.out_w; item += blockDim.x) {
                const uint32_t i = item / rtp.out_w, ow = item - i * rtp.out_w;
                const int32_t* vr = V + i * Wpo + S_ * ow;
                uint32_t sum = 0;
                for (uint32_t q = 0; q < rtp.kw; ++q) sum += (uint32_t)vr[q];
                rtp.rt[((uint64_t)n * rtp.out_h + hv0 + i) * rtp.out_w + ow] = (int32_t)(sum * 128u);
            }
        }
    }
}

// Virtual weights -> N-major planes (layout as conv_weights_kernel): row
// k' = r'*KR_pad + u'*Cp + (th*s + tw)*C + c holds w[m][c][s*r' + th][s*u' + tw], zero past
// the original kernel.  Thread per (k', m); the weights are small.
// With row stacking (T = 2) channel c2 = (t, th, tw, c) of stacked kernel row r2 is
// virtual kernel row T*r2 + t.
__global__ void __launch_bounds__(256) conv_s2d_weights_kernel(const int16_t* __restrict__ w, uint32_t M, uint32_t C,
                                                               uint32_t kh, uint32_t kw, uint32_t s, uint32_t kw2,
                                                               uint32_t Cp, uint32_t KR_pad, uint32_t Kt, uint32_t pitch,
                                                               uint64_t plane, int8_t* __restrict__ planes, uint32_t T) {
    griddep_wait();
    const uint64_t total = (uint64_t)Kt * M;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t kp = (uint32_t)(t / M), m = (uint32_t)(t - (uint64_t)kp * M);
        const uint32_t r2 = kp / KR_pad, rem = kp - r2 * KR_pad;
        const uint32_t u2 = rem / Cp, c2 = rem - u2 * Cp;
        int8_t hi = 0, lo = 0;
        if (u2 < kw2 && c2 < T * s * s * C) {
            const uint32_t st = c2 / (s * s * C), c2b = c2 - st * (s * s * C);
            const uint32_t blk = c2b / C, c = c2b - blk * C, th = blk / s, tw = blk - th * s;
            const uint32_t r = s * (T * r2 + st) + th, q = s * u2 + tw;
            if (r < kh && q < kw) {
                const int16_t v = __ldg(w + (((uint64_t)m * C + c) * kh + r) * kw + q);
                hi = (int8_t)(v >> 8);
                lo = (int8_t)((v & 255) - 128);
            }
        }
        planes[(uint64_t)kp * pitch + m] = hi;
        planes[plane + (uint64_t)kp * pitch + m] = lo;
    }
}

}  // namespace
}  // namespace cm

using namespace cm;

// A channels-last plane image of an activation x [n][C][H][W]: hi / lo' planes
// [2][n][Hp][Wp][Cp] (Hp = pt + H + pb, Wp = pl + W + pr, Cp = C rounded up to 16)
// and per-pixel channel sums S [n][Hp][Wp] = sum_c (x - 128); the frame and the
// channels past C hold x = 0.  It is the A operand of every implicit-GEMM conv
// that reads x, so a conv whose GEMM epilogue writes it spares its consumers the
// split pass.
struct cm_planes {
    int8_t* planes = nullptr;
    int32_t* S = nullptr;
    uint64_t plane_pitch = 0;   // bytes from the hi plane to the lo plane
    uint32_t n = 0, C = 0, H = 0, W = 0, Cp = 0, Hp = 0, Wp = 0, pt = 0, pl = 0;
    int device = -1;
};

namespace {

// The path a standard conv call takes, in the order conv_core tests them.
enum ConvPath { CP_DEPTHWISE, CP_BIAS_FILL, CP_DIRECT, CP_TOO_LONG, CP_IMPLICIT, CP_S2D, CP_EXPLICIT };

ConvPath conv_path(uint64_t direct_max_macs, unsigned batch, unsigned in_ch, unsigned out_ch, unsigned out_h,
                   unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                   unsigned dilation_w, unsigned is_depthwise, ImplicitPlan* ip) {
    if (is_depthwise) return CP_DEPTHWISE;
    const uint64_t K64 = (uint64_t)in_ch * kh * kw;
    if (K64 == 0) return CP_BIAS_FILL;
    const uint64_t total = (uint64_t)batch * out_ch * out_h * out_w;
    if ((unsigned __int128)total * K64 <= direct_max_macs) return CP_DIRECT;
    if (K64 > kMaxGemmK) return CP_TOO_LONG;
    if (plan_implicit(in_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, ip)) return CP_IMPLICIT;
    S2dPlan sp;
    if (plan_s2d(in_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, &sp)) return CP_S2D;
    return CP_EXPLICIT;
}

// Whether plane image `xp` can be the A operand of an implicit conv with plan `ip`:
// the same tensor, and a frame at least as wide as the conv's padded extent.
bool planes_fit(const cm_planes* xp, unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned pad_top,
                unsigned pad_left, const ImplicitPlan& ip) {
    // (a box reads up to one kernel row past the last pixel: the image keeps 64 KB of slack)
    return xp && ip.KR <= 65536u && xp->n == batch && xp->C == in_ch && xp->H == in_h && xp->W == in_w && xp->Cp == ip.Cp &&
           xp->pt >= pad_top && xp->pl >= pad_left && (uint64_t)(xp->pt - pad_top) + ip.Hp <= xp->Hp &&
           (uint64_t)(xp->pl - pad_left) + ip.Wp <= xp->Wp;
}

// x (NCHW words) -> plane image yp, by the split kernels (producers whose GEMM does
// not write the image itself).  The frame was written when yp was created.
int planes_from_tensor(const Context* cx, const int16_t* x, cm_planes* yp, cudaStream_t s) {
    const uint64_t HW = (uint64_t)yp->H * yp->W;
    const uint64_t img_plane = (uint64_t)yp->Hp * yp->Wp * yp->Cp;
    const NhwcGeom ng{yp->C, yp->H, yp->W, yp->Cp, yp->Hp, yp->Wp, yp->pt, yp->pl, yp->n};
    const bool quads = HW % 4 == 0 && ((uintptr_t)x & 7u) == 0 && HW < (1ull << 31);
    const uint32_t gx = quads ? (uint32_t)((HW / 4 + 63) / 64) : (uint32_t)(((uint64_t)yp->Hp * yp->Wp + kNhwcPix - 1) / kNhwcPix);
    ProfScope ps_(PK_SPLIT, s);
    for (uint32_t b0 = 0; b0 < yp->n; b0 += 65535u) {
        const uint32_t bz = std::min(65535u, yp->n - b0);
        const int16_t* xb = x + (uint64_t)b0 * yp->C * HW;
        int8_t* pb = yp->planes + (uint64_t)b0 * img_plane;
        int32_t* Sb = yp->S + (uint64_t)b0 * yp->Hp * yp->Wp;
        if (quads) launch_k(conv_nhwc_split4_kernel, dim3(gx, bz), 256, 0, s, xb, ng, pb, Sb);
        else launch_k(conv_nhwc_split_kernel, dim3(gx, bz), 256, 0, s, xb, ng, pb, Sb);
        count_launch();
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv planes split");
}

// Clears the channel sums of plane image yp (images [n0, n0 + nb)) before a GEMM
// epilogue adds into them.
int planes_reset(cm_planes* yp, cudaStream_t s) {
    const Context* cx = ctx();
    const uint64_t img = (uint64_t)yp->Hp * yp->Wp;
    const uint32_t per = (uint32_t)std::max<uint64_t>(1, ((1ull << 31) / img));   // images per launch: words < 2^31
    for (uint32_t b0 = 0; b0 < yp->n; b0 += per) {
        const uint32_t nb = std::min(per, yp->n - b0);
        const uint64_t total = nb * img;
        launch_k(planes_reset_S_kernel, grid_for(cx, total, 256, 4), 256, 0, s, 
            yp->S + (uint64_t)b0 * img, total, FastDiv(yp->Wp), FastDiv(yp->Hp), yp->H, yp->W, yp->pt, yp->pl,
            (int32_t)(0u - 128u * yp->C));
        count_launch();
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv planes reset");
}

// The GEMM epilogue's view of plane image yp from image n0 on.
PlaneOut plane_out(cm_planes* yp, uint64_t n0) {
    PlaneOut o;
    o.planes = yp->planes + n0 * yp->Hp * yp->Wp * yp->Cp;
    o.S = yp->S + n0 * yp->Hp * yp->Wp;
    o.plane_pitch = yp->plane_pitch;
    o.Hp = yp->Hp; o.Wp = yp->Wp; o.Cp = yp->Cp; o.pt = yp->pt; o.pl = yp->pl;
    return o;
}

// The space-to-depth plan conv_core uses: row stacking where the row-staged split kernel
// serves it and it saves K blocks.
bool choose_s2d(uint32_t in_ch, uint32_t in_w, uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t sh,
                uint32_t sw, uint32_t dh, uint32_t dw, S2dPlan* sp) {
    if (!plan_s2d(in_ch, out_h, out_w, kh, kw, sh, sw, dh, dw, sp)) return false;
    S2dPlan sp2;
    if (sh == 2 && in_ch == 3 && 4ull * in_ch * in_w * 2 <= kS2dRowSmem &&
        plan_s2d(in_ch, out_h, out_w, kh, kw, sh, sw, dh, dw, &sp2, 2) &&
        sp2.kh3 * (sp2.ip.KR_pad / 128) < sp->kh3 * (sp->ip.KR_pad / 128))
        *sp = sp2;
    return true;
}

}  // namespace

// Conv weights prepared once (cm_conv_weights_create): the weight planes and column terms
// the tensor-core paths read, built for one geometry, so calls with constant weights skip
// the per-call preparation.
struct cm_conv_weights {
    const int16_t* weight = nullptr;
    const int16_t* bias = nullptr;
    unsigned g[17] = {};               // batch .. is_depthwise, as the conv entry points take them
    int path = -1;                     // cm::ConvPath the planes were built for
    int8_t* planes = nullptr;          // conv_weights layout of that path
    int32_t* colterm = nullptr;
    int8_t* rows = nullptr;            // <= 64 channels: the weights-as-A rows [128][Kt]
    void* mem = nullptr;
    int device = -1;
};

namespace {

// xv: a plane image that fits this conv's implicit plan (read instead of x); po:
// the output's plane image, written by the GEMM epilogue (implicit / space-to-depth
// paths only; y may then be null); rp: the residual's plane image (same paths; resid
// may then be null).
// pw: prepared weight planes and column terms of this geometry's path (null: built here).
int conv_core(const int16_t* x, const cm_planes* xv, const int16_t* weight, const int16_t* bias, int16_t* y,
              cm_planes* po, const cm_planes* rp, unsigned batch, unsigned in_ch,
              unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh, unsigned kw,
              unsigned stride_h, unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
              unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned epi, const int16_t* resid,
              cm_stream_t stream, const cm_conv_weights* pw = nullptr) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    // epilogue bit 3: y is channels-last [batch][out_h][out_w][out_ch] (implicit-GEMM paths)
    const bool nhwc = (epi & 8u) != 0 && y != nullptr;
    epi &= 7u;
    const uint64_t P = (uint64_t)out_h * out_w;
    if (batch == 0 || out_ch == 0 || P == 0) return CM_OK;
    if ((!y && !po) || (has_bias && !bias)) return set_error(CM_EINVAL, "cm_conv: null buffer");
    if (P >= (1ull << 31)) return set_error(CM_EUNSUPPORTED, "cm_conv: output plane too large");
    cudaStream_t s = (cudaStream_t)stream;
    const uint64_t total = (uint64_t)batch * out_ch * P;

    if (nhwc && (is_depthwise || (uint64_t)in_ch * kh * kw == 0))
        return set_error(CM_EUNSUPPORTED, "cm_conv: channels-last output only on the implicit-GEMM paths");
    if (is_depthwise) {
        if (out_ch > in_ch)
            return set_error(CM_EINVAL, "cm_conv: depthwise needs out_ch <= in_ch (output channel m reads input channel m)");
        if ((uint64_t)kh * kw > 0 && (!x || !weight)) return set_error(CM_EINVAL, "cm_conv: null buffer");
        DwArgs a{in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left,
                 has_bias ? 1u : 0u};
        {
            ProfScope ps_(PK_CONV_AUX, s);
            launch_k(conv_depthwise_kernel, grid_for(cx, total, 256, 8), 256, 0, s, x, weight, bias, y, a, total);
            if (epi) launch_k(conv_epilogue_kernel, grid_for(cx, total, 256, 8), 256, 0, s, y, resid, total, epi);
        }
        count_launch(epi ? 2 : 1);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv depthwise");
    }

    const uint64_t K64 = (uint64_t)in_ch * kh * kw;
    if (K64 == 0) {
        {
            ProfScope ps_(PK_CONV_AUX, s);
            launch_k(conv_bias_fill_kernel, grid_for(cx, total, 256, 8), 256, 0, s, bias, y, out_ch, P, total, has_bias ? 1u : 0u);
            if (epi) launch_k(conv_epilogue_kernel, grid_for(cx, total, 256, 8), 256, 0, s, y, resid, total, epi);
        }
        count_launch(epi ? 2 : 1);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv bias fill");
    }
    if ((!x && !xv) || !weight) return set_error(CM_EINVAL, "cm_conv: null buffer");
    if (nhwc && (unsigned __int128)total * K64 <= cx->direct_max_macs)
        return set_error(CM_EUNSUPPORTED, "cm_conv: channels-last output only on the implicit-GEMM paths");
    if ((unsigned __int128)total * K64 <= cx->direct_max_macs) {
        DwArgs a{in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left,
                 has_bias ? 1u : 0u};
        {
            ProfScope ps_(PK_CONV_AUX, s);
            const uint32_t G = direct_lanes(cx, total, (uint64_t)in_ch * kh);
            launch_k(conv_direct_kernel, grid_for(cx, total * G, 256, 8), 256, 0, s, x, weight, bias, y, a, total, G, epi, resid);
        }
        count_launch();
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv direct");
    }
    if (K64 > kMaxGemmK) return set_error(CM_EUNSUPPORTED, "cm_conv: in_ch*kh*kw = %llu exceeds %u", (unsigned long long)K64, kMaxGemmK);
    const uint32_t K = (uint32_t)K64, K_pad = pad_k(K);

    ImplicitPlan ip;
    if (plan_implicit(in_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, &ip)) {
        // rows = output pixels of a chunk of images, columns = output channels
        const uint32_t M_pad = pad_c(out_ch);
        const bool packed = out_ch <= 64;                 // one 64-column tile
        const uint32_t w_pitch = packed ? 128u : M_pad;
        const uint64_t w_plane = packed ? 64u : (uint64_t)ip.Kt * M_pad;
        const uint64_t img_plane = (uint64_t)ip.Hp * ip.Wp * ip.Cp;
        uint64_t chunk = kNhwcBudget / (2 * img_plane);
        if (chunk == 0) chunk = 1;
        if (chunk > batch || xv) chunk = batch;           // a plane image holds every image already
        if (chunk > (1u << 24)) chunk = 1u << 24;
        // prepared weights (pw) replace the per-call weight planes and column terms
        const uint64_t w_bytes = pw ? 0 : ((uint64_t)ip.Kt * (packed ? 128 : 2 * M_pad) + 255) & ~255ull;
        const uint64_t ct_bytes = pw ? 0 : ((uint64_t)out_ch * 4 + 255) & ~255ull;
        const uint64_t a_bytes = xv ? 0 : (2 * chunk * img_plane + ip.KR + 256 + 255) & ~255ull;   // + slack past the last pixel
        const uint64_t s_bytes = xv ? 0 : (chunk * ip.Hp * ip.Wp * 4 + 255) & ~255ull;
        const uint64_t rt_bytes = (chunk * P * 4 + 255) & ~255ull;
        void* scratch = nullptr;
        rc = scratch_alloc(&scratch, w_bytes + ct_bytes + a_bytes + s_bytes + rt_bytes, s);
        if (rc) return rc;
        int8_t* wpl = pw ? pw->planes : (int8_t*)scratch;
        int32_t* ct = pw ? pw->colterm : (int32_t*)((int8_t*)scratch + w_bytes);
        int8_t* apl = (int8_t*)scratch + w_bytes + ct_bytes;
        int32_t* S = (int32_t*)(apl + a_bytes);
        int32_t* rt = (int32_t*)((int8_t*)S + s_bytes);
        if (!pw)
            rc = conv_weights(cx, weight, has_bias ? bias : nullptr, out_ch, in_ch, kh, kw, ip.Cp, ip.KR_pad, w_pitch,
                              w_plane, w_bytes, wpl, ct, s);
        // a plane-image input runs in one chunk: its row-term launch also clears the output
        // image's sums; otherwise a reset launch of its own
        if (!rc && po && !xv) rc = planes_reset(po, s);
        // a plane image read in place: the conv's padded window starts (dt, dl) into its frame
        const uint32_t dt = xv ? xv->pt - pad_top : 0u, dl = xv ? xv->pl - pad_left : 0u;
        for (uint64_t n0 = 0; !rc && n0 < batch; n0 += chunk) {
            const uint32_t nb = (uint32_t)((batch - n0) < chunk ? (batch - n0) : chunk);
            const NhwcGeom ng{in_ch, in_h, in_w, ip.Cp, ip.Hp, ip.Wp, pad_top, pad_left, nb};
            if (xv) {
                ProfScope ps_(PK_SPLIT, s);
                SumsReset z;
                if (po) z = SumsReset{po->S, nb, po->Hp, po->Wp, po->H, po->W, po->pt, po->pl, (int32_t)(0u - 128u * po->C)};
                rowterm_launch(cx, xv->S + (uint64_t)dt * xv->Wp + dl, xv->Hp, xv->Wp, out_h, out_w, kh, kw, stride_h,
                               stride_w, dilation_h, nb, rt, s, z);
            } else {
                ProfScope ps_(PK_SPLIT, s);
                const uint64_t HW = (uint64_t)in_h * in_w;
                const bool quads = HW % 4 == 0 && ((uintptr_t)x & 7u) == 0 && HW < (1ull << 31);
                const uint64_t img_smem = (((uint64_t)in_ch * HW * 2 + 15) & ~15ull) + (uint64_t)ip.Hp * ip.Wp * 4;
                const bool whole = !quads && img_smem <= kImgSplitSmem;
                if (whole) {
                    static bool attr = false;
                    if (!attr) {
                        cudaError_t e = cudaFuncSetAttribute(conv_nhwc_split_img_kernel,
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kImgSplitSmem);
                        if (e != cudaSuccess) { scratch_free(scratch, s); return cuda_error(e, "cudaFuncSetAttribute(split_img)"); }
                        attr = true;
                    }
                }
                const uint32_t gx = quads ? (uint32_t)((HW / 4 + 63) / 64)
                                          : (uint32_t)(((uint64_t)ip.Hp * ip.Wp + kNhwcPix - 1) / kNhwcPix);
                for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
                    const uint32_t bz = std::min(65535u, nb - b0);
                    // the plane stride stays that of the whole chunk (ng.nimg = nb)
                    const int16_t* xb = x + (n0 + b0) * (uint64_t)in_ch * in_h * in_w;
                    int8_t* pb = apl + (uint64_t)b0 * img_plane;
                    int32_t* Sb = S + (uint64_t)b0 * ip.Hp * ip.Wp;
                    if (quads) {
                        launch_k(conv_nhwc_split4_kernel, dim3(gx, bz), 256, 0, s, xb, ng, pb, Sb);
                        count_launch();
                    } else if (whole) {
                        launch_k(conv_nhwc_split_img_kernel, bz, kImgSplitThreads, (size_t)img_smem, s, xb, ng, pb, Sb);
                        count_launch();
                    } else {
                        launch_k(conv_nhwc_split_kernel, dim3(gx, bz), 256, 0, s, xb, ng, pb, Sb);
                        count_launch();
                    }
                }
                if (quads && (pad_top || pad_left || ip.Hp > pad_top + in_h || ip.Wp > pad_left + in_w)) {
                    const uint64_t frame = (uint64_t)2 * (ip.Hp + ip.Wp) * (pad_top + pad_left + ip.Hp + ip.Wp) * (ip.Cp / 16);
                    const uint32_t bx = (uint32_t)std::min<uint64_t>(8, (frame + 255) / 256);
                    for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
                        NhwcGeom gb = ng;
                        const uint32_t bz = std::min(65535u, nb - b0);
                        // images b0.. of the chunk: shift the planes / S bases, keep the chunk's plane stride
                        launch_k(conv_nhwc_border_kernel, dim3(bx, bz), 256, 0, s, gb, apl + (uint64_t)b0 * img_plane,
                                                                            S + (uint64_t)b0 * ip.Hp * ip.Wp);
                        count_launch();
                    }
                }
                rowterm_launch(cx, S, ip.Hp, ip.Wp, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, nb, rt, s);
            }
            uint32_t bw, bh, bn;
            pick_tiles(out_h, out_w, stride_h, stride_w, nb, y != nullptr && !nhwc, &bw, &bh, &bn);
            ConvA ca{apl, nb, ip.Cp, ip.Hp, ip.Wp, ip.KR, ip.KR_pad, kh, stride_h, stride_w, dilation_h,
                     out_h, out_w, log2u(bw), log2u(bh), log2u(bn)};
            if (xv) {
                // the plane image's own layout; boxes may read its whole frame past the plan's extent
                ca.planes = xv->planes + ((uint64_t)dt * xv->Wp + dl) * xv->Cp;
                ca.Hp = xv->Hp - dt; ca.Wp = xv->Wp - dl;
                ca.row_pitch = (uint64_t)xv->Wp * xv->Cp;
                ca.img_pitch = (uint64_t)xv->Hp * xv->Wp * xv->Cp;
                ca.plane_pitch = xv->plane_pitch;
            }
            GemmPlan p{nullptr, 0, 1, wpl, out_ch, 1, ip.Kt, ip.Kt, M_pad, rt, ct,
                       y ? y + n0 * (uint64_t)out_ch * P : nullptr, nhwc ? out_ch : 0u, nhwc ? 1u : P,
                       (uint64_t)out_ch * P, 1};
            p.conv = &ca;
            p.b_packed = packed ? 1u : 0u;
            p.wa_rows = pw ? pw->rows : nullptr;
            p.epi = epi;
            p.resid = resid ? resid + n0 * (uint64_t)out_ch * P : nullptr;
            if (po) p.po = plane_out(po, n0);
            if (rp) p.rp = plane_out(const_cast<cm_planes*>(rp), n0);
            rc = gemm_launch(cx, p, s);
        }
        scratch_free(scratch, s);
        if (rc) return rc;
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv");
    }

    S2dPlan sp;
    if (choose_s2d(in_ch, in_w, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, &sp)) {
        const ImplicitPlan& vp = sp.ip;
        const uint32_t M_pad = pad_c(out_ch);
        const bool packed = out_ch <= 64;
        const uint32_t w_pitch = packed ? 128u : M_pad;
        const uint64_t w_plane = packed ? 64u : (uint64_t)vp.Kt * M_pad;
        const uint64_t img_plane = (uint64_t)vp.Hp * vp.Wp * vp.Cp;
        const uint64_t img_so = (uint64_t)sp.Hpo * sp.Wpo;
        uint64_t chunk = kNhwcBudget / (2 * img_plane + 4 * img_so);
        if (chunk == 0) chunk = 1;
        if (chunk > batch) chunk = batch;
        if (chunk > (1u << 24)) chunk = 1u << 24;
        const uint64_t w_bytes = pw ? 0 : ((uint64_t)vp.Kt * (packed ? 128 : 2 * M_pad) + 255) & ~255ull;
        const uint64_t ct_bytes = pw ? 0 : ((uint64_t)out_ch * 4 + 255) & ~255ull;
        const uint64_t a_bytes = (2 * chunk * img_plane + vp.KR + 256 + 255) & ~255ull;
        const uint64_t s_bytes = (chunk * img_so * 4 + 255) & ~255ull;
        const uint64_t rt_bytes = (chunk * P * 4 + 255) & ~255ull;
        void* scratch = nullptr;
        rc = scratch_alloc(&scratch, w_bytes + ct_bytes + a_bytes + s_bytes + rt_bytes, s);
        if (rc) return rc;
        int8_t* wpl = pw ? pw->planes : (int8_t*)scratch;
        int32_t* ct = pw ? pw->colterm : (int32_t*)((int8_t*)scratch + w_bytes);
        int8_t* apl = (int8_t*)scratch + w_bytes + ct_bytes;
        int32_t* So = (int32_t*)(apl + a_bytes);
        int32_t* rt = (int32_t*)((int8_t*)So + s_bytes);
        // column terms from the original weights (real taps, bias), planes of the virtual kernel
        if (!pw) rc = conv_weights(cx, weight, has_bias ? bias : nullptr, out_ch, in_ch, kh, kw, 0, 0, 0, 0, 0, nullptr, ct, s);
        if (!rc && po) rc = planes_reset(po, s);
        if (!rc && !pw) {
            ProfScope ps_(PK_SPLIT, s);
            const uint64_t wtot = (uint64_t)vp.Kt * out_ch;
            launch_k(conv_s2d_weights_kernel, grid_for(cx, wtot, 256, 8), 256, 0, s, weight, out_ch, in_ch, kh, kw, sp.s, sp.kw2,
                                                                              vp.Cp, vp.KR_pad, vp.Kt, w_pitch, w_plane, wpl,
                                                                              sp.T);
            count_launch();
        }
        for (uint64_t n0 = 0; !rc && n0 < batch; n0 += chunk) {
            const uint32_t nb = (uint32_t)((batch - n0) < chunk ? (batch - n0) : chunk);
            const S2dGeom sg{in_ch, in_h, in_w, sp.s, sp.C2, vp.Cp, vp.Hp, vp.Wp, pad_top, pad_left, sp.Hpo, sp.Wpo, nb};
            const uint64_t vtot = (uint64_t)nb * vp.Hp * vp.Wp;
            {
                ProfScope ps_(PK_SPLIT, s);
                const int16_t* xc = x + n0 * (uint64_t)in_ch * in_h * in_w;
                const uint64_t row_smem = (uint64_t)sp.T * sp.s * in_ch * in_w * 2;
                bool rt_done = false;
                if (sp.T == 2) {
                    // bands of 4 virtual rows when their input rows fit, else 2, else 1
                    const uint64_t row_bytes = (uint64_t)in_ch * in_w * 2;
                    const uint32_t rb = s2d_band_rows(2, 2, 4) * row_bytes <= kS2dRowSmem ? 4u
                                        : s2d_band_rows(2, 2, 2) * row_bytes <= kS2dRowSmem ? 2u : 1u;
                    // the 7 x 7 stride-2 stem: the band also computes its output rows' row terms
                    // (13 staged rows instead of 10, no So, no row-term launch)
                    const uint64_t fused_smem = s2d_stage_rows(2, 2, 4, 7) * row_bytes + 16 + 4ull * 4 * sp.Wpo;
                    const bool fuse_rt = rb == 4 && kh == 7 && kw <= 16 && dilation_h == 1 && dilation_w == 1 &&
                                         fused_smem <= kS2dRowSmem;
                    const size_t band_smem = fuse_rt ? (size_t)fused_smem : (size_t)(s2d_band_rows(2, 2, rb) * row_bytes);
                    const uint32_t gx = (vp.Hp + rb - 1) / rb;
                    for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
                        const uint32_t bz = std::min(65535u, nb - b0);
                        const int16_t* xb = xc + (uint64_t)b0 * in_ch * in_h * in_w;
                        int8_t* pb = apl + (uint64_t)b0 * img_plane;
                        int32_t* sb = So + (uint64_t)b0 * img_so;
                        const S2dRt none{nullptr, 0, 0, 0};
                        if (fuse_rt) {
                            const S2dRt fr{rt + (uint64_t)b0 * P, out_h, out_w, kw};
                            launch_k(conv_s2d_rows_kernel<2, 3, 2, 4, 7>, dim3(gx, bz), kS2dRowThreads, band_smem, s, xb, sg, pb, sb, fr);
                        }
                        else if (rb == 4) launch_k(conv_s2d_rows_kernel<2, 3, 2, 4>, dim3(gx, bz), kS2dRowThreads, band_smem, s, xb, sg, pb, sb, none);
                        else if (rb == 2) launch_k(conv_s2d_rows_kernel<2, 3, 2, 2>, dim3(gx, bz), kS2dRowThreads, band_smem, s, xb, sg, pb, sb, none);
                        else launch_k(conv_s2d_rows_kernel<2, 3, 2, 1>, dim3(gx, bz), kS2dRowThreads, band_smem, s, xb, sg, pb, sb, none);
                        count_launch();
                    }
                    rt_done = fuse_rt;
                } else if (sp.s == 2 && in_ch == 3 && row_smem <= kS2dRowSmem && vp.Hp < (1u << 31)) {
                    for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
                        const uint32_t bz = std::min(65535u, nb - b0);
                        // images b0..: shift the input, planes and So bases; the plane stride stays the chunk's
                        launch_k(conv_s2d_rows_kernel<2, 3>, dim3(vp.Hp, bz), kS2dRowThreads, (size_t)row_smem, s, 
                            xc + (uint64_t)b0 * in_ch * in_h * in_w, sg, apl + (uint64_t)b0 * img_plane, So + (uint64_t)b0 * img_so,
                            S2dRt{nullptr, 0, 0, 0});
                        count_launch();
                    }
                } else if (sp.s == 2 && in_ch == 3) {
                    launch_k(conv_s2d_split_kernel<2, 3>, grid_for(cx, vtot, 256, 8), 256, 0, s, xc, sg, vtot, apl, So);
                    count_launch();
                } else {
                    launch_k(conv_s2d_split_kernel<0, 0>, grid_for(cx, vtot, 256, 8), 256, 0, s, xc, sg, vtot, apl, So);
                    count_launch();
                }
                if (!rt_done) rowterm_launch(cx, So, sp.Hpo, sp.Wpo, out_h, out_w, kh, kw, sp.s, sp.s, 1, nb, rt, s);
            }
            uint32_t bw, bh, bn;
            pick_tiles(out_h, out_w, 1, 1, nb, y != nullptr && !nhwc, &bw, &bh, &bn);
            const ConvA ca{apl, nb, vp.Cp, vp.Hp, vp.Wp, vp.KR, vp.KR_pad, sp.kh3, 1, 1, sp.T,
                           out_h, out_w, log2u(bw), log2u(bh), log2u(bn)};
            GemmPlan p{nullptr, 0, 1, wpl, out_ch, 1, vp.Kt, vp.Kt, M_pad, rt, ct,
                       y ? y + n0 * (uint64_t)out_ch * P : nullptr, nhwc ? out_ch : 0u, nhwc ? 1u : P,
                       (uint64_t)out_ch * P, 1};
            p.conv = &ca;
            p.b_packed = packed ? 1u : 0u;
            p.wa_rows = pw ? pw->rows : nullptr;
            p.epi = epi;
            p.resid = resid ? resid + n0 * (uint64_t)out_ch * P : nullptr;
            if (po) p.po = plane_out(po, n0);
            if (rp) p.rp = plane_out(const_cast<cm_planes*>(rp), n0);
            rc = gemm_launch(cx, p, s);
        }
        scratch_free(scratch, s);
        if (rc) return rc;
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv");
    }

    // Explicit im2col: rows = output pixels of a chunk of images (K-major planes),
    // columns = output channels, K in the weight layout's (c, r, s) order.
    const uint32_t M_pad = pad_c(out_ch);
    if (nhwc) return set_error(CM_EUNSUPPORTED, "cm_conv: channels-last output only on the implicit-GEMM paths");
    const bool packed = out_ch <= 64;
    const uint32_t w_pitch = packed ? 128u : M_pad;
    const uint64_t w_plane = packed ? 64u : (uint64_t)K * M_pad;
    const uint64_t per_img = 2 * (uint64_t)K_pad * P;
    uint64_t chunk = kIm2colBudget / per_img;
    if (chunk == 0) chunk = 1;
    if (chunk > batch) chunk = batch;
    if (chunk * P >= (1ull << 31)) chunk = ((1ull << 31) - 1) / P;
    const uint64_t w_bytes = pw ? 0 : ((uint64_t)K * (packed ? 128 : 2 * M_pad) + 255) & ~255ull;
    const uint64_t ct_bytes = pw ? 0 : ((uint64_t)out_ch * 4 + 255) & ~255ull;
    const uint64_t a_bytes = (chunk * per_img + 255) & ~255ull;
    const uint64_t rt_bytes = (chunk * P * 4 + 255) & ~255ull;
    void* scratch = nullptr;
    rc = scratch_alloc(&scratch, w_bytes + ct_bytes + a_bytes + rt_bytes, s);
    if (rc) return rc;
    int8_t* wpl = pw ? pw->planes : (int8_t*)scratch;
    int32_t* ct = pw ? pw->colterm : (int32_t*)((int8_t*)scratch + w_bytes);
    int8_t* apl = (int8_t*)scratch + w_bytes + ct_bytes;
    int32_t* rt = (int32_t*)(apl + a_bytes);

    // natural tap order: kh = kw = 1, C = Cp = KR_pad = K
    if (!pw)
        rc = conv_weights(cx, weight, has_bias ? bias : nullptr, out_ch, K, 1, 1, K, K, w_pitch, w_plane, w_bytes, wpl, ct,
                          s);
    const ConvGeom geo{in_ch, in_h, in_w, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left};
    // shared-memory window im2col when one block's window (C x kh rows x the columns
    // 128 pixels span) fits; the direct gather otherwise
    const uint64_t WC64 = (uint64_t)(std::min<uint32_t>(out_w, kIcRows) - 1) * stride_w + (uint64_t)(kw - 1) * dilation_w + 1;
    const uint64_t win_bytes = ((uint64_t)in_ch * kh * WC64 + (uint64_t)(kIcRows - 1) * stride_w + 1) * 2;
    const uint32_t WC = (uint32_t)std::min<uint64_t>(WC64, 1u << 20);
    size_t win_smem = 0;
    if (win_bytes <= kWinMax && out_h <= 65535 && batch <= 65535) {
        win_smem = (size_t)2 * kIcRows * kIcPitch + kIcSlice * 4 + (size_t)win_bytes;
        if (cudaFuncSetAttribute(im2col_win_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)win_smem) != cudaSuccess) {
            cudaGetLastError();
            win_smem = 0;
        }
    }
    for (uint64_t n0 = 0; !rc && n0 < batch; n0 += chunk) {
        const uint32_t nb = (uint32_t)((batch - n0) < chunk ? (batch - n0) : chunk);
        const uint64_t rows = (uint64_t)nb * P;
        {
            ProfScope ps_(PK_SPLIT, s);
            const int16_t* xc = x + n0 * (uint64_t)in_ch * in_h * in_w;
            if (win_smem) {
                const dim3 grid((out_w + kIcRows - 1) / kIcRows, out_h, nb);
                launch_k(im2col_win_kernel, grid, kIcRows, win_smem, s, xc, geo, (uint32_t)P, rows, K, K_pad, WC, FastDiv(WC),
                                                                  FastDiv(kh), apl, rt);
            } else {
                launch_k(im2col_rows_kernel, (unsigned)((rows + kIcRows - 1) / kIcRows), kIcRows, 0, s, xc, geo, (uint32_t)P, rows,
                                                                                              K, K_pad, apl, rt);
            }
        }
        count_launch();
        GemmPlan p{apl, (uint32_t)rows, 1, wpl, out_ch, 1, K, K_pad, M_pad, rt, ct,
                   y + n0 * (uint64_t)out_ch * P, 0, P, (uint64_t)out_ch * P, 1};
        p.b_packed = packed ? 1u : 0u;
        p.rows_per_img = (uint32_t)P;
        p.epi = epi;
        p.resid = resid ? resid + n0 * (uint64_t)out_ch * P : nullptr;
        rc = gemm_launch(cx, p, s);
    }
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv");
}

// Conv with optional plane images on either side: xp replaces x when this conv's
// path is the implicit GEMM and xp's frame covers its padding (else x is read and
// must be given); yp receives the output as a plane image -- written by the GEMM
// epilogue on the implicit and space-to-depth paths, by the split kernels from y
// (or a scratch copy of it when y is null) otherwise.
int conv_impl(const int16_t* x, const cm_planes* xp, const int16_t* weight, const int16_t* bias, int16_t* y,
              cm_planes* yp, unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
              unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
              unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
              unsigned is_depthwise, unsigned epi, const int16_t* resid, const cm_planes* rp, cm_stream_t stream,
              const cm_conv_weights* pw = nullptr) {
    if (!(epi & 2u)) rp = nullptr;
    if (!xp && !yp && !rp)
        return conv_core(x, nullptr, weight, bias, y, nullptr, nullptr, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
                         stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epi,
                         resid, stream, pw);
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if ((xp && xp->device != cx->device) || (yp && yp->device != cx->device))
        return set_error(CM_EINVAL, "cm_conv: plane image of another device");
    if (yp && (yp->n != batch || yp->C != out_ch || yp->H != out_h || yp->W != out_w))
        return set_error(CM_EINVAL, "cm_conv: output plane image is %ux%ux%ux%u, the output %ux%ux%ux%u", yp->n, yp->C,
                         yp->H, yp->W, batch, out_ch, out_h, out_w);
    if (rp && (rp->device != cx->device || rp->n != batch || rp->C != out_ch || rp->H != out_h || rp->W != out_w))
        return set_error(CM_EINVAL, "cm_conv: residual plane image does not match the output");
    ImplicitPlan ip;
    const ConvPath path = conv_path(cx->direct_max_macs, batch, in_ch, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                                    dilation_h, dilation_w, is_depthwise, &ip);
    const cm_planes* xv = path == CP_IMPLICIT && planes_fit(xp, batch, in_ch, in_h, in_w, pad_top, pad_left, ip) ? xp : nullptr;
    if (!xv && !x && path != CP_BIAS_FILL)
        return set_error(CM_EINVAL, "cm_conv: x is null and this conv cannot read the plane image (not an implicit-GEMM "
                                    "conv, or the image's tensor or frame does not match)");
    const bool gemm_epi = path == CP_IMPLICIT || path == CP_S2D;   // epilogue in the tensor-core GEMM
    const cm_planes* rv = gemm_epi ? rp : nullptr;
    if (rp && !rv && !resid)
        return set_error(CM_EINVAL, "cm_conv: resid is null and this conv cannot read the residual plane image");
    if (!rv && (epi & 2u) && !resid) return set_error(CM_EINVAL, "cm_conv: residual buffer is null");
    const bool epi_writes = yp && gemm_epi;
    if (!yp || epi_writes)
        return conv_core(x, xv, weight, bias, y, epi_writes ? yp : nullptr, rv, batch, in_ch, in_h, in_w, out_ch, out_h,
                         out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias,
                         is_depthwise, epi, resid, stream, pw);
    cudaStream_t s = (cudaStream_t)stream;
    int16_t* yw = y;
    void* tmp = nullptr;
    if (!yw) {
        rc = scratch_alloc(&tmp, ((uint64_t)batch * out_ch * out_h * out_w * 2 + 255) & ~255ull, s);
        if (rc) return rc;
        yw = (int16_t*)tmp;
    }
    rc = conv_core(x, xv, weight, bias, yw, nullptr, rv, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                   stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epi, resid, stream, pw);
    if (!rc) rc = planes_from_tensor(cx, yw, yp, s);
    if (tmp) scratch_free(tmp, s);
    return rc;
}

}  // namespace

extern "C" int cm_conv_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                             unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h,
                             unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
                             unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                             unsigned has_bias, unsigned is_depthwise, cm_stream_t stream) {
    return conv_impl(x, nullptr, weight, bias, y, nullptr, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
                     stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, 0u, nullptr,
                     nullptr, stream);
}

extern "C" int cm_conv_fused_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
                                   unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                                   unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                                   unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                                   unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned epilogue,
                                   const int16_t* resid, cm_stream_t stream) {
    if (epilogue > 3u) return set_error(CM_EINVAL, "cm_conv_fused: epilogue must be 0..3");
    if ((epilogue & 2u) && !resid) return set_error(CM_EINVAL, "cm_conv_fused: residual buffer is null");
    return conv_impl(x, nullptr, weight, bias, y, nullptr, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
                     stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epilogue,
                     resid, nullptr, stream);
}

extern "C" int cm_conv_pool_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
                                  unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                                  unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                                  unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                                  unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned epilogue,
                                  const int16_t* resid, unsigned p_batch, unsigned p_channels, unsigned p_in_h,
                                  unsigned p_in_w, unsigned p_out_h, unsigned p_out_w, unsigned pool_h, unsigned pool_w,
                                  unsigned p_stride_h, unsigned p_stride_w, unsigned p_pad_top, unsigned p_pad_left,
                                  unsigned p_dil_h, unsigned p_dil_w, unsigned pool_type, unsigned lp_order,
                                  unsigned count_include_pad, cm_stream_t stream) {
    (void)lp_order; (void)count_include_pad;
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (epilogue > 3u) return set_error(CM_EINVAL, "cm_conv_pool: epilogue must be 0..3");
    if (p_batch != batch || p_channels != out_ch || p_in_h != out_h || p_in_w != out_w)
        return set_error(CM_EINVAL, "cm_conv_pool: the pool's input is not the conv's output");
    if (pool_type != CM_POOL_MAX) return set_error(CM_EUNSUPPORTED, "cm_conv_pool: MAX pooling only");
    if (is_depthwise) return set_error(CM_EUNSUPPORTED, "cm_conv_pool: standard convs only");
    const uint64_t total = (uint64_t)batch * out_ch * p_out_h * p_out_w;
    if (total == 0) return CM_OK;
    if (!x || !weight || !y || (has_bias && !bias) || ((epilogue & 2u) && !resid))
        return set_error(CM_EINVAL, "cm_conv_pool: null buffer");
    const DwArgs a{in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top,
                   pad_left, has_bias ? 1u : 0u};
    const PoolGeo q{p_out_h, p_out_w, pool_h, pool_w, p_stride_h, p_stride_w, p_pad_top, p_pad_left, p_dil_h, p_dil_w};
    cudaStream_t s = (cudaStream_t)stream;
    {
        ProfScope ps_(PK_CONV_AUX, s);
        // tap slots: the pool window's taps rounded up to a power of two; then reduction lanes
        // while the slots x lanes stay within a warp
        uint32_t T = 1;
        while (T < (uint64_t)pool_h * pool_w && T < 32) T *= 2;
        uint32_t G = direct_lanes(cx, total * T, (uint64_t)in_ch * kh);
        while (G * T > 32) G /= 2;
        launch_k(conv_pool_direct_kernel, grid_for(cx, total * G * T, 256, 8), 256, 0, s, x, weight, bias, y, a, q, total,
                 G, T, epilogue, resid);
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv_pool");
}

extern "C" int cm_conv_pool(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                            unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h,
                            unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
                            unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                            unsigned has_bias, unsigned is_depthwise, unsigned epilogue, const int16_t* resid,
                            unsigned p_batch, unsigned p_channels, unsigned p_in_h, unsigned p_in_w, unsigned p_out_h,
                            unsigned p_out_w, unsigned pool_h, unsigned pool_w, unsigned p_stride_h,
                            unsigned p_stride_w, unsigned p_pad_top, unsigned p_pad_left, unsigned p_dil_h,
                            unsigned p_dil_w, unsigned pool_type, unsigned lp_order, unsigned count_include_pad) {
    int rc = cm_conv_pool_async(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                                stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epilogue,
                                resid, p_batch, p_channels, p_in_h, p_in_w, p_out_h, p_out_w, pool_h, pool_w,
                                p_stride_h, p_stride_w, p_pad_top, p_pad_left, p_dil_h, p_dil_w, pool_type, lp_order,
                                count_include_pad, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_conv_fused(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                             unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h,
                             unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
                             unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                             unsigned has_bias, unsigned is_depthwise, unsigned epilogue, const int16_t* resid) {
    int rc = cm_conv_fused_async(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                                 stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epilogue,
                                 resid, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_conv(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                       unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w,
                       unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                       unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
                       unsigned is_depthwise) {
    int rc = cm_conv_async(x, weight, bias, y, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                           stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

// ---------------------------------------------------------------------------
// Plane images (no reference counterpart): a conv's output written directly as
// the next implicit-GEMM conv's A operand
// ---------------------------------------------------------------------------
extern "C" cm_planes_t* cm_planes_create(unsigned batch, unsigned channels, unsigned h, unsigned w, unsigned pad_top,
                                         unsigned pad_left, unsigned pad_bottom, unsigned pad_right) {
    const Context* cx;
    if (enter(&cx)) return nullptr;
    if (batch == 0 || channels == 0 || h == 0 || w == 0) {
        set_error(CM_EINVAL, "cm_planes_create: empty tensor");
        return nullptr;
    }
    const uint64_t Cp = (channels + 15ull) & ~15ull, Hp = (uint64_t)pad_top + h + pad_bottom,
                   Wp = (uint64_t)pad_left + w + pad_right;
    if (Cp > 8192 || Hp * Wp >= (1ull << 31) || (uint64_t)batch * Hp * Wp * Cp >= (1ull << 40)) {
        set_error(CM_EUNSUPPORTED, "cm_planes_create: image too large");
        return nullptr;
    }
    cm_planes* p = new (std::nothrow) cm_planes();
    if (!p) return nullptr;
    p->n = batch; p->C = channels; p->H = h; p->W = w; p->Cp = (uint32_t)Cp; p->Hp = (uint32_t)Hp; p->Wp = (uint32_t)Wp;
    p->pt = pad_top; p->pl = pad_left; p->device = cx->device;
    p->plane_pitch = (uint64_t)batch * Hp * Wp * Cp;
    // slack past the lo plane: a conv box reads up to a kernel row (kw * Cp bytes) past a pixel
    const uint64_t slack = 65536 + 256;
    cudaError_t e = cudaMalloc(&p->planes, 2 * p->plane_pitch + slack);
    if (e == cudaSuccess) e = cudaMalloc(&p->S, (uint64_t)batch * Hp * Wp * 4);
    // x = 0 everywhere (hi 0, lo' 0x80): the frame and the channels past C keep it for good
    if (e == cudaSuccess) e = cudaMemset(p->planes, 0, p->plane_pitch);
    if (e == cudaSuccess) e = cudaMemset(p->planes + p->plane_pitch, 0x80, p->plane_pitch + slack);
    if (e == cudaSuccess && planes_reset(p, nullptr) != CM_OK) e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) {
        cuda_error(e, "cm_planes_create");
        cudaFree(p->planes);
        cudaFree(p->S);
        delete p;
        return nullptr;
    }
    return p;
}

extern "C" void cm_planes_destroy(cm_planes_t* p) {
    if (!p) return;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(p->device);
    cudaFree(p->planes);
    cudaFree(p->S);
    if (cur >= 0) cudaSetDevice(cur);
    delete p;
}

extern "C" int cm_conv_plane_frame(unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                                   unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                                   unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                                   unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned* frame) {
    (void)has_bias;
    const Context* c = ctx();
    const uint64_t limit = c ? c->direct_max_macs : (1ull << 22);
    ImplicitPlan ip;
    if (batch == 0 || out_ch == 0 || (uint64_t)out_h * out_w == 0 ||
        conv_path(limit, batch, in_ch, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w,
                  is_depthwise, &ip) != CP_IMPLICIT)
        return 0;
    if (frame) {
        frame[0] = pad_top;
        frame[1] = pad_left;
        frame[2] = ip.Hp > (uint64_t)pad_top + in_h ? ip.Hp - pad_top - in_h : 0u;
        frame[3] = ip.Wp > (uint64_t)pad_left + in_w ? ip.Wp - pad_left - in_w : 0u;
    }
    return 1;
}

extern "C" int cm_conv_writes_nhwc(unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                                   unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                                   unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                                   unsigned pad_left, unsigned has_bias, unsigned is_depthwise) {
    (void)in_h; (void)in_w; (void)pad_top; (void)pad_left; (void)has_bias;
    const Context* c = ctx();
    const uint64_t limit = c ? c->direct_max_macs : (1ull << 22);
    ImplicitPlan ip;
    if (batch == 0 || out_ch == 0 || (uint64_t)out_h * out_w == 0) return 0;
    const ConvPath path = conv_path(limit, batch, in_ch, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h,
                                    dilation_w, is_depthwise, &ip);
    return path == CP_IMPLICIT || path == CP_S2D ? 1 : 0;
}

extern "C" int cm_conv_planes_async(const int16_t* x, const cm_planes_t* xp, const int16_t* weight, const int16_t* bias,
                                    int16_t* y, cm_planes_t* yp, unsigned batch, unsigned in_ch, unsigned in_h,
                                    unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh,
                                    unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                                    unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
                                    unsigned is_depthwise, unsigned epilogue, const int16_t* resid,
                                    const cm_planes_t* resid_planes, cm_stream_t stream) {
    if ((epilogue & ~8u) > 3u) return set_error(CM_EINVAL, "cm_conv_planes: epilogue must be 0..3, plus 8 for channels-last y");
    if ((epilogue & 2u) && !resid && !resid_planes) return set_error(CM_EINVAL, "cm_conv_planes: residual buffer is null");
    if (!y && !yp) return set_error(CM_EINVAL, "cm_conv_planes: neither y nor an output plane image");
    return conv_impl(x, xp, weight, bias, y, yp, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h,
                     stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise, epilogue, resid,
                     resid_planes, stream);
}

extern "C" int cm_conv_planes(const int16_t* x, const cm_planes_t* xp, const int16_t* weight, const int16_t* bias,
                              int16_t* y, cm_planes_t* yp, unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w,
                              unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh, unsigned kw,
                              unsigned stride_h, unsigned stride_w, unsigned dilation_h, unsigned dilation_w,
                              unsigned pad_top, unsigned pad_left, unsigned has_bias, unsigned is_depthwise,
                              unsigned epilogue, const int16_t* resid, const cm_planes_t* resid_planes) {
    int rc = cm_conv_planes_async(x, xp, weight, bias, y, yp, batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw,
                                  stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise,
                                  epilogue, resid, resid_planes, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_planes_fill_async(cm_planes_t* p, const int16_t* x, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!p || !x) return set_error(CM_EINVAL, "cm_planes_fill: null argument");
    if (p->device != cx->device) return set_error(CM_EINVAL, "cm_planes_fill: plane image of another device");
    return planes_from_tensor(cx, x, p, (cudaStream_t)stream);
}

extern "C" int cm_planes_fill(cm_planes_t* p, const int16_t* x) {
    int rc = cm_planes_fill_async(p, x, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_pool_planes_async(const cm_planes_t* xp, cm_planes_t* yp, unsigned batch, unsigned channels,
                                    unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h,
                                    unsigned pool_w, unsigned stride_h, unsigned stride_w, unsigned pad_top,
                                    unsigned pad_left, unsigned dil_h, unsigned dil_w, unsigned pool_type,
                                    unsigned lp_order, unsigned count_include_pad, cm_stream_t stream) {
    (void)lp_order;
    (void)count_include_pad;
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!xp || !yp) return set_error(CM_EINVAL, "cm_pool_planes: null plane image");
    if (pool_type != CM_POOL_MAX) return set_error(CM_EUNSUPPORTED, "cm_pool_planes: MAX pooling only");
    if (xp->device != cx->device || yp->device != cx->device)
        return set_error(CM_EINVAL, "cm_pool_planes: plane image of another device");
    if (xp->n != batch || xp->C != channels || xp->H != in_h || xp->W != in_w || yp->n != batch ||
        yp->C != channels || yp->H != out_h || yp->W != out_w || xp->Cp != yp->Cp)
        return set_error(CM_EINVAL, "cm_pool_planes: plane images do not match the pool's tensors");
    const uint64_t total = (uint64_t)batch * out_h * out_w;
    if (total == 0) return CM_OK;
    if (total >= (1ull << 32)) return set_error(CM_EUNSUPPORTED, "cm_pool_planes: output too large");
    PoolPlanesGeo g{in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top, pad_left, dil_h, dil_w,
                    channels, xp->Cp, xp->Hp, xp->Wp, xp->pt, xp->pl, yp->Hp, yp->Wp, yp->pt, yp->pl,
                    xp->plane_pitch, yp->plane_pitch};
    cudaStream_t s = (cudaStream_t)stream;
    {
        ProfScope ps_(PK_POOL, s);
        launch_k(pool_max_planes_kernel, grid_for(cx, total, 256, 8), 256, 0, s, xp->planes, yp->planes, yp->S, g, total,
                                                                        FastDiv(out_w), FastDiv(out_h));
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_pool_planes");
}

extern "C" int cm_pool_planes(const cm_planes_t* xp, cm_planes_t* yp, unsigned batch, unsigned channels,
                              unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h,
                              unsigned pool_w, unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                              unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                              unsigned count_include_pad) {
    int rc = cm_pool_planes_async(xp, yp, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h,
                                  stride_w, pad_top, pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad,
                                  nullptr);
    return rc ? rc : finish_sync(nullptr);
}

extern "C" int cm_pool_nhwc_planes_async(const int16_t* x, cm_planes_t* yp, unsigned batch, unsigned channels,
                                         unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h,
                                         unsigned pool_w, unsigned stride_h, unsigned stride_w, unsigned pad_top,
                                         unsigned pad_left, unsigned dil_h, unsigned dil_w, unsigned pool_type,
                                         cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!x || !yp) return set_error(CM_EINVAL, "cm_pool_nhwc_planes: null buffer");
    if (pool_type != CM_POOL_MAX) return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc_planes: MAX pooling only");
    if (channels % 16u != 0) return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc_planes: channels must be a multiple of 16");
    if (yp->device != cx->device) return set_error(CM_EINVAL, "cm_pool_nhwc_planes: plane image of another device");
    if (yp->n != batch || yp->C != channels || yp->H != out_h || yp->W != out_w)
        return set_error(CM_EINVAL, "cm_pool_nhwc_planes: the plane image does not match the pool's output");
    uint32_t g_log = 0;
    while ((16u << g_log) < yp->Cp) ++g_log;
    if ((16u << g_log) != yp->Cp || g_log > 5)
        return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc_planes: %u padded channels (16 x a power of two up to 512)", yp->Cp);
    const uint64_t total = ((uint64_t)batch * out_h * out_w) << g_log;
    if (total == 0) return CM_OK;
    if (total >= (1ull << 32)) return set_error(CM_EUNSUPPORTED, "cm_pool_nhwc_planes: output too large");
    PoolPlanesGeo g{in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top, pad_left, dil_h, dil_w,
                    channels, yp->Cp, 0, 0, 0, 0, yp->Hp, yp->Wp, yp->pt, yp->pl, 0, yp->plane_pitch};
    cudaStream_t s = (cudaStream_t)stream;
    {
        ProfScope ps_(PK_POOL, s);
        launch_k(pool_max_nhwc_planes_kernel, grid_for(cx, total, 256, 8), 256, 0, s, x, yp->planes, yp->S, g, total,
                 g_log, FastDiv(out_w), FastDiv(out_h));
    }
    count_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_pool_nhwc_planes");
}

extern "C" int cm_pool_nhwc_planes(const int16_t* x, cm_planes_t* yp, unsigned batch, unsigned channels, unsigned in_h,
                                   unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                                   unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                                   unsigned dil_h, unsigned dil_w, unsigned pool_type) {
    int rc = cm_pool_nhwc_planes_async(x, yp, batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h,
                                       stride_w, pad_top, pad_left, dil_h, dil_w, pool_type, nullptr);
    return rc ? rc : finish_sync(nullptr);
}

// ---------------------------------------------------------------------------
// Prepared conv weights (no reference counterpart): the tensor-core paths' weight planes,
// column terms and weights-as-A rows built once for one geometry.
// ---------------------------------------------------------------------------
extern "C" int cm_conv_weights_create(const int16_t* weight, const int16_t* bias, unsigned batch, unsigned in_ch,
                                      unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w,
                                      unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
                                      unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                                      unsigned has_bias, unsigned is_depthwise, cm_conv_weights_t** out) {
    if (out) *out = nullptr;                // null on every failure
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!out) return set_error(CM_EINVAL, "cm_conv_weights_create: null result pointer");
    if (has_bias && !bias) return set_error(CM_EINVAL, "cm_conv_weights_create: null bias");
    const uint64_t K64 = (uint64_t)in_ch * kh * kw;
    if (K64 > 0 && !weight) return set_error(CM_EINVAL, "cm_conv_weights_create: null weight");
    cm_conv_weights* w = new (std::nothrow) cm_conv_weights;
    if (!w) return set_error(CM_ENOMEM, "cm_conv_weights_create: out of host memory");
    w->weight = weight;
    w->bias = has_bias ? bias : nullptr;
    const unsigned g[17] = {batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                            dilation_h, dilation_w, pad_top, pad_left, has_bias, is_depthwise};
    std::copy(g, g + 17, w->g);
    w->device = cx->device;
    ImplicitPlan ip;
    const ConvPath path = (batch == 0 || out_ch == 0 || (uint64_t)out_h * out_w == 0)
                              ? CP_BIAS_FILL
                              : conv_path(cx->direct_max_macs, batch, in_ch, out_ch, out_h, out_w, kh, kw, stride_h, stride_w,
                                          dilation_h, dilation_w, is_depthwise, &ip);
    w->path = (int)path;
    const uint32_t M_pad = pad_c(out_ch);
    const bool packed = out_ch <= 64;
    uint32_t Kt = 0;
    S2dPlan sp;
    if (path == CP_IMPLICIT) Kt = ip.Kt;
    else if (path == CP_S2D && choose_s2d(in_ch, in_w, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, &sp))
        Kt = sp.ip.Kt;
    else if (path == CP_EXPLICIT) Kt = (uint32_t)K64;
    if (Kt == 0) {                  // nothing to prepare on this path: calls read weight and bias
        w->path = path == CP_S2D ? -1 : (int)path;
        *out = w;
        return CM_OK;
    }
    const uint64_t w_bytes = ((uint64_t)Kt * (packed ? 128 : 2 * M_pad) + 255) & ~255ull;
    const uint64_t ct_bytes = ((uint64_t)out_ch * 4 + 255) & ~255ull;
    const bool rows = packed && path != CP_EXPLICIT;      // the weights-as-A form is a conv-mode GEMM
    const uint64_t r_bytes = rows ? ((uint64_t)Kt * 128 + 255) & ~255ull : 0;
    cudaError_t e = cudaMalloc(&w->mem, w_bytes + ct_bytes + r_bytes);
    if (e != cudaSuccess) { delete w; return cuda_error(e, "cm_conv_weights_create: cudaMalloc"); }
    w->planes = (int8_t*)w->mem;
    w->colterm = (int32_t*)((int8_t*)w->mem + w_bytes);
    w->rows = rows ? (int8_t*)w->mem + w_bytes + ct_bytes : nullptr;
    cudaStream_t s = nullptr;
    const uint32_t w_pitch = packed ? 128u : M_pad;
    if (path == CP_IMPLICIT) {
        rc = conv_weights(cx, weight, w->bias, out_ch, in_ch, kh, kw, ip.Cp, ip.KR_pad, w_pitch,
                          packed ? 64u : (uint64_t)Kt * M_pad, w_bytes, w->planes, w->colterm, s);
    } else if (path == CP_S2D) {
        rc = conv_weights(cx, weight, w->bias, out_ch, in_ch, kh, kw, 0, 0, 0, 0, 0, nullptr, w->colterm, s);
        if (!rc) {
            const ImplicitPlan& vp = sp.ip;
            const uint64_t wtot = (uint64_t)Kt * out_ch;
            launch_k(conv_s2d_weights_kernel, grid_for(cx, wtot, 256, 8), 256, 0, s, weight, out_ch, in_ch, kh, kw, sp.s, sp.kw2,
                                                                              vp.Cp, vp.KR_pad, Kt, w_pitch,
                                                                              packed ? 64u : (uint64_t)Kt * M_pad, w->planes,
                                                                              sp.T);
            count_launch();
        }
    } else {
        rc = conv_weights(cx, weight, w->bias, out_ch, (uint32_t)K64, 1, 1, (uint32_t)K64, (uint32_t)K64, w_pitch,
                          packed ? 64u : (uint64_t)Kt * M_pad, w_bytes, w->planes, w->colterm, s);
    }
    if (!rc && rows) rc = weights_to_rows(cx, w->planes, Kt, w->rows, s);
    if (!rc) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_error(e, "cm_conv_weights_create");
    }
    if (rc) {
        cudaFree(w->mem);
        delete w;
        return rc;
    }
    *out = w;
    return CM_OK;
}

extern "C" void cm_conv_weights_destroy(cm_conv_weights_t* w) {
    if (!w) return;
    if (w->mem) {
        int cur = -1;
        cudaGetDevice(&cur);
        if (w->device >= 0 && cur != w->device) cudaSetDevice(w->device);
        cudaFree(w->mem);
        if (cur >= 0 && cur != w->device) cudaSetDevice(cur);
    }
    delete w;
}

extern "C" int cm_conv_prepared_async(const cm_conv_weights_t* w, const int16_t* x, const cm_planes_t* xp, int16_t* y,
                                      cm_planes_t* yp, unsigned epilogue, const int16_t* resid,
                                      const cm_planes_t* resid_planes, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (!w) return set_error(CM_EINVAL, "cm_conv_prepared: null prepared weights");
    if (w->device != cx->device) return set_error(CM_EINVAL, "cm_conv_prepared: weights prepared on another device");
    if ((epilogue & ~8u) > 3u) return set_error(CM_EINVAL, "cm_conv_prepared: epilogue %u (0..3, plus 8 for channels-last y)", epilogue);
    const unsigned* g = w->g;
    // the planes serve only the path they were built for (the direct-path limit may have
    // changed since); otherwise this call prepares its own from weight and bias
    ImplicitPlan ip;
    const ConvPath path = (g[0] == 0 || g[4] == 0 || (uint64_t)g[5] * g[6] == 0)
                              ? CP_BIAS_FILL
                              : conv_path(cx->direct_max_macs, g[0], g[1], g[4], g[5], g[6], g[7], g[8], g[9], g[10], g[11],
                                          g[12], g[16], &ip);
    const cm_conv_weights* pw = (w->planes && (int)path == w->path) ? w : nullptr;
    return conv_impl(x, xp, w->weight, w->bias, y, yp, g[0], g[1], g[2], g[3], g[4], g[5], g[6], g[7], g[8], g[9], g[10],
                     g[11], g[12], g[13], g[14], g[15], g[16], epilogue, resid, resid_planes, stream, pw);
}

extern "C" int cm_conv_prepared(const cm_conv_weights_t* w, const int16_t* x, const cm_planes_t* xp, int16_t* y,
                                cm_planes_t* yp, unsigned epilogue, const int16_t* resid, const cm_planes_t* resid_planes) {
    int rc = cm_conv_prepared_async(w, x, xp, y, yp, epilogue, resid, resid_planes, nullptr);
    return rc ? rc : finish_sync(nullptr);
}
