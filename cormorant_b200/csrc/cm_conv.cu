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
// Explicit im2col (everything else): rows = output channels (weights
// [M][C*kh*kw], already K-major), columns = output pixels of one image, K in
// the weight layout's (c, r, s) order; the im2col pre-pass gathers each
// column's taps into N-major planes.  Images are processed in chunks so that
// either form's scratch stays bounded.
//
// Depthwise conv (is_depthwise = 1, ConvKernel.cpp:251-319) is a per-channel
// kh x kw stencil: CUDA cores, one thread per output pixel, int32 wrap sum.
#include <algorithm>

#include "cm_gemm.cuh"

namespace cm {
namespace {

struct DwArgs {
    uint32_t C, H, W, M, out_h, out_w, kh, kw, sh, sw, dh, dw, pt, pl, has_bias;
};

__global__ void __launch_bounds__(256) conv_depthwise_kernel(const int16_t* __restrict__ x, const int16_t* __restrict__ w,
                                                             const int16_t* __restrict__ bias, int16_t* __restrict__ y,
                                                             DwArgs a, uint64_t total) {
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

// Empty reduction (in_ch * kh * kw == 0): every output is bias (or 0).
__global__ void conv_bias_fill_kernel(const int16_t* __restrict__ bias, int16_t* __restrict__ y, uint32_t M,
                                      uint64_t ohw, uint64_t total, uint32_t has_bias) {
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
// Block = one padded input row segment of `wchunk` pixels: the segment is read
// channel by channel (coalesced along w) into shared memory, then written
// pixel by pixel (coalesced along c).
__global__ void __launch_bounds__(256) conv_nhwc_split_kernel(const int16_t* __restrict__ x, NhwcGeom g, uint32_t wchunk,
                                                              int8_t* __restrict__ planes, int32_t* __restrict__ S) {
    extern __shared__ int16_t tile[];                       // [wchunk][Cp + 2]
    const uint32_t pitch = g.Cp + 2;
    int32_t* ssum = (int32_t*)(tile + (uint64_t)wchunk * pitch);
    const uint32_t n = blockIdx.z, hp = blockIdx.y, w0 = blockIdx.x * wchunk;
    const uint32_t nw = min(wchunk, g.Wp - w0);
    const int32_t ih = (int32_t)hp - (int32_t)g.pt;
    const bool row_in = ih >= 0 && ih < (int32_t)g.H;
    for (uint32_t t = threadIdx.x; t < nw; t += blockDim.x) ssum[t] = 0;
    const int16_t* xr = x + (uint64_t)n * g.C * g.H * g.W + (row_in ? (uint64_t)ih * g.W : 0);
    for (uint32_t t = threadIdx.x; t < g.Cp * nw; t += blockDim.x) {
        const uint32_t c = t / nw, w = t - c * nw;
        const int32_t iw = (int32_t)(w0 + w) - (int32_t)g.pl;
        int16_t v = 0;
        if (c < g.C && row_in && iw >= 0 && iw < (int32_t)g.W) v = __ldg(xr + (uint64_t)c * g.H * g.W + (uint32_t)iw);
        tile[w * pitch + c] = v;
    }
    __syncthreads();
    const uint32_t cq = g.Cp / 4;
    const uint64_t base = (((uint64_t)n * g.Hp + hp) * g.Wp + w0) * g.Cp;
    const uint64_t plane = (uint64_t)g.nimg * g.Hp * g.Wp * g.Cp;
    for (uint32_t t = threadIdx.x; t < cq * nw; t += blockDim.x) {
        const uint32_t w = t / cq, c4 = (t - w * cq) * 4;
        const int16_t* tp = tile + w * pitch + c4;
        uint32_t hi = 0, lo = 0;
        int32_t sum = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int16_t v = tp[j];
            hi |= (uint32_t)(uint8_t)(v >> 8) << (8 * j);
            lo |= (uint32_t)(((uint32_t)v & 255u) ^ 0x80u) << (8 * j);
            if (c4 + j < g.C) sum += (int32_t)v - 128;
        }
        const uint64_t o = base + (uint64_t)w * g.Cp + c4;
        *(uint32_t*)(planes + o) = hi;
        *(uint32_t*)(planes + plane + o) = lo;
        atomicAdd(&ssum[w], sum);
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < nw; t += blockDim.x)
        S[((uint64_t)n * g.Hp + hp) * g.Wp + w0 + t] = ssum[t];
}

// rowterm of output pixel (n, oh, ow) = 128 * sum over its kh x kw taps of S.
__global__ void __launch_bounds__(256) conv_rowterm_kernel(const int32_t* __restrict__ S, uint32_t Hp, uint32_t Wp,
                                                           uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw,
                                                           uint32_t sh, uint32_t sw, uint32_t dh, uint64_t total,
                                                           int32_t* __restrict__ rowterm) {
    const uint64_t P = (uint64_t)out_h * out_w;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t n = t / P, p = t - n * P;
        const uint32_t oh = (uint32_t)(p / out_w), ow = (uint32_t)(p - (uint64_t)oh * out_w);
        const int32_t* b = S + ((uint64_t)n * Hp + (uint64_t)oh * sh) * Wp + (uint64_t)ow * sw;
        uint32_t sum = 0;
        for (uint32_t r = 0; r < kh; ++r)
            for (uint32_t s = 0; s < kw; ++s) sum += (uint32_t)__ldg(b + (uint64_t)r * dh * Wp + s);
        rowterm[t] = (int32_t)(sum * 128u);
    }
}

// weights [M][C][kh][kw] -> N-major planes [2][Kt][M_pad], row k' = r*KR_pad + s*Cp + c;
// k' outside the real taps holds h = l' = 0 and so adds nothing to any product.
__global__ void __launch_bounds__(256) conv_weight_kn_kernel(const int16_t* __restrict__ w, uint32_t M, uint32_t C,
                                                             uint32_t kh, uint32_t kw, uint32_t Cp, uint32_t KR_pad,
                                                             uint32_t M_pad, uint32_t Kt, int8_t* __restrict__ planes) {
    const uint64_t total = (uint64_t)Kt * M;
    const uint64_t plane = (uint64_t)Kt * M_pad;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t kp = (uint32_t)(t / M), m = (uint32_t)(t - (uint64_t)kp * M);
        const uint32_t r = kp / KR_pad, rem = kp - r * KR_pad;
        const uint32_t s = rem / Cp, c = rem - s * Cp;
        int8_t hi = 0, lo = 0;
        if (s < kw && c < C) {
            const int16_t v = __ldg(w + (((uint64_t)m * C + c) * kh + r) * kw + s);
            hi = (int8_t)(v >> 8);
            lo = (int8_t)((v & 255) - 128);
        }
        planes[(uint64_t)kp * M_pad + m] = hi;
        planes[plane + (uint64_t)kp * M_pad + m] = lo;
    }
}

// colterm[m] = 128 * sum_k (w - 128) + 16384 * K + (bias ? bias[m] << 8 : 0)  (mod 2^32); warp per m.
__global__ void __launch_bounds__(256) conv_colterm_kernel(const int16_t* __restrict__ w, const int16_t* __restrict__ bias,
                                                           uint32_t M, uint32_t K, int32_t* __restrict__ colterm) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warps = (uint64_t)gridDim.x * blockDim.x / 32;
    for (uint64_t m = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; m < M; m += warps) {
        const int16_t* wr = w + m * K;
        int32_t sum = 0;
        for (uint32_t k = lane; k < K; k += 32) sum += (int32_t)__ldg(wr + k) - 128;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
        if (lane == 0) {
            uint32_t term = (uint32_t)sum * 128u + K * 16384u;
            if (bias) term += (uint32_t)((int32_t)bias[m] * 256);
            colterm[m] = (int32_t)term;
        }
    }
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
// (<= 8), and padding every kernel row's kw*Cp bytes up to 128 costs at most
// half again the real reduction length.
bool plan_implicit(uint32_t C, uint32_t out_h, uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t sh, uint32_t sw,
                   uint32_t dh, uint32_t dw, ImplicitPlan* ip) {
    if (dw != 1 || sh == 0 || sw == 0 || sh > 8 || sw > 8 || kh == 0 || kw == 0 || C == 0) return false;
    const uint64_t Cp = (C + 15ull) & ~15ull;
    if (Cp > 8192) return false;
    const uint64_t KR = (uint64_t)kw * Cp, KR_pad = (KR + 127) & ~127ull, Kt = KR_pad * kh;
    const uint64_t Kreal = (uint64_t)C * kh * kw;
    if (2 * Kt > 3 * Kreal || Kt > (1ull << 30)) return false;
    const uint64_t Hp = (uint64_t)(out_h - 1) * sh + (uint64_t)(kh - 1) * dh + 1;
    const uint64_t Wp = (uint64_t)(out_w - 1) * sw + (kw - 1) + 1;
    if (Hp >= (1ull << 31) || Wp >= (1ull << 31)) return false;
    uint32_t bw = std::min<uint32_t>(pow2_ceil(out_w), 128);
    while (bw * sw > 256) bw >>= 1;
    uint32_t bh = std::min<uint32_t>(pow2_ceil(out_h), 128 / bw);
    while (bh * sh > 256) bh >>= 1;
    ip->Cp = (uint32_t)Cp; ip->Hp = (uint32_t)Hp; ip->Wp = (uint32_t)Wp;
    ip->KR = (uint32_t)KR; ip->KR_pad = (uint32_t)KR_pad; ip->Kt = (uint32_t)Kt;
    ip->bw = bw; ip->bh = bh; ip->bn = 128 / (bw * bh);
    return true;
}

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_conv_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                             unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h,
                             unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w,
                             unsigned dilation_h, unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                             unsigned has_bias, unsigned is_depthwise, cm_stream_t stream) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    const uint64_t P = (uint64_t)out_h * out_w;
    if (batch == 0 || out_ch == 0 || P == 0) return CM_OK;
    if (!y || (has_bias && !bias)) return set_error(CM_EINVAL, "cm_conv: null buffer");
    if (P >= (1ull << 31)) return set_error(CM_EUNSUPPORTED, "cm_conv: output plane too large");
    cudaStream_t s = (cudaStream_t)stream;
    const uint64_t total = (uint64_t)batch * out_ch * P;

    if (is_depthwise) {
        if (out_ch > in_ch)
            return set_error(CM_EINVAL, "cm_conv: depthwise needs out_ch <= in_ch (output channel m reads input channel m)");
        if ((uint64_t)kh * kw > 0 && (!x || !weight)) return set_error(CM_EINVAL, "cm_conv: null buffer");
        DwArgs a{in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left,
                 has_bias ? 1u : 0u};
        {
            ProfScope ps_(PK_CONV_AUX, s);
            conv_depthwise_kernel<<<grid_for(cx, total, 256, 8), 256, 0, s>>>(x, weight, bias, y, a, total);
        }
        count_launch();
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv depthwise");
    }

    const uint64_t K64 = (uint64_t)in_ch * kh * kw;
    if (K64 == 0) {
        {
            ProfScope ps_(PK_CONV_AUX, s);
            conv_bias_fill_kernel<<<grid_for(cx, total, 256, 8), 256, 0, s>>>(bias, y, out_ch, P, total, has_bias ? 1u : 0u);
        }
        count_launch();
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv bias fill");
    }
    if (!x || !weight) return set_error(CM_EINVAL, "cm_conv: null buffer");
    if (K64 > kMaxGemmK) return set_error(CM_EUNSUPPORTED, "cm_conv: in_ch*kh*kw = %llu exceeds %u", (unsigned long long)K64, kMaxGemmK);
    const uint32_t K = (uint32_t)K64, K_pad = pad_k(K);

    ImplicitPlan ip;
    if (plan_implicit(in_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, &ip)) {
        // rows = output pixels of a chunk of images, columns = output channels
        const uint32_t M_pad = pad_c(out_ch);
        const uint64_t img_plane = (uint64_t)ip.Hp * ip.Wp * ip.Cp;
        uint64_t chunk = kNhwcBudget / (2 * img_plane);
        if (chunk == 0) chunk = 1;
        if (chunk > batch) chunk = batch;
        if (chunk > (1u << 24)) chunk = 1u << 24;
        const uint64_t w_bytes = ((uint64_t)2 * ip.Kt * M_pad + 255) & ~255ull;
        const uint64_t ct_bytes = ((uint64_t)out_ch * 4 + 255) & ~255ull;
        const uint64_t a_bytes = (2 * chunk * img_plane + ip.KR + 256 + 255) & ~255ull;   // + slack past the last pixel
        const uint64_t s_bytes = (chunk * ip.Hp * ip.Wp * 4 + 255) & ~255ull;
        const uint64_t rt_bytes = (chunk * P * 4 + 255) & ~255ull;
        void* scratch = nullptr;
        rc = scratch_alloc(&scratch, w_bytes + ct_bytes + a_bytes + s_bytes + rt_bytes, s);
        if (rc) return rc;
        int8_t* wpl = (int8_t*)scratch;
        int32_t* ct = (int32_t*)(wpl + w_bytes);
        int8_t* apl = (int8_t*)ct + ct_bytes;
        int32_t* S = (int32_t*)(apl + a_bytes);
        int32_t* rt = (int32_t*)((int8_t*)S + s_bytes);
        {
            ProfScope ps_(PK_SPLIT, s);
            const uint64_t wtot = (uint64_t)ip.Kt * out_ch;
            conv_weight_kn_kernel<<<grid_for(cx, wtot, 256, 8), 256, 0, s>>>(weight, out_ch, in_ch, kh, kw, ip.Cp, ip.KR_pad,
                                                                            M_pad, ip.Kt, wpl);
            conv_colterm_kernel<<<grid_for(cx, (uint64_t)out_ch * 32, 256, 8), 256, 0, s>>>(
                weight, has_bias ? bias : nullptr, out_ch, K, ct);
        }
        count_launch();
        count_launch();
        const uint32_t wchunk = std::min<uint32_t>(ip.Wp, std::max<uint32_t>(1u, 46000u / (2 * (ip.Cp + 2) + 4)));
        const size_t nhwc_smem = (size_t)wchunk * (ip.Cp + 2) * 2 + (size_t)wchunk * 4;
        for (uint64_t n0 = 0; !rc && n0 < batch; n0 += chunk) {
            const uint32_t nb = (uint32_t)((batch - n0) < chunk ? (batch - n0) : chunk);
            const NhwcGeom ng{in_ch, in_h, in_w, ip.Cp, ip.Hp, ip.Wp, pad_top, pad_left, nb};
            const uint64_t tot = (uint64_t)nb * P;
            {
                ProfScope ps_(PK_SPLIT, s);
                for (uint32_t b0 = 0; b0 < nb; b0 += 65535u) {
                    const uint32_t bz = std::min(65535u, nb - b0);
                    NhwcGeom gb = ng;
                    const dim3 grid((ip.Wp + wchunk - 1) / wchunk, ip.Hp, bz);
                    // the plane stride stays that of the whole chunk
                    conv_nhwc_split_kernel<<<grid, 256, nhwc_smem, s>>>(
                        x + (n0 + b0) * (uint64_t)in_ch * in_h * in_w, gb, wchunk, apl + (uint64_t)b0 * img_plane,
                        S + (uint64_t)b0 * ip.Hp * ip.Wp);
                    count_launch();
                }
                conv_rowterm_kernel<<<grid_for(cx, tot, 256, 8), 256, 0, s>>>(S, ip.Hp, ip.Wp, out_h, out_w, kh, kw, stride_h,
                                                                            stride_w, dilation_h, tot, rt);
                count_launch();
            }
            const ConvA ca{apl, nb, ip.Cp, ip.Hp, ip.Wp, ip.KR, ip.KR_pad, kh, stride_h, stride_w, dilation_h,
                           out_h, out_w, log2u(ip.bw), log2u(ip.bh), log2u(ip.bn)};
            GemmPlan p{nullptr, 0, 1, wpl, out_ch, 1, ip.Kt, ip.Kt, M_pad, rt, ct,
                       y + n0 * (uint64_t)out_ch * P, 0, P, (uint64_t)out_ch * P, 1};
            p.conv = &ca;
            rc = gemm_launch(cx, p, s);
        }
        scratch_free(scratch, s);
        if (rc) return rc;
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv");
    }

    const uint64_t per_img = 2 * (uint64_t)K * pad_c((uint32_t)P);
    uint64_t chunk = kIm2colBudget / per_img;
    if (chunk == 0) chunk = 1;
    if (chunk > batch) chunk = batch;
    const uint64_t w_bytes = ((uint64_t)2 * out_ch * K_pad + 255) & ~255ull;
    const uint64_t rt_bytes = ((uint64_t)out_ch * 4 + 255) & ~255ull;
    const uint64_t b_bytes = (chunk * per_img + 255) & ~255ull;
    const uint64_t ct_bytes = (chunk * P * 4 + 255) & ~255ull;
    void* scratch = nullptr;
    rc = scratch_alloc(&scratch, w_bytes + rt_bytes + b_bytes + ct_bytes, s);
    if (rc) return rc;
    int8_t* wp = (int8_t*)scratch;
    int32_t* rt = (int32_t*)(wp + w_bytes);
    int8_t* bp = (int8_t*)rt + rt_bytes;
    int32_t* ct = (int32_t*)(bp + b_bytes);

    rc = split_rows(cx, weight, 0, K, out_ch, K, 1, wp, rt, has_bias ? bias : nullptr, s);
    const ConvGeom geo{in_ch, in_h, in_w, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_left};
    for (uint64_t n0 = 0; !rc && n0 < batch; n0 += chunk) {
        const uint32_t nb = (uint32_t)((batch - n0) < chunk ? (batch - n0) : chunk);
        rc = split_im2col(cx, x + n0 * (uint64_t)in_ch * in_h * in_w, geo, nb, bp, ct, s);
        if (rc) break;
        GemmPlan p{wp, out_ch, 1, bp, (uint32_t)P, nb, K, K_pad, pad_c((uint32_t)P), rt, ct,
                   y + n0 * (uint64_t)out_ch * P, P, 1, (uint64_t)out_ch * P, nb};
        rc = gemm_launch(cx, p, s);
    }
    scratch_free(scratch, s);
    if (rc) return rc;
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CM_OK : cuda_error(e, "cm_conv");
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
