// cm_conv.cu -- ConvKernel on B200 (reference: kernels/conv/kernel/ConvKernel.cpp).
//
// Standard conv (group = 1) runs as a GEMM on the tcgen05 Q8.8 core
// (cm_gemm.cu): rows = output channels (weights [M][C*kh*kw], already K-major),
// columns = output pixels p = oh*out_w + ow of one image, K = C*kh*kw in the
// weight layout's (c, r, s) order.  The im2col pre-pass gathers each
// column's taps (out-of-range taps read 0, ConvKernel.cpp:184-202), splits
// them into hi/lo planes and forms the column terms; the weight split adds
// bias << 8 to the row terms (ConvKernel.cpp:160-169).  The GEMM epilogue
// writes y[n][m][p], i.e. NCHW directly.  Images are processed in chunks so
// that the im2col scratch stays bounded.
//
// Depthwise conv (is_depthwise = 1, ConvKernel.cpp:251-319) is a per-channel
// kh x kw stencil: CUDA cores, one thread per output pixel, int32 wrap sum.
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
                   y + n0 * (uint64_t)out_ch * P, P, (uint64_t)out_ch * P, nb};
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
