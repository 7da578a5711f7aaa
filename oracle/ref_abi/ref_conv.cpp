// C-ABI entry for the reference ConvKernel compiled against the oracle's
// fixed-point shim (kernels/conv/include/ConvKernel.h:79-101).
#include <cstdint>
#include "ConvKernel.h"
static_assert(sizeof(Data_t) == 2, "Data_t must be a 16-bit word");
extern "C" void cmref_conv(const int16_t* x, const int16_t* w, const int16_t* bias, int16_t* y,
                           unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w,
                           unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh, unsigned kw,
                           unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                           unsigned dilation_w, unsigned pad_top, unsigned pad_left,
                           unsigned has_bias, unsigned is_depthwise) {
    ConvKernel(reinterpret_cast<const Data_t*>(x), reinterpret_cast<const Data_t*>(w),
               reinterpret_cast<const Data_t*>(bias), reinterpret_cast<Data_t*>(y), batch, in_ch,
               in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w,
               pad_top, pad_left, has_bias, is_depthwise);
}
extern "C" unsigned cmref_conv_max_kh(void) { return kMaxKH; }
extern "C" unsigned cmref_conv_max_kw(void) { return kMaxKW; }
