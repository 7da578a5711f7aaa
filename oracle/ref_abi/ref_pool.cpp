// C-ABI entry for the reference PoolingKernel compiled against the oracle's
// fixed-point shim (kernels/pool/include/PoolingKernel.h:63-83).
#include <cstdint>
#include "PoolingKernel.h"
static_assert(sizeof(Data_t) == 2, "Data_t must be a 16-bit word");
extern "C" void cmref_pool(const int16_t* x, int16_t* y, unsigned batch, unsigned channels,
                           unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w,
                           unsigned pool_h, unsigned pool_w, unsigned stride_h, unsigned stride_w,
                           unsigned pad_top, unsigned pad_left, unsigned dil_h, unsigned dil_w,
                           unsigned pool_type, unsigned lp_order, unsigned count_include_pad) {
    PoolingKernel(reinterpret_cast<const Data_t*>(x), reinterpret_cast<Data_t*>(y), batch, channels,
                  in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top, pad_left,
                  dil_h, dil_w, pool_type, lp_order, count_include_pad);
}
extern "C" unsigned cmref_pool_max_window(void) { return kMaxPoolH; }
