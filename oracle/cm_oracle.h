/* cm_oracle.h -- CPU restatement of the four Cormorant kernels on raw Q8.8
 * words.  TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg as the parity checker.  Never linked into
 * or called by libcormorant_cuda.so.
 *
 * Every buffer holds int16 raw words of ap_fixed<16,8> (value = raw / 256).
 * Argument lists and meanings are those of the reference kernels:
 *   VectorOPKernel  kernels/vectorop/include/VectorOP.h:86-95
 *   MatmulKernel    kernels/matmul/include/MatmulKernel.h:68-79
 *   ConvKernel      kernels/conv/include/ConvKernel.h:79-101
 *   PoolingKernel   kernels/pool/include/PoolingKernel.h:63-83
 * Index arithmetic is 64-bit; it equals the reference's 32-bit unsigned
 * arithmetic whenever the latter does not wrap (i.e. for every in-bounds call).
 */
#ifndef CM_ORACLE_H
#define CM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void orc_set_threads(int n);
int orc_get_threads(void);

int16_t orc_vectorop_scalar(uint32_t op, int16_t a, int16_t b);

void orc_vectorop(const int16_t* a, const int16_t* b, int16_t* c, uint32_t size, uint32_t op,
                  uint32_t outer, uint32_t a_inc, uint32_t b_inc);

/* Exhaustive check helper: got[(ia - a_first) * 65536 + (b + 32768)] must equal
 * op(ia, b) for ia in [a_first, a_first + a_count) and every int16 b.
 * Returns the number of mismatches; *first_bad receives the first bad index. */
uint64_t orc_vectorop_check_pairs(uint32_t op, int32_t a_first, uint32_t a_count,
                                  const int16_t* got, int64_t* first_bad);

void orc_matmul(const int16_t* a, const int16_t* b, int16_t* c, uint32_t n, uint32_t k, uint32_t m,
                uint32_t batch, uint32_t a_batch_stride, uint32_t b_batch_stride,
                uint32_t c_batch_stride);

/* Rows (bidx[i], ridx[i]) of the matmul output, written to out[i * m + col]. */
void orc_matmul_rows(const int16_t* a, const int16_t* b, uint32_t n, uint32_t k, uint32_t m,
                     uint32_t a_batch_stride, uint32_t b_batch_stride, const uint32_t* bidx,
                     const uint32_t* ridx, uint32_t count, int16_t* out);

void orc_conv(const int16_t* x, const int16_t* w, const int16_t* bias, int16_t* y, uint32_t batch,
              uint32_t in_ch, uint32_t in_h, uint32_t in_w, uint32_t out_ch, uint32_t out_h,
              uint32_t out_w, uint32_t kh, uint32_t kw, uint32_t stride_h, uint32_t stride_w,
              uint32_t dilation_h, uint32_t dilation_w, uint32_t pad_top, uint32_t pad_left,
              uint32_t has_bias, uint32_t is_depthwise);

/* Output planes (nidx[i], midx[i]) of the conv, written to out[i * out_h * out_w + p]. */
void orc_conv_planes(const int16_t* x, const int16_t* w, const int16_t* bias, uint32_t in_ch,
                     uint32_t in_h, uint32_t in_w, uint32_t out_ch, uint32_t out_h, uint32_t out_w,
                     uint32_t kh, uint32_t kw, uint32_t stride_h, uint32_t stride_w,
                     uint32_t dilation_h, uint32_t dilation_w, uint32_t pad_top,
                     uint32_t pad_left, uint32_t has_bias, uint32_t is_depthwise,
                     const uint32_t* nidx, const uint32_t* midx, uint32_t count, int16_t* out);

void orc_pool(const int16_t* x, int16_t* y, uint32_t batch, uint32_t channels, uint32_t in_h,
              uint32_t in_w, uint32_t out_h, uint32_t out_w, uint32_t pool_h, uint32_t pool_w,
              uint32_t stride_h, uint32_t stride_w, uint32_t pad_top, uint32_t pad_left,
              uint32_t dil_h, uint32_t dil_w, uint32_t pool_type, uint32_t lp_order,
              uint32_t count_include_pad);

#ifdef __cplusplus
}
#endif
#endif
