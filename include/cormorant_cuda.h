/*
 * cormorant_cuda.h -- C ABI of libcormorant_cuda.so, the B200 (sm_100a)
 * implementation of Cormorant's four Q8.8 kernels.
 *
 * Every kernel entry keeps the reference kernel's argument list, order and
 * meaning; only the buffer arguments change from "physical DDR address
 * programmed into an AXI-Lite register" to "CUDA device pointer".  Data are
 * raw ap_fixed<16,8> words (int16, value = raw / 256); outputs are bit-exact
 * with the reference C-simulation.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   cm_vectorop  <- VectorOPKernel   kernels/vectorop/include/VectorOP.h:86-95,
 *                   programmed by run_op()       inference-scheduler/src/codegen/_source.py:175-217
 *   cm_matmul    <- MatmulKernel     kernels/matmul/include/MatmulKernel.h:68-79,
 *                   programmed by run_matmul()   _source.py:220-258
 *   cm_matmul_at <- run_matmul_at()  _source.py:261-299 (element offsets added to a/b/c)
 *   cm_conv      <- ConvKernel       kernels/conv/include/ConvKernel.h:79-101,
 *                   programmed by run_conv()     _source.py:302-362
 *   cm_pool      <- PoolingKernel    kernels/pool/include/PoolingKernel.h:63-83,
 *                   programmed by run_pool()     _source.py:365-420
 *   cm_init / cm_release  <- X<Kernel>_Initialize(&inst, name) / X<Kernel>_Release
 *                   (_source.py:602-634: int rc, 0 = OK)
 *   cm_buf_*     <- inference_buf_*  inference-scheduler/src/codegen/_buf_impl.py:25-236
 *                   ("phys" becomes the device address)
 *
 * Conventions
 *   - Every call returns CM_OK (0) or a negative CM_E* code; nothing aborts or
 *     throws across the ABI.  cm_last_error() describes the last failure of
 *     the calling thread.
 *   - The plain entry points are synchronous, like the reference's
 *     Start + while(!IsDone) helpers: they return after the work is complete
 *     and report device-side errors.  The *_async twins enqueue on `stream`
 *     (a cudaStream_t; NULL = legacy default stream) and return at once;
 *     cm_synchronize(stream) waits and reports device-side errors.
 *   - `b` (unary ops) and `bias` (has_bias == 0) may be NULL, as in the reference.
 *   - The caller owns every input/output buffer.  Scratch for the tensor-core
 *     kernels comes from the device's stream-ordered memory pool on the call's
 *     stream, so concurrent calls on different streams do not share scratch.
 */
#ifndef CORMORANT_CUDA_H
#define CORMORANT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define CM_OK            0
#define CM_EINVAL       (-1)  /* bad argument (null pointer, size overflow, ...) */
#define CM_EUNSUPPORTED (-2)  /* valid for the reference but not implemented here */
#define CM_ECUDA        (-3)  /* a CUDA runtime/driver call failed */
#define CM_ETIMEOUT     (-4)  /* a device-side bounded wait expired; the kernel returned early */
#define CM_ENOMEM       (-5)  /* device or pinned-host allocation failed */
#define CM_ENOINIT      (-6)  /* cm_init has not succeeded in this process */

/* ---- operation codes (VectorOP.h:50-57, PoolingKernel Config.h.in:35-51) -- */
#define CM_OP_ADD   0u
#define CM_OP_SUB   1u
#define CM_OP_MUL   2u
#define CM_OP_DIV   3u
#define CM_OP_RELU  4u
#define CM_OP_RELU6 5u
#define CM_POOL_MAX 0u
#define CM_POOL_AVG 1u
#define CM_POOL_LP  2u

typedef void* cm_stream_t; /* cudaStream_t */

/* ---- lifecycle ------------------------------------------------------------ */
/* instance: device ordinal as text ("0", "cuda:1"); NULL or "" = device 0.
 * Mirrors X<Kernel>_Initialize(&inst, "<uio name>") (_source.py:602-608). */
int cm_init(const char* instance);
int cm_release(void);
int cm_device(void);                          /* ordinal chosen by cm_init, or CM_ENOINIT */
const char* cm_strerror(int status);
const char* cm_last_error(void);
int cm_synchronize(cm_stream_t stream);       /* wait, then read + clear the device status word */
uint64_t cm_launch_count(void);               /* kernels launched by this library so far */
/* MatMul / standard Conv calls of at most `macs` multiply-accumulates run as one
 * CUDA-core kernel instead of the split + tensor-core pipeline (default 2^22, or
 * the CM_DIRECT_MAX_MACS environment variable at cm_init; 0 = never).  Returns the
 * previous limit.  No reference counterpart; both paths are bit-exact. */
uint64_t cm_set_direct_limit(uint64_t macs);
/* K-split tensor-core GEMMs: a launch whose tiles fill at most half the SMs (CTA pairs)
 * divides each tile's K blocks among 2-4 units that add up exactly (int32 wrap).
 * splits < 0: chosen per launch (default, or the CM_GEMM_SPLIT environment variable at
 * cm_init); 0 or 1: never; k >= 2: k units per tile whenever the tile has at least 2k K
 * blocks and the grid is at most four waves (each unit's int32 slab comes from the
 * stream-ordered scratch pool).  Returns the previous setting.  No reference counterpart;
 * every setting is bit-exact. */
int cm_set_gemm_split(int splits);
const char* cm_version(void);

/* ---- failure-path self test (no reference counterpart) ------------------------
 * Launches one kernel whose bounded mbarrier wait can never be satisfied; after
 * timeout_ms (1..10000) it records CM_ETIMEOUT and returns.  Returns CM_ETIMEOUT
 * (the status word is read and cleared), and the library stays usable. */
int cm_selftest_wait_timeout(unsigned timeout_ms);

/* ---- int8 tensor-pipe ceiling (a measurement; no reference counterpart) --------
 * Runs the MatMul GEMM's MMA stream (tcgen05.mma kind::i8, M = 128 per CTA,
 * N = 256, 32 deep) with its operands resident in shared memory -- no memory
 * traffic -- on every SM: one CTA per SM (pairs = 0) or CTA pairs with
 * cta_group::2 (pairs = 1), `iters` (1..65536) rounds of 8 MMAs each, after one
 * untimed launch.  Returns the int8 ops per second reached (TOPS, 2 ops per
 * multiply-add) and the timed launch's device time in ms: the roofline
 * denominator of the Q8.8 GEMM, measured at the clocks of the moment.  `sm_mhz`
 * (may be NULL) receives the SM clock over the timed stream (clock64 ticks per
 * %globaltimer microsecond in CTA 0), so the ceiling can be scaled to the clock
 * another measurement ran at. */
int cm_int8_mma_rate(unsigned pairs, unsigned iters, double* tops, double* ms, double* sm_mhz);

/* ---- device timing of this library's launches (no reference counterpart) --
 * Between cm_profile_begin and cm_profile_end every kernel launch is bracketed
 * by CUDA events on its own stream.  cm_profile_read waits for those events
 * and returns the summed device time and launch count of one kernel family:
 * "gemm_q88", "split", "vectorop", "pool" or "conv_aux". */
int cm_profile_begin(void);
int cm_profile_end(void);
int cm_profile_read(const char* kernel, double* total_ms, uint64_t* launches);
/* The mean SM clock (MHz) of the tensor-core GEMM launches since cm_profile_begin (each launch
 * times its first CTA with the SM cycle counter and the global nanosecond timer); 0 if none
 * ran.  Synchronizes the device.  A measurement aid with no reference counterpart: the GEMM's
 * roofline divides by the int8 pipe's per-clock ceiling at this clock. */
int cm_profile_gemm_clock(double* sm_mhz);

/* ---- VectorOPKernel ----------------------------------------------------------
 * c[o*(a_inc+b_inc) + i] = op(a[o*a_inc + i], b[o*b_inc + i]),  o < outer, i < size.
 * op: CM_OP_*; any other value copies a (VectorOP.cpp:108). */
int cm_vectorop(const int16_t* a, const int16_t* b, int16_t* c, unsigned size, unsigned op,
                unsigned outer, unsigned a_inc, unsigned b_inc);
int cm_vectorop_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned size, unsigned op,
                      unsigned outer, unsigned a_inc, unsigned b_inc, cm_stream_t stream);

/* ---- MatmulKernel --------------------------------------------------------------
 * c[bi*c_bs + r*m + j] = sat(floor((sum_t a[bi*a_bs + r*k + t] * b[bi*b_bs + t*m + j]) / 256)),
 * accumulated in int32 modulo 2^32; a stride of 0 broadcasts that operand. */
int cm_matmul(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
              unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
              unsigned c_batch_stride);
int cm_matmul_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k,
                    unsigned m, unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                    unsigned c_batch_stride, cm_stream_t stream);
/* Allocation-free MatMul (no counterpart in the reference).  Same arguments and
 * result as cm_matmul, enqueued on `stream` (wait with cm_synchronize).  For
 * callers that cannot call cudaMalloc once running -- e.g. a run loop that,
 * like the reference's generated inference_run(), must not allocate after
 * initialisation, or code whose device memory is owned by another allocator.
 * It never allocates: its scratch is a fixed device array inside this library
 * of CM_MATMUL_NOALLOC_SCRATCH_BYTES, held on every GPU that loads the library
 * until the process exits.  Calls whose scratch need exceeds it return
 * CM_EINVAL; the need is, in bytes (each term rounded up to 256):
 *   A_b*2*n*K16 + B_b*2*k*M16 + A_b*n*4 + B_b*m*4,
 *   K16, M16 = k, m rounded up to 16, A_b = (a_batch_stride ? batch : 1), B_b likewise.
 * Calls of at most cm_set_direct_limit multiply-accumulates run on the one-kernel
 * CUDA-core path, as cm_matmul does, and use no scratch.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture.  All calls share the one array: calls that can overlap on the GPU
 * (different streams without ordering between them) race and must not be issued. */
#define CM_MATMUL_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)
int cm_matmul_noalloc(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k,
                      unsigned m, unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                      unsigned c_batch_stride, cm_stream_t stream);

/* ---- MatMul with a fused bias / ReLU epilogue (no reference counterpart) -----------
 * The same product as cm_matmul, then on every narrowed output word v of row r, column j:
 *   epilogue bit 1: v = sat16(v + bias[j])   (VectorOP ADD, size m, outer n, a_inc m, b_inc 0:
 *                                             the bias row broadcast over the rows)
 *   epilogue bit 0: v = max(v, 0)            (VectorOP RELU)
 * 0 = plain cm_matmul, 1 = MatMul+Relu, 2 = MatMul+Add, 3 = MatMul+Add+Relu: the scheduler's
 * Gemm decomposition (MatMul then the broadcast bias Add, graph.py:83-188) and a following
 * Relu, word for word, in one launch.  The same bias row serves every batch step. */
int cm_matmul_fused(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k, unsigned m,
                    unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                    unsigned c_batch_stride, unsigned epilogue, const int16_t* bias);
int cm_matmul_fused_async(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k,
                          unsigned m, unsigned batch, unsigned a_batch_stride, unsigned b_batch_stride,
                          unsigned c_batch_stride, unsigned epilogue, const int16_t* bias,
                          cm_stream_t stream);

/* run_matmul_at(): the same call with element offsets applied to each buffer. */
int cm_matmul_at(const int16_t* a, unsigned a_off, const int16_t* b, unsigned b_off, int16_t* c,
                 unsigned c_off, unsigned n, unsigned k, unsigned m, unsigned batch,
                 unsigned a_batch_stride, unsigned b_batch_stride, unsigned c_batch_stride);

/* ---- ConvKernel ----------------------------------------------------------------
 * NCHW conv; weights [out_ch][in_ch][kh][kw] (depthwise: [out_ch][1][kh][kw],
 * input channel = output channel); out-of-range input taps read 0; bias[m]
 * initialises the accumulator as bias << 8. */
int cm_conv(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
            unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
            unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
            unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
            unsigned pad_left, unsigned has_bias, unsigned is_depthwise);
int cm_conv_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
                  unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                  unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                  unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                  unsigned pad_left, unsigned has_bias, unsigned is_depthwise,
                  cm_stream_t stream);

/* ---- Conv with a fused elementwise epilogue (no reference counterpart) -------
 * The same convolution as cm_conv, then on every narrowed output word v:
 *   epilogue bit 1: v = sat16(v + resid[i])   (VectorOP ADD, resid laid out like y)
 *   epilogue bit 0: v = max(v, 0)             (VectorOP RELU)
 * 0 = plain cm_conv, 1 = Conv+Relu, 2 = Conv+Add, 3 = Conv+Add+Relu -- the result equals
 * the reference's ConvKernel followed by those VectorOP calls, word for word, without
 * writing and re-reading the intermediate tensors. */
int cm_conv_fused(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
                  unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                  unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                  unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                  unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned epilogue,
                  const int16_t* resid);
int cm_conv_fused_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y,
                        unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                        unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                        unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                        unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned epilogue,
                        const int16_t* resid, cm_stream_t stream);
/* ConvKernel (+ cm_conv_fused's epilogue) followed by a MAX PoolingKernel of its output, in one
 * CUDA-core launch; the conv's 17 scalars and epilogue / resid as cm_conv_fused, then the pool's
 * 17 scalars as cm_pool (its batch, channels, in_h, in_w must be the conv's batch, out_ch, out_h,
 * out_w). y is the pool's output; the conv output is never written. The words of cm_conv_fused
 * followed by cm_pool. No reference counterpart: for launch-bound networks (LeNet-5 batch 1),
 * where a Conv -> Relu -> MaxPool chain whose intermediate has no other reader becomes one
 * launch. MAX pools and standard (not depthwise) convs only, else CM_EUNSUPPORTED. */
int cm_conv_pool(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                 unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w,
                 unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                 unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias, unsigned is_depthwise,
                 unsigned epilogue, const int16_t* resid, unsigned p_batch, unsigned p_channels, unsigned p_in_h,
                 unsigned p_in_w, unsigned p_out_h, unsigned p_out_w, unsigned pool_h, unsigned pool_w,
                 unsigned p_stride_h, unsigned p_stride_w, unsigned p_pad_top, unsigned p_pad_left,
                 unsigned p_dil_h, unsigned p_dil_w, unsigned pool_type, unsigned lp_order,
                 unsigned count_include_pad);
int cm_conv_pool_async(const int16_t* x, const int16_t* weight, const int16_t* bias, int16_t* y, unsigned batch,
                       unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w,
                       unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                       unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
                       unsigned is_depthwise, unsigned epilogue, const int16_t* resid, unsigned p_batch,
                       unsigned p_channels, unsigned p_in_h, unsigned p_in_w, unsigned p_out_h, unsigned p_out_w,
                       unsigned pool_h, unsigned pool_w, unsigned p_stride_h, unsigned p_stride_w,
                       unsigned p_pad_top, unsigned p_pad_left, unsigned p_dil_h, unsigned p_dil_w,
                       unsigned pool_type, unsigned lp_order, unsigned count_include_pad, cm_stream_t stream);

/* ---- Plane images: conv outputs produced as the next conv's operand ----------------
 * (no reference counterpart; results are those of the plain calls, word for word)
 * The tensor-core conv reads its input x [batch][C][H][W] as channels-last int8 hi/lo
 * planes with the spatial padding written out, which a split pass normally builds
 * from x on every call.  A cm_planes_t holds that form of one tensor; a conv whose
 * output feeds such convs can write it directly from its GEMM epilogue, and the
 * consumers read it instead of x:
 *   cm_planes_create     -- a plane image of a [batch][channels][h][w] tensor with the
 *                           given frame (rows / columns of padding on each side);
 *                           needs cm_init; NULL on failure (cm_last_error)
 *   cm_conv_plane_frame  -- 1 if a conv with these arguments reads its input from a
 *                           plane image (its tensor-core implicit-GEMM path, at the
 *                           current cm_set_direct_limit), filling frame[4] = the
 *                           padding {top, left, bottom, right} it needs; else 0
 *   cm_conv_planes       -- cm_conv_fused with plane images: xp (may be NULL) replaces x
 *                           when the conv reads plane images and xp's tensor matches and
 *                           its frame covers the needed padding (otherwise x is read,
 *                           and a NULL x is CM_EINVAL); yp (may be NULL) receives the
 *                           output, y may then be NULL.  A consumer whose padding is
 *                           smaller than the frame reads the image in place.
 *                           resid_planes (may be NULL): a plane image of the residual
 *                           (epilogue bit 1) with the output's shape, read instead of
 *                           resid by convs that read plane images (resid may then be
 *                           NULL; others need resid).  Epilogue bit 3 (value 8): y is
 *                           channels-last, [batch][out_h][out_w][out_ch] (an NCHW resid
 *                           is then read in that layout too); implicit-GEMM convs only,
 *                           others return CM_EUNSUPPORTED. */
typedef struct cm_planes cm_planes_t;
cm_planes_t* cm_planes_create(unsigned batch, unsigned channels, unsigned h, unsigned w, unsigned pad_top,
                              unsigned pad_left, unsigned pad_bottom, unsigned pad_right);
void cm_planes_destroy(cm_planes_t* planes);
/* x [batch][channels][h][w] (NCHW words) -> plane image p: the split pass a conv would run,
 * for a tensor no conv produced (a pool output, the network input) that several convs read. */
int cm_planes_fill(cm_planes_t* p, const int16_t* x);
int cm_planes_fill_async(cm_planes_t* p, const int16_t* x, cm_stream_t stream);
/* PoolingKernel (MAX only) from plane image xp to plane image yp, the same words as
 * cm_pool on the NCHW tensors: a conv -> max pool -> conv chain stays in plane form. */
int cm_pool_planes(const cm_planes_t* xp, cm_planes_t* yp, unsigned batch, unsigned channels, unsigned in_h,
                   unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                   unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                   unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                   unsigned count_include_pad);
int cm_pool_planes_async(const cm_planes_t* xp, cm_planes_t* yp, unsigned batch, unsigned channels,
                         unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h,
                         unsigned pool_w, unsigned stride_h, unsigned stride_w, unsigned pad_top,
                         unsigned pad_left, unsigned dil_h, unsigned dil_w, unsigned pool_type,
                         unsigned lp_order, unsigned count_include_pad, cm_stream_t stream);
/* PoolingKernel (MAX only) from a channels-last tensor x [batch][in_h][in_w][channels]
 * (a conv's y under epilogue bit 3; channels a multiple of 16) to plane image yp: the words
 * of cm_pool on the NCHW tensors, in the form the next convs read.  A conv -> max pool ->
 * conv chain then writes no NCHW tensor and runs no split pass. */
int cm_pool_nhwc_planes(const int16_t* x, cm_planes_t* yp, unsigned batch, unsigned channels, unsigned in_h,
                        unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                        unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left, unsigned dil_h,
                        unsigned dil_w, unsigned pool_type);
int cm_pool_nhwc_planes_async(const int16_t* x, cm_planes_t* yp, unsigned batch, unsigned channels,
                              unsigned in_h, unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h,
                              unsigned pool_w, unsigned stride_h, unsigned stride_w, unsigned pad_top,
                              unsigned pad_left, unsigned dil_h, unsigned dil_w, unsigned pool_type,
                              cm_stream_t stream);
int cm_conv_plane_frame(unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                        unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                        unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                        unsigned pad_left, unsigned has_bias, unsigned is_depthwise, unsigned* frame);
/* 1 if a conv with these arguments (at the current cm_set_direct_limit) runs on an
 * implicit-GEMM path and can write a channels-last y (epilogue bit 3), else 0. */
int cm_conv_writes_nhwc(unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w, unsigned out_ch,
                        unsigned out_h, unsigned out_w, unsigned kh, unsigned kw, unsigned stride_h,
                        unsigned stride_w, unsigned dilation_h, unsigned dilation_w, unsigned pad_top,
                        unsigned pad_left, unsigned has_bias, unsigned is_depthwise);
int cm_conv_planes(const int16_t* x, const cm_planes_t* xp, const int16_t* weight, const int16_t* bias,
                   int16_t* y, cm_planes_t* yp, unsigned batch, unsigned in_ch, unsigned in_h, unsigned in_w,
                   unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh, unsigned kw,
                   unsigned stride_h, unsigned stride_w, unsigned dilation_h, unsigned dilation_w,
                   unsigned pad_top, unsigned pad_left, unsigned has_bias, unsigned is_depthwise,
                   unsigned epilogue, const int16_t* resid, const cm_planes_t* resid_planes);
int cm_conv_planes_async(const int16_t* x, const cm_planes_t* xp, const int16_t* weight, const int16_t* bias,
                         int16_t* y, cm_planes_t* yp, unsigned batch, unsigned in_ch, unsigned in_h,
                         unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w, unsigned kh,
                         unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                         unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
                         unsigned is_depthwise, unsigned epilogue, const int16_t* resid,
                         const cm_planes_t* resid_planes, cm_stream_t stream);

/* ---- Prepared conv weights (no reference counterpart) ---------------------------------
 * A network's conv weights do not change between runs, but every conv call turns them into
 * the GEMM's weight planes and column terms again (one to three small launches per call).
 * cm_conv_weights_create does that once for one call's geometry (the scalars of cm_conv_planes
 * from batch to is_depthwise, the same meaning) and keeps the result on the device;
 * cm_conv_prepared[_async] then runs that conv (cm_conv_planes' x, xp, y, yp, epilogue, resid,
 * resid_planes) without the preparation.  Results are cm_conv_planes' words as long as weight
 * and bias still hold the values they held at creation: the prepared planes are a snapshot,
 * while convs small enough for the CUDA-core paths (and depthwise convs) read weight and bias
 * at each call, so both buffers must stay allocated.  Creation runs on the default stream and
 * waits for it (not inside a stream capture); *out is null unless it returns CM_OK.
 * Destroy frees the planes (null is accepted). */
typedef struct cm_conv_weights cm_conv_weights_t;
int cm_conv_weights_create(const int16_t* weight, const int16_t* bias, unsigned batch, unsigned in_ch,
                           unsigned in_h, unsigned in_w, unsigned out_ch, unsigned out_h, unsigned out_w,
                           unsigned kh, unsigned kw, unsigned stride_h, unsigned stride_w, unsigned dilation_h,
                           unsigned dilation_w, unsigned pad_top, unsigned pad_left, unsigned has_bias,
                           unsigned is_depthwise, cm_conv_weights_t** out);
void cm_conv_weights_destroy(cm_conv_weights_t* w);
int cm_conv_prepared(const cm_conv_weights_t* w, const int16_t* x, const cm_planes_t* xp, int16_t* y,
                     cm_planes_t* yp, unsigned epilogue, const int16_t* resid, const cm_planes_t* resid_planes);
int cm_conv_prepared_async(const cm_conv_weights_t* w, const int16_t* x, const cm_planes_t* xp, int16_t* y,
                           cm_planes_t* yp, unsigned epilogue, const int16_t* resid,
                           const cm_planes_t* resid_planes, cm_stream_t stream);

/* ---- Prepared MatMul B (no reference counterpart) -------------------------------------
 * A network's Gemm weights (B, k x m, broadcast over the batch) do not change between runs,
 * but every MatMul call splits them into the GEMM's planes and column terms again (one
 * launch; 14 us for ResNet-18's 512 x 1000 classifier).  cm_matmul_weights_create does that
 * once; cm_matmul_prepared[_async] then returns cm_matmul_fused's words for (a, b, c, n, k,
 * m, batch, a_batch_stride, 0, c_batch_stride, epilogue, bias) while b keeps the values it
 * held at creation (the planes are a snapshot; calls that cm_matmul runs on another path --
 * launch-bound sizes, overlapping output steps, the row-strided form -- read b itself, so b
 * must stay allocated).  Creation runs on the default stream and waits for it (not inside a
 * stream capture); *out is null unless it returns CM_OK.  Destroy frees the planes (null is
 * accepted). */
typedef struct cm_matmul_weights cm_matmul_weights_t;
int cm_matmul_weights_create(const int16_t* b, unsigned k, unsigned m, cm_matmul_weights_t** out);
void cm_matmul_weights_destroy(cm_matmul_weights_t* w);
int cm_matmul_prepared(const cm_matmul_weights_t* w, const int16_t* a, int16_t* c, unsigned n, unsigned batch,
                       unsigned a_batch_stride, unsigned c_batch_stride, unsigned epilogue, const int16_t* bias);
int cm_matmul_prepared_async(const cm_matmul_weights_t* w, const int16_t* a, int16_t* c, unsigned n, unsigned batch,
                             unsigned a_batch_stride, unsigned c_batch_stride, unsigned epilogue, const int16_t* bias,
                             cm_stream_t stream);

/* ---- Small call lists in one launch (no reference counterpart) ----------------------
 * A list of small kernel calls -- a batch-1 network, bound by launch latency -- run as ONE
 * CTA that executes them in order, with the results of the entry points named below,
 * word for word.  Supported: CM_CALL_CONV (cm_conv_fused's arguments: args = its 17
 * scalars, epilogue 0..3, in0 x, in1 weight, in2 bias, resid), CM_CALL_MATMUL
 * (cm_matmul_fused: args = its 7 scalars, epilogue 0..3, in0 a, in1 b, in2 bias row),
 * CM_CALL_POOL (cm_pool with pool_type MAX: args = its 17 scalars, in0 x) and
 * CM_CALL_VECTOROP (cm_vectorop except DIV: args = size, op, outer, a_inc, b_inc, in0 a,
 * in1 b); at most 2^20 outputs and 2^22 multiply-accumulates per call, no overlapping
 * output rows.  cm_calls_supported says whether a list qualifies (1) or not (0);
 * cm_calls_async refuses a list that does not with CM_EUNSUPPORTED. */
#define CM_CALL_VECTOROP 0u
#define CM_CALL_MATMUL   1u
#define CM_CALL_CONV     2u
#define CM_CALL_POOL     3u
#define CM_CALLS_MAX     24u
typedef struct cm_call {
    unsigned kind;           /* CM_CALL_* */
    unsigned epilogue;       /* conv / matmul: the fused epilogue bits */
    const int16_t* in0;
    const int16_t* in1;
    const int16_t* in2;
    const int16_t* resid;
    int16_t* out;
    unsigned args[17];       /* the entry point's scalar arguments, in its order */
} cm_call_t;
int cm_calls_supported(const cm_call_t* calls, unsigned count);
int cm_calls(const cm_call_t* calls, unsigned count);
int cm_calls_async(const cm_call_t* calls, unsigned count, cm_stream_t stream);

/* ---- PoolingKernel -------------------------------------------------------------
 * pool_type CM_POOL_MAX / AVG / LP (any value >= 2 is LP); lp_order 1 = sum|x|,
 * any other value = sqrt(sum x^2); count_include_pad selects the AVG divisor. */
int cm_pool(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
            unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
            unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
            unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
            unsigned count_include_pad);
int cm_pool_async(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                  unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                  unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                  unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                  unsigned count_include_pad, cm_stream_t stream);
/* PoolingKernel's global pools (the window covers the whole plane: out 1x1, pool = in
 * size, no padding) on a channels-last tensor x [batch][in_h][in_w][channels] -- a conv's
 * y under epilogue bit 3 -- with cm_pool's arguments and words; y is [batch][channels].
 * No reference counterpart: a conv whose only reader is a global pool (ResNet's last
 * block before GlobalAveragePool) then writes channels-last rows instead of scattered NCHW
 * words.  channels a multiple of 8, x and y 16-byte aligned; other pools and layouts
 * return CM_EUNSUPPORTED. */
int cm_pool_nhwc(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                 unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                 unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                 unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                 unsigned count_include_pad);
int cm_pool_nhwc_async(const int16_t* x, int16_t* y, unsigned batch, unsigned channels, unsigned in_h,
                       unsigned in_w, unsigned out_h, unsigned out_w, unsigned pool_h, unsigned pool_w,
                       unsigned stride_h, unsigned stride_w, unsigned pad_top, unsigned pad_left,
                       unsigned dil_h, unsigned dil_w, unsigned pool_type, unsigned lp_order,
                       unsigned count_include_pad, cm_stream_t stream);

/* ---- outputs written across GPUs (no reference counterpart) -----------------------
 * The batch-sharded multi-GPU drivers (one process per GPU) gather a step's outputs
 * on one GPU by letting every rank's kernels write their shard straight into that
 * GPU's buffers: the root exports a device buffer (cm_ipc_export), every other rank
 * maps it (cm_ipc_open, CUDA IPC; peer access over NVLink / NVSwitch enabled as
 * needed) and passes the mapped address, offset to its shard, as the output of
 * cm_matmul / cm_vectorop / cm_pool.  Those kernels write outputs with ordinary
 * stores only, so each word crosses NVLink once, while it is computed.  The
 * exporter keeps the buffer alive until every importer has called cm_ipc_close.
 * Ordering across processes is the caller's (e.g. a barrier after each rank's
 * cm_synchronize). */
typedef struct cm_ipc_handle {
    unsigned char handle[64];   /* cudaIpcMemHandle_t of the allocation holding the buffer */
    uint64_t      offset;       /* bytes from the allocation's start to the buffer */
    int           device;       /* the exporting process's device ordinal */
    int           reserved;
} cm_ipc_handle_t;
int cm_ipc_export(const void* dev_ptr, cm_ipc_handle_t* handle);
int cm_ipc_open(const cm_ipc_handle_t* handle, void** dev_ptr);
int cm_ipc_close(void* dev_ptr);
/* One device-to-device copy enqueued on `stream` (a copy engine; `dst` or `src` may be
 * a cm_ipc_open mapping of a peer GPU's buffer): pushes a finished output shard to the
 * root while the next kernels run. */
int cm_copy_async(void* dst, const void* src, size_t bytes, cm_stream_t stream);

/* ---- buffers: mirror of inference_buf_* (_buf_impl.py:25-236) ------------------
 * An owner buffer is a device allocation plus a pinned host mirror of the same
 * size; views alias a slice of an owner.  `virt` is the host mirror, `dev` the
 * device address handed to the kernels (the reference's "phys"). */
typedef struct cm_buf {
    void*    virt;
    uint64_t dev;
    unsigned count;      /* elements (int16 words) */
    unsigned refcount;
    unsigned is_owner;
    int      device;
} cm_buf_t;

cm_buf_t* cm_buf_alloc(unsigned n_elem);
void      cm_buf_free(cm_buf_t* buf);
void      cm_buf_retain(cm_buf_t* buf);
void      cm_buf_release(cm_buf_t* buf);
int16_t*  cm_buf_ptr(cm_buf_t* buf);
uint64_t  cm_buf_dev(const cm_buf_t* buf);
unsigned  cm_buf_count(const cm_buf_t* buf);
void      cm_buf_init_view(cm_buf_t* view, cm_buf_t* base, unsigned offset_elems,
                           unsigned count_elems);
int       cm_buf_sync_to_device(cm_buf_t* buf);
int       cm_buf_sync_from_device(cm_buf_t* buf);
/* Stream-ordered twins of the two syncs (no reference counterpart: the reference's
 * syncs are cache maintenance on one shared DDR): one cudaMemcpyAsync between the
 * pinned mirror and the device buffer, enqueued on `stream`, so that a caller can
 * overlap the copies of one call with the kernels of another.  Wait with
 * cm_synchronize(stream) or any later work ordered after it on the GPU. */
int       cm_buf_sync_to_device_async(cm_buf_t* buf, cm_stream_t stream);
int       cm_buf_sync_from_device_async(cm_buf_t* buf, cm_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* CORMORANT_CUDA_H */
