// cm_gemm.cuh -- the Q8.8 tensor-core GEMM shared by MatMul and Conv.
//
// Data layout in HBM (all produced by the split pre-passes in cm_gemm.cu):
//   A planes  [a_batches][2][rows][K_pad] int8   K-major (rows of A, K contiguous)
//   B planes  [b_batches][2][K][C_pad]    int8   N-major (rows of B, N contiguous)
//   plane 0 = hi = x >> 8 (signed), plane 1 = lo' = (x & 255) - 128 (signed)
//   K_pad = K rounded up to 16, C_pad = cols rounded up to 16 (16-byte TMA strides)
//   rowterm   [a_batches][rows] int32, colterm [b_batches][cols] int32
//   out[z*out_bs + row*ldo + col*ldc] = sat16(floor(acc / 256)), with
//   acc = 2^16*HH + 2^8*(HL + LH) + LL + rowterm[row] + colterm[col]  (mod 2^32)
// which equals the exact sum of int16 products (see cm_gemm.cu).
#pragma once

#include "cm_common.cuh"

namespace cm {

// Implicit-GEMM A operand of a convolution (rows = output pixels, K = taps):
// planes [2][nimg][Hp][Wp][Cp] int8, the input in channels-last order with the
// spatial zero padding written out (x = 0 is h = 0, l' = -128), Cp = C rounded up
// to 16.  For fixed kernel row r the taps (s, c) of one output pixel are the
// kw*Cp consecutive bytes starting at its first input pixel, so K is ordered
// (r, s, c) with each r's kw*Cp bytes padded to KR_pad (a multiple of 128) and
// the A tile of K block (r, kb) is one TMA box {128 k, bw pixels (stride sw),
// bh rows (stride sh), bn images} at (kb*128, ow0*sw, oh0*sh + r*dh, n0).
// Tile rows are (image, row, column) in that order with bw*bh*bn = 128,
// all three powers of two.
// Hp and Wp are the extents the boxes may read (rows and columns past them read as
// zero); the pitches give the layout, so a view into a larger plane image (a
// channels-last image with a wider padding frame) is a shifted base pointer with
// the image's own pitches.  Pitches of 0 mean the dense layout of these extents.
struct ConvA {
    const int8_t* planes;
    uint32_t nimg, Cp, Hp, Wp, KR, KR_pad, kh, sh, sw, dh;
    uint32_t out_h, out_w, bw_log, bh_log, bn_log;
    uint64_t row_pitch = 0, img_pitch = 0, plane_pitch = 0;   // bytes
};

// Channels-last plane image written by a conv GEMM's epilogue (the consumer convs'
// A operand, produced without a separate split pass): output pixel (n, oh, ow),
// channel c -> hi byte at planes[((n*Hp + oh + pt)*Wp + ow + pl)*Cp + c], lo' byte
// plane_pitch further, and S[(n*Hp + oh + pt)*Wp + ow + pl] += x - 128 (atomic;
// the producer clears S first).
struct PlaneOut {
    int8_t* planes = nullptr;
    int32_t* S = nullptr;
    uint64_t plane_pitch = 0;
    uint32_t Hp = 0, Wp = 0, Cp = 0, pt = 0, pl = 0;
};

struct GemmPlan {
    const int8_t* a_planes; uint32_t rows; uint32_t a_batches;
    const int8_t* b_planes; uint32_t cols; uint32_t b_batches;
    uint32_t K, K_pad, C_pad;
    const int32_t* rowterm;
    const int32_t* colterm;
    int16_t* out; uint64_t ldo, ldc, out_bs;     // out[z*out_bs + row*ldo + col*ldc]
    uint32_t batch;
    // Conv implicit GEMM (a_planes, rows, a_batches, K_pad and batch unused):
    // output pixel (n, oh, ow), channel col -> out[n*out_bs + (oh*out_w + ow)*ldo + col*ldc]
    // (ldo 0 means 1: NCHW with ldc = out_h*out_w; channels-last: ldo = cols, ldc = 1),
    // rowterm[n*out_h*out_w + oh*out_w + ow]; K = kh*KR_pad.
    const ConvA* conv = nullptr;
    // B planes packed for one 64-column tile: [b_batches][K][128] int8, each K row
    // = [64 hi | 64 lo] (cols <= 64; C_pad unused).
    uint32_t b_packed = 0;
    // packed B already regrouped as weights-as-A rows [128][K] (prepared weights), or null
    const int8_t* wa_rows = nullptr;
    // rows_per_img != 0 (plain mode): row = n*rows_per_img + p is written to
    // out[n*out_bs + p + col*ldc] (conv output pixels of several images, NCHW)
    uint32_t rows_per_img = 0;
    // 1: never divide the tiles' K blocks among units (a K-split launch allocates its slabs;
    // the allocation-free entry may not)
    uint32_t no_split = 0;
    // fused epilogue: bit 1 = add `resid` (same indexing as out, saturating), then
    // bit 0 = ReLU -- VectorOP ADD / RELU applied to the narrowed words
    uint32_t epi = 0;
    const int16_t* resid = nullptr;
    // conv mode: also write the output as a plane image (out may then be null)
    PlaneOut po;
    // conv mode: read the residual from this plane image (same shape as the output)
    PlaneOut rp;
};

constexpr uint32_t kMaxGemmK = 65535;  // per-accumulator sums stay below 2^31 in magnitude

inline uint32_t pad_k(uint32_t K) { return (K + 15u) & ~15u; }
inline uint32_t pad_c(uint32_t C) { return (C + 15u) & ~15u; }

// Launch the tcgen05 GEMM (all arguments device-resident, stream-ordered).
int gemm_launch(const Context* cx, const GemmPlan& g, cudaStream_t s);
int gemm_launch_conv(const Context* cx, const GemmPlan& g, cudaStream_t s);

// Packed weight planes [Kt][64 hi | 64 lo] -> weights-as-A rows [128][Kt] (row 2m + p =
// byte p*64 + m of every K row); Kt a multiple of 128.
int weights_to_rows(const Context* cx, const int8_t* packed, uint32_t Kt, int8_t* rows, cudaStream_t s);

// Split int16 rows into hi/lo planes + row terms:
//   element (bt, r, k) = src[bt*src_bs + r*ld + k], r < rows, k < K, bt < nbt;
//   rowterm[bt*rows + r] = 128*sum_k(x - 128) + 16384*K + (bias ? bias[r] << 8 : 0).
int split_rows(const Context* cx, const int16_t* src, uint64_t src_bs, uint64_t ld, uint32_t rows, uint32_t K,
               uint32_t nbt, int8_t* planes, int32_t* rowterm, const int16_t* bias, cudaStream_t s);

// Split int16 matrix rows of B into N-major hi/lo planes + column terms:
//   element (bt, k, c) = src[bt*src_bs + k*ld + c], c < cols, k < K;
//   planes[((bt*2 + p)*K + k)*C_pad + c]; colterm[bt*cols + c] = 128*sum_k(x - 128).
//   packed = true (cols <= 64): planes[bt*K*128 + k*128 + p*64 + c] instead.
int split_kn(const Context* cx, const int16_t* src, uint64_t src_bs, uint64_t ld, uint32_t cols, uint32_t K,
             uint32_t nbt, int8_t* planes, int32_t* colterm, cudaStream_t s, bool packed = false);

// Convolution geometry (input C x H x W, output out_h x out_w, kernel kh x kw).
struct ConvGeom {
    uint32_t C, H, W, out_h, out_w, kh, kw, sh, sw, dh, dw, pt, pl;
};

// Lanes per output word for the launch-bound CUDA-core kernels (power of two <= 32).
uint32_t direct_lanes(const Context* cx, uint64_t outputs, uint64_t red);

// Zero-fill out[z*out_bs + r*ldo + c] (the K == 0 case: an empty sum narrows to 0).
int fill_zero(const Context* cx, int16_t* out, uint32_t batch, uint32_t rows, uint32_t cols, uint64_t ldo,
              uint64_t out_bs, cudaStream_t s);

}  // namespace cm
