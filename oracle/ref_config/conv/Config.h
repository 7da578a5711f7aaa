// Build configuration for compiling the reference ConvKernel as a CPU parity
// checker (kernels/conv/include/Config.h.in).  Types, tile sizes and the 7x7
// filter limit are the reference CMake defaults (kernels/conv/CMakeLists.txt:35-56).
#pragma once
#include <cstdint>
#include "ap_fixed.h"
#define CONV_HAVE_APFIXED
using Data_t    = ap_fixed<16, 8>;
using AccData_t = ap_fixed<32, 16>;
static constexpr unsigned kTileM  = 8;
static constexpr unsigned kTileIC = 16;
static constexpr unsigned kMaxKH  = 7;
static constexpr unsigned kMaxKW  = 7;
static constexpr unsigned kSeed   = 42;
