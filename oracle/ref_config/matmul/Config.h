// Build configuration for compiling the reference MatmulKernel as a CPU
// parity checker (kernels/matmul/include/Config.h.in).  Types and tile sizes
// are the reference CMake defaults (kernels/matmul/CMakeLists.txt:36-57);
// kMaxK is raised from 2048 to 16384 so that the K=4096 sweep shapes fit the
// kernel's static a_buf (the reference has no run-time check of this limit).
#pragma once
#include <cstdint>
#include "ap_fixed.h"
#define MATMUL_HAVE_APFIXED
using Data_t    = ap_fixed<16, 8>;
using AccData_t = ap_fixed<32, 16>;
static constexpr unsigned kTileN = 4;
static constexpr unsigned kTileM = 16;
static constexpr unsigned kTileK = 256;
static constexpr unsigned kMaxK  = 16384;
static constexpr unsigned kSeed  = 42;
