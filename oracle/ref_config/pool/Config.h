// Build configuration for compiling the reference PoolingKernel as a CPU
// parity checker (kernels/pool/include/Config.h.in).  Types, channel tile and
// sentinels are the reference CMake defaults (kernels/pool/CMakeLists.txt:35-60);
// the window limit is raised from 7x7 to 128x128 so that global pools over
// 112x112 planes fit the kernel's static win_buf.
#pragma once
#include <cstdint>
#include "ap_fixed.h"
#define POOL_HAVE_APFIXED
using Data_t    = ap_fixed<16, 8>;
using AccData_t = ap_fixed<32, 16>;
static constexpr unsigned kTileC    = 8;
static constexpr unsigned kMaxPoolH = 128;
static constexpr unsigned kMaxPoolW = 128;
static constexpr unsigned kPoolMax = 0u;
static constexpr unsigned kPoolAvg = 1u;
static constexpr unsigned kPoolLp  = 2u;
static constexpr float kDataMin = -128.0f;
static constexpr float kAccMin  = -32768.0f;
static constexpr unsigned kSeed = 42;
