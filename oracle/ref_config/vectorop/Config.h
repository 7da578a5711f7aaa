// Build configuration for compiling the reference VectorOPKernel as a CPU
// parity checker.  Plays the role of the reference's CMake-generated Config.h
// (kernels/vectorop/include/Config.h.in) with Data_t = ap_fixed<16,8>.
#pragma once
#include <cstddef>
#include "ap_fixed.h"
using Data_t = ap_fixed<16, 8>;
constexpr unsigned kDataWidthBits = 16;
constexpr unsigned kSeed = 42;
