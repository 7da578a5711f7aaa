// C-ABI entry for the reference VectorOPKernel compiled against the oracle's
// fixed-point shim (kernels/vectorop/include/VectorOP.h:86-95).  Buffers are
// raw int16 Q8.8 words, exactly the in-memory layout of ap_fixed<16,8>.
#include <cstdint>
#include "VectorOP.h"
static_assert(sizeof(Data_t) == 2, "Data_t must be a 16-bit word");
extern "C" void cmref_vectorop(const int16_t* a, const int16_t* b, int16_t* c, unsigned size,
                               unsigned op, unsigned outer, unsigned a_inc, unsigned b_inc) {
    VectorOPKernel(reinterpret_cast<const Data_t*>(a), reinterpret_cast<const Data_t*>(b),
                   reinterpret_cast<Data_t*>(c), size, op, outer, a_inc, b_inc);
}
