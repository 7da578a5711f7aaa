// C-ABI entry for the reference MatmulKernel compiled against the oracle's
// fixed-point shim (kernels/matmul/include/MatmulKernel.h:68-79).
#include <cstdint>
#include "MatmulKernel.h"
static_assert(sizeof(Data_t) == 2, "Data_t must be a 16-bit word");
extern "C" void cmref_matmul(const int16_t* a, const int16_t* b, int16_t* c, unsigned n, unsigned k,
                             unsigned m, unsigned batch, unsigned a_batch_stride,
                             unsigned b_batch_stride, unsigned c_batch_stride) {
    MatmulKernel(reinterpret_cast<const Data_t*>(a), reinterpret_cast<const Data_t*>(b),
                 reinterpret_cast<Data_t*>(c), n, k, m, batch, a_batch_stride, b_batch_stride,
                 c_batch_stride);
}
extern "C" unsigned cmref_matmul_max_k(void) { return kMaxK; }
