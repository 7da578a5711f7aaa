// cm_common.cuh -- shared internals of libcormorant_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cormorant_cuda.h"

namespace cm {

// ---------------------------------------------------------------------------
// Host side: context, errors, scratch
// ---------------------------------------------------------------------------
struct Context {
    int device = -1;
    int sm_count = 0;
    int* status = nullptr;          // device status word (0 = ok, else a CM_E* code)
    uint64_t timeout_ns = 2000000000ull;  // bounded device-side waits
    // MatMul / standard conv with at most this many MACs run as one CUDA-core
    // kernel (launch-bound sizes: no split pre-passes, no tensor-core pipeline)
    uint64_t direct_max_macs = 1ull << 22;
    // 128-column GEMM tiles run on CTA pairs (tcgen05 cta_group::2); CM_GEMM_PAIRS=0 turns it off
    int gemm_pairs = 1;
    int gemm_wa = 1;          // weights-as-A GEMM for conv outputs of at most 64 channels
    // large MatMul calls split batch chunk j+1 on this stream while chunk j's GEMM runs on
    // the caller's (CM_MATMUL_OVERLAP=0 at cm_init turns it off)
    cudaStream_t aux_stream = nullptr;
    int matmul_overlap = 1;
    // implicit-GEMM convs with packed weights read one input window per K block
    // (CM_CONV_WINDOW=0 at cm_init turns it off)
    int conv_window = 1;
    // K-split GEMM units for grids of few tiles: -1 = chosen per launch, 0 / 1 = never,
    // k >= 2 = k units per tile whenever the K blocks allow (CM_GEMM_SPLIT at cm_init,
    // cm_set_gemm_split)
    int gemm_split = -1;
};
// K-split launches keep at most this many (tile, CTA, epilogue warp) arrival counters
constexpr uint32_t kSplitCounters = 1u << 16;

Context* ctx();                      // nullptr before cm_init
int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
int enter(const Context** out);      // checks init, selects the device
void count_launch(unsigned n = 1);
int finish_sync(cm_stream_t stream); // synchronize + read/clear the status word

// Stream-ordered scratch from the device's default memory pool.
int scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

// Opt-in device timing of the library's own launches: CUDA events recorded on
// the launch stream around each kernel while profiling is on (cm_profile_*).
enum ProfKind { PK_GEMM = 0, PK_SPLIT, PK_VECTOROP, PK_POOL, PK_CONV_AUX, PK_COUNT };
// Device counters {SM cycles, nanoseconds} that GEMM launches add their CTA 0 span to while
// profiling is on (cm_profile_begin .. cm_profile_end); nullptr otherwise.
unsigned long long* prof_gemm_clock();

struct ProfScope {
    int kind; cudaStream_t s; cudaEvent_t a = nullptr;
    ProfScope(int k, cudaStream_t st);
    ~ProfScope();
};

// Programmatic dependent launch.  Every kernel of the library is launched with
// launch_k, which lets the next kernel on the stream be scheduled before this one has
// finished (cudaLaunchAttributeProgrammaticStreamSerialization; CM_PDL=0 at cm_init
// turns it off), and every kernel begins with griddep_wait(), which returns once the
// grids it depends on have completed and their memory is visible -- so no kernel
// touches its operands before its predecessor is done, and what overlaps is the
// launch, the block scheduling and the code before the wait.  Kernels whose CTAs are
// all resident at once (the persistent GEMM) also call griddep_launch_dependents()
// after their wait so that the next kernel is launched while they run; others let the
// trigger fire as their blocks exit, so a dependent's waiting blocks never hold slots
// their later waves need.  (Measured: LeNet-5 b1 27.2 -> 24.6 us per image; an early
// trigger in every grid of at most one block per SM added nothing.)
extern int g_pdl;

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... P, typename... A>
inline void launch_k(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, A&&... args) {
    cudaLaunchConfig_t q{};
    q.gridDim = grid;
    q.blockDim = block;
    q.dynamicSmemBytes = smem;
    q.stream = s;
    cudaLaunchAttribute at{};
    at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at.val.programmaticStreamSerializationAllowed = g_pdl ? 1 : 0;
    q.attrs = &at;
    q.numAttrs = 1;
    (void)cudaLaunchKernelEx(&q, kernel, static_cast<A&&>(args)...);   // errors: cudaGetLastError
}

// Grid size for a grid-stride kernel: a multiple of the SM count.
inline unsigned grid_for(const Context* c, uint64_t work_items, unsigned block, unsigned per_sm) {
    const uint64_t need = (work_items + block - 1) / block;
    const uint64_t cap = (uint64_t)c->sm_count * per_sm;
    return (unsigned)(need < cap ? (need ? need : 1) : cap);
}

// ---------------------------------------------------------------------------
// Device side: Q8.8 narrowing
// ---------------------------------------------------------------------------
__device__ __forceinline__ int16_t sat16(int32_t v) {
    return (int16_t)max(-32768, min(32767, v));
}

// saturate_cast<ap_fixed<16,8>>(ap_fixed<32,16> acc): floor by 8 bits, clamp.
// `acc` is the raw Q16.16 accumulator, already reduced mod 2^32.
__device__ __forceinline__ int16_t narrow_acc(uint32_t acc) {
    return sat16(((int32_t)acc) >> 8);   // arithmetic shift == floor
}

// Unsigned 32-bit division by a run-time invariant divisor with a
// multiply-high and a shift (Granlund & Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994, Fig. 4.1).
struct FastDiv {
    uint32_t d, mul, shift;
    FastDiv() : d(1), mul(0), shift(0) {}
    explicit FastDiv(uint32_t div) : d(div ? div : 1) {
        uint32_t l = 0;
        while (l < 32 && (1ull << l) < d) ++l;
        shift = l;
        mul = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        const uint64_t t = __umulhi(n, mul);
        return (uint32_t)((t + n) >> shift);
    }
};

}  // namespace cm
