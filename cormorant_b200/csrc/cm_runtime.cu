// cm_runtime.cu -- lifecycle, status word, errors, scratch and the
// inference_buf_* mirror of libcormorant_cuda.so.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "cm_common.cuh"

namespace cm {

static Context g_ctx;
static bool g_ready = false;
static std::mutex g_mu;
static std::atomic<uint64_t> g_launches{0};
static thread_local char t_err[512] = "";

Context* ctx() { return g_ready ? &g_ctx : nullptr; }

int g_pdl = 1;   // programmatic dependent launch of the library's kernels (CM_PDL=0 at cm_init: off)

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(e == cudaErrorMemoryAllocation ? CM_ENOMEM : CM_ECUDA, "%s: %s", what,
                     cudaGetErrorString(e));
}

int enter(const Context** out) {
    if (!g_ready) return set_error(CM_ENOINIT, "cm_init has not been called");
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != g_ctx.device) {
        cudaError_t e = cudaSetDevice(g_ctx.device);
        if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    }
    *out = &g_ctx;
    return CM_OK;
}

void count_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int finish_sync(cm_stream_t stream) {
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamSynchronize");
    int st = 0;
    e = cudaMemcpy(&st, g_ctx.status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_error(e, "reading device status");
    if (st != 0) {
        const int zero = 0;
        cudaMemcpy(g_ctx.status, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return set_error(st, "device-side status %d (%s)", st, cm_strerror(st));
    }
    return CM_OK;
}

// ---- profiling --------------------------------------------------------------
static const char* kProfNames[PK_COUNT] = {"gemm_q88", "split", "vectorop", "pool", "conv_aux"};
struct ProfPair { int kind; cudaEvent_t a, b; };
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static std::vector<ProfPair> g_prof_pairs;
static std::vector<cudaEvent_t> g_prof_free;

static cudaEvent_t prof_event() {
    cudaEvent_t e = nullptr;
    if (!g_prof_free.empty()) { e = g_prof_free.back(); g_prof_free.pop_back(); }
    else cudaEventCreate(&e);
    return e;
}

ProfScope::ProfScope(int k, cudaStream_t st) : kind(k), s(st) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on) return;
    a = prof_event();
    cudaEventRecord(a, s);
}

ProfScope::~ProfScope() {
    if (!a) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEvent_t b = prof_event();
    cudaEventRecord(b, s);
    g_prof_pairs.push_back({kind, a, b});
}

// the GEMM clock counters live in the status buffer, after the status word
static unsigned long long* gemm_clock_words() {
    return g_ready ? (unsigned long long*)((char*)g_ctx.status + 64) : nullptr;
}

unsigned long long* prof_gemm_clock() {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    return g_prof_on ? gemm_clock_words() : nullptr;
}

int scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
    *p = nullptr;
    if (bytes == 0) return CM_OK;
    cudaError_t e = cudaMallocAsync(p, bytes, s);
    if (e != cudaSuccess) return cuda_error(e, "cudaMallocAsync (scratch)");
    return CM_OK;
}

void scratch_free(void* p, cudaStream_t s) {
    if (p) cudaFreeAsync(p, s);
}

}  // namespace cm

using namespace cm;

extern "C" {

const char* cm_version(void) { return "cormorant_b200 0.1 (sm_100a)"; }

const char* cm_strerror(int status) {
    switch (status) {
        case CM_OK: return "ok";
        case CM_EINVAL: return "invalid argument";
        case CM_EUNSUPPORTED: return "unsupported";
        case CM_ECUDA: return "CUDA error";
        case CM_ETIMEOUT: return "device-side wait timed out";
        case CM_ENOMEM: return "out of memory";
        case CM_ENOINIT: return "not initialised";
        default: return "unknown status";
    }
}

const char* cm_last_error(void) { return t_err; }

int cm_init(const char* instance) {
    std::lock_guard<std::mutex> lk(g_mu);
    int dev = 0;
    if (instance && *instance) {
        const char* s = instance;
        if (!strncmp(s, "cuda:", 5)) s += 5;
        char* end = nullptr;
        long v = strtol(s, &end, 10);
        if (end == s || *end != '\0' || v < 0) return set_error(CM_EINVAL, "bad instance '%s'", instance);
        dev = (int)v;
    }
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceCount");
    if (dev >= n) return set_error(CM_EINVAL, "device %d not present (%d devices)", dev, n);
    if (g_ready && g_ctx.device == dev) return CM_OK;
    if (g_ready) {
        cudaSetDevice(g_ctx.device);
        cudaFree(g_ctx.status);
        if (g_ctx.aux_stream) cudaStreamDestroy(g_ctx.aux_stream);
        g_ready = false;
    }
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceProperties");
    if (prop.major != 10) return set_error(CM_EUNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", dev, prop.major, prop.minor);
    Context c;
    c.device = dev;
    c.sm_count = prop.multiProcessorCount;
    e = cudaMalloc(&c.status, 256);
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc(status)");
    cudaMemset(c.status, 0, 256);
    // Keep freed scratch cached in the pool instead of returning it to the OS.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t thr = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
    const char* tmo = getenv("CM_TIMEOUT_MS");
    if (tmo && *tmo) c.timeout_ns = (uint64_t)strtoull(tmo, nullptr, 10) * 1000000ull;
    const char* gp = getenv("CM_GEMM_PAIRS");
    if (gp && *gp) c.gemm_pairs = atoi(gp) != 0;
    const char* gw = getenv("CM_GEMM_WA");
    if (gw && *gw) c.gemm_wa = atoi(gw) != 0;
    const char* dm = getenv("CM_DIRECT_MAX_MACS");
    if (dm && *dm) c.direct_max_macs = (uint64_t)strtoull(dm, nullptr, 10);
    const char* mo = getenv("CM_MATMUL_OVERLAP");
    if (mo && *mo) c.matmul_overlap = atoi(mo) != 0;
    const char* cw = getenv("CM_CONV_WINDOW");
    if (cw && *cw) c.conv_window = atoi(cw) != 0;
    const char* gs = getenv("CM_GEMM_SPLIT");
    if (gs && *gs) c.gemm_split = atoi(gs);
    const char* pd = getenv("CM_PDL");
    g_pdl = (pd && *pd) ? (atoi(pd) != 0) : 1;
    e = cudaStreamCreateWithFlags(&c.aux_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        cudaFree(c.status);
        return cuda_error(e, "cudaStreamCreate(aux)");
    }
    g_ctx = c;
    g_ready = true;
    return CM_OK;
}

int cm_release(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ready) return CM_OK;
    cudaSetDevice(g_ctx.device);
    cudaDeviceSynchronize();
    cudaFree(g_ctx.status);
    if (g_ctx.aux_stream) cudaStreamDestroy(g_ctx.aux_stream);
    g_ready = false;
    return CM_OK;
}

int cm_device(void) { return g_ready ? g_ctx.device : CM_ENOINIT; }

uint64_t cm_launch_count(void) { return g_launches.load(); }

int cm_profile_begin(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& pp : g_prof_pairs) { g_prof_free.push_back(pp.a); g_prof_free.push_back(pp.b); }
    g_prof_pairs.clear();
    if (gemm_clock_words()) cudaMemset(gemm_clock_words(), 0, 2 * sizeof(unsigned long long));
    g_prof_on = true;
    return CM_OK;
}

int cm_profile_gemm_clock(double* sm_mhz) {
    if (!sm_mhz) return set_error(CM_EINVAL, "cm_profile_gemm_clock: null result");
    *sm_mhz = 0.0;
    if (!g_ready) return set_error(CM_ENOINIT, "cm_profile_gemm_clock: cm_init has not been called");
    unsigned long long w[2] = {0, 0};
    cudaError_t e = cudaMemcpy(w, gemm_clock_words(), sizeof w, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_error(e, "cm_profile_gemm_clock");
    *sm_mhz = w[1] ? (double)w[0] / (double)w[1] * 1000.0 : 0.0;
    return CM_OK;
}

int cm_profile_end(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_on = false;
    return CM_OK;
}

int cm_profile_read(const char* kernel, double* total_ms, uint64_t* launches) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    int kind = -1;
    for (int i = 0; i < PK_COUNT; ++i)
        if (kernel && !strcmp(kernel, kProfNames[i])) kind = i;
    if (kind < 0) return set_error(CM_EINVAL, "unknown kernel '%s'", kernel ? kernel : "(null)");
    double ms = 0.0;
    uint64_t n = 0;
    for (auto& pp : g_prof_pairs) {
        if (pp.kind != kind) continue;
        cudaError_t e = cudaEventSynchronize(pp.b);
        if (e != cudaSuccess) return cuda_error(e, "cudaEventSynchronize");
        float t = 0.f;
        e = cudaEventElapsedTime(&t, pp.a, pp.b);
        if (e != cudaSuccess) return cuda_error(e, "cudaEventElapsedTime");
        ms += t;
        ++n;
    }
    if (total_ms) *total_ms = ms;
    if (launches) *launches = n;
    return CM_OK;
}

uint64_t cm_set_direct_limit(uint64_t macs) {
    std::lock_guard<std::mutex> lk(g_mu);
    const uint64_t old = g_ctx.direct_max_macs;
    g_ctx.direct_max_macs = macs;
    return old;
}

int cm_set_gemm_split(int splits) {
    std::lock_guard<std::mutex> lk(g_mu);
    const int old = g_ctx.gemm_split;
    g_ctx.gemm_split = splits < 0 ? -1 : splits;
    return old;
}

int cm_synchronize(cm_stream_t stream) {
    const Context* c;
    int rc = enter(&c);
    if (rc) return rc;
    return finish_sync(stream);
}

// ---- inference_buf_* mirror ------------------------------------------------

cm_buf_t* cm_buf_alloc(unsigned n_elem) {
    const Context* c;
    if (enter(&c)) return nullptr;
    cm_buf_t* b = (cm_buf_t*)calloc(1, sizeof(cm_buf_t));
    if (!b) return nullptr;
    const size_t bytes = (size_t)(n_elem ? n_elem : 1) * sizeof(int16_t);
    void* d = nullptr;
    void* h = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) { free(b); set_error(CM_ENOMEM, "cudaMalloc(%zu)", bytes); return nullptr; }
    if (cudaMallocHost(&h, bytes) != cudaSuccess) { cudaFree(d); free(b); set_error(CM_ENOMEM, "cudaMallocHost(%zu)", bytes); return nullptr; }
    memset(h, 0, bytes);
    cudaMemset(d, 0, bytes);
    b->virt = h;
    b->dev = (uint64_t)(uintptr_t)d;
    b->count = n_elem;
    b->refcount = 1;
    b->is_owner = 1;
    b->device = c->device;
    return b;
}

static void buf_dealloc(cm_buf_t* b) {
    cudaSetDevice(b->device);
    cudaFreeHost(b->virt);
    cudaFree((void*)(uintptr_t)b->dev);
    free(b);
}

void cm_buf_retain(cm_buf_t* b) {
    if (b && b->is_owner) b->refcount++;
}

void cm_buf_release(cm_buf_t* b) {
    if (!b || !b->is_owner) return;
    if (--b->refcount == 0u) buf_dealloc(b);
}

void cm_buf_free(cm_buf_t* b) { cm_buf_release(b); }

int16_t* cm_buf_ptr(cm_buf_t* b) { return b ? (int16_t*)b->virt : nullptr; }
uint64_t cm_buf_dev(const cm_buf_t* b) { return b ? b->dev : 0; }
unsigned cm_buf_count(const cm_buf_t* b) { return b ? b->count : 0; }

void cm_buf_init_view(cm_buf_t* view, cm_buf_t* base, unsigned offset_elems, unsigned count_elems) {
    const uint64_t off = (uint64_t)offset_elems * sizeof(int16_t);
    view->virt = (char*)base->virt + off;
    view->dev = base->dev + off;
    view->count = count_elems;
    view->refcount = 0;
    view->is_owner = 0;
    view->device = base->device;
}

int cm_buf_sync_to_device(cm_buf_t* b) {
    if (!b) return set_error(CM_EINVAL, "null buffer");
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpy((void*)(uintptr_t)b->dev, b->virt, (size_t)b->count * 2, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? CM_OK : cuda_error(e, "sync_to_device");
}

int cm_buf_sync_from_device(cm_buf_t* b) {
    if (!b) return set_error(CM_EINVAL, "null buffer");
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpy(b->virt, (void*)(uintptr_t)b->dev, (size_t)b->count * 2, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? CM_OK : cuda_error(e, "sync_from_device");
}

int cm_buf_sync_to_device_async(cm_buf_t* b, cm_stream_t stream) {
    if (!b) return set_error(CM_EINVAL, "null buffer");
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpyAsync((void*)(uintptr_t)b->dev, b->virt, (size_t)b->count * 2, cudaMemcpyHostToDevice,
                                    (cudaStream_t)stream);
    return e == cudaSuccess ? CM_OK : cuda_error(e, "sync_to_device_async");
}

int cm_buf_sync_from_device_async(cm_buf_t* b, cm_stream_t stream) {
    if (!b) return set_error(CM_EINVAL, "null buffer");
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpyAsync(b->virt, (void*)(uintptr_t)b->dev, (size_t)b->count * 2, cudaMemcpyDeviceToHost,
                                    (cudaStream_t)stream);
    return e == cudaSuccess ? CM_OK : cuda_error(e, "sync_from_device_async");
}

}  // extern "C"
