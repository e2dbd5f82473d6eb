// Error reporting, device status word, TMA descriptor encoding.
#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "dc_internal.h"

namespace dc {

static thread_local char g_last_error[512] = "";

int fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = '\0'; }

static constexpr int kMaxDevices = 64;
static int *g_status[kMaxDevices] = {nullptr};
static std::atomic<int> g_sms[kMaxDevices];
static std::mutex g_dev_mutex;

int *device_status_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_status[dev]) {
        int *p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
        g_status[dev] = p;
    }
    return g_status[dev];
}

int sm_count()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    int n = g_sms[dev].load(std::memory_order_relaxed);
    if (!n) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        n = n > 0 ? n : 148;
        g_sms[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_tmap(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                CUtensorMapSwizzle swizzle)
{
    EncodeTiledFn fn = get_encode();
    if (!fn) return fail(DC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void *>(base),
                    reinterpret_cast<const cuuint64_t *>(dims),
                    reinterpret_cast<const cuuint64_t *>(strides_bytes),
                    reinterpret_cast<const cuuint32_t *>(box), estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(DC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rank=%d dims=%llu,%llu box=%u,%u",
                    (int)r, rank, (unsigned long long)dims[0],
                    (unsigned long long)(rank > 1 ? dims[1] : 0), box[0], rank > 1 ? box[1] : 0);
    return DC_OK;
}

// ------------------------------------------------------------ kernel timing
struct TimedLaunch {
    const char *name;
    cudaEvent_t a, b;
};
static std::mutex g_prof_mutex;
static bool g_prof_on = false;
static std::vector<TimedLaunch> g_prof;

bool profiling_enabled() { return g_prof_on; }

KernelTimer::KernelTimer(const char *n, cudaStream_t s) : name(n), stream(s)
{
    if (!g_prof_on) return;
    if (cudaEventCreate(&start) != cudaSuccess) {
        start = nullptr;
        return;
    }
    cudaEventRecord(start, stream);
}

KernelTimer::~KernelTimer()
{
    if (!start) return;
    cudaEvent_t end;
    if (cudaEventCreate(&end) != cudaSuccess) {
        cudaEventDestroy(start);
        return;
    }
    cudaEventRecord(end, stream);
    std::lock_guard<std::mutex> lock(g_prof_mutex);
    g_prof.push_back({name, start, end});
}

}  // namespace dc

extern "C" {

// Turn per-launch kernel timing on (1) or off (0); either way the records
// collected so far are dropped.
int dc_profile_enable(int on)
{
    std::lock_guard<std::mutex> lock(dc::g_prof_mutex);
    for (auto &r : dc::g_prof) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    dc::g_prof.clear();
    dc::g_prof_on = on != 0;
    return DC_OK;
}

// Synchronise the recorded events and aggregate them by kernel name.
// Writes up to max_entries rows: names (NUL-separated, each < 64 bytes, in
// names[64*k]), total milliseconds and launch counts.  Returns the number of
// distinct kernels (may exceed max_entries).
int dc_profile_read(char *names, float *total_ms, int *counts, int max_entries)
{
    std::lock_guard<std::mutex> lock(dc::g_prof_mutex);
    std::vector<std::string> keys;
    std::vector<float> ms;
    std::vector<int> cnt;
    for (auto &r : dc::g_prof) {
        cudaEventSynchronize(r.b);
        float t = 0.f;
        cudaEventElapsedTime(&t, r.a, r.b);
        size_t k = 0;
        while (k < keys.size() && keys[k] != r.name) ++k;
        if (k == keys.size()) {
            keys.push_back(r.name);
            ms.push_back(0.f);
            cnt.push_back(0);
        }
        ms[k] += t;
        cnt[k] += 1;
    }
    for (size_t k = 0; k < keys.size() && (int)k < max_entries; ++k) {
        if (names) snprintf(names + 64 * k, 64, "%s", keys[k].c_str());
        if (total_ms) total_ms[k] = ms[k];
        if (counts) counts[k] = cnt[k];
    }
    return (int)keys.size();
}

const char *dc_last_error(void) { return dc::g_last_error; }

const char *dc_version(void) { return "dart_cuda_b200 0.1 (sm_100a)"; }

int dc_device_status(void *stream, int *bits)
{
    int *w = dc::device_status_word();
    if (!w) return dc::fail(DC_ERR_CUDA, "no device status word");
    DC_CUDA_TRY(cudaStreamSynchronize(dc::as_stream(stream)));
    int h = 0;
    DC_CUDA_TRY(cudaMemcpy(&h, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (bits) *bits = h;
    if (h) {
        DC_CUDA_TRY(cudaMemset(w, 0, sizeof(int)));
        return dc::fail(DC_ERR_DEVICE, "device status bits 0x%x (0x1-0x10: a bounded wait gave up; "
                        "0x20: token id out of range; 0x40: decode past capacity; "
                        "0x80: AFT input outside the factorised range)", h);
    }
    return DC_OK;
}

}  // extern "C"
