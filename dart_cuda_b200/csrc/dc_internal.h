// Host-side helpers shared by the translation units of libmat_mul.so.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/dart_cuda_b200.h"

namespace dc {

// Record a message for dc_last_error() and return `code`.
int fail(int code, const char *fmt, ...);
void clear_error();

// Convert and check a CUDA runtime result.
#define DC_CUDA_TRY(expr)                                                             \
    do {                                                                              \
        cudaError_t _e = (expr);                                                      \
        if (_e != cudaSuccess)                                                        \
            return ::dc::fail(DC_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,            \
                              cudaGetErrorString(_e), __FILE__, __LINE__);            \
    } while (0)

#define DC_TRY(...)                  \
    do {                             \
        int _s = (__VA_ARGS__);      \
        if (_s != DC_OK) return _s;  \
    } while (0)

// Per-device status word that kernels OR error bits into (bounded waits).
int *device_status_word();

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point,
// so the library does not link libcuda directly.
int encode_tmap(CUtensorMap *map, CUtensorMapDataType dtype, int rank, const void *base,
                const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Kernel timing (off unless dc_profile_enable(1)): brackets a launch with
// CUDA events on its stream and files the pair under `name`.
struct KernelTimer {
    const char *name;
    cudaStream_t stream;
    cudaEvent_t start = nullptr;
    KernelTimer(const char *n, cudaStream_t s);
    ~KernelTimer();
};
bool profiling_enabled();

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Launch with programmatic stream serialisation (the kernel calls
// grid_dep_wait() before its first dependent memory access) and, when
// cluster > 1, as clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, int cluster, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cluster > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

}  // namespace dc
