// Shared pieces of the handle runtime (runtime.cu) used by the op wrappers
// of the reference ABI (runtime.cu, legacy_ops.cu).
#pragma once
#include <functional>
#include <memory>
#include <vector>

#include "dc_internal.h"

namespace dc {
namespace rt {

// All handle-ABI work is issued on the legacy default stream.
constexpr cudaStream_t kStream = 0;

// Stream-ordered device buffer kept alive by an op for its backward.
struct DevBuf {
    void *p = nullptr;
    explicit DevBuf(size_t bytes)
    {
        if (bytes && cudaMallocAsync(&p, bytes, kStream) != cudaSuccess) p = nullptr;
    }
    ~DevBuf()
    {
        if (p) cudaFreeAsync(p, kStream);
    }
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
};

// An engine-owned fp32 tensor: data + grad buffers, its op inputs (kept
// alive for backward) and the closure that propagates its grad.
struct Node {
    float *data = nullptr;
    float *grad = nullptr;
    int rows = 0, cols = 0;
    size_t size = 0;
    std::vector<std::shared_ptr<Node>> inputs;
    std::function<void()> backward_fn;
    std::vector<std::shared_ptr<DevBuf>> saved;

    Node(int r, int c);
    ~Node();
};

std::shared_ptr<Node> ref(void *h);  // owning reference to a live handle
Node *make(int r, int c);            // new registered tensor (grad zeroed)
void report(int status, const char *what);

inline unsigned blocks_for(size_t n)
{
    size_t b = (n + 255) / 256;
    if (b < 1) b = 1;
    if (b > 148 * 16) b = 148 * 16;
    return (unsigned)b;
}

}  // namespace rt
}  // namespace dc
