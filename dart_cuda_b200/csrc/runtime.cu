// The reference's handle ABI (native/src/engine.cu) on top of the dc_ entry
// points: engine-owned fp32 tensors with a grad buffer, ops that record a
// backward closure, and backward(root) that runs the tape in reverse
// topological order.
//
// Design: a handle is a pointer to a `Node`.  The registry owns one
// shared_ptr per live handle; every op output holds shared_ptrs to its inputs,
// so destroy_tensor on an input that a live output still needs only drops the
// registry entry (the same ownership rule as engine.cu:19-122).  Device
// buffers come from the stream-ordered pool; all work is issued on the legacy
// default stream, so host copies (which synchronise) observe every prior op.
#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <unordered_set>

#include "runtime.h"

namespace dc {
namespace rt {

Node::Node(int r, int c) : rows(r), cols(c), size((size_t)std::max(r, 0) * std::max(c, 0))
{
    if (size) {
        if (cudaMallocAsync(&data, size * 4, kStream) != cudaSuccess) data = nullptr;
        if (cudaMallocAsync(&grad, size * 4, kStream) != cudaSuccess) grad = nullptr;
        if (grad) cudaMemsetAsync(grad, 0, size * 4, kStream);
    }
}

Node::~Node()
{
    if (data) cudaFreeAsync(data, kStream);
    if (grad) cudaFreeAsync(grad, kStream);
}

static std::unordered_map<Node *, std::shared_ptr<Node>> g_registry;
static std::mutex g_mutex;

std::shared_ptr<Node> ref(void *h)
{
    if (!h) return nullptr;
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_registry.find(static_cast<Node *>(h));
    if (it != g_registry.end()) return it->second;
    // a handle that is no longer registered but still alive as somebody's
    // input: borrow it without ownership
    return std::shared_ptr<Node>(std::shared_ptr<Node>{}, static_cast<Node *>(h));
}

Node *make(int r, int c)
{
    auto n = std::make_shared<Node>(r, c);
    Node *raw = n.get();
    std::lock_guard<std::mutex> lock(g_mutex);
    g_registry[raw] = std::move(n);
    return raw;
}

void report(int status, const char *what)
{
    if (status != DC_OK) fprintf(stderr, "[libmat_mul] %s: %s\n", what, dc_last_error());
}

// -------------------------------------------------------------- elementwise
__global__ void k_add(const float *a, const float *b, float *o, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        o[i] = a[i] + b[i];
}
__global__ void k_add_bwd(const float *g, float *ga, float *gb, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        ga[i] += g[i];
        gb[i] += g[i];
    }
}
__global__ void k_mul(const float *a, const float *b, float *o, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        o[i] = a[i] * b[i];
}
__global__ void k_mul_bwd(const float *a, const float *b, const float *g, float *ga, float *gb,
                          size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        ga[i] += g[i] * b[i];
        gb[i] += g[i] * a[i];
    }
}
__global__ void k_sum(const float *a, size_t n, float scale, float *out)
{
    __shared__ float red[32];
    float s = 0.f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) s += a[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) out[0] = s * scale;
    }
}
__global__ void k_bcast_add(const float *g, float scale, float *ga, size_t n)
{
    const float v = g[0] * scale;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        ga[i] += v;
}
__global__ void k_fill(float *p, float v, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        p[i] = v;
}
__global__ void k_step(float *d, float *g, float lr, size_t n)
{
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        d[i] -= lr * g[i];
        g[i] = 0.f;
    }
}

}  // namespace rt
}  // namespace dc

using namespace dc;
using namespace dc::rt;

extern "C" {

void *create_tensor(int r, int c, float *host)
{
    Node *t = make(r, c);
    if (host && t->size) cudaMemcpy(t->data, host, t->size * 4, cudaMemcpyHostToDevice);
    return t;
}

void destroy_tensor(void *h)
{
    if (!h) return;
    std::shared_ptr<Node> kept;
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        auto it = g_registry.find(static_cast<Node *>(h));
        if (it == g_registry.end()) return;
        kept = std::move(it->second);
        g_registry.erase(it);
    }
}

void get_tensor_data(void *h, float *out)
{
    Node *t = static_cast<Node *>(h);
    if (t && out && t->size) cudaMemcpy(out, t->data, t->size * 4, cudaMemcpyDeviceToHost);
}

void tensor_to_host(void *h, float *out) { get_tensor_data(h, out); }

void get_tensor_grad(void *h, float *out)
{
    Node *t = static_cast<Node *>(h);
    if (t && out && t->size) cudaMemcpy(out, t->grad, t->size * 4, cudaMemcpyDeviceToHost);
}

void set_tensor_data(void *h, float *in)
{
    Node *t = static_cast<Node *>(h);
    if (!t || !in || !t->size) return;
    cudaError_t e = cudaMemcpy(t->data, in, t->size * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) fprintf(stderr, "[libmat_mul] set_tensor_data: %s\n", cudaGetErrorString(e));
}

void zero_grad(void *h)
{
    Node *t = static_cast<Node *>(h);
    if (t && t->size) cudaMemsetAsync(t->grad, 0, t->size * 4, kStream);
}

void tensor_step(void *h, float lr)
{
    Node *t = static_cast<Node *>(h);
    if (t && t->size) k_step<<<blocks_for(t->size), 256, 0, kStream>>>(t->data, t->grad, lr, t->size);
}

void backward(void *h)
{
    Node *root = static_cast<Node *>(h);
    if (!root) return;
    // iterative post-order DFS over the inputs (engine.cu:145-195)
    std::vector<Node *> topo;
    std::unordered_set<Node *> seen;
    std::vector<std::pair<Node *, size_t>> stack;
    seen.insert(root);
    stack.push_back({root, 0});
    while (!stack.empty()) {
        auto &top = stack.back();
        Node *v = top.first;
        if (top.second < v->inputs.size()) {
            Node *c = v->inputs[top.second++].get();
            if (c && seen.insert(c).second) stack.push_back({c, 0});
        } else {
            topo.push_back(v);
            stack.pop_back();
        }
    }
    if (root->size) k_fill<<<blocks_for(root->size), 256, 0, kStream>>>(root->grad, 1.0f, root->size);
    for (auto it = topo.rbegin(); it != topo.rend(); ++it)
        if ((*it)->backward_fn) (*it)->backward_fn();
    cudaStreamSynchronize(kStream);
}

// ----------------------------------------------------------------- AFT ops
void *aft_forward(void *qh, void *kh, void *vh, void *wh, bool masked)
{
    auto Q = ref(qh), K = ref(kh), V = ref(vh), W = ref(wh);
    const int T = Q->rows, D = Q->cols;
    Node *out = make(T, D);
    out->inputs = {Q, K, V, W};
    // the forward keeps r and 1/den so the backward skips its second contraction
    const int flags = (masked ? DC_AFT_CAUSAL : 0) | DC_AFT_SAVE_STATS;
    size_t bytes = 0;
    dc_aft_workspace_size(1, T, T, D, DC_F32, flags, &bytes);
    auto ws = std::make_shared<DevBuf>(bytes);
    out->saved.push_back(ws);
    // WB is read with row stride T = Q->rows (attention.cuh:20)
    report(dc_aft_fwd(Q->data, K->data, V->data, W->data, T, out->data, 1, T, T, D, DC_F32,
                      flags, ws->p, bytes, kStream),
           "aft_forward");
    Node *o = out;
    Node *q = Q.get(), *k = K.get(), *v = V.get(), *w = W.get();
    out->backward_fn = [o, q, k, v, w, T, D, flags, ws, bytes]() {
        report(dc_aft_bwd(q->data, k->data, v->data, w->data, T, o->grad, q->grad, k->grad,
                          v->grad, w->grad, 1, T, T, D, DC_F32,
                          flags | DC_AFT_ACCUMULATE | DC_AFT_WS_VALID, ws->p, bytes, kStream),
               "aft_forward backward");
    };
    return out;
}

void *aft_cross_forward(void *qh, void *kh, void *vh, void *wh)
{
    auto Q = ref(qh), K = ref(kh), V = ref(vh), W = ref(wh);
    const int TDec = Q->rows, TEnc = K->rows, D = Q->cols;
    Node *out = make(TDec, D);
    out->inputs = {Q, K, V, W};
    size_t bytes = 0;
    dc_aft_workspace_size(1, TDec, TEnc, D, DC_F32, DC_AFT_SAVE_STATS, &bytes);
    auto ws = std::make_shared<DevBuf>(bytes);
    out->saved.push_back(ws);
    report(dc_aft_fwd(Q->data, K->data, V->data, W->data, TEnc, out->data, 1, TDec, TEnc, D,
                      DC_F32, DC_AFT_SAVE_STATS, ws->p, bytes, kStream),
           "aft_cross_forward");
    Node *o = out;
    Node *q = Q.get(), *k = K.get(), *v = V.get(), *w = W.get();
    out->backward_fn = [o, q, k, v, w, TDec, TEnc, D, ws, bytes]() {
        report(dc_aft_bwd(q->data, k->data, v->data, w->data, TEnc, o->grad, q->grad, k->grad,
                          v->grad, w->grad, 1, TDec, TEnc, D, DC_F32,
                          DC_AFT_SAVE_STATS | DC_AFT_ACCUMULATE | DC_AFT_WS_VALID, ws->p, bytes,
                          kStream),
               "aft_cross_forward backward");
    };
    return out;
}

// --------------------------------------------------------- row-wise ops
void *layernorm_forward(void *xh, void *gh, void *bh, float eps)
{
    auto X = ref(xh), G = ref(gh), Bt = ref(bh);
    Node *out = make(X->rows, X->cols);
    out->inputs = {X, G, Bt};
    report(dc_layernorm_fwd(X->data, G->data, Bt->data, out->data, X->rows, X->cols, eps, kStream),
           "layernorm_forward");
    Node *o = out, *x = X.get(), *g = G.get(), *b = Bt.get();
    out->backward_fn = [o, x, g, b, eps]() {
        report(dc_layernorm_bwd(x->data, g->data, o->grad, x->grad, g->grad, b->grad, x->rows,
                                x->cols, eps, 1, kStream),
               "layernorm backward");
    };
    return out;
}

void *add_tensor_row_broadcast(void *ah, void *bh)
{
    auto A = ref(ah), Bt = ref(bh);
    const int M = A->rows, N = A->cols;
    Node *out = make(M, N);
    out->inputs = {A, Bt};
    report(dc_bias_fwd(A->data, Bt->data, out->data, M, N, kStream), "add_tensor_row_broadcast");
    Node *o = out, *a = A.get(), *b = Bt.get();
    out->backward_fn = [o, a, b, M, N]() {
        report(dc_bias_bwd(o->grad, a->grad, b->grad, M, N, 1, kStream), "bias backward");
    };
    return out;
}

void *cross_entropy_loss(void *lh, int32_t *host_targets, int32_t T, int32_t V)
{
    auto L = ref(lh);
    Node *out = make(1, 1);
    out->inputs = {L};
    auto tg = std::make_shared<DevBuf>((size_t)std::max(T, 0) * 4);
    out->saved.push_back(tg);
    if (T > 0) cudaMemcpy(tg->p, host_targets, (size_t)T * 4, cudaMemcpyHostToDevice);
    // label smoothing fixed at 0.1 (engine.cu:825)
    report(dc_ce_fwd(L->data, (const int32_t *)tg->p, out->data, nullptr, T, V, 0.1f, kStream),
           "cross_entropy_loss");
    Node *o = out, *l = L.get();
    out->backward_fn = [o, l, tg, T, V]() {
        report(dc_ce_bwd(l->data, (const int32_t *)tg->p, o->grad, l->grad, T, V, 0.1f, kStream),
               "cross_entropy backward");
    };
    return out;
}

void adam_step(void *ph, void *mh, void *vh, int32_t t, float lr, float b1, float b2, float eps)
{
    Node *p = static_cast<Node *>(ph), *m = static_cast<Node *>(mh), *v = static_cast<Node *>(vh);
    // weight decay 0.001 as hard-coded in the reference (loss_optim.cuh:268)
    report(dc_adam_step(p->data, p->grad, m->data, v->data, (int64_t)p->size, t, lr, b1, b2, eps,
                        0.001f, kStream),
           "adam_step");
}

// ---------------------------------------------------- elementwise support
void *add_tensors(void *ah, void *bh)
{
    auto A = ref(ah), Bt = ref(bh);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A, Bt};
    const size_t n = out->size;
    if (n) k_add<<<blocks_for(n), 256, 0, kStream>>>(A->data, Bt->data, out->data, n);
    Node *o = out, *a = A.get(), *b = Bt.get();
    out->backward_fn = [o, a, b, n]() {
        if (n) k_add_bwd<<<blocks_for(n), 256, 0, kStream>>>(o->grad, a->grad, b->grad, n);
    };
    return out;
}

void *mul_tensors(void *ah, void *bh)
{
    auto A = ref(ah), Bt = ref(bh);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A, Bt};
    const size_t n = out->size;
    if (n) k_mul<<<blocks_for(n), 256, 0, kStream>>>(A->data, Bt->data, out->data, n);
    Node *o = out, *a = A.get(), *b = Bt.get();
    out->backward_fn = [o, a, b, n]() {
        if (n) k_mul_bwd<<<blocks_for(n), 256, 0, kStream>>>(a->data, b->data, o->grad, a->grad,
                                                             b->grad, n);
    };
    return out;
}

static void *reduce_op(void *ah, bool mean)
{
    auto A = ref(ah);
    Node *out = make(1, 1);
    out->inputs = {A};
    const size_t n = A->size;
    const float scale = mean ? 1.0f / (float)std::max<size_t>(n, 1) : 1.0f;
    k_sum<<<1, 1024, 0, kStream>>>(A->data, n, scale, out->data);
    Node *o = out, *a = A.get();
    out->backward_fn = [o, a, n, scale]() {
        if (n) k_bcast_add<<<blocks_for(n), 256, 0, kStream>>>(o->grad, scale, a->grad, n);
    };
    return out;
}

void *sum_tensor(void *ah) { return reduce_op(ah, false); }
void *mean_tensor(void *ah) { return reduce_op(ah, true); }

}  // extern "C"
