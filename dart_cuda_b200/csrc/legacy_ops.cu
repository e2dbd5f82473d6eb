// The rest of the reference's handle ABI (native/src/engine.cu), so that its
// Dart and Python loaders — which bind every symbol eagerly
// (lib/core/tensor/cuda_engine.dart:320-420,
//  python/dart_cuda/core/tensor/cuda_engine.py:99-199) — open this library.
// These ops sit outside the AFT training hot path; each is a plain, correct
// kernel with the reference's forward/backward semantics (grads accumulate).
#include <curand_kernel.h>
#include <math.h>

#include <algorithm>
#include <vector>

#include "runtime.h"

namespace dc {
namespace rt {

#define GRID_STRIDE(i, n)                                                        \
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n);      \
         i += (size_t)gridDim.x * blockDim.x)

// ------------------------------------------------------------- elementwise
__global__ void k_sub(const float *a, const float *b, float *o, size_t n)
{
    GRID_STRIDE(i, n) o[i] = a[i] - b[i];
}
__global__ void k_sub_bwd(const float *g, float *ga, float *gb, size_t n)
{
    GRID_STRIDE(i, n)
    {
        ga[i] += g[i];
        gb[i] -= g[i];
    }
}

// reciprocal with the reference's |b| >= 1e-20 floor (elementwise.cuh:200-207)
__device__ __forceinline__ float safe_recip(float b)
{
    const float fl = 1e-20f;
    const float bs = (fabsf(b) < fl) ? copysignf(fl, b == 0.0f ? 1.0f : b) : b;
    return 1.0f / bs;
}
__global__ void k_div(const float *a, const float *b, float *o, size_t n)
{
    GRID_STRIDE(i, n) o[i] = a[i] * safe_recip(b[i]);
}
__global__ void k_div_bwd(const float *a, const float *b, const float *g, float *ga, float *gb,
                          size_t n)
{
    GRID_STRIDE(i, n)
    {
        const float ib = safe_recip(b[i]);
        ga[i] += g[i] * ib;
        gb[i] -= g[i] * a[i] * ib * ib;
    }
}

// scalar-broadcast ops: b is one element (engine.cu:196-316)
enum ScalarOp { S_ADD = 0, S_SUB = 1, S_MUL = 2, S_DIV = 3 };
__global__ void k_scalar(int op, const float *a, const float *b, float *o, size_t n)
{
    const float s = b[0];
    GRID_STRIDE(i, n)
    {
        const float x = a[i];
        o[i] = op == S_ADD ? x + s : op == S_SUB ? x - s : op == S_MUL ? x * s : x / s;
    }
}
__global__ void k_scalar_bwd(int op, const float *a, const float *b, const float *g, float *ga,
                             float *gb, size_t n)
{
    __shared__ float red[32];
    float s = b[0];
    if (op == S_DIV && fabsf(s) < 1e-20f) s = copysignf(1e-20f, s == 0.0f ? 1.0f : s);
    float acc = 0.f;
    GRID_STRIDE(i, n)
    {
        const float gi = g[i];
        if (op == S_ADD) {
            ga[i] += gi;
            acc += gi;
        } else if (op == S_SUB) {
            ga[i] += gi;
            acc -= gi;
        } else if (op == S_MUL) {
            ga[i] += s * gi;
            acc += a[i] * gi;
        } else {
            const float ib = 1.0f / s;
            ga[i] += gi * ib;
            acc -= a[i] * gi * ib * ib;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        acc = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (threadIdx.x == 0) atomicAdd(gb, acc);
    }
}

// unary ops (elementwise.cuh:209-426)
enum UnaryOp { U_RELU, U_GELU, U_TANH, U_SIGMOID, U_LOG, U_ABS, U_POW };

__device__ __forceinline__ float intpow(float b, int e)
{
    if (e == 0) return 1.0f;
    const bool neg = e < 0;
    if (neg) e = -e;
    float r = 1.0f;
    while (e > 0) {
        if (e & 1) r *= b;
        b *= b;
        e >>= 1;
    }
    return neg ? (r == 0.0f ? 0.0f : 1.0f / r) : r;
}
__device__ __forceinline__ bool int_exp(float e, int *k)
{
    const int r = __float2int_rn(e);
    if (fabsf(e - (float)r) < 1e-6f) {
        *k = r;
        return true;
    }
    return false;
}

__global__ void k_unary(int op, float p, const float *a, float *o, size_t n)
{
    GRID_STRIDE(i, n)
    {
        const float x = a[i];
        float y;
        switch (op) {
        case U_RELU: y = fmaxf(0.0f, x); break;
        case U_GELU: y = 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))); break;
        case U_TANH: y = tanhf(x); break;
        case U_SIGMOID: y = 1.0f / (1.0f + expf(-x)); break;
        case U_LOG: y = logf(x + 1e-7f); break;
        case U_ABS: y = fabsf(x); break;
        default: {
            int k;
            y = int_exp(p, &k) ? intpow(x, k) : (x > 0.0f ? powf(x, p) : 0.0f);
        }
        }
        o[i] = y;
    }
}
__global__ void k_unary_bwd(int op, float p, const float *a, const float *out, const float *g,
                            float *ga, size_t n)
{
    GRID_STRIDE(i, n)
    {
        const float x = a[i];
        float d;
        switch (op) {
        case U_RELU: d = x > 0 ? 1.0f : 0.0f; break;
        case U_GELU: {
            const float t = tanhf(0.7978845608f * (x + 0.044715f * x * x * x));
            d = 0.5f * (1.0f + t) +
                0.5f * x * (1.0f - t * t) * 0.7978845608f * (1.0f + 3.0f * 0.044715f * x * x);
            break;
        }
        case U_TANH: d = 1.0f - out[i] * out[i]; break;
        case U_SIGMOID: d = out[i] * (1.0f - out[i]); break;
        case U_LOG: d = 1.0f / (x + 1e-7f); break;
        case U_ABS: d = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); break;
        default: {
            int k;
            if (int_exp(p, &k))
                d = (float)k * intpow(x, k - 1);
            else if (x > 0.0f)
                d = p * powf(x, p - 1.0f);
            else
                d = 0.0f;
        }
        }
        ga[i] += d * g[i];
    }
}

// ------------------------------------------------------------------ GEMM
// C[M,N] (+)= sum_k A(m,k) B(k,n) with element strides, 32x32 smem tiles
// (16x16 threads, 2x2 outputs each).  Plain fp32 on CUDA cores, as the
// reference's 32x32 tiled matmul (matmul.cuh:27-131).
__global__ void k_gemm(const float *A, long sam, long sak, const float *B, long sbk, long sbn,
                       float *C, int M, int N, int K, int accumulate)
{
    __shared__ float As[32][33], Bs[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;
    const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int r = ty; r < 32; r += 16)
            for (int c = tx; c < 32; c += 16) {
                const int m = m0 + r, k = k0 + c;
                As[r][c] = (m < M && k < K) ? A[m * sam + k * sak] : 0.f;
                const int kk = k0 + r, n = n0 + c;
                Bs[r][c] = (kk < K && n < N) ? B[kk * sbk + n * sbn] : 0.f;
            }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            const float a0 = As[ty][k], a1 = As[ty + 16][k];
            const float b0 = Bs[k][tx], b1 = Bs[k][tx + 16];
            acc[0][0] += a0 * b0;
            acc[0][1] += a0 * b1;
            acc[1][0] += a1 * b0;
            acc[1][1] += a1 * b1;
        }
        __syncthreads();
    }
    for (int i = 0; i < 2; ++i)
        for (int j = 0; j < 2; ++j) {
            const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m < M && n < N) {
                float *c = C + (size_t)m * N + n;
                *c = accumulate ? *c + acc[i][j] : acc[i][j];
            }
        }
}

static void gemm(const float *A, long sam, long sak, const float *B, long sbk, long sbn, float *C,
                 int M, int N, int K, int accumulate)
{
    if (M <= 0 || N <= 0) return;
    dim3 grid((N + 31) / 32, (M + 31) / 32);
    k_gemm<<<grid, dim3(16, 16), 0, kStream>>>(A, sam, sak, B, sbk, sbn, C, M, N, K, accumulate);
}

// ------------------------------------------------------------ row kernels
// softmax with the reference's +1e-9 on the denominator (engine.cu:1048-1083)
__global__ void k_softmax(const float *x, float *y, int R, int V)
{
    __shared__ float red[32];
    __shared__ float bc;
    const int row = blockIdx.x;
    const float *xr = x + (size_t)row * V;
    float *yr = y + (size_t)row * V;
    float mx = -1e30f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, xr[v]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -1e30f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
        bc = m;
    }
    __syncthreads();
    mx = bc;
    float s = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float e = expf(xr[v] - mx);
        yr[v] = e;
        s += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        bc = 1.0f / (t + 1e-9f);
    }
    __syncthreads();
    const float inv = bc;
    for (int v = threadIdx.x; v < V; v += blockDim.x) yr[v] *= inv;
}

// gx += y * (gy - sum(y*gy))  (transpose.cuh:56-79); also the non-affine
// layer norm rows: one block per row, `mode` selects the formula.
__device__ float block_sum_bcast(float v, float *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    return t;
}

__global__ void k_softmax_bwd(const float *y, const float *gy, float *gx, int V)
{
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *yr = y + (size_t)row * V, *gr = gy + (size_t)row * V;
    float *xr = gx + (size_t)row * V;
    float dot = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) dot += yr[v] * gr[v];
    dot = block_sum_bcast(dot, red);
    for (int v = threadIdx.x; v < V; v += blockDim.x) xr[v] += yr[v] * (gr[v] - dot);
}

// non-affine layer norm (layernorm_embed.cuh:46-138)
__global__ void k_lnorm(const float *x, float *y, const float *g, float *gx, int C, float eps,
                        int backward)
{
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = x + (size_t)row * C;
    float s = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) s += xr[j];
    const float mean = block_sum_bcast(s, red) / (float)C;
    float q = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float d = xr[j] - mean;
        q += d * d;
    }
    const float inv = rsqrtf(block_sum_bcast(q, red) / (float)C + eps);
    if (!backward) {
        for (int j = threadIdx.x; j < C; j += blockDim.x) y[(size_t)row * C + j] = (xr[j] - mean) * inv;
        return;
    }
    const float *gr = g + (size_t)row * C;
    float dy = 0.f, dyy = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float yv = (xr[j] - mean) * inv;
        dy += gr[j];
        dyy += gr[j] * yv;
    }
    dy = block_sum_bcast(dy, red);
    dyy = block_sum_bcast(dyy, red);
    const float invC = 1.0f / (float)C;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float yv = (xr[j] - mean) * inv;
        gx[(size_t)row * C + j] += inv * (gr[j] - dy * invC - yv * dyy * invC);
    }
}

// ----------------------------------------------------- layout / gather ops
__global__ void k_transpose(const float *a, float *o, int R, int C, int accumulate)
{
    __shared__ float tile[32][33];
    const int x = blockIdx.x * 32 + threadIdx.x, y0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += 8)
        if (x < C && y0 + j < R) tile[j][threadIdx.x] = a[(size_t)(y0 + j) * C + x];
    __syncthreads();
    const int ox = blockIdx.y * 32 + threadIdx.x, oy0 = blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += 8)
        if (ox < R && oy0 + j < C) {
            float *p = o + (size_t)(oy0 + j) * R + ox;
            *p = accumulate ? *p + tile[threadIdx.x][j] : tile[threadIdx.x][j];
        }
}

// concat along columns: out[r, k*cols + c] = in_k[r, c]
__global__ void k_concat1(const float *const *ins, float *out, int nt, int rows, int cols,
                          int backward)
{
    const size_t total = (size_t)rows * cols * nt;
    GRID_STRIDE(i, total)
    {
        const int tc = cols * nt;
        const int r = (int)(i / tc), c = (int)(i % tc);
        const int k = c / cols, lc = c % cols;
        float *src = const_cast<float *>(ins[k]) + (size_t)r * cols + lc;
        if (backward)
            *src += out[i];
        else
            out[i] = *src;
    }
}

// concat along rows: offs has nt+1 entries
__global__ void k_concat0(const float *const *ins, const int *offs, float *out, int nt, int cols,
                          int backward)
{
    const size_t total = (size_t)offs[nt] * cols;
    GRID_STRIDE(i, total)
    {
        const int r = (int)(i / cols), c = (int)(i % cols);
        int k = 0;
        while (k + 1 < nt && r >= offs[k + 1]) ++k;
        float *src = const_cast<float *>(ins[k]) + (size_t)(r - offs[k]) * cols + c;
        if (backward)
            *src += out[i];
        else
            out[i] = *src;
    }
}

__global__ void k_embed(const int *idx, const float *wte, const float *wpe, float *out, int T,
                        int D)
{
    const size_t total = (size_t)T * D;
    GRID_STRIDE(i, total)
    {
        const int t = (int)(i / D), d = (int)(i % D);
        out[i] = wte[(size_t)idx[t] * D + d] + wpe[i];
    }
}
__global__ void k_embed_bwd(const int *idx, const float *g, float *gwte, float *gwpe, int T, int D)
{
    const size_t total = (size_t)T * D;
    GRID_STRIDE(i, total)
    {
        const int t = (int)(i / D), d = (int)(i % D);
        atomicAdd(gwte + (size_t)idx[t] * D + d, g[i]);
        gwpe[i] += g[i];
    }
}

__global__ void k_copy_offset(const float *src, float *dst, size_t n, int backward)
{
    GRID_STRIDE(i, n)
    {
        if (backward)
            dst[i] += src[i];
        else
            dst[i] = src[i];
    }
}

__global__ void k_sgd(float *p, const float *g, size_t n, float lr)
{
    GRID_STRIDE(i, n) p[i] = p[i] - lr * g[i] - lr * p[i];
}
__global__ void k_clip(float *g, float lim, size_t n)
{
    GRID_STRIDE(i, n) g[i] = fminf(fmaxf(g[i], -lim), lim);
}

// (loss_optim / conv_misc.cuh:54-67): uniform(-limit, limit) from cuRAND
__global__ void k_xavier(float *p, size_t n, int n_in, int n_out, unsigned long seed)
{
    GRID_STRIDE(i, n)
    {
        curandState st;
        curand_init(seed, i, 0, &st);
        const float lim = sqrtf(6.0f / (float)(n_in + n_out));
        p[i] = (curand_uniform(&st) * 2.0f - 1.0f) * lim;
    }
}

__global__ void k_cost(const float *pb, const float *gb, float *cm, int nq, int ng)
{
    const size_t total = (size_t)nq * ng;
    GRID_STRIDE(i, total)
    {
        const int q = (int)(i / ng), g = (int)(i % ng);
        float s = 0.f;
        for (int k = 0; k < 4; ++k) s += fabsf(pb[q * 4 + k] - gb[g * 4 + k]);
        cm[i] = s;
    }
}

// im2col / col2im (conv_misc.cuh:69-149)
__global__ void k_im2col(const float *im, int C, int H, int W, int kh, int kw, int ph, int pw,
                         int sh, int sw, int Ho, int Wo, float *col)
{
    const size_t total = (size_t)C * Ho * Wo;
    GRID_STRIDE(idx, total)
    {
        const int wo = (int)(idx % Wo), ho = (int)((idx / Wo) % Ho), c = (int)(idx / ((size_t)Ho * Wo));
        const int h0 = ho * sh - ph, w0 = wo * sw - pw;
        for (int i = 0; i < kh; ++i)
            for (int j = 0; j < kw; ++j) {
                const int r = h0 + i, q = w0 + j;
                const size_t row = (size_t)c * kh * kw + i * kw + j;
                col[row * Ho * Wo + (size_t)ho * Wo + wo] =
                    (r >= 0 && r < H && q >= 0 && q < W) ? im[((size_t)c * H + r) * W + q] : 0.f;
            }
    }
}
__global__ void k_col2im(const float *col, int C, int H, int W, int k, int p, int s, int Ho, int Wo,
                         float *im)
{
    const size_t total = (size_t)C * H * W;
    GRID_STRIDE(idx, total)
    {
        const int w = (int)(idx % W) + p, h = (int)((idx / W) % H) + p, c = (int)(idx / ((size_t)H * W));
        float v = 0.f;
        for (int a = 0; a < k; ++a)
            for (int bq = 0; bq < k; ++bq) {
                int ho = h - a, wo = w - bq;
                if (ho % s == 0 && wo % s == 0) {
                    ho /= s;
                    wo /= s;
                    if (ho >= 0 && ho < Ho && wo >= 0 && wo < Wo)
                        v += col[(((size_t)c * k + a) * k + bq) * Ho * Wo + (size_t)ho * Wo + wo];
                }
            }
        im[idx] = v;
    }
}

// ---------------------------------------------------------------- helpers
static void *binary(void *ah, void *bh, int which)
{
    auto A = ref(ah), Bt = ref(bh);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A, Bt};
    const size_t n = out->size;
    Node *o = out, *a = A.get(), *b = Bt.get();
    if (which == 0) {
        if (n) k_sub<<<blocks_for(n), 256, 0, kStream>>>(a->data, b->data, o->data, n);
        out->backward_fn = [o, a, b, n]() {
            if (n) k_sub_bwd<<<blocks_for(n), 256, 0, kStream>>>(o->grad, a->grad, b->grad, n);
        };
    } else {
        if (n) k_div<<<blocks_for(n), 256, 0, kStream>>>(a->data, b->data, o->data, n);
        out->backward_fn = [o, a, b, n]() {
            if (n)
                k_div_bwd<<<blocks_for(n), 256, 0, kStream>>>(a->data, b->data, o->grad, a->grad,
                                                              b->grad, n);
        };
    }
    return out;
}

static void *scalar(void *ah, void *bh, int op)
{
    auto A = ref(ah), Bt = ref(bh);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A, Bt};
    const size_t n = out->size;
    Node *o = out, *a = A.get(), *b = Bt.get();
    if (n) k_scalar<<<blocks_for(n), 256, 0, kStream>>>(op, a->data, b->data, o->data, n);
    out->backward_fn = [o, a, b, n, op]() {
        if (n)
            k_scalar_bwd<<<blocks_for(n), 256, 0, kStream>>>(op, a->data, b->data, o->grad,
                                                             a->grad, b->grad, n);
    };
    return out;
}

static void *unary(void *ah, int op, float p = 0.f)
{
    auto A = ref(ah);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A};
    const size_t n = out->size;
    Node *o = out, *a = A.get();
    if (n) k_unary<<<blocks_for(n), 256, 0, kStream>>>(op, p, a->data, o->data, n);
    out->backward_fn = [o, a, n, op, p]() {
        if (n)
            k_unary_bwd<<<blocks_for(n), 256, 0, kStream>>>(op, p, a->data, o->data, o->grad,
                                                            a->grad, n);
    };
    return out;
}

// device copy of a host pointer table, owned by the op
static std::shared_ptr<DevBuf> upload(const void *host, size_t bytes)
{
    auto buf = std::make_shared<DevBuf>(bytes);
    if (buf->p && bytes) cudaMemcpy(buf->p, host, bytes, cudaMemcpyHostToDevice);
    return buf;
}

}  // namespace rt
}  // namespace dc

using namespace dc;
using namespace dc::rt;

extern "C" {

void *sub_tensors(void *a, void *b) { return binary(a, b, 0); }
void *div_tensors(void *a, void *b) { return binary(a, b, 1); }
void *add_tensor_scalar(void *a, void *b) { return scalar(a, b, S_ADD); }
void *sub_tensor_scalar(void *a, void *b) { return scalar(a, b, S_SUB); }
void *mul_tensor_scalar(void *a, void *b) { return scalar(a, b, S_MUL); }
void *div_tensor_scalar(void *a, void *b) { return scalar(a, b, S_DIV); }
void *relu_tensor(void *a) { return unary(a, U_RELU); }
void *gelu_tensor(void *a) { return unary(a, U_GELU); }
void *tanh_tensor(void *a) { return unary(a, U_TANH); }
void *sigmoid_tensor(void *a) { return unary(a, U_SIGMOID); }
void *log_tensor(void *a) { return unary(a, U_LOG); }
void *abs_tensor(void *a) { return unary(a, U_ABS); }
void *pow_tensor(void *a, float e) { return unary(a, U_POW, e); }

void *matmul_tensors(void *ah, void *bh)
{
    auto A = ref(ah), Bt = ref(bh);
    const int M = A->rows, K = A->cols, N = Bt->cols;
    Node *out = make(M, N);
    out->inputs = {A, Bt};
    Node *o = out, *a = A.get(), *b = Bt.get();
    gemm(a->data, K, 1, b->data, N, 1, o->data, M, N, K, 0);
    out->backward_fn = [o, a, b, M, N, K]() {
        gemm(o->grad, N, 1, b->data, 1, N, a->grad, M, K, N, 1);  // dA += dC B^T
        gemm(a->data, 1, K, o->grad, N, 1, b->grad, K, N, M, 1);  // dB += A^T dC
    };
    return out;
}

void *softmax_forward(void *ah)
{
    auto A = ref(ah);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A};
    Node *o = out, *a = A.get();
    if (o->size) k_softmax<<<a->rows, 256, 0, kStream>>>(a->data, o->data, a->rows, a->cols);
    out->backward_fn = [o, a]() {
        if (o->size) k_softmax_bwd<<<a->rows, 256, 0, kStream>>>(o->data, o->grad, a->grad, a->cols);
    };
    return out;
}

void *transpose_tensor(void *ah)
{
    auto A = ref(ah);
    const int R = A->rows, C = A->cols;
    Node *out = make(C, R);
    out->inputs = {A};
    Node *o = out, *a = A.get();
    if (o->size)
        k_transpose<<<dim3((C + 31) / 32, (R + 31) / 32), dim3(32, 8), 0, kStream>>>(a->data, o->data,
                                                                                      R, C, 0);
    out->backward_fn = [o, a, R, C]() {
        if (o->size)
            k_transpose<<<dim3((R + 31) / 32, (C + 31) / 32), dim3(32, 8), 0, kStream>>>(
                o->grad, a->grad, C, R, 1);
    };
    return out;
}

void *concat_tensors_gpu(void **handles, int num)
{
    std::vector<std::shared_ptr<Node>> ts;
    for (int i = 0; i < num; ++i) ts.push_back(ref(handles[i]));
    const int rows = ts[0]->rows, cols = ts[0]->cols;
    Node *out = make(rows, cols * num);
    out->inputs = ts;
    std::vector<const float *> dptr, gptr;
    for (auto &t : ts) {
        dptr.push_back(t->data);
        gptr.push_back(t->grad);
    }
    auto dtab = upload(dptr.data(), num * sizeof(float *));
    auto gtab = upload(gptr.data(), num * sizeof(float *));
    out->saved = {dtab, gtab};
    Node *o = out;
    if (o->size)
        k_concat1<<<blocks_for(o->size), 256, 0, kStream>>>((const float *const *)dtab->p, o->data,
                                                            num, rows, cols, 0);
    out->backward_fn = [o, gtab, num, rows, cols]() {
        if (o->size)
            k_concat1<<<blocks_for(o->size), 256, 0, kStream>>>((const float *const *)gtab->p,
                                                                o->grad, num, rows, cols, 1);
    };
    return out;
}

void *concat_tensors_axis0_gpu(void **handles, int num)
{
    std::vector<std::shared_ptr<Node>> ts;
    for (int i = 0; i < num; ++i) ts.push_back(ref(handles[i]));
    const int cols = ts[0]->cols;
    std::vector<int> offs(num + 1, 0);
    for (int i = 0; i < num; ++i) offs[i + 1] = offs[i] + ts[i]->rows;
    Node *out = make(offs[num], cols);
    out->inputs = ts;
    std::vector<const float *> dptr, gptr;
    for (auto &t : ts) {
        dptr.push_back(t->data);
        gptr.push_back(t->grad);
    }
    auto dtab = upload(dptr.data(), num * sizeof(float *));
    auto gtab = upload(gptr.data(), num * sizeof(float *));
    auto otab = upload(offs.data(), (num + 1) * sizeof(int));
    out->saved = {dtab, gtab, otab};
    Node *o = out;
    if (o->size)
        k_concat0<<<blocks_for(o->size), 256, 0, kStream>>>((const float *const *)dtab->p,
                                                            (const int *)otab->p, o->data, num,
                                                            cols, 0);
    out->backward_fn = [o, gtab, otab, num, cols]() {
        if (o->size)
            k_concat0<<<blocks_for(o->size), 256, 0, kStream>>>((const float *const *)gtab->p,
                                                                (const int *)otab->p, o->grad, num,
                                                                cols, 1);
    };
    return out;
}

void *embedding_forward(int *h_idx, void *wteh, void *wpeh, int T, int D)
{
    auto WTE = ref(wteh), WPE = ref(wpeh);
    Node *out = make(T, D);
    out->inputs = {WTE, WPE};
    auto idx = upload(h_idx, (size_t)std::max(T, 0) * sizeof(int));
    out->saved = {idx};
    Node *o = out, *te = WTE.get(), *pe = WPE.get();
    if (o->size)
        k_embed<<<blocks_for(o->size), 256, 0, kStream>>>((const int *)idx->p, te->data, pe->data,
                                                          o->data, T, D);
    out->backward_fn = [o, te, pe, idx, T, D]() {
        if (o->size)
            k_embed_bwd<<<blocks_for(o->size), 256, 0, kStream>>>((const int *)idx->p, o->grad,
                                                                  te->grad, pe->grad, T, D);
    };
    return out;
}

void *slice_tensor(void *h, int start, int num)
{
    auto A = ref(h);
    if (start < 0) start = 0;
    if (start + num > A->rows) num = A->rows - start;
    num = std::max(num, 0);
    const int cols = A->cols;
    Node *out = make(num, cols);
    out->inputs = {A};
    Node *o = out, *a = A.get();
    const size_t off = (size_t)start * cols, n = o->size;
    if (n) k_copy_offset<<<blocks_for(n), 256, 0, kStream>>>(a->data + off, o->data, n, 0);
    out->backward_fn = [o, a, off, n]() {
        if (n) k_copy_offset<<<blocks_for(n), 256, 0, kStream>>>(o->grad, a->grad + off, n, 1);
    };
    return out;
}

void *layer_norm_tensor(void *ah, float eps)
{
    auto A = ref(ah);
    Node *out = make(A->rows, A->cols);
    out->inputs = {A};
    Node *o = out, *a = A.get();
    if (o->size) k_lnorm<<<a->rows, 256, 0, kStream>>>(a->data, o->data, nullptr, nullptr, a->cols, eps, 0);
    out->backward_fn = [o, a, eps]() {
        if (o->size)
            k_lnorm<<<a->rows, 256, 0, kStream>>>(a->data, nullptr, o->grad, a->grad, a->cols, eps, 1);
    };
    return out;
}

// SGD as the reference applies it: p -= lr*g + lr*p (loss_optim.cuh:300-340)
void sdg_step(void *ph, void *mh, void *vh, int t, float lr)
{
    (void)mh;
    (void)vh;
    (void)t;
    Node *p = static_cast<Node *>(ph);
    if (p && p->size) k_sgd<<<blocks_for(p->size), 256, 0, kStream>>>(p->data, p->grad, p->size, lr);
}

void clip_gradients(void *h, float limit)
{
    Node *t = static_cast<Node *>(h);
    if (t && t->size) k_clip<<<blocks_for(t->size), 256, 0, kStream>>>(t->grad, limit, t->size);
}

void tensor_xavier_init(void *ph, int n_in, int n_out, int seed)
{
    Node *p = static_cast<Node *>(ph);
    if (p && p->size)
        k_xavier<<<blocks_for(p->size), 256, 0, kStream>>>(p->data, p->size, n_in, n_out,
                                                           (unsigned long)seed);
}

void tensor_zero_init(void *ph)
{
    Node *p = static_cast<Node *>(ph);
    if (p && p->size) cudaMemsetAsync(p->data, 0, p->size * 4, kStream);
}

void compute_cost_matrix(void *pbh, void *gbh, void *cmh)
{
    Node *pb = static_cast<Node *>(pbh), *gb = static_cast<Node *>(gbh), *cm = static_cast<Node *>(cmh);
    const size_t n = (size_t)pb->rows * gb->rows;
    if (n) k_cost<<<blocks_for(n), 256, 0, kStream>>>(pb->data, gb->data, cm->data, pb->rows, gb->rows);
    cudaStreamSynchronize(kStream);
}

void im2col_cuda(void *inh, int C, int H, int W, int kh, int kw, int ph, int pw, int sh, int sw,
                 void *outh)
{
    Node *in = static_cast<Node *>(inh), *out = static_cast<Node *>(outh);
    const int Ho = (H + 2 * ph - kh) / sh + 1, Wo = (W + 2 * pw - kw) / sw + 1;
    const size_t n = (size_t)C * Ho * Wo;
    if (n > 0 && Ho > 0 && Wo > 0)
        k_im2col<<<blocks_for(n), 256, 0, kStream>>>(in->data, C, H, W, kh, kw, ph, pw, sh, sw, Ho,
                                                     Wo, out->data);
    cudaStreamSynchronize(kStream);
}

// takes raw device pointers, as the reference's col2im_cuda does (engine.cu:1280)
void col2im_cuda(float *d_col, int c, int h, int w, int k, int p, int s, float *d_im)
{
    const int Ho = (h + 2 * p - k) / s + 1, Wo = (w + 2 * p - k) / s + 1;
    const size_t n = (size_t)c * h * w;
    if (n == 0) return;
    k_col2im<<<blocks_for(n), 256, 0, kStream>>>(d_col, c, h, w, k, p, s, Ho, Wo, d_im);
    cudaStreamSynchronize(kStream);
}

}  // extern "C"
