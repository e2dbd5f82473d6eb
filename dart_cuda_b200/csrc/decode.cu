// Incremental AFT-full decode over a per-layer K/V history.
//
// The reference generates by re-running the whole decoder over the context
// for every new token (example/bin/shakespear4.dart:176-214), an O(t^2 d)
// step.  The causal AFT row of the newest position t needs only the history:
//
//   Z[b,t,c] = sigmoid(q[b,c]) * sum_{i<=t} e^{k_i[b,c] + w[t,i]} v_i[b,c]
//                              / sum_{i<=t} e^{k_i[b,c] + w[t,i]}
//
// (native/src/kernels/attention.cuh:6-40, one row t), so a step keeps k and v
// of every earlier position (the cache) and streams them once: O(t d) bytes,
// HBM-bound.  The sum runs as an online softmax (running maximum, rescale)
// in fp32, which is the reference's joint-max stabilisation computed in one
// pass; the position's own k, v come from the fresh projection and are
// appended to the cache by the same launch.
//
// Cache layout per layer: [Tmax][B*D/4][8] fp32 -- for every 4 consecutive
// columns c (b-major, then head, then channel) the 4 k values then the 4 v
// values, so one thread moves one 32-byte sector per history row.
//
// Launch: blocks of 256 threads x 4 columns (a 1024-column slab) times
// chunks of the history rows; each block leaves (max, num, den) per column
// and the last block of a slab to finish (atomic counter after a fence)
// merges the chunks and applies the sigmoid gate.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "dc_internal.h"
#include "dc_ptx.cuh"

namespace dc {
namespace dec {

constexpr int kThreads = 256;
constexpr int kSlab = kThreads * 4;  // columns per block
constexpr int kGroup = 8;            // history rows per online-softmax update
constexpr int kMaxRows = 256;        // history rows per block at most
constexpr int kMaxChunks = 16;       // blocks per slab at most (merged in registers)
constexpr int kMaxHeads = 8;         // heads one slab may touch

struct Params {
    const float *qkv;  // [B, 3*D] rows: q | k | v, heads of hs channels each
    int ldq;
    const float *w;    // posBias of head h: w + h * wh, row t at t * ldw
    int ldw;
    long long wh;
    float *cache;      // [Tmax][B*D/4][8]
    int B, H, hs, D, Tmax;
    const int *pos;    // device: the position t being decoded
    int rows;          // history rows per chunk (multiple of kGroup), set on the device
    int *status;
    int t, chunks;     // set on the device from *pos
    float *Z;
    int ldz;
    float *part;       // [chunks][B*D][3]: max, num, den
    int *counter;      // [slabs], zero between launches
};

__device__ __forceinline__ float sigm(float q) { return 1.0f / (1.0f + __expf(-q)); }

__global__ void __launch_bounds__(kThreads) aft_decode_kernel(Params p)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    // the grid covers Tmax rows; blocks past the history of position t leave
    p.t = *p.pos;
    if (p.t < 0 || p.t >= p.Tmax) {
        if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) atomicOr(p.status, 0x40);
        return;
    }
    // the t+1 history rows split evenly over the grid's chunks, so every
    // block streams about the same number of rows whatever t is
    p.rows = ((p.t + (int)gridDim.y) / (int)gridDim.y + kGroup - 1) / kGroup * kGroup;
    p.chunks = p.t / p.rows + 1;
    if ((int)blockIdx.y >= p.chunks) return;
    const int cols = p.B * p.D;
    const int slab = blockIdx.x, chunk = blockIdx.y;
    const int c0 = slab * kSlab + threadIdx.x * 4;  // first of this thread's 4 columns
    const bool active = c0 < cols;
    const int b = active ? c0 / p.D : 0;
    const int ch = active ? c0 % p.D : 0;  // channel within the concatenated heads
    const int h = ch / p.hs;
    const int i0 = chunk * p.rows, i1 = min(p.t + 1, i0 + p.rows);

    // this block's heads' bias rows w_h[t, i0:i1] (a slab spans whole heads)
    __shared__ float ws[kMaxHeads][kMaxRows];
    const int h_first = (slab * kSlab % p.D) / p.hs;
    const int nh = min(p.H, (kSlab + p.hs - 1) / p.hs + 1);
    const int span = i1 - i0;
    for (int k = threadIdx.x; k < nh * span; k += kThreads) {
        const int hh = (h_first + k / span) % p.H, i = i0 + k % span;
        ws[k / span][k % span] = p.w[hh * p.wh + (size_t)p.t * p.ldw + i];
    }
    __syncthreads();
    const int hl = (h - h_first + p.H) % p.H;  // this thread's head within ws

    float m[4], num[4], den[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        m[j] = -INFINITY;
        num[j] = den[j] = 0.f;
    }
    const size_t rowstride = (size_t)cols * 2;  // floats per cache row
    const float *qrow = p.qkv + (size_t)b * p.ldq;
    if (active) {
        for (int g0 = i0; g0 < i1; g0 += kGroup) {
            float kk[kGroup][4], vv[kGroup][4];
#pragma unroll
            for (int r = 0; r < kGroup; ++r) {
                const int i = g0 + r;
                if (i < i1 && i < p.t) {
                    const float4 *src =
                        reinterpret_cast<const float4 *>(p.cache + (size_t)i * rowstride + (size_t)c0 * 2);
                    const float4 a = __ldcs(src), v = __ldcs(src + 1);
                    kk[r][0] = a.x; kk[r][1] = a.y; kk[r][2] = a.z; kk[r][3] = a.w;
                    vv[r][0] = v.x; vv[r][1] = v.y; vv[r][2] = v.z; vv[r][3] = v.w;
                } else if (i == p.t) {
                    // the newest position: fresh projection, appended to the cache
                    const float4 a = *reinterpret_cast<const float4 *>(qrow + p.D + ch);
                    const float4 v = *reinterpret_cast<const float4 *>(qrow + 2 * p.D + ch);
                    float4 *dst =
                        reinterpret_cast<float4 *>(p.cache + (size_t)i * rowstride + (size_t)c0 * 2);
                    dst[0] = a;
                    dst[1] = v;
                    kk[r][0] = a.x; kk[r][1] = a.y; kk[r][2] = a.z; kk[r][3] = a.w;
                    vv[r][0] = v.x; vv[r][1] = v.y; vv[r][2] = v.z; vv[r][3] = v.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        kk[r][j] = -INFINITY;
                        vv[r][j] = 0.f;
                    }
                }
            }
            float s[kGroup][4], mx[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) mx[j] = m[j];
#pragma unroll
            for (int r = 0; r < kGroup; ++r) {
                const int i = g0 + r;
                const float wv = i < i1 ? ws[hl][i - i0] : 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    s[r][j] = kk[r][j] + wv;
                    mx[j] = fmaxf(mx[j], s[r][j]);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (mx[j] == -INFINITY) continue;
                const float scale = __expf(m[j] - mx[j]);  // 0 when m = -inf
                num[j] *= scale;
                den[j] *= scale;
                m[j] = mx[j];
#pragma unroll
                for (int r = 0; r < kGroup; ++r) {
                    const float e = __expf(s[r][j] - mx[j]);  // 0 for padded rows
                    num[j] += e * vv[r][j];
                    den[j] += e;
                }
            }
        }
        float *pp = p.part + ((size_t)chunk * cols + c0) * 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            pp[3 * j] = m[j];
            pp[3 * j + 1] = num[j];
            pp[3 * j + 2] = den[j];
        }
    }
    // the last block of this slab merges the chunks
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        const int done = atomicAdd(p.counter + slab, 1);
        last = done == p.chunks - 1;
        if (last) p.counter[slab] = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!last || !active) return;
    __threadfence();
    // every chunk's 12 partials of this thread's 4 columns are contiguous:
    // loads of four chunks are issued together, then combined
    float M[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, n[4] = {0.f, 0.f, 0.f, 0.f},
          d[4] = {0.f, 0.f, 0.f, 0.f};
    for (int q0 = 0; q0 < p.chunks; q0 += 4) {
        float4 pr[4][3];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (q0 + u < p.chunks) {
                const float4 *src =
                    reinterpret_cast<const float4 *>(p.part + ((size_t)(q0 + u) * cols + c0) * 3);
                pr[u][0] = __ldcg(src);
                pr[u][1] = __ldcg(src + 1);
                pr[u][2] = __ldcg(src + 2);
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (q0 + u < p.chunks) {
                const float v[12] = {pr[u][0].x, pr[u][0].y, pr[u][0].z, pr[u][0].w,
                                     pr[u][1].x, pr[u][1].y, pr[u][1].z, pr[u][1].w,
                                     pr[u][2].x, pr[u][2].y, pr[u][2].z, pr[u][2].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float mq = v[3 * j];
                    if (mq == -INFINITY) continue;
                    const float nm = fmaxf(M[j], mq);
                    const float a = __expf(M[j] - nm), b_ = __expf(mq - nm);
                    n[j] = n[j] * a + v[3 * j + 1] * b_;
                    d[j] = d[j] * a + v[3 * j + 2] * b_;
                    M[j] = nm;
                }
            }
    }
    const float4 qv = *reinterpret_cast<const float4 *>(qrow + ch);
    float4 z;
    z.x = sigm(qv.x) * (n[0] / d[0]);
    z.y = sigm(qv.y) * (n[1] / d[1]);
    z.z = sigm(qv.z) * (n[2] / d[2]);
    z.w = sigm(qv.w) * (n[3] / d[3]);
    *reinterpret_cast<float4 *>(p.Z + (size_t)b * p.ldz + ch) = z;
}

// Copy k and v of positions [0, T) of a prefill's fused projection
// ([B*T, 3*D] rows, row stride ldq) into the cache layout.
__global__ void cache_fill_kernel(const float *__restrict__ qkv, int ldq, int B, int T, int D,
                                  float *__restrict__ cache)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // 4-column group
    const size_t groups = (size_t)B * D / 4;
    if (g >= groups * T) return;
    const int t = (int)(g / groups);
    const size_t cg = g % groups;
    const int b = (int)(cg * 4 / D), ch = (int)(cg * 4 % D);
    const float *row = qkv + ((size_t)b * T + t) * ldq;
    float4 *dst = reinterpret_cast<float4 *>(cache + ((size_t)t * groups + cg) * 8);
    dst[0] = *reinterpret_cast<const float4 *>(row + D + ch);
    dst[1] = *reinterpret_cast<const float4 *>(row + 2 * D + ch);
}

}  // namespace dec
}  // namespace dc

using namespace dc;

extern "C" {

size_t dc_aft_decode_workspace_size(int B, int D, int Tmax)
{
    const size_t cols = (size_t)B * D;
    const size_t slabs = (cols + dec::kSlab - 1) / dec::kSlab;
    const size_t chunks = ((size_t)Tmax + dec::kGroup - 1) / dec::kGroup;
    return round_up((int64_t)(slabs * sizeof(int)), 256) + chunks * cols * 3 * sizeof(float);
}

int dc_aft_decode(const float *qkv, int ldq, const float *w, int ldw, long long head_stride_w,
                  float *cache, int B, int H, int hs, const int *pos, int Tmax, float *Z, int ldz,
                  void *workspace, size_t workspace_bytes, void *stream)
{
    using namespace dc::dec;
    clear_error();
    const int D = H * hs;
    if (B <= 0 || H <= 0 || hs <= 0 || Tmax <= 0)
        return fail(DC_ERR_INVALID, "bad decode shape B=%d H=%d hs=%d Tmax=%d", B, H, hs, Tmax);
    if (hs % 4 || ldq % 4 || ldz % 4 || ldq < 3 * D || ldz < D || ldw < Tmax)
        return fail(DC_ERR_INVALID,
                    "hs, ldq and ldz must be multiples of 4, ldq >= 3D, ldz >= D, ldw >= Tmax");
    if (!pos || !qkv || !w || !cache || !Z || !workspace) return fail(DC_ERR_INVALID, "null pointer");
    if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(cache) |
          reinterpret_cast<uintptr_t>(Z)) & 15) != 0)
        return fail(DC_ERR_INVALID, "qkv, cache and Z need 16-byte alignment");
    if (workspace_bytes < dc_aft_decode_workspace_size(B, D, Tmax))
        return fail(DC_ERR_NOMEM, "decode workspace too small");
    // the heads one slab touches must fit the block's bias rows
    if (std::min(H, (kSlab + hs - 1) / hs + 1) > kMaxHeads)
        return fail(DC_ERR_UNSUPPORTED, "more than %d heads per %d-column slab", kMaxHeads, kSlab);
    const int cols = B * D;
    const int slabs = (cols + kSlab - 1) / kSlab;
    // history chunks: the grid holds about two blocks per SM (slabs x
    // chunks); the kernel splits the t+1 rows of each step over them, at
    // most kMaxRows rows a chunk
    const int min_chunks = (Tmax + kMaxRows - 1) / kMaxRows;
    if (min_chunks > kMaxChunks)
        return fail(DC_ERR_UNSUPPORTED, "Tmax %d above %d", Tmax, kMaxRows * kMaxChunks);
    const int max_chunks =
        std::min(kMaxChunks, std::max(min_chunks, std::max(1, 2 * sm_count() / slabs)));
    Params p{};
    p.qkv = qkv;
    p.ldq = ldq;
    p.w = w;
    p.ldw = ldw;
    p.wh = head_stride_w;
    p.cache = cache;
    p.B = B;
    p.H = H;
    p.hs = hs;
    p.D = D;
    p.Tmax = Tmax;
    p.pos = pos;
    p.status = device_status_word();
    p.Z = Z;
    p.ldz = ldz;
    char *ws = static_cast<char *>(workspace);
    p.counter = reinterpret_cast<int *>(ws);
    p.part = reinterpret_cast<float *>(ws + round_up((int64_t)(slabs * sizeof(int)), 256));
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("aft_decode", st);
    (void)launch_pdl(aft_decode_kernel, dim3(slabs, max_chunks), dim3(kThreads), 0, st, 1, p);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_kv_cache_fill(const float *qkv, int ldq, int B, int T, int D, float *cache, void *stream)
{
    clear_error();
    if (B < 0 || T < 0 || D % 4 || ldq % 4 || ldq < 3 * D) return fail(DC_ERR_INVALID, "bad shape");
    const size_t n = (size_t)B * D / 4 * T;
    if (n == 0) return DC_OK;
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("kv_cache_fill", st);
    (void)launch_pdl(dec::cache_fill_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st,
                     1, qkv, ldq, B, T, D, cache);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

}  // extern "C"
