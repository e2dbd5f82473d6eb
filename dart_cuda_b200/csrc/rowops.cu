// HBM-bound row kernels of the training step: affine LayerNorm, row-broadcast
// bias add, label-smoothed cross-entropy with fused log-softmax, AdamW.
//
// Each kernel touches every element once in the forward (one read, one
// write) and reduces with warp shuffles; column reductions of the backward
// (dgamma, dbeta, bias grad) are two-stage (per-CTA partials, then a column
// pass) instead of the reference's per-row atomics.
#include <math.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "dc_internal.h"
#include "dc_ptx.cuh"

namespace dc {
namespace rows {

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// block-wide sum; `red` holds >= 32 floats; every thread gets the result
__device__ __forceinline__ float block_sum(float v, float *red)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float r = (lane < nw) ? red[lane] : 0.f;
    return warp_sum(r);
}
__device__ __forceinline__ float block_max(float v, float *red)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    const int nw = (blockDim.x + 31) >> 5;
    float r = (lane < nw) ? red[lane] : -INFINITY;
    return warp_max(r);
}

// ====================================================================== LN
// One warp per row, the row held in registers (NV float4 per lane, C <= 128*NV).
// Two-pass mean/variance over the registers, as the reference computes it
// (native/src/kernels/layernorm_embed.cuh:140-176), with one global read.
template <int NV>
__global__ void ln_fwd_warp(const float *__restrict__ x, const float *__restrict__ gamma,
                            const float *__restrict__ beta, float *__restrict__ y, int R, int C,
                            float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= R) return;
    const int C4 = C >> 2;
    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * C);
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int j = lane + 32 * k;
        v[k] = (j < C4) ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    const float mean = warp_sum(s) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int j = lane + 32 * k;
        if (j < C4) {
            float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
            q += (a * a + b * b) + (c * c + d * d);
        }
    }
    const float inv_std = rsqrtf(warp_sum(q) / (float)C + eps);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    const float4 *b4 = reinterpret_cast<const float4 *>(beta);
    float4 *yr = reinterpret_cast<float4 *>(y + (size_t)row * C);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int j = lane + 32 * k;
        if (j < C4) {
            const float4 g = g4[j], bb = b4[j];
            float4 o;
            o.x = (v[k].x - mean) * inv_std * g.x + bb.x;
            o.y = (v[k].y - mean) * inv_std * g.y + bb.y;
            o.z = (v[k].z - mean) * inv_std * g.z + bb.z;
            o.w = (v[k].w - mean) * inv_std * g.w + bb.w;
            yr[j] = o;
        }
    }
}

// General fallback: one block per row, loops over the row (any C).
__global__ void ln_fwd_block(const float *__restrict__ x, const float *__restrict__ gamma,
                             const float *__restrict__ beta, float *__restrict__ y, int R, int C,
                             float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = x + (size_t)row * C;
    float s = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) s += xr[j];
    const float mean = block_sum(s, red) / (float)C;
    float q = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        float d = xr[j] - mean;
        q += d * d;
    }
    const float inv_std = rsqrtf(block_sum(q, red) / (float)C + eps);
    float *yr = y + (size_t)row * C;
    for (int j = threadIdx.x; j < C; j += blockDim.x)
        yr[j] = (xr[j] - mean) * inv_std * gamma[j] + beta[j];
}

// Backward, one warp per row; each CTA also accumulates its rows'
// contributions to dgamma/dbeta and writes them as one partial row
// part[blockIdx.x][0:C] (dgamma) and part[blockIdx.x][C:2C] (dbeta).
template <int NV>
__global__ void ln_bwd_warp(const float *__restrict__ x, const float *__restrict__ gamma,
                            const float *__restrict__ dy, float *__restrict__ dx,
                            float *__restrict__ part, int R, int C, float eps, int accumulate,
                            int rows_per_cta)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    extern __shared__ float sh[];  // [nwarps][2C]
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int C4 = C >> 2;
    float4 gg[NV], gb[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        gg[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        gb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(R, r0 + rows_per_cta);
    // with accumulate, rows of up to 512 columns also load the old dx with
    // x and dy (one memory round trip a row instead of two)
    constexpr bool kEarlyOld = NV <= 4;
    for (int row = r0 + wid; row < r1; row += nw) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)row * C);
        const float4 *gr = reinterpret_cast<const float4 *>(dy + (size_t)row * C);
        float4 *dr = reinterpret_cast<float4 *>(dx + (size_t)row * C);
        float4 v[NV], g[NV], old[kEarlyOld ? NV : 1];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int j = lane + 32 * k;
            const bool in = j < C4;
            v[k] = in ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            g[k] = in ? gr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            if (kEarlyOld) old[kEarlyOld ? k : 0] = in && accumulate ? dr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < NV; ++k) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        const float mean = warp_sum(s) / (float)C;
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int j = lane + 32 * k;
            if (j < C4) {
                float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
                q += (a * a + b * b) + (c * c + d * d);
            }
        }
        const float inv_std = rsqrtf(warp_sum(q) / (float)C + eps);
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int j = lane + 32 * k;
            if (j < C4) {
                const float4 ga = g4[j];
                float4 xh;
                xh.x = (v[k].x - mean) * inv_std;
                xh.y = (v[k].y - mean) * inv_std;
                xh.z = (v[k].z - mean) * inv_std;
                xh.w = (v[k].w - mean) * inv_std;
                s1 += (g[k].x * ga.x + g[k].y * ga.y) + (g[k].z * ga.z + g[k].w * ga.w);
                s2 += (g[k].x * ga.x * xh.x + g[k].y * ga.y * xh.y) +
                      (g[k].z * ga.z * xh.z + g[k].w * ga.w * xh.w);
                gg[k].x += g[k].x * xh.x;
                gg[k].y += g[k].y * xh.y;
                gg[k].z += g[k].z * xh.z;
                gg[k].w += g[k].w * xh.w;
                gb[k].x += g[k].x;
                gb[k].y += g[k].y;
                gb[k].z += g[k].z;
                gb[k].w += g[k].w;
                v[k] = xh;
            }
        }
        const float invC = 1.0f / (float)C;
        const float m1 = warp_sum(s1) * invC, m2 = warp_sum(s2) * invC;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int j = lane + 32 * k;
            if (j < C4) {
                const float4 ga = g4[j];
                float4 o;
                o.x = inv_std * (g[k].x * ga.x - m1 - v[k].x * m2);
                o.y = inv_std * (g[k].y * ga.y - m1 - v[k].y * m2);
                o.z = inv_std * (g[k].z * ga.z - m1 - v[k].z * m2);
                o.w = inv_std * (g[k].w * ga.w - m1 - v[k].w * m2);
                if (accumulate) {
                    const float4 a = kEarlyOld ? old[kEarlyOld ? k : 0] : dr[j];
                    o.x += a.x;
                    o.y += a.y;
                    o.z += a.z;
                    o.w += a.w;
                }
                dr[j] = o;
            }
        }
    }
    // CTA partials of dgamma/dbeta
    float4 *myg = reinterpret_cast<float4 *>(sh + (size_t)wid * 2 * C);
    float4 *myb = reinterpret_cast<float4 *>(sh + (size_t)wid * 2 * C + C);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        const int j = lane + 32 * k;
        if (j < C4) {
            myg[j] = gg[k];
            myb[j] = gb[k];
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < 2 * C; j += blockDim.x) {
        float acc = 0.f;
        for (int w = 0; w < nw; ++w) acc += sh[(size_t)w * 2 * C + j];
        part[(size_t)blockIdx.x * 2 * C + j] = acc;
    }
}

// Generic backward, one block per row; partials one row per CTA (= per row).
__global__ void ln_bwd_block(const float *__restrict__ x, const float *__restrict__ gamma,
                             const float *__restrict__ dy, float *__restrict__ dx,
                             float *__restrict__ part, int R, int C, float eps, int accumulate)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = x + (size_t)row * C;
    const float *gr = dy + (size_t)row * C;
    float s = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) s += xr[j];
    const float mean = block_sum(s, red) / (float)C;
    float q = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        float d = xr[j] - mean;
        q += d * d;
    }
    const float inv_std = rsqrtf(block_sum(q, red) / (float)C + eps);
    float s1 = 0.f, s2 = 0.f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float xh = (xr[j] - mean) * inv_std;
        const float dxh = gr[j] * gamma[j];
        s1 += dxh;
        s2 += dxh * xh;
        part[(size_t)row * 2 * C + j] = gr[j] * xh;
        part[(size_t)row * 2 * C + C + j] = gr[j];
    }
    const float invC = 1.0f / (float)C;
    const float m1 = block_sum(s1, red) * invC;
    const float m2 = block_sum(s2, red) * invC;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const float xh = (xr[j] - mean) * inv_std;
        float o = inv_std * (gr[j] * gamma[j] - m1 - xh * m2);
        if (accumulate) o += dx[(size_t)row * C + j];
        dx[(size_t)row * C + j] = o;
    }
}

// Sum `nparts` partial rows of width W into out (+= when accumulate).  A
// block (32 x kColLanes) covers 32 columns; lane y adds partials y, y +
// kColLanes, ... with four loads in flight, and the lanes' sums are added in
// a fixed order (deterministic).  One thread per column walking all partials
// was latency-bound: hundreds of dependent L2 round trips on a handful of SMs.
constexpr int kColLanes = 16;
__global__ void __launch_bounds__(32 * kColLanes)
    colsum_parts(const float *__restrict__ part, int nparts, int W, float *out0, float *out1,
                 int split, int accumulate)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[kColLanes][33];
    const int j = blockIdx.x * 32 + threadIdx.x;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (j < W) {
        int p = threadIdx.y;
        for (; p + 3 * kColLanes < nparts; p += 4 * kColLanes) {
            const float *q = part + (size_t)p * W + j;
            a0 += q[0];
            a1 += q[(size_t)kColLanes * W];
            a2 += q[(size_t)2 * kColLanes * W];
            a3 += q[(size_t)3 * kColLanes * W];
        }
        for (; p < nparts; p += kColLanes) a0 += part[(size_t)p * W + j];
    }
    red[threadIdx.y][threadIdx.x] = (a0 + a1) + (a2 + a3);
    __syncthreads();
    if (threadIdx.y == 0 && j < W) {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < kColLanes; ++k) acc += red[k][threadIdx.x];
        float *o = (j < split) ? out0 + j : out1 + (j - split);
        *o = accumulate ? *o + acc : acc;
    }
}

// ==================================================================== bias
__global__ void bias_fwd_vec(const float4 *__restrict__ a, const float4 *__restrict__ b,
                             float4 *__restrict__ out, size_t n4, int N4)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], y = b[i % N4];
        out[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    }
}
__global__ void bias_fwd_scalar(const float *__restrict__ a, const float *__restrict__ b,
                                float *__restrict__ out, size_t n, int N)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = a[i] + b[i % N];
}

// block (32, 8): 32 columns x row slice; da (+)= dy; column partial sums.
__global__ void bias_bwd_kernel(const float *__restrict__ dy, float *__restrict__ da,
                                float *__restrict__ part, int M, int N, int rows_per_cta,
                                int accumulate)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[8][33];
    const int col = blockIdx.x * 32 + threadIdx.x;
    const int r0 = blockIdx.y * rows_per_cta, r1 = min(M, r0 + rows_per_cta);
    float acc = 0.f;
    if (col < N) {
        for (int r = r0 + threadIdx.y; r < r1; r += 8) {
            const size_t o = (size_t)r * N + col;
            const float g = dy[o];
            acc += g;
            if (da) da[o] = accumulate ? da[o] + g : g;
        }
    }
    red[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && col < N) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x];
        part[(size_t)blockIdx.y * N + col] = s;
    }
}

// 16-byte variant (N % 4 == 0, aligned rows): a block covers 128 columns x 8
// row lanes, each lane two rows per iteration so four loads are in flight.
__global__ void bias_bwd_vec4(const float4 *__restrict__ dy, float4 *__restrict__ da,
                              float *__restrict__ part, int M, int N4, int rows_per_cta,
                              int accumulate)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float4 red[8][33];
    const int col = blockIdx.x * 32 + threadIdx.x;
    const int r0 = blockIdx.y * rows_per_cta, r1 = min(M, r0 + rows_per_cta);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col < N4) {
        int r = r0 + threadIdx.y;
        for (; r + 8 < r1; r += 16) {
            const size_t o0 = (size_t)r * N4 + col, o1 = o0 + (size_t)8 * N4;
            const float4 g0 = __ldcs(dy + o0), g1 = __ldcs(dy + o1);
            acc.x += g0.x + g1.x;
            acc.y += g0.y + g1.y;
            acc.z += g0.z + g1.z;
            acc.w += g0.w + g1.w;
            if (da) {
                float4 a0 = g0, a1 = g1;
                if (accumulate) {
                    const float4 p0 = da[o0], p1 = da[o1];
                    a0 = make_float4(p0.x + g0.x, p0.y + g0.y, p0.z + g0.z, p0.w + g0.w);
                    a1 = make_float4(p1.x + g1.x, p1.y + g1.y, p1.z + g1.z, p1.w + g1.w);
                }
                da[o0] = a0;
                da[o1] = a1;
            }
        }
        for (; r < r1; r += 8) {
            const size_t o = (size_t)r * N4 + col;
            const float4 g = __ldcs(dy + o);
            acc.x += g.x;
            acc.y += g.y;
            acc.z += g.z;
            acc.w += g.w;
            if (da) {
                float4 a = g;
                if (accumulate) {
                    const float4 p = da[o];
                    a = make_float4(p.x + g.x, p.y + g.y, p.z + g.z, p.w + g.w);
                }
                da[o] = a;
            }
        }
    }
    red[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && col < N4) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            s.x += red[k][threadIdx.x].x;
            s.y += red[k][threadIdx.x].y;
            s.z += red[k][threadIdx.x].z;
            s.w += red[k][threadIdx.x].w;
        }
        reinterpret_cast<float4 *>(part)[(size_t)blockIdx.y * N4 + col] = s;
    }
}

// Column sums on clusters, one launch: the CL CTAs of a cluster (grid x)
// split the rows of one block of 4*QN columns (grid y).  A CTA's 512 threads
// are 512/QN row lanes x QN float4 column lanes with four rows in flight
// each; lanes of a column meet by shuffles and shared memory, and rank 0 adds
// the cluster's CTA sums, read from distributed shared memory in rank order.
// The sums are deterministic and no partial rows go through global memory
// (the two-pass form spent a second launch and an L2 round trip on them).
// QN = 4 (16 columns, 64-byte row segments): 8-column blocks doubled the
// CTAs but halved the bytes per L1 wavefront and ran at half the bandwidth.
// 16-CTA clusters (a non-portable size) for narrow matrices, to fill the
// SMs with 256 CTAs at [262144, 256], ran slower still; tall matrices of at
// most 1024 columns take the row-contiguous form below instead.
constexpr int kSumCluster = 8;
constexpr int kSumThreads = 512;

__device__ __forceinline__ void add4(float4 &a, const float4 &b)
{
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
}

template <int QN, int CL>
__global__ void __launch_bounds__(kSumThreads)
    bias_bwd_cluster(const float4 *__restrict__ dy, float4 *__restrict__ da,
                     float *__restrict__ db, int M, int N4, int accumulate)
{
    constexpr int kRowLanes = kSumThreads / QN;
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float4 wsum[kSumThreads / 32][QN];
    __shared__ float csum[4 * QN];
    const int q = threadIdx.x % QN, rl = threadIdx.x / QN;
    const int c4 = blockIdx.y * QN + q;
    const int rpc = (M + CL - 1) / CL;
    const int r0 = (int)cluster_rank() * rpc, r1 = min(M, r0 + rpc);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c4 < N4) {
        int r = r0 + rl;
        for (; r + 3 * kRowLanes < r1; r += 4 * kRowLanes) {
            float4 g[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) g[k] = __ldcs(dy + (size_t)(r + k * kRowLanes) * N4 + c4);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                add4(acc, g[k]);
                if (da) {
                    const size_t o = (size_t)(r + k * kRowLanes) * N4 + c4;
                    float4 a = g[k];
                    if (accumulate) add4(a, da[o]);
                    da[o] = a;
                }
            }
        }
        for (; r < r1; r += kRowLanes) {
            const size_t o = (size_t)r * N4 + c4;
            const float4 g = __ldcs(dy + o);
            add4(acc, g);
            if (da) {
                float4 a = g;
                if (accumulate) add4(a, da[o]);
                da[o] = a;
            }
        }
    }
#pragma unroll
    for (int off = QN; off < 32; off <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
    }
    if ((threadIdx.x & 31) < QN) wsum[threadIdx.x >> 5][q] = acc;
    __syncthreads();
    if (threadIdx.x < 4 * QN) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSumThreads / 32; ++w)
            v += reinterpret_cast<const float *>(&wsum[w][0])[threadIdx.x];
        csum[threadIdx.x] = v;
    }
    cluster_sync_all();
    if (cluster_rank() == 0 && threadIdx.x < 4 * QN) {
        const int j = blockIdx.y * 4 * QN + threadIdx.x;
        const uint32_t mine = (uint32_t)__cvta_generic_to_shared(&csum[threadIdx.x]);
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < CL; ++r) v += ld_dsmem_f32(smem_in_cta(mine, r));
        if (j < 4 * N4) db[j] = accumulate ? db[j] + v : v;
    }
    cluster_sync_all();  // the CTA sums stay readable until rank 0 has added them
}

// Column sums of a tall matrix of at most 1024 columns, whole rows: the rows
// go in units of 512/N4 (one row per N4 float4 lanes of the 512 threads), and
// the units round-robin over the CTAs, four in flight a thread, so the grid
// streams one contiguous front as a copy does (whole row ranges a CTA ran at
// 0.77 of HBM, 296 separate streams; round-robin units 0.80).  Every warp
// reads and writes contiguous bytes.  A CTA adds its rows per column in
// shared memory in row-lane order and writes its partial sums; the CTA that
// finishes last (an atomic count, no CTA waits for another) adds the
// partials in CTA order, so the sums are deterministic.  It resets the count
// for the next call.
__global__ void __launch_bounds__(kSumThreads)
    bias_bwd_rows(const float4 *__restrict__ dy, float4 *__restrict__ da, float *__restrict__ db,
                  float4 *__restrict__ part, unsigned *__restrict__ done, int M, int N4,
                  int accumulate)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float4 red[kSumThreads];
    __shared__ bool last;
    const int lanes = kSumThreads / N4;  // rows in flight per step (>= 2)
    const int c4 = threadIdx.x % N4, rl = threadIdx.x / N4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rl < lanes) {
        const int units = (M + lanes - 1) / lanes, G = (int)gridDim.x;
        int u = blockIdx.x;
        for (; u + 3 * G < units; u += 4 * G) {
            float4 g[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int r = (u + k * G) * lanes + rl;
                g[k] = r < M ? __ldcs(dy + (size_t)r * N4 + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int r = (u + k * G) * lanes + rl;
                add4(acc, g[k]);
                if (da && r < M) {
                    const size_t o = (size_t)r * N4 + c4;
                    float4 a = g[k];
                    if (accumulate) add4(a, da[o]);
                    __stcs(da + o, a);
                }
            }
        }
        for (; u < units; u += G) {
            const int r = u * lanes + rl;
            if (r >= M) continue;
            const size_t o = (size_t)r * N4 + c4;
            const float4 g = __ldcs(dy + o);
            add4(acc, g);
            if (da) {
                float4 a = g;
                if (accumulate) add4(a, da[o]);
                __stcs(da + o, a);
            }
        }
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < N4) {
        float4 v = red[threadIdx.x];
        for (int k = 1; k < lanes; ++k) add4(v, red[k * N4 + threadIdx.x]);
        part[(size_t)blockIdx.x * N4 + threadIdx.x] = v;
    }
    __threadfence();  // this CTA's partials are visible before it is counted
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int j = threadIdx.x; j < 4 * N4; j += blockDim.x) {
        const float *pf = reinterpret_cast<const float *>(part);
        float v = 0.f;
        for (int c = 0; c < (int)gridDim.x; ++c) v += __ldcg(pf + (size_t)c * 4 * N4 + j);
        db[j] = accumulate ? db[j] + v : v;
    }
    if (threadIdx.x == 0) *done = 0u;
}

// ===================================================================== CE
// One warp per row (V small) or one block per row; online max/sum-exp with a
// single read of the row.  loss_row = (1-eps)(lse - x_y) + eps(lse - mean x),
// lse = max + log(sum exp(x - max) + 1e-12)  (loss_optim.cuh:163-205).
__device__ __forceinline__ void online_update(float &m, float &s, float x)
{
    if (x > m) {
        s = s * __expf(m - x) + 1.0f;
        m = x;
    } else {
        s += __expf(x - m);
    }
}
__device__ __forceinline__ void online_merge(float &m, float &s, float m2, float s2)
{
    const float mm = fmaxf(m, m2);
    if (mm == -INFINITY) return;
    s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
    m = mm;
}

__global__ void ce_fwd_warp(const float *__restrict__ logits, const int32_t *__restrict__ tgt,
                            float *__restrict__ row_loss, int T, int V, float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= T) return;
    const float *xr = logits + (size_t)row * V;
    float m = -INFINITY, s = 0.f, sx = 0.f;
    for (int v = lane; v < V; v += 32) {
        const float x = xr[v];
        online_update(m, s, x);
        sx += x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        online_merge(m, s, m2, s2);
    }
    sx = warp_sum(sx);
    if (lane == 0) {
        const float lse = m + logf(s + 1e-12f);
        const float xt = xr[tgt[row]];
        row_loss[row] = (1.0f - eps) * (lse - xt) + eps * (lse - sx / (float)V);
    }
}

__global__ void ce_fwd_block(const float *__restrict__ logits, const int32_t *__restrict__ tgt,
                             float *__restrict__ row_loss, int T, int V, float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float rm[32], rs[32], red[32];
    const int row = blockIdx.x;
    const float *xr = logits + (size_t)row * V;
    float m = -INFINITY, s = 0.f, sx = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float x = xr[v];
        online_update(m, s, x);
        sx += x;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        online_merge(m, s, m2, s2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        rm[wid] = m;
        rs[wid] = s;
    }
    sx = block_sum(sx, red);
    if (wid == 0) {
        m = lane < nw ? rm[lane] : -INFINITY;
        s = lane < nw ? rs[lane] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
            online_merge(m, s, m2, s2);
        }
        if (lane == 0) {
            const float lse = m + logf(s + 1e-12f);
            const float xt = xr[tgt[row]];
            row_loss[row] = (1.0f - eps) * (lse - xt) + eps * (lse - sx / (float)V);
        }
    }
}

// Wide rows (1024 < V <= 1024*NV4, V % 4 == 0, 16-byte aligned): one block
// of 256 threads per row holds the whole row in registers (NV4 float4 per
// thread, all loads issued up front), so the forward reads each logit once
// and the backward reads once and writes once.  Two block reductions: the
// row maximum, then sum e^{x-max} and sum x.
template <int NV4>
__device__ __forceinline__ void ce_row_regs(const float *__restrict__ xr, int V, float4 (&x)[NV4],
                                            float &mx, float &s, float &sx, float *red)
{
    const float4 *x4 = reinterpret_cast<const float4 *>(xr);
    const int n4 = V >> 2;
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = threadIdx.x + k * 256;
        x[k] = i < n4 ? __ldcs(x4 + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        m = fmaxf(m, fmaxf(fmaxf(x[k].x, x[k].y), fmaxf(x[k].z, x[k].w)));
    }
    mx = block_max(m, red);
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        if (threadIdx.x + k * 256 < n4) {
            a += __expf(x[k].x - mx) + __expf(x[k].y - mx) + __expf(x[k].z - mx) + __expf(x[k].w - mx);
            b += (x[k].x + x[k].y) + (x[k].z + x[k].w);
        }
    }
    s = block_sum(a, red);
    sx = block_sum(b, red);
}

template <int NV4>
__global__ void __launch_bounds__(256) ce_fwd_regs(const float *__restrict__ logits,
                                                   const int32_t *__restrict__ tgt,
                                                   float *__restrict__ row_loss, int T, int V,
                                                   float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = logits + (size_t)row * V;
    float4 x[NV4];
    float mx, s, sx;
    ce_row_regs<NV4>(xr, V, x, mx, s, sx, red);
    if (threadIdx.x == 0) {
        const float lse = mx + logf(s + 1e-12f);
        const float xt = xr[tgt[row]];
        row_loss[row] = (1.0f - eps) * (lse - xt) + eps * (lse - sx / (float)V);
    }
}

template <int NV4>
__global__ void __launch_bounds__(256) ce_bwd_regs(const float *__restrict__ logits,
                                                   const int32_t *__restrict__ tgt,
                                                   const float *__restrict__ gscale,
                                                   float *__restrict__ grad, int T, int V,
                                                   float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = logits + (size_t)row * V;
    float4 x[NV4];
    float mx, s, sx;
    ce_row_regs<NV4>(xr, V, x, mx, s, sx, red);
    const float inv = 1.0f / (s + 1e-12f);
    const float scale = (gscale ? gscale[0] : 1.0f) / (float)T;
    const int y = tgt[row];
    const float off = eps / (float)V;
    float4 *g4 = reinterpret_cast<float4 *>(grad + (size_t)row * V);
    const int n4 = V >> 2;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = threadIdx.x + k * 256;
        if (i < n4) {
            const int v0 = 4 * i;
            float4 g;
            g.x = (__expf(x[k].x - mx) * inv - ((v0 == y ? 1.0f - eps : 0.f) + off)) * scale;
            g.y = (__expf(x[k].y - mx) * inv - ((v0 + 1 == y ? 1.0f - eps : 0.f) + off)) * scale;
            g.z = (__expf(x[k].z - mx) * inv - ((v0 + 2 == y ? 1.0f - eps : 0.f) + off)) * scale;
            g.w = (__expf(x[k].w - mx) * inv - ((v0 + 3 == y ? 1.0f - eps : 0.f) + off)) * scale;
            __stcs(g4 + i, g);
        }
    }
}

// mean of the row losses (ce_mean_reduce, engine.cu:829-837), deterministic
__global__ void mean_kernel(const float *__restrict__ v, int n, float *__restrict__ out)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float red[32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
    s = block_sum(s, red);
    if (threadIdx.x == 0) out[0] = s / (float)n;
}

// grad = (softmax - ((1-eps) 1_y + eps/V)) * g / T, written (not accumulated)
// (loss_optim.cuh:207-244)
__global__ void ce_bwd_warp(const float *__restrict__ logits, const int32_t *__restrict__ tgt,
                            const float *__restrict__ gscale, float *__restrict__ grad, int T,
                            int V, float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= T) return;
    const float *xr = logits + (size_t)row * V;
    float m = -INFINITY, s = 0.f;
    for (int v = lane; v < V; v += 32) online_update(m, s, xr[v]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        online_merge(m, s, m2, s2);
    }
    const float inv = 1.0f / (s + 1e-12f);
    const float scale = (gscale ? gscale[0] : 1.0f) / (float)T;
    const int y = tgt[row];
    const float off = eps / (float)V;
    float *gr = grad + (size_t)row * V;
    for (int v = lane; v < V; v += 32) {
        const float sm = __expf(xr[v] - m) * inv;
        const float tp = (v == y ? (1.0f - eps) : 0.f) + off;
        gr[v] = (sm - tp) * scale;
    }
}

__global__ void ce_bwd_block(const float *__restrict__ logits, const int32_t *__restrict__ tgt,
                             const float *__restrict__ gscale, float *__restrict__ grad, int T,
                             int V, float eps)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float rm[32], rs[32];
    const int row = blockIdx.x;
    const float *xr = logits + (size_t)row * V;
    float m = -INFINITY, s = 0.f;
    for (int v = threadIdx.x; v < V; v += blockDim.x) online_update(m, s, xr[v]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        online_merge(m, s, m2, s2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) {
        rm[wid] = m;
        rs[wid] = s;
    }
    __syncthreads();
    m = lane < nw ? rm[lane] : -INFINITY;
    s = lane < nw ? rs[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        online_merge(m, s, m2, s2);
    }
    const float inv = 1.0f / (s + 1e-12f);
    const float scale = (gscale ? gscale[0] : 1.0f) / (float)T;
    const int y = tgt[row];
    const float off = eps / (float)V;
    float *gr = grad + (size_t)row * V;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float sm = __expf(xr[v] - m) * inv;
        const float tp = (v == y ? (1.0f - eps) : 0.f) + off;
        gr[v] = (sm - tp) * scale;
    }
}

// =================================================================== Adam
// loss_optim.cuh:255-298: step = t+1, p -= lr*mhat/(sqrt(vhat)+eps) + lr*wd*p
__global__ void adam_kernel(float *__restrict__ p, const float *__restrict__ g,
                            float *__restrict__ m, float *__restrict__ v, int64_t n, float lr,
                            float b1, float b2, float eps, float wd, float c1, float c2)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gr = g[i];
        const float mi = b1 * m[i] + (1.0f - b1) * gr;
        const float vi = b2 * v[i] + (1.0f - b2) * (gr * gr);
        m[i] = mi;
        v[i] = vi;
        const float mh = mi / c1, vh = vi / c2;
        const float pi = p[i];
        p[i] = pi - lr * mh / (sqrtf(vh) + eps) - lr * wd * pi;
    }
}

}  // namespace rows
}  // namespace dc

using namespace dc;
using namespace dc::rows;


// Cross-entropy rows: a warp per row up to V = 1024; wider rows held in
// registers by a block per row when V % 4 == 0 (up to 16384); otherwise a
// streaming block per row.
static void ce_fwd_launch(const float *logits, const int32_t *targets, float *rows, int T, int V,
                          float eps, cudaStream_t st)
{
    const bool regs = V > 1024 && V % 4 == 0 && V <= 16384 && aligned16(logits);
    if (V <= 1024)
        (void)launch_pdl(ce_fwd_warp, dim3((T + 7) / 8), dim3(256), 0, st, 1, logits, targets,
                         rows, T, V, eps);
    else if (regs && V <= 2048)
        (void)launch_pdl(ce_fwd_regs<2>, dim3(T), dim3(256), 0, st, 1, logits, targets, rows, T,
                         V, eps);
    else if (regs && V <= 4096)
        (void)launch_pdl(ce_fwd_regs<4>, dim3(T), dim3(256), 0, st, 1, logits, targets, rows, T,
                         V, eps);
    else if (regs && V <= 8192)
        (void)launch_pdl(ce_fwd_regs<8>, dim3(T), dim3(256), 0, st, 1, logits, targets, rows, T,
                         V, eps);
    else if (regs)
        (void)launch_pdl(ce_fwd_regs<16>, dim3(T), dim3(256), 0, st, 1, logits, targets, rows, T,
                         V, eps);
    else
        (void)launch_pdl(ce_fwd_block, dim3(T), dim3(256), 0, st, 1, logits, targets, rows, T, V,
                         eps);
}

static void ce_bwd_launch(const float *logits, const int32_t *targets, const float *gscale,
                          float *dlogits, int T, int V, float eps, cudaStream_t st)
{
    const bool regs = V > 1024 && V % 4 == 0 && V <= 16384 && aligned16(logits) && aligned16(dlogits);
    if (V <= 1024)
        (void)launch_pdl(ce_bwd_warp, dim3((T + 7) / 8), dim3(256), 0, st, 1, logits, targets,
                         gscale, dlogits, T, V, eps);
    else if (regs && V <= 2048)
        (void)launch_pdl(ce_bwd_regs<2>, dim3(T), dim3(256), 0, st, 1, logits, targets, gscale,
                         dlogits, T, V, eps);
    else if (regs && V <= 4096)
        (void)launch_pdl(ce_bwd_regs<4>, dim3(T), dim3(256), 0, st, 1, logits, targets, gscale,
                         dlogits, T, V, eps);
    else if (regs && V <= 8192)
        (void)launch_pdl(ce_bwd_regs<8>, dim3(T), dim3(256), 0, st, 1, logits, targets, gscale,
                         dlogits, T, V, eps);
    else if (regs)
        (void)launch_pdl(ce_bwd_regs<16>, dim3(T), dim3(256), 0, st, 1, logits, targets, gscale,
                         dlogits, T, V, eps);
    else
        (void)launch_pdl(ce_bwd_block, dim3(T), dim3(256), 0, st, 1, logits, targets, gscale,
                         dlogits, T, V, eps);
}

extern "C" {

int dc_layernorm_fwd(const float *x, const float *gamma, const float *beta, float *y, int R,
                     int C, float eps, void *stream)
{
    clear_error();
    if (R < 0 || C < 0) return fail(DC_ERR_INVALID, "negative shape");
    if ((long long)R * C == 0) return DC_OK;
    if (!x || !gamma || !beta || !y) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(y) && aligned16(gamma) &&
                     aligned16(beta);
    const int wpb = 8;
    const unsigned grid = (unsigned)((R + wpb - 1) / wpb);
    KernelTimer kt("layernorm_fwd", st);
    if (vec && C <= 128)
        (void)launch_pdl(ln_fwd_warp<1>, dim3(grid), dim3(32 * wpb), 0, st, 1, x, gamma, beta, y,
                         R, C, eps);
    else if (vec && C <= 256)
        (void)launch_pdl(ln_fwd_warp<2>, dim3(grid), dim3(32 * wpb), 0, st, 1, x, gamma, beta, y,
                         R, C, eps);
    else if (vec && C <= 512)
        (void)launch_pdl(ln_fwd_warp<4>, dim3(grid), dim3(32 * wpb), 0, st, 1, x, gamma, beta, y,
                         R, C, eps);
    else if (vec && C <= 1024)
        (void)launch_pdl(ln_fwd_warp<8>, dim3(grid), dim3(32 * wpb), 0, st, 1, x, gamma, beta, y,
                         R, C, eps);
    else
        (void)launch_pdl(ln_fwd_block, dim3(R), dim3(256), 0, st, 1, x, gamma, beta, y, R, C, eps);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_layernorm_bwd(const float *x, const float *gamma, const float *dy, float *dx,
                     float *dgamma, float *dbeta, int R, int C, float eps, int accumulate,
                     void *stream)
{
    clear_error();
    if (R < 0 || C < 0) return fail(DC_ERR_INVALID, "negative shape");
    if ((long long)R * C == 0) return DC_OK;
    if (!x || !gamma || !dy || !dx || !dgamma || !dbeta)
        return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    const bool vec = (C % 4 == 0) && aligned16(x) && aligned16(dy) && aligned16(dx) &&
                     aligned16(gamma) && C <= 1024;
    int nparts;
    int rows_per_cta = 0;
    const int wpb = 8;
    if (vec) {
        const int target = sm_count() * 4;
        rows_per_cta = std::max(wpb, (R + target - 1) / target);
        nparts = (R + rows_per_cta - 1) / rows_per_cta;
    } else {
        nparts = R;
    }
    float *part = nullptr;
    DC_CUDA_TRY(cudaMallocAsync(&part, (size_t)nparts * 2 * C * sizeof(float), st));
    const size_t shbytes = (size_t)wpb * 2 * C * sizeof(float);
    int rc = DC_OK;
    KernelTimer kt("layernorm_bwd", st);
    if (vec) {
        if (C <= 128)
            (void)launch_pdl(ln_bwd_warp<1>, dim3(nparts), dim3(32 * wpb), shbytes, st, 1, x,
                             gamma, dy, dx, part, R, C, eps, accumulate, rows_per_cta);
        else if (C <= 256)
            (void)launch_pdl(ln_bwd_warp<2>, dim3(nparts), dim3(32 * wpb), shbytes, st, 1, x,
                             gamma, dy, dx, part, R, C, eps, accumulate, rows_per_cta);
        else if (C <= 512)
            (void)launch_pdl(ln_bwd_warp<4>, dim3(nparts), dim3(32 * wpb), shbytes, st, 1, x,
                             gamma, dy, dx, part, R, C, eps, accumulate, rows_per_cta);
        else {
            // idempotent: concurrent first calls may both set it
            cudaFuncSetAttribute(ln_bwd_warp<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)shbytes);
            (void)launch_pdl(ln_bwd_warp<8>, dim3(nparts), dim3(32 * wpb), shbytes, st, 1, x,
                             gamma, dy, dx, part, R, C, eps, accumulate, rows_per_cta);
        }
    } else {
        (void)launch_pdl(ln_bwd_block, dim3(R), dim3(256), 0, st, 1, x, gamma, dy, dx, part, R, C,
                         eps, accumulate);
    }
    if (cudaGetLastError() != cudaSuccess) rc = fail(DC_ERR_CUDA, "layernorm bwd launch failed");
    if (rc == DC_OK) {
        (void)launch_pdl(colsum_parts, dim3((2 * C + 31) / 32), dim3(32, kColLanes), 0, st, 1, part,
                         nparts, 2 * C, dgamma, dbeta, C, accumulate);
        if (cudaGetLastError() != cudaSuccess)
            rc = fail(DC_ERR_CUDA, "layernorm colsum launch failed");
    }
    cudaFreeAsync(part, st);
    return rc;
}

int dc_bias_fwd(const float *a, const float *b, float *out, int M, int N, void *stream)
{
    clear_error();
    if (M < 0 || N < 0) return fail(DC_ERR_INVALID, "negative shape");
    if ((long long)M * N == 0) return DC_OK;
    if (!a || !b || !out) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    const size_t n = (size_t)M * N;
    const int blocks = (int)std::min<size_t>((n + 1023) / 1024, (size_t)sm_count() * 8);
    KernelTimer kt("bias_fwd", st);
    if (N % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out))
        (void)launch_pdl(bias_fwd_vec, dim3(blocks), dim3(256), 0, st, 1, (const float4 *)a,
                         (const float4 *)b, (float4 *)out, n / 4, N / 4);
    else
        (void)launch_pdl(bias_fwd_scalar, dim3(blocks), dim3(256), 0, st, 1, a, b, out, n, N);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_bias_bwd(const float *dy, float *da, float *db, int M, int N, int accumulate,
                void *stream)
{
    clear_error();
    if (M < 0 || N < 0) return fail(DC_ERR_INVALID, "negative shape");
    if ((long long)M * N == 0) return DC_OK;
    if (!dy || !db) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    const bool vec = N % 4 == 0 && aligned16(dy) && (!da || aligned16(da));
    // tall matrices of at most 1024 columns: the row-contiguous form (whole
    // rows per CTA; its partial sums and the finishing count in a scratch of
    // the stream-ordered allocator).  From 131072 rows on: below, the last
    // CTA's serial sum of the partials outweighs the streaming gain (the
    // decoder's [16384, 256..1024] gradients ran 309 -> 516 us a step)
    if (vec && N <= 1024 && M >= 131072) {
        const int N4 = N / 4, lanes = kSumThreads / N4;
        const int grid = std::max(1, std::min(2 * sm_count(), (M + 4 * lanes - 1) / (4 * lanes)));
        char *scratch = nullptr;
        const size_t pbytes = (size_t)grid * N * sizeof(float);
        DC_CUDA_TRY(cudaMallocAsync(&scratch, pbytes + 256, st));
        unsigned *done = reinterpret_cast<unsigned *>(scratch + round_up((int64_t)pbytes, 256));
        cudaError_t e = cudaMemsetAsync(done, 0, sizeof(unsigned), st);
        if (e == cudaSuccess) {
            KernelTimer kt("bias_bwd", st);
            e = launch_pdl(bias_bwd_rows, dim3(grid), dim3(kSumThreads), 0, st, 1,
                           reinterpret_cast<const float4 *>(dy), reinterpret_cast<float4 *>(da), db,
                           reinterpret_cast<float4 *>(scratch), done, M, N4, accumulate);
        }
        cudaFreeAsync(scratch, st);
        if (e != cudaSuccess) return fail(DC_ERR_CUDA, "bias bwd: %s", cudaGetErrorString(e));
        return DC_OK;
    }
    // one-launch cluster form when its CTAs (a cluster per 16 columns) fill
    // at least half the SMs
    const int nb16 = (N + 15) / 16;
    if (vec && 2 * nb16 * kSumCluster >= sm_count() && nb16 <= 65535) {
        KernelTimer kt("bias_bwd", st);
        {
            DC_CUDA_TRY(launch_pdl(bias_bwd_cluster<4, kSumCluster>, dim3(kSumCluster, nb16),
                                   dim3(kSumThreads), 0, st, kSumCluster, reinterpret_cast<const float4 *>(dy),
                                   reinterpret_cast<float4 *>(da), db, M, N / 4, accumulate));
        }
        return DC_OK;
    }
    const int cblocks = vec ? (N / 4 + 31) / 32 : (N + 31) / 32;
    const int target = std::max(1, sm_count() * 8 / cblocks);
    const int rows_per_cta = std::max(16, (M + target - 1) / target);
    const int rblocks = (M + rows_per_cta - 1) / rows_per_cta;
    float *part = nullptr;
    DC_CUDA_TRY(cudaMallocAsync(&part, (size_t)rblocks * N * sizeof(float), st));
    KernelTimer kt("bias_bwd", st);
    if (vec)
        (void)launch_pdl(bias_bwd_vec4, dim3(cblocks, rblocks), dim3(32, 8), 0, st, 1,
                         reinterpret_cast<const float4 *>(dy), reinterpret_cast<float4 *>(da),
                         part, M, N / 4, rows_per_cta, accumulate);
    else
        (void)launch_pdl(bias_bwd_kernel, dim3(cblocks, rblocks), dim3(32, 8), 0, st, 1, dy, da,
                         part, M, N, rows_per_cta, accumulate);
    (void)launch_pdl(colsum_parts, dim3((N + 31) / 32), dim3(32, kColLanes), 0, st, 1, part, rblocks, N,
                     db, db, N, accumulate);
    cudaError_t e = cudaGetLastError();
    cudaFreeAsync(part, st);
    if (e != cudaSuccess) return fail(DC_ERR_CUDA, "bias bwd: %s", cudaGetErrorString(e));
    return DC_OK;
}

int dc_ce_fwd(const float *logits, const int32_t *targets, float *loss, float *row_loss, int T,
              int V, float eps, void *stream)
{
    clear_error();
    if (T < 0 || V <= 0) return fail(DC_ERR_INVALID, "bad shape T=%d V=%d", T, V);
    if (T == 0) return DC_OK;
    if (!logits || !targets || !loss) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    float *rows = row_loss;
    if (!rows) DC_CUDA_TRY(cudaMallocAsync(&rows, (size_t)T * sizeof(float), st));
    KernelTimer kt("ce_fwd", st);
    ce_fwd_launch(logits, targets, rows, T, V, eps, st);
    (void)launch_pdl(mean_kernel, dim3(1), dim3(1024), 0, st, 1, rows, T, loss);
    cudaError_t e = cudaGetLastError();
    if (!row_loss) cudaFreeAsync(rows, st);
    if (e != cudaSuccess) return fail(DC_ERR_CUDA, "ce fwd: %s", cudaGetErrorString(e));
    return DC_OK;
}

// ---------------------------------------------------------------------------
// Cross-entropy forward for callers that must not allocate device memory.
//
// dc_ce_fwd needs T floats of scratch for the per-row losses before it
// reduces them to the mean; without a caller buffer it takes them from the
// stream-ordered allocator.  Some callers cannot allow any allocation inside
// the loss call: a host runtime that owns all device memory up front and
// forbids the library from allocating, or a step that must never wait on or
// grow the allocator pool.  This entry point keeps the per-row losses in a
// fixed array compiled into the library instead.
//
// Limit: T <= DC_CE_NOALLOC_MAX_ROWS (65536 rows, 256 KiB per GPU).  The array
// exists on every GPU that loads the library and stays resident until the
// process exits.  It is shared by every call on a device and holds the last
// call's row losses; each call overwrites all T entries it reads, so nothing
// needs clearing, but calls that overlap on the GPU (other streams, other
// host threads) race on it and must be serialised by the caller.  Calls
// queued back to back on one stream are ordered: every kernel of a call waits
// for the previous kernel on the stream to finish before it touches memory.
// The first call on each device looks the array's device address up (the
// host-side symbol is only a stand-in for it) and caches it; make that first
// call before any stream capture.  The cache does not survive a device reset:
// after cudaDeviceReset the module is loaded again and the array may move, so
// a process that resets a device must not call this entry point afterwards.
// ---------------------------------------------------------------------------
#define DC_CE_NOALLOC_MAX_ROWS 65536

static __device__ __align__(256) float g_ce_noalloc_rows[DC_CE_NOALLOC_MAX_ROWS];

static float *ce_noalloc_rows_ptr()
{
    static float *ptrs[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_ce_noalloc_rows) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<float *>(p);
    }
    return ptrs[dev];
}

int dc_ce_fwd_noalloc(const float *logits, const int32_t *targets, float *loss, int T, int V,
                      float eps, void *stream)
{
    clear_error();
    if (T < 0 || V <= 0) return fail(DC_ERR_INVALID, "bad shape T=%d V=%d", T, V);
    if (T > DC_CE_NOALLOC_MAX_ROWS)
        return fail(DC_ERR_INVALID, "dc_ce_fwd_noalloc: T=%d rows exceeds the fixed scratch of %d rows",
                    T, DC_CE_NOALLOC_MAX_ROWS);
    if (T == 0) return DC_OK;
    if (!logits || !targets || !loss) return fail(DC_ERR_INVALID, "null pointer");
    float *rows = ce_noalloc_rows_ptr();
    if (!rows) return fail(DC_ERR_CUDA, "dc_ce_fwd_noalloc: cannot resolve the scratch array address");
    cudaStream_t st = as_stream(stream);
    ce_fwd_launch(logits, targets, rows, T, V, eps, st);
    (void)launch_pdl(mean_kernel, dim3(1), dim3(1024), 0, st, 1, rows, T, loss);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DC_ERR_CUDA, "ce fwd noalloc: %s", cudaGetErrorString(e));
    return DC_OK;
}

int dc_ce_bwd(const float *logits, const int32_t *targets, const float *grad_scale,
              float *dlogits, int T, int V, float eps, void *stream)
{
    clear_error();
    if (T < 0 || V <= 0) return fail(DC_ERR_INVALID, "bad shape T=%d V=%d", T, V);
    if (T == 0) return DC_OK;
    if (!logits || !targets || !dlogits) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("ce_bwd", st);
    ce_bwd_launch(logits, targets, grad_scale, dlogits, T, V, eps, st);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_adam_step(float *p, const float *g, float *m, float *v, int64_t n, int t, float lr,
                 float b1, float b2, float eps, float weight_decay, void *stream)
{
    clear_error();
    if (n < 0) return fail(DC_ERR_INVALID, "negative size");
    if (n == 0) return DC_OK;
    if (!p || !g || !m || !v) return fail(DC_ERR_INVALID, "null pointer");
    const float step = (float)t + 1.0f;
    const float c1 = 1.0f - powf(b1, step), c2 = 1.0f - powf(b2, step);
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
    KernelTimer kt("adam", as_stream(stream));
    (void)launch_pdl(adam_kernel, dim3(blocks), dim3(256), 0, as_stream(stream), 1, p, g, m, v, n,
                     lr, b1, b2, eps, weight_decay, c1, c2);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

}  // extern "C"
