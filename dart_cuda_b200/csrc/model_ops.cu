// Element-wise and gather kernels of the AFT decoder step around the dense
// layers and the AFT operator:
//
//   embedding   x[b,t,:] = wte[idx[b,t],:] + wpe[t,:]
//               (reference embedding_fwd / embedding_bwd,
//                native/src/kernels/layernorm_embed.cuh:242-269)
//   gate        z = sigmoid(q) * v0: the AFT cross-attention against a single
//               encoder row (native/src/kernels/attention.cuh:41-128 with
//               TEnc = 1), where the one weight e^{k+w} cancels and
//               Z = sigmoid(Q) * V exactly; the decoder's dummy [1, D]
//               encoder (lib/core/transformers/aft/transformer_decoder_block.dart:63-67)
//   greedy      next token = argmax of a logits row, fused with the embedding
//               of that token at the next position
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "dc_internal.h"
#include "dc_ptx.cuh"

namespace dc {
namespace model {

constexpr int DC_DEVERR_INDEX = 0x20;  // a token id outside [0, V)

__global__ void embed_fwd_kernel(const int32_t *__restrict__ idx, const float *__restrict__ wte,
                                 const float *__restrict__ wpe, float *__restrict__ out, int T,
                                 int D, int V, int *status)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int row = blockIdx.x;  // b*T + t
    const int t = row % T;
    const int tok = idx[row];
    const bool ok = tok >= 0 && tok < V;
    if (!ok && threadIdx.x == 0) atomicOr(status, DC_DEVERR_INDEX);
    const float *e = wte + (size_t)(ok ? tok : 0) * D;
    const float *p = wpe + (size_t)t * D;
    float *o = out + (size_t)row * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) o[d] = ok ? e[d] + p[d] : 0.f;
}

// dwte[idx] += dx rows (atomics: several rows may share a token);
// dwpe[t] += sum_b dx[b, t] (one thread per (t, d), no atomics).
__global__ void embed_bwd_tok_kernel(const int32_t *__restrict__ idx, const float *__restrict__ dx,
                                     float *__restrict__ dwte, int D, int V)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int row = blockIdx.x;
    const int tok = idx[row];
    if (tok < 0 || tok >= V) return;
    const float *g = dx + (size_t)row * D;
    float *dst = dwte + (size_t)tok * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) atomicAdd(dst + d, g[d]);
}

__global__ void embed_bwd_pos_kernel(const float *__restrict__ dx, float *__restrict__ dwpe, int B,
                                     int T, int D)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)T * D) return;
    const int t = (int)(i / D), d = (int)(i % D);
    float s = 0.f;
    for (int b = 0; b < B; ++b) s += dx[((size_t)b * T + t) * D + d];
    dwpe[i] += s;
}

__device__ __forceinline__ float sigm(float q) { return 1.0f / (1.0f + __expf(-q)); }

__global__ void gate_fwd_kernel(const float *__restrict__ q, int ldq, const float *__restrict__ v0,
                                float *__restrict__ out, int ldo, int M, int N)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * N) return;
    const int m = (int)(i / N), n = (int)(i % N);
    out[(size_t)m * ldo + n] = sigm(q[(size_t)m * ldq + n]) * v0[n];
}

// 16-byte form (N, ldq, ldo multiples of 4, aligned bases): 32 float4
// columns x 8 row lanes a block, four rows in flight per thread.
__device__ __forceinline__ float4 sigm4(float4 q)
{
    return make_float4(sigm(q.x), sigm(q.y), sigm(q.z), sigm(q.w));
}

__global__ void gate_fwd_vec(const float4 *__restrict__ q, int ldq4, const float4 *__restrict__ v0,
                             float4 *__restrict__ out, int ldo4, int M, int N4)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    const int c = blockIdx.x * 32 + (threadIdx.x & 31);
    if (c >= N4) return;
    const float4 v = v0[c];
    const int step = gridDim.y * 8;
    int m = blockIdx.y * 8 + (threadIdx.x >> 5);
    for (; m + 3 * step < M; m += 4 * step) {
        float4 x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = __ldcs(q + (size_t)(m + k * step) * ldq4 + c);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float4 s = sigm4(x[k]);
            out[(size_t)(m + k * step) * ldo4 + c] = make_float4(s.x * v.x, s.y * v.y, s.z * v.z, s.w * v.w);
        }
    }
    for (; m < M; m += step) {
        const float4 s = sigm4(__ldcs(q + (size_t)m * ldq4 + c));
        out[(size_t)m * ldo4 + c] = make_float4(s.x * v.x, s.y * v.y, s.z * v.z, s.w * v.w);
    }
}

__global__ void gate_bwd_vec(const float4 *__restrict__ q, int ldq4, const float4 *__restrict__ v0,
                             const float4 *__restrict__ dz, int ldz4, float4 *__restrict__ dq,
                             int lddq4, float *__restrict__ dv0, int M, int N4)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float4 part[8][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + tx;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < N4) {
        const float4 v = v0[c];
        const int step = gridDim.y * 8;
        int m = blockIdx.y * 8 + ty;
        auto one = [&](const float4 x, const float4 g, size_t o) {
            const float4 s = sigm4(x);
            dq[o] = make_float4(g.x * v.x * s.x * (1.0f - s.x), g.y * v.y * s.y * (1.0f - s.y),
                                g.z * v.z * s.z * (1.0f - s.z), g.w * v.w * s.w * (1.0f - s.w));
            acc.x += g.x * s.x;
            acc.y += g.y * s.y;
            acc.z += g.z * s.z;
            acc.w += g.w * s.w;
        };
        for (; m + 3 * step < M; m += 4 * step) {
            float4 x[4], g[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                x[k] = __ldcs(q + (size_t)(m + k * step) * ldq4 + c);
                g[k] = __ldcs(dz + (size_t)(m + k * step) * ldz4 + c);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) one(x[k], g[k], (size_t)(m + k * step) * lddq4 + c);
        }
        for (; m < M; m += step)
            one(__ldcs(q + (size_t)m * ldq4 + c), __ldcs(dz + (size_t)m * ldz4 + c),
                (size_t)m * lddq4 + c);
    }
    part[ty][tx] = acc;
    __syncthreads();
    if (ty == 0 && c < N4) {
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            s.x += part[r][tx].x;
            s.y += part[r][tx].y;
            s.z += part[r][tx].z;
            s.w += part[r][tx].w;
        }
        atomicAdd(dv0 + 4 * c, s.x);
        atomicAdd(dv0 + 4 * c + 1, s.y);
        atomicAdd(dv0 + 4 * c + 2, s.z);
        atomicAdd(dv0 + 4 * c + 3, s.w);
    }
}

// dq = dz * v0 * s (1 - s); dv0 += sum_m dz * s.  Block: 32 columns x 8 row
// lanes; partial column sums meet in shared memory, one atomic per column.
__global__ void gate_bwd_kernel(const float *__restrict__ q, int ldq, const float *__restrict__ v0,
                                const float *__restrict__ dz, int ldz, float *__restrict__ dq,
                                int lddq, float *__restrict__ dv0, int M, int N, int rows_per_block)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float part[8][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int n = blockIdx.x * 32 + tx;
    const int m0 = blockIdx.y * rows_per_block, m1 = min(M, m0 + rows_per_block);
    float acc = 0.f;
    if (n < N) {
        const float v = v0[n];
        for (int m = m0 + ty; m < m1; m += 8) {
            const float s = sigm(q[(size_t)m * ldq + n]);
            const float g = dz[(size_t)m * ldz + n];
            dq[(size_t)m * lddq + n] = g * v * s * (1.0f - s);
            acc += g * s;
        }
    }
    part[ty][tx] = acc;
    __syncthreads();
    if (ty == 0 && n < N) {
        float s = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) s += part[r][tx];
        atomicAdd(dv0 + n, s);
    }
}

// One block per batch row: argmax over V logits (first index on ties) of the
// position *pos_dev, stored as the token of position p = *pos_dev + 1, then
// x[b,:] = wte[tok,:] + wpe[p,:] for the next decode step.  The position
// lives in device memory so a captured decode step replays unchanged;
// advance_kernel moves it on once every block has read it.
__global__ void greedy_embed_kernel(const float *__restrict__ logits, int ldl, int V,
                                    const float *__restrict__ wte, const float *__restrict__ wpe,
                                    const int *pos_dev, int D, int32_t *__restrict__ tokens, int ldt,
                                    float *__restrict__ x)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int pos = *pos_dev + 1;
    if (pos < 0 || pos >= ldt) return;  // sequence full: advance_kernel flags it
    const int b = blockIdx.x;
    const float *l = logits + (size_t)b * ldl;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    auto take = [&](float x_, int v) {
        if (x_ > best || (x_ == best && v < bi)) {
            best = x_;
            bi = v;
        }
    };
    if (((ldl | V) & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        // 16-byte loads, several in flight per thread
        const float4 *l4 = reinterpret_cast<const float4 *>(l);
#pragma unroll 4
        for (int v = threadIdx.x; v < V / 4; v += blockDim.x) {
            const float4 x4 = l4[v];
            take(x4.x, 4 * v);
            take(x4.y, 4 * v + 1);
            take(x4.z, 4 * v + 2);
            take(x4.w, 4 * v + 3);
        }
    } else {
        for (int v = threadIdx.x; v < V; v += blockDim.x) take(l[v], v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        best = lane < nw ? sv[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) si[0] = bi < V ? bi : 0;  // all-NaN row: token 0
    }
    __syncthreads();
    const int tok = si[0];
    if (threadIdx.x == 0) tokens[(size_t)b * ldt + pos] = tok;
    if (x) {
        const float *e = wte + (size_t)tok * D;
        const float *p = wpe + (size_t)pos * D;
        for (int d = threadIdx.x; d < D; d += blockDim.x) x[(size_t)b * D + d] = e[d] + p[d];
    }
}

constexpr int DC_DEVERR_FULL = 0x40;  // decode ran past the sequence capacity

__global__ void advance_kernel(int *pos, int cap, int *status)
{
    grid_dep_wait();  // programmatic dependent launch: inputs are ready
    grid_dep_launch();
    if (*pos + 1 >= cap) {
        atomicOr(status, DC_DEVERR_FULL);
        return;
    }
    *pos += 1;
}

}  // namespace model
}  // namespace dc

using namespace dc;
using namespace dc::model;

extern "C" {

int dc_embedding_fwd(const int32_t *idx, const float *wte, const float *wpe, float *out, int B,
                     int T, int D, int V, void *stream)
{
    clear_error();
    if (B < 0 || T < 0 || D < 0 || V <= 0) return fail(DC_ERR_INVALID, "bad shape");
    if ((long long)B * T * D == 0) return DC_OK;
    if (!idx || !wte || !wpe || !out) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("embedding_fwd", st);
    (void)launch_pdl(embed_fwd_kernel, dim3(B * T), dim3(128), 0, st, 1, idx, wte, wpe, out, T, D,
                     V, device_status_word());
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_embedding_bwd(const int32_t *idx, const float *dx, float *dwte, float *dwpe, int B, int T,
                     int D, int V, void *stream)
{
    clear_error();
    if (B < 0 || T < 0 || D < 0 || V <= 0) return fail(DC_ERR_INVALID, "bad shape");
    if ((long long)B * T * D == 0) return DC_OK;
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("embedding_bwd", st);
    if (dwte) (void)launch_pdl(embed_bwd_tok_kernel, dim3(B * T), dim3(128), 0, st, 1, idx, dx,
                               dwte, D, V);
    if (dwpe) {
        const size_t n = (size_t)T * D;
        (void)launch_pdl(embed_bwd_pos_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                         st, 1, dx, dwpe, B, T, D);
    }
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_gate_fwd(const float *q, int ldq, const float *v0, float *out, int ldo, int M, int N,
                void *stream)
{
    clear_error();
    if (M < 0 || N < 0 || ldq < N || ldo < N) return fail(DC_ERR_INVALID, "bad shape");
    if ((long long)M * N == 0) return DC_OK;
    cudaStream_t st = as_stream(stream);
    const size_t n = (size_t)M * N;
    KernelTimer kt("gate_fwd", st);
    if (N % 4 == 0 && ldq % 4 == 0 && ldo % 4 == 0 && aligned16(q) && aligned16(v0) && aligned16(out)) {
        // one row a thread for short inputs (the decode step's 64 rows are
        // latency-bound), up to eight blocks an SM for long ones
        const int cb = (N / 4 + 31) / 32;
        const int rb = std::max(1, std::min((M + 7) / 8, (8 * sm_count() + cb - 1) / cb));
        DC_CUDA_TRY(launch_pdl(gate_fwd_vec, dim3(cb, rb), dim3(256), 0, st, 1, (const float4 *)q,
                               ldq / 4, (const float4 *)v0, (float4 *)out, ldo / 4, M, N / 4));
        return DC_OK;
    }
    (void)launch_pdl(gate_fwd_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, 1, q,
                     ldq, v0, out, ldo, M, N);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_gate_bwd(const float *q, int ldq, const float *v0, const float *dz, int ldz, float *dq,
                int lddq, float *dv0, int M, int N, void *stream)
{
    clear_error();
    if (M < 0 || N < 0 || ldq < N || ldz < N || lddq < N) return fail(DC_ERR_INVALID, "bad shape");
    if ((long long)M * N == 0) return DC_OK;
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("gate_bwd", st);
    if (N % 4 == 0 && ldq % 4 == 0 && ldz % 4 == 0 && lddq % 4 == 0 && aligned16(q) &&
        aligned16(v0) && aligned16(dz) && aligned16(dq)) {
        // two blocks an SM: eight 16-byte loads in flight per thread suffice,
        // and fewer blocks mean fewer atomics on each dv0 column
        const int cb4 = (N / 4 + 31) / 32;
        const int rb = std::max(1, std::min((M + 31) / 32, (2 * sm_count() + cb4 - 1) / cb4));
        DC_CUDA_TRY(launch_pdl(gate_bwd_vec, dim3(cb4, rb), dim3(256), 0, st, 1, (const float4 *)q,
                               ldq / 4, (const float4 *)v0, (const float4 *)dz, ldz / 4,
                               (float4 *)dq, lddq / 4, dv0, M, N / 4));
        return DC_OK;
    }
    const int cb = (N + 31) / 32;
    int rsplit = std::max(1, std::min((M + 63) / 64, (4 * sm_count() + cb - 1) / cb));
    const int rows = (M + rsplit - 1) / rsplit;
    rsplit = (M + rows - 1) / rows;
    (void)launch_pdl(gate_bwd_kernel, dim3(cb, rsplit), dim3(256), 0, st, 1, q, ldq, v0, dz, ldz,
                     dq, lddq, dv0, M, N, rows);
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_greedy_embed(const float *logits, int ldl, int B, int V, const float *wte,
                    const float *wpe, int *pos, int D, int32_t *tokens, int ldt, float *x,
                    void *stream)
{
    clear_error();
    if (B < 0 || V <= 0 || ldl < V || ldt <= 0 || !pos) return fail(DC_ERR_INVALID, "bad shape");
    if (B == 0) return DC_OK;
    if (x && (!wte || !wpe || D <= 0)) return fail(DC_ERR_INVALID, "embedding tables needed");
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("greedy_embed", st);
    (void)launch_pdl(greedy_embed_kernel, dim3(B), dim3(256), 0, st, 1, logits, ldl, V, wte, wpe,
                     pos, D, tokens, ldt, x);
    (void)launch_pdl(advance_kernel, dim3(1), dim3(1), 0, st, 1, pos, ldt, device_status_word());
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_copy2d(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t width_bytes,
              size_t rows, void *stream)
{
    clear_error();
    if (rows == 0 || width_bytes == 0) return DC_OK;
    DC_CUDA_TRY(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, rows,
                                  cudaMemcpyDeviceToDevice, as_stream(stream)));
    return DC_OK;
}

}  // extern "C"
