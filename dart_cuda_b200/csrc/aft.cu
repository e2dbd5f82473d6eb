// AFT-full forward and backward on sm_100a.
//
// The reference computes, per (t, d), a joint-max-stabilised softmax-like
// weighted sum over i <= t with one CUDA thread per query row
// (native/src/kernels/attention.cuh:6-40, native/src/engine.cu:522-590).
// Here the same operator is factorised into dense contractions that run on
// the 5th-generation tensor cores:
//
//   m_t  = max_{i in S(t)} w[t,i]            c_{b,d} = max_i K[b,i,d]
//   A'   = [i in S(t)] * exp(w - m)  (Tq x Tk, shared by the batch)
//   E'   = exp(K - c);  PV = E' * V;  PE = E'          ([B, Tk, D] each)
//   num' = A' PV, den' = A' PE,  r = num'/den',  Z = sigmoid(Q) * r
//
// The scale factors e^{m_t} and e^{c_{b,d}} cancel exactly in r and in every
// gradient, so the result equals the reference's up to rounding.  Backward:
//
//   g = dZ*sigmoid(Q)/den',  n = -g*r,  dQ = dZ*r*sigmoid(Q)*(1-sigmoid(Q))
//   H1 = A'^T g, H2 = A'^T n          ->  dV = E'*H1,  dK = E'*(V*H1 + H2)
//   dW = A' (.) sum_b (g_b PV_b^T + n_b PE_b^T)
//
// Four tcgen05 contraction modes share one persistent, warp-specialised
// kernel (aft_tc.cuh):
//   FWD   : acc[t, d] = sum_i A'[t,i] PV[i,d]  (and PE)  -> Z
//   BWD1  : same contraction                             -> dQ, g, n
//   HGRAD : acc[i, d] = sum_t A'[t,i] G[t,d]   (and N)   -> dK, dV
//   WGRAD : acc[t, i] = sum_{b,d} G[b,t,d] P[b,i,d]      -> dW (split-K, atomics)
// Operands are staged by TMA into 128-byte-swizzled shared memory; one thread
// issues the MMAs into double-buffered TMEM accumulators; twelve warps read
// TMEM back and apply the element-wise epilogue with 32-byte accesses.
#include <cuda_bf16.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <initializer_list>

#include "dc_internal.h"
#include "dc_ptx.cuh"

namespace dc {
namespace aft {

constexpr int BM = 128;        // accumulator rows = TMEM lanes
constexpr int BN = 128;        // accumulator columns (one accumulator)
constexpr int T_ALIGN = 128;   // workspace padding of Tq and Tk (tf32 operands)
constexpr int T_ALIGN2 = 256;  // ... with bf16 operands: CTA pairs cover 256 rows
constexpr int D_ALIGN = 128;   // workspace padding of D (64 for narrow heads, make_layout)

enum Mode { FWD = 0, BWD1 = 1, HGRAD = 2, WGRAD = 3 };

// ------------------------------------------------------------ element I/O
__device__ __forceinline__ float ld_io(const float *p, size_t i) { return p[i]; }
__device__ __forceinline__ float ld_io(const __nv_bfloat16 *p, size_t i)
{
    return __bfloat162float(p[i]);
}
__device__ __forceinline__ void st_io(float *p, size_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st_io(__nv_bfloat16 *p, size_t i, float v)
{
    p[i] = __float2bfloat16_rn(v);
}

// operand precision: bf16, or fp32 rounded to tf32 (round-to-nearest-away)
template <class E> __device__ __forceinline__ E to_op(float v);
template <> __device__ __forceinline__ __nv_bfloat16 to_op<__nv_bfloat16>(float v)
{
    return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ float to_op<float>(float v)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}
__device__ __forceinline__ float from_op(float v) { return v; }
__device__ __forceinline__ float from_op(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float sigmoidf_(float q) { return 1.0f / (1.0f + __expf(-q)); }

// ------------------------------------------------------------ parameters
struct Params {
    int B, Tq, Tk, D, Tqp, Tkp, dp;
    int causal, accumulate;
    int ldi;          // row stride of Q, K, V, dQ, dK, dV (elements, >= D)
    int ldo;          // row stride of Z and dZ (elements, >= D)
    int n_tiles;      // tensor-core path: number of output tiles of the launch
    int kpb;          // WGRAD: K steps per batch element (dp / BKe)
    int narrow;       // dp = 64 < BN: every FWD/BWD1/HGRAD tile is a half tile (half 0)
    int bundled;      // FWD/BWD1/HGRAD: tiles dealt in equal-work bundles of two
    int n_full;       // FWD/BWD1/HGRAD without bundles: units before the half tiles
    int zero_dw;      // BWD1 / saved-statistics kernel: also zero dW[Tq][Tk] (stride ldw)
    int splits;       // WGRAD: split-K factor
    int sk_tiles;     // WGRAD: dW tiles
    int sk_lo;        // WGRAD: leading tiles that also run a low-part pass
    int vec_io;       // user tensors allow 32-byte vector access along D
    int vec_w;        // w / dW allow 32-byte vector access along a row
    int spare_sms;    // host only: SMs the persistent launch leaves free
    const void *Q, *K, *V, *dZ;
    void *Z, *dQ, *dK, *dV;
    float *dW;
    const float *w;
    int ldw;
    const float *m;   // [Tqp]
    const float *c;   // [B][dp]
    void *G1, *G2;    // g and n = -g*r, [B][Tqp][dp] operand precision
    void *G1l, *G2l;  // their rounding residuals (g - G1, n - G2), same layout
    int lo_rows;      // the residuals exist for query rows t < lo_rows (multiple of 128)
    // forward statistics r = num/den and 1/den (Rs == nullptr: not kept):
    // fp32 [B][stat_lo][dp] for query rows t < stat_lo (= lo_rows, where the
    // backward keeps g and n to better than operand precision), operand
    // precision [B][Tqp][dp] (Rb, Ib; rows from stat_lo on) for the rest
    float *Rs, *Is;
    void *Rb, *Ib;
    int stat_lo;
    int dw_packed;    // dW in the block-packed causal layout (dw_packed_row)
    int *status;
    unsigned long long *trace;  // optional per-tile timeline (nullptr: off)
#ifdef DC_TEST_WITHHOLD
    int test_withhold;  // test build only: CTA 0 skips its first stage's load
#endif
};

#ifdef DC_TEST_WITHHOLD
// Test build only (the library built with -DDC_TEST_WITHHOLD and a short
// DC_WAIT_NS, never the product library): dc_test_withhold_next(1) makes the
// next tensor-core launch's CTA 0 skip the TMA load and the arrival of its
// first pipeline stage, so the MMA issuer's bounded wait for that stage runs
// out and the abort path (status bit, drains, TMEM release) is exercised.
static int g_test_withhold = 0;
#endif

// Test hook: the two-launch prep (prep_wc_kernel + prep_p_kernel) instead of
// the one-launch clustered prep, to cross-check the two (dc_aft_prep_mode).
static int g_prep_two_launch = 0;

// Per-tile timeline of the tensor-core launches whose mode bit is set in
// g_trace_modes (bit MODE); see trace_at() in aft_tc.cuh.
static unsigned long long *g_trace_buf = nullptr;
static int g_trace_modes = 0;

// ------------------------------------------------------------ packed dW
// Block-packed causal dW (DC_AFT_DW_PACKED): query rows in blocks of 256;
// block k holds its rows' causal extent only, min(Tk8, 256 (k + 1)) columns
// (Tk8 = Tk rounded up to 8), row after row, so every row starts 32-byte
// aligned and the blocks before k (all of full width) take 256^2 k(k+1)/2
// floats.  At T = 4096 that is 53% of the full matrix: the data-parallel
// all-reduce of dW moves half the bytes (the upper triangle is zero on every
// rank).
constexpr int kDwBlock = 256;

__host__ __device__ __forceinline__ size_t dw_packed_width(int t, int Tk)
{
    const size_t k = (size_t)t / kDwBlock, tk8 = ((size_t)Tk + 7) & ~(size_t)7;
    const size_t full = (k + 1) * kDwBlock;
    return full < tk8 ? full : tk8;
}

__host__ __device__ __forceinline__ size_t dw_packed_row(int t, int Tk)
{
    const size_t k = (size_t)t / kDwBlock;
    return (size_t)kDwBlock * kDwBlock * k * (k + 1) / 2 + ((size_t)t - k * kDwBlock) * dw_packed_width(t, Tk);
}

__host__ __device__ __forceinline__ size_t dw_packed_floats(int Tq, int Tk)
{
    return Tq > 0 ? dw_packed_row(Tq - 1, Tk) + dw_packed_width(Tq - 1, Tk) : 0;
}

// start of dW's row t in the caller's layout
__device__ __forceinline__ float *dw_row(const Params &p, int t)
{
    return p.dW + (p.dw_packed ? dw_packed_row(t, p.Tk) : (size_t)t * p.ldw);
}

// ------------------------------------------------------------ epilogues
// Shared by the tensor-core and CUDA-core paths so both apply identical
// element-wise maths to the contraction results.
template <class IO>
__device__ __forceinline__ void epi_fwd(const Params &p, int b, int t, int d, float num,
                                        float den)
{
    if (t < p.Tq && d < p.D) {
        const size_t row = (size_t)b * p.Tq + t;
        float s = sigmoidf_(ld_io((const IO *)p.Q, row * p.ldi + d));
        st_io((IO *)p.Z, row * p.ldo + d, s * (num / den));
        if (p.status && (!(den >= 0x1p-100f) || !(fabsf(num) <= 3.0e38f))) atomicOr(p.status, DC_DEVERR_RANGE);
    }
}

template <class IO, class E>
__device__ __forceinline__ void epi_bwd1(const Params &p, int b, int t, int d, float num,
                                         float den)
{
    float g = 0.f, n = 0.f;
    if (t < p.Tq && d < p.D) {
        const size_t row = (size_t)b * p.Tq + t;
        const size_t o = row * p.ldi + d;
        float s = sigmoidf_(ld_io((const IO *)p.Q, o));
        float dz = ld_io((const IO *)p.dZ, row * p.ldo + d);
        float r = num / den;
        if (p.status && (!(den >= 0x1p-100f) || !(fabsf(num) <= 3.0e38f))) atomicOr(p.status, DC_DEVERR_RANGE);
        float dq = dz * r * s * (1.0f - s);
        if (p.accumulate) dq += ld_io((const IO *)p.dQ, o);
        st_io((IO *)p.dQ, o, dq);
        g = dz * s / den;
        n = -g * r;
    }
    // hi/lo split: the dW contraction sums g*E'V + n*E' over d, which cancel
    // where V ~ r; rounding g and n alone would leave an error of the
    // operand precision times |g E' V| there, so the residuals are kept too.
    size_t go = ((size_t)b * p.Tqp + t) * p.dp + d;
    const E gh = to_op<E>(g), nh = to_op<E>(n);
    ((E *)p.G1)[go] = gh;
    ((E *)p.G2)[go] = nh;
    ((E *)p.G1l)[go] = to_op<E>(g - from_op(gh));
    ((E *)p.G2l)[go] = to_op<E>(n - from_op(nh));
}

template <class IO>
__device__ __forceinline__ void epi_hgrad(const Params &p, int b, int i, int d, float h1,
                                          float h2)
{
    if (i < p.Tk && d < p.D) {
        const size_t o = ((size_t)b * p.Tk + i) * p.ldi + d;
        float e = __expf(ld_io((const IO *)p.K, o) - p.c[(size_t)b * p.dp + d]);
        float v = ld_io((const IO *)p.V, o);
        float dv = e * h1;
        float dk = e * (v * h1 + h2);
        if (p.accumulate) {
            dv += ld_io((const IO *)p.dV, o);
            dk += ld_io((const IO *)p.dK, o);
        }
        st_io((IO *)p.dV, o, dv);
        st_io((IO *)p.dK, o, dk);
    }
}

__device__ __forceinline__ void epi_wgrad(const Params &p, int t, int i, float acc)
{
    if (t < p.Tq && i < p.Tk && (!p.causal || i <= t)) {
        float a = __expf(p.w[(size_t)t * p.ldw + i] - p.m[t]);
        atomicAdd(dw_row(p, t) + i, a * acc);
    }
}

// ------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float block_max(float v, float *red)
{
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0) red[wid] = v;
    __syncthreads();
    int nw = (blockDim.x + 31) >> 5;
    v = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : -INFINITY;
    if (wid == 0) v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
    __syncthreads();
    v = red[0];
    __syncthreads();
    return v;
}

// ------------------------------------------------------------ prep kernels
// Eight operand-precision values, one 16-byte (bf16) or two (tf32) stores.
__device__ __forceinline__ void st8op(__nv_bfloat16 *p, const float (&v)[8])
{
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)  // paired conversions, v[2k] in the low half
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w[k]) : "f"(v[2 * k + 1]), "f"(v[2 * k]));
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void st8op(float *p, const float (&v)[8])
{
    float4 a, b;
    a.x = to_op<float>(v[0]); a.y = to_op<float>(v[1]); a.z = to_op<float>(v[2]); a.w = to_op<float>(v[3]);
    b.x = to_op<float>(v[4]); b.y = to_op<float>(v[5]); b.z = to_op<float>(v[6]); b.w = to_op<float>(v[7]);
    reinterpret_cast<float4 *>(p)[0] = a;
    reinterpret_cast<float4 *>(p)[1] = b;
}

// Row maxima m_t over the visible set and A' = exp(w - m) (0 outside the
// set and in the padding), one warp per padded row t.
template <class E>
__device__ __forceinline__ void prep_w_row(int t, int lane, const float *__restrict__ w, int ldw,
                                           int Tq, int Tk, int Tkp, int causal,
                                           float *__restrict__ m, E *__restrict__ Ap)
{
    E *row = Ap + (size_t)t * Tkp;
    const int lim = t < Tq ? (causal ? min(t + 1, Tk) : Tk) : 0;
    const float *wr = w + (size_t)t * ldw;
    // 16-byte loads when a row starts on a 16-byte boundary (ldw % 4 == 0):
    // a float4 at a multiple of 4 below lim then stays inside the row
    const bool vec = (ldw % 4 == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
    float mx = -INFINITY;
    if (vec) {
        for (int i = lane * 4; i < lim; i += 128) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(wr + i));
            mx = fmaxf(mx, v.x);
            if (i + 1 < lim) mx = fmaxf(mx, v.y);
            if (i + 2 < lim) mx = fmaxf(mx, v.z);
            if (i + 3 < lim) mx = fmaxf(mx, v.w);
        }
    } else {
        for (int i = lane; i < lim; i += 32) mx = fmaxf(mx, wr[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) m[t] = t < Tq ? mx : 0.f;
    // eight A' entries per lane and step, one vector store (Tkp is a multiple of 8)
    for (int i = lane * 8; i < Tkp; i += 256) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
        if (i < lim) {
            if (vec) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(wr + i));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                if (i + 4 < lim) {
                    const float4 b = __ldg(reinterpret_cast<const float4 *>(wr + i + 4));
                    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (i + k < lim) v[k] = wr[i + k];
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = i + k < lim ? __expf(v[k] - mx) : 0.f;
        }
        st8op(row + i, v);
    }
}

// Partial column maxima of K over row slices: cpart[s][b][d].  Block of
// 32 x 8 threads: each thread owns 8 consecutive columns (one 16-byte load
// for bf16) and every 8th row of the slice; the 8 row lanes then combine.
__device__ __forceinline__ void ld8(const float *p, float (&v)[8])
{
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void ld8(const __nv_bfloat16 *p, float (&v)[8])
{
    const uint4 x = __ldg(reinterpret_cast<const uint4 *>(p));
    v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xFFFF0000u);
    v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xFFFF0000u);
    v[4] = __uint_as_float(x.z << 16); v[5] = __uint_as_float(x.z & 0xFFFF0000u);
    v[6] = __uint_as_float(x.w << 16); v[7] = __uint_as_float(x.w & 0xFFFF0000u);
}

template <class IO>
__device__ __forceinline__ void prep_colmax_block(int bx, int s, int b, const IO *__restrict__ K,
                                                  int B, int Tk, int D, int ldk, int dp,
                                                  int rows_per_split, int vec,
                                                  float *__restrict__ cpart)
{
    __shared__ float red[8][32 * 8 + 1];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int d0 = (bx * 32 + tx) * 8;
    const int i0 = s * rows_per_split, i1 = min(Tk, i0 + rows_per_split);
    const IO *Kb = K + (size_t)b * Tk * ldk;
    float mx[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
    if (vec && d0 + 8 <= D) {
        for (int i = i0 + ty; i < i1; i += 8) {
            float v[8];
            ld8(Kb + (size_t)i * ldk + d0, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], v[k]);
        }
    } else if (d0 < D) {
        for (int i = i0 + ty; i < i1; i += 8)
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (d0 + k < D) mx[k] = fmaxf(mx[k], ld_io(Kb, (size_t)i * ldk + d0 + k));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) red[ty][tx * 8 + k] = mx[k];
    __syncthreads();
    // 256 threads finish 256 columns: column j = threadIdx.x of this block
    const int j = threadIdx.x;
    float m = red[0][j];
#pragma unroll
    for (int r = 1; r < 8; ++r) m = fmaxf(m, red[r][j]);
    const int d = bx * 256 + j;
    if (d < D) cpart[((size_t)s * B + b) * dp + d] = m;
}

// First prep launch: blocks [0, Tqp/8) build the rows of A' and m; the
// remaining blocks compute the partial column maxima of K (ncb column blocks
// of 256 x nsplit row slices x B).
template <class IO, class E>
__global__ void __launch_bounds__(256)
    prep_wc_kernel(const float *__restrict__ w, int ldw, int Tq, int Tk, int Tkp, int causal,
                   float *__restrict__ m, E *__restrict__ Ap, const IO *__restrict__ K, int B,
                   int D, int ldk, int dp, int ncb, int nsplit, int rows_per_split, int vec,
                   float *__restrict__ cpart)
{
    grid_dep_wait();  // launched early (programmatic dependent launch)
    grid_dep_launch();
    const int bid = blockIdx.x;
    const int wblocks = gridDim.x - ncb * nsplit * B;  // eight rows of A' each
    if (bid < wblocks) {
        prep_w_row<E>(bid * 8 + (threadIdx.x >> 5), threadIdx.x & 31, w, ldw, Tq, Tk, Tkp, causal,
                      m, Ap);
        return;
    }
    const int q = bid - wblocks;
    prep_colmax_block<IO>(q % ncb, (q / ncb) % nsplit, q / (ncb * nsplit), K, B, Tk, D, ldk, dp,
                          rows_per_split, vec, cpart);
}

// E'V and E' (eight columns from d0, bf16 K and V) of rows ia and ib of one
// sequence: the four 16-byte loads are issued before any is converted (a
// conversion waits for its load); rows at or past Tk are written as zeros.
template <class E>
__device__ __forceinline__ void panel_rows2(const __nv_bfloat16 *__restrict__ Kb,
                                            const __nv_bfloat16 *__restrict__ Vb, int ldk, int Tk,
                                            int ia, int ib, int d0, const float (&cc)[8],
                                            E *__restrict__ PVa, E *__restrict__ PEa,
                                            E *__restrict__ PVb, E *__restrict__ PEb)
{
    uint4 ka = make_uint4(0u, 0u, 0u, 0u), va = ka, kb = ka, vb = ka;
    if (ia < Tk) {
        ka = __ldg(reinterpret_cast<const uint4 *>(Kb + (size_t)ia * ldk + d0));
        va = __ldg(reinterpret_cast<const uint4 *>(Vb + (size_t)ia * ldk + d0));
    }
    if (ib < Tk) {
        kb = __ldg(reinterpret_cast<const uint4 *>(Kb + (size_t)ib * ldk + d0));
        vb = __ldg(reinterpret_cast<const uint4 *>(Vb + (size_t)ib * ldk + d0));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const bool in = (h ? ib : ia) < Tk;
        const uint4 kw = h ? kb : ka, vw = h ? vb : va;
        const uint32_t kx[4] = {kw.x, kw.y, kw.z, kw.w}, vx[4] = {vw.x, vw.y, vw.z, vw.w};
        float pv[8], pe[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float kv = __uint_as_float(u ? (kx[q] & 0xFFFF0000u) : (kx[q] << 16));
                const float vv = __uint_as_float(u ? (vx[q] & 0xFFFF0000u) : (vx[q] << 16));
                const int k = 2 * q + u;
                pe[k] = in ? __expf(kv - cc[k]) : 0.f;
                pv[k] = pe[k] * vv;
            }
        }
        st8op(h ? PVb : PVa, pv);
        st8op(h ? PEb : PEa, pe);
    }
}

// PV = exp(K - c) * V and PE = exp(K - c) over the padded [B, Tkp, dp] space,
// eight consecutive d per thread (16-byte loads and stores when `vec`).

// Block (128 columns x 16 row lanes) of batch b = blockIdx.z: the block first
// finishes the column maxima of its 128 columns from the nsplit partials (and
// stores them to c for the backward's epilogue), then walks its row range.
template <class IO, class E>
__global__ void __launch_bounds__(256)
    prep_p_kernel(const IO *__restrict__ K, const IO *__restrict__ V,
                  const float *__restrict__ cpart, int nsplit, float *__restrict__ c, int B,
                  int Tk, int D, int ldk, int Tkp, int dp, int rows_per_block, int vec,
                  E *__restrict__ PV, E *__restrict__ PE)
{
    grid_dep_wait();  // launched early (programmatic dependent launch)
    grid_dep_launch();
    __shared__ __align__(16) float cs[128];
    __shared__ float half_mx[128];
    const int b = blockIdx.z;
    const int dblk = blockIdx.x * 128;
    {
        // the column maxima of this block's 128 columns from the nsplit
        // partials: two threads a column, each over half of the partials
        // (independent loads, unrolled), then combined in shared memory
        const int col = threadIdx.x & 127, h = threadIdx.x >> 7;
        const int d = dblk + col;
        float mx = -INFINITY;
        if (d < D) {
#pragma unroll 4
            for (int s = h; s < nsplit; s += 2) mx = fmaxf(mx, __ldg(cpart + ((size_t)s * B + b) * dp + d));
        }
        if (h) half_mx[col] = mx;
        __syncthreads();
        if (!h) {
            mx = d < D ? fmaxf(mx, half_mx[col]) : 0.f;
            cs[col] = mx;
            if (blockIdx.y == 0 && d < dp) c[(size_t)b * dp + d] = mx;
        }
    }
    __syncthreads();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int d0 = dblk + tx * 8;
    if (d0 >= dp) return;  // narrow panels: 64 columns
    float cc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) cc[k] = cs[tx * 8 + k];
    const int r0 = blockIdx.y * rows_per_block, r1 = min(Tkp, r0 + rows_per_block);
    // one row a step: two rows a step with all four loads ahead (panel_rows2,
    // as the clustered prep does) measured slower at T = 4096 (48-53 -> 60 us)
    for (int i = r0 + ty; i < r1; i += 16) {
        float pv[8], pe[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) pv[k] = pe[k] = 0.f;
        if (i < Tk) {
            const size_t src = ((size_t)b * Tk + i) * ldk + d0;
            if (vec && d0 + 8 <= D) {
                float k8[8], v8[8];
                ld8(K + src, k8);
                ld8(V + src, v8);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    pe[k] = __expf(k8[k] - cc[k]);
                    pv[k] = pe[k] * v8[k];
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (d0 + k < D) {
                        pe[k] = __expf(ld_io(K, src + k) - cc[k]);
                        pv[k] = pe[k] * ld_io(V, src + k);
                    }
            }
        }
        const size_t dst = ((size_t)b * Tkp + i) * dp + d0;
        st8op(PV + dst, pv);
        st8op(PE + dst, pe);
    }
}

// One-launch prep: clusters of kPrepCluster CTAs along x.  The first `wcl`
// clusters build A' rows and m (8 rows a CTA, a warp a row).  Every other
// cluster owns one (sequence b, 128-column block) of the panels: CTA `rank`
// reads its rows [rank * rpb, ...) of K for their partial column maxima, the
// cluster combines the kPrepCluster partials over distributed shared memory
// (rank 0 also stores c for the backward's epilogue), and each CTA then reads
// its rows of K again — the same 1 MB column block moments later, an L2 hit —
// with V to write its rows of E'V and E'.  K comes from DRAM once and the
// partial maxima never leave the cluster: prep_wc_kernel's column pass and a
// launch boundary are gone.
constexpr int kPrepCluster = 8;

template <class IO, class E>
__global__ void __launch_bounds__(256)
    prep_fused_kernel(const float *__restrict__ w, int ldw, int Tq, int Tqp, int Tk, int Tkp, int causal,
                      float *__restrict__ m, E *__restrict__ Ap, const IO *__restrict__ K,
                      const IO *__restrict__ V, int D, int ldk, int dp, int ndb, int rpb, int vec,
                      int wcl, float *__restrict__ c, E *__restrict__ PV, E *__restrict__ PE)
{
    grid_dep_wait();  // launched early (programmatic dependent launch)
    grid_dep_launch();
    const int cl = blockIdx.x / kPrepCluster;
    if (cl < wcl) {  // A' rows: every CTA of these clusters, no cluster barrier
        const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
        if (t < Tqp) prep_w_row<E>(t, threadIdx.x & 31, w, ldw, Tq, Tk, Tkp, causal, m, Ap);
        return;
    }
    __shared__ float red[16][129];
    __shared__ float cpart_s[128];
    __shared__ float cs[128];
    const int g = cl - wcl, b = g / ndb, dblk = (g % ndb) * 128;
    const uint32_t rank = cluster_rank();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int d0 = dblk + tx * 8;
    const int r0 = (int)rank * rpb, r1 = min(Tkp, r0 + rpb), rk1 = min(r1, Tk);
    const IO *Kb = K + (size_t)b * Tk * ldk;
    const IO *Vb = V + (size_t)b * Tk * ldk;
    // pass 1: partial column maxima of this CTA's rows
    float mx[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
    if (vec && d0 + 8 <= D) {
        int i = r0 + ty;
        for (; i + 16 < rk1; i += 32) {
            float a[8], a2[8];
            ld8(Kb + (size_t)i * ldk + d0, a);
            ld8(Kb + (size_t)(i + 16) * ldk + d0, a2);
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], fmaxf(a[k], a2[k]));
        }
        for (; i < rk1; i += 16) {
            float a[8];
            ld8(Kb + (size_t)i * ldk + d0, a);
#pragma unroll
            for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], a[k]);
        }
    } else if (d0 < D) {
        for (int i = r0 + ty; i < rk1; i += 16)
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (d0 + k < D) mx[k] = fmaxf(mx[k], ld_io(Kb, (size_t)i * ldk + d0 + k));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) red[ty][tx * 8 + k] = mx[k];
    __syncthreads();
    if (threadIdx.x < 128) {
        float v = red[0][threadIdx.x];
#pragma unroll
        for (int r = 1; r < 16; ++r) v = fmaxf(v, red[r][threadIdx.x]);
        cpart_s[threadIdx.x] = v;
    }
    // the cluster's partials, combined over distributed shared memory in rank order
    cluster_sync_all();
    if (threadIdx.x < 128) {
        const int d = dblk + threadIdx.x;
        const uint32_t mine = (uint32_t)__cvta_generic_to_shared(&cpart_s[threadIdx.x]);
        float v = -INFINITY;
#pragma unroll
        for (int r = 0; r < kPrepCluster; ++r) v = fmaxf(v, ld_dsmem_f32(smem_in_cta(mine, r)));
        v = d < D ? v : 0.f;
        cs[threadIdx.x] = v;
        if (rank == 0 && d < dp) c[(size_t)b * dp + d] = v;
    }
    cluster_sync_all();  // every CTA has read the partials; cs is visible in the CTA
    // pass 2: E'V and E' of this CTA's rows (K again, from L2)
    if (d0 >= dp) return;  // narrow panels: 64 columns
    float cc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) cc[k] = cs[tx * 8 + k];
    int i0 = r0 + ty;
    if constexpr (sizeof(IO) == 2) {
        if (vec && d0 + 8 <= D) {
            for (; i0 + 16 < r1; i0 += 32) {
                const size_t da = ((size_t)b * Tkp + i0) * dp + d0, db = da + (size_t)16 * dp;
                panel_rows2<E>(Kb, Vb, ldk, Tk, i0, i0 + 16, d0, cc, PV + da, PE + da, PV + db, PE + db);
            }
        }
    }
    for (int i = i0; i < r1; i += 16) {
        float pv[8], pe[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) pv[k] = pe[k] = 0.f;
        if (i < Tk) {
            const size_t src = (size_t)i * ldk + d0;
            if (vec && d0 + 8 <= D) {
                float k8[8], v8[8];
                ld8(Kb + src, k8);
                ld8(Vb + src, v8);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    pe[k] = __expf(k8[k] - cc[k]);
                    pv[k] = pe[k] * v8[k];
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (d0 + k < D) {
                        pe[k] = __expf(ld_io(Kb, src + k) - cc[k]);
                        pv[k] = pe[k] * ld_io(Vb, src + k);
                    }
            }
        }
        const size_t dst = ((size_t)b * Tkp + i) * dp + d0;
        st8op(PV + dst, pv);
        st8op(PE + dst, pe);
    }
}

// ------------------------------------------------------------ CUDA-core path
// Same contractions on CUDA cores in fp32 (cross-check of the tensor-core
// path and of the prep kernels; not the product's fast path).
template <int MODE, class E, class IO>
__global__ void aft_simt_kernel(const Params p, const E *__restrict__ Ap,
                                const E *__restrict__ PV, const E *__restrict__ PE)
{
    const E *G1 = (const E *)p.G1;
    const E *G2 = (const E *)p.G2;
    if (MODE == FWD || MODE == BWD1) {
        const size_t total = (size_t)p.B * p.Tqp * p.dp;
        const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (idx >= total) return;
        const int d = (int)(idx % p.dp);
        const int t = (int)((idx / p.dp) % p.Tqp);
        const int b = (int)(idx / ((size_t)p.dp * p.Tqp));
        float num = 0.f, den = 0.f;
        const int lim = p.causal ? min(t + 1, p.Tkp) : p.Tkp;
        for (int i = 0; i < lim; ++i) {
            const float a = from_op(Ap[(size_t)t * p.Tkp + i]);
            const size_t o = ((size_t)b * p.Tkp + i) * p.dp + d;
            num += a * from_op(PV[o]);
            den += a * from_op(PE[o]);
        }
        if (MODE == FWD)
            epi_fwd<IO>(p, b, t, d, num, den);
        else
            epi_bwd1<IO, E>(p, b, t, d, num, den);
    } else if (MODE == HGRAD) {
        const size_t total = (size_t)p.B * p.Tkp * p.dp;
        const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (idx >= total) return;
        const int d = (int)(idx % p.dp);
        const int i = (int)((idx / p.dp) % p.Tkp);
        const int b = (int)(idx / ((size_t)p.dp * p.Tkp));
        float h1 = 0.f, h2 = 0.f;
        for (int t = p.causal ? i : 0; t < p.Tqp; ++t) {
            const float a = from_op(Ap[(size_t)t * p.Tkp + i]);
            const size_t o = ((size_t)b * p.Tqp + t) * p.dp + d;
            h1 += a * from_op(G1[o]);
            h2 += a * from_op(G2[o]);
            if (sizeof(E) == 4) {  // tf32 operands: add the low parts, as the tensor-core path does
                h1 += a * from_op(((const E *)p.G1l)[o]);
                h2 += a * from_op(((const E *)p.G2l)[o]);
            }
        }
        epi_hgrad<IO>(p, b, i, d, h1, h2);
    } else {
        const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (idx >= (size_t)p.Tq * p.Tk) return;
        const int t = (int)(idx / p.Tk), i = (int)(idx % p.Tk);
        if (p.causal && i > t) return;
        float acc = 0.f;
        for (int b = 0; b < p.B; ++b)
            for (int d = 0; d < p.dp; ++d) {
                const size_t og = ((size_t)b * p.Tqp + t) * p.dp + d;
                const size_t op = ((size_t)b * p.Tkp + i) * p.dp + d;
                const float gg = from_op(G1[og]) + from_op(((const E *)p.G1l)[og]);
                const float nn = from_op(G2[og]) + from_op(((const E *)p.G2l)[og]);
                acc += gg * from_op(PV[op]) + nn * from_op(PE[op]);
            }
        epi_wgrad(p, t, i, acc);
    }
}

// ------------------------------------------------------------ tensor-core path
}  // namespace aft
}  // namespace dc

#include "aft_tc.cuh"

namespace dc {
namespace aft {

// Backward from the forward's saved statistics: the element-wise maths of the
// recompute epilogue (epi16_bwd1) with r and 1/den read back, so the backward
// needs no second pass of the forward contraction.  One thread per 16
// columns of one padded row; consecutive threads walk a row.
template <class IO, class E>
__global__ void __launch_bounds__(256, 3) bwd_stats_kernel(const Params p)
{
    grid_dep_wait();  // launched early (programmatic dependent launch)
    grid_dep_launch();
    if (p.zero_dw)
        zero_dw(p, (size_t)blockIdx.x * blockDim.x + threadIdx.x, (size_t)gridDim.x * blockDim.x);
    const int groups = p.dp / 16;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)p.B * p.Tqp * groups) return;
    const int d0 = (int)(idx % groups) * 16;
    const size_t bt = idx / groups;
    const int t = (int)(bt % p.Tqp);
    const int b = (int)(bt / p.Tqp);
    // every load of the thread is issued before any of its data is used:
    // the bf16 statistics and the Q and dZ runs as raw words, so the four
    // requests are in flight together (converting the statistics as they
    // arrived held the Q and dZ loads back by a whole memory round trip)
    uint32_t rw[8], iw[8];
    bool raw_stats = false;
    EpiPre pf;
    pf.ok = false;
    if (t < p.Tq) {
        if constexpr (sizeof(E) == 2) {
            if (t >= p.stat_lo) {
                const size_t so = ((size_t)b * p.Tqp + t) * p.dp + d0;
                ld32B_nc((const E *)p.Rb + so, rw);
                ld32B_nc((const E *)p.Ib + so, iw);
                raw_stats = true;
            }
        }
        if constexpr (sizeof(IO) == 2) {
            if (p.vec_io && d0 + 16 <= p.D) {
                const size_t row = (size_t)b * p.Tq + t;
                ld32B_nc((const IO *)p.Q + row * p.ldi + d0, pf.a);
                ld32B_nc((const IO *)p.dZ + row * p.ldo + d0, pf.b);
                pf.ok = true;
            }
        }
    }
    float r[16], inv[16];
    if (raw_stats) {
        words_to_bf16(rw, r);
        words_to_bf16(iw, inv);
    } else if (t < p.Tq) {
        if (t < p.stat_lo) {
            const size_t so = ((size_t)b * p.stat_lo + t) * p.dp + d0;
            ld16g(p.Rs + so, r);
            ld16g(p.Is + so, inv);
        } else {
            const size_t so = ((size_t)b * p.Tqp + t) * p.dp + d0;
            ld16g((const E *)p.Rb + so, r);
            ld16g((const E *)p.Ib + so, inv);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = inv[j] = 0.f;
    }
    // the forward's range guard, on 1/den' and r
    if (t < p.Tq) {
        bool bad = false;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            bad |= d0 + j < p.D && (!(inv[j] <= 0x1p100f) || !(fabsf(r[j]) <= 3.0e38f));
        if (bad) report_range(p);
    }
    epi16_grads<IO, E>(p, b, t, d0, r, inv, pf);
}

// Block-packed dW to the caller's [Tq][ldw] layout, zeros past each row's
// packed extent: one warp per row, lanes on consecutive columns.
__global__ void __launch_bounds__(256)
    dw_unpack_kernel(const float *__restrict__ packed, float *__restrict__ dW, int ldw, int Tq, int Tk)
{
    grid_dep_wait();  // launched early (programmatic dependent launch)
    grid_dep_launch();
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= Tq) return;
    const float *src = packed + dw_packed_row(t, Tk);
    const int width = (int)dw_packed_width(t, Tk) < Tk ? (int)dw_packed_width(t, Tk) : Tk;
    float *dst = dW + (size_t)t * ldw;
    // 16-byte accesses when the rows of dW start on 16-byte boundaries (the
    // packed rows always do; their widths are multiples of 8 unless clipped
    // to Tk, and Tk % 4 == 0 keeps whole float4s inside the row)
    if ((ldw % 4) == 0 && (Tk % 4) == 0 && (reinterpret_cast<uintptr_t>(dW) & 15) == 0) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = lane; i < Tk / 4; i += 32)
            d4[i] = 4 * i < width ? __ldg(s4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    for (int i = lane; i < Tk; i += 32) dst[i] = i < width ? src[i] : 0.f;
}

// ------------------------------------------------------------ host side
struct Layout {
    int B, Tq, Tk, D, Tqp, Tkp, dp, esz, nsplit, rows_per_split;
    int ldi, ldo;  // row strides of the user tensors (Q, K, V and grads; Z and dZ)
    size_t off_m, off_c, off_cpart, off_ap, off_pv, off_pe, off_g1, off_g2, off_g1l, off_g2l;
    size_t off_rs, off_is;  // saved forward statistics, fp32 rows t < stat_lo (DC_AFT_SAVE_STATS)
    size_t off_rb, off_ib;  // the same in operand precision, rows t >= stat_lo
    int stat_lo;
    size_t total;
};

static int operand_size(int dtype, int flags)
{
    return (dtype == DC_F32 && !(flags & DC_AFT_COMPUTE_BF16)) ? 4 : 2;
}

// Long sequences with bf16 operands run as CTA pairs (M = 256 per MMA, each
// CTA loading half of B): the main loops dominate there.  Short ones keep one
// CTA per tile: their element-wise epilogues dominate, and twice as many
// independent workers drain them faster.
static bool use_pairs(const Layout &L) { return L.esz == 2 && std::max(L.Tqp, L.Tkp) >= 1024; }

// Query rows whose g and n keep their rounding residuals (g - G1, n - G2):
// dW's terms g*E'V + n*E' cancel most (and g = dZ*sigmoid(Q)/den' is largest)
// in the first query rows, where den' sums few terms; with bf16 operands the
// residuals of rows t < 128 (256 when CTA-pair tiles span two 128-row blocks)
// bring dW to the accuracy of keeping them all.  tf32 keeps them everywhere
// (they also enter dK/dV there).  The saved statistics of these rows stay
// fp32, those of the others take the operand precision (their g and n are
// rounded to it anyway).
static int lo_rows_of(const Layout &L)
{
    return L.esz == 4 ? L.Tqp : std::min(L.Tqp, use_pairs(L) ? 2 * BM : BM);
}

static Layout make_layout(int B, int Tq, int Tk, int D, int dtype, int flags)
{
    Layout L{};
    L.B = B;
    L.Tq = Tq;
    L.Tk = Tk;
    L.D = D;
    L.ldi = L.ldo = D;
    const int talign = operand_size(dtype, flags) == 2 ? T_ALIGN2 : T_ALIGN;
    L.Tqp = (int)round_up(std::max(Tq, 1), talign);
    L.Tkp = (int)round_up(std::max(Tk, 1), talign);
    L.esz = operand_size(dtype, flags);
    // Narrow heads (D <= 64, e.g. the reference's 4 x 64-channel heads) pad
    // D to 64 rather than 128 where every tile can be a 64-column half tile
    // (single CTAs: not the CTA-pair regime of long bf16 sequences, whose
    // tiles span 128 columns): half the operand panels, B loads, MMA work and
    // dW's K range.
    L.dp = D <= 64 && !use_pairs(L) ? 64 : (int)round_up(std::max(D, 1), D_ALIGN);
    const int dblocks = (D + 255) / 256;
    int want = (8 * 148 + dblocks * B - 1) / std::max(1, dblocks * B);
    // (at most 32 row slices: prep_p combines the slices' partial maxima of
    // every column before its panel rows, so more of them only lengthen
    // that serial part; small batches asked for up to 128)
    L.nsplit = std::max(1, std::min(std::min(want, 32), (Tk + 31) / 32));
    L.rows_per_split = (Tk + L.nsplit - 1) / L.nsplit;
    L.nsplit = std::max(1, (Tk + L.rows_per_split - 1) / L.rows_per_split);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += round_up((int64_t)bytes, 1024);
        return o;
    };
    L.off_m = take((size_t)L.Tqp * 4);
    L.off_c = take((size_t)B * L.dp * 4);
    L.off_cpart = take((size_t)L.nsplit * B * L.dp * 4);
    L.off_ap = take((size_t)L.Tqp * L.Tkp * L.esz);
    L.off_pv = take((size_t)B * L.Tkp * L.dp * L.esz);
    L.off_pe = take((size_t)B * L.Tkp * L.dp * L.esz);
    L.off_g1 = take((size_t)B * L.Tqp * L.dp * L.esz);
    L.off_g2 = take((size_t)B * L.Tqp * L.dp * L.esz);
    L.off_g1l = take((size_t)B * L.Tqp * L.dp * L.esz);
    L.off_g2l = take((size_t)B * L.Tqp * L.dp * L.esz);
    // saved statistics: fp32 for the rows whose g and n keep their rounding
    // residuals (lo_rows_of), operand precision for the rest
    L.stat_lo = lo_rows_of(L);
    const bool keep = (flags & DC_AFT_SAVE_STATS) != 0;
    const size_t nlo = keep ? (size_t)B * L.stat_lo * L.dp * 4 : 0;
    const size_t nhi = keep && L.stat_lo < L.Tqp ? (size_t)B * L.Tqp * L.dp * L.esz : 0;
    L.off_rs = take(nlo);
    L.off_is = take(nlo);
    L.off_rb = take(nhi);
    L.off_ib = take(nhi);
    L.total = off;
    return L;
}

static int validate(const void *Q, const void *K, const void *V, const float *w, int ldw,
                    int B, int Tq, int Tk, int D, int dtype, int flags)
{
    if (B < 0 || Tq < 0 || Tk < 0 || D < 0)
        return fail(DC_ERR_INVALID, "negative shape B=%d Tq=%d Tk=%d D=%d", B, Tq, Tk, D);
    if (dtype != DC_F32 && dtype != DC_BF16) return fail(DC_ERR_INVALID, "dtype %d", dtype);
    if ((flags & DC_AFT_CAUSAL) && Tq != Tk)
        return fail(DC_ERR_INVALID, "causal AFT needs Tq == Tk (got %d, %d)", Tq, Tk);
    if ((long long)B * Tq * D == 0) return DC_OK;
    if (Tk == 0) return fail(DC_ERR_INVALID, "Tk must be positive when Tq*D*B > 0");
    if (ldw < Tk) return fail(DC_ERR_INVALID, "ldw (%d) < Tk (%d)", ldw, Tk);
    if (!Q || !K || !V || !w) return fail(DC_ERR_INVALID, "null input pointer");
    if ((long long)B * std::max(Tq, Tk) * (long long)D >= (1ll << 40))
        return fail(DC_ERR_INVALID, "tensor too large");
    return DC_OK;
}

// Workspace handed in or allocated on the stream.
struct Workspace {
    char *base = nullptr;
    bool owned = false;
    cudaStream_t stream = nullptr;
    ~Workspace()
    {
        if (owned && base) cudaFreeAsync(base, stream);
    }
};

static int get_workspace(Workspace &ws, const Layout &L, void *workspace, size_t bytes,
                         cudaStream_t stream)
{
    ws.stream = stream;
    if (workspace) {
        if (bytes < L.total)
            return fail(DC_ERR_NOMEM, "workspace of %zu bytes < %zu needed", bytes, L.total);
        if ((reinterpret_cast<uintptr_t>(workspace) & 1023) != 0)
            return fail(DC_ERR_INVALID, "workspace must be 1024-byte aligned");
        ws.base = static_cast<char *>(workspace);
        return DC_OK;
    }
    void *p = nullptr;
    DC_CUDA_TRY(cudaMallocAsync(&p, L.total, stream));
    ws.base = static_cast<char *>(p);
    ws.owned = true;
    return DC_OK;
}

template <class IO, class E>
static int run_prep(const Layout &L, const IO *K, const IO *V, const float *w, int ldw,
                    int causal, char *ws, cudaStream_t st)
{
    float *m = reinterpret_cast<float *>(ws + L.off_m);
    float *c = reinterpret_cast<float *>(ws + L.off_c);
    float *cpart = reinterpret_cast<float *>(ws + L.off_cpart);
    E *Ap = reinterpret_cast<E *>(ws + L.off_ap);
    E *PV = reinterpret_cast<E *>(ws + L.off_pv);
    E *PE = reinterpret_cast<E *>(ws + L.off_pe);
    // 16-byte access to K and V rows: D a multiple of 8 and aligned bases
    const int vec = (L.D % 8 == 0) && (L.ldi % 8 == 0) &&
                    ((reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V)) & 15) == 0;
    // one launch for panels of up to 16 M elements (measured: C2 31.6 -> 28.3
    // us, the decoder's heads 306 -> 204 us of prep a step); larger ones keep
    // the two launches, whose column pass streams K at the full rate (C4:
    // 82 us against 92 us in one launch, whose second read of K and the A'
    // rows' stream then compete for L2)
    if (!g_prep_two_launch && (long long)L.B * L.Tkp * L.dp <= (16ll << 20)) {
        // one launch: A' clusters first, then a cluster per (b, 128 columns)
        KernelTimer kt("aft_prep", st);
        const int ndb = (L.dp + 127) / 128;
        const int rpb = (L.Tkp + kPrepCluster - 1) / kPrepCluster;
        const int wcl = (L.Tqp + 8 * kPrepCluster - 1) / (8 * kPrepCluster);
        const long long clusters = (long long)wcl + (long long)L.B * ndb;
        if (clusters * kPrepCluster > 0x7fffffffLL) return fail(DC_ERR_INVALID, "prep grid too large");
        DC_CUDA_TRY(launch_pdl(prep_fused_kernel<IO, E>, dim3((unsigned)(clusters * kPrepCluster)), dim3(256), 0,
                               st, kPrepCluster, w, ldw, L.Tq, L.Tqp, L.Tk, L.Tkp, causal, m, Ap, K, V, L.D,
                               L.ldi, L.dp, ndb, rpb, vec, wcl, c, PV, PE));
        DC_CUDA_TRY(cudaGetLastError());
        return DC_OK;
    }
    {
        // A' rows and the partial column maxima of K in one launch
        KernelTimer kt("aft_prep_w_colmax", st);
        const int ncb = (L.D + 255) / 256;
        const int grid = L.Tqp / 8 + ncb * L.nsplit * L.B;
        DC_CUDA_TRY(launch_pdl(prep_wc_kernel<IO, E>, dim3(grid), dim3(256), 0, st, 1, w, ldw, L.Tq,
                               L.Tk, L.Tkp, causal, m, Ap, K, L.B, L.D, L.ldi, L.dp, ncb,
                               L.nsplit, L.rows_per_split, vec, cpart));
    }
    {
        KernelTimer kt("aft_prep_p", st);
        const int ndb = (L.dp + 127) / 128;
        const int target = sm_count() * 4;
        int rsplit = std::max(1, (target + ndb * L.B - 1) / (ndb * L.B));
        rsplit = std::min(rsplit, std::max(1, L.Tkp / 16));
        const int rows_per_block = (L.Tkp + rsplit - 1) / rsplit;
        rsplit = (L.Tkp + rows_per_block - 1) / rows_per_block;
        DC_CUDA_TRY(launch_pdl(prep_p_kernel<IO, E>, dim3(ndb, rsplit, L.B), dim3(256), 0, st, 1,
                               K, V, cpart, L.nsplit, c, L.B, L.Tk, L.D, L.ldi, L.Tkp, L.dp,
                               rows_per_block, vec, PV, PE));
    }
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

// dW output tiles (128 query rows x 256 keys) before split-K; causal
// launches skip the pairs above the diagonal.
static int wgrad_tiles(const Layout &L, int causal)
{
    if (use_pairs(L)) {  // CTA pairs: 256 query rows x 256 keys
        const int mt = L.Tqp / T_ALIGN2, nt = L.Tkp / T_ALIGN2;
        return causal ? mt * (mt + 1) / 2 : mt * nt;
    }
    const int mt = L.Tqp / BM, nt = L.Tkp / BN;
    return causal ? wgrad_pairs_before(mt) : mt * ((nt + 1) / 2);
}

static CUtensorMapDataType tmap_type(int esz)
{
    return esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Swizzle of a TMA box: MN-major tiles of 32-bit operands need the 32-byte
// atom variant of the 128-byte swizzle (the smem form tcgen05 reads for
// MN-major tf32); everything else uses the 16-byte-atom 128-byte swizzle.
static CUtensorMapSwizzle tile_swizzle(const Layout &L, bool mn_major, int krow = 128)
{
    if (mn_major)
        return L.esz == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    return krow == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
}

// [B][rows][dp] operand buffer; box of `bx` (inner, d) x `by` rows.  K-major
// boxes of `krow` bytes per row use the matching 128- or 64-byte swizzle.
static int map_3d(CUtensorMap *m, const void *base, const Layout &L, int rows, uint32_t bx,
                  uint32_t by, bool mn_major, int krow = 128)
{
    uint64_t dims[3] = {(uint64_t)L.dp, (uint64_t)rows, (uint64_t)L.B};
    uint64_t strides[2] = {(uint64_t)L.dp * L.esz, (uint64_t)rows * L.dp * L.esz};
    uint32_t box[3] = {bx, by, 1};
    return encode_tmap(m, tmap_type(L.esz), 3, base, dims, strides, box,
                       tile_swizzle(L, mn_major, krow));
}

// A' [Tqp][Tkp]; box of `bx` (inner, i) x `by` rows (t).
static int map_ap(CUtensorMap *m, const void *base, const Layout &L, uint32_t bx, uint32_t by,
                  bool mn_major)
{
    uint64_t dims[2] = {(uint64_t)L.Tkp, (uint64_t)L.Tqp};
    uint64_t strides[1] = {(uint64_t)L.Tkp * L.esz};
    uint32_t box[2] = {bx, by};
    return encode_tmap(m, tmap_type(L.esz), 2, base, dims, strides, box,
                       tile_swizzle(L, mn_major));
}

template <int MODE, class E, class IO, bool P>
static int launch_tc(Params p, const Layout &L, char *ws, cudaStream_t st)
{
    static_assert(!P || sizeof(E) == 2, "CTA pairs run bf16 operands");
    using C = TcCfg<MODE, E, P>;
    constexpr int RB = P ? 2 * BM : BM;
    // per instantiation and device; host threads may race to set them (the
    // attribute call is idempotent), the flags themselves are atomic
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    DC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DC_ERR_UNSUPPORTED, "device ordinal %d", dev);
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        DC_CUDA_TRY(cudaFuncSetAttribute(aft_tc_kernel<MODE, E, IO, P>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES));
        attr_set[dev].store(true, std::memory_order_release);
    }
    // tensor maps: A, B1..B4 (B3/B4 only for the tf32 dK/dV low parts), A2..A4 (dW)
    CUtensorMap mA, mB1, mB2, mB3, mB4, mA2, mA3, mA4;
    const uint32_t BK = C::BKe, BOX = C::BOX_MN;
    const int nd = (L.dp + BN - 1) / BN;
    if (MODE == FWD || MODE == BWD1) {
        DC_TRY(map_ap(&mA, ws + L.off_ap, L, BK, BM, false));
        DC_TRY(map_3d(&mB1, ws + L.off_pv, L, L.Tkp, BOX, BK, true));
        DC_TRY(map_3d(&mB2, ws + L.off_pe, L, L.Tkp, BOX, BK, true));
        mB3 = mB4 = mA2 = mA3 = mA4 = mA;
        p.n_tiles = (L.Tqp / RB) * nd * L.B;
    } else if (MODE == HGRAD) {
        DC_TRY(map_ap(&mA, ws + L.off_ap, L, BOX, BK, true));
        DC_TRY(map_3d(&mB1, ws + L.off_g1, L, L.Tqp, BOX, BK, true));
        DC_TRY(map_3d(&mB2, ws + L.off_g2, L, L.Tqp, BOX, BK, true));
        DC_TRY(map_3d(&mB3, ws + L.off_g1l, L, L.Tqp, BOX, BK, true));
        DC_TRY(map_3d(&mB4, ws + L.off_g2l, L, L.Tqp, BOX, BK, true));
        mA2 = mA3 = mA4 = mA;
        p.n_tiles = (L.Tkp / RB) * nd * L.B;
    } else {
        const int kr = C::KROW;
        DC_TRY(map_3d(&mA, ws + L.off_g1, L, L.Tqp, BK, BM, false, kr));
        DC_TRY(map_3d(&mA2, ws + L.off_g2, L, L.Tqp, BK, BM, false, kr));
        DC_TRY(map_3d(&mA3, ws + L.off_g1l, L, L.Tqp, BK, BM, false, kr));
        DC_TRY(map_3d(&mA4, ws + L.off_g2l, L, L.Tqp, BK, BM, false, kr));
        DC_TRY(map_3d(&mB1, ws + L.off_pv, L, L.Tkp, BK, C::BROWS, false, kr));
        DC_TRY(map_3d(&mB2, ws + L.off_pe, L, L.Tkp, BK, C::BROWS, false, kr));
        mB3 = mB4 = mB1;
        p.n_tiles = (p.sk_tiles + p.sk_lo) * p.splits;
    }
    p.trace = (g_trace_modes >> MODE) & 1 ? g_trace_buf : nullptr;
#ifdef DC_TEST_WITHHOLD
    p.test_withhold = g_test_withhold;
    g_test_withhold = 0;
#endif
    static const char *names[4] = {"aft_tc_fwd", "aft_tc_bwd_recompute", "aft_tc_dkdv",
                                   "aft_tc_dw"};
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = P ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // persistent: one CTA (or CTA pair) per SM (pair); shared memory admits one.
    // Pairs need two SMs of one GPC: ask how many clusters fit at once.
    static std::atomic<int> max_clusters[64];
    if (P && max_clusters[dev].load(std::memory_order_acquire) == 0) {
        cfg.gridDim = dim3(2 * (sm_count() / 2));
        int n = 0;
        DC_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, aft_tc_kernel<MODE, E, IO, P>, &cfg));
        max_clusters[dev].store(std::max(1, n), std::memory_order_release);
    }
    const int workers = P ? std::max(1, max_clusters[dev].load(std::memory_order_acquire) -
                                            (p.spare_sms + 1) / 2)
                          : std::max(1, sm_count() - p.spare_sms);
    // Schedule (decode_tile): bundles only pay with at least two tiles a
    // worker (with fewer they would leave workers idle).  Where whole rounds
    // leave a partial last one, its tiles can run as halves spread over all
    // workers instead, when that shortens the schedule (counting a half as
    // half a tile; single CTAs with two B tiles a stage).
    p.bundled = 0;
    p.n_full = p.n_tiles;
    p.narrow = MODE != WGRAD && L.dp < BN;
    if (p.narrow && !C::HALF_OK && MODE != HGRAD)
        return fail(DC_ERR_UNSUPPORTED, "narrow panels need half tiles");  // excluded by make_layout
    if (p.narrow) {
        p.bundled = p.n_tiles >= 2 * workers;
    } else if (MODE != WGRAD) {
        const int U = p.n_tiles;
        const double rounds = (double)((U + workers - 1) / workers);
        const int F = U / workers * workers, R = U - F;
        const double with_halves = (double)(U / workers) + 0.5 * ((2 * R + workers - 1) / workers);
        if (C::HALF_OK && R > 0 && with_halves < 0.95 * rounds) {
            p.n_full = F;
            p.n_tiles = F + 2 * R;
        } else {
            p.bundled = U >= 2 * workers;
        }
    }
    const dim3 grid((P ? 2 : 1) * std::max(1, std::min(p.n_tiles, workers)));
    {
        KernelTimer kt(names[MODE], st);
        DC_CUDA_TRY(launch_pdl(aft_tc_kernel<MODE, E, IO, P>, grid, dim3(kTcThreads), C::SMEM_BYTES,
                               st, P ? 2 : 1, p, mA, mB1, mB2, mB3, mB4, mA2, mA3, mA4));
    }
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

template <int MODE, class E, class IO>
static int launch_simt(const Params &p, const Layout &L, char *ws, cudaStream_t st)
{
    size_t n;
    if (MODE == FWD || MODE == BWD1)
        n = (size_t)L.B * L.Tqp * L.dp;
    else if (MODE == HGRAD)
        n = (size_t)L.B * L.Tkp * L.dp;
    else
        n = (size_t)L.Tq * L.Tk;
    KernelTimer kt("aft_simt", st);
    aft_simt_kernel<MODE, E, IO><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        p, reinterpret_cast<const E *>(ws + L.off_ap), reinterpret_cast<const E *>(ws + L.off_pv),
        reinterpret_cast<const E *>(ws + L.off_pe));
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

template <int MODE, class E, class IO>
static int launch(const Params &p, const Layout &L, char *ws, cudaStream_t st, int flags)
{
    if (flags & DC_AFT_SIMT) return launch_simt<MODE, E, IO>(p, L, ws, st);
    if constexpr (sizeof(E) == 2)
        if (use_pairs(L)) return launch_tc<MODE, E, IO, true>(p, L, ws, st);
    return launch_tc<MODE, E, IO, false>(p, L, ws, st);
}

// The tensor-core forward keeps r and 1/den for the backward.
static bool saves_stats(int flags)
{
    return (flags & DC_AFT_SAVE_STATS) && !(flags & DC_AFT_SIMT);
}

static Params make_params(const Layout &L, char *ws, int flags)
{
    Params p{};
    p.B = L.B;
    p.Tq = L.Tq;
    p.Tk = L.Tk;
    p.D = L.D;
    p.ldi = L.ldi;
    p.ldo = L.ldo;
    p.Tqp = L.Tqp;
    p.Tkp = L.Tkp;
    p.dp = L.dp;
    p.causal = (flags & DC_AFT_CAUSAL) ? 1 : 0;
    p.accumulate = (flags & DC_AFT_ACCUMULATE) ? 1 : 0;
    p.m = reinterpret_cast<const float *>(ws + L.off_m);
    p.c = reinterpret_cast<const float *>(ws + L.off_c);
    p.G1 = ws + L.off_g1;
    p.G2 = ws + L.off_g2;
    p.G1l = ws + L.off_g1l;
    p.G2l = ws + L.off_g2l;
    p.lo_rows = lo_rows_of(L);
    if (saves_stats(flags)) {
        p.Rs = reinterpret_cast<float *>(ws + L.off_rs);
        p.Is = reinterpret_cast<float *>(ws + L.off_is);
        p.Rb = ws + L.off_rb;
        p.Ib = ws + L.off_ib;
        p.stat_lo = L.stat_lo;
    }
    p.spare_sms = (flags >> 16) & 0xff;
    p.status = device_status_word();
    return p;
}

// 32-byte vector access along D: every 16-element run of a row starts on a
// 32-byte boundary when both row strides are multiples of 32 bytes and every
// base pointer is 32-byte aligned.
template <class IO>
static int vec_ok(const Layout &L, std::initializer_list<const void *> ptrs)
{
    if ((L.ldi * (int)sizeof(IO)) % 32 != 0 || (L.ldo * (int)sizeof(IO)) % 32 != 0) return 0;
    for (const void *q : ptrs)
        if (reinterpret_cast<uintptr_t>(q) & 31) return 0;
    return 1;
}

template <class IO, class E>
static int fwd_impl(const void *Q, const void *K, const void *V, const float *w, int ldw,
                    void *Z, const Layout &L, int flags, char *ws, cudaStream_t st)
{
    if (!(flags & DC_AFT_WS_VALID))
        DC_TRY(run_prep<IO, E>(L, (const IO *)K, (const IO *)V, w, ldw,
                               (flags & DC_AFT_CAUSAL) ? 1 : 0, ws, st));
    Params p = make_params(L, ws, flags);
    p.Q = Q;
    p.K = K;
    p.V = V;
    p.Z = Z;
    p.w = w;
    p.ldw = ldw;
    p.vec_io = vec_ok<IO>(L, {Q, Z});
    return launch<FWD, E, IO>(p, L, ws, st, flags);
}

template <class IO, class E>
static int bwd_impl(const void *Q, const void *K, const void *V, const float *w, int ldw,
                    const void *dZ, void *dQ, void *dK, void *dV, float *dW, const Layout &L,
                    int flags, char *ws, cudaStream_t st)
{
    const int causal = (flags & DC_AFT_CAUSAL) ? 1 : 0;
    Params p = make_params(L, ws, flags);
    p.Q = Q;
    p.K = K;
    p.V = V;
    p.dZ = dZ;
    p.dQ = dQ;
    p.dK = dK;
    p.dV = dV;
    p.dW = dW;
    p.w = w;
    p.ldw = ldw;
    p.vec_io = vec_ok<IO>(L, {Q, K, V, dZ, dQ, dK, dV});
    p.vec_w = (ldw % 8 == 0) && ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(dW)) & 31) == 0;
    p.dw_packed = (flags & DC_AFT_DW_PACKED) ? 1 : 0;
    // dQ, g and n, then dW (which needs only g, n and the prep panels), then
    // dK and dV: a caller that splits the call can reduce dW across ranks
    // while the last contraction runs
    if (!(flags & DC_AFT_BWD_DKDV)) {
        if (!(flags & DC_AFT_WS_VALID))
            DC_TRY(run_prep<IO, E>(L, (const IO *)K, (const IO *)V, w, ldw, causal, ws, st));
        // dW starts at zero for the split-K atomics: the tensor-core and
        // statistics kernels clear it themselves (no memset node between
        // them and the dW launch); the CUDA-core cross-check path does not
        if (!(flags & DC_AFT_ACCUMULATE)) {
            if ((flags & DC_AFT_SIMT) && p.dw_packed)
                DC_CUDA_TRY(cudaMemsetAsync(dW, 0, dw_packed_floats(L.Tq, L.Tk) * 4, st));
            else if (flags & DC_AFT_SIMT)
                DC_CUDA_TRY(cudaMemset2DAsync(dW, (size_t)ldw * 4, 0, (size_t)L.Tk * 4, L.Tq, st));
            else
                p.zero_dw = 1;
        }
        if ((flags & DC_AFT_WS_VALID) && saves_stats(flags)) {
            KernelTimer kt("aft_bwd_from_stats", st);
            const size_t n = (size_t)L.B * L.Tqp * (L.dp / 16);
            DC_CUDA_TRY(launch_pdl(bwd_stats_kernel<IO, E>, dim3((unsigned)((n + 255) / 256)),
                                   dim3(256), 0, st, 1, p));
            DC_CUDA_TRY(cudaGetLastError());
        } else {
            DC_TRY((launch<BWD1, E, IO>(p, L, ws, st, flags)));
        }
        // dW: tiles, then the low-part passes of the first rows' tiles as
        // tiles of their own, each split into `splits` K ranges.  The split
        // count is the one whose units fill the persistent workers (CTAs, or
        // CTA pairs) in the least time, waves x time per unit, where a unit
        // costs at least its epilogue (the scaled atomic adds of a 128 x 256
        // block per CTA: measured at about 4 K steps of 128 B, 8 of the 64 B
        // steps a single CTA runs, of its main loop; for pairs, whose
        // epilogues contend for the same dW lines, splitting below ~40 steps
        // measured slower), so splitting finer than that only adds atomics.
        // All units then have one K length and the workers walk K together,
        // which keeps the operand slices they read in L2.
        Params pw = p;
        pw.zero_dw = 0;
        const bool pairs = use_pairs(L);
        pw.kpb = L.dp / (pairs ? TcCfg<WGRAD, E, sizeof(E) == 2>::BKe : TcCfg<WGRAD, E, false>::BKe);
        const int rb = pairs ? 2 * BM : BM;
        const int lo_blocks = std::min((p.lo_rows + rb - 1) / rb, L.Tqp / rb);
        pw.sk_tiles = wgrad_tiles(L, causal);
        pw.sk_lo = !causal ? lo_blocks * ((L.Tkp / BN + 1) / 2)
                   : pairs ? lo_blocks * (lo_blocks + 1) / 2 : wgrad_pairs_before(lo_blocks);
        const int tiles = pw.sk_tiles + pw.sk_lo;
        const int ktot = L.B * pw.kpb;
        const int workers = pairs ? sm_count() / 2 : sm_count();
        const double kEpiSteps = pairs ? 40.0 : 8.0;  // in K steps of the launched tile
        int best = 1;
        double best_cost = 1e30;
        for (int sp = 1; sp <= std::max(1, ktot / 8); ++sp) {
            const int waves = (tiles * sp + workers - 1) / workers;
            const double cost = waves * std::max((double)ktot / sp, kEpiSteps);
            if (cost < 0.97 * best_cost) {  // more splits only for a clear gain (atomics)
                best_cost = cost;
                best = sp;
            }
        }
        pw.splits = best;
        DC_TRY((launch<WGRAD, E, IO>(pw, L, ws, st, flags)));
    }
    if (!(flags & DC_AFT_BWD_NO_DKDV)) DC_TRY((launch<HGRAD, E, IO>(p, L, ws, st, flags)));
    return DC_OK;
}

}  // namespace aft
}  // namespace dc

using namespace dc;
using namespace dc::aft;

extern "C" {

#ifdef DC_TEST_WITHHOLD
int dc_test_withhold_next(int on)
{
    g_test_withhold = on ? 1 : 0;
    return DC_OK;
}
#endif

int dc_aft_trace(void *device_buffer, size_t bytes, int mode_mask)
{
    const size_t need = (size_t)sm_count() * 64 * 8 * sizeof(unsigned long long);
    if (device_buffer && bytes < need)
        return fail(DC_ERR_NOMEM, "trace buffer needs %zu bytes", need);
    g_trace_buf = static_cast<unsigned long long *>(device_buffer);
    g_trace_modes = device_buffer ? mode_mask : 0;
    return DC_OK;
}

int dc_aft_prep_mode(int two_launch)
{
    g_prep_two_launch = two_launch ? 1 : 0;
    return DC_OK;
}

int dc_aft_dw_packed_size(int Tq, int Tk, size_t *floats)
{
    clear_error();
    if (!floats) return fail(DC_ERR_INVALID, "floats is NULL");
    if (Tq < 0 || Tk < 0) return fail(DC_ERR_INVALID, "negative shape");
    *floats = dw_packed_floats(Tq, Tk);
    return DC_OK;
}

int dc_aft_dw_unpack(const float *packed, float *dW, int ldw, int Tq, int Tk, void *stream)
{
    clear_error();
    if (Tq < 0 || Tk < 0 || ldw < Tk) return fail(DC_ERR_INVALID, "bad shape Tq=%d Tk=%d ldw=%d", Tq, Tk, ldw);
    if ((long long)Tq * Tk == 0) return DC_OK;
    if (!packed || !dW) return fail(DC_ERR_INVALID, "null pointer");
    cudaStream_t st = as_stream(stream);
    KernelTimer kt("aft_dw_unpack", st);
    DC_CUDA_TRY(launch_pdl(dw_unpack_kernel, dim3((unsigned)((Tq + 7) / 8)), dim3(256), 0, st, 1, packed, dW,
                           ldw, Tq, Tk));
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

int dc_aft_workspace_size(int B, int Tq, int Tk, int D, int dtype, int flags, size_t *bytes)
{
    clear_error();
    if (!bytes) return fail(DC_ERR_INVALID, "bytes is NULL");
    if (B < 0 || Tq < 0 || Tk < 0 || D < 0) return fail(DC_ERR_INVALID, "negative shape");
    *bytes = make_layout(B, Tq, Tk, D, dtype, flags).total;
    return DC_OK;
}

int dc_aft_fwd(const void *Q, const void *K, const void *V, const float *w, int ldw, void *Z,
               int B, int Tq, int Tk, int D, int dtype, int flags, void *workspace,
               size_t workspace_bytes, void *stream)
{
    return dc_aft_fwd_strided(Q, K, V, w, ldw, Z, B, Tq, Tk, D, D, D, dtype, flags, workspace,
                              workspace_bytes, stream);
}

int dc_aft_bwd(const void *Q, const void *K, const void *V, const float *w, int ldw,
               const void *dZ, void *dQ, void *dK, void *dV, float *dW, int B, int Tq, int Tk,
               int D, int dtype, int flags, void *workspace, size_t workspace_bytes,
               void *stream)
{
    return dc_aft_bwd_strided(Q, K, V, w, ldw, dZ, dQ, dK, dV, dW, B, Tq, Tk, D, D, D, dtype,
                              flags, workspace, workspace_bytes, stream);
}

int dc_aft_fwd_strided(const void *Q, const void *K, const void *V, const float *w, int ldw,
                       void *Z, int B, int Tq, int Tk, int D, int ldi, int ldo, int dtype,
                       int flags, void *workspace, size_t workspace_bytes, void *stream)
{
    clear_error();
    DC_TRY(validate(Q, K, V, w, ldw, B, Tq, Tk, D, dtype, flags));
    if ((long long)B * Tq * D == 0) return DC_OK;
    if (!Z) return fail(DC_ERR_INVALID, "Z is NULL");
    if (ldi < D || ldo < D) return fail(DC_ERR_INVALID, "row strides (%d, %d) < D (%d)", ldi, ldo, D);
    cudaStream_t st = as_stream(stream);
    Layout L = make_layout(B, Tq, Tk, D, dtype, flags);
    L.ldi = ldi;
    L.ldo = ldo;
    Workspace ws;
    DC_TRY(get_workspace(ws, L, workspace, workspace_bytes, st));
    if (dtype == DC_BF16)
        return fwd_impl<__nv_bfloat16, __nv_bfloat16>(Q, K, V, w, ldw, Z, L, flags, ws.base, st);
    if (L.esz == 2)
        return fwd_impl<float, __nv_bfloat16>(Q, K, V, w, ldw, Z, L, flags, ws.base, st);
    return fwd_impl<float, float>(Q, K, V, w, ldw, Z, L, flags, ws.base, st);
}

int dc_aft_bwd_strided(const void *Q, const void *K, const void *V, const float *w, int ldw,
                       const void *dZ, void *dQ, void *dK, void *dV, float *dW, int B, int Tq,
                       int Tk, int D, int ldi, int ldo, int dtype, int flags, void *workspace,
                       size_t workspace_bytes, void *stream)
{
    clear_error();
    DC_TRY(validate(Q, K, V, w, ldw, B, Tq, Tk, D, dtype, flags));
    if ((long long)B * Tq * D == 0) return DC_OK;
    const bool part1 = !(flags & DC_AFT_BWD_DKDV), part2 = !(flags & DC_AFT_BWD_NO_DKDV);
    if (!part1 && !part2)
        return fail(DC_ERR_INVALID, "DC_AFT_BWD_NO_DKDV and DC_AFT_BWD_DKDV together");
    if (!part1 && !(flags & DC_AFT_WS_VALID))
        return fail(DC_ERR_INVALID, "DC_AFT_BWD_DKDV needs DC_AFT_WS_VALID (g, n of an earlier call)");
    if ((part1 && (!dZ || !dQ || !dW)) || (part2 && (!dK || !dV)))
        return fail(DC_ERR_INVALID, "null gradient pointer");
    if (ldi < D || ldo < D) return fail(DC_ERR_INVALID, "row strides (%d, %d) < D (%d)", ldi, ldo, D);
    if ((flags & DC_AFT_DW_PACKED) && !(flags & DC_AFT_CAUSAL))
        return fail(DC_ERR_INVALID, "DC_AFT_DW_PACKED needs DC_AFT_CAUSAL (the packed layout holds the causal extent)");
    cudaStream_t st = as_stream(stream);
    Layout L = make_layout(B, Tq, Tk, D, dtype, flags);
    L.ldi = ldi;
    L.ldo = ldo;
    Workspace ws;
    DC_TRY(get_workspace(ws, L, workspace, workspace_bytes, st));
    if (dtype == DC_BF16)
        return bwd_impl<__nv_bfloat16, __nv_bfloat16>(Q, K, V, w, ldw, dZ, dQ, dK, dV, dW, L,
                                                      flags, ws.base, st);
    if (L.esz == 2)
        return bwd_impl<float, __nv_bfloat16>(Q, K, V, w, ldw, dZ, dQ, dK, dV, dW, L, flags,
                                              ws.base, st);
    return bwd_impl<float, float>(Q, K, V, w, ldw, dZ, dQ, dK, dV, dW, L, flags, ws.base, st);
}

}  // extern "C"
