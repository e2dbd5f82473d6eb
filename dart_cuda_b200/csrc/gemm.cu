// General tcgen05 GEMM of the decoder's dense layers (Q/K/V, projections,
// FFN, LM head) and of their backward:
//
//   C[M,N] = epilogue( alpha * op(A)[M,K] . op(B)[K,N] )
//
// op(A) = A ([M,K] row-major, K-major for the tensor core) or A^T (A stored
// [K,M], MN-major); op(B) = B ([K,N] row-major, MN-major) or B^T (B stored
// [N,K], K-major).  Forward layers are NN (X . W), the input gradient is NT
// (dY . W^T) and the weight gradient TN (X^T . dY).  fp32 tensors run with
// tf32 operands, bf16 tensors with bf16 operands; accumulation and C are
// fp32.  The epilogue fuses what follows a layer's product in the reference
// (native/src/engine.cu:480-507 matmul, :352-372 row-broadcast bias,
// native/src/kernels/elementwise.cuh:328-351 tanh GELU and its derivative,
// residual adds): bias, GELU (keeping the pre-activation for the backward),
// the GELU derivative, and a residual / accumulate input; and the decoder's
// cross-attention gate, sigmoid(value) * v0 (dc_gate_fwd).
//
// One persistent CTA per SM walks 128 x BN output tiles (split along K when
// the tiles alone cannot fill the SMs: with atomics into C for a linear
// epilogue, else over a cluster of CTAs a tile, see below): warp 16
// issues TMA loads into a ring of stages (six of 32 KB with BN = 128, four of
// 48 KB with BN = 256), warp 17 owns TMEM and issues the MMAs into a
// double-buffered accumulator, warps 0-15 drain it.  BN = 256 (one N = 256
// MMA a K slice) serves products with enough 128 x 256 tiles to fill the SMs
// unsplit: each A tile then feeds twice the outputs from shared memory, and
// the tall, short-K layers of the decoder take half as many rounds.
#include <cuda_bf16.h>

#include <atomic>

#include "dc_internal.h"
#include "dc_ptx.cuh"

namespace dc {
namespace gemm {

constexpr int BM = 128, BN = 128;  // BN: the narrow tile; Cfg::TBN the launched one
constexpr int kEpiWarps = 16;
constexpr int kThreads = (kEpiWarps + 2) * 32;

enum : int {
    EPI_BIAS = 1,      // + bias[n] (split 0 only under split-K)
    EPI_GELU = 2,      // aux = pre-activation (if aux), C = gelu(pre)
    EPI_GELU_BWD = 4,  // C = value * gelu'(aux)
    EPI_RESID = 8,     // + R[m, n] before the activation (R may alias C)
    EPI_ATOMIC = 16,   // split-K: C += value with atomics (C pre-initialised)
    EPI_GATE = 32,     // C = sigmoid(value) * gate[n] (after bias and residual)
};

template <class E, bool A_MN, bool B_MN, int TBN_ = BN>
struct Cfg {
    static constexpr int TBN = TBN_;
    static constexpr bool TF32 = sizeof(E) == 4;
    static constexpr int BKe = 128 / (int)sizeof(E);     // K elements per stage (128 B rows)
    static constexpr int UK = TF32 ? 8 : 16;             // K per MMA instruction
    static constexpr int NSUB = BKe / UK;
    static constexpr int BOX_MN = 128 / (int)sizeof(E);  // MN elements in one 128 B block
    static constexpr int TILE_BYTES = 128 * 128;        // A: 128 rows x 128 B of K
    static constexpr int B_BYTES = TBN * 128;           // B: TBN columns x 128 B of K
    static constexpr int STAGE_BYTES = TILE_BYTES + B_BYTES;
    static constexpr int STAGES = TBN == 128 ? 6 : 4;
    static_assert(kEpiWarps * 2048 <= STAGES * STAGE_BYTES, "epilogue staging fits the stages");
    static constexpr uint32_t IDESC = umma_idesc(TF32 ? 2u : 1u, BM, TBN, A_MN, B_MN);
    static constexpr uint32_t MN_LBO = BKe * 128;
    static constexpr uint32_t MN_LAYOUT = TF32 ? 1u : 2u;
    static constexpr uint32_t MN_SBO = TF32 ? 512u : 1024u;
    static constexpr uint32_t TMEM_COLS = 2 * TBN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
    // cluster split-K: a CTA's partial tile, rows padded by 16 bytes, in the stages
    static constexpr int RED_LD = TBN + 4;
    static_assert(BM * RED_LD * 4 <= STAGES * STAGE_BYTES, "partial tile fits the stages");
};

struct Params {
    int M, N, K;
    int ldc, ldr, ldx;
    float alpha;
    float *C;
    const float *R;
    const float *bias;
    float *aux;
    int epi;
    int tiles_m, tiles_n, splits, ksteps, n_tiles;
    int vec;
    int *status;
    const float *gate;  // EPI_GATE: [N]
    // cluster split-K: the `cl` splits of one tile are consecutive CTAs of
    // one cluster and add their partial tiles over distributed shared
    // memory before the epilogue (0: off)
    int cl;
};

// tanh-approximated GELU and its derivative, the forms of the reference's
// gelu_fwd / gelu_bwd (native/src/kernels/elementwise.cuh:328-351).
__device__ __forceinline__ float gelu_f(float x)
{
    return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
}
__device__ __forceinline__ float gelu_d(float x)
{
    const float x2 = x * x;
    const float t = tanhf(0.7978845608f * (x + 0.044715f * x2 * x));
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * 0.7978845608f * (1.0f + 3.0f * 0.044715f * x2);
}

// the sigmoid of the cross-attention gate (dc_gate_fwd's form)
__device__ __forceinline__ float sigm_f(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ void ld16f(const float *p, float (&v)[16])
{
    const float4 *q = reinterpret_cast<const float4 *>(p);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 f = q[k];
        v[4 * k] = f.x;
        v[4 * k + 1] = f.y;
        v[4 * k + 2] = f.z;
        v[4 * k + 3] = f.w;
    }
}
__device__ __forceinline__ void st16f(float *p, const float (&v)[16])
{
#pragma unroll
    for (int h = 0; h < 2; ++h)
        asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p + 8 * h),
                     "r"(__float_as_uint(v[8 * h])), "r"(__float_as_uint(v[8 * h + 1])),
                     "r"(__float_as_uint(v[8 * h + 2])), "r"(__float_as_uint(v[8 * h + 3])),
                     "r"(__float_as_uint(v[8 * h + 4])), "r"(__float_as_uint(v[8 * h + 5])),
                     "r"(__float_as_uint(v[8 * h + 6])), "r"(__float_as_uint(v[8 * h + 7]))
                     : "memory");
}

// 16 consecutive accumulator columns of one row.  EXT: the kernel form
// that also has the gate (a separate instantiation: the plain GEMMs carry
// none of its code, which measured slower even where it never ran).
template <bool EXT>
__device__ __forceinline__ void epilogue16(const Params &p, int r, int c0, int split,
                                           float (&v)[16])
{
    if (r >= p.M || c0 >= p.N) return;
    const bool first = split == 0;
    const int epi = p.epi;
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= p.alpha;
    if (p.vec && c0 + 16 <= p.N) {
        float t[16];
        if ((epi & EPI_BIAS) && first) {
            ld16f(p.bias + c0, t);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += t[j];
        }
        float *c = p.C + (size_t)r * p.ldc + c0;
        if (epi & EPI_ATOMIC) {
            float4 *c4 = reinterpret_cast<float4 *>(c);
#pragma unroll
            for (int k = 0; k < 4; ++k)
                atomicAdd(c4 + k, make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]));
            return;
        }
        if (epi & EPI_RESID) {
            ld16f(p.R + (size_t)r * p.ldr + c0, t);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += t[j];
        }
        if (epi & EPI_GELU) {
            if (p.aux) st16f(p.aux + (size_t)r * p.ldx + c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = gelu_f(v[j]);
        } else if (epi & EPI_GELU_BWD) {
            ld16f(p.aux + (size_t)r * p.ldx + c0, t);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] *= gelu_d(t[j]);
        } else if (EXT && (epi & EPI_GATE)) {
            ld16f(p.gate + c0, t);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = sigm_f(v[j]) * t[j];
        }
        st16f(c, v);
        return;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int c = c0 + j;
        if (c >= p.N) break;
        float x = v[j];
        if ((epi & EPI_BIAS) && first) x += p.bias[c];
        float *dst = p.C + (size_t)r * p.ldc + c;
        if (epi & EPI_ATOMIC) {
            atomicAdd(dst, x);
            continue;
        }
        if (epi & EPI_RESID) x += p.R[(size_t)r * p.ldr + c];
        if (epi & EPI_GELU) {
            if (p.aux) p.aux[(size_t)r * p.ldx + c] = x;
            x = gelu_f(x);
        } else if (epi & EPI_GELU_BWD) {
            x *= gelu_d(p.aux[(size_t)r * p.ldx + c]);
        } else if (EXT && (epi & EPI_GATE)) {
            x = sigm_f(x) * p.gate[c];
        }
        *dst = x;
    }
}

// Four consecutive columns of one row of a tile reduced over its cluster:
// the whole epilogue (the bias once, no atomics).
__device__ __forceinline__ void epilogue4(const Params &p, int r, int c0, float4 acc)
{
    if (r >= p.M || c0 >= p.N) return;
    const int epi = p.epi;
    float v[4] = {acc.x * p.alpha, acc.y * p.alpha, acc.z * p.alpha, acc.w * p.alpha};
    if (p.vec && c0 + 4 <= p.N) {
        if (epi & EPI_BIAS) {
            const float4 b = *reinterpret_cast<const float4 *>(p.bias + c0);
            v[0] += b.x; v[1] += b.y; v[2] += b.z; v[3] += b.w;
        }
        if (epi & EPI_RESID) {
            const float4 t = *reinterpret_cast<const float4 *>(p.R + (size_t)r * p.ldr + c0);
            v[0] += t.x; v[1] += t.y; v[2] += t.z; v[3] += t.w;
        }
        if (epi & EPI_GELU) {
            if (p.aux)
                *reinterpret_cast<float4 *>(p.aux + (size_t)r * p.ldx + c0) = make_float4(v[0], v[1], v[2], v[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = gelu_f(v[j]);
        } else if (epi & EPI_GELU_BWD) {
            const float4 t = *reinterpret_cast<const float4 *>(p.aux + (size_t)r * p.ldx + c0);
            v[0] *= gelu_d(t.x); v[1] *= gelu_d(t.y); v[2] *= gelu_d(t.z); v[3] *= gelu_d(t.w);
        } else if (epi & EPI_GATE) {
            const float4 t = *reinterpret_cast<const float4 *>(p.gate + c0);
            v[0] = sigm_f(v[0]) * t.x; v[1] = sigm_f(v[1]) * t.y;
            v[2] = sigm_f(v[2]) * t.z; v[3] = sigm_f(v[3]) * t.w;
        }
        *reinterpret_cast<float4 *>(p.C + (size_t)r * p.ldc + c0) = make_float4(v[0], v[1], v[2], v[3]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = c0 + j;
        if (c >= p.N) break;
        float x = v[j];
        if (epi & EPI_BIAS) x += p.bias[c];
        if (epi & EPI_RESID) x += p.R[(size_t)r * p.ldr + c];
        if (epi & EPI_GELU) {
            if (p.aux) p.aux[(size_t)r * p.ldx + c] = x;
            x = gelu_f(x);
        } else if (epi & EPI_GELU_BWD) {
            x *= gelu_d(p.aux[(size_t)r * p.ldx + c]);
        } else if (epi & EPI_GATE) {
            x = sigm_f(x) * p.gate[c];
        }
        p.C[(size_t)r * p.ldc + c] = x;
    }
}

struct Tile {
    int m0, n0, k0, k1, split;
};

__device__ __forceinline__ void st_shared4(uint32_t a, float x, float y, float z, float w)
{
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w)
                 : "memory");
}
__device__ __forceinline__ float4 ld_shared4(uint32_t a)
{
    float4 x;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                 : "r"(a)
                 : "memory");
    return x;
}

// Epilogue of 16 accumulator columns of a warp's 32 rows (all in bounds,
// 16-byte path; split-K partial sums are added with 16-byte atomics).  The tcgen05 load gives lane i row i;
// writing every lane's 64 bytes to global memory directly puts 32 rows, 32
// sectors of 32 different lines, behind each store instruction.  Instead
// the block goes through 2 KB of shared memory (16-byte chunk k of row i at
// chunk k ^ ((i >> 1) & 3), conflict-free both ways) and comes back as four
// lanes per row: every instruction then covers 8 rows x 64 contiguous bytes.
// The streamed inputs (residual, GELU pre-activation) of all 4 passes are
// loaded before the first store (R may alias C: same elements, read first).
template <bool EXT>
__device__ __forceinline__ void epilogue16_staged(const Params &p, int row0, int c0, int split,
                                                  const float (&v)[16], uint32_t sbase, int lane)
{
    const int epi = p.epi;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        st_shared4(sbase + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4), v[4 * k], v[4 * k + 1],
                   v[4 * k + 2], v[4 * k + 3]);
    __syncwarp();
    const int c = lane & 3;
    const int gc = c0 + 4 * c;
    float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
    if ((epi & EPI_BIAS) && split == 0) bb = *reinterpret_cast<const float4 *>(p.bias + gc);
    float4 gt = make_float4(0.f, 0.f, 0.f, 0.f);
    if (EXT && (epi & EPI_GATE)) gt = *reinterpret_cast<const float4 *>(p.gate + gc);
    float4 in[4];
    if (epi & (EPI_RESID | EPI_GELU_BWD)) {
        const float *src = (epi & EPI_RESID) ? p.R : p.aux;
        const int ld = (epi & EPI_RESID) ? p.ldr : p.ldx;
#pragma unroll
        for (int it = 0; it < 4; ++it)
            in[it] = *reinterpret_cast<const float4 *>(
                src + (size_t)(row0 + it * 8 + (lane >> 2)) * ld + gc);
    }
#pragma unroll
    for (int it = 0; it < 4; ++it) {
        const int r = it * 8 + (lane >> 2);
        float4 x = ld_shared4(sbase + r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
        x.x = x.x * p.alpha + bb.x;
        x.y = x.y * p.alpha + bb.y;
        x.z = x.z * p.alpha + bb.z;
        x.w = x.w * p.alpha + bb.w;
        const size_t grow = (size_t)(row0 + r);
        if (epi & EPI_ATOMIC) {
            atomicAdd(reinterpret_cast<float4 *>(p.C + grow * p.ldc + gc), x);
            continue;
        }
        if (epi & EPI_RESID) {
            x.x += in[it].x;
            x.y += in[it].y;
            x.z += in[it].z;
            x.w += in[it].w;
        }
        if (epi & EPI_GELU) {
            if (p.aux) *reinterpret_cast<float4 *>(p.aux + grow * p.ldx + gc) = x;
            x = make_float4(gelu_f(x.x), gelu_f(x.y), gelu_f(x.z), gelu_f(x.w));
        } else if (epi & EPI_GELU_BWD) {
            x.x *= gelu_d(in[it].x);
            x.y *= gelu_d(in[it].y);
            x.z *= gelu_d(in[it].z);
            x.w *= gelu_d(in[it].w);
        } else if (EXT && (epi & EPI_GATE)) {
            x = make_float4(sigm_f(x.x) * gt.x, sigm_f(x.y) * gt.y, sigm_f(x.z) * gt.z,
                            sigm_f(x.w) * gt.w);
        }
        *reinterpret_cast<float4 *>(p.C + grow * p.ldc + gc) = x;
    }
    __syncwarp();  // the staging block is rewritten by the next pass
}

template <int TBN, bool EXT>
__device__ __forceinline__ Tile decode_tile(const Params &p, int idx)
{
    Tile t;
    const int per = p.tiles_m * p.tiles_n;
    // split-major, except under cluster split-K, where a tile's splits are
    // consecutive CTAs (one cluster)
    const bool cl = EXT && p.cl;
    t.split = cl ? idx % p.splits : idx / per;
    const int rem = cl ? idx / p.splits : idx % per;
    t.m0 = (rem / p.tiles_n) * BM;
    t.n0 = (rem % p.tiles_n) * TBN;
    t.k0 = (int)(((long long)t.split * p.ksteps) / p.splits);
    t.k1 = (int)(((long long)(t.split + 1) * p.ksteps) / p.splits);
    return t;
}

__device__ __forceinline__ int sched_tile(int j, int ntiles)
{
    const int t = j * (int)gridDim.x + (int)blockIdx.x;
    return t < ntiles ? t : -1;
}

template <class E, bool A_MN, bool B_MN, int TBN, bool EXT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap mapA,
                   const __grid_constant__ CUtensorMap mapB)
{
    using C = Cfg<E, A_MN, B_MN, TBN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // the staged epilogue's 2 KB a warp: the pipeline stages, free once a
    // CTA's last tile is in TMEM (its MMAs have read every stage, no load follows)
    const uint32_t stg = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = bars + C::STAGES;
    uint64_t *accf = bars + 2 * C::STAGES;
    uint64_t *acce = accf + 2;
    uint64_t *drainb = acce + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drainb + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&accf[s]), 1);
            mbar_init(smem_u32(&acce[s]), kEpiWarps);
        }
        mbar_init(smem_u32(drainb), 1);
        fence_mbar_init();
    }
    if (warp == kEpiWarps && lane == 0) {
        tma_prefetch(&mapA);
        tma_prefetch(&mapB);
    }
    if (warp == kEpiWarps + 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    // programmatic dependent launch: the set-up above overlapped the previous
    // kernel's tail; its outputs are visible from here on
    grid_dep_wait();
    grid_dep_launch();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = p.n_tiles;

    if (warp == kEpiWarps) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool stop = false;
            for (int jt = 0; !stop; ++jt) {
                const int tile = sched_tile(jt, ntiles);
                if (tile < 0) break;
                const Tile tl = decode_tile<TBN, EXT>(p, tile);
                for (int k = tl.k0; k < tl.k1; ++k, ++g) {
                    const int s = g % C::STAGES;
                    if (!mbar_wait(smem_u32(&empty[s]), ((g / C::STAGES) & 1) ^ 1, abort_flag,
                                   p.status, DC_DEVERR_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
                    const uint32_t fb = smem_u32(&full[s]);
                    mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::TILE_BYTES;
                    const int kx = k * C::BKe;
                    if (A_MN) {
#pragma unroll
                        for (int j = 0; j < BM / C::BOX_MN; ++j)
                            tma_load_2d(sa + j * C::MN_LBO, &mapA, fb, tl.m0 + j * C::BOX_MN, kx);
                    } else {
                        tma_load_2d(sa, &mapA, fb, kx, tl.m0);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int j = 0; j < TBN / C::BOX_MN; ++j)
                            tma_load_2d(sb + j * C::MN_LBO, &mapB, fb, tl.n0 + j * C::BOX_MN, kx);
                    } else {
                        // K-major rows in 128-row boxes; the 8-row swizzle
                        // atoms of the second continue those of the first
#pragma unroll
                        for (int j = 0; j < TBN / 128; ++j)
                            tma_load_2d(sb + j * C::TILE_BYTES, &mapB, fb, kx, tl.n0 + 128 * j);
                    }
                }
            }
            if (*abort_flag) {
                const uint32_t first = g > (uint32_t)C::STAGES ? g - C::STAGES : 0;
                for (uint32_t q = first; q < g; ++q)
                    mbar_wait(smem_u32(&full[q % C::STAGES]), (q / C::STAGES) & 1, nullptr,
                              p.status, DC_DEVERR_TIMEOUT_DRAIN);
            }
        }
    } else if (warp == kEpiWarps + 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t g = 0;
            bool stop = false;
            for (uint32_t j = 0; !stop; ++j) {
                const int tile = sched_tile(j, ntiles);
                if (tile < 0) break;
                const Tile tl = decode_tile<TBN, EXT>(p, tile);
                const uint32_t buf = j & 1, use = j >> 1;
                if (!mbar_wait(smem_u32(&acce[buf]), (use & 1) ^ 1, abort_flag, p.status,
                               DC_DEVERR_TIMEOUT_ACC))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + buf * TBN;
                for (int k = tl.k0; k < tl.k1; ++k, ++g) {
                    const int s = g % C::STAGES;
                    if (!mbar_wait(smem_u32(&full[s]), (g / C::STAGES) & 1, abort_flag, p.status,
                                   DC_DEVERR_TIMEOUT_FULL)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::TILE_BYTES;
#pragma unroll
                    for (int u = 0; u < C::NSUB; ++u) {
                        const uint32_t koff = u * C::UK * (int)sizeof(E);
                        const uint32_t moff = u * C::UK * 128;
                        const uint64_t a = A_MN ? sw128_desc(sa + moff, C::MN_LBO, C::MN_SBO,
                                                             C::MN_LAYOUT)
                                                : sw128_desc(sa + koff, 16, 1024, 2);
                        const uint64_t b = B_MN ? sw128_desc(sb + moff, C::MN_LBO, C::MN_SBO,
                                                             C::MN_LAYOUT)
                                                : sw128_desc(sb + koff, 16, 1024, 2);
                        umma<C::TF32>(acc, a, b, C::IDESC, (k == tl.k0 && u == 0) ? 0u : 1u);
                    }
                    umma_commit(smem_u32(&empty[s]));
                }
                if (stop) break;
                umma_commit(smem_u32(&accf[buf]));
            }
            if (*abort_flag) {
                umma_commit(smem_u32(drainb));
                mbar_wait(smem_u32(drainb), 0, nullptr, p.status, DC_DEVERR_TIMEOUT_DRAIN);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0-15)
        const int quad = warp & 3;
        const int slice = warp >> 2;
        const int row = quad * 32 + lane;
        for (uint32_t j = 0;; ++j) {
            const int tile = sched_tile(j, ntiles);
            if (tile < 0) break;
            const Tile tl = decode_tile<TBN, EXT>(p, tile);
            const uint32_t buf = j & 1, use = j >> 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&accf[buf]), use & 1,
                                                              abort_flag, p.status,
                                                              DC_DEVERR_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            // a quarter of the tile's columns per warp of a lane quadrant
            constexpr int QC = TBN / 4;
            const uint32_t lane_addr = tmem + buf * TBN + ((uint32_t)(quad * 32) << 16) + slice * QC;
            if constexpr (EXT) {
                if (p.cl) {
                    // cluster split-K (one tile a CTA): the partial tile goes
                    // to this CTA's stages, free now that its MMAs are
                    // complete, and the cluster adds the partials below
                    if (quad * 32 < p.M - tl.m0) {
#pragma unroll 1
                        for (int sb = 0; sb < QC / 16; ++sb) {
                            float v[16];
                            tmem_ld16(lane_addr + sb * 16, v);
                            const uint32_t dst = stg + (uint32_t)(row * C::RED_LD + slice * QC + sb * 16) * 4u;
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                st_shared4(dst + 16 * k, v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
                        }
                    }
                    tc_fence_before();
                    break;
                }
            }
            // a CTA's last tile (under split-K its only one) goes through the
            // staged form where the warp's 32 rows and the tile's columns are
            // in bounds on the 16-byte path: its shared memory is then free (a
            // residual together with GELU' keeps the row-per-lane form).
            // Staging through memory of its own instead (32 KB more a CTA)
            // sped the GEMMs up alone but slowed the decoder step: fewer other
            // kernels' CTAs could share the SM.
            const bool staged = sched_tile(j + 1, ntiles) < 0 && p.vec &&
                                (p.epi & (EPI_RESID | EPI_GELU_BWD)) != (EPI_RESID | EPI_GELU_BWD) &&
                                tl.m0 + quad * 32 + 32 <= p.M && tl.n0 + TBN <= p.N;
#pragma unroll 1
            for (int sb = 0; sb < QC / 16; ++sb) {
                float v[16];
                tmem_ld16(lane_addr + sb * 16, v);
                if (staged)
                    epilogue16_staged<EXT>(p, tl.m0 + quad * 32, tl.n0 + slice * QC + sb * 16, tl.split, v,
                                           stg + warp * 2048, lane);
                else
                    epilogue16<EXT>(p, tl.m0 + row, tl.n0 + slice * QC + sb * 16, tl.split, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acce[buf]));
        }
    }
    if constexpr (EXT) {
        if (p.cl) {
            // every role of every CTA of the cluster passes both barriers
            __syncwarp();
            cluster_sync_all();  // the cluster's partial tiles are in shared memory
            if (warp < kEpiWarps && !*abort_flag) {
                // CTA `rank` finishes a 1/cl share of the tile's 16-byte
                // cells: the partials added in rank order (the same bits on
                // every run), then the whole epilogue
                const Tile tl = decode_tile<TBN, EXT>(p, blockIdx.x);
                constexpr int C4 = TBN / 4;
                const int total = min(BM, p.M - tl.m0) * C4;
                const int rank = (int)cluster_rank();
                const int beg = (int)((long long)total * rank / p.cl);
                const int end = (int)((long long)total * (rank + 1) / p.cl);
                for (int i = beg + (int)threadIdx.x; i < end; i += kEpiWarps * 32) {
                    const int r = i / C4, c4 = i % C4;
                    const uint32_t a = stg + (uint32_t)(r * C::RED_LD + 4 * c4) * 4u;
                    float4 acc = ld_dsmem_f32x4(smem_in_cta(a, 0));
                    for (int q = 1; q < p.cl; ++q) {
                        const float4 v = ld_dsmem_f32x4(smem_in_cta(a, (uint32_t)q));
                        acc.x += v.x;
                        acc.y += v.y;
                        acc.z += v.z;
                        acc.w += v.w;
                    }
                    epilogue4(p, tl.m0 + r, tl.n0 + 4 * c4, acc);
                }
            }
            __syncwarp();
            cluster_sync_all();  // no CTA leaves while another reads its partial
        }
    }
    __syncthreads();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------ host side
static CUtensorMapDataType tmap_type(int esz)
{
    return esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// Row-major [rows, cols] operand with leading dimension ld (elements).
// K-major: box of BKe (K) x 128 rows, 128-byte swizzle.  MN-major: box of
// one 128-byte MN block x BKe K-rows, in the swizzle tcgen05 reads for that
// majorness (32-byte atoms for 32-bit operands).
static int map_operand(CUtensorMap *m, const void *base, int esz, int rows, int cols, int ld,
                       bool mn_major)
{
    const uint32_t bke = 128 / esz;
    uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
    uint64_t strides[1] = {(uint64_t)ld * esz};
    uint32_t box[2];
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
    if (mn_major) {
        box[0] = 128 / esz;
        box[1] = bke;
        if (esz == 4) sw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    } else {
        box[0] = bke;
        box[1] = 128;
    }
    return encode_tmap(m, tmap_type(esz), 2, base, dims, strides, box, sw);
}

template <class E, bool A_MN, bool B_MN, int TBN, bool EXT>
static int launch(Params p, const void *A, int lda, const void *B, int ldb, cudaStream_t st)
{
    using C = Cfg<E, A_MN, B_MN, TBN>;
    auto kernel = gemm_tc_kernel<E, A_MN, B_MN, TBN, EXT>;
    // per instantiation and device; host threads may race to set them (the
    // attribute call is idempotent), the flags themselves are atomic
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    DC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DC_ERR_UNSUPPORTED, "device ordinal %d", dev);
    if (!attr_set[dev].load(std::memory_order_acquire)) {
        DC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM_BYTES));
        attr_set[dev].store(true, std::memory_order_release);
    }
    const int esz = (int)sizeof(E);
    CUtensorMap mA, mB;
    // A: op(A) is [M,K]; stored [M,K] (K-major) or [K,M] (MN-major)
    DC_TRY(A_MN ? map_operand(&mA, A, esz, p.K, p.M, lda, true)
                : map_operand(&mA, A, esz, p.M, p.K, lda, false));
    // B: op(B) is [K,N]; stored [K,N] (MN-major) or [N,K] (K-major)
    DC_TRY(B_MN ? map_operand(&mB, B, esz, p.K, p.N, ldb, true)
                : map_operand(&mB, B, esz, p.N, p.K, ldb, false));
    if (EXT && p.cl) {
        // cluster split-K: the largest cluster (at most the one asked for)
        // of which one per tile can be resident at once (a cluster's CTAs
        // share a GPC, one CTA fills an SM), so no tile waits for a second wave
        static std::atomic<int> fits[64][9];
        const int tiles = p.tiles_m * p.tiles_n;
        int cl = p.cl;
        for (; cl > 1; --cl) {
            int n = fits[dev][cl].load(std::memory_order_acquire);
            if (n == 0) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3(cl * std::max(1, sm_count() / cl));
                cfg.blockDim = dim3(kThreads);
                cfg.dynamicSmemBytes = C::SMEM_BYTES;
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeClusterDimension;
                at[0].val.clusterDim.x = cl;
                at[0].val.clusterDim.y = 1;
                at[0].val.clusterDim.z = 1;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                DC_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg));
                n = std::max(n, 1);
                fits[dev][cl].store(n, std::memory_order_release);
            }
            if (tiles <= n) break;
        }
        p.cl = cl > 1 ? cl : 0;
        p.splits = cl;
        p.n_tiles = tiles * cl;
    }
    const int grid = p.cl ? p.n_tiles : std::max(1, std::min(p.n_tiles, sm_count()));
    {
        KernelTimer kt("gemm_tc", st);
        DC_CUDA_TRY(launch_pdl(kernel, dim3(grid), dim3(kThreads), C::SMEM_BYTES, st,
                               p.cl ? p.cl : 1, p, mA, mB));
    }
    DC_CUDA_TRY(cudaGetLastError());
    return DC_OK;
}

template <class E, int TBN, bool EXT>
static int dispatch(const Params &p, bool ta, bool tb, const void *A, int lda, const void *B,
                    int ldb, cudaStream_t st)
{
    // op(B) = B   -> B stored [K,N] -> MN-major;  op(B) = B^T -> K-major
    if (!ta && !tb) return launch<E, false, true, TBN, EXT>(p, A, lda, B, ldb, st);
    if (!ta && tb) return launch<E, false, false, TBN, EXT>(p, A, lda, B, ldb, st);
    if (ta && !tb) return launch<E, true, true, TBN, EXT>(p, A, lda, B, ldb, st);
    return launch<E, true, false, TBN, EXT>(p, A, lda, B, ldb, st);
}

template <class E, int TBN>
static int dispatch_ext(const Params &p, bool ta, bool tb, const void *A, int lda, const void *B,
                        int ldb, cudaStream_t st)
{
    // the gate and the cluster split-K live in their own instantiations
    if (p.cl || (p.epi & EPI_GATE)) return dispatch<E, TBN, true>(p, ta, tb, A, lda, B, ldb, st);
    return dispatch<E, TBN, false>(p, ta, tb, A, lda, B, ldb, st);
}

static bool aligned(const void *q, int bytes)
{
    return (reinterpret_cast<uintptr_t>(q) & (uintptr_t)(bytes - 1)) == 0;
}

// dc_gemm and dc_gemm_gate: shapes and flags checked, tiles and splits chosen.
static int gemm_impl(const void *A, int lda, const void *B, int ldb, float *C, int ldc, int M,
                     int N, int K, int dtype, int flags, float alpha, const float *bias,
                     const float *R, int ldr, float *aux, int ldaux, const float *gate, void *stream)
{
    if (M < 0 || N < 0 || K < 0) return fail(DC_ERR_INVALID, "negative shape M=%d N=%d K=%d", M, N, K);
    if ((long long)M * N == 0) return DC_OK;
    if (K == 0) return fail(DC_ERR_INVALID, "K == 0");
    if (dtype != DC_F32 && dtype != DC_BF16) return fail(DC_ERR_INVALID, "dtype %d", dtype);
    if (!A || !B || !C) return fail(DC_ERR_INVALID, "null operand");
    const bool ta = flags & DC_GEMM_TRANS_A, tb = flags & DC_GEMM_TRANS_B;
    const int esz = dtype == DC_F32 ? 4 : 2;
    if (lda < (ta ? M : K) || ldb < (tb ? K : N) || ldc < N)
        return fail(DC_ERR_INVALID, "leading dimension too small (lda=%d ldb=%d ldc=%d)", lda, ldb, ldc);
    if ((lda * esz) % 16 || (ldb * esz) % 16 || !aligned(A, 16) || !aligned(B, 16))
        return fail(DC_ERR_INVALID, "A and B need 16-byte aligned bases and row strides");
    const bool gelu = flags & DC_GEMM_GELU, gelu_bwd = flags & DC_GEMM_GELU_BWD;
    if ((int)gelu + (int)gelu_bwd + (int)(gate != nullptr) > 1)
        return fail(DC_ERR_INVALID, "GELU, GELU_BWD and the gate are exclusive");
    if (gelu_bwd && !aux) return fail(DC_ERR_INVALID, "GELU_BWD needs the pre-activation in aux");
    if ((flags & DC_GEMM_BIAS) && !bias) return fail(DC_ERR_INVALID, "BIAS without a bias vector");
    if (flags & DC_GEMM_ACCUMULATE) {
        if (R && R != C) return fail(DC_ERR_INVALID, "ACCUMULATE with a separate residual");
        R = C;
        ldr = ldc;
    }
    if (R && ldr < N) return fail(DC_ERR_INVALID, "ldr < N");
    if (aux && ldaux < N) return fail(DC_ERR_INVALID, "ldaux < N");

    Params p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.ldc = ldc;
    p.ldr = ldr;
    p.ldx = ldaux;
    p.alpha = alpha;
    p.C = C;
    p.R = R;
    p.bias = bias;
    p.aux = aux;
    p.gate = gate;
    p.epi = ((flags & DC_GEMM_BIAS) ? EPI_BIAS : 0) | (gelu ? EPI_GELU : 0) |
            (gelu_bwd ? EPI_GELU_BWD : 0) | (R ? EPI_RESID : 0) | (gate ? EPI_GATE : 0);
    p.tiles_m = (M + BM - 1) / BM;
    const int sms = sm_count();
    const bool linear = !gelu && !gelu_bwd && !gate;
    // 128 x 256 tiles where they fill at least half the SMs unsplit, or
    // where K is long enough to be split into many long units (the weight
    // gradients' K = B*T): each A tile then feeds twice the outputs
    const int wide_tiles = p.tiles_m * ((N + 255) / 256);
    const int bke = 128 / esz;
    p.ksteps = (K + bke - 1) / bke;
    const bool long_k = linear && p.ksteps >= 128 && 2 * wide_tiles <= sms;
    const int tbn = N >= 256 && (2 * wide_tiles >= sms || long_k) ? 256 : BN;
    p.tiles_n = (N + tbn - 1) / tbn;
    // split K when the tiles leave SMs idle, down to one K step a split (the
    // decode step's 64-row products are latency bound: more, shorter splits
    // measured faster).  A linear epilogue adds the splits with atomics into
    // C (initialised with the residual, or zero, unless the residual is C
    // itself); any other splits over a cluster of up to 8 CTAs a tile that
    // add their partial tiles over distributed shared memory before the
    // epilogue.  Measured on the decode step's 64-row layers (graph-replayed
    // launches): GELU 10.1 us unsplit, 6.9 us over a cluster; a linear layer
    // 5.9 us with atomics and the initialising memset, 6.7 us over a cluster.
    const int tiles = p.tiles_m * p.tiles_n;
    int splits = 1;
    p.cl = 0;
    if (tiles * 2 <= sms) {
        const int most = std::max(1, std::min(sms / tiles, p.ksteps));
        if (linear)
            splits = most;
        else if (std::min(most, 8) >= 2)
            p.cl = splits = std::min(most, 8);
    }
    p.splits = splits;
    p.n_tiles = tiles * splits;
    p.vec = (ldc % 8 == 0) && gemm::aligned(C, 32) && (!R || (ldr % 8 == 0 && gemm::aligned(R, 32))) &&
            (!aux || (ldaux % 8 == 0 && gemm::aligned(aux, 32))) && (!bias || gemm::aligned(bias, 32)) &&
            (!gate || gemm::aligned(gate, 32));
    p.status = device_status_word();
    cudaStream_t st = as_stream(stream);
    if (splits > 1 && !p.cl) {
        // C starts as the residual (or zero) and every split adds its part
        if (!R)
            DC_CUDA_TRY(cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, M, st));
        else if (R != C)
            DC_CUDA_TRY(cudaMemcpy2DAsync(C, (size_t)ldc * 4, R, (size_t)ldr * 4, (size_t)N * 4, M,
                                          cudaMemcpyDeviceToDevice, st));
        p.epi = (p.epi & EPI_BIAS) | EPI_ATOMIC;
    }
    if (tbn == 256) {
        if (dtype == DC_F32) return dispatch_ext<float, 256>(p, ta, tb, A, lda, B, ldb, st);
        return dispatch_ext<__nv_bfloat16, 256>(p, ta, tb, A, lda, B, ldb, st);
    }
    if (dtype == DC_F32) return dispatch_ext<float, BN>(p, ta, tb, A, lda, B, ldb, st);
    return dispatch_ext<__nv_bfloat16, BN>(p, ta, tb, A, lda, B, ldb, st);
}

}  // namespace gemm
}  // namespace dc

using namespace dc;

extern "C" int dc_gemm(const void *A, int lda, const void *B, int ldb, float *C, int ldc, int M,
                       int N, int K, int dtype, int flags, float alpha, const float *bias,
                       const float *R, int ldr, float *aux, int ldaux, void *stream)
{
    clear_error();
    return gemm::gemm_impl(A, lda, B, ldb, C, ldc, M, N, K, dtype, flags, alpha, bias, R, ldr, aux,
                           ldaux, nullptr, stream);
}

extern "C" int dc_gemm_gate(const void *A, int lda, const void *B, int ldb, float *C, int ldc,
                            int M, int N, int K, int dtype, int flags, float alpha,
                            const float *bias, const float *R, int ldr, const float *gate,
                            void *stream)
{
    clear_error();
    if (!gate) return fail(DC_ERR_INVALID, "dc_gemm_gate without a gate vector");
    return gemm::gemm_impl(A, lda, B, ldb, C, ldc, M, N, K, dtype, flags, alpha, bias, R, ldr,
                           nullptr, 0, gate, stream);
}
