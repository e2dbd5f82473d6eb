// Persistent, warp-specialised tcgen05 contraction kernel of the AFT-full
// operator (included by aft.cu; uses its Params, element helpers and modes).
//
// Accumulator rows (TMEM lanes) are the query / key positions and columns are
// channels d, so every epilogue thread owns contiguous runs of d and moves
// them with 32-byte vector loads and stores:
//
//   FWD, BWD1 : acc[t, d]  = sum_i A'[t,i] PV[i,d]   and   sum_i A'[t,i] PE[i,d]
//   HGRAD     : acc[i, d]  = sum_t A'[t,i] G[t,d]    and   sum_t A'[t,i] N[t,d]
//   WGRAD     : acc[t, i]  = sum_{b,d} (G PV^T + N PE^T + G_lo PV^T + N_lo PE^T)
//
// Warp roles (448 threads): warps 0-11 epilogue (warp w reads TMEM lanes
// 32*(w%4).. and, of each row's 16-column sub-blocks, every third one starting
// at w/4), warp 12 TMA producer, warp 13 TMEM allocator + MMA issuer.  Each
// CTA walks its tiles (sched_tile); the accumulator is double-buffered in
// TMEM so the epilogue of one tile overlaps the main loop of the next.
#pragma once

namespace dc {
namespace aft {

// Epilogue warps, a multiple of 4 (a quarter per TMEM lane quadrant).  Twelve
// give 14 warps a CTA, at most 4 per SM sub-partition, so each thread has 128
// registers; sixteen (5 warps on some sub-partitions, 96 registers) measured
// slower in the backward epilogues.
constexpr int kEpiWarps = 12;
constexpr int kTcThreads = (kEpiWarps + 2) * 32;
constexpr int kSmemBudget = 227 * 1024;

// P: the launch runs CTA pairs (cta_group::2): every MMA is M = 256 over the
// pair, each CTA loading its 128 rows of A and half of B.  bf16 operands.
template <int MODE, class E, bool P = false>
struct TcCfg {
    static constexpr bool PAIR = P;
    static constexpr bool TF32 = sizeof(E) == 4;
    static constexpr bool W = MODE == WGRAD;
    static constexpr bool H = MODE == HGRAD;
    // bytes of K per operand row and stage.  dW's four K-major tiles per stage
    // take 128 B rows with CTA pairs (two stages): TMA moves whole 128 B row
    // segments at a markedly higher rate than 64 B ones, which outweighs the
    // shallower pipeline (dW at T = 4096: 354 -> 228 us); single CTAs (short
    // sequences) measured faster with 64 B rows and four stages (T = 512:
    // 32.6 -> 30.3 us).
    static constexpr int KROW = W ? (P ? 128 : 64) : 128;
    static constexpr int BKe = KROW / (int)sizeof(E);  // K elements per stage
    static constexpr int UK = TF32 ? 8 : 16;           // K per MMA instruction
    static constexpr int NSUB = BKe / UK;              // MMAs per stage and operand pair
    static constexpr int BOX_MN = 128 / (int)sizeof(E);// elements in one 128 B MN block
    static constexpr int TILE_BYTES = 128 * KROW;      // one operand tile of 128 rows
    // dW accumulates a 128 x 256 tile (two i blocks): its B tiles have 256 rows
    static constexpr int WN = W ? 2 * BN : BN;         // accumulator columns of one product
    // dW: B rows of one product held by one CTA (K-major)
    static constexpr int BROWS = P ? WN / 2 : WN;
    // One B tile: dW a K-major [BROWS rows] tile; otherwise one MN-major
    // [BN columns] tile of one product (E'V or E'; g or n).  The other modes
    // issue one N = 256 MMA over two adjacent tiles (num | den), so a CTA
    // holds both (or, in a pair, the even CTA the first and the odd the second).
    static constexpr int TILE_B = W ? BROWS * KROW : BN * BKe * (int)sizeof(E);
    static constexpr int MMA_N = W ? WN : 2 * BN;
    // K-major descriptor: swizzle mode (2 = 128 B, 4 = 64 B), 8-row atom stride
    static constexpr uint32_t K_LAYOUT = KROW == 64 ? 4u : 2u;
    static constexpr uint32_t K_SBO = 8 * KROW;
    // dK/dV at tf32 also adds the low parts of g and n (1e-3 bar); dW adds
    // them as a second pass over K with the low-part panels as A
    static constexpr bool LO = H && TF32;
    static constexpr int NA = W ? 2 : 1;               // A tiles per stage
    static constexpr int NB = W ? 2 : (P ? 1 : (LO ? 4 : 2));  // B tiles per stage and CTA
    static constexpr int STAGE_BYTES = NA * TILE_BYTES + NB * TILE_B;
    static constexpr int STAGES_FIT = (kSmemBudget - 2048) / STAGE_BYTES;
    static constexpr int STAGES_MAX = P ? 6 : 4;
    static constexpr int STAGES = STAGES_FIT < STAGES_MAX ? STAGES_FIT : STAGES_MAX;
    static constexpr int NACC = W ? 1 : 2;             // accumulators per tile
    static constexpr uint32_t ACC_COLS = W ? WN : NACC * BN;
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;  // double buffered
    static constexpr uint32_t A_MN = H ? 1 : 0;
    static constexpr uint32_t B_MN = W ? 0 : 1;
    static constexpr uint32_t IDESC = umma_idesc(TF32 ? 2u : 1u, P ? 2 * BM : BM, MMA_N, A_MN, B_MN);
    // half tiles: 64 of a tile's BN columns, one N = 128 MMA over [num | den]
    // (single CTAs with the two B tiles of a stage; see decode_tile)
    static constexpr bool HALF_OK = !W && !P && NB == 2;
    static constexpr uint32_t IDESC_HALF = umma_idesc(TF32 ? 2u : 1u, BM, BN, A_MN, B_MN);
    static_assert(!P || !TF32, "CTA pairs run bf16 operands");
    static constexpr uint32_t MN_LBO = BKe * 128;      // bytes between 128 B MN blocks
    static constexpr uint32_t MN_LAYOUT = TF32 ? 1u : 2u;
    static constexpr uint32_t MN_SBO = TF32 ? 512u : 1024u;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 512;
    static_assert(STAGES >= 2, "pipeline needs two stages");
    static_assert(W || TILE_B == (BN / BOX_MN) * (int)MN_LBO,
                  "adjacent B tiles must continue the MN-block stride (one N = 256 operand)");
    static_assert(SMEM_BYTES <= kSmemBudget, "shared memory budget");
};

// ----------------------------------------------------------- vector I/O
// bf16 <-> fp32 by bit placement: a bf16 is the high half of an fp32.
// One paired conversion (a in the low half): converting the two values one at
// a time costs two instructions on the special-function pipe, which the
// epilogues' exponentials and reciprocals already keep busy.
__device__ __forceinline__ uint32_t pack2(float a, float b)
{
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}
// 256-bit accesses: one full 32-byte sector per thread per instruction
// (sm_100 global v8 loads/stores); callers guarantee 32-byte alignment.
__device__ __forceinline__ void ld32B_nc(const void *p, uint32_t (&r)[8])
{
    asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "l"(p));
}
__device__ __forceinline__ void ld32B(const void *p, uint32_t (&r)[8])
{
    asm volatile("ld.global.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "l"(p)
                 : "memory");
}
__device__ __forceinline__ void st32B(void *p, const uint32_t (&r)[8])
{
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void words_to_f32(const uint32_t (&r)[8], float (&v)[16], int o)
{
#pragma unroll
    for (int k = 0; k < 8; ++k) v[o + k] = __uint_as_float(r[k]);
}
__device__ __forceinline__ void words_to_bf16(const uint32_t (&r)[8], float (&v)[16])
{
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        v[2 * k] = __uint_as_float(r[k] << 16);
        v[2 * k + 1] = __uint_as_float(r[k] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ void ld16g(const float *p, float (&v)[16])
{
    uint32_t r[8];
    ld32B_nc(p, r);
    words_to_f32(r, v, 0);
    ld32B_nc(p + 8, r);
    words_to_f32(r, v, 8);
}
__device__ __forceinline__ void ld16g(const __nv_bfloat16 *p, float (&v)[16])
{
    uint32_t r[8];
    ld32B_nc(p, r);
    words_to_bf16(r, v);
}
// plain (coherent) loads for outputs read back when accumulating
__device__ __forceinline__ void ld16(const float *p, float (&v)[16])
{
    uint32_t r[8];
    ld32B(p, r);
    words_to_f32(r, v, 0);
    ld32B(p + 8, r);
    words_to_f32(r, v, 8);
}
__device__ __forceinline__ void ld16(const __nv_bfloat16 *p, float (&v)[16])
{
    uint32_t r[8];
    ld32B(p, r);
    words_to_bf16(r, v);
}
__device__ __forceinline__ void st16(float *p, const float (&v)[16])
{
    uint32_t r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = __float_as_uint(v[k]);
    st32B(p, r);
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = __float_as_uint(v[8 + k]);
    st32B(p + 8, r);
}
__device__ __forceinline__ void st16(__nv_bfloat16 *p, const float (&v)[16])
{
    uint32_t r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = pack2(v[2 * k], v[2 * k + 1]);
    st32B(p, r);
}
// operand-precision store: bf16, or tf32-rounded fp32
__device__ __forceinline__ void st16op(__nv_bfloat16 *p, const float (&v)[16]) { st16(p, v); }
__device__ __forceinline__ void st16op(float *p, const float (&v)[16])
{
    float r[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) r[k] = to_op<float>(v[k]);
    st16(p, r);
}
__device__ __forceinline__ void round16(const float (&v)[16], float (&hi)[16], float (&lo)[16],
                                        bool bf16)
{
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
        if (bf16) {
            const uint32_t w = pack2(v[k], v[k + 1]);
            hi[k] = __uint_as_float(w << 16);
            hi[k + 1] = __uint_as_float(w & 0xFFFF0000u);
        } else {
            hi[k] = to_op<float>(v[k]);
            hi[k + 1] = to_op<float>(v[k + 1]);
        }
        lo[k] = v[k] - hi[k];
        lo[k + 1] = v[k + 1] - hi[k + 1];
    }
}

__device__ __forceinline__ float fast_sigmoid(float q) { return __fdividef(1.0f, 1.0f + __expf(-q)); }

// ----------------------------------------------------------- epilogues
// One thread, one accumulator row, 16 consecutive columns starting at c0.
// `full` = the row and all 16 columns are inside the logical tensor and the
// tensors allow 32-byte vector access; otherwise an element-wise path runs.

// The epilogue's element-wise inputs (Q; Q and dZ; K and V) for bf16 tensors,
// loaded before the accumulator is ready so their latency overlaps the main
// loop.  ok = false: the epilogue loads them itself (other types, partial
// columns or rows, accumulate mode).  Used by the forward only: holding the
// two inputs of the backward epilogues this way spills under the 128-register
// budget and measured slower.
struct EpiPre {
    uint32_t a[8], b[8];
    bool ok;
};

template <int MODE, class IO>
__device__ __forceinline__ void epi_prefetch(const Params &p, int bb, int r, int c0, EpiPre &pf)
{
    pf.ok = false;
    if constexpr (sizeof(IO) == 2 && MODE == FWD) {
        const int rows = MODE == HGRAD ? p.Tk : p.Tq;
        if (!p.vec_io || p.accumulate || c0 + 16 > p.D || r >= rows) return;
        const size_t o = ((size_t)bb * rows + r) * p.ldi + c0;
        if (MODE == HGRAD) {
            ld32B_nc((const IO *)p.K + o, pf.a);
            ld32B_nc((const IO *)p.V + o, pf.b);
        } else {
            ld32B_nc((const IO *)p.Q + o, pf.a);
            if (MODE == BWD1)
                ld32B_nc((const IO *)p.dZ + ((size_t)bb * rows + r) * p.ldo + c0, pf.b);
        }
        pf.ok = true;
    }
}

// Range guard of the factorised stabilisation: an output whose denominator
// den' (the sum of e^{w-m_t} e^{K-c_d} over the visible keys) is below 2^-100,
// or whose numerator is not finite, is outside the range the factorisation
// resolves (the reference's joint maximum never is); the call then reports
// DC_DEVERR_RANGE in the device status word instead of passing inf or NaN on
// silently.  Terms below 2^-126 that the operands or products lose are then
// at most 2^-26 of den'.
__device__ __forceinline__ bool out_of_range(float num, float den)
{
    return !(den >= 0x1p-100f) || !(fabsf(num) <= 3.0e38f);
}
__device__ __forceinline__ void report_range(const Params &p)
{
    if (p.status) atomicOr(p.status, DC_DEVERR_RANGE);
}

template <class IO, class E>
__device__ __forceinline__ void epi16_fwd(const Params &p, int b, int t, int d0,
                                          const float (&num)[16], const float (&den)[16],
                                          const EpiPre &pf)
{
    if (t >= p.Tq) return;
    {
        bool bad = false;
#pragma unroll
        for (int j = 0; j < 16; ++j) bad |= d0 + j < p.D && out_of_range(num[j], den[j]);
        if (bad) report_range(p);
    }
    if (p.Rs) {  // r and 1/den for the backward, exactly as epi16_bwd1 forms them
        float r[16], inv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            inv[j] = __fdividef(1.0f, den[j]);
            r[j] = num[j] * inv[j];
        }
        if (t < p.stat_lo) {  // fp32 (rows whose g and n keep residuals)
            const size_t so = ((size_t)b * p.stat_lo + t) * p.dp + d0;
            st16(p.Rs + so, r);
            st16(p.Is + so, inv);
        } else {              // operand precision
            const size_t so = ((size_t)b * p.Tqp + t) * p.dp + d0;
            st16op((E *)p.Rb + so, r);
            st16op((E *)p.Ib + so, inv);
        }
    }
    const size_t row = (size_t)b * p.Tq + t;
    const size_t o = row * p.ldi + d0, oz = row * p.ldo + d0;
    if (p.vec_io && d0 + 16 <= p.D) {
        float q[16], z[16];
        if (pf.ok)
            words_to_bf16(pf.a, q);
        else
            ld16g((const IO *)p.Q + o, q);
#pragma unroll
        for (int j = 0; j < 16; ++j) z[j] = __fdividef(num[j], den[j] * (1.0f + __expf(-q[j])));
        st16((IO *)p.Z + oz, z);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (d0 + j >= p.D) break;
            const float q = ld_io((const IO *)p.Q, o + j);
            st_io((IO *)p.Z, oz + j, __fdividef(num[j], den[j] * (1.0f + __expf(-q))));
        }
    }
}

// dQ, and g = dZ*sigmoid(Q)/den and n = -g*r as operand panels, from the
// forward's r = num/den and inv = 1/den of 16 columns of row t.
template <class IO, class E>
__device__ __forceinline__ void epi16_grads(const Params &p, int b, int t, int d0,
                                            const float (&rr)[16], const float (&iv)[16],
                                            const EpiPre &pf)
{
    float g[16], n[16];
    const bool trow = t < p.Tq;
    const size_t row = (size_t)b * p.Tq + t;
    const size_t o = row * p.ldi + d0, oz = row * p.ldo + d0;
    if (trow && p.vec_io && d0 + 16 <= p.D) {
        float q[16], dz[16], dq[16];
        if (pf.ok) {
            words_to_bf16(pf.a, q);
            words_to_bf16(pf.b, dz);
        } else {
            ld16g((const IO *)p.Q + o, q);
            ld16g((const IO *)p.dZ + oz, dz);
        }
        if (p.accumulate) ld16((const IO *)p.dQ + o, dq);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float s = fast_sigmoid(q[j]);
            const float inv = iv[j];
            const float r = rr[j];
            const float add = dz[j] * r * s * (1.0f - s);
            dq[j] = p.accumulate ? dq[j] + add : add;
            g[j] = dz[j] * s * inv;
            n[j] = -g[j] * r;
        }
        st16((IO *)p.dQ + o, dq);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            g[j] = 0.f;
            n[j] = 0.f;
        }
        if (trow) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                if (d0 + j >= p.D) break;
                const float q = ld_io((const IO *)p.Q, o + j);
                const float dz = ld_io((const IO *)p.dZ, oz + j);
                const float s = fast_sigmoid(q);
                const float inv = iv[j];
                const float r = rr[j];
                float dq = dz * r * s * (1.0f - s);
                if (p.accumulate) dq += ld_io((const IO *)p.dQ, o + j);
                st_io((IO *)p.dQ, o + j, dq);
                g[j] = dz * s * inv;
                n[j] = -g[j] * r;
            }
        }
    }
    // g, n and their rounding residuals, over the whole padded tile
    const size_t go = ((size_t)b * p.Tqp + t) * p.dp + d0;
    float hi[16], lo[16];
    constexpr bool BF = sizeof(E) == 2;
    if (t < p.lo_rows) {
        round16(g, hi, lo, BF);
        st16op((E *)p.G1 + go, hi);
        st16op((E *)p.G1l + go, lo);
        round16(n, hi, lo, BF);
        st16op((E *)p.G2 + go, hi);
        st16op((E *)p.G2l + go, lo);
    } else {  // the operand-precision store rounds exactly as round16's hi
        st16op((E *)p.G1 + go, g);
        st16op((E *)p.G2 + go, n);
    }
}

template <class IO, class E>
__device__ __forceinline__ void epi16_bwd1(const Params &p, int b, int t, int d0,
                                           const float (&num)[16], const float (&den)[16],
                                           const EpiPre &pf)
{
    if (t < p.Tq) {  // the range guard of epi16_fwd
        bool bad = false;
#pragma unroll
        for (int j = 0; j < 16; ++j) bad |= d0 + j < p.D && out_of_range(num[j], den[j]);
        if (bad) report_range(p);
    }
    float r[16], inv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        inv[j] = __fdividef(1.0f, den[j]);
        r[j] = num[j] * inv[j];
    }
    epi16_grads<IO, E>(p, b, t, d0, r, inv, pf);
}

template <class IO>
__device__ __forceinline__ void epi16_hgrad(const Params &p, int b, int i, int d0,
                                            const float (&h1)[16], const float (&h2)[16],
                                            const EpiPre &pf)
{
    if (i >= p.Tk) return;
    const size_t o = ((size_t)b * p.Tk + i) * p.ldi + d0;
    const float *cb = p.c + (size_t)b * p.dp + d0;
    if (p.vec_io && d0 + 16 <= p.D) {
        float k[16], v[16], c[16], dk[16], dv[16];
        if (pf.ok) {
            words_to_bf16(pf.a, k);
            words_to_bf16(pf.b, v);
        } else {
            ld16g((const IO *)p.K + o, k);
            ld16g((const IO *)p.V + o, v);
        }
        ld16g(cb, c);
        if (p.accumulate) {
            ld16((const IO *)p.dK + o, dk);
            ld16((const IO *)p.dV + o, dv);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float e = __expf(k[j] - c[j]);
            const float a = e * h1[j], bk = e * (v[j] * h1[j] + h2[j]);
            dv[j] = p.accumulate ? dv[j] + a : a;
            dk[j] = p.accumulate ? dk[j] + bk : bk;
        }
        st16((IO *)p.dV + o, dv);
        st16((IO *)p.dK + o, dk);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (d0 + j >= p.D) break;
            const float e = __expf(ld_io((const IO *)p.K, o + j) - cb[j]);
            const float v = ld_io((const IO *)p.V, o + j);
            float dv = e * h1[j], dk = e * (v * h1[j] + h2[j]);
            if (p.accumulate) {
                dv += ld_io((const IO *)p.dV, o + j);
                dk += ld_io((const IO *)p.dK, o + j);
            }
            st_io((IO *)p.dV, o + j, dv);
            st_io((IO *)p.dK, o + j, dk);
        }
    }
}

__device__ __forceinline__ void epi16_wgrad(const Params &p, int t, int i0, const float (&acc)[16])
{
    if (t >= p.Tq || i0 >= p.Tk || (p.causal && i0 > t)) return;
    const float m = __ldg(p.m + t);
    const float *w = p.w + (size_t)t * p.ldw;
    float *dW = dw_row(p, t);
    if (p.vec_w && i0 + 16 <= p.Tk && (!p.causal || i0 + 15 <= t)) {
        float wv[16];
        ld16g(w + i0, wv);
        float4 *d4 = reinterpret_cast<float4 *>(dW + i0);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float4 v;
            v.x = __expf(wv[4 * k] - m) * acc[4 * k];
            v.y = __expf(wv[4 * k + 1] - m) * acc[4 * k + 1];
            v.z = __expf(wv[4 * k + 2] - m) * acc[4 * k + 2];
            v.w = __expf(wv[4 * k + 3] - m) * acc[4 * k + 3];
            atomicAdd(d4 + k, v);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = i0 + j;
            if (i < p.Tk && (!p.causal || i <= t)) atomicAdd(dW + i, __expf(__ldg(w + i) - m) * acc[j]);
        }
    }
}

// dW[Tq][Tk] (row stride ldw) set to zero by `count` threads, this one being
// thread `i` of them: the first backward kernel clears it for dW's split-K
// atomics (the dW launch waits for that kernel to complete).
__device__ __forceinline__ void zero_dw(const Params &p, size_t i, size_t count)
{
    if (p.dw_packed) {  // one contiguous run (a multiple of 8 floats)
        const size_t n = dw_packed_floats(p.Tq, p.Tk);
        if (p.vec_w) {
            for (size_t e = i; e < n / 4; e += count)
                reinterpret_cast<float4 *>(p.dW)[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            for (size_t e = i; e < n; e += count) p.dW[e] = 0.f;
        }
        return;
    }
    if (p.vec_w) {  // rows of whole float4s (ldw % 8 == 0, 32-byte aligned base)
        const size_t per = (size_t)(p.Tk + 3) / 4, n = per * p.Tq;
        for (size_t e = i; e < n; e += count) {
            const size_t t = e / per, c = (e % per) * 4;
            float *row = p.dW + t * p.ldw;
            if (c + 3 < (size_t)p.Tk) {
                *reinterpret_cast<float4 *>(row + c) = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                for (size_t k = c; k < (size_t)p.Tk; ++k) row[k] = 0.f;
            }
        }
    } else {
        const size_t n = (size_t)p.Tq * p.Tk;
        for (size_t e = i; e < n; e += count) p.dW[(e / p.Tk) * p.ldw + e % p.Tk] = 0.f;
    }
}

// ----------------------------------------------------------- tile schedule
struct Tile {
    int b, mrow, ncol;  // mrow/ncol: 128-row block of the accumulator / column block
    int k0, k1;         // K steps [k0, k1); WGRAD: of the tile's passes laid end to end
    int kt;             // WGRAD: K steps of one pass (steps from kt on read the low parts)
    int half;           // -1: all BN columns; 0 or 1: that half of them (N = 128 MMA)
};

// dW tiles of a causal launch: row block r holds r/2 + 1 column pairs, so
// the rows before r hold S(r) pairs: S(2m) = m(m+1), S(2m+1) = (m+1)^2.
__host__ __device__ __forceinline__ int wgrad_pairs_before(int r)
{
    const int m = r >> 1;
    return (r & 1) ? (m + 1) * (m + 1) : m * (m + 1);
}

// A tile's rows are 128-blocks (one CTA) or pairs of 128-blocks (P: the two
// CTAs of a pair, block 2*mrow + rank each); RB is the rows it spans.
template <int MODE, int BKe, bool P = false>
__device__ __forceinline__ Tile decode_tile(const Params &p, int idx)
{
    constexpr int RB = P ? 2 * BM : BM;
    Tile t{};
    t.kt = 0x7fffffff;
    t.half = -1;
    if (MODE != WGRAD) {
        // Tiles in bundles of two of one group g = (b, column block d): row
        // levels q and nm-1-q, whose K lengths sum to the same total for every
        // q (causal; all equal otherwise), heavy tile first.  Bundles run
        // group-major; with nm odd the middle-level tiles of all groups follow,
        // paired with each other.
        // Without bundles the tiles come heavy level first, one per unit;
        // units from n_full on are halves of the remaining (lightest) tiles,
        // which spread a last, partial round over all workers.
        const int nd = (p.dp + BN - 1) / BN;
        const int nm = (MODE == HGRAD ? p.Tkp : p.Tqp) / RB;
        const int nb = nm / 2;
        const int bundles = nd * p.B * nb;
        const int u = idx >> 1;
        int g, level;  // level 0 = the lightest row level
        if (!p.bundled) {
            int tt = idx;
            if (idx >= p.n_full) {
                tt = p.n_full + ((idx - p.n_full) >> 1);
                t.half = (idx - p.n_full) & 1;
            }
            g = tt % (nd * p.B);
            level = nm - 1 - tt / (nd * p.B);
        } else if (u < bundles) {
            g = u / nb;
            const int q = u % nb;
            level = (idx & 1) ? q : nm - 1 - q;
        } else {
            g = idx - 2 * bundles;
            level = nm / 2;
        }
        t.ncol = g % nd;
        t.b = g / nd;
        // narrow panels (64 columns): every tile is the first half of one
        // (HGRAD at tf32 keeps whole tiles: its loads past column 64 read the
        // tensor maps' zero fill and its epilogue stops at D)
        if (p.narrow && !(MODE == HGRAD && BKe == 32)) t.half = 0;
        if (MODE == HGRAD) {  // early key rows see the most query rows
            t.mrow = nm - 1 - level;
            t.k0 = p.causal ? (t.mrow * RB) / BKe : 0;
            t.k1 = p.Tqp / BKe;
        } else {
            t.mrow = level;
            t.k0 = 0;
            t.k1 = (p.causal ? min(p.Tkp, (t.mrow + 1) * RB) : p.Tkp) / BKe;
        }
    } else {
        // RB query rows x 256 keys (two 128-blocks); ncol counts the key pairs.
        // Units: split s of tile u, where tiles sk_tiles.. are the low-part
        // passes of the first sk_lo tiles (kept separate so that every unit
        // has the same K length and all workers walk K together)
        const int u = idx / p.splits, s = idx % p.splits;
        const bool lo = u >= p.sk_tiles;
        const int pair = lo ? u - p.sk_tiles : u;
        if (!p.causal) {
            const int np = (p.Tkp / BN + 1) / 2;
            t.mrow = pair / np;
            t.ncol = pair % np;
        } else if (P) {
            // row pair m holds key pairs 0..m: triangular
            int r = (int)((sqrtf(8.0f * (float)pair + 1.0f) - 1.0f) * 0.5f);
            while ((r + 1) * (r + 2) / 2 <= pair) ++r;
            while (r * (r + 1) / 2 > pair) --r;
            t.mrow = r;
            t.ncol = pair - r * (r + 1) / 2;
        } else {
            int r = (int)(2.0f * sqrtf((float)pair)) - 1;  // S(r) ~ r^2/4: start just below
            if (r < 0) r = 0;
            while (r > 0 && wgrad_pairs_before(r) > pair) --r;
            while (wgrad_pairs_before(r + 1) <= pair) ++r;
            t.mrow = r;
            t.ncol = pair - wgrad_pairs_before(r);
        }
        const int kt = p.kpb * p.B;
        t.kt = kt;
        t.k0 = (int)(((long long)s * kt) / p.splits) + (lo ? kt : 0);
        t.k1 = (int)(((long long)(s + 1) * kt) / p.splits) + (lo ? kt : 0);
    }
    return t;
}

// Tile of this CTA's (or CTA pair's) j-th iteration, -1 once it has no more.
// Units are dealt boustrophedon (round r even: worker c, odd: G-1-c): for
// FWD/BWD1/HGRAD with at least two tiles a worker (p.bundled) a unit is a
// bundle of two tiles with equal K sums (decode_tile), so every worker gets
// the same main-loop work up to one bundle; otherwise, and for WGRAD, a unit
// is one tile (WGRAD: one split of one tile or low-part pass).
template <int MODE, bool P = false>
__device__ __forceinline__ int sched_tile(const Params &p, int j, int ntiles)
{
    const int G = P ? gridDim.x >> 1 : gridDim.x, c = P ? blockIdx.x >> 1 : blockIdx.x;
    const bool bundles = MODE != WGRAD && p.bundled;
    const int r = bundles ? j >> 1 : j;
    const int unit = r * G + ((r & 1) ? (G - 1 - c) : c);
    const int t = bundles ? 2 * unit + (j & 1) : unit;
    return t < ntiles ? t : -1;
}

// Optional per-tile timeline (Params::trace): 8 words per (CTA, local tile):
// 0 producer start, 1 MMA start, 2 MMA done, 3 epilogue start, 4 epilogue
// done (global-timer ns), 5 tile index, 6 K steps.  Up to 64 tiles per CTA.
__device__ __forceinline__ void trace_at(const Params &p, int j, int field, unsigned long long v)
{
    if (p.trace && j < 64) p.trace[((size_t)blockIdx.x * 64 + j) * 8 + field] = v;
}

// ----------------------------------------------------------- the kernel
// With P the grid is made of 2-CTA clusters: both CTAs load their halves of
// every stage (completion counted on the even CTA's barrier), the even CTA
// issues the pair's MMAs and signals both CTAs' barriers, and each CTA's
// epilogue drains its own 128 accumulator rows and reports to the even CTA.
template <int MODE, class E, class IO, bool P>
__global__ void __launch_bounds__(kTcThreads, 1)
    aft_tc_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap mapA,
                  const __grid_constant__ CUtensorMap mapB1,
                  const __grid_constant__ CUtensorMap mapB2,
                  const __grid_constant__ CUtensorMap mapB3,
                  const __grid_constant__ CUtensorMap mapB4,
                  const __grid_constant__ CUtensorMap mapA2,
                  const __grid_constant__ CUtensorMap mapA3,
                  const __grid_constant__ CUtensorMap mapA4)
{
    using C = TcCfg<MODE, E, P>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full = bars;                   // [STAGES]  TMA -> MMA
    uint64_t *empty = bars + C::STAGES;      // [STAGES]  MMA -> TMA
    uint64_t *accf = bars + 2 * C::STAGES;   // [2]       MMA -> epilogue
    uint64_t *acce = accf + 2;               // [2]       epilogue -> MMA
    uint64_t *drainb = acce + 2;             // [1]       MMA drain after an abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drainb + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = P ? cluster_rank() : 0;  // CTA of the pair (0 issues the MMAs)
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&accf[s]), 1);
            mbar_init(smem_u32(&acce[s]), P ? 2 * kEpiWarps : kEpiWarps);
        }
        mbar_init(smem_u32(drainb), 1);
        fence_mbar_init();
    }
    if (warp == kEpiWarps && lane == 0) {
        tma_prefetch(&mapA);
        tma_prefetch(&mapB1);
        tma_prefetch(&mapB2);
        if (C::NB == 4) {
            tma_prefetch(&mapB3);
            tma_prefetch(&mapB4);
        }
        if (C::W) {
            tma_prefetch(&mapA2);
            tma_prefetch(&mapA3);
            tma_prefetch(&mapA4);
        }
    }
    if (warp == kEpiWarps + 1) {
        if constexpr (P) {
            tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    // a pair's barriers must be initialised before either CTA signals them
    if constexpr (P)
        cluster_sync_all();
    else
        __syncthreads();
    tc_fence_after();
    // the set-up above overlapped the previous kernel's tail; its results are
    // visible from here on (programmatic dependent launch)
    grid_dep_wait();
    grid_dep_launch();
    const uint32_t tmem = *tmem_slot;
    const int ntiles = p.n_tiles;
    auto ld2 = [&](uint32_t dst, const CUtensorMap *m, uint32_t bar, int c0, int c1) {
        if constexpr (P)
            tma_load_2d_pair(dst, m, bar, c0, c1);
        else
            tma_load_2d(dst, m, bar, c0, c1);
    };
    auto ld3 = [&](uint32_t dst, const CUtensorMap *m, uint32_t bar, int c0, int c1, int c2) {
        if constexpr (P)
            tma_load_3d_pair(dst, m, bar, c0, c1, c2);
        else
            tma_load_3d(dst, m, bar, c0, c1, c2);
    };

    if (warp == kEpiWarps) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t g = 0;
            bool stop = false;
            for (int jt = 0; !stop; ++jt) {
                const int tile = sched_tile<MODE, P>(p, jt, ntiles);
                if (tile < 0) break;
                const Tile tl = decode_tile<MODE, C::BKe, P>(p, tile);
                trace_at(p, jt, 0, global_timer());
                // this CTA's accumulator rows and its share of B's columns / rows
                const int m0 = (P ? 2 * tl.mrow + (int)rank : tl.mrow) * BM;
                const int bofs = (int)rank * C::BROWS;  // dW: this CTA's key rows
                for (int e = tl.k0; e < tl.k1; ++e, ++g) {
                    const bool lo = e >= tl.kt;  // dW: the low-part pass
                    const int k = lo ? e - tl.kt : e;
                    const int s = g % C::STAGES;
                    const uint32_t ph = (g / C::STAGES) & 1;
                    if (!mbar_wait<P>(smem_u32(&empty[s]), ph ^ 1, abort_flag, p.status,
                                   DC_DEVERR_TIMEOUT_EMPTY)) {
                        stop = true;
                        break;
                    }
#ifdef DC_TEST_WITHHOLD
                    // test build: CTA 0 withholds its first stage (no arrival,
                    // no copy), so the consumer's bounded wait runs out
                    if (p.test_withhold && blockIdx.x == 0 && jt == 0 && e == tl.k0) continue;
#endif
                    // both CTAs' copies complete on the even CTA's barrier
                    const uint32_t fb = P ? smem_in_cta(smem_u32(&full[s]), 0) : smem_u32(&full[s]);
                    // a half tile loads half of each B tile
                    const int bytes = C::STAGE_BYTES - (tl.half >= 0 ? C::TILE_B : 0);
                    if (leader) mbar_arrive_expect_tx(smem_u32(&full[s]), (P ? 2 : 1) * bytes);
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::NA * C::TILE_BYTES;
                    if (MODE == FWD || MODE == BWD1 || MODE == HGRAD) {
                        if (MODE == HGRAD) {
                            // A: A'[t rows (K), i cols (M)] MN-major
#pragma unroll
                            for (int j = 0; j < BM / C::BOX_MN; ++j)
                                ld2(sa + j * C::MN_LBO, &mapA, fb, m0 + j * C::BOX_MN, k * C::BKe);
                        } else {
                            // A: A'[t rows, i cols] K-major
                            ld2(sa, &mapA, fb, k * C::BKe, m0);
                        }
                        // B: [PV | PE] or [G | N] (then [G lo | N lo]) [K rows, d cols]
                        // MN-major, one BN-column tile each; a pair splits them.
                        // A half tile loads its half of both, the second right
                        // after the first (one N = 128 operand).
                        const int nbx = (tl.half >= 0 ? BN / 2 : BN) / C::BOX_MN;
                        const int x0 = tl.ncol * BN + (tl.half > 0 ? BN / 2 : 0);
#pragma unroll
                        for (int j = 0; j < BN / C::BOX_MN; ++j) {
                            if (j >= nbx) break;
                            const int x = x0 + j * C::BOX_MN;
                            const uint32_t o = sb + j * C::MN_LBO;
                            if (P) {
                                ld3(o, rank ? &mapB2 : &mapB1, fb, x, k * C::BKe, tl.b);
                            } else {
                                ld3(o, &mapB1, fb, x, k * C::BKe, tl.b);
                                ld3(o + nbx * C::MN_LBO, &mapB2, fb, x, k * C::BKe, tl.b);
                                if (C::NB == 4) {
                                    ld3(o + 2 * C::TILE_B, &mapB3, fb, x, k * C::BKe, tl.b);
                                    ld3(o + 3 * C::TILE_B, &mapB4, fb, x, k * C::BKe, tl.b);
                                }
                            }
                        }
                    } else {
                        // A: G, N (first pass) or their low parts (second pass) [t rows, d]
                        // K-major; B: PV, PE [256 i rows, d] K-major
                        const int bb = k / p.kpb, x = (k % p.kpb) * C::BKe;
                        ld3(sa, lo ? &mapA3 : &mapA, fb, x, m0, bb);
                        ld3(sa + C::TILE_BYTES, lo ? &mapA4 : &mapA2, fb, x, m0, bb);
                        ld3(sb, &mapB1, fb, x, tl.ncol * C::WN + bofs, bb);
                        ld3(sb + C::TILE_B, &mapB2, fb, x, tl.ncol * C::WN + bofs, bb);
                    }
                }
            }
            if (*abort_flag && leader) {
                // let the copies already in flight land before the CTA exits (a
                // pair's barriers live in the even CTA, which the odd one awaits
                // at the final cluster barrier)
                const uint32_t first = g > (uint32_t)C::STAGES ? g - C::STAGES : 0;
                for (uint32_t q = first; q < g; ++q)
                    mbar_wait(smem_u32(&full[q % C::STAGES]), (q / C::STAGES) & 1, nullptr,
                              p.status, DC_DEVERR_TIMEOUT_DRAIN);
            }
        }
    } else if (warp == kEpiWarps + 1) {
        // ------------------------------------------------ MMA issuer (even CTA of a pair)
        auto mma = [&](uint32_t d, uint64_t a, uint64_t b, uint32_t acc_on,
                       uint32_t idesc = C::IDESC) {
            if constexpr (P)
                umma_pair(d, a, b, idesc, acc_on);
            else
                umma<C::TF32>(d, a, b, idesc, acc_on);
        };
        auto commit = [&](uint32_t bar) {
            if constexpr (P)
                umma_commit_pair(bar);
            else
                umma_commit(bar);
        };
        if (lane == 0 && leader) {
            uint32_t g = 0, j = 0;
            bool stop = false;
            for (; !stop; ++j) {
                const int tile = sched_tile<MODE, P>(p, j, ntiles);
                if (tile < 0) break;
                const Tile tl = decode_tile<MODE, C::BKe, P>(p, tile);
                const uint32_t buf = j & 1, use = j >> 1;
                // both CTAs' epilogues report here (cluster-scope acquire)
                if (!mbar_wait<P>(smem_u32(&acce[buf]), (use & 1) ^ 1, abort_flag, p.status,
                                  DC_DEVERR_TIMEOUT_ACC))
                    break;
                tc_fence_after();
                trace_at(p, j, 1, global_timer());
                trace_at(p, j, 5, tile);
                trace_at(p, j, 6, tl.k1 - tl.k0);
                const uint32_t acc = tmem + buf * C::ACC_COLS;
                const int nsteps = tl.k1 - tl.k0;
                for (int js = 0; js < nsteps; ++js, ++g) {
                    const int s = g % C::STAGES;
                    if (!mbar_wait<P>(smem_u32(&full[s]), (g / C::STAGES) & 1, abort_flag, p.status,
                                   DC_DEVERR_TIMEOUT_FULL)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::NA * C::TILE_BYTES;
#pragma unroll
                    for (int u = 0; u < C::NSUB; ++u) {
                        const uint32_t first = (js == 0 && u == 0) ? 0u : 1u;
                        const uint32_t koff = u * C::UK * (int)sizeof(E);  // K-major step
                        const uint32_t moff = u * C::UK * 128;             // MN-major step
                        if (C::W) {
                            // acc[128 or 256 t, 256 i] += G . PV^T + N . PE^T (or their low parts)
                            const uint64_t b1 = sw128_desc(sb + koff, 16, C::K_SBO, C::K_LAYOUT);
                            const uint64_t b2 =
                                sw128_desc(sb + C::TILE_B + koff, 16, C::K_SBO, C::K_LAYOUT);
                            mma(acc, sw128_desc(sa + koff, 16, C::K_SBO, C::K_LAYOUT), b1, first);
                            mma(acc, sw128_desc(sa + C::TILE_BYTES + koff, 16, C::K_SBO, C::K_LAYOUT),
                                b2, 1u);
                        } else {
                            const uint64_t a = C::H ? sw128_desc(sa + moff, C::MN_LBO, C::MN_SBO,
                                                                 C::MN_LAYOUT)
                                                    : sw128_desc(sa + koff, 16, C::K_SBO, C::K_LAYOUT);
                            // acc[:, 0:2BN] = [num | den]: one N = 256 MMA over the
                            // two adjacent B tiles (their MN blocks are MN_LBO apart)
                            const uint64_t b = sw128_desc(sb + moff, C::MN_LBO, C::MN_SBO, C::MN_LAYOUT);
                            mma(acc, a, b, first, tl.half >= 0 ? C::IDESC_HALF : C::IDESC);
                            if (C::NB == 4) {
                                const uint64_t bl = sw128_desc(sb + 2 * C::TILE_B + moff, C::MN_LBO,
                                                               C::MN_SBO, C::MN_LAYOUT);
                                mma(acc, a, bl, 1u);
                            }
                        }
                    }
                    commit(smem_u32(&empty[s]));
                }
                if (stop) break;
                commit(smem_u32(&accf[buf]));
                trace_at(p, j, 2, global_timer());
            }
            if (*abort_flag) {  // MMAs must finish before TMEM is released
                commit(smem_u32(drainb));
                mbar_wait(smem_u32(drainb), 0, nullptr, p.status, DC_DEVERR_TIMEOUT_DRAIN);
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps
        // warp w reads TMEM lanes 32*(w%4).. (its quadrant's rows) and, of the
        // row's 16-column sub-blocks, every QW-th starting at w/4
        constexpr int QW = kEpiWarps / 4;          // warps per lane quadrant
        constexpr int NSB = C::WN / 16;            // 16-column sub-blocks per row
        constexpr int MAXK = (NSB + QW - 1) / QW;  // sub-blocks per warp, at most
        const int quad = warp & 3;
        const int slice = warp >> 2;
        const int row = quad * 32 + lane;
        for (uint32_t j = 0;; ++j) {
            const int tile = sched_tile<MODE, P>(p, j, ntiles);
            if (tile < 0) break;
            const Tile tl = decode_tile<MODE, C::BKe, P>(p, tile);
            const uint32_t buf = j & 1, use = j >> 1;
            // t (FWD, BWD1, WGRAD) or i (HGRAD): this CTA's 128 rows of the tile
            const int r = (P ? 2 * tl.mrow + (int)rank : tl.mrow) * BM + row;
            // first column (d, or i for WGRAD); a half tile's 64 columns hold
            // num and den at accumulator columns 0 and 64 (else 0 and BN)
            const int cb0 = tl.ncol * C::WN + (tl.half > 0 ? BN / 2 : 0);
            const int nsb = tl.half >= 0 ? NSB / 2 : NSB;
            const uint32_t dofs = tl.half >= 0 ? BN / 2 : BN;
            // element-wise inputs requested while the main loop still runs
            EpiPre pf[C::W ? 1 : MAXK];
            if constexpr (!C::W) {
#pragma unroll
                for (int k = 0; k < MAXK; ++k) {
                    const int sb = slice + k * QW;
                    pf[k].ok = false;
                    if (sb < nsb) epi_prefetch<MODE, IO>(p, tl.b, r, cb0 + sb * 16, pf[k]);
                }
            }
            // warp-uniform, because the TMEM loads below are warp-collective
            const bool ok = __all_sync(0xffffffffu, mbar_wait<P>(smem_u32(&accf[buf]), use & 1,
                                                                 abort_flag, p.status,
                                                                 DC_DEVERR_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            if (threadIdx.x == 0) trace_at(p, j, 3, global_timer());
            const uint32_t lane_addr = tmem + buf * C::ACC_COLS + ((uint32_t)(quad * 32) << 16);
            if constexpr (C::W) {
#pragma unroll 1
                for (int sb = slice; sb < NSB; sb += QW) {
                    float v1[16];
                    tmem_ld16(lane_addr + sb * 16, v1);
                    epi16_wgrad(p, r, cb0 + sb * 16, v1);
                }
            } else {
#pragma unroll
                for (int k = 0; k < MAXK; ++k) {
                    const int sb = slice + k * QW;  // warp-uniform
                    if (sb >= nsb) break;
                    float v1[16], v2[16];
                    tmem_ld16(lane_addr + sb * 16, v1);
                    tmem_ld16(lane_addr + dofs + sb * 16, v2);
                    const int c0 = cb0 + sb * 16;
                    if (MODE == FWD)
                        epi16_fwd<IO, E>(p, tl.b, r, c0, v1, v2, pf[k]);
                    else if (MODE == BWD1)
                        epi16_bwd1<IO, E>(p, tl.b, r, c0, v1, v2, pf[k]);
                    else
                        epi16_hgrad<IO>(p, tl.b, r, c0, v1, v2, pf[k]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (P)
                    mbar_arrive_remote(smem_in_cta(smem_u32(&acce[buf]), 0));
                else
                    mbar_arrive(smem_u32(&acce[buf]));
            }
            if (threadIdx.x == 0) trace_at(p, j, 4, global_timer());
        }
        if constexpr (MODE == BWD1)
            if (p.zero_dw)
                zero_dw(p, (size_t)blockIdx.x * (kEpiWarps * 32) + threadIdx.x,
                        (size_t)gridDim.x * (kEpiWarps * 32));
    }
    // neither CTA of a pair leaves while the other may still signal its barriers
    if constexpr (P)
        cluster_sync_all();
    else
        __syncthreads();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        if constexpr (P)
            tmem_dealloc_pair(tmem, C::TMEM_COLS);
        else
            tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace aft
}  // namespace dc
