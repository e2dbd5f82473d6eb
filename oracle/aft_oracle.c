/*
 * CPU oracle for the G-Tensor (KellyKinyama/dart_cuda) training hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links or calls
 * this file; only the test suite, the smoke check and the CPU-baseline leg of
 * the benchmark use it, and only as the checker / the timed CPU baseline.
 *
 * Each function restates one reference kernel loop for loop, with the same
 * constants, the same fp32 arithmetic and the same summation order along the
 * reduced axis.  The reference runs one CUDA thread per row; here the row loop
 * is an OpenMP loop.  Where the reference accumulates with atomicAdd from many
 * threads, the restatement keeps the per-thread contributions private and
 * reduces them afterwards, which changes only the order of the cross-row sum.
 *
 * Reference files (paths inside the reference project):
 *   aft_full_fwd ........ native/src/kernels/attention.cuh:6-40
 *   aft_full_bwd ........ native/src/engine.cu:522-590
 *   aft_cross_fwd ....... native/src/kernels/attention.cuh:41-72
 *   aft_cross_bwd ....... native/src/kernels/attention.cuh:73-128
 *   layernorm_fwd/bwd ... native/src/kernels/layernorm_embed.cuh:140-240
 *   add_row_broadcast ... native/src/kernels/elementwise.cuh:64-89
 *   cross_entropy ....... native/src/kernels/loss_optim.cuh:163-244,
 *                         native/src/engine.cu:825-877 (eps 0.1, mean over T)
 *   adam_kernel ......... native/src/kernels/loss_optim.cuh:255-298
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int oracle_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int oracle_thread_id(void)
{
#ifdef _OPENMP
    return omp_get_thread_num();
#else
    return 0;
#endif
}

int oracle_num_threads(void) { return oracle_threads(); }

void oracle_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------
 * AFT-full forward, one sequence.  attention.cuh:6-40.
 * WB is read as WB[t*ldw + tp]; the reference always passes ldw == T
 * (it indexes WB with the query row count even when the bias tensor was
 * allocated [maxSeqLen, maxSeqLen]).
 * ---------------------------------------------------------------------- */
static void aft_full_fwd_row(const float *Q, const float *K, const float *V,
                             const float *WB, float *out, int T, int D,
                             int masked, int ldw, int t, float *scratch)
{
    /* The reference's per-(t,d) loops over tp, evaluated for all d of row t
     * at once (d innermost, so K and V rows are read contiguously).  Every
     * (t,d) sees exactly the reference's sequence of operations: the max over
     * tp in increasing tp, then num and den summed in increasing tp. */
    float *max_val = scratch, *numerator = scratch + D, *denominator = scratch + 2 * D;
    int limit = masked ? (t + 1) : T;
    const float *wrow = WB + (size_t)t * ldw;
    for (int d = 0; d < D; d++) {
        max_val[d] = -1e20f;
        numerator[d] = 0.0f;
        denominator[d] = 0.0f;
    }
    for (int tp = 0; tp < limit; tp++) {
        const float wv = wrow[tp];
        const float *k = K + (size_t)tp * D;
        for (int d = 0; d < D; d++) {
            float val = k[d] + wv;
            if (val > max_val[d]) max_val[d] = val;
        }
    }
    for (int tp = 0; tp < limit; tp++) {
        const float wv = wrow[tp];
        const float *k = K + (size_t)tp * D, *v = V + (size_t)tp * D;
        for (int d = 0; d < D; d++) {
            float w = expf(k[d] + wv - max_val[d]);
            numerator[d] += w * v[d];
            denominator[d] += w;
        }
    }
    for (int d = 0; d < D; d++) {
        float sigQ = 1.0f / (1.0f + expf(-Q[(size_t)t * D + d]));
        out[(size_t)t * D + d] = sigQ * (numerator[d] / (denominator[d] + 1e-6f));
    }
}

/* Batched forward: B independent sequences [B,T,D] sharing one WB. */
void oracle_aft_full_fwd(const float *Q, const float *K, const float *V,
                         const float *WB, float *out, int B, int T, int D,
                         int masked, int ldw)
{
    size_t sd = (size_t)T * D;
    long total = (long)B * T;
#pragma omp parallel
    {
        float *scratch = (float *)malloc((size_t)3 * D * sizeof(float));
#pragma omp for schedule(dynamic, 1)
        for (long bt = total - 1; bt >= 0; bt--) {
            int b = (int)(bt / T), t = (int)(bt % T);
            if (scratch)
                aft_full_fwd_row(Q + b * sd, K + b * sd, V + b * sd, WB, out + b * sd,
                                 T, D, masked, ldw, t, scratch);
        }
        free(scratch);
    }
}

/* ------------------------------------------------------------------------
 * AFT-full backward, one query row t of one sequence.  engine.cu:522-590.
 * dQ, dK, dV, dWB accumulate (+=), as the reference's atomicAdd does.
 * gK/gV here are the calling thread's private accumulators; row t of gWB is
 * written by this call alone (one thread owns each query row), and its
 * entries receive their d contributions in increasing d, as the reference's
 * loop nest (d outer, tp inner) adds them.
 * ---------------------------------------------------------------------- */
static void aft_full_bwd_row(const float *Q, const float *K, const float *V,
                             const float *WB, const float *gout, float *gQ,
                             float *gK, float *gV, float *gWB, int T, int D,
                             int masked, int ldw, int t, float *scratch)
{
    float *max_val = scratch, *num = scratch + D, *den = scratch + 2 * D;
    float *den_inv = scratch + 3 * D, *ratio = scratch + 4 * D, *gs = scratch + 5 * D;
    int limit = masked ? (t + 1) : T;
    const float *wrow = WB + (size_t)t * ldw;
    for (int d = 0; d < D; d++) {
        max_val[d] = -1e20f;
        num[d] = 0.0f;
        den[d] = 0.0f;
    }
    for (int tp = 0; tp < limit; tp++) {
        const float wv = wrow[tp];
        const float *k = K + (size_t)tp * D;
        for (int d = 0; d < D; d++) {
            float v = k[d] + wv;
            if (v > max_val[d]) max_val[d] = v;
        }
    }
    for (int tp = 0; tp < limit; tp++) {
        const float wv = wrow[tp];
        const float *k = K + (size_t)tp * D, *vv = V + (size_t)tp * D;
        for (int d = 0; d < D; d++) {
            float w = expf(k[d] + wv - max_val[d]);
            num[d] += w * vv[d];
            den[d] += w;
        }
    }
    for (int d = 0; d < D; d++) {
        den_inv[d] = 1.0f / (den[d] + 1e-9f);
        ratio[d] = num[d] * den_inv[d];
        float sigQ = 1.0f / (1.0f + expf(-Q[(size_t)t * D + d]));
        float dSigQ = sigQ * (1.0f - sigQ);
        float gO = gout[(size_t)t * D + d];
        gQ[(size_t)t * D + d] += gO * ratio[d] * dSigQ;
        gs[d] = gO * sigQ;
    }
    for (int tp = 0; tp < limit; tp++) {
        const float wv = wrow[tp];
        const float *k = K + (size_t)tp * D, *vv = V + (size_t)tp * D;
        float *gk = gK + (size_t)tp * D, *gv = gV + (size_t)tp * D;
        float acc = gWB[(size_t)t * ldw + tp];
        for (int d = 0; d < D; d++) {
            float w = expf(k[d] + wv - max_val[d]);
            float dV = gs[d] * (w * den_inv[d]);
            gv[d] += dV;
            float dW = gs[d] * w * (vv[d] - ratio[d]) * den_inv[d];
            gk[d] += dW;
            acc += dW;
        }
        gWB[(size_t)t * ldw + tp] = acc;
    }
}

/* Batched backward.  Grad buffers accumulate.  gWB has rows of stride ldw
 * and T rows; it is shared by all B sequences (their grads add up, as B
 * sequential reference calls on one bias tensor would). */
void oracle_aft_full_bwd(const float *Q, const float *K, const float *V,
                         const float *WB, const float *gout, float *gQ,
                         float *gK, float *gV, float *gWB, int B, int T, int D,
                         int masked, int ldw)
{
    size_t sd = (size_t)T * D;
    int nth = oracle_threads();
    /* private dK/dV per thread for one sequence at a time; dWB rows belong
     * to the thread that owns the query row */
    float *priv = (float *)calloc((size_t)nth * 2 * sd, sizeof(float));
    if (!priv) return;
    for (int b = 0; b < B; b++) {
        memset(priv, 0, (size_t)nth * 2 * sd * sizeof(float));
#pragma omp parallel
        {
            float *scratch = (float *)malloc((size_t)6 * D * sizeof(float));
            float *mine = priv + (size_t)oracle_thread_id() * 2 * sd;
#pragma omp for schedule(dynamic, 1)
            for (int t = T - 1; t >= 0; t--) {
                if (scratch)
                    aft_full_bwd_row(Q + b * sd, K + b * sd, V + b * sd, WB,
                                     gout + b * sd, gQ + b * sd, mine, mine + sd,
                                     gWB, T, D, masked, ldw, t, scratch);
            }
            free(scratch);
        }
        /* reduce the private accumulators */
#pragma omp parallel for schedule(static)
        for (long j = 0; j < (long)sd; j++) {
            float sk = 0.0f, sv = 0.0f;
            for (int h = 0; h < nth; h++) {
                float *mine = priv + (size_t)h * 2 * sd;
                sk += mine[j];
                sv += mine[sd + j];
            }
            gK[b * sd + j] += sk;
            gV[b * sd + j] += sv;
        }
    }
    free(priv);
}

/* ------------------------------------------------------------------------
 * AFT-cross forward / backward.  attention.cuh:41-128.  Q is [TDec,D],
 * K,V are [TEnc,D], WB is read with row stride TEnc.  Not causal.
 * ---------------------------------------------------------------------- */
void oracle_aft_cross_fwd(const float *Q, const float *K, const float *V,
                          const float *WB, float *out, int TDec, int TEnc,
                          int D)
{
#pragma omp parallel for schedule(static)
    for (int t = 0; t < TDec; t++) {
        for (int d = 0; d < D; d++) {
            float max_val = -1e20f;
            for (int tp = 0; tp < TEnc; tp++) {
                float val = K[tp * D + d] + WB[(size_t)t * TEnc + tp];
                if (val > max_val) max_val = val;
            }
            float numerator = 0.0f, denominator = 0.0f;
            for (int tp = 0; tp < TEnc; tp++) {
                float w = expf(K[tp * D + d] + WB[(size_t)t * TEnc + tp] - max_val);
                numerator += w * V[tp * D + d];
                denominator += w;
            }
            float sigQ = 1.0f / (1.0f + expf(-Q[t * D + d]));
            out[t * D + d] = sigQ * (numerator / (denominator + 1e-6f));
        }
    }
}

void oracle_aft_cross_bwd(const float *Q, const float *K, const float *V,
                          const float *WB, const float *gout, float *gQ,
                          float *gK, float *gV, float *gWB, int TDec, int TEnc,
                          int D)
{
    /* serial: the cross op is small in every configuration that uses it */
    for (int t = 0; t < TDec; t++) {
        for (int d = 0; d < D; d++) {
            float max_val = -1e20f;
            for (int tp = 0; tp < TEnc; tp++) {
                float v = K[tp * D + d] + WB[(size_t)t * TEnc + tp];
                if (v > max_val) max_val = v;
            }
            float num = 0.0f, den = 0.0f;
            for (int tp = 0; tp < TEnc; tp++) {
                float w = expf(K[tp * D + d] + WB[(size_t)t * TEnc + tp] - max_val);
                num += w * V[tp * D + d];
                den += w;
            }
            float den_inv = 1.0f / (den + 1e-6f);
            float ratio = num * den_inv;
            float sigQ = 1.0f / (1.0f + expf(-Q[t * D + d]));
            float gO = gout[t * D + d];
            gQ[t * D + d] += gO * ratio * sigQ * (1.0f - sigQ);
            for (int tp = 0; tp < TEnc; tp++) {
                float w = expf(K[tp * D + d] + WB[(size_t)t * TEnc + tp] - max_val);
                gV[tp * D + d] += gO * sigQ * (w * den_inv);
                float dW = gO * sigQ * w * (V[tp * D + d] - ratio) * den_inv;
                gK[tp * D + d] += dW;
                gWB[(size_t)t * TEnc + tp] += dW;
            }
        }
    }
}

/* ------------------------------------------------------------------------
 * Affine LayerNorm.  layernorm_embed.cuh:140-240.  Two-pass mean/variance,
 * y = (x-mean)*rsqrt(var+eps)*gamma + beta.  Backward accumulates into
 * gx, gGamma, gBeta.  rsqrtf is restated as 1/sqrtf.
 * ---------------------------------------------------------------------- */
void oracle_layernorm_fwd(const float *x, const float *gamma,
                          const float *beta, float *out, int R, int C,
                          float eps)
{
#pragma omp parallel for schedule(static)
    for (int r = 0; r < R; r++) {
        const float *xr = x + (size_t)r * C;
        float *yr = out + (size_t)r * C;
        float s = 0.0f;
        for (int j = 0; j < C; j++) s += xr[j];
        float mean = s / (float)C;
        float sq = 0.0f;
        for (int j = 0; j < C; j++) {
            float d = xr[j] - mean;
            sq += d * d;
        }
        float inv_std = 1.0f / sqrtf(sq / (float)C + eps);
        for (int j = 0; j < C; j++)
            yr[j] = (xr[j] - mean) * inv_std * gamma[j] + beta[j];
    }
}

void oracle_layernorm_bwd(const float *x, const float *gamma, const float *go,
                          float *gx, float *gGamma, float *gBeta, int R, int C,
                          float eps)
{
    for (int r = 0; r < R; r++) {
        const float *xr = x + (size_t)r * C;
        const float *gr = go + (size_t)r * C;
        float *gxr = gx + (size_t)r * C;
        float s = 0.0f;
        for (int j = 0; j < C; j++) s += xr[j];
        float mean = s / (float)C;
        float sq = 0.0f;
        for (int j = 0; j < C; j++) {
            float d = xr[j] - mean;
            sq += d * d;
        }
        float inv_std = 1.0f / sqrtf(sq / (float)C + eps);
        float dxh_sum = 0.0f, dxh_xh_sum = 0.0f;
        for (int j = 0; j < C; j++) {
            float xh = (xr[j] - mean) * inv_std;
            float dxh = gr[j] * gamma[j];
            dxh_sum += dxh;
            dxh_xh_sum += dxh * xh;
            gGamma[j] += gr[j] * xh;
            gBeta[j] += gr[j];
        }
        float invC = 1.0f / (float)C;
        for (int j = 0; j < C; j++) {
            float xh = (xr[j] - mean) * inv_std;
            float dxh = gr[j] * gamma[j];
            gxr[j] += inv_std * (dxh - dxh_sum * invC - xh * dxh_xh_sum * invC);
        }
    }
}

/* ------------------------------------------------------------------------
 * Row-broadcast bias add.  elementwise.cuh:64-89.  ga += g, gb[j] += sum_i g.
 * ---------------------------------------------------------------------- */
void oracle_add_row_broadcast_fwd(const float *a, const float *b, float *out,
                                  int M, int N)
{
    for (long i = 0; i < M; i++)
        for (int j = 0; j < N; j++) out[i * N + j] = a[i * N + j] + b[j];
}

void oracle_add_row_broadcast_bwd(const float *go, float *ga, float *gb,
                                  int M, int N)
{
    for (long i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            float g = go[i * N + j];
            ga[i * N + j] += g;
            gb[j] += g;
        }
}

/* ------------------------------------------------------------------------
 * Label-smoothed cross-entropy.  loss_optim.cuh:163-244 and the wrapper at
 * engine.cu:825-877: per-row loss (1-eps)(lse - x_y) + eps(lse - mean_v x),
 * lse = max + log(sum exp(x-max) + 1e-12); scalar = mean over T rows.
 * Backward WRITES (not +=) grad = (softmax - ((1-eps)1_y + eps/V)) * g/T.
 * ---------------------------------------------------------------------- */
void oracle_ce_fwd(const float *logits, const int *targets, float *loss_rows,
                   int T, int V, float eps)
{
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        const float *row = logits + (size_t)t * V;
        float mx = -1e30f;
        for (int v = 0; v < V; v++) mx = fmaxf(mx, row[v]);
        float se = 0.0f, sl = 0.0f;
        for (int v = 0; v < V; v++) {
            se += expf(row[v] - mx);
            sl += row[v];
        }
        float lse = mx + logf(se + 1e-12f);
        float ce = lse - row[targets[t]];
        float smooth = lse - sl / (float)V;
        loss_rows[t] = (1.0f - eps) * ce + eps * smooth;
    }
}

float oracle_ce_mean(const float *loss_rows, int T)
{
    float s = 0.0f;
    for (int t = 0; t < T; t++) s += loss_rows[t];
    return s / (float)T;
}

void oracle_ce_bwd(const float *logits, const int *targets, float *grad,
                   int T, int V, float grad_output, float eps)
{
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        const float *row = logits + (size_t)t * V;
        float *gr = grad + (size_t)t * V;
        float mx = -1e30f;
        for (int v = 0; v < V; v++) mx = fmaxf(mx, row[v]);
        float se = 0.0f;
        for (int v = 0; v < V; v++) se += expf(row[v] - mx);
        se += 1e-12f;
        float scale = grad_output / (float)T;
        for (int v = 0; v < V; v++) {
            float sm = expf(row[v] - mx) / se;
            float ind = (v == targets[t]) ? 1.0f : 0.0f;
            float tp = (1.0f - eps) * ind + eps / (float)V;
            gr[v] = (sm - tp) * scale;
        }
    }
}

/* ------------------------------------------------------------------------
 * AdamW as the reference implements it.  loss_optim.cuh:255-298:
 * step = t+1, weight decay 0.001 applied as p -= lr*wd*p (old p).
 * ---------------------------------------------------------------------- */
void oracle_adam(float *p, const float *g, float *m, float *v, int size, int t,
                 float lr, float b1, float b2, float eps)
{
    float step = (float)t + 1.0f;
    float wd = 0.001f;
    for (int i = 0; i < size; i++) {
        float grad = g[i];
        m[i] = b1 * m[i] + (1.0f - b1) * grad;
        v[i] = b2 * v[i] + (1.0f - b2) * (grad * grad);
        float m_hat = m[i] / (1.0f - powf(b1, step));
        float v_hat = v[i] / (1.0f - powf(b2, step));
        float delta = lr * m_hat / (sqrtf(v_hat) + eps);
        p[i] = p[i] - delta - (lr * wd * p[i]);
    }
}
