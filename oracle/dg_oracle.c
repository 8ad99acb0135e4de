/*
 * dg_oracle.c -- CPU restatement of DeltaGrid's recurrence hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see dg_oracle.h).  Every function cites the
 * reference file:line it restates.  Paths are relative to the reference
 * project root (hsameerc/deltagrid).
 */
#include "dg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* storage-dtype rounding (IEEE 754 binary16 / bfloat16, round to nearest even) */
/* ------------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static uint16_t f32_to_f16_bits(float f) {
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);          /* >= 65520 -> inf */
    if (ax < 0x38800000u) {                                             /* below 2^-14 */
        float scaled = u2f(ax) * 16777216.0f;                           /* exact: x * 2^24 */
        uint32_t m = (uint32_t)rintf(scaled);                           /* nearest-even */
        return (uint16_t)(sign | m);
    }
    uint32_t e = (ax >> 23) - 127u + 15u;
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

static float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e - 15u + 127u) << 23) | (m << 13));
}

static float round_bf16(float f) {
    uint32_t x = f2u(f);
    if ((x & 0x7fffffffu) > 0x7f800000u) return u2f((x | 0x00400000u) & 0xffff0000u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return u2f(x & 0xffff0000u);
}

float orc_round(float x, int dtype) {
    switch (dtype) {
    case ORC_F16: return f16_bits_to_f32(f32_to_f16_bits(x));
    case ORC_BF16: return round_bf16(x);
    default: return x;
    }
}

void orc_round_array(float* x, int64_t n, int dtype) {
    if (dtype != ORC_F16 && dtype != ORC_BF16) return;
    for (int64_t i = 0; i < n; ++i) x[i] = orc_round(x[i], dtype);
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* dense recurrence                                                          */
/* ------------------------------------------------------------------------ */

/*
 * Per lane (b,h) and step t (src/cpp/delta_kernel.cu:78-112; the PyTorch loop
 * src/modules/memory.py:524-539 computes the same three lines):
 *   y_t = wq_t^T S,  r_t = v_t - wk_t^T S,  S = alpha_t S + (beta_t wk_t) r_t^T
 * S stays fp32 for all T (delta_kernel.cu:64-76, :116-121).  The sums over the
 * slot index run in increasing slot order, as in delta_kernel.cu:92-98.
 */
void orc_dense_forward(int B, int H, int T, int S, int Dh,
                       const float* v, const float* beta, const float* wk, const float* wq,
                       const float* decay, int dynamic_decay, const float* s_init,
                       float* out, float* s_final, float* err_out) {
    const int lanes = B * H;
#pragma omp parallel for schedule(dynamic, 1)
    for (int lane = 0; lane < lanes; ++lane) {
        const int h = lane % H;
        float* st = s_final + (int64_t)lane * S * Dh;
        if (s_init) memcpy(st, s_init + (int64_t)lane * S * Dh, sizeof(float) * (size_t)S * Dh);
        else memset(st, 0, sizeof(float) * (size_t)S * Dh);
        float* acc_y = (float*)malloc(sizeof(float) * (size_t)Dh * 2);
        float* acc_p = acc_y + Dh;
        for (int t = 0; t < T; ++t) {
            const int64_t bt_idx = (int64_t)lane * T + t;
            const float alpha = dynamic_decay ? decay[bt_idx] : decay[h];
            const float bt = beta[bt_idx];
            const float* wkt = wk + bt_idx * S;
            const float* wqt = wq + bt_idx * S;
            const float* vt = v + bt_idx * Dh;
            for (int d = 0; d < Dh; ++d) { acc_y[d] = 0.0f; acc_p[d] = 0.0f; }
            for (int m = 0; m < S; ++m) {
                const float a = wqt[m], b = wkt[m];
                const float* row = st + (int64_t)m * Dh;
                for (int d = 0; d < Dh; ++d) {
                    acc_y[d] += a * row[d];
                    acc_p[d] += b * row[d];
                }
            }
            float* yt = out + bt_idx * Dh;
            for (int d = 0; d < Dh; ++d) {
                yt[d] = acc_y[d];
                acc_p[d] = vt[d] - acc_p[d];                 /* r_t */
                if (err_out) err_out[bt_idx * Dh + d] = acc_p[d];
            }
            for (int m = 0; m < S; ++m) {
                const float bw = bt * wkt[m];
                float* row = st + (int64_t)m * Dh;
                for (int d = 0; d < Dh; ++d) row[d] = alpha * row[d] + bw * acc_p[d];
            }
        }
        free(acc_y);
    }
}

/* ------------------------------------------------------------------------ */
/* sparse Delta-PKM recurrence                                               */
/* ------------------------------------------------------------------------ */

/*
 * Per lane and step (src/cpp/delta_kernel.cu:885-920):
 *   gather s_m = S[idx_m] (and save it, :899-901), y = sum_m wq_m s_m,
 *   pred = sum_m wk_m s_m, r = v - pred, beta_r = beta * r,
 *   S[idx_m] = cast(alpha * s_m + beta_r * wk_m)   (:918; rounded every step)
 * The PyTorch loop (src/ops/_autograd.py:148-167) computes the same values.
 */
void orc_pkm_forward(int B, int H, int T, int A, int64_t total_slots, int Dh,
                     const float* v, const float* beta, const float* wk, const float* wq,
                     const int64_t* idx, const float* decay, int dynamic_decay,
                     float* state, int state_dtype, float* out, float* saved_s_act) {
    const int lanes = B * H;
#pragma omp parallel for schedule(dynamic, 1)
    for (int lane = 0; lane < lanes; ++lane) {
        const int h = lane % H;
        float* st = state + (int64_t)lane * total_slots * Dh;
        float* acc_y = (float*)malloc(sizeof(float) * (size_t)Dh * 2);
        float* acc_r = acc_y + Dh;
        for (int t = 0; t < T; ++t) {
            const int64_t bt_idx = (int64_t)lane * T + t;
            const float alpha = dynamic_decay ? decay[bt_idx] : decay[h];
            const float bt = beta[bt_idx];
            const float* wkt = wk + bt_idx * A;
            const float* wqt = wq + bt_idx * A;
            const int64_t* it = idx + bt_idx * A;
            const float* vt = v + bt_idx * Dh;
            for (int d = 0; d < Dh; ++d) { acc_y[d] = 0.0f; acc_r[d] = 0.0f; }
            for (int m = 0; m < A; ++m) {
                const float* row = st + it[m] * Dh;
                if (saved_s_act) memcpy(saved_s_act + (bt_idx * A + m) * Dh, row, sizeof(float) * (size_t)Dh);
                const float a = wqt[m], b = wkt[m];
                for (int d = 0; d < Dh; ++d) {
                    acc_y[d] += a * row[d];
                    acc_r[d] += b * row[d];
                }
            }
            float* yt = out + bt_idx * Dh;
            for (int d = 0; d < Dh; ++d) {
                yt[d] = acc_y[d];
                acc_r[d] = bt * (vt[d] - acc_r[d]);            /* beta * r_t */
            }
            for (int m = 0; m < A; ++m) {
                float* row = st + it[m] * Dh;
                const float w = wkt[m];
                for (int d = 0; d < Dh; ++d) row[d] = orc_round(alpha * row[d] + acc_r[d] * w, state_dtype);
            }
        }
        free(acc_y);
    }
}

/* ------------------------------------------------------------------------ */
/* two-axis product-key router                                               */
/* ------------------------------------------------------------------------ */

void orc_topk_desc(const float* scores, int n, int K, float* vals, int32_t* idx) {
    /* insertion into a sorted list with strict '>' comparison: among equal
       scores the earlier (lower) index stays ahead (deltagrid_math.cpp:155-167) */
    int filled = 0;
    for (int i = 0; i < n; ++i) {
        const float s = scores[i];
        if (filled == K && !(s > vals[K - 1])) continue;
        int pos = (filled < K) ? filled++ : K - 1;
        while (pos > 0 && s > vals[pos - 1]) {
            vals[pos] = vals[pos - 1];
            idx[pos] = idx[pos - 1];
            --pos;
        }
        vals[pos] = s;
        idx[pos] = i;
    }
}

static float dot_seq(const float* a, const float* b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

/* F.normalize(x, p=2, dim=-1): x / max(||x||_2, 1e-12) (memory.py:265, :270) */
static void l2norm_inplace(float* x, int n) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    float nrm = (float)sqrt(ss);
    if (nrm < 1e-12f) nrm = 1e-12f;
    for (int i = 0; i < n; ++i) x[i] = x[i] / nrm;
}

/*
 * src/modules/memory.py:258-279 for two axes without subspace slicing:
 *   s_a = axes_proj_k[a](k); (val, idx_a) = topk(s_a, K); u_k,a = normalize(val)
 *   u_q,a = normalize(gather(axes_proj_q[a](q), idx_a))      (query read at key indices)
 *   wk = u_k,0 (x) u_k,1;  wq = u_q,0 (x) u_q,1;  idx = idx_0 * G1 + idx_1
 * q_scale (memory.py:453-455) multiplies wq when given.
 */
void orc_pkm_route(int64_t N, int Dh, int G0, int G1, int K,
                   const float* k, const float* q,
                   const float* wk0, const float* wk1, const float* wq0, const float* wq1,
                   const float* q_scale, float* wk, float* wq, int64_t* idx, float* margin) {
    const int Gmax = G0 > G1 ? G0 : G1;
#pragma omp parallel
    {
        float* sc = (float*)malloc(sizeof(float) * (size_t)Gmax);
        float* vals = (float*)malloc(sizeof(float) * (size_t)(K + 1) * 2);
        int32_t* ix = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K + 1) * 2);
        float uk[2][64], uq[2][64];
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; ++n) {
            const float* kn = k + n * Dh;
            const float* qn = q + n * Dh;
            float mg = INFINITY;
            for (int a = 0; a < 2; ++a) {
                const int G = a ? G1 : G0;
                const float* Wk = a ? wk1 : wk0;
                const float* Wq = a ? wq1 : wq0;
                for (int g = 0; g < G; ++g) sc[g] = dot_seq(Wk + (int64_t)g * Dh, kn, Dh);
                const int KK = (K < G) ? K + 1 : K;
                orc_topk_desc(sc, G, KK, vals + a * (K + 1), ix + a * (K + 1));
                if (KK > K) {
                    float gap = vals[a * (K + 1) + K - 1] - vals[a * (K + 1) + K];
                    if (gap < mg) mg = gap;
                }
                for (int j = 0; j < K; ++j) {
                    uk[a][j] = vals[a * (K + 1) + j];
                    uq[a][j] = dot_seq(Wq + (int64_t)ix[a * (K + 1) + j] * Dh, qn, Dh);
                }
                l2norm_inplace(uk[a], K);
                l2norm_inplace(uq[a], K);
            }
            const float qs = q_scale ? q_scale[n] : 1.0f;
            for (int i = 0; i < K; ++i) {
                for (int j = 0; j < K; ++j) {
                    const int64_t o = n * K * K + i * K + j;
                    wk[o] = uk[0][i] * uk[1][j];
                    wq[o] = (uq[0][i] * uq[1][j]) * qs;
                    idx[o] = (int64_t)ix[i] * G1 + ix[(K + 1) + j];
                }
            }
            if (margin) margin[n] = mg;
        }
        free(sc);
        free(vals);
        free(ix);
    }
}

/* ------------------------------------------------------------------------ */
/* Q16.16 fixed-point                                                        */
/* ------------------------------------------------------------------------ */

#define FXP_HALF (1 << 15)

/* include/deltagrid_math_fxp.h:16-19: (a*b + 2^15) >> 16 in 64-bit */
int32_t orc_fxp_mul(int32_t a, int32_t b) {
    int64_t p = (int64_t)a * (int64_t)b;
    return (int32_t)((p + FXP_HALF) >> 16);
}

/* deltagrid_fxp.cpp:380-405 (dense) -- int64 MACs, round, residual, update */
void orc_fxp_dense_forward(int L, int T, int S, int Dh,
                           const int32_t* wk, const int32_t* wq, const int32_t* v,
                           const int32_t* beta, const int32_t* alpha,
                           int32_t* state, int32_t* y) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int l = 0; l < L; ++l) {
        int32_t* st = state + (int64_t)l * S * Dh;
        int64_t* ya = (int64_t*)malloc(sizeof(int64_t) * (size_t)Dh * 2);
        int64_t* pa = ya + Dh;
        int32_t* rt = (int32_t*)malloc(sizeof(int32_t) * (size_t)Dh);
        for (int t = 0; t < T; ++t) {
            const int64_t lt = (int64_t)l * T + t;
            const int32_t* wkt = wk + lt * S;
            const int32_t* wqt = wq + lt * S;
            for (int d = 0; d < Dh; ++d) { ya[d] = 0; pa[d] = 0; }
            for (int s = 0; s < S; ++s) {
                const int32_t* row = st + (int64_t)s * Dh;
                const int64_t a = wqt[s], b = wkt[s];
                for (int d = 0; d < Dh; ++d) { ya[d] += a * row[d]; pa[d] += b * row[d]; }
            }
            for (int d = 0; d < Dh; ++d) {
                y[lt * Dh + d] = (int32_t)((ya[d] + FXP_HALF) >> 16);
                const int32_t pred = (int32_t)((pa[d] + FXP_HALF) >> 16);
                rt[d] = (int32_t)((uint32_t)v[lt * Dh + d] - (uint32_t)pred);
            }
            const int32_t al = alpha[lt], be = beta[lt];
            for (int s = 0; s < S; ++s) {
                int32_t* row = st + (int64_t)s * Dh;
                const int32_t bw = orc_fxp_mul(be, wkt[s]);
                for (int d = 0; d < Dh; ++d)
                    row[d] = (int32_t)((uint32_t)orc_fxp_mul(al, row[d]) + (uint32_t)orc_fxp_mul(bw, rt[d]));
            }
        }
        free(ya);
        free(rt);
    }
}

/* deltagrid_fxp.cpp:298-326 (sparse PKM) -- gather rows, int64 MACs, update in place */
void orc_fxp_pkm_forward(int L, int T, int A, int64_t total_slots, int Dh,
                         const int32_t* wk, const int32_t* wq, const int32_t* idx,
                         const int32_t* v, const int32_t* beta, const int32_t* alpha,
                         int32_t* state, int32_t* y) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int l = 0; l < L; ++l) {
        int32_t* st = state + (int64_t)l * total_slots * Dh;
        int64_t* ya = (int64_t*)malloc(sizeof(int64_t) * (size_t)Dh * 2);
        int64_t* pa = ya + Dh;
        int32_t* rt = (int32_t*)malloc(sizeof(int32_t) * (size_t)Dh);
        for (int t = 0; t < T; ++t) {
            const int64_t lt = (int64_t)l * T + t;
            const int32_t* wkt = wk + lt * A;
            const int32_t* wqt = wq + lt * A;
            const int32_t* it = idx + lt * A;
            for (int d = 0; d < Dh; ++d) { ya[d] = 0; pa[d] = 0; }
            for (int m = 0; m < A; ++m) {
                const int32_t* row = st + (int64_t)it[m] * Dh;
                const int64_t a = wqt[m], b = wkt[m];
                for (int d = 0; d < Dh; ++d) { ya[d] += a * row[d]; pa[d] += b * row[d]; }
            }
            for (int d = 0; d < Dh; ++d) {
                y[lt * Dh + d] = (int32_t)((ya[d] + FXP_HALF) >> 16);
                const int32_t pred = (int32_t)((pa[d] + FXP_HALF) >> 16);
                rt[d] = (int32_t)((uint32_t)v[lt * Dh + d] - (uint32_t)pred);
            }
            const int32_t al = alpha[lt], be = beta[lt];
            for (int m = 0; m < A; ++m) {
                int32_t* row = st + (int64_t)it[m] * Dh;
                const int32_t bw = orc_fxp_mul(be, wkt[m]);
                for (int d = 0; d < Dh; ++d)
                    row[d] = (int32_t)((uint32_t)orc_fxp_mul(al, row[d]) + (uint32_t)orc_fxp_mul(bw, rt[d]));
            }
        }
        free(ya);
        free(rt);
    }
}

/* dg_matmul_fxp without bias (deltagrid_math_fxp.cpp:5-27) for one output row */
static int32_t fxp_dot(const int32_t* row, const int32_t* x, int n) {
    int64_t s = 0;
    for (int j = 0; j < n; ++j) s += (int64_t)row[j] * (int64_t)x[j];
    return (int32_t)((s + FXP_HALF) >> 16);
}

/* dg_topk_descending_fxp (deltagrid_math_fxp.cpp:104-129): strict '>' keeps lower index first */
static void fxp_topk(const int32_t* sc, int n, int K, int32_t* vals, int32_t* ix) {
    int filled = 0;
    for (int i = 0; i < n; ++i) {
        const int32_t s = sc[i];
        if (filled == K && !(s > vals[K - 1])) continue;
        int pos = (filled < K) ? filled++ : K - 1;
        while (pos > 0 && s > vals[pos - 1]) { vals[pos] = vals[pos - 1]; ix[pos] = ix[pos - 1]; --pos; }
        vals[pos] = s;
        ix[pos] = i;
    }
}

/* dg_l2_normalize_fxp (deltagrid_math_fxp.cpp:86-102): fp32 norm, truncating Q16.16 reciprocal */
static void fxp_l2norm(int32_t* x, int n) {
    float ss = 0.0f;
    for (int i = 0; i < n; ++i) { float f = (float)x[i] / 65536.0f; ss += f * f; }
    float nrm = sqrtf(ss);
    float den = (nrm > 1e-12f) ? nrm : 1e-12f;
    int32_t inv = (int32_t)((1.0f / den) * 65536.0f);
    for (int i = 0; i < n; ++i) x[i] = orc_fxp_mul(x[i], inv);
}

/* deltagrid_fxp.cpp:246-296 for two axes, then q_scale (:294-296) */
void orc_fxp_pkm_route(int Dh, int G0, int G1, int K, const int32_t* k, const int32_t* q,
                       const int32_t* wk0, const int32_t* wk1, const int32_t* wq0,
                       const int32_t* wq1, int32_t q_scale,
                       int32_t* wk, int32_t* wq, int32_t* idx) {
    int32_t uk[2][64], uq[2][64], ix[2][64];
    const int Gmax = G0 > G1 ? G0 : G1;
    int32_t* sc = (int32_t*)malloc(sizeof(int32_t) * (size_t)Gmax);
    for (int a = 0; a < 2; ++a) {
        const int G = a ? G1 : G0;
        const int32_t* Wk = a ? wk1 : wk0;
        const int32_t* Wq = a ? wq1 : wq0;
        for (int g = 0; g < G; ++g) sc[g] = fxp_dot(Wk + (int64_t)g * Dh, k, Dh);
        fxp_topk(sc, G, K, uk[a], ix[a]);
        fxp_l2norm(uk[a], K);
        for (int j = 0; j < K; ++j) uq[a][j] = fxp_dot(Wq + (int64_t)ix[a][j] * Dh, q, Dh);
        fxp_l2norm(uq[a], K);
    }
    free(sc);
    for (int i = 0; i < K; ++i)
        for (int j = 0; j < K; ++j) {
            wk[i * K + j] = orc_fxp_mul(uk[0][i], uk[1][j]);
            wq[i * K + j] = orc_fxp_mul(orc_fxp_mul(uq[0][i], uq[1][j]), q_scale);
            idx[i * K + j] = ix[0][i] * G1 + ix[1][j];
        }
}
