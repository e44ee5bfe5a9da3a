/* CPU oracle: plain-C restatement of the reference's fp32 CPU emit.
 * TEST INFRASTRUCTURE ONLY (see ns_oracle.h). Compiled with the same flags
 * as the reference's emitted units (-O3 -march=x86-64-v3, default FP
 * contraction) so that scalar accumulation chains contract to FMA the same
 * way; every reduction below is sequential in the reference's index order.
 */
#include "ns_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* src/codegen/codegen.cpp:1244-1255 (ns_act2). GELU divides by the float
 * literal 1.41421356f, unlike the MoE expert's GELU which multiplies by
 * 0.7071067811865476f (codegen.cpp:1938). */
float orc_act(float x, int code) {
    switch (code) {
        case 1: return x > 0 ? x : 0.f;
        case 2: return x > 0 ? x : 0.01f * x;
        case 3: return 1.f / (1.f + expf(-x));
        case 4: return tanhf(x);
        case 5: return x / (1.f + expf(-x));
        case 6: return 0.5f * x * (1.f + erff(x / 1.41421356f));
        default: return x;
    }
}

/* codegen.cpp:1305-1315 (ns_act_deriv). */
float orc_act_deriv(float x, int code) {
    switch (code) {
        case 1: return x > 0.f ? 1.f : 0.f;
        case 2: return x > 0.f ? 1.f : 0.01f;
        case 3: { float s = 1.f / (1.f + expf(-x)); return s * (1.f - s); }
        case 4: { float t = tanhf(x); return 1.f - t * t; }
        case 5: { float s = x / (1.f + expf(-x)); return s + x * (1.f - s); }
        case 6: {
            float u = x / 1.41421356f;
            float p = 0.5f * (1.f + erff(u));
            return p + x * expf(-u * u) / 2.50662827f;
        }
        default: return 1.f;
    }
}

void orc_act_vec(const float* in, float* out, size_t n, int code) {
    for (size_t i = 0; i < n; i++) out[i] = orc_act(in[i], code);
}

/* codegen.cpp:1340-1343 (ns_act_grad): dOut = dIn * act'(pre-activation). */
void orc_act_grad(const float* din, const float* act_in, float* dout, size_t n, int code) {
    for (size_t i = 0; i < n; i++) dout[i] = din[i] * orc_act_deriv(act_in[i], code);
}

/* codegen.cpp:1257-1265 (ns_matmul): C[M,N] = A[M,K] B[K,N], k innermost. */
void orc_matmul(const float* A, const float* B, float* C, int64_t M, int64_t K, int64_t N) {
    for (int64_t i = 0; i < M; i++) {
        const float* a = A + (size_t)i * K;
        for (int64_t j = 0; j < N; j++) {
            float acc = 0.f;
            for (int64_t k = 0; k < K; k++) acc += a[k] * B[(size_t)k * N + j];
            C[(size_t)i * N + j] = acc;
        }
    }
}

/* codegen.cpp:1318-1326 (ns_matmul_grad_a): dA[M,K] = dC[M,N] B[K,N]^T. */
void orc_matmul_grad_a(const float* dC, const float* B, float* dA, int64_t M, int64_t K, int64_t N) {
    for (int64_t i = 0; i < M; i++) {
        const float* d = dC + (size_t)i * N;
        for (int64_t k = 0; k < K; k++) {
            const float* b = B + (size_t)k * N;
            float acc = 0.f;
            for (int64_t j = 0; j < N; j++) acc += d[j] * b[j];
            dA[(size_t)i * K + k] = acc;
        }
    }
}

/* codegen.cpp:1329-1337 (ns_matmul_grad_w): dB[K,N] = A[M,K]^T dC[M,N],
 * summed over rows i in order. */
void orc_matmul_grad_w(const float* A, const float* dC, float* dB, int64_t M, int64_t K, int64_t N) {
    for (int64_t k = 0; k < K; k++)
        for (int64_t j = 0; j < N; j++) {
            float acc = 0.f;
            for (int64_t i = 0; i < M; i++) acc += A[(size_t)i * K + k] * dC[(size_t)i * N + j];
            dB[(size_t)k * N + j] = acc;
        }
}

/* codegen.cpp:1267-1278 (ns_binop): C[i] = A[i] op B[i % nb]. */
void orc_binop(const float* A, size_t na, const float* B, size_t nb, float* C, int op) {
    for (size_t i = 0; i < na; i++) {
        float b = nb > 0 ? B[i % nb] : 0.f;
        switch (op) {
            case 0: C[i] = A[i] + b; break;
            case 1: C[i] = A[i] - b; break;
            case 2: C[i] = A[i] * b; break;
            case 3: C[i] = A[i] / b; break;
            default: C[i] = A[i]; break;
        }
    }
}

/* codegen.cpp:1280-1291 (ns_layernorm): two-pass mean / biased variance,
 * eps 1e-5, no affine. Out-of-place here; the reference copies then
 * normalises in place, which is the same arithmetic. */
void orc_layernorm(const float* in, float* out, int64_t rows, int64_t last) {
    for (int64_t r = 0; r < rows; r++) {
        const float* x = in + (size_t)r * last;
        float* y = out + (size_t)r * last;
        float mean = 0.f, var = 0.f;
        for (int64_t j = 0; j < last; j++) mean += x[j];
        mean /= last;
        for (int64_t j = 0; j < last; j++) { float d = x[j] - mean; var += d * d; }
        var /= last;
        float inv = 1.f / sqrtf(var + 1e-5f);
        for (int64_t j = 0; j < last; j++) y[j] = (x[j] - mean) * inv;
    }
}

/* codegen.cpp:1346-1371 (ns_layernorm_grad): statistics recomputed from the
 * LayerNorm input x. */
void orc_layernorm_grad(const float* dout, const float* x, float* dx, int64_t rows, int64_t last) {
    for (int64_t r = 0; r < rows; r++) {
        const float* xr = x + (size_t)r * last;
        const float* dr = dout + (size_t)r * last;
        float* o = dx + (size_t)r * last;
        float mean_x = 0.f, mean_d = 0.f;
        for (int64_t j = 0; j < last; j++) { mean_x += xr[j]; mean_d += dr[j]; }
        mean_x /= last;
        mean_d /= last;
        float var_x = 0.f, gamma = 0.f;
        for (int64_t j = 0; j < last; j++) {
            float xj = xr[j] - mean_x;
            var_x += xj * xj;
            gamma += xj * dr[j];
        }
        var_x /= last;
        gamma /= last;
        float inv = 1.f / sqrtf(var_x + 1e-5f);
        for (int64_t j = 0; j < last; j++) {
            float xj = xr[j] - mean_x;
            o[j] = (dr[j] - mean_d - xj * gamma) * inv;
        }
    }
}

/* codegen.cpp:1293-1302 (ns_softmax). */
void orc_softmax(const float* in, float* out, int64_t rows, int64_t last) {
    for (int64_t r = 0; r < rows; r++) {
        const float* x = in + (size_t)r * last;
        float* y = out + (size_t)r * last;
        float mx = x[0];
        for (int64_t j = 1; j < last; j++) mx = mx > x[j] ? mx : x[j];
        float s = 0.f;
        for (int64_t j = 0; j < last; j++) { y[j] = expf(x[j] - mx); s += y[j]; }
        for (int64_t j = 0; j < last; j++) y[j] /= s;
    }
}

/* codegen.cpp:1711-1718 (ns_embedding): ids are fp32 truncated toward zero;
 * out-of-range ids read row 0. */
void orc_embedding(const float* W, const float* idx, float* out, int64_t n, int64_t V, int64_t D) {
    for (int64_t i = 0; i < n; i++) {
        int64_t k = (int64_t)idx[i];
        if (k < 0 || k >= V) k = 0;
        memcpy(out + (size_t)i * D, W + (size_t)k * D, (size_t)D * sizeof(float));
    }
}

/* codegen.cpp:1374-1383 (ns_embedding_grad_w): zero, then add dOut rows in
 * row order; out-of-range ids are skipped. */
void orc_embedding_grad_w(const float* dout, const float* idx, float* dW, int64_t M, int64_t D, int64_t V) {
    memset(dW, 0, (size_t)V * (size_t)D * sizeof(float));
    for (int64_t i = 0; i < M; i++) {
        int64_t row = (int64_t)idx[i];
        if (row < 0 || row >= V) continue;
        for (int64_t j = 0; j < D; j++) dW[(size_t)row * D + j] += dout[(size_t)i * D + j];
    }
}

/* Per-(b,h) probabilities P[S,S] = softmax(Q K^T * scale), with the score
 * formed as (dot) * scale like codegen.cpp:1757-1767. */
static void attn_probs(const float* Q, const float* K, float* P, int64_t b, int64_t h,
                       int64_t S, int64_t D, int64_t Dk, float scale) {
    for (int64_t i = 0; i < S; i++) {
        float* row = P + (size_t)i * S;
        const float* q = Q + (size_t)(b * S + i) * D + h * Dk;
        for (int64_t j = 0; j < S; j++) {
            const float* k = K + (size_t)(b * S + j) * D + h * Dk;
            float a = 0.f;
            for (int64_t d = 0; d < Dk; d++) a += q[d] * k[d];
            row[j] = a * scale;
        }
        float mx = row[0];
        for (int64_t j = 1; j < S; j++) mx = mx > row[j] ? mx : row[j];
        float s = 0.f;
        for (int64_t j = 0; j < S; j++) { row[j] = expf(row[j] - mx); s += row[j]; }
        for (int64_t j = 0; j < S; j++) row[j] /= s;
    }
}

/* codegen.cpp:1724-1777 (ns_attention_fwd): Q/K/V projections, per
 * (sequence, head) softmax attention over S = BS / B positions, output
 * projection. Non-causal, no biases. */
void orc_attention_fwd(const float* x, const float* Wq, const float* Wk, const float* Wv,
                       const float* Wo, float* out, int64_t BS, int64_t D, int64_t H, int64_t S) {
    int64_t Dk = D / H;
    float scale = 1.0f / sqrtf((float)Dk);
    size_t n = (size_t)BS * D;
    float* Q = (float*)malloc(n * sizeof(float));
    float* K = (float*)malloc(n * sizeof(float));
    float* V = (float*)malloc(n * sizeof(float));
    float* O = (float*)calloc(n, sizeof(float));
    float* P = (float*)malloc((size_t)S * S * sizeof(float));
    orc_matmul(x, Wq, Q, BS, D, D);
    orc_matmul(x, Wk, K, BS, D, D);
    orc_matmul(x, Wv, V, BS, D, D);
    int64_t B = BS / S;
    for (int64_t b = 0; b < B; b++)
        for (int64_t h = 0; h < H; h++) {
            attn_probs(Q, K, P, b, h, S, D, Dk, scale);
            for (int64_t i = 0; i < S; i++)
                for (int64_t d = 0; d < Dk; d++) {
                    float a = 0.f;
                    for (int64_t j = 0; j < S; j++) a += P[(size_t)i * S + j] * V[(size_t)(b * S + j) * D + h * Dk + d];
                    O[(size_t)(b * S + i) * D + h * Dk + d] = a;
                }
        }
    orc_matmul(O, Wo, out, BS, D, D);
    free(Q); free(K); free(V); free(O); free(P);
}

/* codegen.cpp:1785-1907 (ns_attention_bwd). All five gradients from one
 * recompute; each output equals what the reference produces when asked for
 * that output alone. */
void orc_attention_bwd(const float* dout, const float* x, const float* Wq, const float* Wk,
                       const float* Wv, const float* Wo, float* dX, float* dWq, float* dWk,
                       float* dWv, float* dWo, int64_t BS, int64_t D, int64_t H, int64_t S) {
    if (D <= 0 || H <= 0 || S <= 0) return;
    int64_t Dk = D / H;
    float scale = 1.0f / sqrtf((float)Dk);
    int64_t B = BS / S;
    if (B <= 0) B = 1;
    size_t n = (size_t)BS * D;
    float* Q = (float*)malloc(n * sizeof(float));
    float* K = (float*)malloc(n * sizeof(float));
    float* V = (float*)malloc(n * sizeof(float));
    float* dQ = (float*)calloc(n, sizeof(float));
    float* dK = (float*)calloc(n, sizeof(float));
    float* dV = (float*)calloc(n, sizeof(float));
    float* dPre = (float*)malloc(n * sizeof(float));
    float* O = (float*)calloc(n, sizeof(float));
    float* P = (float*)malloc((size_t)S * S * sizeof(float));
    float* dp = (float*)malloc((size_t)S * S * sizeof(float));
    float* ds = (float*)malloc((size_t)S * S * sizeof(float));
    orc_matmul(x, Wq, Q, BS, D, D);
    orc_matmul(x, Wk, K, BS, D, D);
    orc_matmul(x, Wv, V, BS, D, D);
    /* dPre = dout Wo^T (codegen.cpp:1839-1844) */
    orc_matmul_grad_a(dout, Wo, dPre, BS, D, D);
    for (int64_t b = 0; b < B; b++)
        for (int64_t h = 0; h < H; h++) {
            attn_probs(Q, K, P, b, h, S, D, Dk, scale);
            for (int64_t i = 0; i < S; i++)
                for (int64_t d = 0; d < Dk; d++) {
                    float a = 0.f;
                    for (int64_t j = 0; j < S; j++) a += P[(size_t)i * S + j] * V[(size_t)(b * S + j) * D + h * Dk + d];
                    O[(size_t)(b * S + i) * D + h * Dk + d] = a;
                }
            for (int64_t j = 0; j < S; j++)
                for (int64_t d = 0; d < Dk; d++) {
                    float a = 0.f;
                    for (int64_t i = 0; i < S; i++) a += P[(size_t)i * S + j] * dPre[(size_t)(b * S + i) * D + h * Dk + d];
                    dV[(size_t)(b * S + j) * D + h * Dk + d] += a;
                }
            for (int64_t i = 0; i < S; i++) {
                for (int64_t j = 0; j < S; j++) {
                    float a = 0.f;
                    for (int64_t d = 0; d < Dk; d++)
                        a += V[(size_t)(b * S + j) * D + h * Dk + d] * dPre[(size_t)(b * S + i) * D + h * Dk + d];
                    dp[(size_t)i * S + j] = a;
                }
                float dot = 0.f;
                for (int64_t j = 0; j < S; j++) dot += P[(size_t)i * S + j] * dp[(size_t)i * S + j];
                for (int64_t j = 0; j < S; j++) ds[(size_t)i * S + j] = P[(size_t)i * S + j] * (dp[(size_t)i * S + j] - dot);
            }
            for (int64_t i = 0; i < S; i++)
                for (int64_t d = 0; d < Dk; d++) {
                    float a = 0.f;
                    for (int64_t j = 0; j < S; j++) a += ds[(size_t)i * S + j] * K[(size_t)(b * S + j) * D + h * Dk + d];
                    dQ[(size_t)(b * S + i) * D + h * Dk + d] += a * scale;
                }
            for (int64_t j = 0; j < S; j++)
                for (int64_t d = 0; d < Dk; d++) {
                    float a = 0.f;
                    for (int64_t i = 0; i < S; i++) a += ds[(size_t)i * S + j] * Q[(size_t)(b * S + i) * D + h * Dk + d];
                    dK[(size_t)(b * S + j) * D + h * Dk + d] += a * scale;
                }
        }
    if (dWq) orc_matmul_grad_w(x, dQ, dWq, BS, D, D);
    if (dWk) orc_matmul_grad_w(x, dK, dWk, BS, D, D);
    if (dWv) orc_matmul_grad_w(x, dV, dWv, BS, D, D);
    if (dWo) orc_matmul_grad_w(O, dout, dWo, BS, D, D);
    if (dX) {
        /* dX = dQ Wq^T + dK Wk^T + dV Wv^T, summed as (gq + gk) + gv
         * (codegen.cpp:1898-1904). */
        float* gq = (float*)malloc(n * sizeof(float));
        float* gk = (float*)malloc(n * sizeof(float));
        float* gv = (float*)malloc(n * sizeof(float));
        orc_matmul_grad_a(dQ, Wq, gq, BS, D, D);
        orc_matmul_grad_a(dK, Wk, gk, BS, D, D);
        orc_matmul_grad_a(dV, Wv, gv, BS, D, D);
        for (size_t i = 0; i < n; i++) dX[i] = gq[i] + gk[i] + gv[i];
        free(gq); free(gk); free(gv);
    }
    free(Q); free(K); free(V); free(dQ); free(dK); free(dV); free(dPre); free(O);
    free(P); free(dp); free(ds);
}

/* Router of codegen.cpp:1915-1931 / :1393-1412: logits a_e = sum_k x_k Wg[k,e]
 * (sequential in k), mx = max over live, weights expf(a_e - mx) over live,
 * best = first live maximum of the exp'd weights, p = w / sum. */
void orc_moe_route(const float* x, const float* Wg, const uint8_t* active, int32_t* best,
                   float* pbest, float* p, int64_t M, int64_t D, int64_t E) {
    float* lg = (float*)malloc((size_t)E * sizeof(float));
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        float mx = -1.0e30f, sum = 0.f;
        for (int64_t e = 0; e < E; e++) {
            float a = 0.f;
            for (int64_t k = 0; k < D; k++) a += xr[k] * Wg[(size_t)k * E + e];
            lg[e] = a;
            if ((!active || active[e]) && a > mx) mx = a;
        }
        int64_t b = -1;
        for (int64_t e = 0; e < E; e++) {
            if (active && !active[e]) continue;
            lg[e] = expf(lg[e] - mx);
            sum += lg[e];
            if (b < 0 || lg[e] > lg[b]) b = e;
        }
        best[i] = (int32_t)b;
        float pb = 0.f;
        if (sum > 0.f && b >= 0) pb = lg[b] / sum;
        if (pbest) pbest[i] = pb;
        if (p) {
            for (int64_t e = 0; e < E; e++)
                p[(size_t)i * E + e] = ((!active || active[e]) && sum > 0.f) ? lg[e] / sum : 0.f;
        }
    }
    free(lg);
}

/* Exact-erf GELU and its derivative as written in the MoE helpers
 * (codegen.cpp:1938 and :1430-1431). */
static inline float moe_gelu(float u) { return 0.5f * u * (1.f + erff(u * 0.7071067811865476f)); }
static inline float moe_gelu_d(float u) {
    return 0.5f * (1.f + erff(u * 0.7071067811865476f)) + u * expf(-u * u * 0.5f) * 0.3989422804014327f;
}

/* Expert pre-activation hpre[a] = x . We1[best][:, a] (k sequential). */
static void moe_hpre(const float* xr, const float* We1, int64_t b, int64_t D, int64_t H, float* hpre) {
    for (int64_t a = 0; a < H; a++) {
        float acc = 0.f;
        for (int64_t k = 0; k < D; k++) acc += xr[k] * We1[(size_t)b * D * H + (size_t)k * H + a];
        hpre[a] = acc;
    }
}

/* codegen.cpp:1915-1945 (ns_moe_fwd): y = p_best * GELU(x We1[b]) We2[b]. */
void orc_moe_fwd(const float* x, const float* Wg, const float* We1, const float* We2,
                 const uint8_t* active, float* out, int64_t M, int64_t D, int64_t H, int64_t E) {
    int32_t* best = (int32_t*)malloc((size_t)M * sizeof(int32_t));
    float* pb = (float*)malloc((size_t)M * sizeof(float));
    float* h = (float*)malloc((size_t)H * sizeof(float));
    orc_moe_route(x, Wg, active, best, pb, NULL, M, D, E);
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        int64_t b = best[i];
        if (b < 0) { memset(out + (size_t)i * D, 0, (size_t)D * sizeof(float)); continue; }
        moe_hpre(xr, We1, b, D, H, h);
        for (int64_t a = 0; a < H; a++) h[a] = moe_gelu(h[a]);
        for (int64_t j = 0; j < D; j++) {
            float acc = 0.f;
            for (int64_t a = 0; a < H; a++) acc += h[a] * We2[(size_t)b * H * D + (size_t)a * D + j];
            out[(size_t)i * D + j] = pb[i] * acc;
        }
    }
    free(best); free(pb); free(h);
}

/* dpre2[a] = dout . We2[b][a, :] (j sequential). */
static void moe_dpre2(const float* dr, const float* We2, int64_t b, int64_t D, int64_t H, float* dpre2) {
    for (int64_t a = 0; a < H; a++) {
        float acc = 0.f;
        for (int64_t j = 0; j < D; j++) acc += dr[j] * We2[(size_t)b * H * D + (size_t)a * D + j];
        dpre2[a] = acc;
    }
}

/* codegen.cpp:1388-1443 (ns_moe_grad_x): gate path through the live softmax
 * plus the routed expert path. dx is ACCUMULATED into (the reference zeroes
 * it first at the call site, codegen.cpp:3070). */
void orc_moe_grad_x(const float* dout, const float* x, const float* Wg, const float* We1,
                    const float* We2, const uint8_t* active, float* dx,
                    int64_t M, int64_t D, int64_t H, int64_t E) {
    int32_t* best = (int32_t*)malloc((size_t)M * sizeof(int32_t));
    float* pb = (float*)malloc((size_t)M * sizeof(float));
    float* p = (float*)malloc((size_t)M * E * sizeof(float));
    float* h = (float*)malloc((size_t)H * sizeof(float));
    float* dpre2 = (float*)malloc((size_t)H * sizeof(float));
    float* dH = (float*)malloc((size_t)H * sizeof(float));
    orc_moe_route(x, Wg, active, best, pb, p, M, D, E);
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        const float* dr = dout + (size_t)i * D;
        float* o = dx + (size_t)i * D;
        int64_t b = best[i];
        if (b < 0) continue; /* the reference would index We1 at -1 here */
        moe_hpre(xr, We1, b, D, H, h);
        moe_dpre2(dr, We2, b, D, H, dpre2);
        float dpb = 0.f;
        for (int64_t a = 0; a < H; a++) {
            const float u = h[a];
            const float ga = moe_gelu(u);
            const float gd = moe_gelu_d(u);
            dpb += ga * dpre2[a];
            dH[a] = dpre2[a] * pb[i] * gd;
        }
        const float sd = dpb * pb[i];
        for (int64_t e = 0; e < E; e++) {
            const float dg = p[(size_t)i * E + e] * ((e == b ? dpb : 0.f) - sd);
            for (int64_t k = 0; k < D; k++) o[k] += dg * Wg[(size_t)k * E + e];
        }
        for (int64_t k = 0; k < D; k++) {
            float acc = 0.f;
            for (int64_t a = 0; a < H; a++) acc += dH[a] * We1[(size_t)b * D * H + (size_t)k * H + a];
            o[k] += acc;
        }
    }
    free(best); free(pb); free(p); free(h); free(dpre2); free(dH);
}

/* codegen.cpp:1446-1491 (ns_moe_grad_wg): dWg[k,e] = sum_i x[i,k] dg[i,e],
 * accumulated token by token. */
void orc_moe_grad_wg(const float* dout, const float* x, const float* Wg, const float* We1,
                     const float* We2, const uint8_t* active, float* dWg,
                     int64_t M, int64_t D, int64_t H, int64_t E) {
    int32_t* best = (int32_t*)malloc((size_t)M * sizeof(int32_t));
    float* pb = (float*)malloc((size_t)M * sizeof(float));
    float* p = (float*)malloc((size_t)M * E * sizeof(float));
    float* h = (float*)malloc((size_t)H * sizeof(float));
    float* dpre2 = (float*)malloc((size_t)H * sizeof(float));
    orc_moe_route(x, Wg, active, best, pb, p, M, D, E);
    memset(dWg, 0, (size_t)D * E * sizeof(float));
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        const float* dr = dout + (size_t)i * D;
        int64_t b = best[i];
        float dpb = 0.f;
        if (b >= 0) {
            moe_hpre(xr, We1, b, D, H, h);
            for (int64_t a = 0; a < H; a++) h[a] = moe_gelu(h[a]);
            moe_dpre2(dr, We2, b, D, H, dpre2);
            for (int64_t a = 0; a < H; a++) dpb += h[a] * dpre2[a];
        }
        const float sd = dpb * pb[i];
        for (int64_t e = 0; e < E; e++) {
            const float dg = p[(size_t)i * E + e] * ((e == b ? dpb : 0.f) - sd);
            for (int64_t k = 0; k < D; k++) dWg[(size_t)k * E + e] += xr[k] * dg;
        }
    }
    free(best); free(pb); free(p); free(h); free(dpre2);
}

/* codegen.cpp:1494-1540 (ns_moe_grad_we1): dWe1[b][k,a] += x[i,k] dH[i,a]. */
void orc_moe_grad_we1(const float* dout, const float* x, const float* Wg, const float* We1,
                      const float* We2, const uint8_t* active, float* dWe1,
                      int64_t M, int64_t D, int64_t H, int64_t E) {
    int32_t* best = (int32_t*)malloc((size_t)M * sizeof(int32_t));
    float* pb = (float*)malloc((size_t)M * sizeof(float));
    float* h = (float*)malloc((size_t)H * sizeof(float));
    float* dpre2 = (float*)malloc((size_t)H * sizeof(float));
    orc_moe_route(x, Wg, active, best, pb, NULL, M, D, E);
    memset(dWe1, 0, (size_t)E * D * H * sizeof(float));
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        const float* dr = dout + (size_t)i * D;
        int64_t b = best[i];
        if (b < 0) continue;
        moe_hpre(xr, We1, b, D, H, h);
        moe_dpre2(dr, We2, b, D, H, dpre2);
        for (int64_t a = 0; a < H; a++) {
            const float dHa = dpre2[a] * pb[i] * moe_gelu_d(h[a]);
            for (int64_t k = 0; k < D; k++) dWe1[(size_t)b * D * H + (size_t)k * H + a] += xr[k] * dHa;
        }
    }
    free(best); free(pb); free(h); free(dpre2);
}

/* codegen.cpp:1543-1579 (ns_moe_grad_we2): dWe2[b][a,j] += gelu(h)[a] * p * dout[j]. */
void orc_moe_grad_we2(const float* dout, const float* x, const float* Wg, const float* We1,
                      const float* We2, const uint8_t* active, float* dWe2,
                      int64_t M, int64_t D, int64_t H, int64_t E) {
    (void)We2;
    int32_t* best = (int32_t*)malloc((size_t)M * sizeof(int32_t));
    float* pb = (float*)malloc((size_t)M * sizeof(float));
    float* h = (float*)malloc((size_t)H * sizeof(float));
    orc_moe_route(x, Wg, active, best, pb, NULL, M, D, E);
    memset(dWe2, 0, (size_t)E * H * D * sizeof(float));
    for (int64_t i = 0; i < M; i++) {
        const float* xr = x + (size_t)i * D;
        const float* dr = dout + (size_t)i * D;
        int64_t b = best[i];
        if (b < 0) continue;
        moe_hpre(xr, We1, b, D, H, h);
        for (int64_t a = 0; a < H; a++) h[a] = moe_gelu(h[a]);
        for (int64_t a = 0; a < H; a++)
            for (int64_t j = 0; j < D; j++)
                dWe2[(size_t)b * H * D + (size_t)a * D + j] += h[a] * pb[i] * dr[j];
    }
    free(best); free(pb); free(h);
}

/* codegen.cpp:1582-1595 (ns_loss_grad): d = (softmax(preds) - labels) / denom.
 * The reference divides by the local row count; a data-parallel step
 * divides by the global row count instead, hence the explicit denom. */
void orc_loss_grad(const float* preds, const float* labels, float* d, int64_t rows, int64_t C,
                   float denom) {
    for (int64_t r = 0; r < rows; r++) {
        const float* x = preds + (size_t)r * C;
        float mx = x[0];
        for (int64_t j = 1; j < C; j++) mx = mx > x[j] ? mx : x[j];
        float s = 0.f;
        for (int64_t j = 0; j < C; j++) s += expf(x[j] - mx);
        for (int64_t j = 0; j < C; j++) {
            float p = expf(x[j] - mx) / s;
            d[(size_t)r * C + j] = (p - labels[(size_t)r * C + j]) / denom;
        }
    }
}

/* codegen.cpp:1598-1613 (ns_cross_entropy): -sum_{y>0} log p, per row. */
void orc_cross_entropy_rows(const float* preds, const float* labels, float* row_loss,
                            int64_t rows, int64_t C) {
    for (int64_t r = 0; r < rows; r++) {
        const float* x = preds + (size_t)r * C;
        float mx = x[0];
        for (int64_t j = 1; j < C; j++) mx = mx > x[j] ? mx : x[j];
        float s = 0.f;
        for (int64_t j = 0; j < C; j++) s += expf(x[j] - mx);
        float l = 0.f;
        for (int64_t j = 0; j < C; j++) {
            float p = expf(x[j] - mx) / s;
            if (labels[(size_t)r * C + j] > 0.f) l -= logf(p);
        }
        row_loss[r] = l;
    }
}

/* The reference accumulates one running float over all rows and divides by
 * the row count (codegen.cpp:1598-1613). */
float orc_cross_entropy(const float* preds, const float* labels, int64_t rows, int64_t C) {
    float loss = 0.f;
    for (int64_t r = 0; r < rows; r++) {
        const float* x = preds + (size_t)r * C;
        float mx = x[0];
        for (int64_t j = 1; j < C; j++) mx = mx > x[j] ? mx : x[j];
        float s = 0.f;
        for (int64_t j = 0; j < C; j++) s += expf(x[j] - mx);
        for (int64_t j = 0; j < C; j++) {
            float p = expf(x[j] - mx) / s;
            if (labels[(size_t)r * C + j] > 0.f) loss -= logf(p);
        }
    }
    return loss / (float)rows;
}

/* codegen.cpp:1617-1633 (ns_orthonom): modified Gram-Schmidt over the
 * columns of G (M >= N) or over its rows (M < N). */
void orc_orthonom(float* G, size_t M, size_t N) {
    int tr = M < N;
    size_t R = tr ? N : M;
    size_t C = tr ? M : N;
#define AT(k, j) (*(tr ? &G[(j) * R + (k)] : &G[(k) * N + (j)]))
    for (size_t j = 0; j < C; j++) {
        for (size_t i = 0; i < j; i++) {
            float dot = 0.f;
            for (size_t k = 0; k < R; k++) dot += AT(k, i) * AT(k, j);
            for (size_t k = 0; k < R; k++) AT(k, j) -= dot * AT(k, i);
        }
        float nrm = 0.f;
        for (size_t k = 0; k < R; k++) nrm += AT(k, j) * AT(k, j);
        nrm = sqrtf(nrm) + 1e-30f;
        for (size_t k = 0; k < R; k++) AT(k, j) /= nrm;
    }
#undef AT
}

/* include/ns/optim/optim_params.hpp:54-62, emitted as ns_lr_schedule by
 * src/codegen/codegen.cpp:23-39. */
float orc_lr_schedule(int64_t step, int kind, int64_t warmup, int64_t total, float min_factor) {
    if (kind == 0) return 1.0f;
    if (warmup <= 0) return 1.0f;
    if (step < warmup) return (float)step / (float)warmup;
    const int64_t end = total > warmup ? total : warmup + 1;
    const int64_t s = step >= end ? end : step;
    const float t = (float)(s - warmup) / (float)(end - warmup);
    return min_factor + 0.5f * (1.0f - min_factor) * (1.0f + cosf(3.14159265f * t));
}

/* codegen.cpp:3108-3120: bias-corrected AdamW with decoupled decay scaled by
 * lr, per-tensor step counter t. */
void orc_adamw_step(float* w, const float* g, float* m, float* v, size_t n, int64_t t, float lr,
                    float beta1, float beta2, float one_minus_beta1, float one_minus_beta2,
                    float eps, float decay) {
    float b1t = 1.f - powf(beta1, (float)t), b2t = 1.f - powf(beta2, (float)t);
    for (size_t i = 0; i < n; i++) {
        float gg = g[i];
        m[i] = beta1 * m[i] + one_minus_beta1 * gg;
        v[i] = beta2 * v[i] + one_minus_beta2 * gg * gg;
        float mh = m[i] / b1t, vh = v[i] / b2t;
        w[i] -= (lr * mh / (sqrtf(vh) + eps)) + (decay * lr) * w[i];
    }
}

/* codegen.cpp:3099-3107: m = momentum*m + g; MGS(m); w -= lr*sqrt(min(r,c))*m
 * + (decay*lr)*w; m = 0. */
void orc_muon_mgs_step(float* w, const float* g, float* mom, int64_t r, int64_t c, float lr,
                       float momentum, float decay) {
    size_t n = (size_t)r * (size_t)c;
    for (size_t i = 0; i < n; i++) mom[i] = momentum * mom[i] + g[i];
    orc_orthonom(mom, (size_t)r, (size_t)c);
    float rank = sqrtf((float)(r < c ? r : c));
    float le = lr * rank;
    for (size_t i = 0; i < n; i++) w[i] -= le * mom[i] + (decay * lr) * w[i];
    memset(mom, 0, n * sizeof(float));
}

/* Newton-Schulz quintic iteration X <- aX + (bA + cA^2) X, A = X X^T, on the
 * orientation with rows <= cols, after normalising by the Frobenius norm
 * (coefficients as cited in include/ns/optim/muon.hpp:19-21). fp32, with
 * double accumulators for the oracle's own accuracy. */
void orc_newton_schulz5(float* X, int64_t r, int64_t c, int steps) {
    const double a = 3.4445, b = -4.7750, cc = 2.0315;
    int tr = r > c;
    int64_t R = tr ? c : r, C = tr ? r : c;
    double* Y = (double*)malloc((size_t)R * C * sizeof(double));
    double* A = (double*)malloc((size_t)R * R * sizeof(double));
    double* B = (double*)malloc((size_t)R * R * sizeof(double));
    double* T = (double*)malloc((size_t)R * C * sizeof(double));
    double nrm = 0.0;
    for (int64_t i = 0; i < R; i++)
        for (int64_t j = 0; j < C; j++) {
            double v = tr ? X[(size_t)j * c + i] : X[(size_t)i * c + j];
            Y[(size_t)i * C + j] = v;
            nrm += v * v;
        }
    nrm = sqrt(nrm) + 1e-7;
    for (size_t i = 0; i < (size_t)R * C; i++) Y[i] /= nrm;
    for (int s = 0; s < steps; s++) {
        for (int64_t i = 0; i < R; i++)
            for (int64_t j = 0; j < R; j++) {
                double acc = 0.0;
                for (int64_t k = 0; k < C; k++) acc += Y[(size_t)i * C + k] * Y[(size_t)j * C + k];
                A[(size_t)i * R + j] = acc;
            }
        for (int64_t i = 0; i < R; i++)
            for (int64_t j = 0; j < R; j++) {
                double acc = 0.0;
                for (int64_t k = 0; k < R; k++) acc += A[(size_t)i * R + k] * A[(size_t)k * R + j];
                B[(size_t)i * R + j] = b * A[(size_t)i * R + j] + cc * acc;
            }
        for (int64_t i = 0; i < R; i++)
            for (int64_t j = 0; j < C; j++) {
                double acc = 0.0;
                for (int64_t k = 0; k < R; k++) acc += B[(size_t)i * R + k] * Y[(size_t)k * C + j];
                T[(size_t)i * C + j] = a * Y[(size_t)i * C + j] + acc;
            }
        memcpy(Y, T, (size_t)R * C * sizeof(double));
    }
    for (int64_t i = 0; i < R; i++)
        for (int64_t j = 0; j < C; j++) {
            float v = (float)Y[(size_t)i * C + j];
            if (tr) X[(size_t)j * c + i] = v; else X[(size_t)i * c + j] = v;
        }
    free(Y); free(A); free(B); free(T);
}

float orc_mse(const float* p, const float* y, size_t n) {
    double acc = 0.0;
    for (size_t i = 0; i < n; i++) { double d = (double)p[i] - (double)y[i]; acc += d * d; }
    return (float)(acc / (double)n);
}

void orc_mse_grad(const float* p, const float* y, float* d, size_t n, float denom) {
    for (size_t i = 0; i < n; i++) d[i] = 2.0f * (p[i] - y[i]) / denom;
}

/* ---- data movement: the reference's CPU helpers (emitted into every CPU
 * unit by src/codegen/codegen.cpp; CUDA forms cuda_backend.cpp:93-171).
 * Scatters write updates in increasing k, so a repeated index keeps its
 * last update. Index reads outside the source (undefined in the reference)
 * read 0 here, as the device kernels do. */
void orc_transpose2d(const float* in, float* out, int64_t rows, int64_t cols) {
    for (int64_t i = 0; i < rows; i++)
        for (int64_t j = 0; j < cols; j++) out[j * rows + i] = in[i * cols + j];
}
void orc_concat2(const float* a, const float* b, float* out, int64_t rows, int64_t ca, int64_t cb) {
    for (int64_t r = 0; r < rows; r++) {
        memcpy(out + r * (ca + cb), a + r * ca, (size_t)ca * sizeof(float));
        memcpy(out + r * (ca + cb) + ca, b + r * cb, (size_t)cb * sizeof(float));
    }
}
void orc_concat0(const float* a, const float* b, float* out, int64_t ba, int64_t bb, int64_t d) {
    memcpy(out, a, (size_t)(ba * d) * sizeof(float));
    memcpy(out + ba * d, b, (size_t)(bb * d) * sizeof(float));
}
void orc_slice2(const float* in, float* out, int64_t M, int64_t C, int64_t cs, int64_t ce) {
    for (int64_t r = 0; r < M; r++) memcpy(out + r * (ce - cs), in + r * C + cs, (size_t)(ce - cs) * sizeof(float));
}
void orc_slicerows(const float* in, float* out, int64_t C, int64_t rs, int64_t re) {
    memcpy(out, in + rs * C, (size_t)((re - rs) * C) * sizeof(float));
}
void orc_index2(const float* in, const int64_t* idx, float* out, int64_t M, int64_t C, int64_t L) {
    for (int64_t r = 0; r < M; r++)
        for (int64_t k = 0; k < L; k++) out[r * L + k] = (idx[k] >= 0 && idx[k] < C) ? in[r * C + idx[k]] : 0.f;
}
void orc_indexrows(const float* in, int64_t R, const int64_t* idx, float* out, int64_t L, int64_t C) {
    for (int64_t k = 0; k < L; k++)
        for (int64_t c = 0; c < C; c++) out[k * C + c] = (idx[k] >= 0 && idx[k] < R) ? in[idx[k] * C + c] : 0.f;
}
void orc_scatter2(const float* in, const int64_t* idx, const float* upd, float* out, int64_t M, int64_t C, int64_t L) {
    memcpy(out, in, (size_t)(M * C) * sizeof(float));
    for (int64_t r = 0; r < M; r++)
        for (int64_t k = 0; k < L; k++)
            if (idx[k] >= 0 && idx[k] < C) out[r * C + idx[k]] = upd[r * L + k];
}
void orc_scatterrows(const float* in, const int64_t* idx, const float* upd, float* out, int64_t R, int64_t C,
                     int64_t L) {
    memcpy(out, in, (size_t)(R * C) * sizeof(float));
    for (int64_t k = 0; k < L; k++)
        if (idx[k] >= 0 && idx[k] < R) memcpy(out + idx[k] * C, upd + k * C, (size_t)C * sizeof(float));
}

/* ---- dropout mask (no reference counterpart for the values: the reference
 * draws its CPU mask from std::mt19937 via bernoulli_distribution,
 * codegen.cpp:2874-2893, and its CUDA mask from curand). Counter-based
 * Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC 2011), restated here
 * independently of the device code: element i keeps its value when the top
 * 24 bits of word i % 4 of Philox(counter = {i/4 lo, i/4 hi, step, site},
 * key = {k0, k1}) / 2^24 >= rate; kept elements are scaled by 1/(1 - rate). */
static uint32_t orc_mulhilo(uint32_t a, uint32_t b, uint32_t* hi) {
    uint64_t p = (uint64_t)a * (uint64_t)b;
    *hi = (uint32_t)(p >> 32);
    return (uint32_t)p;
}
void orc_dropout_mask(float* mask, size_t n, float rate, uint32_t k0, uint32_t k1, uint32_t step, uint32_t site) {
    const float scale = 1.0f / (1.0f - rate);
    for (size_t q = 0; 4 * q < n; q++) {
        uint32_t c0 = (uint32_t)q, c1 = (uint32_t)((uint64_t)q >> 32), c2 = step, c3 = site;
        uint32_t a = k0, b = k1;
        for (int r = 0; r < 10; r++) {
            uint32_t hi0, hi1;
            uint32_t lo0 = orc_mulhilo(0xD2511F53u, c0, &hi0);
            uint32_t lo1 = orc_mulhilo(0xCD9E8D57u, c2, &hi1);
            uint32_t n0 = hi1 ^ c1 ^ a, n2 = hi0 ^ c3 ^ b;
            c0 = n0;
            c1 = lo1;
            c2 = n2;
            c3 = lo0;
            a += 0x9E3779B9u;
            b += 0xBB67AE85u;
        }
        const uint32_t w[4] = {c0, c1, c2, c3};
        for (int j = 0; j < 4 && 4 * q + j < n; j++)
            mask[4 * q + j] = (float)(w[j] >> 8) * (1.0f / 16777216.0f) >= rate ? scale : 0.f;
    }
}
