/*
 * moe_oracle.c -- CPU restatement of Apertura's Gemma-4 MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed CPU
 * baseline.  The product (apertura_b200/libapt_moe.so) never links, loads or
 * calls it; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may.
 *
 * It restates, step for step and with the same rounding points, the mx:: op
 * sequence of:
 *   aptransformer/ESRouter.mm:14-32    ESRouter::routeTopK
 *   aptransformer/ESRouter.mm:34-40    ESRouter::routeWeights
 *   aptransformer/ESExperts.mm:44-60   ESExperts::sparseForward (bf16 and quantised)
 *   aptransformer/ESExperts.mm:28-42   ESExperts::forward (dense, all experts)
 *   aptransformer/ESOps.h:29-37        geluTanh (f32 internal, rounded once)
 * plus MLX's published affine quantisation (mx::quantize / mx::dequantize,
 * ml-explore/mlx @ 057cdc9ec, not vendored; called at ESExperts.mm:14,16).
 *
 * Rounding points (bf16 path, in order):
 *   router entirely f32, only w rounded to bf16            (ESRouter.mm:31)
 *   gate_up product rounded to bf16 (gather_mm out dtype)   (ESExperts.mm:52)
 *   gelu in f32, rounded to bf16                            (ESOps.h:29-37)
 *   gelu(g)*up : bf16 x bf16 -> bf16                        (ESExperts.mm:54)
 *   down product rounded to bf16                            (ESExperts.mm:57)
 *   w*out rounded to bf16, summed over k, rounded to bf16   (ESExperts.mm:59)
 * MLX's accumulator precision inside gather_mm / sum is not visible here (MLX
 * is not vendored).  This oracle accumulates every dot product in f32 with
 * eight interleaved partial sums combined pairwise, and the k-sum in f32 in k
 * order, rounding once.
 *
 * Parity status: the router structure and gelu are pinned by the reference's
 * own tests (ESPrimitivesTests.mm:44-56,71-91,171-189); the full block is
 * pinned against HF transformers' Gemma4TextRouter / Gemma4TextExperts golden
 * vectors (tests/golden/).  The reference publishes no expert-level fixtures.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------- bf16 helpers ---------------- */

static inline float bf2f(uint16_t b) {
    uint32_t u = ((uint32_t)b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* round to nearest even; NaN stays NaN */
static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rbf(float f) { return bf2f(f2bf(f)); }

float oracle_bf16_round(float f) { return rbf(f); }

/* f32 dot product: 8 interleaved partial sums, combined pairwise. */
static float dot_f32_f32(const float *a, const float *b, int n) {
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) s[l] += a[i + l] * b[i + l];
    for (; i < n; ++i) s[i & 7] += a[i] * b[i];
    float s01 = s[0] + s[1], s23 = s[2] + s[3], s45 = s[4] + s[5], s67 = s[6] + s[7];
    return (s01 + s23) + (s45 + s67);
}

/* ---------------- gelu (ESOps.h:29-37) ---------------- */

/* f32 gelu_pytorch_tanh with the reference's op order:
 *   x3 = (x*x)*x; inner = c0*(x + c1*x3); y = (0.5*x)*(1 + tanh(inner)) */
float oracle_gelu_tanh_f32(float x) {
    float x3 = (x * x) * x;
    float inner = 0.7978845608028654f * (x + 0.044715f * x3);
    return (0.5f * x) * (1.0f + tanhf(inner));
}

/* geluTanh on bf16 input: f32 internal, rounded once to bf16 */
void oracle_gelu_tanh_bf16(const uint16_t *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f2bf(oracle_gelu_tanh_f32(bf2f(x[i])));
}

/* ---------------- RMSNorm (ESRMSNorm.mm:14-28, unfused path) ----------------
 * out = bf16( (xf * rsqrt(mean(xf^2) + eps)) * f32(weight) ), weight may be NULL
 * (weightless).  Used for pre_ff_ln_2 / post_ff_ln_2 around the MoE block
 * (ESDecoderLayer.mm:67-75). */
void oracle_rms_norm(const uint16_t *x, const uint16_t *weight, int T, int H, float eps,
                     uint16_t *out) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        const uint16_t *xr = x + (int64_t)t * H;
        float s8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= H; i += 8)
            for (int l = 0; l < 8; ++l) s8[l] += bf2f(xr[i + l]) * bf2f(xr[i + l]);
        for (; i < H; ++i) s8[i & 7] += bf2f(xr[i]) * bf2f(xr[i]);
        float ss = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
        float inv = 1.0f / sqrtf(ss * (1.0f / (float)H) + eps);
        for (int j = 0; j < H; ++j) {
            float v = bf2f(xr[j]) * inv;
            if (weight) v = v * bf2f(weight[j]);
            out[(int64_t)t * H + j] = f2bf(v);
        }
    }
}

/* ---------------- router (ESRouter.mm:14-32) ---------------- */

/*
 * x [T,H] bf16, proj [E,H] bf16, scale [H] bf16, pes [E] bf16.
 * Outputs: idx [T,K] int32 (descending probability, lower index first on
 * exact ties -- argsort(-probs) ordering), w [T,K] bf16, and optionally
 * scores [T,E] f32 (pre-softmax logits), probs [T,E] f32, w_f32 [T,K] (before
 * the bf16 cast).
 */
void oracle_route_topk(const uint16_t *x, int T, int H, const uint16_t *proj,
                       const uint16_t *scale, const uint16_t *pes, int E, int K,
                       float eps, int32_t *idx, uint16_t *w, float *scores_out,
                       float *probs_out, float *w_f32_out) {
    const float root = (float)(1.0 / sqrt((double)H)); /* ESRouter.mm:12 */
    float *projf = (float *)malloc(sizeof(float) * (size_t)E * H);
    for (int64_t i = 0; i < (int64_t)E * H; ++i) projf[i] = bf2f(proj[i]);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) {
        float *h = (float *)malloc(sizeof(float) * H);
        float *sc = (float *)malloc(sizeof(float) * E);
        float *p = (float *)malloc(sizeof(float) * E);
        int *ord = (int *)malloc(sizeof(int) * E);
        const uint16_t *xr = x + (int64_t)t * H;
        /* weightless RMSNorm: ms = mean(xf*xf); h = xf * rsqrt(ms + eps) */
        float ss = 0.f;
        for (int i = 0; i < H; ++i) {
            float v = bf2f(xr[i]);
            h[i] = v;
        }
        {
            float s8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int i = 0;
            for (; i + 8 <= H; i += 8)
                for (int l = 0; l < 8; ++l) s8[l] += h[i + l] * h[i + l];
            for (; i < H; ++i) s8[i & 7] += h[i] * h[i];
            ss = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
        }
        float ms = ss * (1.0f / (float)H);
        float r = 1.0f / sqrtf(ms + eps);
        /* h = (h * scale) * H^-1/2, each product rounded in f32 */
        for (int i = 0; i < H; ++i) h[i] = ((h[i] * r) * bf2f(scale[i])) * root;
        /* scores = h . proj^T */
        for (int e = 0; e < E; ++e) sc[e] = dot_f32_f32(h, projf + (int64_t)e * H, H);
        /* softmax(precise): max-subtracted, f32 */
        float m = sc[0];
        for (int e = 1; e < E; ++e) m = sc[e] > m ? sc[e] : m;
        float den = 0.f;
        for (int e = 0; e < E; ++e) {
            p[e] = expf(sc[e] - m);
            den += p[e];
        }
        for (int e = 0; e < E; ++e) p[e] = p[e] / den;
        /* argsort(-p): descending, stable (lower index first on equal p) */
        for (int e = 0; e < E; ++e) ord[e] = e;
        for (int a = 1; a < E; ++a) { /* insertion sort, stable */
            int v = ord[a];
            int b = a - 1;
            while (b >= 0 && p[ord[b]] < p[v]) {
                ord[b + 1] = ord[b];
                --b;
            }
            ord[b + 1] = v;
        }
        float sum = 0.f;
        for (int k = 0; k < K; ++k) sum += p[ord[k]];
        for (int k = 0; k < K; ++k) {
            int e = ord[k];
            float wk = p[e] / sum;
            wk = wk * bf2f(pes[e]);
            idx[(int64_t)t * K + k] = e;
            w[(int64_t)t * K + k] = f2bf(wk);
            if (w_f32_out) w_f32_out[(int64_t)t * K + k] = wk;
        }
        if (scores_out) memcpy(scores_out + (int64_t)t * E, sc, sizeof(float) * E);
        if (probs_out) memcpy(probs_out + (int64_t)t * E, p, sizeof(float) * E);
        free(h);
        free(sc);
        free(p);
        free(ord);
    }
    free(projf);
}

/* routeWeights (ESRouter.mm:34-40): dense [T,E] bf16, zero except at idx */
void oracle_route_weights(const int32_t *idx, const uint16_t *w, int T, int E, int K,
                          uint16_t *W) {
    memset(W, 0, sizeof(uint16_t) * (size_t)T * E);
    for (int t = 0; t < T; ++t)
        for (int k = 0; k < K; ++k) W[(int64_t)t * E + idx[(int64_t)t * K + k]] = w[(int64_t)t * K + k];
}

/* ---------------- affine quantisation (mx::quantize, affine mode) ---------------- */

/*
 * mx::quantize, affine mode (called at ESExperts.mm:14,16 and
 * ESWeightLoader.mm:221), restated from MLX's published source at the pinned
 * commit ml-explore/mlx @ 057cdc9ec (mlx/fast.cpp `affine_quantize`, the CPU
 * fallback; the Metal kernel `affine_quantize` in
 * mlx/backend/metal/kernels/quantized.h computes the same per-group values).
 * Per group of `gs` consecutive elements along the last (input) axis, in f32:
 *   n = 2^bits - 1;  mask = |min| > |max|
 *   scale = max((max - min) / n, 1e-7), negated when !mask
 *   edge  = mask ? min : max         (the larger-magnitude end)
 *   q0 = rint(edge / scale);  if q0 != 0: scale = edge / q0  (zero lands on a code)
 *   bias = q0 == 0 ? 0 : edge
 *   q = clip(rint((w - bias) / scale), 0, n)   with the f32 scale and bias
 * and only then are scale and bias stored as bf16 (the weight dtype).  The
 * scale is negative when the group's larger-magnitude end is its maximum.
 * Packing: 32/bits values per uint32, element i of a row at word i*bits/32,
 * bit offset (i*bits) % 32 (low bits first), as MLX's power-of-two shifts.
 * w [rows, cols] bf16 -> q [rows, cols*bits/32] u32, s, b [rows, cols/gs] bf16.
 * Dequantisation (mx::dequantize, gather_qmm): w = scale*q + bias with the
 * stored bf16 scale and bias.
 */
void oracle_affine_params(float mn, float mx, int bits, float *scale, float *bias) {
    const float n = (float)((1 << bits) - 1);
    const int mask = fabsf(mn) > fabsf(mx);
    float sc = (mx - mn) / n;
    if (sc < 1e-7f) sc = 1e-7f;
    if (!mask) sc = -sc;
    const float edge = mask ? mn : mx;
    const float q0 = nearbyintf(edge / sc);
    if (q0 != 0.0f) sc = edge / q0;
    *scale = sc;
    *bias = q0 == 0.0f ? 0.0f : edge;
}

int oracle_quantize_affine(const uint16_t *w, int64_t rows, int cols, int gs, int bits,
                           uint32_t *q, uint16_t *s, uint16_t *b) {
    if (bits != 4 && bits != 8) return 1;
    if (cols % gs || cols % (32 / bits) || gs % (32 / bits)) return 1;
    const int per_word = 32 / bits;
    const int qmax = (1 << bits) - 1;
    const int ng = cols / gs;
    const int words = cols / per_word;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t *wr = w + r * cols;
        uint32_t *qr = q + r * words;
        for (int g = 0; g < ng; ++g) {
            float mn = bf2f(wr[g * gs]), mx = mn;
            for (int i = 1; i < gs; ++i) {
                float v = bf2f(wr[g * gs + i]);
                mn = v < mn ? v : mn;
                mx = v > mx ? v : mx;
            }
            float sc, bi;
            oracle_affine_params(mn, mx, bits, &sc, &bi);
            s[r * ng + g] = f2bf(sc);
            b[r * ng + g] = f2bf(bi);
            for (int i = 0; i < gs; i += per_word) {
                uint32_t word = 0;
                for (int l = 0; l < per_word; ++l) {
                    float v = (bf2f(wr[g * gs + i + l]) - bi) / sc;
                    int qi = (int)nearbyintf(v);
                    qi = qi < 0 ? 0 : (qi > qmax ? qmax : qi);
                    word |= ((uint32_t)qi) << (l * bits);
                }
                qr[(g * gs + i) / per_word] = word;
            }
        }
    }
    return 0;
}

/* dequantised row element: scale*q + bias in f32 */
static inline float deq(const uint32_t *qr, const uint16_t *sr, const uint16_t *br, int i,
                        int gs, int bits) {
    int per_word = 32 / bits;
    uint32_t word = qr[i / per_word];
    int qi = (int)((word >> ((i % per_word) * bits)) & ((1u << bits) - 1u));
    int g = i / gs;
    return bf2f(sr[g]) * (float)qi + bf2f(br[g]);
}

void oracle_dequantize_affine(const uint32_t *q, const uint16_t *s, const uint16_t *b,
                              int64_t rows, int cols, int gs, int bits, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const uint32_t *qr = q + r * (cols * bits / 32);
        for (int i = 0; i < cols; ++i)
            out[r * cols + i] = deq(qr, s + r * (cols / gs), b + r * (cols / gs), i, gs, bits);
    }
}

/* ---------------- experts (ESExperts.mm:44-60) ---------------- */

/* Weight source: either bf16 (gate_up [E,2I,H], down [E,H,I]) or quantised
 * triples.  Rows are converted to f32 on the fly. */
typedef struct {
    const uint16_t *gu, *dn;                     /* bf16 */
    const uint32_t *gu_q, *dn_q;                 /* packed */
    const uint16_t *gu_s, *gu_b, *dn_s, *dn_b;   /* scale / bias */
    int bits, gs;
} wsrc_t;

static void row_f32(const wsrc_t *ws, int which, int64_t row, int cols, float *dst) {
    if (!ws->bits) {
        const uint16_t *src = (which ? ws->dn : ws->gu) + row * cols;
        for (int i = 0; i < cols; ++i) dst[i] = bf2f(src[i]);
    } else {
        const uint32_t *q = (which ? ws->dn_q : ws->gu_q) + row * (cols * ws->bits / 32);
        const uint16_t *s = (which ? ws->dn_s : ws->gu_s) + row * (cols / ws->gs);
        const uint16_t *b = (which ? ws->dn_b : ws->gu_b) + row * (cols / ws->gs);
        for (int i = 0; i < cols; ++i) dst[i] = deq(q, s, b, i, ws->gs, ws->bits);
    }
}

/* One (token, expert) pair: o [H] bf16 = down(geglu(gate_up(x))) */
static void expert_one(const wsrc_t *ws, const uint16_t *xr, int H, int I, int e, uint16_t *o,
                       float *xf, float *wrow, float *y) {
    for (int i = 0; i < H; ++i) xf[i] = bf2f(xr[i]);
    int64_t gu_base = (int64_t)e * 2 * I;
    for (int j = 0; j < I; ++j) {
        row_f32(ws, 0, gu_base + j, H, wrow);
        float g = rbf(dot_f32_f32(xf, wrow, H));
        row_f32(ws, 0, gu_base + I + j, H, wrow);
        float u = rbf(dot_f32_f32(xf, wrow, H));
        float ge = rbf(oracle_gelu_tanh_f32(g));
        y[j] = rbf(ge * u);
    }
    int64_t dn_base = (int64_t)e * H;
    for (int h = 0; h < H; ++h) {
        row_f32(ws, 1, dn_base + h, I, wrow);
        o[h] = f2bf(dot_f32_f32(y, wrow, I));
    }
}

static void experts_sparse(const wsrc_t *ws, const uint16_t *x, int T, int H, int I, int K,
                           const int32_t *idx, const uint16_t *w, uint16_t *out,
                           uint16_t *pair_out) {
    int64_t P = (int64_t)T * K;
    uint16_t *po = pair_out ? pair_out : (uint16_t *)malloc(sizeof(uint16_t) * P * H);
    int maxd = H > I ? H : I;
#pragma omp parallel
    {
        float *xf = (float *)malloc(sizeof(float) * H);
        float *wrow = (float *)malloc(sizeof(float) * maxd);
        float *y = (float *)malloc(sizeof(float) * I);
#pragma omp for schedule(dynamic, 1)
        for (int64_t p = 0; p < P; ++p) {
            int t = (int)(p / K);
            expert_one(ws, x + (int64_t)t * H, H, I, idx[p], po + p * H, xf, wrow, y);
        }
        free(xf);
        free(wrow);
        free(y);
    }
    /* weighted sum over k: bf16(w*out) accumulated in f32, rounded once */
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
        for (int h = 0; h < H; ++h) {
            float acc = 0.f;
            for (int k = 0; k < K; ++k) {
                int64_t p = (int64_t)t * K + k;
                acc += rbf(bf2f(w[p]) * bf2f(po[p * H + h]));
            }
            out[(int64_t)t * H + h] = f2bf(acc);
        }
    if (!pair_out) free(po);
}

/* sparseForward with bf16 experts.  pair_out [T*K, H] (optional) receives the
 * per-(token,k) bf16 expert outputs before the weighted sum. */
void oracle_experts_sparse(const uint16_t *x, int T, int H, int I, int K, const uint16_t *gate_up,
                           const uint16_t *down, const int32_t *idx, const uint16_t *w,
                           uint16_t *out, uint16_t *pair_out) {
    wsrc_t ws;
    memset(&ws, 0, sizeof ws);
    ws.gu = gate_up;
    ws.dn = down;
    experts_sparse(&ws, x, T, H, I, K, idx, w, out, pair_out);
}

/* sparseForward with quantised experts (gather_qmm path). */
void oracle_experts_sparse_q(const uint16_t *x, int T, int H, int I, int K, const uint32_t *gu_q,
                             const uint16_t *gu_s, const uint16_t *gu_b, const uint32_t *dn_q,
                             const uint16_t *dn_s, const uint16_t *dn_b, int bits, int gs,
                             const int32_t *idx, const uint16_t *w, uint16_t *out,
                             uint16_t *pair_out) {
    wsrc_t ws;
    memset(&ws, 0, sizeof ws);
    ws.gu_q = gu_q;
    ws.gu_s = gu_s;
    ws.gu_b = gu_b;
    ws.dn_q = dn_q;
    ws.dn_s = dn_s;
    ws.dn_b = dn_b;
    ws.bits = bits;
    ws.gs = gs;
    experts_sparse(&ws, x, T, H, I, K, idx, w, out, pair_out);
}

/*
 * Dense forward (ESExperts.mm:28-42): out[t] = sum_e bf16(W[t,e] * y_e[t]).
 * Experts whose weight is exactly zero contribute exactly zero, so they are
 * skipped; the sum runs over experts in index order, f32, rounded once.
 */
void oracle_experts_dense(const uint16_t *x, int T, int H, int I, int E, const uint16_t *gate_up,
                          const uint16_t *down, const uint16_t *W, uint16_t *out) {
    wsrc_t ws;
    memset(&ws, 0, sizeof ws);
    ws.gu = gate_up;
    ws.dn = down;
    int maxd = H > I ? H : I;
#pragma omp parallel
    {
        float *xf = (float *)malloc(sizeof(float) * H);
        float *wrow = (float *)malloc(sizeof(float) * maxd);
        float *y = (float *)malloc(sizeof(float) * I);
        uint16_t *o = (uint16_t *)malloc(sizeof(uint16_t) * H);
        float *acc = (float *)malloc(sizeof(float) * H);
#pragma omp for schedule(dynamic, 1)
        for (int t = 0; t < T; ++t) {
            for (int h = 0; h < H; ++h) acc[h] = 0.f;
            for (int e = 0; e < E; ++e) {
                uint16_t we = W[(int64_t)t * E + e];
                if ((we & 0x7fff) == 0) continue;
                expert_one(&ws, x + (int64_t)t * H, H, I, e, o, xf, wrow, y);
                for (int h = 0; h < H; ++h) acc[h] += rbf(bf2f(we) * bf2f(o[h]));
            }
            for (int h = 0; h < H; ++h) out[(int64_t)t * H + h] = f2bf(acc[h]);
        }
        free(xf);
        free(wrow);
        free(y);
        free(o);
        free(acc);
    }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
