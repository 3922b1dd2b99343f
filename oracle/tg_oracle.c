/* ==========================================================================
 *  oracle/tg_oracle.c -- TEST INFRASTRUCTURE ONLY (the parity checker).
 *
 *  A plain-C restatement of the TinyGNN CPU algorithms on the GNN inference
 *  hot path.  It is the oracle the CUDA path is checked against: only
 *  tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load it.
 *  The product library never links, loads or falls back to this code.
 *
 *  Arithmetic is restated operation for operation, so that results are
 *  bit-identical to the reference compiled as its own build does
 *  (-O3 + AVX2/FMA, GCC's default floating-point contraction):
 *    - every `c += a * b` of the reference becomes an explicit fmaf(a, b, c),
 *      which is what the AVX2 `_mm256_fmadd_ps` bodies and GCC's contraction
 *      of the scalar tails produce;
 *    - plain sums stay plain sums in the reference's order;
 *    - exp/log/tanh are the same libm calls the reference makes.
 *  This file is compiled with -ffp-contract=off so that the compiler adds
 *  no contraction of its own; every fused multiply-add is spelled out.
 *
 *  Each function names the reference lines it follows
 *  (paths relative to the TinyGNN source tree).
 * ========================================================================== */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

#ifdef _OPENMP
#include <omp.h>
#endif

/* Host threads the parallel loops below use (OpenMP's default team size). */
EXPORT int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets that team size (n > 0). */
EXPORT void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ── matmul: src/ops.cpp:70-162 ───────────────────────────────────────────
 * (i, k, j) loop order; C starts at zero; every C[i][j] is one fused
 * multiply-add chain over k in increasing order (ops.cpp:121-159). */
EXPORT void orc_matmul(int64_t M, int64_t K, int64_t N, const float* A,
                       const float* B, float* C) {
    memset(C, 0, (size_t)(M * N) * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i) {
        float* ci = C + i * N;
        for (int64_t k = 0; k < K; ++k) {
            const float a = A[i * K + k];
            const float* bk = B + k * N;
            for (int64_t j = 0; j < N; ++j) ci[j] = fmaf(a, bk[j], ci[j]);
        }
    }
}

/* ── spmm: src/ops.cpp:198-297 ────────────────────────────────────────────
 * Row-wise CSR x dense; C starts at zero; per output element one fused
 * multiply-add chain over the row's stored entries in stored order
 * (ops.cpp:252-294).  Empty operands return zeros (ops.cpp:234). */
EXPORT void orc_spmm(int64_t M, const int32_t* rp, const int32_t* ci,
                     const float* v, const float* B, int64_t F, float* C) {
    memset(C, 0, (size_t)(M * F) * sizeof(float));
    if (M == 0 || F == 0) return;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < M; ++i) {
        float* crow = C + i * F;
        for (int32_t nz = rp[i]; nz < rp[i + 1]; ++nz) {
            const float a = v[nz];
            const float* brow = B + (int64_t)ci[nz] * F;
            for (int64_t j = 0; j < F; ++j) crow[j] = fmaf(a, brow[j], crow[j]);
        }
    }
}

/* ── activations: src/ops.cpp:328-560 ──────────────────────────────────────
 * kind 0 relu (328), 1 leaky_relu (355), 2 elu (380), 3 sigmoid (411),
 * 4 tanh (441), 5 gelu (469), 6 softmax (506), 7 log_softmax (565). */
EXPORT int orc_activation(int kind, float alpha, float* X, int64_t rows,
                          int64_t cols) {
    const int64_t n = rows * cols;
    switch (kind) {
        case 0:
            for (int64_t i = 0; i < n; ++i) X[i] = X[i] > 0.0f ? X[i] : 0.0f; /* std::max(0.0f, x) */
            return 0;
        case 1:
            for (int64_t i = 0; i < n; ++i) X[i] = X[i] >= 0.0f ? X[i] : alpha * X[i];
            return 0;
        case 2:
            for (int64_t i = 0; i < n; ++i)
                if (X[i] < 0.0f) X[i] = alpha * (expf(X[i]) - 1.0f);
            return 0;
        case 3:
            for (int64_t i = 0; i < n; ++i) {
                if (X[i] >= 0.0f) {
                    X[i] = 1.0f / (1.0f + expf(-X[i]));
                } else {
                    const float ex = expf(X[i]);
                    X[i] = ex / (1.0f + ex);
                }
            }
            return 0;
        case 4:
            for (int64_t i = 0; i < n; ++i) X[i] = tanhf(X[i]);
            return 0;
        case 5: {
            /* ops.cpp:477-482: inner = S * (x + C*x*x*x); the add contracts
             * with the last multiply: fma((C*x)*x, x, x). */
            const float S = 0.7978845608f, Cf = 0.044715f;
            for (int64_t i = 0; i < n; ++i) {
                const float x = X[i];
                const float inner = S * fmaf((Cf * x) * x, x, x);
                X[i] = (0.5f * x) * (1.0f + tanhf(inner));
            }
            return 0;
        }
        case 6:
        case 7:
            if (cols == 0) return 1; /* softmax over an empty row: invalid (ops.cpp:510,569) */
            for (int64_t i = 0; i < rows; ++i) {
                float* row = X + i * cols;
                float mx = row[0];
                for (int64_t j = 1; j < cols; ++j)
                    if (row[j] > mx) mx = row[j];
                if (kind == 6) {
                    float s = 0.0f;
                    for (int64_t j = 0; j < cols; ++j) {
                        row[j] = expf(row[j] - mx);
                        s += row[j];
                    }
                    const float inv = 1.0f / s;
                    for (int64_t j = 0; j < cols; ++j) row[j] *= inv;
                } else {
                    float s = 0.0f;
                    for (int64_t j = 0; j < cols; ++j) s += expf(row[j] - mx);
                    const float lse = mx + logf(s);
                    for (int64_t j = 0; j < cols; ++j) row[j] -= lse;
                }
            }
            return 0;
        default:
            return 1;
    }
}

/* ── add_bias: src/ops.cpp:622-661 ── X[i][j] += b[j] */
EXPORT void orc_add_bias(float* X, int64_t rows, int64_t cols, const float* b) {
    for (int64_t i = 0; i < rows; ++i)
        for (int64_t j = 0; j < cols; ++j) X[i * cols + j] += b[j];
}

/* ── add_self_loops: src/layers.cpp:71-144 ─────────────────────────────────
 * Rows keep their stored order; a missing diagonal (1.0) is inserted before
 * the first column > i, or appended; an existing diagonal becomes v + 1.
 * Returns the output nnz.  Output arrays must hold nnz + N entries. */
EXPORT int64_t orc_add_self_loops(int64_t N, const int32_t* rp, const int32_t* ci,
                                  const float* v, int32_t* rp_out,
                                  int32_t* ci_out, float* v_out) {
    int64_t o = 0;
    for (int64_t i = 0; i < N; ++i) {
        int has_diag = 0;
        for (int32_t nz = rp[i]; nz < rp[i + 1]; ++nz)
            if (ci[nz] == (int32_t)i) { has_diag = 1; break; }
        rp_out[i] = (int32_t)o;
        int written = 0;
        for (int32_t nz = rp[i]; nz < rp[i + 1]; ++nz) {
            const int32_t c = ci[nz];
            if (!written && !has_diag && c > (int32_t)i) {
                ci_out[o] = (int32_t)i; v_out[o] = 1.0f; ++o; written = 1;
            }
            if (c == (int32_t)i) {
                ci_out[o] = c; v_out[o] = v[nz] + 1.0f; ++o; written = 1;
            } else {
                ci_out[o] = c; v_out[o] = v[nz]; ++o;
            }
        }
        if (!written) { ci_out[o] = (int32_t)i; v_out[o] = 1.0f; ++o; }
    }
    rp_out[N] = (int32_t)o;
    return o;
}

/* ── gcn_norm: src/layers.cpp:158-208 ──────────────────────────────────────
 * deg[i] = sequential float sum of the self-looped row's values (170-178);
 * dis = deg > 0 ? 1/sqrtf(deg) : 0 (181-187); v' = (v * dis_i) * dis_j
 * (190-198).  Output arrays must hold nnz + N entries. */
EXPORT int64_t orc_gcn_norm(int64_t N, const int32_t* rp, const int32_t* ci,
                            const float* v, int32_t* rp_out, int32_t* ci_out,
                            float* v_out) {
    const int64_t nnz = orc_add_self_loops(N, rp, ci, v, rp_out, ci_out, v_out);
    float* dis = (float*)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
    /* rows are independent: parallel over rows as the reference's
     * OpenMP loops are (layers.cpp:170, 190), each row's sum sequential */
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < N; ++i) {
        float d = 0.0f;
        for (int32_t nz = rp_out[i]; nz < rp_out[i + 1]; ++nz) d += v_out[nz];
        dis[i] = d > 0.0f ? 1.0f / sqrtf(d) : 0.0f;
    }
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < N; ++i) {
        const float di = dis[i];
        for (int32_t nz = rp_out[i]; nz < rp_out[i + 1]; ++nz)
            v_out[nz] = (v_out[nz] * di) * dis[ci_out[nz]];
    }
    free(dis);
    return nnz;
}

/* ── edge_list_to_csr: src/graph_loader.cpp:211-281 ────────────────────────
 * Count out-degree, exclusive prefix sum, place in input order, sort each
 * row ascending, values 1.0.  No de-duplication.  Endpoints are validated
 * first; returns the index of the first bad edge, or -1 when all are valid
 * (graph_loader.cpp:228-242).  Also the CSR step of load_cora_binary
 * (src/model.cpp:89-122), which uses the same algorithm. */
static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return (x > y) - (x < y);
}

EXPORT int64_t orc_edge_list_to_csr(int64_t N, int64_t E, const int32_t* src,
                                    const int32_t* dst, int32_t* rp,
                                    int32_t* ci, float* v) {
    for (int64_t e = 0; e < E; ++e)
        if (src[e] < 0 || src[e] >= N || dst[e] < 0 || dst[e] >= N) return e;
    int32_t* cur = (int32_t*)calloc((size_t)(N > 0 ? N : 1), sizeof(int32_t));
    memset(rp, 0, (size_t)(N + 1) * sizeof(int32_t));
    for (int64_t e = 0; e < E; ++e) rp[src[e] + 1]++;
    for (int64_t i = 0; i < N; ++i) rp[i + 1] += rp[i];
    for (int64_t e = 0; e < E; ++e) {
        const int32_t s = src[e];
        ci[rp[s] + cur[s]++] = dst[e];
    }
#pragma omp parallel for schedule(dynamic, 256)
    for (int64_t i = 0; i < N; ++i)
        qsort(ci + rp[i], (size_t)(rp[i + 1] - rp[i]), sizeof(int32_t), cmp_i32);
    for (int64_t e = 0; e < E; ++e) v[e] = 1.0f;
    free(cur);
    return -1;
}

/* ── edge_softmax: src/layers.cpp:768-822 ──────────────────────────────────
 * Per row: max, exp(v - max) with a sequential sum, scale by 1/sum; empty
 * rows untouched (their outputs are zero-initialised in the reference). */
EXPORT void orc_edge_softmax(int64_t N, const int32_t* rp, const float* v,
                             float* out) {
    for (int64_t i = 0; i < N; ++i) {
        const int32_t s = rp[i], e = rp[i + 1];
        if (s == e) continue;
        float mx = v[s];
        for (int32_t nz = s + 1; nz < e; ++nz) mx = v[nz] > mx ? v[nz] : mx;
        float sum = 0.0f;
        for (int32_t nz = s; nz < e; ++nz) {
            out[nz] = expf(v[nz] - mx);
            sum += out[nz];
        }
        if (sum > 0.0f) {
            const float inv = 1.0f / sum;
            for (int32_t nz = s; nz < e; ++nz) out[nz] *= inv;
        }
    }
}

/* ── sage_max_aggregate: src/layers.cpp:359-435 ────────────────────────────
 * Element-wise max over neighbours starting from -inf; empty rows are 0.
 * Full groups of 8 use _mm256_max_ps(r, h) = (r > h) ? r : h (411-415);
 * the tail uses std::max(r, h) = (r < h) ? h : r (416).  The two differ
 * only for signed zeros and NaN. */
EXPORT void orc_sage_max_aggregate(int64_t N, const int32_t* rp, const int32_t* ci,
                                   const float* H, int64_t F, float* out) {
    memset(out, 0, (size_t)(N * F) * sizeof(float));
    const int64_t F8 = (F / 8) * 8;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t i = 0; i < N; ++i) {
        if (rp[i] == rp[i + 1]) continue;
        float* r = out + i * F;
        for (int64_t f = 0; f < F; ++f) r[f] = -INFINITY;
        for (int32_t nz = rp[i]; nz < rp[i + 1]; ++nz) {
            const float* h = H + (int64_t)ci[nz] * F;
            for (int64_t f = 0; f < F8; ++f) r[f] = (r[f] > h[f]) ? r[f] : h[f];
            for (int64_t f = F8; f < F; ++f) r[f] = (r[f] < h[f]) ? h[f] : r[f];
        }
    }
}

/* ── GCNLayer::forward: src/layers.cpp:286-339 ─────────────────────────────
 * out = act(spmm(A_norm, matmul(H, W)) + b). */
EXPORT void orc_gcn_layer(int64_t N, const int32_t* rp, const int32_t* ci,
                          const float* v, const float* H, int64_t F_in,
                          int64_t F_out, const float* W, const float* bias,
                          int relu, float* out) {
    float* HW = (float*)malloc((size_t)(N * F_out > 0 ? N * F_out : 1) * sizeof(float));
    orc_matmul(N, F_in, F_out, H, W, HW);
    orc_spmm(N, rp, ci, v, HW, F_out, out);
    if (bias) orc_add_bias(out, N, F_out, bias);
    if (relu) orc_activation(0, 0.0f, out, N, F_out);
    free(HW);
}

/* ── SAGELayer::forward: src/layers.cpp:538-752 ────────────────────────────
 * Per row: agg = neighbour sum (plain adds, stored order; Mean) or max
 * from -inf (Max; empty rows 0), Mean scales by 1/deg with deg the row
 * length; then out[fo] accumulates over fi in increasing order with two
 * fused multiply-adds per step, neighbour term first (AVX2 body,
 * layers.cpp:643-664).  Columns past the last full group of 8 use the
 * scalar tail `out += a*wn + h*ws` (665-667), which GCC contracts to
 * out + fma(a, wn, h*ws).  Then bias (738) and activation (742-749). */
EXPORT void orc_sage_layer(int64_t N, const int32_t* rp, const int32_t* ci,
                           const float* H, int64_t F_in, int64_t F_out,
                           const float* Wn, const float* Ws, const float* bias,
                           int agg_max, int relu, float* out) {
    memset(out, 0, (size_t)(N * F_out) * sizeof(float));
    const int64_t F8 = (F_out / 8) * 8;
#pragma omp parallel
    {
        float* agg = (float*)malloc((size_t)(F_in > 0 ? F_in : 1) * sizeof(float));
#pragma omp for schedule(dynamic, 64)
        for (int64_t i = 0; i < N; ++i) {
            const int32_t s = rp[i], e = rp[i + 1];
            for (int64_t f = 0; f < F_in; ++f) agg[f] = 0.0f;
            if (!agg_max) {
                for (int32_t nz = s; nz < e; ++nz) {
                    const float* h = H + (int64_t)ci[nz] * F_in;
                    for (int64_t f = 0; f < F_in; ++f) agg[f] += h[f];
                }
                const float deg = (float)(e - s);
                if (deg > 0.0f) {
                    const float inv = 1.0f / deg;
                    for (int64_t f = 0; f < F_in; ++f) agg[f] *= inv;
                }
            } else if (s < e) {
                for (int64_t f = 0; f < F_in; ++f) agg[f] = -INFINITY;
                for (int32_t nz = s; nz < e; ++nz) {
                    const float* h = H + (int64_t)ci[nz] * F_in;
                    for (int64_t f = 0; f < F_in; ++f) agg[f] = agg[f] < h[f] ? h[f] : agg[f];
                }
            }
            float* o = out + i * F_out;
            const float* hi = H + i * F_in;
            for (int64_t fi = 0; fi < F_in; ++fi) {
                const float a = agg[fi], hv = hi[fi];
                const float* wn = Wn + fi * F_out;
                const float* ws = Ws + fi * F_out;
                for (int64_t fo = 0; fo < F8; ++fo) o[fo] = fmaf(hv, ws[fo], fmaf(a, wn[fo], o[fo]));
                for (int64_t fo = F8; fo < F_out; ++fo) o[fo] = o[fo] + fmaf(a, wn[fo], hv * ws[fo]);
            }
        }
        free(agg);
    }
    if (bias) orc_add_bias(out, N, F_out, bias);
    if (relu) orc_activation(0, 0.0f, out, N, F_out);
}

/* ── GATLayer::forward: src/layers.cpp:945-1129 ────────────────────────────
 * Wh = matmul(H, W) (982).  Scores (994-1026): eight lane accumulators
 * take fused multiply-adds over full groups of 8 features, are summed in
 * lane order from 0, and the remaining features are fused in one by one.
 * Per row (1052-1112): e = LeakyReLU(src_i + dst_j), running max from
 * -inf, exp(e - max) with a sequential sum, alpha = e * (1/sum), then
 * out = fma(alpha, Wh_j, out) in stored order.  Bias, activation. */
EXPORT void orc_gat_layer(int64_t N, const int32_t* rp, const int32_t* ci,
                          const float* H, int64_t F_in, int64_t F_out,
                          const float* W, const float* al, const float* ar,
                          const float* bias, float slope, int relu, float* out) {
    float* Wh = (float*)malloc((size_t)(N * F_out > 0 ? N * F_out : 1) * sizeof(float));
    float* ss = (float*)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
    float* ds = (float*)malloc((size_t)(N > 0 ? N : 1) * sizeof(float));
    orc_matmul(N, F_in, F_out, H, W, Wh);
    const int64_t F8 = (F_out / 8) * 8;
    for (int64_t i = 0; i < N; ++i) {
        const float* w = Wh + i * F_out;
        float ls[8] = {0}, ld[8] = {0};
        for (int64_t f = 0; f < F8; f += 8)
            for (int l = 0; l < 8; ++l) {
                ls[l] = fmaf(al[f + l], w[f + l], ls[l]);
                ld[l] = fmaf(ar[f + l], w[f + l], ld[l]);
            }
        float s = 0.0f, d = 0.0f;
        for (int l = 0; l < 8; ++l) { s += ls[l]; d += ld[l]; }
        int64_t f = F8;
        /* The reference build's vectoriser turns a tail of four or more
         * features into an in-order reduction: the first four products are
         * rounded separately and added one by one; the remaining tail
         * features are fused one by one. */
        if (F_out - F8 >= 4) {
            for (; f < F8 + 4; ++f) {
                s = s + al[f] * w[f];
                d = d + ar[f] * w[f];
            }
        }
        for (; f < F_out; ++f) {
            s = fmaf(al[f], w[f], s);
            d = fmaf(ar[f], w[f], d);
        }
        ss[i] = s;
        ds[i] = d;
    }
    memset(out, 0, (size_t)(N * F_out) * sizeof(float));
#pragma omp parallel
    {
        int32_t cap = 1;
        for (int64_t i = 0; i < N; ++i)
            if (rp[i + 1] - rp[i] > cap) cap = rp[i + 1] - rp[i];
        float* att = (float*)malloc((size_t)cap * sizeof(float));
#pragma omp for schedule(dynamic, 64)
        for (int64_t i = 0; i < N; ++i) {
            const int32_t s0 = rp[i], len = rp[i + 1] - rp[i];
            if (len == 0) continue;
            const float si = ss[i];
            float mx = -INFINITY;
            for (int32_t k = 0; k < len; ++k) {
                float e = si + ds[ci[s0 + k]];
                e = e >= 0.0f ? e : slope * e;
                att[k] = e;
                mx = mx < e ? e : mx; /* std::max(row_max, e) */
            }
            float sum = 0.0f;
            for (int32_t k = 0; k < len; ++k) {
                att[k] = expf(att[k] - mx);
                sum += att[k];
            }
            const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
            for (int32_t k = 0; k < len; ++k) att[k] *= inv;
            float* o = out + i * F_out;
            for (int32_t k = 0; k < len; ++k) {
                const float* wj = Wh + (int64_t)ci[s0 + k] * F_out;
                for (int64_t f = 0; f < F_out; ++f) o[f] = fmaf(att[k], wj[f], o[f]);
            }
        }
        free(att);
    }
    if (bias) orc_add_bias(out, N, F_out, bias);
    if (relu) orc_activation(0, 0.0f, out, N, F_out);
    free(Wh);
    free(ss);
    free(ds);
}
