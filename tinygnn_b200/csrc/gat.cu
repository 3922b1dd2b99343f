// ============================================================================
//  gat.cu -- multi-head graph attention in one pass over the graph.
//
//  Reference: GATLayer::forward (src/layers.cpp:945-1129) run once per head
//  by Model::forward (src/model.cpp:403-422), which traverses the graph
//  `heads` times and stores per-head outputs before concatenating them.
//
//  Here:
//   1. Wh = H . W_all for all heads at once (exact GEMM, gemm.cu);
//   2. gat_scores_kernel: per node and head, src = a_left.Wh_i and
//      dst = a_right.Wh_i with the reference's AVX2 summation order
//      (eight lane accumulators over full groups of 8, summed in lane order,
//      tail folded as the reference build's vectoriser does) -> bit-identical
//      scores and logits;
//   3. gat_aggregate_kernel: one sub-warp per destination row holds all
//      heads' output features; for each incoming edge (stored order) it
//      forms e = LeakyReLU(src_i,h + dst_j,h) and folds it into an online
//      (max-rescaled) softmax and the weighted sum of Wh_j.  The E x heads
//      score tensor is never written; per edge the kernel reads col (4 B),
//      the neighbour's dst scores (4*heads B) and its Wh row (4*heads*d B).
//  Epilogue: 1/sum, + bias, layer activation, post activation, written at
//  the head's column offset (concat).
// ============================================================================
#include "launch.cuh"

namespace tg {

void gemm(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
          int64_t ldc, const float* bias, int act, float alpha, int mode, cudaStream_t s);
void csr_degree_order(int64_t M, const int32_t* rp, int32_t* out, cudaStream_t s);

namespace {

// Scores: thread per (node, head).  sd[i*2H + h] = src, sd[i*2H + H + h] = dst.
__global__ void gat_scores_kernel(int64_t N, int H, int d, const float* Wh, int64_t ldw, const float* al,
                                  const float* ar, float* sd) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= N * H) return;
    const int64_t i = t / H;
    const int h = static_cast<int>(t % H);
    const float* w = Wh + i * ldw + static_cast<int64_t>(h) * d;
    const float* pa = al + static_cast<int64_t>(h) * d;
    const float* pr = ar + static_cast<int64_t>(h) * d;
    const int d8 = (d / 8) * 8;
    float ls[8], ld[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) { ls[l] = 0.0f; ld[l] = 0.0f; }
    for (int f = 0; f < d8; f += 8)
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float x = w[f + l];
            ls[l] = fmaf(pa[f + l], x, ls[l]);
            ld[l] = fmaf(pr[f + l], x, ld[l]);
        }
    float s = 0.0f, dd = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) { s = __fadd_rn(s, ls[l]); dd = __fadd_rn(dd, ld[l]); }
    int f = d8;
    if (d - d8 >= 4)
        for (; f < d8 + 4; ++f) {
            s = __fadd_rn(s, __fmul_rn(pa[f], w[f]));
            dd = __fadd_rn(dd, __fmul_rn(pr[f], w[f]));
        }
    for (; f < d; ++f) {
        s = fmaf(pa[f], w[f], s);
        dd = fmaf(pr[f], w[f], dd);
    }
    sd[i * 2 * H + h] = s;
    sd[i * 2 * H + H + h] = dd;
}

struct GatArgs {
    int64_t N;
    const int32_t* rp; const int32_t* ci; const int32_t* order;
    const float* Wh; int64_t ldw;      // N x (H*d)
    const float* sd;                   // N x 2H scores
    int H, d;
    float slope;
    const float* bias;                 // H*d, nullable
    int act, post;                     // layer activation, post activation (ELU/ReLU/none)
    float* out; int64_t ldo;           // N x (H*d) concat
};

template <int VEC>
__device__ __forceinline__ void ldv(const float* p, float (&x)[VEC]) {
    if constexpr (VEC == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p));
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else if constexpr (VEC == 2) {
        const float2 t = __ldg(reinterpret_cast<const float2*>(p));
        x[0] = t.x; x[1] = t.y;
    } else {
        x[0] = __ldg(p);
    }
}

// One sub-warp of LPR lanes per destination row; lane l owns the VEC
// features starting at (s*LPR + l)*VEC, which lie inside one head (VEC | d).
template <int VEC, int LPR, int SPL>
__global__ void __launch_bounds__(256) gat_aggregate_kernel(const GatArgs a) {
    constexpr int RPW = 32 / LPR;
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const unsigned mask = (LPR == 32) ? 0xffffffffu : (((1u << LPR) - 1u) << (sub * LPR));
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
    if (slot >= a.N) return;
    const int64_t row = a.order ? static_cast<int64_t>(__ldg(a.order + slot)) : slot;
    const int HD = a.H * a.d;

    int fo[SPL], hd[SPL];
    bool live[SPL];
    float si[SPL], m[SPL], ssum[SPL], acc[SPL][VEC];
#pragma unroll
    for (int s = 0; s < SPL; ++s) {
        fo[s] = (s * LPR + l) * VEC;
        live[s] = fo[s] < HD;
        hd[s] = live[s] ? fo[s] / a.d : 0;
        si[s] = live[s] ? __ldg(a.sd + row * 2 * a.H + hd[s]) : 0.0f;
        m[s] = -INFINITY;
        ssum[s] = 0.0f;
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[s][k] = 0.0f;
    }

    const int32_t start = __ldg(a.rp + row), end = __ldg(a.rp + row + 1);
    for (int32_t base = start; base < end; base += LPR) {
        const int n = min(LPR, end - base);
        const int my_c = (l < n) ? __ldg(a.ci + base + l) : 0;
        for (int e0 = 0; e0 < n; e0 += U) {
            const int ne = min(U, n - e0);
            int c[U];
            float w[U][SPL][VEC], dj[U][SPL];
#pragma unroll
            for (int u = 0; u < U; ++u) c[u] = __shfl_sync(mask, my_c, min(e0 + u, n - 1), LPR);
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (u < ne)
#pragma unroll
                    for (int s = 0; s < SPL; ++s)
                        if (live[s]) {
                            ldv<VEC>(a.Wh + static_cast<int64_t>(c[u]) * a.ldw + fo[s], w[u][s]);
                            dj[u][s] = __ldg(a.sd + static_cast<int64_t>(c[u]) * 2 * a.H + a.H + hd[s]);
                        }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (u < ne)
#pragma unroll
                    for (int s = 0; s < SPL; ++s)
                        if (live[s]) {
                            float e = __fadd_rn(si[s], dj[u][s]);
                            e = e >= 0.0f ? e : __fmul_rn(a.slope, e);
                            if (e > m[s]) {  // new running max: rescale what we have
                                const float sc = expf(__fsub_rn(m[s], e));
                                ssum[s] = __fmul_rn(ssum[s], sc);
#pragma unroll
                                for (int k = 0; k < VEC; ++k) acc[s][k] = __fmul_rn(acc[s][k], sc);
                                m[s] = e;
                            }
                            const float p = expf(__fsub_rn(e, m[s]));
                            ssum[s] = __fadd_rn(ssum[s], p);
#pragma unroll
                            for (int k = 0; k < VEC; ++k) acc[s][k] = fmaf(p, w[u][s][k], acc[s][k]);
                        }
        }
    }

#pragma unroll
    for (int s = 0; s < SPL; ++s) {
        if (!live[s]) continue;
        const float inv = ssum[s] > 0.0f ? __fdiv_rn(1.0f, ssum[s]) : 0.0f;
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            float v = __fmul_rn(acc[s][k], inv);
            if (a.bias) v = __fadd_rn(v, __ldg(a.bias + fo[s] + k));
            v = apply_act(a.act, v, 0.0f);
            v = apply_act(a.post, v, 1.0f);  // ELU alpha 1 (Model's inter-layer ELU)
            a.out[row * a.ldo + fo[s] + k] = v;
        }
    }
}

template <int VEC, int LPR, int SPL>
void launch_gat(const GatArgs& a, cudaStream_t s) {
    constexpr int RPB = 8 * (32 / LPR);
    launch("gat_aggregate", gat_aggregate_kernel<VEC, LPR, SPL>, dim3(static_cast<unsigned>(ceil_div(a.N, RPB))),
           dim3(256), 0, s, a);
}

template <int VEC>
void dispatch_gat(const GatArgs& a, cudaStream_t s) {
    const int S = a.H * a.d / VEC;
    if (S <= 8) launch_gat<VEC, 8, 1>(a, s);
    else if (S <= 16) launch_gat<VEC, 16, 1>(a, s);
    else if (S <= 32) launch_gat<VEC, 32, 1>(a, s);
    else if (S <= 64) launch_gat<VEC, 32, 2>(a, s);
    else if (S <= 128) launch_gat<VEC, 32, 4>(a, s);
    else invalid("gat: heads*out_features above 512 are not supported");
}

__global__ void head_average_kernel(int64_t N, int H, int d, const float* cat, int64_t ldc, float* out, int64_t ldo,
                                    int post) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= N * d) return;
    const int64_t i = t / d;
    const int f = static_cast<int>(t % d);
    float acc = 0.0f;
    for (int h = 0; h < H; ++h) acc = __fadd_rn(acc, cat[i * ldc + static_cast<int64_t>(h) * d + f]);
    const float inv = __fdiv_rn(1.0f, static_cast<float>(H));
    out[i * ldo + f] = apply_act(post, __fmul_rn(acc, inv), 1.0f);
}

}  // namespace

// Full multi-head layer.  W_all is F_in x (H*d); a_l, a_r, bias are H*d.
void gat_layer(int64_t N, const int32_t* rp, const int32_t* ci, const float* Hf, int64_t ldh, int64_t F_in, int H,
               int d, const float* W_all, const float* al, const float* ar, const float* bias, float slope,
               bool concat, int act, int post, float* out, int64_t ldo, const int32_t* order, int mode,
               cudaStream_t s) {
    if (N == 0) return;
    const int64_t HD = static_cast<int64_t>(H) * d;
    const int64_t ldw = (HD + 3) / 4 * 4;
    Scratch<float> Wh(static_cast<size_t>(N * ldw), s);
    gemm(N, HD, F_in, Hf, ldh, W_all, HD, Wh.p, ldw, nullptr, TG_ACT_NONE, 0.0f, mode, s);
    Scratch<float> sd(static_cast<size_t>(N * 2 * H), s);
    launch("gat_scores", gat_scores_kernel, dim3(static_cast<unsigned>(ceil_div(N * H, 256))), dim3(256), 0, s, N, H,
           d, static_cast<const float*>(Wh.p), ldw, al, ar, sd.p);

    float* cat_out = out;
    int64_t cat_ld = ldo;
    Scratch<float> cat(concat ? 1 : static_cast<size_t>(N * HD), s);
    if (!concat) { cat_out = cat.p; cat_ld = HD; }

    // Longest rows first unless the caller scheduled them (see gather_rows).
    Scratch<int32_t> auto_order(order || N < 16384 ? 1 : static_cast<size_t>(N), s);
    if (!order && N >= 16384) {
        csr_degree_order(N, rp, auto_order.p, s);
        order = auto_order.p;
    }
    GatArgs g{N, rp, ci, order, Wh.p, ldw, sd.p, H, d, slope, bias, act, concat ? post : TG_ACT_NONE, cat_out, cat_ld};
    int vec = (d % 4 == 0) ? 4 : (d % 2 == 0 ? 2 : 1);
    while (vec > 1 && HD / vec < 8) vec /= 2;
    if (vec == 4) dispatch_gat<4>(g, s);
    else if (vec == 2) dispatch_gat<2>(g, s);
    else dispatch_gat<1>(g, s);

    if (!concat)
        launch("head_average", head_average_kernel, dim3(static_cast<unsigned>(ceil_div(N * d, 256))), dim3(256), 0, s,
               N, H, d, static_cast<const float*>(cat.p), HD, out, ldo, post);
}

}  // namespace tg
