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
    // Hub rows: schedule slots [0, *heavy_count) are split into chunks of
    // kGatChunk entries (gat_chunk_kernel + gat_combine_kernel) and skipped by
    // gat_aggregate_kernel.  NULL = none.
    const int32_t* heavy_count = nullptr;
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

constexpr int kGatScan = 16384;   // leading schedule slots examined for hub rows
constexpr int kGatChunk = 512;    // entries per hub-row chunk

// One sub-warp's view of a destination row: lane l owns the VEC features
// starting at (s*LPR + l)*VEC, which lie inside one head (VEC | d), and keeps
// an online (max-rescaled) softmax of that head's scores over the entries
// seen so far: running max m, sum of exp, weighted sum of Wh rows.
template <int VEC, int SPL>
struct GatLane {
    int fo[SPL], hd[SPL];
    bool live[SPL];
    float si[SPL], m[SPL], ssum[SPL], acc[SPL][VEC];

    __device__ __forceinline__ void init(const GatArgs& a, int64_t row, int l, int LPR) {
        const int HD = a.H * a.d;
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
    }

    // Folds entries [start, end) of the CSR (stored order) into the state.
    template <int LPR>
    __device__ __forceinline__ void run(const GatArgs& a, unsigned mask, int l, int32_t start, int32_t end) {
        constexpr int U = 4;
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
    }

    // 1/sum, + bias, layer activation, post activation; stored at the row.
    __device__ __forceinline__ void finish(const GatArgs& a, int64_t row) const {
#pragma unroll
        for (int s = 0; s < SPL; ++s) {
            if (!live[s]) continue;
            const float inv = ssum[s] > 0.0f ? __fdiv_rn(1.0f, ssum[s]) : 0.0f;
            float v[VEC];
#pragma unroll
            for (int k = 0; k < VEC; ++k) v[k] = __fmul_rn(acc[s][k], inv);
            if (a.bias) {
#pragma unroll
                for (int k = 0; k < VEC; ++k) v[k] = __fadd_rn(v[k], __ldg(a.bias + fo[s] + k));
            }
            act_v<VEC>(v, a.act, 0.0f);
            act_v<VEC>(v, a.post, 1.0f);  // ELU alpha 1 (Model's inter-layer ELU)
#pragma unroll
            for (int k = 0; k < VEC; ++k) a.out[row * a.ldo + fo[s] + k] = v[k];
        }
    }
};

// One sub-warp of LPR lanes per destination row (rows of the schedule from
// slot *heavy_count on).
template <int VEC, int LPR, int SPL>
__global__ void __launch_bounds__(256) gat_aggregate_kernel(const GatArgs a) {
    constexpr int RPW = 32 / LPR;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const unsigned mask = (LPR == 32) ? 0xffffffffu : (((1u << LPR) - 1u) << (sub * LPR));
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
    if (slot >= a.N) return;
    if (a.heavy_count && slot < *a.heavy_count) return;  // hub rows: the chunk kernels' slots
    const int64_t row = a.order ? static_cast<int64_t>(__ldg(a.order + slot)) : slot;
    GatLane<VEC, SPL> st;
    st.init(a, row, l, LPR);
    st.template run<LPR>(a, mask, l, __ldg(a.rp + row), __ldg(a.rp + row + 1));
    st.finish(a, row);
}

// ── Hub rows ────────────────────────────────────────────────────────────────
// A row's serial chain is len x (latency / 4); on graphs whose in-degree has
// hubs (R-MAT stored incoming: tens of thousands of entries) it is the whole
// launch.  GAT's result is a softmax-weighted sum, so a hub row can be cut
// into chunks whose online-softmax states merge exactly the way the state
// absorbs one entry (rescale by exp(old max - new max)); the result stays
// within the fp32 tolerance the GAT path is held to.

// One block: hc = the leading schedule slots (at most kGatScan) whose rows
// have at least max(1023, 2^ceil(log2(nnz / 16384)) - 1) entries, shrunk
// until their chunks fit `cap` records; base[0..hc] = exclusive prefix of the
// chunk counts; *total = base[hc].
__global__ void __launch_bounds__(1024) gat_heavy_plan_kernel(int64_t N, const int32_t* rp, const int32_t* order,
                                                              int64_t cap, int32_t* hc_out, int32_t* base,
                                                              int32_t* total_out) {
    __shared__ int32_t first_light;
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t carry, limit;
    const int64_t target = (static_cast<int64_t>(rp[N]) - rp[0]) / 16384;
    int64_t p = 1;
    while (p < target) p <<= 1;
    const int32_t T = static_cast<int32_t>(p - 1 > 1023 ? p - 1 : 1023);
    const int scan = static_cast<int>(N < kGatScan ? N : kGatScan);
    if (threadIdx.x == 0) {
        first_light = scan;
        carry = 0;
        limit = -1;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < scan; t += blockDim.x) {
        const int32_t r = order[t];
        if (rp[r + 1] - rp[r] < T) atomicMin(&first_light, t);
    }
    __syncthreads();
    const int hc = first_light;
    // Exclusive prefix of chunk counts over slots [0, hc), 1024 at a time.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int t0 = 0; t0 < hc; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int32_t cnt = 0;
        if (t < hc) {
            const int32_t r = order[t];
            cnt = (rp[r + 1] - rp[r] + kGatChunk - 1) / kGatChunk;
        }
        int32_t incl = cnt;
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += y;
        }
        if (lane == 31) warp_sums[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int32_t ws = warp_sums[lane];
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t y = __shfl_up_sync(0xffffffffu, ws, d);
                if (lane >= d) ws += y;
            }
            warp_sums[lane] = ws;  // inclusive over warps
        }
        __syncthreads();
        const int32_t before = carry + (warp > 0 ? warp_sums[warp - 1] : 0);
        const int32_t excl = before + incl - cnt;
        if (t < hc) {
            base[t] = excl;
            if (excl + cnt > cap) atomicMin(reinterpret_cast<unsigned*>(&limit), static_cast<unsigned>(t));
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[31];
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int h = limit >= 0 ? limit : hc;  // slots whose chunks fit
        *hc_out = h;
        int32_t tot = 0;
        if (h > 0) {
            const int32_t r = order[h - 1];
            tot = base[h - 1] + (rp[r + 1] - rp[r] + kGatChunk - 1) / kGatChunk;
        }
        base[h] = tot;
        *total_out = tot;
    }
}

// Chunk states: every sub-warp takes chunks c = its index, + the sub-warp
// count, ... < *total; the chunk's slot is found by binary search in base.
// Record of chunk c: per lane slice q = s*LPR + l, (m, sum, acc[VEC]).
template <int VEC, int LPR, int SPL>
__global__ void __launch_bounds__(256) gat_chunk_kernel(const GatArgs a, const int32_t* base, const int32_t* total,
                                                        int64_t cap, float* rec) {
    constexpr int RPW = 32 / LPR;
    constexpr int REC = LPR * SPL * (VEC + 2);
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const unsigned mask = (LPR == 32) ? 0xffffffffu : (((1u << LPR) - 1u) << (sub * LPR));
    const int hc = *a.heavy_count;
    const int64_t n_chunks = *total < cap ? *total : cap;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5) * RPW;
    for (int64_t c = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
         c < n_chunks; c += stride) {
        int lo = 0, hi = hc;  // largest slot with base[slot] <= c
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (base[mid] <= c) lo = mid;
            else hi = mid;
        }
        const int64_t row = static_cast<int64_t>(__ldg(a.order + lo));
        const int32_t rs = __ldg(a.rp + row), re = __ldg(a.rp + row + 1);
        const int32_t cs = rs + static_cast<int32_t>((c - base[lo]) * kGatChunk);
        const int32_t ce = min(re, cs + kGatChunk);
        GatLane<VEC, SPL> st;
        st.init(a, row, l, LPR);
        st.template run<LPR>(a, mask, l, cs, ce);
        float* r = rec + c * REC;
#pragma unroll
        for (int s = 0; s < SPL; ++s) {
            float* q = r + (s * LPR + l) * (VEC + 2);
            q[0] = st.m[s];
            q[1] = st.ssum[s];
#pragma unroll
            for (int k = 0; k < VEC; ++k) q[2 + k] = st.acc[s][k];
        }
    }
}

// One sub-warp per hub slot: its chunks' states merged in chunk order, then
// the row's epilogue.
template <int VEC, int LPR, int SPL>
__global__ void __launch_bounds__(256) gat_combine_kernel(const GatArgs a, const int32_t* base, const float* rec) {
    constexpr int RPW = 32 / LPR;
    constexpr int REC = LPR * SPL * (VEC + 2);
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
    if (slot >= *a.heavy_count) return;
    const int64_t row = static_cast<int64_t>(__ldg(a.order + slot));
    GatLane<VEC, SPL> st;
    st.init(a, row, l, LPR);
    for (int32_t c = base[slot]; c < base[slot + 1]; ++c) {
        const float* r = rec + static_cast<int64_t>(c) * REC;
#pragma unroll
        for (int s = 0; s < SPL; ++s) {
            if (!st.live[s]) continue;
            const float* q = r + (s * LPR + l) * (VEC + 2);
            const float mc = q[0];
            if (mc == -INFINITY) continue;  // a chunk with nothing to add
            if (mc > st.m[s]) {
                const float sc = expf(__fsub_rn(st.m[s], mc));
                st.ssum[s] = __fmul_rn(st.ssum[s], sc);
#pragma unroll
                for (int k = 0; k < VEC; ++k) st.acc[s][k] = __fmul_rn(st.acc[s][k], sc);
                st.m[s] = mc;
            }
            const float w = expf(__fsub_rn(mc, st.m[s]));
            st.ssum[s] = fmaf(q[1], w, st.ssum[s]);
#pragma unroll
            for (int k = 0; k < VEC; ++k) st.acc[s][k] = fmaf(q[2 + k], w, st.acc[s][k]);
        }
    }
    st.finish(a, row);
}

template <int VEC, int LPR, int SPL>
void launch_gat(const GatArgs& a, int64_t nnz, cudaStream_t s) {
    constexpr int RPB = 8 * (32 / LPR);
    if (a.order && a.N >= kGatScan) {
        // Hub rows in chunks; the capacity comes from the caller's nnz, and
        // the plan admits only the hub rows whose chunks fit it.
        constexpr int REC = LPR * SPL * (VEC + 2);
        const int64_t cap = std::max<int64_t>(1, nnz / kGatChunk + kGatScan);
        Scratch<int32_t> meta(static_cast<size_t>(kGatScan + 3), s);  // base[kGatScan+1], hc, total
        Scratch<float> rec(static_cast<size_t>(cap) * REC, s);
        int32_t* hc = meta.p + kGatScan + 1;
        int32_t* total = hc + 1;
        launch("gat_heavy_plan", gat_heavy_plan_kernel, dim3(1), dim3(1024), 0, s, a.N, a.rp, a.order, cap, hc,
               meta.p, total);
        GatArgs h = a;
        h.heavy_count = hc;
        launch("gat_chunk", gat_chunk_kernel<VEC, LPR, SPL>, dim3(static_cast<unsigned>(num_sms() * 8)), dim3(256),
               0, s, h, static_cast<const int32_t*>(meta.p), static_cast<const int32_t*>(total), cap, rec.p);
        launch("gat_combine", gat_combine_kernel<VEC, LPR, SPL>, dim3(static_cast<unsigned>(ceil_div(kGatScan, RPB))),
               dim3(256), 0, s, h, static_cast<const int32_t*>(meta.p), static_cast<const float*>(rec.p));
        launch("gat_aggregate", gat_aggregate_kernel<VEC, LPR, SPL>,
               dim3(static_cast<unsigned>(ceil_div(a.N, RPB))), dim3(256), 0, s, h);
        return;
    }
    launch("gat_aggregate", gat_aggregate_kernel<VEC, LPR, SPL>, dim3(static_cast<unsigned>(ceil_div(a.N, RPB))),
           dim3(256), 0, s, a);
}

template <int VEC>
void dispatch_gat(const GatArgs& a, int64_t nnz, cudaStream_t s) {
    const int S = a.H * a.d / VEC;
    if (S <= 8) launch_gat<VEC, 8, 1>(a, nnz, s);
    else if (S <= 16) launch_gat<VEC, 16, 1>(a, nnz, s);
    else if (S <= 32) launch_gat<VEC, 32, 1>(a, nnz, s);
    else if (S <= 64) launch_gat<VEC, 32, 2>(a, nnz, s);
    else if (S <= 128) launch_gat<VEC, 32, 4>(a, nnz, s);
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
void gat_layer(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci, const float* Hf, int64_t ldh, int64_t F_in, int H,
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
    if (vec == 4) dispatch_gat<4>(g, nnz, s);
    else if (vec == 2) dispatch_gat<2>(g, nnz, s);
    else dispatch_gat<1>(g, nnz, s);

    if (!concat)
        launch("head_average", head_average_kernel, dim3(static_cast<unsigned>(ceil_div(N * d, 256))), dim3(256), 0, s,
               N, H, d, static_cast<const float*>(cat.p), HD, out, ldo, post);
}

}  // namespace tg
