// ============================================================================
//  layers.cu -- GCN / SAGE / GAT layer forwards composed from the kernels.
//
//  GCN  (src/layers.cpp:286-339): HW = H . W into a row-padded scratch
//       (EXACT: k-sequential FMA GEMM, bit-identical; FAST: 3xTF32 tensor
//       cores), then one gather pass out = act(A_norm . HW + b) with bias and
//       activation in its epilogue.
//  SAGE (src/layers.cpp:538-752): aggregate-first (mean/max gather into a
//       scratch, then the interleaved dual product with bias + activation),
//       bit-identical; FAST does the product as one tensor-core GEMM
//       [agg | H] . [Wn; Ws] whose operand loads do the concatenation; or,
//       in FAST mode with F_in > F_out (mean), transform-first: T = H .
//       [Wn | Ws] in one tensor-core pass over H, then one gather of the Wn
//       half with the self half, bias and activation fused -- fewer bytes per
//       edge.
//  GAT  (src/layers.cpp:945-1129 + src/model.cpp:403-422): gat.cu.
// ============================================================================
#include "gather.cuh"
#include "launch.cuh"

namespace tg {

void gemm(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
          int64_t ldc, const float* bias, int act, float alpha, int mode, cudaStream_t s);
void gemm_dual_exact(int64_t M, int64_t N, int64_t K, const float* A1, int64_t lda1, const float* A2, int64_t lda2,
                     const float* B1, const float* B2, int64_t ldb, float* C, int64_t ldc, const float* bias, int act,
                     float alpha, cudaStream_t s);
void gemm_pair(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B1, const float* B2,
               int64_t ldb, float* C1, int64_t ldc1, float* C2, int64_t ldc2, int mode, cudaStream_t s);
void gemm_cat(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1, int64_t K2, const float* A2,
              int64_t lda2, const float* B1, int64_t ldb1, const float* B2, int64_t ldb2, float* C, int64_t ldc,
              const float* bias, int act, float alpha, int mode, cudaStream_t s);
void gat_layer(int64_t N, int64_t nnz, const int32_t* rp, const int32_t* ci, const float* Hf, int64_t ldh, int64_t F_in, int H,
               int d, const float* W_all, const float* al, const float* ar, const float* bias, float slope,
               bool concat, int act, int post, float* out, int64_t ldo, const int32_t* order, int mode,
               cudaStream_t s);

inline int64_t pad4(int64_t n) { return (n + 3) / 4 * 4; }

void gcn_layer(int64_t N, const int32_t* rp, const int32_t* ci, const float* v, const float* H, int64_t ldh,
               int64_t F_in, int64_t F_out, const float* W, const float* bias, int act, float* out, int64_t ldo,
               const int32_t* order, int mode, cudaStream_t s) {
    if (N == 0 || F_out == 0) return;
    const int64_t ldw = pad4(F_out);
    Scratch<float> HW(static_cast<size_t>(N * ldw), s);
    gemm(N, F_out, F_in, H, ldh, W, F_out, HW.p, ldw, nullptr, TG_ACT_NONE, 0.0f, mode | TG_FLAG_C_COLS_PADDED, s);
    GatherArgs a;
    a.M = N; a.rp = rp; a.ci = ci; a.val = v; a.order = order;
    a.B = HW.p; a.ldb = ldw; a.b_padded = true; a.F = F_out;
    a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM;
    gather_rows(a, s);
}

void sage_layer(int64_t N, const int32_t* rp, const int32_t* ci, const float* H, int64_t ldh, int64_t F_in,
                int64_t F_out, const float* Wn, const float* Ws, const float* bias, int agg, int act, float* out,
                int64_t ldo, const int32_t* order, int mode, cudaStream_t s) {
    if (N == 0 || F_out == 0) return;
    const bool fast = (mode & 0xff) == TG_MODE_FAST;
    const bool transform_first = fast && (agg == TG_AGG_MEAN) && (F_in > F_out);
    if (!transform_first) {
        const int64_t lda = pad4(F_in);
        Scratch<float> A(static_cast<size_t>(N * lda), s);
        GatherArgs a;
        a.M = N; a.rp = rp; a.ci = ci; a.order = order; a.B = H; a.ldb = ldh; a.F = F_in;
        a.C = A.p; a.ldc = lda;
        if (agg == TG_AGG_MAX) { a.op = GATHER_MAX; a.max_avx_cols = 0; }
        else { a.op = GATHER_SUM; a.mean = 1; }
        gather_rows(a, s);
        if (fast)  // [agg | H] . [Wn; Ws] + b on the tensor cores, the concatenation in the operand loads
            gemm_cat(N, F_out, F_in, A.p, lda, F_in, H, ldh, Wn, F_out, Ws, F_out, out, ldo, bias, act, 0.0f, mode,
                     s);
        else       // the reference's interleaved dual product, bit for bit
            gemm_dual_exact(N, F_out, F_in, A.p, lda, H, ldh, Wn, Ws, F_out, out, ldo, bias, act, 0.0f, s);
        return;
    }
    // Transform first: Tn = H . Wn and Ts = H . Ws (side by side in one
    // padded buffer, one tensor-core pass over H), then
    // out_i = act(mean_j Tn[j] + Ts[i] + b).
    const int64_t half = pad4(F_out);
    const int64_t ldt = 2 * half;
    Scratch<float> T(static_cast<size_t>(N * ldt), s);
    gemm_pair(N, F_out, F_in, H, ldh, Wn, Ws, F_out, T.p, ldt, T.p + half, ldt, mode | TG_FLAG_C_COLS_PADDED, s);
    GatherArgs a;
    a.M = N; a.rp = rp; a.ci = ci; a.order = order;
    a.B = T.p; a.ldb = ldt; a.b_padded = true; a.F = F_out;
    a.self = T.p + half; a.lds = ldt;
    a.C = out; a.ldc = ldo; a.bias = bias; a.act = act; a.op = GATHER_SUM; a.mean = 1;
    gather_rows(a, s);
}

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_gcn_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                  const float* values, const float* H, int64_t ldh, int64_t F_in, int64_t F_out,
                                  const float* W, const float* bias, int32_t act, float* out, int64_t ldo,
                                  const int32_t* row_order, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (N < 0 || nnz < 0) invalid("GCNLayer::forward: negative size");
        if (F_in <= 0) invalid("GCNLayer: in_features must be > 0.");
        if (F_out <= 0) invalid("GCNLayer: out_features must be > 0.");
        check_ld("GCNLayer::forward", "H", ldh, F_in);
        check_ld("GCNLayer::forward", "out", ldo, F_out);
        check_csr_input(N, N, nnz, row_ptr, col_ind, as_stream(stream), row_order);
        gcn_layer(N, row_ptr, col_ind, values, H, ldh, F_in, F_out, W, bias, act, out, ldo, row_order, mode,
                  as_stream(stream));
    });
}

TG_API tg_status tg_sage_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                   const float* H, int64_t ldh, int64_t F_in, int64_t F_out, const float* W_neigh,
                                   const float* W_self, const float* bias, int32_t aggregator, int32_t act,
                                   float* out, int64_t ldo, const int32_t* row_order, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (N < 0 || nnz < 0) invalid("SAGELayer::forward: negative size");
        if (F_in <= 0) invalid("SAGELayer: in_features must be > 0.");
        if (F_out <= 0) invalid("SAGELayer: out_features must be > 0.");
        check_ld("SAGELayer::forward", "H", ldh, F_in);
        check_ld("SAGELayer::forward", "out", ldo, F_out);
        check_csr_input(N, N, nnz, row_ptr, col_ind, as_stream(stream), row_order);
        sage_layer(N, row_ptr, col_ind, H, ldh, F_in, F_out, W_neigh, W_self, bias, aggregator, act, out, ldo,
                   row_order, mode, as_stream(stream));
    });
}

TG_API tg_status tg_gat_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr, const int32_t* col_ind,
                                  const float* H, int64_t ldh, int64_t F_in, int64_t heads, int64_t F_out,
                                  const float* W, const float* a_left, const float* a_right, const float* bias,
                                  float negative_slope, int32_t concat, int32_t act, float* out, int64_t ldo,
                                  const int32_t* row_order, int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (nnz < 0) invalid("GATLayer: negative nnz");
        if (F_in <= 0) invalid("GATLayer: in_features must be > 0.");
        if (F_out <= 0) invalid("GATLayer: out_features must be > 0.");
        if (heads <= 0) invalid("GATLayer: heads must be > 0.");
        check_ld("GATLayer::forward", "H", ldh, F_in);
        check_ld("GATLayer::forward", "out", ldo, concat ? heads * F_out : F_out);
        if (N < 0) invalid("GATLayer::forward: negative size");
        check_csr_input(N, N, nnz, row_ptr, col_ind, as_stream(stream), row_order);
        gat_layer(N, nnz, row_ptr, col_ind, H, ldh, F_in, static_cast<int>(heads), static_cast<int>(F_out), W, a_left,
                  a_right, bias, negative_slope, concat != 0, act, TG_ACT_NONE, out, ldo, row_order, mode,
                  as_stream(stream));
    });
}

}  // extern "C"
