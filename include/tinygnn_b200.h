/* ============================================================================
 *  tinygnn_b200.h -- the C ABI of the B200 GNN inference engine.
 *
 *  Every entry point is extern "C", takes plain pointers and sizes, and
 *  returns a tg_status; on failure tg_last_error_message() gives the text,
 *  worded like the TinyGNN exception it stands for.  No C++ or torch type
 *  crosses this boundary.
 *
 *  Two levels:
 *   1. Device-pointer entry points (tg_spmm_f32, tg_gemm_f32, ...).  Every
 *      pointer is device memory; nothing is synchronised unless stated; work
 *      is queued on `stream` (a cudaStream_t, NULL = legacy default stream).
 *      Dense matrices are row-major with an explicit leading dimension (ld,
 *      in elements, >= the logical column count).  Results match the
 *      TinyGNN CPU library bit for bit where the entry point says "exact".
 *   2. Handle entry points (tg_tensor_*, tg_model_*, at the end of this
 *      file), the surface TinyGNN's own binding (python/tinygnn_ext.cpp)
 *      exposes: tensors built from host arrays, Model, forward on host
 *      inputs, logits back to the host.
 *
 *  References are to TinyGNN source files, path:line.
 * ========================================================================== */
#ifndef TINYGNN_B200_H
#define TINYGNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TG_API __attribute__((visibility("default")))
#else
#define TG_API
#endif

/* Error model: TinyGNN throws std::invalid_argument for shape/format/bounds
 * violations (src/ops.cpp:73-98, src/tensor.cpp:46-86), std::out_of_range
 * for Tensor::at (src/tensor.cpp:137) and std::runtime_error for I/O and an
 * empty Model (src/model.cpp:52,262,361). */
typedef enum tg_status {
    TG_OK = 0,
    TG_ERR_INVALID_ARGUMENT = 1, /* std::invalid_argument */
    TG_ERR_OUT_OF_RANGE = 2,     /* std::out_of_range */
    TG_ERR_RUNTIME = 3,          /* std::runtime_error */
    TG_ERR_CUDA = 4,             /* a CUDA runtime call failed */
    TG_ERR_NCCL = 5,             /* a collective failed */
    TG_ERR_TIMEOUT = 6,          /* a bounded device or host wait ran out */
    TG_ERR_DEVICE_CHECK = 7,     /* reserved (input checks report TG_ERR_INVALID_ARGUMENT) */
    TG_ERR_NO_DEVICE = 8         /* no CUDA device (the library has no CPU path) */
} tg_status;

/* Activations applied in kernel epilogues and by tg_activation_f32
 * (src/ops.cpp:328 relu, 355 leaky_relu, 380 elu, 411 sigmoid, 441 tanh,
 * 469 gelu). */
typedef enum tg_activation {
    TG_ACT_NONE = 0,
    TG_ACT_RELU = 1,
    TG_ACT_ELU = 2,
    TG_ACT_LEAKY_RELU = 3,
    TG_ACT_SIGMOID = 4,
    TG_ACT_TANH = 5,
    TG_ACT_GELU = 6
} tg_activation;

/* SAGE aggregators (include/tinygnn/layers.hpp SAGELayer::Aggregator). */
typedef enum tg_aggregator { TG_AGG_MEAN = 0, TG_AGG_MAX = 1 } tg_aggregator;

/* Execution modes.
 *  TG_MODE_EXACT: the reference's arithmetic order (bit-identical results
 *                 for spmm/matmul/GCN/SAGE-mean aggregate-first).
 *  TG_MODE_FAST:  the byte- or flop-minimal dataflow, results within the
 *                 fp32 tolerance |d| <= 1e-5 + 1e-4 |ref| (SAGE
 *                 transform-first when F_in > F_out, split long rows). */
typedef enum tg_mode { TG_MODE_EXACT = 0, TG_MODE_FAST = 1 } tg_mode;

/* OR'ed into a gather entry point's `mode`: every row of the gathered
 * operand is readable up to its leading dimension (the buffer holds
 * rows * ld floats), so rows whose width is not a multiple of 4 can still be
 * read with 16-byte loads.  Results do not change. */
#define TG_FLAG_B_ROWS_PADDED 0x100

/* OR'ed into a GEMM's `mode` (tg_gemm_f32, tg_gemm_rowscale_f32,
 * tg_gemm_pair_f32; the `flags` of tg_gemm_peers_f32): the rows of C have
 * room up to round_up(N, 4) columns, which may then be written (the
 * epilogue applied to a zero product: act(0)), so FAST mode can store rows
 * 16 bytes at a time.  Without it nothing past column N is written. */
#define TG_FLAG_C_COLS_PADDED 0x200

/* ── library ─────────────────────────────────────────────────────────────── */
TG_API const char* tg_last_error_message(void); /* thread-local */
TG_API const char* tg_version(void);
TG_API int32_t tg_abi_version(void); /* 2 */
/* Number of CUDA devices; 0 means every compute call returns TG_ERR_NO_DEVICE. */
TG_API int32_t tg_device_count(void);
/* How many kernels this library has launched in this process (all devices);
 * used by benchmarks to count their own launches. */
TG_API uint64_t tg_kernel_launch_count(void);

/* Input CSR checks.  Every entry point that reads a caller's CSR first
 * checks it on the device -- Tensor::sparse_csr's checks (src/tensor.cpp:
 * 46-86): row_ptr non-decreasing, row_ptr[rows] == nnz, every column in
 * [0, cols) -- plus row_ptr[0] >= 0 and every row_order entry in [0, rows),
 * and returns TG_ERR_INVALID_ARGUMENT with the reference's message before
 * any kernel reads through the arrays.  The check reads row_ptr and col_ind
 * once and synchronises the stream.  A caller whose CSRs were checked
 * already (built by this library, or by tg_csr_validate) turns it off for
 * the calling thread with tg_set_csr_checks(0); returns the previous
 * setting (1 = on, the default). */
TG_API int32_t tg_set_csr_checks(int32_t enabled);

/* ── dense ops (level 1) ─────────────────────────────────────────────────── */

/* C[M,N] = A[M,K] . B[K,N]  (TinyGNN matmul, src/ops.cpp:70-162).
 * EXACT: every C[i][j] is one fused multiply-add chain over k = 0..K-1,
 * the reference's order -> bit-identical.  FAST: tcgen05 tensor cores with
 * a 3xTF32 split (within the fp32 tolerance) when lda % 4 == 0, A is
 * 16-byte aligned and N <= 256; otherwise the EXACT kernel.  Optional
 * epilogue: + bias[N] (add_bias, src/ops.cpp:622) then activation `act`
 * with parameter alpha. */
TG_API tg_status tg_gemm_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                             const float* B, int64_t ldb, float* C, int64_t ldc,
                             const float* bias, int32_t act, float alpha, int32_t mode,
                             void* stream);

/* C1 = A . B1 and C2 = A . B2 (B1, B2: K x N, ld ldb).  FAST: one
 * tensor-core pass over A with [B1 | B2] when 2N <= 256 (SAGE's W_neigh and
 * W_self on the same input); otherwise two tg_gemm_f32 products. */
TG_API tg_status tg_gemm_pair_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                                  const float* B1, const float* B2, int64_t ldb, float* C1,
                                  int64_t ldc1, float* C2, int64_t ldc2, int32_t mode, void* stream);

/* C = act([A1 | A2] . [B1; B2] + bias) (A1: M x K1, A2: M x K2, B1: K1 x N,
 * B2: K2 x N): SAGELayer's concat of the aggregate and the node's own row
 * feeding one product (src/layers.cpp:538-752, FAST mode).  FAST with
 * 16-byte aligned rows: one tensor-core GEMM whose operand loads switch
 * from A1 to A2 along K -- the concatenation is never stored; otherwise two
 * products and a sum. */
TG_API tg_status tg_gemm_cat_f32(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1,
                                 int64_t K2, const float* A2, int64_t lda2, const float* B1,
                                 int64_t ldb1, const float* B2, int64_t ldb2, float* C, int64_t ldc,
                                 const float* bias, int32_t act, float alpha, int32_t mode,
                                 void* stream);

/* C = act(diag(row_scale) . (A . B) + bias): tg_gemm_f32 with row i of the
 * product multiplied by row_scale[i] (one rounding) before the bias.  No
 * counterpart in the reference; it carries gcn_norm's column scaling in the
 * FAST GCN forward (tg_gcn_aggregate_f32). */
TG_API tg_status tg_gemm_rowscale_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                                      const float* B, int64_t ldb, float* C, int64_t ldc,
                                      const float* row_scale, const float* bias, int32_t act,
                                      float alpha, int32_t mode, void* stream);

/* C = A1 . B1 and A2 . B2 interleaved per k (the fused dual GEMV of
 * SAGELayer::forward, src/layers.cpp:639-669): for k = 0..K-1,
 * acc = fma(A1[i][k], B1[k][j], acc); acc = fma(A2[i][k], B2[k][j], acc).
 * Columns j >= 8*floor(N/8) follow the reference's scalar tail
 * acc = acc + fma(A1, B1, A2*B2).  Then + bias, activation. */
TG_API tg_status tg_gemm_dual_f32(int64_t M, int64_t N, int64_t K, const float* A1,
                                  int64_t lda1, const float* A2, int64_t lda2,
                                  const float* B1, const float* B2, int64_t ldb, float* C,
                                  int64_t ldc, const float* bias, int32_t act, float alpha,
                                  void* stream);

/* In-place activation on a rows x cols matrix (src/ops.cpp:328-482). */
TG_API tg_status tg_activation_f32(int32_t act, float alpha, float* X, int64_t rows,
                                   int64_t cols, int64_t ld, void* stream);
/* Row-wise softmax / log_softmax in place (src/ops.cpp:506, 565);
 * cols == 0 is rejected like the reference. */
TG_API tg_status tg_softmax_rows_f32(float* X, int64_t rows, int64_t cols, int64_t ld,
                                     void* stream);
TG_API tg_status tg_log_softmax_rows_f32(float* X, int64_t rows, int64_t cols, int64_t ld,
                                         void* stream);
/* X[i][j] += bias[j]  (src/ops.cpp:622-661). */
TG_API tg_status tg_add_bias_f32(float* X, int64_t rows, int64_t cols, int64_t ld,
                                 const float* bias, void* stream);

/* ── sparse ops ──────────────────────────────────────────────────────────── */

/* C[M,F] = A . B for CSR A (M x K, int32 row_ptr[M+1] / col_ind[nnz], fp32
 * values[nnz]) and dense B (K x F)  (TinyGNN spmm, src/ops.cpp:198-297).
 * EXACT: one fused multiply-add chain per output element over the row's
 * entries in stored order -> bit-identical.  row_order (nullable) lists the
 * rows in the order to schedule them (e.g. tg_csr_degree_order); it changes
 * speed only.  Optional fused epilogue + bias[F], activation.  values ==
 * NULL: an unweighted CSR, every entry 1.0 (each update then adds the row
 * with one rounding, as the FMA with 1.0 does) -- no values are read. */
TG_API tg_status tg_spmm_f32(int64_t M, int64_t K, int64_t nnz, const int32_t* row_ptr,
                             const int32_t* col_ind, const float* values, const float* B,
                             int64_t F, int64_t ldb, float* C, int64_t ldc, const float* bias,
                             int32_t act, float alpha, const int32_t* row_order, int32_t mode,
                             void* stream);

/* Column-block passes.  For a CSR whose rows are sorted by column (as
 * TinyGNN's builders produce), tg_csr_column_splits writes the split points
 * of `nblocks` column blocks of `width` columns: splits[q*M + i] is the
 * first entry of row i with column >= q*width (q = 0..nblocks, the last
 * being row_ptr[i+1]).  tg_spmm_segment_f32 then runs one pass over entries
 * [seg_begin[i], seg_end[i]) of every row: with carry = 0 the accumulator
 * starts at zero, with carry = 1 it continues from C; bias and activation
 * are applied only with last = 1.  Passes over q = 0..nblocks-1 in order
 * reproduce tg_spmm_f32 bit for bit, while each pass gathers from only one
 * block of B's rows (an L2-sized working set, or the block another GPU has
 * just delivered).  The same for the SAGE-mean combine (the 1/deg uses the
 * whole row). */
TG_API tg_status tg_csr_column_splits(int64_t M, const int32_t* row_ptr, const int32_t* col_ind,
                                      int32_t nblocks, int64_t width, int32_t* splits_out,
                                      void* stream);
TG_API tg_status tg_spmm_segment_f32(int64_t M, int64_t K, const int32_t* row_ptr,
                                     const int32_t* col_ind, const float* values,
                                     const int32_t* seg_begin, const int32_t* seg_end,
                                     const float* B, int64_t F, int64_t ldb, float* C, int64_t ldc,
                                     const float* bias, int32_t act, float alpha,
                                     const int32_t* row_order, int32_t carry, int32_t last,
                                     int32_t mode, void* stream);
TG_API tg_status tg_sage_mean_combine_segment_f32(int64_t M, int64_t K, const int32_t* row_ptr,
                                                  const int32_t* col_ind, const int32_t* seg_begin,
                                                  const int32_t* seg_end, const float* Tn, int64_t F,
                                                  int64_t ldn, const float* Ts, int64_t lds,
                                                  const float* bias, int32_t act, float* out,
                                                  int64_t ldo, const int32_t* row_order,
                                                  int32_t carry, int32_t last, int32_t mode,
                                                  void* stream);

/* A schedule that starts the longest rows first, into order_out[M]: rows
 * in classes of decreasing stored length -- four classes per power of two
 * of (length + 1) -- and by row id within a class (a stable bucket sort). */
TG_API tg_status tg_csr_degree_order(int64_t M, const int32_t* row_ptr, int32_t* order_out,
                                     void* stream);

/* Neighbour aggregation for SAGE (src/layers.cpp:588-637 mean, 674-700 max):
 * out[i] = mean_j H[j] (plain adds in stored order, then * (1/deg)), or the
 * element-wise max (-inf start, empty rows 0).  CSR values are ignored. */
TG_API tg_status tg_sage_aggregate_f32(int64_t M, int64_t K, int64_t nnz,
                                       const int32_t* row_ptr, const int32_t* col_ind,
                                       const float* H, int64_t F, int64_t ldh, float* out,
                                       int64_t ldo, int32_t aggregator, void* stream);

/* The transform-first SAGE-mean combine (TG_MODE_FAST layers and the
 * row-partitioned driver): with Tn = H . W_neigh (gathered, K x F) and
 * Ts = H . W_self (this block's rows, M x F),
 * out[i] = act(mean_{j in row i} Tn[j] + Ts[i] + bias).  Mean is linear, so
 * this equals SAGELayer's (mean_j H[j]) . W_neigh + H[i] . W_self + b within
 * fp32 tolerance while gathering F instead of F_in floats per edge. */
TG_API tg_status tg_sage_mean_combine_f32(int64_t M, int64_t K, int64_t nnz,
                                          const int32_t* row_ptr, const int32_t* col_ind,
                                          const float* Tn, int64_t F, int64_t ldn, const float* Ts,
                                          int64_t lds, const float* bias, int32_t act, float* out,
                                          int64_t ldo, const int32_t* row_order, int32_t mode,
                                          void* stream);

/* sage_max_aggregate (src/layers.cpp:359-435), exact. */
TG_API tg_status tg_sage_max_aggregate_f32(int64_t M, int64_t K, int64_t nnz,
                                           const int32_t* row_ptr, const int32_t* col_ind,
                                           const float* H, int64_t F, int64_t ldh, float* out,
                                           int64_t ldo, void* stream);

/* edge_softmax (src/layers.cpp:768-822): per-row softmax of CSR values into
 * values_out[nnz]; empty rows produce nothing. */
TG_API tg_status tg_edge_softmax_f32(int64_t M, int64_t nnz, const int32_t* row_ptr,
                                     const float* values, float* values_out, void* stream);

/* ── graph construction (bit-exact) ──────────────────────────────────────── */

/* GraphLoader::edge_list_to_csr (src/graph_loader.cpp:211-281): COO edges
 * (src[E], dst[E]) -> CSR with rows = src, each row's columns sorted
 * ascending, values 1.0, no de-duplication.  Endpoints outside
 * [0, num_nodes) are rejected with the reference's message.  Outputs:
 * row_ptr[num_nodes+1], col_ind[E], values[E].  Synchronises `stream`. */
TG_API tg_status tg_edge_list_to_csr(int64_t num_nodes, int64_t E, const int32_t* src,
                                     const int32_t* dst, int32_t* row_ptr_out,
                                     int32_t* col_ind_out, float* values_out, void* stream);

/* add_self_loops (src/layers.cpp:71-144): capacity of col_ind_out/values_out
 * must be >= nnz + N; *nnz_out receives the result's nnz (host pointer).
 * Synchronises `stream`. */
TG_API tg_status tg_add_self_loops_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                       const int32_t* col_ind, const float* values,
                                       int32_t* row_ptr_out, int32_t* col_ind_out,
                                       float* values_out, int64_t* nnz_out, void* stream);

/* gcn_norm (src/layers.cpp:158-208): D^-1/2 (A + I) D^-1/2 with the
 * reference's float degree sum, 1/sqrtf and (v*dis_i)*dis_j rounding.
 * Same output contract as tg_add_self_loops_f32. */
TG_API tg_status tg_gcn_norm_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                 const int32_t* col_ind, const float* values,
                                 int32_t* row_ptr_out, int32_t* col_ind_out, float* values_out,
                                 int64_t* nnz_out, void* stream);

/* gcn_norm on a block of rows, for row-partitioned graphs.  The three calls
 *   tg_add_self_loops_rows_f32(rows, row_offset, ...)   -> A_r + I_r
 *   tg_csr_degree_inv_sqrt_f32(rows, ...)              -> dis_r (this block)
 *   (all-gather dis_r over the blocks into dis_all)
 *   tg_csr_scale_sym_f32(rows, ..., dis_r, dis_all)     -> (v * dis_i) * dis_j
 * give exactly the rows of tg_gcn_norm_f32's result (src/layers.cpp:158-208).
 * The block holds global rows [row_offset, row_offset + rows) with global
 * column ids; the diagonal of local row i is column i + row_offset. */
TG_API tg_status tg_add_self_loops_rows_f32(int64_t rows, int64_t row_offset, int64_t nnz,
                                            const int32_t* row_ptr, const int32_t* col_ind,
                                            const float* values, int32_t* row_ptr_out,
                                            int32_t* col_ind_out, float* values_out,
                                            int64_t* nnz_out, void* stream);
/* dis[i] = 1/sqrtf(d_i) for d_i = the row's values summed in stored order,
 * 0 when d_i is not > 0 (src/layers.cpp:170-187). */
TG_API tg_status tg_csr_degree_inv_sqrt_f32(int64_t rows, const int32_t* row_ptr,
                                            const float* values, float* dis_out, void* stream);
/* values[k] = (values[k] * dis_row[i]) * dis_col[col_ind[k]] in place
 * (src/layers.cpp:190-198). */
TG_API tg_status tg_csr_scale_sym_f32(int64_t rows, const int32_t* row_ptr, const int32_t* col_ind,
                                      float* values, const float* dis_row, const float* dis_col,
                                      void* stream);

/* The same row-block gcn_norm in two passes over the raw rows instead of
 * five (src/layers.cpp:71-208 for these rows):
 *   tg_gcn_norm_rows_degrees_f32  -> row_ptr_out[rows+1] of the self-looped
 *       block, insert_out[rows] (where each row's diagonal is inserted, -1
 *       when the row holds one) and dis_out[rows] = 1/sqrtf(degree of the
 *       self-looped row, summed in stored order);
 *   (all-gather dis over the blocks into dis_all)
 *   tg_gcn_norm_rows_fill_f32     -> col_ind_out / values_out: the self-looped
 *       rows with values (v * dis_row[i]) * dis_col[j].
 * Bit-identical to the three-call form.  col_ind_out / values_out need
 * row_ptr_out[rows] entries (at most nnz + rows); both calls are
 * asynchronous (read row_ptr_out[rows] for the count).  row_order
 * (nullable; e.g. tg_csr_degree_order of the raw rows) schedules the rows,
 * longest first, so that a hub row does not end the launch alone; it
 * changes speed only. */
TG_API tg_status tg_gcn_norm_rows_degrees_f32(int64_t rows, int64_t row_offset, int64_t nnz,
                                              const int32_t* row_ptr, const int32_t* col_ind,
                                              const float* values, const int32_t* row_order,
                                              int32_t* row_ptr_out, int32_t* insert_out,
                                              float* dis_out, void* stream);
TG_API tg_status tg_gcn_norm_rows_fill_f32(int64_t rows, int64_t row_offset, int64_t n_cols,
                                           const int32_t* row_ptr, const int32_t* col_ind,
                                           const float* values,
                                           const int32_t* row_order, const int32_t* row_ptr_out,
                                           const int32_t* insert, const float* dis_row,
                                           const float* dis_col, int32_t* col_ind_out,
                                           float* values_out, void* stream);

/* Tensor::sparse_csr validation (src/tensor.cpp:46-86) on device arrays:
 * row_ptr[rows] == nnz, row_ptr non-decreasing, 0 <= col_ind < cols.
 * Synchronises `stream`; errors carry the reference's message. */
TG_API tg_status tg_csr_validate(int64_t rows, int64_t cols, int64_t nnz,
                                 const int32_t* row_ptr, const int32_t* col_ind, void* stream);

/* The FAST GCN forward without a normalised copy of A.  gcn_norm's
 * D^-1/2 (A + I) D^-1/2 (src/layers.cpp:158-208) applied to HW factors as
 *   out_i = dis_i * (sum_j a_ij Hs_j + Hs_i),   Hs = diag(dis) . HW,
 * with d_i = (sum of row i's values) + 1 -- A + I's row sum whether or not
 * row i holds its diagonal (that entry becomes a_ii + 1) -- and dis_i =
 * 1/sqrtf(d_i) (0 when d_i <= 0).  Equal to the normalised path in exact
 * arithmetic; the roundings differ, within the fp32 tolerance
 * |d| <= 1e-5 + 1e-4 |ref| (degrees of integer-valued rows are exact).
 * The scale of a row needs only its own row, so row-partitioned callers
 * exchange Hs and need no exchange of dis.  No counterpart in the reference.
 *
 * tg_gcn_norm_scale_f32: dis_out[rows] for a block of raw rows (values read
 *   in any order; nnz = row_ptr[rows] - row_ptr[0] entries).
 * values == NULL in both: an unweighted CSR (every a_ij = 1.0); d_i is then
 *   the row length + 1 from row_ptr alone, and the aggregate reads no
 *   values -- bit-identical to passing an array of ones.
 * tg_gcn_aggregate_f32: out_i = act(dis[i] * (sum_j a_ij Hs[j] + Hs_self[i])
 *   + bias) for the M rows of a block (global columns < K; Hs K x F, ld
 *   ldh; Hs_self / dis this block's rows), the sum one fused multiply-add
 *   chain in stored order.  seg_begin / seg_end (nullable) restrict each row
 *   to entries [seg_begin[i], seg_end[i]) for column-block passes as in
 *   tg_spmm_segment_f32: the chain is carried through `out` (carry != 0)
 *   and the epilogue runs on the pass with last != 0.  mode: the
 *   TG_FLAG_B_ROWS_PADDED bit. */
TG_API tg_status tg_gcn_norm_scale_f32(int64_t rows, int64_t nnz, const int32_t* row_ptr,
                                       const float* values, float* dis_out, void* stream);
TG_API tg_status tg_gcn_aggregate_f32(int64_t M, int64_t K, int64_t nnz, const int32_t* row_ptr,
                                      const int32_t* col_ind, const float* values, const float* Hs,
                                      int64_t F, int64_t ldh, const float* Hs_self, int64_t lds,
                                      const float* dis, const float* bias, int32_t act, float* out,
                                      int64_t ldo, const int32_t* row_order, const int32_t* seg_begin,
                                      const int32_t* seg_end, int32_t carry, int32_t last,
                                      int32_t mode, void* stream);

/* ── layers ──────────────────────────────────────────────────────────────── */

/* GCNLayer::forward (src/layers.cpp:286-339): out = act(A_norm . (H . W) + b)
 * with A_norm an N x N CSR (e.g. from tg_gcn_norm_f32).  W is F_in x F_out,
 * bias nullable.  EXACT -> bit-identical.  Allocates an N x F_out scratch. */
TG_API tg_status tg_gcn_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                  const int32_t* col_ind, const float* values, const float* H,
                                  int64_t ldh, int64_t F_in, int64_t F_out, const float* W,
                                  const float* bias, int32_t act, float* out, int64_t ldo,
                                  const int32_t* row_order, int32_t mode, void* stream);

/* No counterpart in the reference: tg_gcn_layer_f32 for callers that cannot
 * let the library allocate device memory (serving loops that must not call
 * cudaMalloc after start-up, runtimes that own all device memory).  Same
 * arguments and bit-identical results as tg_gcn_layer_f32 in TG_MODE_EXACT,
 * but the N x F_out intermediate H.W lives in a fixed array inside the
 * library (TG_NOALLOC_SCRATCH_BYTES per GPU, held until the process exits),
 * so it allocates nothing: N * round_up(F_out, 4) * 4 bytes must fit, larger
 * layers return TG_ERR_INVALID_ARGUMENT.  Rows run in the caller's
 * row_order, or in natural order when it is NULL (no schedule is computed);
 * every row, hub rows included, runs in the sub-warp gather kernel (the
 * hub-row kernel's counter and side stream would allocate).
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array: calls whose work overlaps on the GPU (other
 * streams, other threads) race on it and must be serialised by the caller. */
#define TG_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
TG_API tg_status tg_gcn_layer_noalloc_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                          const int32_t* col_ind, const float* values,
                                          const float* H, int64_t ldh, int64_t F_in, int64_t F_out,
                                          const float* W, const float* bias, int32_t act, float* out,
                                          int64_t ldo, const int32_t* row_order, void* stream);

/* SAGELayer::forward (src/layers.cpp:538-752) on the raw adjacency (no
 * self-loops): out = act(AGG_j H[j] . Wn + H[i] . Ws + b).  EXACT computes
 * the aggregate first and the interleaved dual product (bit-identical for
 * mean); FAST transforms first when F_in > F_out (mean only). */
TG_API tg_status tg_sage_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                   const int32_t* col_ind, const float* H, int64_t ldh,
                                   int64_t F_in, int64_t F_out, const float* W_neigh,
                                   const float* W_self, const float* bias, int32_t aggregator,
                                   int32_t act, float* out, int64_t ldo,
                                   const int32_t* row_order, int32_t mode, void* stream);

/* Multi-head GATLayer::forward (src/layers.cpp:945-1129) plus the head
 * concat/average of Model::forward (src/model.cpp:403-422), in one pass over
 * the graph.  A is the self-looped adjacency.  W is F_in x (heads*F_out):
 * head h's weight occupies columns [h*F_out, (h+1)*F_out).  a_left, a_right,
 * bias are heads x F_out (bias nullable).  Per head: e_ij = LeakyReLU(
 * a_left.Wh_i + a_right.Wh_j), softmax over the row, out_i = sum a_ij Wh_j
 * + b, activation `act`; then heads are concatenated (out is N x heads*F_out)
 * or averaged (N x F_out).  The E x heads score tensor is never stored. */
TG_API tg_status tg_gat_layer_f32(int64_t N, int64_t nnz, const int32_t* row_ptr,
                                  const int32_t* col_ind, const float* H, int64_t ldh,
                                  int64_t F_in, int64_t heads, int64_t F_out, const float* W,
                                  const float* a_left, const float* a_right, const float* bias,
                                  float negative_slope, int32_t concat, int32_t act,
                                  float* out, int64_t ldo, const int32_t* row_order,
                                  int32_t mode, void* stream);

/* ── Fused GEMM -> exchange over NVLink (one process per GPU) ────────────
 * No counterpart in the reference (it has no multi-GPU path); these replace
 * the NCCL all-gather between a row-partitioned layer's GEMM and its gather.
 *
 * tg_ipc_get_handle: a CUDA IPC handle (TG_IPC_HANDLE_BYTES bytes) of the
 * allocation holding `ptr`, and ptr's offset in it.  tg_ipc_open_handle maps
 * another process's allocation into this one (its base; add the offset);
 * tg_ipc_close_handle unmaps it. */
#define TG_IPC_HANDLE_BYTES 64
#define TG_MAX_PEERS 7
TG_API tg_status tg_ipc_get_handle(const void* ptr, void* handle_out, int64_t* offset_out);
TG_API tg_status tg_ipc_open_handle(const void* handle, void** base_out);
TG_API tg_status tg_ipc_close_handle(void* base);

/* C = act(A . B + bias) on the tensor cores (FAST mode arithmetic; rows
 * scaled by row_scale[i] before the bias when it is not NULL), with
 * every stored row also written at the same offset of peer_C[p] (another
 * GPU's copy of C's buffer, same ldc), for p < npeers (<= TG_MAX_PEERS); once
 * a 128-row tile has landed in every copy, *peer_flags[p] += 1 (a 64-bit
 * counter in that GPU's memory; release, system scope).  Requires N <= 256,
 * lda % 4 == 0 and A 16-byte aligned.  flags: TG_FLAG_C_COLS_PADDED = the
 * rows of C and of its copies have room up to round_up(N, 4) columns, which
 * may then be written (with act(0)) so that rows are stored 16 bytes at a
 * time. */
TG_API tg_status tg_gemm_peers_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                                   const float* B, int64_t ldb, float* C, int64_t ldc,
                                   const float* bias, int32_t act, float alpha,
                                   const float* row_scale, int32_t npeers,
                                   float* const* peer_C, uint64_t* const* peer_flags, int32_t flags,
                                   void* stream);

/* Waits on the device, in stream order, until flags[i] >= targets[i] for
 * every i < n (n <= 8; targets is a host array, 0 = skip), reading with
 * acquire semantics at system scope.  A flag that has not reached its target
 * after timeout_ns gives up: tg_take_device_error then reports
 * TG_ERR_TIMEOUT. */
TG_API tg_status tg_wait_flags(const uint64_t* flags, const uint64_t* targets, int32_t n,
                               int64_t timeout_ns, void* stream);

/* Reads and clears the device error words of the pipelined kernels (the
 * tensor-core GEMM of FAST mode, the heavy-row gather used by every
 * degree-ordered spmm / SAGE aggregation, tg_wait_flags): TG_ERR_TIMEOUT
 * when one of their bounded waits ran out since the last call (that call's
 * output is then invalid).  Synchronises `stream`. */
TG_API tg_status tg_take_device_error(void* stream);

/* ── handles: TinyGNN's Tensor and Model over the C ABI ─────────────────── */
/* The drop-in API (the headers in include/tinygnn: Tensor, Model, layers) behind
 * opaque handles, for callers that bind C rather than C++ -- the surface of
 * TinyGNN's own Python binding (python/tinygnn_ext.cpp:195-452: tensors from
 * host arrays, Model construction, load_weights, forward).  Host buffers are
 * read or written only inside the call; every call here completes (and
 * synchronises the calling thread's stream) before it returns.  Calls run on
 * the current CUDA device. */
typedef struct tg_tensor_s* tg_tensor;
typedef struct tg_model_s* tg_model;

/* Tensor::dense (include/tinygnn/tensor.hpp) from host rows of stride ld
 * (host NULL: zeros). */
TG_API tg_status tg_tensor_create_dense(int64_t rows, int64_t cols, const float* host, int64_t ld,
                                        tg_tensor* out);
/* Tensor::sparse_csr (src/tensor.cpp:142-182) from host arrays: row_ptr
 * [rows+1], col_ind [nnz], values [nnz] (NULL: every value 1.0, an
 * unweighted graph).  Checked on the device after the upload with the
 * reference's checks and messages (TG_ERR_INVALID_ARGUMENT). */
TG_API tg_status tg_tensor_create_csr(int64_t rows, int64_t cols, int64_t nnz, const int32_t* row_ptr,
                                      const int32_t* col_ind, const float* values, tg_tensor* out);
/* A dense tensor's values into host rows of stride ld. */
TG_API tg_status tg_tensor_download(tg_tensor t, float* host, int64_t ld);
/* New values into an existing tensor from the host, its shape and structure
 * kept: a dense tensor's rows x cols from host rows of stride ld; a CSR
 * tensor's nnz values (ld ignored; row_ptr / col_ind unchanged).  A tensor a
 * captured forward reads (tg_model_capture) takes new inputs this way
 * between replays. */
TG_API tg_status tg_tensor_upload(tg_tensor t, const float* host, int64_t ld);
/* rows, cols, nnz (rows*cols for dense) and format (1 = SparseCSR); each
 * pointer nullable. */
TG_API tg_status tg_tensor_shape(tg_tensor t, int64_t* rows, int64_t* cols, int64_t* nnz,
                                 int32_t* is_csr);
TG_API void tg_tensor_free(tg_tensor t);

/* Model (src/model.cpp:191-439).  act: TG_ACT_NONE or TG_ACT_RELU (the
 * layers' Activation); post: 0 none, 1 ReLU, 2 ELU (Model::InterActivation);
 * aggregator: TG_AGG_MEAN / TG_AGG_MAX. */
TG_API tg_status tg_model_create(tg_model* out);
TG_API tg_status tg_model_add_gcn(tg_model m, int64_t in_f, int64_t out_f, int32_t bias, int32_t act,
                                  int32_t post);
TG_API tg_status tg_model_add_sage(tg_model m, int64_t in_f, int64_t out_f, int32_t aggregator,
                                   int32_t bias, int32_t act, int32_t post);
TG_API tg_status tg_model_add_gat(tg_model m, int64_t in_f, int64_t out_f, int64_t heads,
                                  int32_t concat, float slope, int32_t bias, int32_t act,
                                  int32_t post);
/* Model::load_weights from a TGNN file (src/model.cpp:134-185, 258-305). */
TG_API tg_status tg_model_load_weights_file(tg_model m, const char* path);
/* Model::load_weights from named host tensors (the TGNN names
 * "layer{i}.weight" ..., rows x cols each, row-major). */
TG_API tg_status tg_model_load_weights(tg_model m, int32_t count, const char* const* names,
                                       const float* const* data, const int64_t* rows,
                                       const int64_t* cols);
/* Model::forward(adjacency, features) -> *out (a new dense tensor): raw
 * adjacency without self-loops; gcn_norm / add_self_loops once per call like
 * the reference.  With tg_set_fast_math(1) the GCN layers run on the raw
 * adjacency with gcn_norm as per-row scale factors (tg_gcn_aggregate_f32)
 * and the GEMMs on the tensor cores, within the fp32 tolerance; otherwise
 * bit-identical to the reference. */
TG_API tg_status tg_model_forward(tg_model m, tg_tensor adjacency, tg_tensor features, tg_tensor* out);
/* tg_model_forward from host buffers in one call (Model::forward,
 * src/model.cpp:358-439, with the tensors' construction from host arrays,
 * src/tensor.cpp:46-86, folded in): the n x n raw adjacency as CSR arrays
 * (values NULL: an unweighted graph, every value 1.0, written on the device
 * instead of crossing PCIe) and the n x feature_cols features at row stride
 * ld_features in; the last layer's n x out_cols output written to out at row
 * stride ld_out before the call returns.  The uploads are queued on a copy
 * stream and overlap the compute: the CSR first (checked on the device with
 * Tensor::sparse_csr's checks and messages as soon as it has landed), then
 * the features in row blocks; a FAST GCN (or transform-first SAGE-mean)
 * first layer multiplies and gathers block by block as the blocks land, and a one-pass FAST GCN last layer
 * returns its output in row chunks while the next chunk gathers.  Results
 * equal tg_model_forward's on tensors holding the same data.  Pinned
 * (page-locked) host buffers let the copies overlap; pageable ones work with
 * the driver's staging.  Same calling thread rules as the other handle
 * calls. */
TG_API tg_status tg_model_forward_host(tg_model m, int64_t n, int64_t nnz, const int32_t* row_ptr,
                                       const int32_t* col_ind, const float* values, const float* features,
                                       int64_t feature_cols, int64_t ld_features, float* out, int64_t out_cols,
                                       int64_t ld_out);
TG_API void tg_model_free(tg_model m);
/* Model::forward(adjacency, features) recorded once as a CUDA graph (after
 * one eager run) and replayed: for small graphs, where launching a
 * forward's couple of dozen kernels costs more than their work.  The graph
 * reads the two tensors' device memory at each replay, so they must outlive
 * it (new values can be written into them between replays); FAST-mode GCN
 * and SAGE layers only (EXACT gcn_norm and GAT's self-loops read a size back
 * to the host: TG_ERR_RUNTIME).  No counterpart in the reference. */
typedef struct tg_graph_s* tg_graph;
TG_API tg_status tg_model_capture(tg_model m, tg_tensor adjacency, tg_tensor features, tg_graph* out);
/* Runs the captured forward again; complete when it returns. */
TG_API tg_status tg_graph_replay(tg_graph g);
/* The last replay's (or the capture's) output into host rows of stride ld. */
TG_API tg_status tg_graph_download(tg_graph g, float* host, int64_t ld);
TG_API void tg_graph_free(tg_graph g);
/* FAST (1) or EXACT (0) arithmetic for the handle and C++ APIs, process-wide;
 * returns the previous setting (tinygnn::set_fast_math). */
TG_API int32_t tg_set_fast_math(int32_t fast);

/* ── several GPUs: the row-partitioned forward ──────────────────────────── */
/* One process per GPU.  An n-node graph is split into equal 1-D row blocks,
 * R = ceil(n / world) rows each (rank r: rows [r R, min(n, (r+1) R))); a
 * rank holds its rows of the adjacency (global column ids) and of the
 * features.  Each layer's exchanged rows (GCN: H.W -- FAST: scaled by
 * 1/sqrt(deg); SAGE: H.W_neigh, or H when it aggregates first) are
 * all-gathered in place over NCCL, then every rank aggregates its own rows.
 * The logits equal the rows of tg_model_forward on the whole graph (bit for
 * bit in EXACT mode).  No counterpart in the reference, which runs on one
 * CPU.  NCCL (libnccl.so.2) is loaded by tg_dist_init. */
typedef struct tg_dist_s* tg_dist;

/* This rank's row block [*row_begin, *row_end) and, given the whole graph's
 * host row_ptr (nullable), its entry range [*entry_begin, *entry_end).  Host
 * only; every output pointer nullable. */
TG_API tg_status tg_dist_partition_csr(int32_t world, int32_t rank, int64_t n, const int32_t* row_ptr,
                                       int64_t* row_begin, int64_t* row_end, int64_t* entry_begin,
                                       int64_t* entry_end);
/* Joins the communicator of `world` processes on CUDA device `device` (made
 * current).  Rank 0 writes the communicator id to the file id_path (a path
 * every rank can read; remove it afterwards); the others wait for it.  Every
 * wait -- for the file, for all ranks to join, and later for each forward --
 * gives up after timeout_ms: TG_ERR_TIMEOUT, the communicator aborted. */
TG_API tg_status tg_dist_init(int32_t world, int32_t rank, int32_t device, const char* id_path,
                              int32_t timeout_ms, tg_dist* out);
/* Model::forward on this rank's rows: adjacency_rows (rows x n, global
 * columns, no self-loops), feature_rows (rows x F_in) -> *out (rows x
 * F_out).  GCN and SAGE layers.  Every rank calls it with the same model;
 * it returns once this rank's logits are computed. */
TG_API tg_status tg_dist_forward(tg_dist d, tg_model m, int64_t n, tg_tensor adjacency_rows,
                                 tg_tensor feature_rows, tg_tensor* out);
/* Leaves and frees the communicator (every rank, after its last forward). */
TG_API tg_status tg_dist_finalize(tg_dist d);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* TINYGNN_B200_H */
