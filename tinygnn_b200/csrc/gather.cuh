// ============================================================================
//  gather.cuh -- the CSR row-gather kernel family (internal interface).
//
//  One kernel template covers every "for each row, reduce the gathered
//  feature rows of its neighbours" operation on the hot path:
//    spmm (weighted fused multiply-add chain), SAGE mean (sum then 1/deg),
//    SAGE / sage_max_aggregate max, and the transform-first SAGE combine
//    (mean + self term + bias).  Each output row is produced by a sub-warp
//    of LPR lanes that walks the row's entries in stored order, so the
//    per-element arithmetic is the reference's sequential chain.
// ============================================================================
#pragma once

#include "common.cuh"

namespace tg {

enum GatherOp : int { GATHER_SUM = 0, GATHER_MAX = 1 };

struct GatherArgs {
    int64_t M = 0;                    // output rows
    const int32_t* rp = nullptr;      // row_ptr[M+1]
    const int32_t* ci = nullptr;      // col_ind[nnz]
    const float* val = nullptr;       // values[nnz]; NULL = weight 1 (exact add)
    const int32_t* order = nullptr;   // optional row schedule
    const float* B = nullptr;         // gathered rows, K x F, ld ldb
    int64_t ldb = 0;
    int64_t F = 0;
    float* C = nullptr;               // output, M x F, ld ldc
    int64_t ldc = 0;
    const float* self = nullptr;      // optional additive term (row i), ld lds
    int64_t lds = 0;
    const float* row_scale = nullptr; // optional per-row factor (after the self term, before the bias)
    const float* bias = nullptr;      // optional bias[F]
    int act = TG_ACT_NONE;
    float alpha = 0.0f;
    int mean = 0;                     // SUM: multiply by 1/deg when deg > 0
    int64_t max_avx_cols = 0;         // MAX: columns < this use (r > h) ? r : h
    int op = GATHER_SUM;
    // B's rows are readable up to ldb (an internal buffer of K*ldb floats):
    // lets the kernel use vectors wider than F's divisibility allows.
    bool b_padded = false;
    // Without `order`, large launches compute a longest-rows-first schedule
    // in pool memory; false keeps the natural row order and allocates nothing.
    bool allow_auto_order = true;
    // Rows of the schedule long enough for the heavy-row kernel go there
    // (it needs a pool-allocated counter and a side stream); false keeps
    // every row in the sub-warp kernel -- the same arithmetic, bit for bit.
    bool allow_heavy = true;
    // Column-block pass: only entries [seg_lo[i], seg_hi[i]) of row i; the
    // accumulator starts from C (carry) and the epilogue (1/deg with the full
    // row length, self, bias, activation) runs only on the last pass, so the
    // passes in increasing column order reproduce the one-pass arithmetic.
    const int32_t* seg_lo = nullptr;
    const int32_t* seg_hi = nullptr;
    bool carry = false;
    bool last = true;
    // Heavy rows: slots [0, *heavy_count) of `order` are produced by the
    // heavy-row kernel and skipped by the sub-warp kernel (set by
    // gather_rows, never by callers; NULL = none).
    const int32_t* heavy_count = nullptr;
};

// Queues the gather on `s`.
void gather_rows(const GatherArgs& a, cudaStream_t s);

}  // namespace tg
