// ============================================================================
//  gather_kernel.cuh -- the CSR row-gather kernel template (see gather.cuh).
//
//  One sub-warp of LPR lanes owns an output row; lane l holds SPL vectors of
//  VEC floats (features (s*LPR + l)*VEC ..).  Per row:
//   * the row's col/val are read LPR at a time into registers (one entry per
//     lane) and broadcast with shuffles; the next window is prefetched while
//     the current one is consumed;
//   * gathered rows are loaded U at a time before their updates are applied
//     in stored order (per element one fused multiply-add chain, or max);
//   * L2 policy: the CSR arrays are streamed (evict_first), the gathered
//     operand is kept (evict_last) -- it is re-read ~nnz/K times, the CSR once;
//     neither is allocated in L1 (no reuse there).
//  Epilogue: (1/deg) -> (+ self row) -> (x row scale) -> (+ bias) ->
//  activation, one rounding each, then vector or element stores depending on
//  C's alignment.
// ============================================================================
#pragma once

#include "common.cuh"
#include "gather.cuh"

namespace tg {
namespace gk {

__device__ __forceinline__ uint64_t policy_keep() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_stream() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ int32_t ld_i32(const int32_t* p, uint64_t pol) {
    int32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.s32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
    return v;
}

__device__ __forceinline__ float ld_f32(const float* p, uint64_t pol) {
    float v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
    return v;
}

template <int V>
__device__ __forceinline__ void ldv(const float* p, float (&x)[V], uint64_t pol) {
    if constexpr (V == 4) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                     : "=f"(x[0]), "=f"(x[1]), "=f"(x[2]), "=f"(x[3])
                     : "l"(p), "l"(pol));
    } else if constexpr (V == 2) {
        asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0, %1}, [%2], %3;"
                     : "=f"(x[0]), "=f"(x[1])
                     : "l"(p), "l"(pol));
    } else {
        x[0] = ld_f32(p, pol);
    }
}

template <int V>
__device__ __forceinline__ void ldv_plain(const float* p, float (&x)[V]) {
    if constexpr (V == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p));
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else if constexpr (V == 2) {
        const float2 t = __ldg(reinterpret_cast<const float2*>(p));
        x[0] = t.x; x[1] = t.y;
    } else {
        x[0] = __ldg(p);
    }
}

template <int V>
__device__ __forceinline__ void stv(float* p, const float (&x)[V]) {
    if constexpr (V == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else if constexpr (V == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    } else {
        p[0] = x[0];
    }
}

template <int OP>
__device__ __forceinline__ float reduce_step(float acc, float w, float h, bool avx_col) {
    if constexpr (OP == GATHER_SUM) {
        return fmaf(w, h, acc);  // acc += w * h with one rounding: the reference's FMA chain
    } else {
        // _mm256_max_ps(r, h) on full 8-groups, std::max(r, h) elsewhere.
        return avx_col ? ((acc > h) ? acc : h) : ((acc < h) ? h : acc);
    }
}

// Accumulator start for the features [fo, fo+VEC) of `row`: the chain stored
// by the previous column-block pass (carry) or the reduction's identity.
template <int VEC, bool CVEC>
__device__ __forceinline__ void start_acc(const GatherArgs& a, int64_t row, int64_t fo, bool live, bool full,
                                          float init, float (&acc)[VEC]) {
    if (a.carry && live) {
        if (CVEC && full) {
            ldv_plain<VEC>(a.C + row * a.ldc + fo, acc);
        } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k) acc[k] = (fo + k < a.F) ? a.C[row * a.ldc + fo + k] : init;
        }
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] = init;
    }
}

// Stores features [fo, fo+VEC) of `row`: the raw accumulator on an
// intermediate pass, else (1/deg) -> (+ self row) -> (x row scale) ->
// (+ bias) -> activation, one rounding each.
template <int OP, int VEC, bool CVEC>
__device__ __forceinline__ void finish_acc(const GatherArgs& a, int64_t row, int64_t fo, bool full, int32_t deg,
                                           const float (&acc)[VEC]) {
    if (!a.last) {
        if (CVEC && full) {
            stv<VEC>(a.C + row * a.ldc + fo, acc);
        } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k)
                if (fo + k < a.F) a.C[row * a.ldc + fo + k] = acc[k];
        }
        return;
    }
    const float inv_deg = (OP == GATHER_SUM && a.mean && deg > 0) ? __fdiv_rn(1.0f, static_cast<float>(deg)) : 1.0f;
    const float rs = a.row_scale ? a.row_scale[row] : 1.0f;
    const bool vec_io = CVEC && full;
    float x[VEC], sv[VEC], bv[VEC];
    if (vec_io) {
        if (a.self) ldv_plain<VEC>(a.self + row * a.lds + fo, sv);
        if (a.bias) ldv_plain<VEC>(a.bias + fo, bv);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const bool in = fo + k < a.F;
            sv[k] = (a.self && in) ? a.self[row * a.lds + fo + k] : 0.0f;
            bv[k] = (a.bias && in) ? a.bias[fo + k] : 0.0f;
        }
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) x[k] = (OP == GATHER_MAX && deg == 0) ? 0.0f : acc[k];
    if (OP == GATHER_SUM && a.mean && deg > 0) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) x[k] = __fmul_rn(x[k], inv_deg);
    }
    if (a.self) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) x[k] = __fadd_rn(x[k], sv[k]);
    }
    if (a.row_scale) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) x[k] = __fmul_rn(x[k], rs);
    }
    if (a.bias) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) x[k] = __fadd_rn(x[k], bv[k]);
    }
    act_v<VEC>(x, a.act, a.alpha);
    if (vec_io) {
        stv<VEC>(a.C + row * a.ldc + fo, x);
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k)
            if (fo + k < a.F) a.C[row * a.ldc + fo + k] = x[k];
    }
}

// VEC: floats per load; LPR: lanes per row; SPL: vectors per lane;
// OP: GATHER_SUM / GATHER_MAX; U: gathered rows in flight per batch;
// CVEC: C, self and bias use VEC-wide accesses (else element accesses).
template <int VEC, int LPR, int SPL, int OP, int U, bool CVEC>
__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherArgs a) {
    constexpr int RPW = 32 / LPR;
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPR;
    const int l = lane % LPR;
    const unsigned mask = (LPR == 32) ? 0xffffffffu : (((1u << LPR) - 1u) << (sub * LPR));

    const int64_t slot = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
    if (slot >= a.M) return;  // whole sub-warps leave together
    if (a.heavy_count && slot < *a.heavy_count) return;  // the heavy-row kernel's slots
    const uint64_t keep = policy_keep(), stream = policy_stream();
    const int64_t row = a.order ? static_cast<int64_t>(ld_i32(a.order + slot, stream)) : slot;

    const int64_t f0 = static_cast<int64_t>(blockIdx.y) * (LPR * SPL * VEC);  // feature pass
    bool live[SPL], full[SPL];
    int64_t fo[SPL];
#pragma unroll
    for (int s = 0; s < SPL; ++s) {
        fo[s] = f0 + static_cast<int64_t>(s * LPR + l) * VEC;
        live[s] = fo[s] < a.F;          // the vector starts inside the row
        full[s] = fo[s] + VEC <= a.F;   // ... and ends inside it (else B rows are padded)
    }

    float acc[SPL][VEC];
    const float init = (OP == GATHER_SUM) ? 0.0f : -INFINITY;
#pragma unroll
    for (int s = 0; s < SPL; ++s) start_acc<VEC, CVEC>(a, row, fo[s], live[s], full[s], init, acc[s]);

    bool avx[SPL][VEC];
#pragma unroll
    for (int s = 0; s < SPL; ++s)
#pragma unroll
        for (int k = 0; k < VEC; ++k) avx[s][k] = (fo[s] + k) < a.max_avx_cols;

    const int32_t row_begin = ld_i32(a.rp + row, stream);
    const int32_t row_end = ld_i32(a.rp + row + 1, stream);
    // a segment never reaches outside its row
    const int32_t start = a.seg_lo ? max(row_begin, ld_i32(a.seg_lo + row, stream)) : row_begin;
    const int32_t end = a.seg_hi ? min(row_end, ld_i32(a.seg_hi + row, stream)) : row_end;

    // Window of LPR entries: one (col, val) per lane; the next one is loaded
    // before the current one is consumed.
    int nx_c = 0;
    float nx_w = 1.0f;
    if (start + l < end) {
        nx_c = ld_i32(a.ci + start + l, stream);
        if (a.val) nx_w = ld_f32(a.val + start + l, stream);
    }
    for (int32_t base = start; base < end; base += LPR) {
        const int n = min(LPR, end - base);
        const int my_c = nx_c;
        const float my_w = nx_w;
        if (base + LPR + l < end) {
            nx_c = ld_i32(a.ci + base + LPR + l, stream);
            if (a.val) nx_w = ld_f32(a.val + base + LPR + l, stream);
        }
        int e = 0;
        for (; e + U <= n; e += U) {
            int c[U];
            float w[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                c[u] = __shfl_sync(mask, my_c, e + u, LPR);
                w[u] = __shfl_sync(mask, my_w, e + u, LPR);
            }
            float h[U][SPL][VEC];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int s = 0; s < SPL; ++s)
                    if (live[s]) ldv<VEC>(a.B + static_cast<int64_t>(c[u]) * a.ldb + fo[s], h[u][s], keep);
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int s = 0; s < SPL; ++s)
                    if (live[s])
#pragma unroll
                        for (int k = 0; k < VEC; ++k)
                            acc[s][k] = reduce_step<OP>(acc[s][k], w[u], h[u][s][k], avx[s][k]);
        }
        for (; e < n; ++e) {
            const int c = __shfl_sync(mask, my_c, e, LPR);
            const float w = __shfl_sync(mask, my_w, e, LPR);
#pragma unroll
            for (int s = 0; s < SPL; ++s)
                if (live[s]) {
                    float h[VEC];
                    ldv<VEC>(a.B + static_cast<int64_t>(c) * a.ldb + fo[s], h, keep);
#pragma unroll
                    for (int k = 0; k < VEC; ++k) acc[s][k] = reduce_step<OP>(acc[s][k], w, h[k], avx[s][k]);
                }
        }
    }

    const int32_t deg = row_end - row_begin;  // the whole row, whichever segment this pass covered
#pragma unroll
    for (int s = 0; s < SPL; ++s)
        if (live[s]) finish_acc<OP, VEC, CVEC>(a, row, fo[s], full[s], deg, acc[s]);
}

}  // namespace gk
}  // namespace tg
