// ============================================================================
//  gather_heavy.cuh -- the row-gather kernel for long (hub) rows.
//
//  The sub-warp kernel keeps U gathered rows in flight per output row, so a
//  row's time grows as len * latency / U: on a power-law graph the longest
//  row becomes the critical path of the launch once the other rows are
//  spread over enough SMs (a 13.5k-entry row: ~2.4 ms at U = 4).  Here one
//  CTA streams a long row's gathered rows into a shared-memory ring with
//  bulk async copies (~100 KB in flight instead of ~2 KB):
//
//    warp 0      producer: reads the row's (col, val) entries kHeavyAhead
//                chunks ahead, then per chunk of G entries one cp.async.bulk per
//                entry (the feature slice of B's row, 16-byte multiple) into
//                stage k of K, completion counted on full[k];
//    warps 1-4   consumers: thread t owns features f0 + t*VEC .. +VEC and
//                applies the chunk's entries in stored order -- the same
//                per-element fused multiply-add (or max) chain as the
//                sub-warp kernel -- then releases the stage (empty[k]).
//
//  Which rows: heavy_prefix_kernel (below) picks the threshold on the device
//  from the launch's nnz -- a row is heavy when its serial chain would rival
//  the whole launch: len >= max(1023, 2^ceil(log2(nnz / 16384)) - 1) -- and
//  counts the leading slots of the schedule whose rows reach it (with the
//  degree order, whose buckets are powers of two, exactly the heavy rows).
//  This kernel takes slots [0, h) and the sub-warp kernel skips them.
//
//  The kernel is persistent: CTA b takes slots b, b + gridDim.x, ... < h.
//  The stage counter runs on across rows, so the barriers are initialised
//  once.  Carry-in, epilogue and stores are the sub-warp kernel's own
//  functions: results are bit-identical whichever kernel produced a row.
//
//  Every wait is bounded (mbarrier.cuh); after a timeout the CTA records a
//  code in the error word, stops issuing, waits (bounded) for the copies it
//  issued and returns.
//
//  Requirements (checked by the host): a row schedule, ldb % 4 == 0 and B
//  16-byte aligned (bulk-copy source rows), so the copied slice may run up
//  to the padded width pad4(F) <= ldb.
// ============================================================================
#pragma once

#include "gather_kernel.cuh"
#include "mbarrier.cuh"

namespace tg {
namespace gk {

constexpr int kHeavyG = 32;              // entries per stage (one per producer lane)
constexpr int kHeavyConsumers = 128;     // consumer threads
constexpr int kHeavyThreads = 32 + kHeavyConsumers;
constexpr int kHeavyAhead = 8;           // chunks of (col, val) the producer holds ahead

// Dynamic shared memory of the heavy kernel for K stages of `bpe` bytes per entry.
inline size_t heavy_smem_bytes(int K, int bpe) {
    return static_cast<size_t>(K) * kHeavyG * (bpe + 4) + static_cast<size_t>(2 * K) * 8 + 16;
}

template <int V>
__device__ __forceinline__ void ldv_shared(const float* p, float (&x)[V]) {
    if constexpr (V == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else if constexpr (V == 2) {
        const float2 t = *reinterpret_cast<const float2*>(p);
        x[0] = t.x; x[1] = t.y;
    } else {
        x[0] = p[0];
    }
}

constexpr int kHeavyScanThreads = 1024;
constexpr int32_t kHeavyFloor = 1023;     // shortest heavy row
constexpr int64_t kHeavyRatio = 16384;    // ... and at least nnz / kHeavyRatio (rounded to 2^k - 1)

// *count = the number of leading slots of `order` (at most `scan`) whose rows
// have at least T entries; T = min_len if >= 0, else chosen from the nnz.
__global__ void __launch_bounds__(kHeavyScanThreads)
heavy_prefix_kernel(int64_t M, const int32_t* rp, const int32_t* order, int64_t scan, int32_t min_len,
                    int32_t* count) {
    __shared__ int64_t first;
    int32_t T = min_len;
    if (T < 0) {
        const int64_t target = (static_cast<int64_t>(rp[M]) - rp[0]) / kHeavyRatio;
        int64_t p = 1;
        while (p < target) p <<= 1;
        T = static_cast<int32_t>(p - 1 > kHeavyFloor ? p - 1 : kHeavyFloor);
    }
    if (threadIdx.x == 0) first = scan;
    __syncthreads();
    for (int64_t base = 0; base < scan; base += kHeavyScanThreads) {
        const int64_t i = base + threadIdx.x;
        if (i < scan) {
            const int64_t r = order[i];
            if (rp[r + 1] - rp[r] < T) atomicMin(reinterpret_cast<unsigned long long*>(&first),
                                                 static_cast<unsigned long long>(i));
        }
        __syncthreads();
        if (first < scan) break;  // uniform: read after the barrier
        __syncthreads();
    }
    if (threadIdx.x == 0) *count = static_cast<int32_t>(first);
}

template <int VEC, int OP, bool CVEC>
__global__ void __launch_bounds__(kHeavyThreads) gather_heavy_kernel(const GatherArgs a, int K, int bpe, int* err) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int bpf = bpe >> 2;  // floats per staged entry
    float* data = reinterpret_cast<float*>(smem);
    float* wbuf = data + static_cast<size_t>(K) * kHeavyG * bpf;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(wbuf + K * kHeavyG);
    uint64_t* empty_bar = full_bar + K;
    int* abort_flag = reinterpret_cast<int*>(empty_bar + K);

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int k = 0; k < K; ++k) {
            mb::init(&full_bar[k], 1);
            mb::init(&empty_bar[k], kHeavyConsumers / 32);
        }
        *abort_flag = 0;
        mb::fence_init();
    }
    __syncthreads();

    const int64_t f0 = static_cast<int64_t>(blockIdx.y) * (kHeavyConsumers * VEC);  // feature pass
    const int64_t limit = *a.heavy_count;
    const uint64_t keep = policy_keep(), stream = policy_stream();
    int64_t g = 0;  // stages used so far by this CTA (same count in every role)

    if (tid < 32) {
        // ── producer ──
        const int lane = tid;
        const float* src = a.B + f0;
        // Bytes copied per entry: this pass's slice, up to the padded width.
        const int64_t rest = ((a.F + 3) & ~static_cast<int64_t>(3)) - f0;
        const int cpy = static_cast<int>(rest < bpf ? rest : bpf) * 4;
        bool ok = true;
        for (int64_t slot = blockIdx.x; slot < limit && ok; slot += gridDim.x) {
            const int64_t row = ld_i32(a.order + slot, stream);
            const int32_t rb = ld_i32(a.rp + row, stream), re = ld_i32(a.rp + row + 1, stream);
            const int32_t start = a.seg_lo ? ld_i32(a.seg_lo + row, stream) : rb;
            const int32_t end = a.seg_hi ? ld_i32(a.seg_hi + row, stream) : re;
            const int32_t len = end - start;
            const int64_t nch = len > 0 ? (len + kHeavyG - 1) / kHeavyG : 1;
            int col[kHeavyAhead];
            float wv[kHeavyAhead];
#pragma unroll
            for (int p = 0; p < kHeavyAhead; ++p) {
                const int64_t e = static_cast<int64_t>(start) + p * kHeavyG + lane;
                col[p] = e < end ? ld_i32(a.ci + e, stream) : 0;
                wv[p] = (e < end && a.val) ? ld_f32(a.val + e, stream) : 1.0f;
            }
            for (int64_t c0 = 0; c0 < nch && ok; c0 += kHeavyAhead) {
#pragma unroll
                for (int p = 0; p < kHeavyAhead; ++p) {
                    const int64_t c = c0 + p;
                    if (c < nch && ok) {
                        const int k = static_cast<int>(g % K);
                        if (g >= K) {  // wait until the consumers released this stage's previous use
                            bool w = true;
                            if (lane == 0) w = mb::wait(&empty_bar[k], static_cast<uint32_t>((g / K - 1) & 1), err, 11);
                            ok = __shfl_sync(0xffffffffu, w, 0);
                        }
                        if (ok) {
                            const int64_t left = static_cast<int64_t>(len) - c * kHeavyG;
                            const int n = left <= 0 ? 0 : (left < kHeavyG ? static_cast<int>(left) : kHeavyG);
                            wbuf[k * kHeavyG + lane] = wv[p];
                            __syncwarp();
                            if (lane == 0) mb::arrive_expect_tx(&full_bar[k], static_cast<uint32_t>(n * cpy));
                            __syncwarp();
                            if (lane < n)
                                mb::bulk_load(data + (static_cast<size_t>(k) * kHeavyG + lane) * bpf,
                                              src + static_cast<int64_t>(col[p]) * a.ldb, static_cast<uint32_t>(cpy),
                                              &full_bar[k], keep);
                            ++g;
                            const int64_t e = static_cast<int64_t>(start) + (c + kHeavyAhead) * kHeavyG + lane;
                            col[p] = e < end ? ld_i32(a.ci + e, stream) : 0;
                            wv[p] = (e < end && a.val) ? ld_f32(a.val + e, stream) : 1.0f;
                        }
                    }
                }
            }
            if (!ok && lane == 0) atomicExch(abort_flag, 1);
        }
    } else {
        // ── consumers ──
        const int t = tid - 32;
        const int lane = t & 31;
        const int64_t fo = f0 + static_cast<int64_t>(t) * VEC;
        const bool live = fo < a.F;
        const bool fullv = fo + VEC <= a.F;
        bool avx[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) avx[k] = (fo + k) < a.max_avx_cols;
        const float init = (OP == GATHER_SUM) ? 0.0f : -INFINITY;
        bool ok = true;
        for (int64_t slot = blockIdx.x; slot < limit && ok; slot += gridDim.x) {
            const int64_t row = ld_i32(a.order + slot, stream);
            const int32_t rb = ld_i32(a.rp + row, stream), re = ld_i32(a.rp + row + 1, stream);
            const int32_t start = a.seg_lo ? ld_i32(a.seg_lo + row, stream) : rb;
            const int32_t end = a.seg_hi ? ld_i32(a.seg_hi + row, stream) : re;
            const int32_t len = end - start;
            const int64_t nch = len > 0 ? (len + kHeavyG - 1) / kHeavyG : 1;
            float acc[VEC];
            start_acc<VEC, CVEC>(a, row, fo, live, fullv, init, acc);
            for (int64_t c = 0; c < nch; ++c) {
                const int k = static_cast<int>(g % K);
                // Every lane waits (acquire); the warp leaves together if any ran out.
                const bool w = mb::wait(&full_bar[k], static_cast<uint32_t>((g / K) & 1), err, 12);
                if (!__all_sync(0xffffffffu, w)) {
                    ok = false;
                    break;
                }
                const int64_t left = static_cast<int64_t>(len) - c * kHeavyG;
                const int n = left <= 0 ? 0 : (left < kHeavyG ? static_cast<int>(left) : kHeavyG);
                if (live) {
                    const float* st = data + static_cast<size_t>(k) * kHeavyG * bpf + static_cast<int64_t>(t) * VEC;
                    const float* ws = wbuf + k * kHeavyG;
                    int i = 0;
                    for (; i + 4 <= n; i += 4) {
                        float h[4][VEC];
#pragma unroll
                        for (int u = 0; u < 4; ++u) ldv_shared<VEC>(st + static_cast<size_t>(i + u) * bpf, h[u]);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float w = ws[i + u];
#pragma unroll
                            for (int q = 0; q < VEC; ++q) acc[q] = reduce_step<OP>(acc[q], w, h[u][q], avx[q]);
                        }
                    }
                    for (; i < n; ++i) {
                        float h[VEC];
                        ldv_shared<VEC>(st + static_cast<size_t>(i) * bpf, h);
                        const float w = ws[i];
#pragma unroll
                        for (int q = 0; q < VEC; ++q) acc[q] = reduce_step<OP>(acc[q], w, h[q], avx[q]);
                    }
                }
                ++g;
                __syncwarp();
                if (lane == 0) mb::arrive(&empty_bar[k]);
            }
            if (!ok) {
                atomicExch(abort_flag, 1);
                break;
            }
            if (live) finish_acc<OP, VEC, CVEC>(a, row, fo, fullv, re - rb, acc);
        }
    }
    __syncthreads();
    // Before the CTA leaves, every copy it issued must have landed: without a
    // timeout the consumers waited for all of them; after one, the producer
    // (thread 0, whose g counts the issued stages) waits for the last K.
    if (tid == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
        for (int64_t q = (g > K ? g - K : 0); q < g; ++q)
            mb::wait(&full_bar[q % K], static_cast<uint32_t>((q / K) & 1), err, 13);
    }
}

}  // namespace gk
}  // namespace tg
