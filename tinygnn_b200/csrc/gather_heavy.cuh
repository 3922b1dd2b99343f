// ============================================================================
//  gather_heavy.cuh -- the row-gather kernel for long (hub) rows.
//
//  The sub-warp kernel keeps U gathered rows in flight per output row, so a
//  row's time grows as len * latency / U: on a power-law graph the longest
//  row becomes the critical path of the launch once the other rows are
//  spread over enough SMs (a 13.5k-entry row: ~1.4 ms at U = 4).  Each
//  element's sum must stay ONE sequential chain (bit-exact results), so the
//  row cannot be split by entries; this kernel splits it by features and
//  feeds each chain from a deep shared-memory pipeline instead:
//
//    * one CTA per (row group, 32-feature slice): a hub row at F = 128 is
//      served by 4 CTAs, each moving 128 B per gathered row;
//    * 8 loader warps fill a ring of kHeavyStages stages of G = 32 entries;
//      warp w fills chunks w, w + 8, ... of the CTA's chunk stream (its
//      rows, one after another) -- and so always stages w and w + 8: column
//      ids with plain loads (the next chunk's are loaded while the current
//      one is issued), the gathered rows as 16-byte cp.async pieces (4 rows
//      per instruction), the weights as 4-byte cp.async, and a descriptor
//      (row, count, first / last, degree); the stage completes when the
//      copies land (cp.async.mbarrier.arrive.noinc per lane + lane 0's
//      arrival);
//    * one consumer warp (lane t = feature f0 + t) applies the chunks in
//      stored order -- the same per-element fused multiply-add (or max)
//      chain as the sub-warp kernel -- and releases each stage.
//
//  Why this shape (measured on one 13.5k-entry row, F = 128): a warp keeps
//  only a few memory instructions in flight, and one bulk (TMA) copy per
//  gathered row costs ~40 ns of the SM's copy engine whatever its size, so
//  one or two producer warps per row -- with bulk copies, cp.async groups
//  or register prefetch -- all stalled at 40-50 ns per entry, whatever the
//  stage count.  Many loader warps per CTA and several CTAs per row lift
//  that bound.
//
//  Which rows: heavy_prefix_kernel (below) picks the threshold on the device
//  from the launch's nnz -- a row is heavy when its serial chain would rival
//  the whole launch: len >= max(1023, 2^ceil(log2(nnz / 16384)) - 1) -- and
//  counts the leading slots of the schedule whose rows reach it (with the
//  degree order, whose buckets are powers of two, exactly the heavy rows).
//  This kernel takes slots [0, h) and the sub-warp kernel skips them.
//  Carry-in, epilogue and stores are the sub-warp kernel's own functions:
//  results are bit-identical whichever kernel produced a row.
//
//  Every mbarrier wait is bounded (mbarrier.cuh).  A timeout records a code
//  in the error word and sets the CTA's abort flag; every role checks it per
//  chunk and leaves at the next batch barrier, and each loader thread waits
//  for its own copies (cp.async.wait_all) before the CTA returns.
//
//  Requirements (checked by the host): a row schedule, ldb % 4 == 0 and B
//  16-byte aligned (16-byte copy pieces), so a slice's copy may run up to
//  the padded width pad4(F) <= ldb.
// ============================================================================
#pragma once

#include "gather_kernel.cuh"
#include "mbarrier.cuh"

namespace tg {
namespace gk {

constexpr int kHeavyG = 32;              // entries per chunk (stage)
constexpr int kHeavySlice = 32;          // features per CTA (one consumer warp)
constexpr int kHeavyLoaders = 8;         // loader warps
constexpr int kHeavyThreads = 32 * (kHeavyLoaders + 1);
constexpr int kHeavyStages = 2 * kHeavyLoaders;  // warp w fills stages w and w + kHeavyLoaders
constexpr int kHeavyTable = 64;          // rows per batch
constexpr int kHeavyCtasPerSm = 3;

struct HeavyDesc {
    int32_t row;
    int32_t n;       // entries in this chunk
    int32_t flags;   // 1 = first chunk of the row, 2 = last
    int32_t deg;     // the row's full length (mean, max of an empty row)
};

struct HeavyRow {
    int32_t row, start, len, deg, nch;
};

struct HeavySmem {
    float data[kHeavyStages][kHeavyG][kHeavySlice];
    float w[kHeavyStages][kHeavyG];
    HeavyDesc desc[kHeavyStages];
    uint64_t full[kHeavyStages], empty[kHeavyStages];
    HeavyRow table[kHeavyTable];
    int32_t chunk0[kHeavyTable + 1];     // first chunk of each table row (prefix sums)
    int abort_flag;
};

constexpr int kHeavyScanThreads = 1024;
constexpr int32_t kHeavyFloor = 1023;     // shortest heavy row
constexpr int64_t kHeavyRatio = 16384;    // ... and at least nnz / kHeavyRatio (rounded to 2^k - 1)

// *count = the number of leading slots of `order` (at most `scan`) whose rows
// have at least T entries; T = min_len if >= 0, else chosen from the nnz.
__global__ void __launch_bounds__(kHeavyScanThreads)
heavy_prefix_kernel(int64_t M, const int32_t* rp, const int32_t* order, int64_t scan, int32_t min_len,
                    int32_t* count) {
    __shared__ unsigned long long first;
    int32_t T = min_len;
    if (T < 0) {
        const int64_t target = (static_cast<int64_t>(rp[M]) - rp[0]) / kHeavyRatio;
        int64_t p = 1;
        while (p < target) p <<= 1;
        T = static_cast<int32_t>(p - 1 > kHeavyFloor ? p - 1 : kHeavyFloor);
    }
    if (threadIdx.x == 0) first = static_cast<unsigned long long>(scan);
    __syncthreads();
    for (int64_t base = 0; base < scan; base += kHeavyScanThreads) {
        const int64_t i = base + threadIdx.x;
        if (i < scan) {
            const int64_t r = order[i];
            if (rp[r + 1] - rp[r] < T) atomicMin(&first, static_cast<unsigned long long>(i));
        }
        __syncthreads();
        const bool done = first < static_cast<unsigned long long>(scan);  // uniform: read after the barrier
        __syncthreads();
        if (done) break;
    }
    if (threadIdx.x == 0) *count = static_cast<int32_t>(first);
}

// Grid: passes * groups CTAs; CTA b serves feature pass b % passes and the
// slots g, g + groups, ... of row group g = b / passes.
template <int OP>
__global__ void __launch_bounds__(kHeavyThreads) gather_heavy_kernel(const GatherArgs a, int passes, int* err) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    HeavySmem& S = *reinterpret_cast<HeavySmem*>(smem_raw);
    volatile int* aborted = &S.abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int k = 0; k < kHeavyStages; ++k) {
            mb::init(&S.full[k], 33);  // the filling warp's 32 copy-completion arrivals + its lane 0
            mb::init(&S.empty[k], 1);  // the consumer warp's lane 0
        }
        S.abort_flag = 0;
        mb::fence_init();
    }
    __syncthreads();

    const int pass = static_cast<int>(blockIdx.x % passes);
    const int64_t group = blockIdx.x / passes, groups = gridDim.x / passes;
    const int64_t f0 = static_cast<int64_t>(pass) * kHeavySlice;
    const int64_t limit = *a.heavy_count;
    const uint64_t keep = policy_keep(), stream = policy_stream();
    // 16-byte pieces copied per gathered row: this slice, up to the padded width.
    const int64_t rest = ((a.F + 3) & ~static_cast<int64_t>(3)) - f0;
    const int ppe = static_cast<int>(rest < kHeavySlice ? rest : kHeavySlice) >> 2;  // 1..8
    const int epi = 32 / ppe;  // rows per copy instruction (4..32)

    const bool consumer = warp == kHeavyLoaders;
    const int64_t fo = f0 + lane;  // consumer: this lane's feature
    const bool live = fo < a.F;
    const bool avx = fo < a.max_avx_cols;
    const float init = (OP == GATHER_SUM) ? 0.0f : -INFINITY;
    float acc[1] = {init};
    int32_t gbase = 0;  // stages used by earlier batches

    for (int64_t tb = group; tb < limit; tb += static_cast<int64_t>(kHeavyTable) * groups) {
        // Row table of this batch (threads 0..63), then chunk prefix sums.
        const int64_t left = (limit - tb + groups - 1) / groups;
        const int nrows = static_cast<int>(left < kHeavyTable ? left : kHeavyTable);
        if (tid < nrows) {
            const int32_t row = ld_i32(a.order + tb + static_cast<int64_t>(tid) * groups, stream);
            const int32_t rb = ld_i32(a.rp + row, stream), re = ld_i32(a.rp + row + 1, stream);
            const int32_t s = a.seg_lo ? max(rb, ld_i32(a.seg_lo + row, stream)) : rb;  // inside the row
            const int32_t e = a.seg_hi ? min(re, ld_i32(a.seg_hi + row, stream)) : re;
            S.table[tid] = HeavyRow{row, s, e - s, re - rb, e > s ? (e - s + kHeavyG - 1) / kHeavyG : 1};
        }
        __syncthreads();
        if (tid == 0) {
            int32_t c = 0;
            for (int i = 0; i < nrows; ++i) {
                S.chunk0[i] = c;
                c += S.table[i].nch;
            }
            S.chunk0[nrows] = c;
        }
        __syncthreads();
        const int32_t total = S.chunk0[nrows];

        if (!consumer) {
            // ── loader warp: chunks warp, warp + kHeavyLoaders, ... ──
            int ti = 0;
            int32_t c = warp;
            while (ti < nrows && S.chunk0[ti + 1] <= c) ++ti;
            auto ids_of = [&](int t, int32_t cc) -> int {  // this lane's column id of chunk cc (row t)
                if (t >= nrows) return 0;
                const HeavyRow r = S.table[t];
                const int64_t e =
                    static_cast<int64_t>(r.start) + static_cast<int64_t>(cc - S.chunk0[t]) * kHeavyG + lane;
                return e < static_cast<int64_t>(r.start) + r.len ? ld_i32(a.ci + e, stream) : 0;
            };
            int col = ids_of(ti, c);
            for (; c < total; c += kHeavyLoaders) {
                const int32_t g = gbase + c;
                const int k = g % kHeavyStages;
                bool ok = true;
                if (lane == 0) {  // one lane decides for the warp
                    if (g >= kHeavyStages)
                        ok = mb::wait_sleepy(&S.empty[k], static_cast<uint32_t>((g / kHeavyStages - 1) & 1), err, 11,
                                             200);  // the consumer warp is the critical path: poll gently
                    ok = ok && !*aborted;
                    if (!ok) atomicExch(&S.abort_flag, 1);
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) break;
                const HeavyRow r = S.table[ti];
                const int cj = c - S.chunk0[ti];
                const int done = cj * kHeavyG;
                const int n = r.len - done < kHeavyG ? (r.len - done > 0 ? r.len - done : 0) : kHeavyG;
                if (lane < n) {
                    if (a.val) mb::cp_async4(&S.w[k][lane], a.val + r.start + done + lane, stream);
                    else S.w[k][lane] = 1.0f;
                }
                if (lane == 0) S.desc[k] = HeavyDesc{r.row, n, (cj == 0 ? 1 : 0) | (cj == r.nch - 1 ? 2 : 0), r.deg};
                const float* src = a.B + f0 + (lane % ppe) * 4;
                for (int e0 = 0; e0 < n; e0 += epi) {
                    const int ent = e0 + lane / ppe;
                    const int cc = __shfl_sync(0xffffffffu, col, ent < 32 ? ent : 31);
                    if (lane / ppe < epi && ent < n)
                        mb::cp_async16(&S.data[k][ent][(lane % ppe) * 4], src + static_cast<int64_t>(cc) * a.ldb,
                                       keep);
                }
                mb::cp_async_arrive(&S.full[k]);
                __syncwarp();
                if (lane == 0) mb::arrive(&S.full[k]);  // publishes stored weights + descriptor
                // The next chunk of this warp, and its column ids.
                const int32_t cn = c + kHeavyLoaders;
                while (ti < nrows && S.chunk0[ti + 1] <= cn) ++ti;
                col = ids_of(ti, cn);
            }
        } else {
            // ── consumer warp ──
            for (int32_t c = 0; c < total; ++c) {
                const int32_t g = gbase + c;
                const int k = g % kHeavyStages;
                // (A loader that gave up publishes nothing more: this wait then
                // runs out too, so the abort flag is not polled per chunk.)
                const bool w = mb::wait(&S.full[k], static_cast<uint32_t>((g / kHeavyStages) & 1), err, 12);
                if (!__all_sync(0xffffffffu, w)) {
                    if (lane == 0) atomicExch(&S.abort_flag, 1);
                    break;
                }
                const HeavyDesc d = S.desc[k];
                if (d.flags & 1) start_acc<1, true>(a, d.row, fo, live, live, init, acc);
                if (live) {
                    const float* st = &S.data[k][0][lane];
                    const float* ws = S.w[k];
                    if (d.n == kHeavyG) {
                        // A full chunk: every load first (one shared-memory latency
                        // per chunk, not per 8 entries), then the chain.
                        float h[kHeavyG], wv[kHeavyG];
#pragma unroll
                        for (int u = 0; u < kHeavyG; ++u) h[u] = st[u * kHeavySlice];
#pragma unroll
                        for (int u = 0; u < kHeavyG; u += 4) {
                            const float4 t = *reinterpret_cast<const float4*>(ws + u);
                            wv[u] = t.x;
                            wv[u + 1] = t.y;
                            wv[u + 2] = t.z;
                            wv[u + 3] = t.w;
                        }
#pragma unroll
                        for (int u = 0; u < kHeavyG; ++u) acc[0] = reduce_step<OP>(acc[0], wv[u], h[u], avx);
                    } else {
                        for (int i = 0; i < d.n; ++i) acc[0] = reduce_step<OP>(acc[0], ws[i], st[i * kHeavySlice], avx);
                    }
                }
                __syncwarp();
                if (lane == 0) mb::arrive(&S.empty[k]);
                if ((d.flags & 2) && live) finish_acc<OP, 1, true>(a, d.row, fo, true, d.deg, acc);
            }
        }
        gbase += total;
        __syncthreads();  // the table is rewritten next batch; every role leaves together on abort
        if (*aborted) break;
    }
    // Every copy a loader thread issued has landed before the CTA may leave.
    if (!consumer) asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
}

}  // namespace gk
}  // namespace tg
