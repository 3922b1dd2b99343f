// ============================================================================
//  gather_heavy.cuh -- the row-gather kernel for long (hub) rows.
//
//  The sub-warp kernel keeps U gathered rows in flight per output row, so a
//  row's time grows as len * latency / U: on a power-law graph the longest
//  row becomes the critical path of the launch once the other rows are
//  spread over enough SMs (a 13.5k-entry row: ~2.4 ms at U = 4).  Here one
//  CTA streams long rows' gathered rows into a shared-memory ring of K
//  stages (G = 32 entries each; ~100 KB in flight instead of ~2 KB):
//
//    warps 0-1   producers.  The CTA's rows (slots b, b + gridDim.x, ... of
//                the schedule) sit in a row table in shared memory; the
//                producers walk them as ONE stream of chunks, loading the
//                (col, val) of the chunk kHeavyAhead chunks ahead -- across
//                row boundaries, so a new row starts without a latency
//                bubble (each producer warp keeps its own table and cursors:
//                the two warps meet only at the stage barriers).  Per chunk
//                each producer warp copies half of the
//                entries' rows (this pass's feature slice, <= 512 B) as
//                16-byte cp.async pieces, several entries per instruction
//                when rows are short, and arrives on full[k] when its pieces
//                land (cp.async.mbarrier.arrive.noinc); warp 0 also writes
//                the chunk's weights and a descriptor (row, count, first /
//                last, degree) and arrives normally to publish them.
//    warps 2-5   consumers: thread t owns feature f0 + t and applies the
//                chunk's entries in stored order -- the same per-element
//                fused multiply-add (or max) chain as the sub-warp kernel --
//                then releases the stage (empty[k]); a descriptor with count
//                < 0 ends the stream.
//
//  Measured before this shape: one producer warp issuing one bulk (TMA)
//  copy per gathered row, or all the 16-byte pieces itself, could not feed
//  the consumers (~63 SM cycles per entry at F = 128).
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
//  in the error word and sets the CTA's abort flag, which every role checks
//  per chunk; the producers then wait for their own copies (cp.async
//  completion) before the CTA returns.
//
//  Requirements (checked by the host): a row schedule, ldb % 4 == 0 and B
//  16-byte aligned (16-byte copy pieces), so the copied slice may run up to
//  the padded width pad4(F) <= ldb.
// ============================================================================
#pragma once

#include "gather_kernel.cuh"
#include "mbarrier.cuh"

namespace tg {
namespace gk {

constexpr int kHeavyG = 32;              // entries per stage
constexpr int kHeavyProducers = 2;       // producer warps
constexpr int kHeavyConsumers = 128;     // consumer threads = features per pass
constexpr int kHeavyThreads = 32 * kHeavyProducers + kHeavyConsumers;
constexpr int kHeavyAhead = 8;           // chunks of (col, val) the producers hold ahead
constexpr int kHeavyTable = 64;          // rows per row-table batch

struct HeavyDesc {
    int32_t row;
    int32_t n;       // entries in this chunk; < 0 ends the stream
    int32_t flags;   // 1 = first chunk of the row, 2 = last
    int32_t deg;     // the row's full length (mean, max of an empty row)
};

struct HeavyRow {
    int32_t row, start, len, deg, nch;
};

// Dynamic shared memory of the heavy kernel for K stages of `bpe` bytes per entry.
inline size_t heavy_smem_bytes(int K, int bpe) {
    return static_cast<size_t>(K) * (kHeavyG * (bpe + 4) + sizeof(HeavyDesc)) + static_cast<size_t>(2 * K) * 8 +
           kHeavyProducers * kHeavyTable * sizeof(HeavyRow) + 16;
}

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

template <int OP>
__global__ void __launch_bounds__(kHeavyThreads) gather_heavy_kernel(const GatherArgs a, int K, int bpe, int* err) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int bpf = bpe >> 2;  // floats per staged entry
    float* data = reinterpret_cast<float*>(smem);
    float* wbuf = data + static_cast<size_t>(K) * kHeavyG * bpf;
    HeavyDesc* desc = reinterpret_cast<HeavyDesc*>(wbuf + K * kHeavyG);
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(desc + K);
    uint64_t* empty_bar = full_bar + K;
    HeavyRow* tables = reinterpret_cast<HeavyRow*>(empty_bar + K);  // one per producer warp
    int* abort_flag = reinterpret_cast<int*>(tables + kHeavyProducers * kHeavyTable);
    volatile int* aborted = abort_flag;

    const int tid = threadIdx.x;
    constexpr int kProdThreads = 32 * kHeavyProducers;
    if (tid == 0) {
        for (int k = 0; k < K; ++k) {
            mb::init(&full_bar[k], kProdThreads + 1);  // copy-completion arrivals + warp 0's publish
            mb::init(&empty_bar[k], kHeavyConsumers / 32);
        }
        *abort_flag = 0;
        mb::fence_init();
    }
    __syncthreads();

    const int64_t f0 = static_cast<int64_t>(blockIdx.y) * kHeavyConsumers;  // feature pass
    const int64_t limit = *a.heavy_count;
    const uint64_t keep = policy_keep(), stream = policy_stream();
    int k = 0;          // ring stage of the next chunk
    uint32_t ph = 0;    // its use count's parity
    bool wrapped = false;  // every stage used at least once

    if (tid < kProdThreads) {
        // ── producers ──
        const int lane = tid & 31, pw = tid >> 5;
        HeavyRow* table = tables + pw * kHeavyTable;
        const float* src = a.B + f0;
        // Bytes copied per entry: this pass's slice, up to the padded width.
        const int64_t rest = ((a.F + 3) & ~static_cast<int64_t>(3)) - f0;
        const int cpy = static_cast<int>(rest < bpf ? rest : bpf) * 4;
        const int ppe = cpy >> 4;               // 16-byte pieces per entry (1..32)
        const int epi = 32 / ppe;               // entries per copy instruction
        const int sub = lane / ppe, q = lane % ppe;
        const bool copy_lane = sub < epi;
        constexpr int kHalf = kHeavyG / kHeavyProducers;
        const int e_lo = pw * kHalf;            // this warp's entries of a chunk
        bool ok = true;

        // Waits until stage k may be refilled and claims it; false on timeout or abort.
        auto claim = [&]() -> bool {
            bool w = true;
            if (lane == 0) {  // one lane decides for the warp
                if (wrapped) w = mb::wait(&empty_bar[k], ph ^ 1u, err, 11);
                w = w && !*aborted;
                if (!w) atomicExch(abort_flag, 1);
            }
            return __shfl_sync(0xffffffffu, w, 0);
        };
        auto publish = [&]() {
            mb::cp_async_arrive(&full_bar[k]);
            if (pw == 0) {
                __syncwarp();
                if (lane == 0) mb::arrive(&full_bar[k]);  // releases weights + descriptor
            }
            if (++k == K) {
                k = 0;
                ph ^= 1u;
                wrapped = true;
            }
        };

        for (int64_t tb = blockIdx.x; tb < limit && ok; tb += static_cast<int64_t>(kHeavyTable) * gridDim.x) {
            // Row table: up to kHeavyTable rows of this CTA.  Each producer
            // warp keeps its own copy, so the warps never wait on each other
            // except through the (bounded) stage barriers.
            for (int i = lane; i < kHeavyTable; i += 32) {
                const int64_t slot = tb + static_cast<int64_t>(i) * gridDim.x;
                if (slot < limit) {
                    const int32_t row = ld_i32(a.order + slot, stream);
                    const int32_t rb = ld_i32(a.rp + row, stream), re = ld_i32(a.rp + row + 1, stream);
                    const int32_t s = a.seg_lo ? ld_i32(a.seg_lo + row, stream) : rb;
                    const int32_t e = a.seg_hi ? ld_i32(a.seg_hi + row, stream) : re;
                    table[i] = HeavyRow{row, s, e - s, re - rb, e > s ? (e - s + kHeavyG - 1) / kHeavyG : 1};
                }
            }
            const int64_t left = (limit - tb + gridDim.x - 1) / gridDim.x;
            const int nrows = static_cast<int>(left < kHeavyTable ? left : kHeavyTable);
            __syncwarp();

            // Two cursors over the table's chunk stream: issue (ti, cj) and
            // prefetch (pti, pcj), kHeavyAhead chunks apart.
            int ti = 0, cj = 0, pti = 0, pcj = 0;
            // Raw loaded values only: nothing may consume a prefetched load
            // before its chunk is issued (an address formed here would stall
            // the warp for a full load latency per chunk).
            int colr[kHeavyAhead];
            float wv[kHeavyAhead];
            auto load_chunk = [&](int& c, float& w) {
                c = 0;
                w = 1.0f;
                if (pti < nrows) {
                    const HeavyRow r = table[pti];
                    const int64_t e = static_cast<int64_t>(r.start) + static_cast<int64_t>(pcj) * kHeavyG + lane;
                    if (e < static_cast<int64_t>(r.start) + r.len) {
                        c = ld_i32(a.ci + e, stream);
                        if (a.val) w = ld_f32(a.val + e, stream);
                    }
                    if (++pcj >= r.nch) {
                        ++pti;
                        pcj = 0;
                    }
                }
            };
#pragma unroll
            for (int p = 0; p < kHeavyAhead; ++p) load_chunk(colr[p], wv[p]);
            while (ti < nrows && ok) {
#pragma unroll
                for (int p = 0; p < kHeavyAhead; ++p) {
                    if (ti < nrows && ok) {
                        ok = claim();
                        if (ok) {
                            const HeavyRow r = table[ti];
                            const int done = cj * kHeavyG;
                            const int n = r.len - done < kHeavyG ? (r.len - done > 0 ? r.len - done : 0) : kHeavyG;
                            if (pw == 0) {
                                wbuf[k * kHeavyG + lane] = wv[p];
                                if (lane == 0)
                                    desc[k] = HeavyDesc{r.row, n, (cj == 0 ? 1 : 0) | (cj == r.nch - 1 ? 2 : 0), r.deg};
                            }
                            float* stage = data + static_cast<size_t>(k) * kHeavyG * bpf;
                            const int e_hi = n < e_lo + kHalf ? n : e_lo + kHalf;
                            for (int e0 = e_lo; e0 < e_hi; e0 += epi) {  // uniform trip count per warp
                                const int ent = e0 + sub;
                                const int col = __shfl_sync(0xffffffffu, colr[p], ent < 32 ? ent : 31);
                                if (copy_lane && ent < e_hi)
                                    mb::cp_async16(stage + static_cast<size_t>(ent) * bpf + q * 4,
                                                   src + static_cast<int64_t>(col) * a.ldb + q * 4, keep);
                            }
                            publish();
                            if (++cj >= r.nch) {
                                ++ti;
                                cj = 0;
                            }
                            load_chunk(colr[p], wv[p]);
                        }
                    }
                }
            }
            __syncwarp();  // the table is rewritten next batch
        }
        // End of stream.  After an abort the consumers stop on the flag.
        if (ok && claim()) {
            if (pw == 0 && lane == 0) desc[k] = HeavyDesc{0, -1, 0, 0};
            publish();
        }
        // Every copy this thread issued has landed before the CTA may leave.
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
        // ── consumers ──
        const int t = tid - kProdThreads;
        const int lane = t & 31;
        const int64_t fo = f0 + t;
        const bool live = fo < a.F;
        const bool avx = fo < a.max_avx_cols;
        const float init = (OP == GATHER_SUM) ? 0.0f : -INFINITY;
        float acc[1] = {init};
        for (;;) {
            // Every lane waits (acquire); the warp leaves together if any ran
            // out or the CTA aborted.
            const bool w = mb::wait(&full_bar[k], ph, err, 12);
            if (!__all_sync(0xffffffffu, w && !*aborted)) {
                if (lane == 0) atomicExch(abort_flag, 1);
                break;
            }
            const HeavyDesc d = desc[k];
            if (d.n < 0) break;
            if (d.flags & 1) start_acc<1, true>(a, d.row, fo, live, live, init, acc);
            if (live) {
                const float* st = data + static_cast<size_t>(k) * kHeavyG * bpf + t;
                const float* ws = wbuf + k * kHeavyG;
                int i = 0;
                for (; i + 8 <= d.n; i += 8) {
                    float h[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) h[u] = st[static_cast<size_t>(i + u) * bpf];
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[0] = reduce_step<OP>(acc[0], ws[i + u], h[u], avx);
                }
                for (; i < d.n; ++i) acc[0] = reduce_step<OP>(acc[0], ws[i], st[static_cast<size_t>(i) * bpf], avx);
            }
            __syncwarp();
            if (lane == 0) mb::arrive(&empty_bar[k]);
            if (++k == K) {
                k = 0;
                ph ^= 1u;
            }
            if ((d.flags & 2) && live) finish_acc<OP, 1, true>(a, d.row, fo, true, d.deg, acc);
        }
    }
    __syncthreads();
}

}  // namespace gk
}  // namespace tg
