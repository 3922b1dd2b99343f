// ============================================================================
//  gemm_tc.cu -- C = A . B on the 5th-generation tensor cores (FAST mode).
//
//  fp32 inputs through tcgen05.mma kind::tf32 with the 3xTF32 split:
//      A = Ah + Al,  Ah = round-to-nearest tf32(A),  Al = A - Ah (exact)
//      A.B ~= Ah.Bh + Ah.Bl + Al.Bh      (fp32 accumulation in TMEM)
//  which keeps the product within ~3e-6 relative of fp32 -- inside the
//  1e-5 + 1e-4|ref| tolerance -- at tensor-core rate.  (Plain TF32 would
//  miss it: a 10-bit mantissa over K = 602.)
//
//  One CTA owns a 128-row tile of C and all of its N (<= 256) columns:
//    warp 0      TMA producer: A tile (128 x 32 fp32, 128B swizzle) and the
//                pre-split B^T hi/lo tiles per k-block, into a 3-stage ring;
//    warp 1      allocates TMEM and issues the MMAs (one thread);
//    warps 2-5   split each A tile into Ah (in place) / Al in shared memory,
//                then run the epilogue: TMEM -> registers, + bias,
//                activation, store.
//  The persistent form (gemm_tcp_kernel, further down) walks several tiles
//  per CTA with two TMEM accumulators, so a tile's epilogue -- including its
//  stores to peer GPUs' copies -- overlaps the next tile's main loop; it is
//  chosen for long K with 16-byte-aligned outputs (use_persistent).
//  Nothing is written past an output's N columns unless the caller declares
//  row padding writable (a TMA store writes whole 16-byte pieces of a row).
//  Every mbarrier wait is bounded; a wait that runs out records a code in
//  a device error word, the CTA drains its copies, frees TMEM and returns.
//  A is read once from HBM (the tile's B^T comes from L2): the kernel is
//  bound by max(A bytes / HBM BW, 3 * 2MNK / tf32 peak).
//
//  Requirements (else the caller uses the exact SIMT kernel): lda % 4 == 0
//  and A 16-byte aligned (TMA row stride), N <= 256.
// ============================================================================
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "launch.cuh"
#include "mbarrier.cuh"

namespace tg {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;       // fp32 per 128-byte swizzled row

// Pipeline depth from the per-stage footprint (A, Al, Bh, Bl) within ~200 KB.
constexpr int stages_for(int BN) {
    return (200 * 1024) / ((2 * BM * BK + 2 * BN * BK) * 4) > 4 ? 4 : (200 * 1024) / ((2 * BM * BK + 2 * BN * BK) * 4);
}

__device__ int g_tc_error = 0;  // first timeout code seen (0 = none)

using mb::smem_u32;

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) { mb::init(bar, count); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) { mb::arrive_expect_tx(bar, bytes); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) { mb::arrive(bar); }

// Bounded wait; false (and the error word set) when it runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
    return mb::wait(bar, parity, &g_tc_error, code);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    const uint32_t a = smem_u32(p);
    uint64_t d = 0;
    d |= static_cast<uint64_t>((a >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(1) << 16;              // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;      // SBO
    d |= static_cast<uint64_t>(1) << 46;              // version
    d |= static_cast<uint64_t>(2) << 61;              // SWIZZLE_128B
    return d;
}

// Shared -> global tensor store of one box (async proxy; the issuing thread
// commits and waits for it before the CTA may exit).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ float tf32_rn(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

template <int BN, int STAGES_>
struct TcSmem {
    static constexpr int STAGES = STAGES_;
    float A[STAGES][BM * BK];     // raw tile, split in place into Ah
    float Al[STAGES][BM * BK];
    float Bh[STAGES][BN * BK];
    float Bl[STAGES][BN * BK];
    uint64_t full[STAGES], split[STAGES], empty[STAGES], acc, drain;
    uint32_t tmem;
};

struct TcArgs {
    float* C;
    int64_t ldc, M, N, K;
    const float* bias;
    int act;
    float alpha;
    int64_t ncols;  // columns stored: N, or round_up(N, 4) when the rows are padded (vec)
    int vec;        // 16-byte stores allowed (ldc % 4 == 0, outputs 16-byte aligned, ncols % 4 == 0)
    const float* rs;  // nullable: row i of the product scaled by rs[i] before the bias (one rounding)
    // Column split (local epilogue only): columns [nsplit, N) go to C2 at
    // column - nsplit (ld ldc2); nsplit == N: everything to C.
    float* C2;
    int64_t ldc2, nsplit;
    // Concat along K: k-blocks [0, kb1) come from tmA, the rest from tmA2
    // (A = [A1 | A2], B = [B1; B2] with B1 zero-padded to kb1 * BK rows).
    int kb1;
    // The epilogue stores through tmC / tmC2 (TMA, 32 x 32 boxes, 128-byte
    // swizzle): C rows 16-byte aligned, and nsplit a multiple of 32.
    int tma_store;
    // Column split with a gap: product columns [gap_lo, nsplit) are zero
    // padding stored nowhere (C holds gap_lo columns); 0 = no gap.
    int64_t gap_lo = 0;
    // The caller's rows have room up to round_up(width, 4) columns of each
    // output, which the epilogue may write (the epilogue of a zero product).
    int pad_ok = 0;
};

// PEERS: the epilogue also stores to peer copies (and may use 16-byte
// stores); false compiles the lean local-only epilogue.
template <int BN, int STAGES_, bool PEERS>
__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmA2,
                                                         const __grid_constant__ CUtensorMap tmBh,
                                                         const __grid_constant__ CUtensorMap tmBl,
                                                         const __grid_constant__ CUtensorMap tmC,
                                                         const __grid_constant__ CUtensorMap tmC2,
                                                         const TcArgs g,
                                                         const __grid_constant__ PeerOut peers) {
    extern __shared__ uint8_t raw[];
    using Smem = TcSmem<BN, STAGES_>;
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    constexpr int STAGES = STAGES_;
    constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
    constexpr uint32_t STAGE_BYTES = (BM * BK + 2 * BN * BK) * 4;
    // tf32 x tf32 -> f32, K-major A and B, M = 128, N = BN.
    constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * BM;
    const int KB = static_cast<int>((g.K + BK - 1) / BK);  // g.K = kb1 * BK + K2 when concatenated

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.split[i], 128);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.acc, 1);
        mbar_init(&s.drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;

    if (warp == 0) {
        // ── TMA producer ──
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int st = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (kb >= STAGES && !mbar_wait(&s.empty[st], ph ^ 1, 1)) break;
                mbar_expect_tx(&s.full[st], STAGE_BYTES);
                if (kb < g.kb1) tma_load_2d(s.A[st], &tmA, kb * BK, static_cast<int>(m0), &s.full[st]);
                else tma_load_2d(s.A[st], &tmA2, (kb - g.kb1) * BK, static_cast<int>(m0), &s.full[st]);
                tma_load_2d(s.Bh[st], &tmBh, kb * BK, 0, &s.full[st]);
                tma_load_2d(s.Bl[st], &tmBl, kb * BK, 0, &s.full[st]);
                ++issued;
            }
            // Every copy issued must have landed before the CTA may exit.
            for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)
                mbar_wait(&s.full[kb % STAGES], (kb / STAGES) & 1, 2);
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            bool ok = true;
            for (int kb = 0; kb < KB && ok; ++kb) {
                const int st = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                if (!(ok = mbar_wait(&s.split[st], ph, 3))) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
                for (int k = 0; k < BK / 8; ++k) {  // K = 8 tf32 (32 bytes) per MMA
                    const uint64_t ah = sw128_desc(s.A[st] + k * 8), al = sw128_desc(s.Al[st] + k * 8);
                    const uint64_t bh = sw128_desc(s.Bh[st] + k * 8), bl = sw128_desc(s.Bl[st] + k * 8);
                    mma_tf32(tmem, al, bh, IDESC, (kb | k) != 0);
                    mma_tf32(tmem, ah, bl, IDESC, 1);
                    mma_tf32(tmem, ah, bh, IDESC, 1);
                }
                mma_commit(&s.empty[st]);  // frees the stage once these MMAs have read it
            }
            mma_commit(&s.acc);            // accumulator complete (or: everything issued has retired)
        }
    } else {
        // ── split (Ah in place, Al) then epilogue: 128 threads ──
        const int t = threadIdx.x - 64;
        bool ok = true, stored = false;
        for (int kb = 0; kb < KB; ++kb) {
            const int st = kb % STAGES;
            const uint32_t ph = (kb / STAGES) & 1;
            if (!(ok = mbar_wait(&s.full[st], ph, 4))) break;
            float4* a = reinterpret_cast<float4*>(s.A[st]);
            float4* l = reinterpret_cast<float4*>(s.Al[st]);
#pragma unroll 4
            for (int i = t; i < BM * BK / 4; i += 128) {
                const float4 x = a[i];
                const float4 h = make_float4(tf32_rn(x.x), tf32_rn(x.y), tf32_rn(x.z), tf32_rn(x.w));
                a[i] = h;
                l[i] = make_float4(__fsub_rn(x.x, h.x), __fsub_rn(x.y, h.y), __fsub_rn(x.z, h.z), __fsub_rn(x.w, h.w));
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
            mbar_arrive(&s.split[st]);
        }
        const bool acc_ready = ok && mbar_wait(&s.acc, 0, 5);
        if (acc_ready && !PEERS && g.tma_store) {
            // TMA-store epilogue.  Measured (clock64 per role, 232,965 x 602 x
            // 128): with one store instruction per 128-byte row segment the
            // epilogue took ~30k of a tile's ~63k cycles -- a latency-bound
            // store stream while the other SMs stream A from HBM.  The last
            // wait is for the boxes to be read out of shared memory only: the
            // CTA may exit while its writes complete.  Here each
            // lane (one row) finishes its 16 columns per TMEM load (row scale,
            // bias, activation), writes them as 16-byte chunks into 32 x 32
            // boxes laid out with the 128-byte swizzle (chunk c of row r at
            // c ^ (r % 8): a warp's 32 writes cover all banks), and one lane
            // hands each box to the TMA engine.
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int q = warp & 3;  // this warp's TMEM lane quarter = its 32 rows of the tile
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
            const int64_t row0 = m0 + q * 32, row = row0 + lane;
            constexpr int kBoxes = (BN + 31) / 32;  // 32 x 32 boxes per warp (a box is 4 KB whatever BN)
            float* stage = reinterpret_cast<float*>(&s) + static_cast<size_t>(q) * kBoxes * 1024;  // the idle ring
            const float sc = (g.rs && row < g.M) ? __ldg(g.rs + row) : 1.0f;
            const bool has_rs = g.rs != nullptr, has_bias = g.bias != nullptr;
            const int act = g.act;
            const float alpha = g.alpha;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15}, [%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(taddr + c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
                if (has_rs) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(v[j], sc);
                }
                if (has_bias) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], c0 + j < g.N ? __ldg(g.bias + c0 + j) : 0.0f);
                }
                act_v<16>(v, act, alpha);
                float* box = stage + (c0 / 32) * 1024;  // 32 rows x 32 floats
                const int cb = (c0 % 32) / 4;           // first 16-byte chunk of these 16 columns
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int phys = (cb + jj) ^ (lane & 7);
                    *reinterpret_cast<float4*>(box + lane * 32 + phys * 4) =
                        make_float4(v[4 * jj], v[4 * jj + 1], v[4 * jj + 2], v[4 * jj + 3]);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> TMA reads
            __syncwarp();
            if (lane == 0 && row0 < g.M) {
                for (int b = 0; b * 32 < BN && b * 32 < g.N; ++b) {
                    const int col = b * 32;
                    if (col < g.nsplit) tma_store_2d(&tmC, stage + b * 1024, col, static_cast<int>(row0));
                    else tma_store_2d(&tmC2, stage + b * 1024, col - static_cast<int>(g.nsplit), static_cast<int>(row0));
                }
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                // the boxes have been read out of shared memory (the writes
                // complete with the grid)
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
            __syncwarp();
            stored = true;
        } else if (acc_ready) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const int q = warp & 3;  // this warp's TMEM lane quarter = its 32 rows of the tile
            const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
            // The accumulator complete means every MMA has read its operands
            // and every copy has landed: the pipeline's shared memory is free.
            // Each warp stages its 32 rows there, then stores them row by row,
            // coalesced.  Local output: 1 column per lane, row stride BN + 1
            // (the column-wise staging writes hit 32 banks).  With peer
            // copies: 4 columns per lane (16-byte stores, 4x fewer NVLink
            // store instructions), row stride BN + 4 (16-byte aligned rows).
            // (Measured on the 232,965 x 602 x 128 GEMM: the 16-byte path is
            // slower for local-only output, 0.42 vs 0.33 ms, and faster with
            // one peer, 0.31 vs 0.38 ms.)
            static_assert(BM * (BN + 4) <= STAGES * (2 * BM * BK + 2 * BN * BK), "staging tile exceeds the ring");
            const bool vec = PEERS && g.vec;
            // Flat: output rows exactly ncols wide (a gather buffer), so a
            // warp's 32 rows are one contiguous block, 128-byte aligned
            // whenever 32 * ncols * 4 is (ncols % 4 == 0): staged at stride
            // ncols and stored as whole 512-byte warp segments -- for narrow
            // rows (44 floats) per-row stores had sent partial lines over
            // NVLink.
            const bool flat = vec && g.ldc == g.ncols;
            const int SB = flat ? static_cast<int>(g.ncols) : (vec ? BN + 4 : BN + 1);
            const bool has_rs = g.rs != nullptr, has_bias = g.bias != nullptr;
            const int act = g.act;
            const float alpha = g.alpha;
            float* tile = reinterpret_cast<float*>(&s) + static_cast<size_t>(q) * 32 * SB;  // the ring's start
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t r[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15}, [%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(taddr + c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        if (!flat || c0 + j < SB)  // flat rows hold ncols columns only
                            *reinterpret_cast<float4*>(tile + lane * SB + c0 + j) =
                                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                            __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) tile[lane * SB + c0 + j] = __uint_as_float(r[j]);
                }
            }
            __syncwarp();
            const int rows = static_cast<int>(g.M - (m0 + q * 32) < 32 ? g.M - (m0 + q * 32) : 32);
            if (flat) {
                // Vector v of the block: element e = 4v is row e / ncols,
                // column e % ncols (a vector never crosses a row).
                const int nc = SB;
                const int nv = rows > 0 ? rows * nc / 4 : 0;
                const int64_t base = (m0 + q * 32) * g.ldc;
#pragma unroll 4
                for (int v = lane; v < nv; v += 32) {
                    const int e = 4 * v, rr = e / nc, col = e - rr * nc;
                    const float4 t4 = *reinterpret_cast<const float4*>(tile + e);
                    float x[4] = {t4.x, t4.y, t4.z, t4.w};
                    if (has_rs) {
                        const float sc = __ldg(g.rs + m0 + q * 32 + rr);
#pragma unroll
                        for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(x[k], sc);
                    }
                    if (has_bias) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) x[k] = __fadd_rn(x[k], col + k < g.N ? __ldg(g.bias + col + k) : 0.0f);
                    }
                    act_v<4>(x, act, alpha);
                    const float4 val = make_float4(x[0], x[1], x[2], x[3]);
                    *reinterpret_cast<float4*>(g.C + base + e) = val;
                    if (PEERS)
                        for (int p = 0; p < peers.n; ++p) *reinterpret_cast<float4*>(peers.c[p] + base + e) = val;
                }
            } else if (vec) {
                // One 16-byte vector of row rr at column col: row scale, bias,
                // activation, then into C and every peer copy (NVLink stores).
                auto put = [&](int rr, int col, const float (&bb)[4]) {
                    const int64_t off = (m0 + q * 32 + rr) * g.ldc;
                    const float sc = g.rs ? __ldg(g.rs + m0 + q * 32 + rr) : 1.0f;
                    const float4 t4 = *reinterpret_cast<const float4*>(tile + rr * SB + col);
                    float x[4] = {t4.x, t4.y, t4.z, t4.w};
                    if (has_rs) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) x[e] = __fmul_rn(x[e], sc);
                    }
                    if (has_bias) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) x[e] = __fadd_rn(x[e], bb[e]);
                    }
                    act_v<4>(x, act, alpha);
                    const float4 v = make_float4(x[0], x[1], x[2], x[3]);
                    *reinterpret_cast<float4*>(g.C + off + col) = v;
                    if (PEERS)
                        for (int p = 0; p < peers.n; ++p) *reinterpret_cast<float4*>(peers.c[p] + off + col) = v;
                };
                // Lanes per row: a row of BN columns is BN / 4 vectors.  Narrow
                // tiles store 32 / G rows per instruction (a 44-float row had
                // kept 21 of 32 lanes idle with one row per instruction).
                constexpr int G = BN / 4 <= 4 ? 4 : (BN / 4 <= 8 ? 8 : (BN / 4 <= 16 ? 16 : 32));
                if constexpr (G < 32) {
                    constexpr int RPI = 32 / G;
                    const int col = (lane % G) * 4;
                    float b4[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) b4[e] = (g.bias && col + e < g.N) ? __ldg(g.bias + col + e) : 0.0f;
                    if (col < g.ncols) {
#pragma unroll 4
                        for (int rr = lane / G; rr < rows; rr += RPI) put(rr, col, b4);
                    }
                } else {
                    constexpr int V4 = (BN / 4 + 31) / 32;  // 4-column groups per lane: lane + 32k
                    float bv[V4][4];
#pragma unroll
                    for (int k = 0; k < V4; ++k)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int col = (lane + 32 * k) * 4 + e;
                            bv[k][e] = (g.bias && col < g.N) ? __ldg(g.bias + col) : 0.0f;  // padding: 0
                        }
#pragma unroll 8
                    for (int rr = 0; rr < rows; ++rr) {  // 8 rows' loads in flight
#pragma unroll
                        for (int k = 0; k < V4; ++k) {
                            const int col = (lane + 32 * k) * 4;
                            if (col < g.ncols) put(rr, col, bv[k]);
                        }
                    }
                }
            } else {
                constexpr int CPL = (BN + 31) / 32;  // columns per lane: lane + 32k
                float bv[CPL];
#pragma unroll
                for (int k = 0; k < CPL; ++k) {
                    const int col = lane + 32 * k;
                    bv[k] = (g.bias && col < g.N) ? __ldg(g.bias + col) : 0.0f;
                }
#pragma unroll 4
                for (int rr = 0; rr < rows; ++rr) {
                    const int64_t row = m0 + q * 32 + rr;
                    const int64_t off = row * g.ldc;
                    const float sc = g.rs ? __ldg(g.rs + row) : 1.0f;
#pragma unroll
                    for (int k = 0; k < CPL; ++k) {
                        const int col = lane + 32 * k;
                        if (col < g.N) {
                            float x[1] = {tile[rr * SB + col]};
                            if (has_rs) x[0] = __fmul_rn(x[0], sc);
                            if (has_bias) x[0] = __fadd_rn(x[0], bv[k]);
                            act_v<1>(x, act, alpha);
                            const float v = x[0];
                            if (!PEERS && col >= g.nsplit) {
                                g.C2[row * g.ldc2 + (col - g.nsplit)] = v;
                                continue;
                            }
                            if (!PEERS && g.gap_lo && col >= g.gap_lo) continue;  // the split's padding gap
                            g.C[off + col] = v;
                            if (PEERS)
                                for (int p = 0; p < peers.n; ++p) peers.c[p][off + col] = v;
                        }
                    }
                }
            }
            stored = true;
        }
        if (PEERS && peers.n > 0) {
            // Signal each peer once this tile is in its memory: every epilogue
            // thread fences its stores at system scope, the 128 threads meet
            // (and agree that all of them stored), then one thread adds 1 to
            // this rank's counter on each peer with release semantics.
            __threadfence_system();
            uint32_t all_stored;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\t"
                "setp.ne.u32 p, %1, 0;\n\t"
                "barrier.cta.red.and.pred q, 1, 128, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(all_stored)
                : "r"(static_cast<uint32_t>(stored))
                : "memory");
            if (t == 0 && all_stored)
                for (int p = 0; p < peers.n; ++p)
                    asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(peers.flag[p]) : "memory");
        }
    }

    // Teardown: all MMAs retired (the acc commit covers every earlier MMA),
    // all copies landed (producer drain), then TMEM is returned.
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        if (lane == 0) {
            mma_commit(&s.drain);
            mbar_wait(&s.drain, 0, 6);
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// ── Persistent form ──────────────────────────────────────────────────────
// One CTA per SM walks the tiles t = blockIdx.x, + gridDim.x, ...  Two TMEM
// accumulators let tile t's epilogue (including its stores to peer copies)
// run while tile t+1's k-blocks are loaded, split and multiplied:
//   warp 0      TMA producer (one ring across tiles);
//   warp 1      TMEM (2 accumulators) and the MMAs into accumulator t % 2;
//   warps 2-5   the 3xTF32 split of each A stage;
//   warps 6-9   the epilogue: 32-column chunks TMEM -> registers -> a
//               per-warp staging buffer -> row segments (+ row scale, bias,
//               activation) into C and every peer copy: with 16-byte stores
//               (g.vec) four rows' 128-byte segments per store instruction,
//               else one row's segment of 4-byte stores; the accumulator is
//               released as soon as its last chunk is read; a tile's peer
//               counters are bumped after its stores (system-scope fence,
//               release add).
template <int BN, int STAGES>
struct TcpSmem {
    float A[STAGES][BM * BK];
    float Al[STAGES][BM * BK];
    float Bh[STAGES][BN * BK];
    float Bl[STAGES][BN * BK];
    float out[4][32 * 36];  // per epilogue warp: 32 rows x 32 columns, row stride 33 (scalar) or 36 (16-byte)
    uint64_t full[STAGES], split[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain;
    uint32_t tmem;
};

// 128 epilogue threads agree (named barrier 2): true iff every one passed `mine`.
__device__ __forceinline__ bool epilogue_all(bool mine) {
    uint32_t all;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.cta.red.and.pred q, 2, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(all)
        : "r"(static_cast<uint32_t>(mine))
        : "memory");
    return all != 0;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(320, 1) gemm_tcp_kernel(const __grid_constant__ CUtensorMap tmA,
                                                          const __grid_constant__ CUtensorMap tmBh,
                                                          const __grid_constant__ CUtensorMap tmBl,
                                                          const TcArgs g,
                                                          const __grid_constant__ PeerOut peers) {
    extern __shared__ uint8_t raw[];
    using Smem = TcpSmem<BN, STAGES>;
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t ACC_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
    constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
    constexpr uint32_t STAGE_BYTES = (BM * BK + 2 * BN * BK) * 4;
    constexpr uint32_t IDESC = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = static_cast<int>((g.K + BK - 1) / BK);
    const int64_t ntiles = (g.M + BM - 1) / BM;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.split[i], 128);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s.acc_full[i], 1);
            mbar_init(&s.acc_empty[i], 4);  // lane 0 of each epilogue warp
        }
        mbar_init(&s.drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = s.tmem;

    if (warp == 0) {
        // ── TMA producer ──
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int st = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (it >= STAGES && !(ok = mbar_wait(&s.empty[st], ph ^ 1, 1))) break;
                    mbar_expect_tx(&s.full[st], STAGE_BYTES);
                    tma_load_2d(s.A[st], &tmA, kb * BK, static_cast<int>(tile * BM), &s.full[st]);
                    tma_load_2d(s.Bh[st], &tmBh, kb * BK, 0, &s.full[st]);
                    tma_load_2d(s.Bl[st], &tmBl, kb * BK, 0, &s.full[st]);
                }
            }
            // Every copy issued must have landed before the CTA may exit.
            for (int q = (it > STAGES ? it - STAGES : 0); q < it; ++q)
                mbar_wait(&s.full[q % STAGES], (q / STAGES) & 1, 2);
        }
    } else if (warp == 1) {
        // ── MMA issuer ──
        if (lane == 0) {
            int it = 0, lt = 0;
            bool ok = true;
            for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++lt) {
                const int acc = lt & 1;
                if (lt >= 2 && !(ok = mbar_wait(&s.acc_empty[acc], ((lt >> 1) & 1) ^ 1, 7))) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint32_t d = tmem + static_cast<uint32_t>(acc) * ACC_COLS;
                for (int kb = 0; kb < KB; ++kb, ++it) {
                    const int st = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!(ok = mbar_wait(&s.split[st], ph, 3))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;");
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {
                        const uint64_t ah = sw128_desc(s.A[st] + k * 8), al = sw128_desc(s.Al[st] + k * 8);
                        const uint64_t bh = sw128_desc(s.Bh[st] + k * 8), bl = sw128_desc(s.Bl[st] + k * 8);
                        mma_tf32(d, al, bh, IDESC, (kb | k) != 0);
                        mma_tf32(d, ah, bl, IDESC, 1);
                        mma_tf32(d, ah, bh, IDESC, 1);
                    }
                    mma_commit(&s.empty[st]);
                }
                if (ok) mma_commit(&s.acc_full[acc]);
            }
        }
    } else if (warp < 6) {
        // ── split: 128 threads ──
        const int t = threadIdx.x - 64;
        int it = 0;
        bool ok = true;
        for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            for (int kb = 0; kb < KB; ++kb, ++it) {
                const int st = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                if (!(ok = mbar_wait(&s.full[st], ph, 4))) break;
                float4* a = reinterpret_cast<float4*>(s.A[st]);
                float4* l = reinterpret_cast<float4*>(s.Al[st]);
#pragma unroll 4
                for (int i = t; i < BM * BK / 4; i += 128) {
                    const float4 x = a[i];
                    const float4 h = make_float4(tf32_rn(x.x), tf32_rn(x.y), tf32_rn(x.z), tf32_rn(x.w));
                    a[i] = h;
                    l[i] = make_float4(__fsub_rn(x.x, h.x), __fsub_rn(x.y, h.y), __fsub_rn(x.z, h.z),
                                       __fsub_rn(x.w, h.w));
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&s.split[st]);
            }
        }
    } else {
        // ── epilogue: 128 threads ──
        const int e = threadIdx.x - 192;
        const int q = warp & 3;  // this warp's TMEM lane quarter = its 32 rows of a tile
        float* buf = s.out[warp - 6];
        const bool vec = g.vec != 0, has_rs = g.rs != nullptr, has_bias = g.bias != nullptr;
        const bool split = g.nsplit < g.N;  // columns [nsplit, N) go to C2 (local output only)
        const int act = g.act;
        const float alpha = g.alpha;
        int lt = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
            const int acc = lt & 1;
            const bool w = mbar_wait(&s.acc_full[acc], (lt >> 1) & 1, 5);
            if (!epilogue_all(w)) break;  // all 128 leave together
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t taddr = tmem + static_cast<uint32_t>(acc) * ACC_COLS + (static_cast<uint32_t>(q * 32) << 16);
            const int64_t r0 = tile * BM + q * 32;
            const int rows = static_cast<int>(g.M - r0 < 32 ? g.M - r0 : 32);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15}, [%16];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                      "=r"(r[15])
                    : "r"(taddr + c0));
                if (c0 + 16 < BN)
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                        "%12, %13, %14, %15}, [%16];"
                        : "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
                          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                          "=r"(r[30]), "=r"(r[31])
                        : "r"(taddr + c0 + 16));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (c0 + 32 >= BN) {  // the accumulator is read: the MMA warp may reuse it
                    asm volatile("tcgen05.fence::before_thread_sync;");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
                }
                if (vec) {
                    // Row stride 36: a quarter-warp's 16-byte writes (rows
                    // lane..lane+7) and reads (8 vectors of one row) each
                    // cover the 32 banks once.
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        if (c0 + j < BN)
                            *reinterpret_cast<float4*>(buf + lane * 36 + j) =
                                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                            __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                    __syncwarp();
                    // Lane = (row in a group of 4, 4-column vector): one store
                    // instruction writes four rows' 128-byte segments.
                    const int cv = (lane & 7) * 4, col = c0 + cv;
                    if (col < g.ncols) {  // ncols = round_up(N, 4) <= BN
                        float b4[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) b4[k] = (has_bias && col + k < g.N) ? __ldg(g.bias + col + k) : 0.0f;
#pragma unroll 4
                        for (int rr = lane >> 3; rr < rows; rr += 4) {
                            const float4 t4 = *reinterpret_cast<const float4*>(buf + rr * 36 + cv);
                            float x[4] = {t4.x, t4.y, t4.z, t4.w};
                            if (has_rs) {
                                const float sc = __ldg(g.rs + r0 + rr);
#pragma unroll
                                for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(x[k], sc);
                            }
                            if (has_bias) {
#pragma unroll
                                for (int k = 0; k < 4; ++k) x[k] = __fadd_rn(x[k], b4[k]);
                            }
                            act_v<4>(x, act, alpha);
                            const float4 v = make_float4(x[0], x[1], x[2], x[3]);
                            if (split && col >= g.nsplit) {  // a vector never straddles nsplit (% 4 == 0)
                                *reinterpret_cast<float4*>(g.C2 + (r0 + rr) * g.ldc2 + (col - g.nsplit)) = v;
                                continue;
                            }
                            if (split && g.gap_lo && col >= g.gap_lo) continue;  // the gap (gap_lo % 4 == 0)
                            const int64_t off = (r0 + rr) * g.ldc + col;
                            *reinterpret_cast<float4*>(g.C + off) = v;
                            for (int p = 0; p < peers.n; ++p) *reinterpret_cast<float4*>(peers.c[p] + off) = v;
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (c0 + j < BN) buf[lane * 33 + j] = __uint_as_float(r[j]);
                    __syncwarp();
                    const int col = c0 + lane;
                    const float bv = (has_bias && col < g.N) ? __ldg(g.bias + col) : 0.0f;
#pragma unroll 4
                    for (int rr = 0; rr < rows; ++rr) {
                        if (col < g.ncols) {
                            float x[1] = {buf[rr * 33 + lane]};
                            if (has_rs) x[0] = __fmul_rn(x[0], __ldg(g.rs + r0 + rr));
                            if (has_bias) x[0] = __fadd_rn(x[0], bv);
                            act_v<1>(x, act, alpha);
                            const float v = x[0];
                            if (split && col >= g.nsplit) {
                                g.C2[(r0 + rr) * g.ldc2 + (col - g.nsplit)] = v;
                                continue;
                            }
                            if (split && g.gap_lo && col >= g.gap_lo) continue;
                            const int64_t off = (r0 + rr) * g.ldc + col;
                            g.C[off] = v;
                            for (int p = 0; p < peers.n; ++p) peers.c[p][off] = v;
                        }
                    }
                }
                __syncwarp();  // buf is rewritten by the next chunk
            }
            if (peers.n > 0) {
                __threadfence_system();
                if (epilogue_all(true) && e == 0)
                    for (int p = 0; p < peers.n; ++p)
                        asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(peers.flag[p]) : "memory");
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 1) {
        if (lane == 0) {
            mma_commit(&s.drain);
            mbar_wait(&s.drain, 0, 6);
        }
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

// B (K x N, ld ldb) -> Bt_hi, Bt_lo: rows n < N, columns k < Kseg of a K-major
// matrix with row stride ldt (zeros for k >= K), tf32 round-to-nearest split.
__global__ void split_bt_kernel(const float* B, int64_t ldb, int64_t K, int64_t N, int64_t Kseg, int64_t ldt,
                                float* hi, float* lo) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= N * Kseg) return;
    const int64_t n = t / Kseg, k = t % Kseg;
    const float x = k < K ? B[k * ldb + n] : 0.0f;
    const float h = tf32_rn(x);
    hi[n * ldt + k] = h;
    lo[n * ldt + k] = __fsub_rn(x, h);
}

void split_bt(const float* B, int64_t ldb, int64_t K, int64_t N, int64_t Kseg, int64_t ldt, float* hi, float* lo,
              cudaStream_t s) {
    if (N * Kseg == 0) return;
    launch("split_bt", split_bt_kernel, dim3(static_cast<unsigned>(ceil_div(N * Kseg, 256))), dim3(256), 0, s, B, ldb,
           K, N, Kseg, ldt, hi, lo);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    if (!fn) fail(TG_ERR_CUDA, "gemm (tensor cores): cuTensorMapEncodeTiled is unavailable");
    return fn;
}

CUtensorMap make_map(const float* base, int64_t inner, int64_t outer, int64_t row_stride_elems, uint32_t box_outer) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(TG_ERR_CUDA, "gemm (tensor cores): tensor map encoding failed (" + std::to_string(r) + ")");
    return m;
}

template <int BN, int STAGES>
void launch_tc_s(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& bh, const CUtensorMap& bl,
                 const CUtensorMap& c, const CUtensorMap& c2, const TcArgs& g, const PeerOut& peers,
                 cudaStream_t s) {
    static_assert(4 * ((BN + 31) / 32) * 4096 <= STAGES * (2 * BM * BK + 2 * BN * BK) * 4,
                  "TMA-store staging exceeds the ring");
    const size_t smem = sizeof(TcSmem<BN, STAGES>) + 1024;
    auto kern = peers.n > 0 ? gemm_tc_kernel<BN, STAGES, true> : gemm_tc_kernel<BN, STAGES, false>;
    TG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    launch("gemm_tc", kern, dim3(static_cast<unsigned>(ceil_div(g.M, BM))), dim3(192), smem, s, a, a2, bh, bl, c, c2,
           g, peers);
}

constexpr int tcp_stages(int BN) {
    return (192 * 1024) / ((2 * BM * BK + 2 * BN * BK) * 4) > 4 ? 4 : (192 * 1024) / ((2 * BM * BK + 2 * BN * BK) * 4);
}

template <int BN>
void launch_tcp(const CUtensorMap& a, const CUtensorMap& bh, const CUtensorMap& bl, const TcArgs& g,
                const PeerOut& peers, cudaStream_t s) {
    constexpr int S = tcp_stages(BN);
    const size_t smem = sizeof(TcpSmem<BN, S>) + 1024;
    auto kern = gemm_tcp_kernel<BN, S>;
    TG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const int64_t tiles = ceil_div(g.M, BM);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(tiles, num_sms()));
    launch("gemm_tc", kern, dim3(grid), dim3(320), smem, s, a, bh, bl, g, peers);
}

// Which kernel.  The persistent one overlaps a tile's epilogue -- above all
// its stores to peer copies -- with the next tile's main loop; the per-tile
// one has the TMA-store epilogue and, for short K, two CTAs per SM.
// Measured on B200 (CUDA events; same-device copies standing in for peers):
//   232,965 x 602 x 128, row-scaled:  local 0.245 vs 0.287 ms, one copy
//   0.27 vs 0.41, three 0.33 vs 0.45; 116,483 rows: local 0.145 vs 0.162,
//   one copy 0.16 vs 0.23; in the 2-GPU forward (copy over NVLink) the
//   layer-1 GEMM 0.215 vs 0.294 ms;
//   232,965 x 128 x 41: local 0.095 vs 0.080, one copy 0.15 vs 0.12;
//   with 4-byte stores (unaligned output) the persistent kernel is slower.
// So: the persistent kernel for K > 256 with 16-byte stores and more tiles
// than SMs, else the per-tile one; TINYGNN_B200_GEMM_PERSISTENT=1 / 0
// forces either (read on every call).
bool use_persistent(bool vec, int64_t K, int64_t tiles) {
    const char* e = std::getenv("TINYGNN_B200_GEMM_PERSISTENT");
    if (e && e[0] == '1') return true;
    if (e && e[0] == '0') return false;
    return vec && K > 8 * BK && tiles > num_sms();
}

// A deep ring for long K; for short K (a few k-blocks per tile, where one
// tile's pipeline fill and epilogue dominate) two stages, so that two CTAs
// share an SM and one's epilogue overlaps the other's main loop (measured:
// the K = 128, N = 41 layer-2 GEMM is latency-bound at one CTA per SM).
template <int BN>
void launch_tc(const CUtensorMap& a, const CUtensorMap& a2, const CUtensorMap& bh, const CUtensorMap& bl,
               const CUtensorMap& c, const CUtensorMap& c2, const TcArgs& g, const PeerOut& peers, cudaStream_t s) {
    constexpr int kShallow = 2;
    constexpr bool two_fit = 2 * (sizeof(TcSmem<BN, kShallow>) + 1024) <= 227 * 1024;
    if (two_fit && g.K <= 8 * BK)
        launch_tc_s<BN, two_fit ? kShallow : stages_for(BN)>(a, a2, bh, bl, c, c2, g, peers, s);
    else launch_tc_s<BN, stages_for(BN)>(a, a2, bh, bl, c, c2, g, peers, s);
}

// Output tile width.  96 (for 65..96 columns, e.g. a pair product of two
// 41-wide weights) keeps a short-K two-stage ring small enough for two CTAs
// per SM, which a 128-wide tile is not.
int tile_n(int64_t N) {
    return N <= 16 ? 16 : N <= 32 ? 32 : N <= 48 ? 48 : N <= 64 ? 64 : N <= 96 ? 96 : N <= 128 ? 128 : 256;
}

// Runs the kernel for a prepared B^T (hi at bt, lo at bt + N * ldt) and
// A maps; g's N, K (and C2 / nsplit / kb1) describe the product.
bool aligned16(const void* p, int64_t ld) { return reinterpret_cast<uintptr_t>(p) % 16 == 0 && ld % 4 == 0; }

void run_tc(const CUtensorMap& ma, const CUtensorMap& ma2, const float* bt, int64_t ldt, TcArgs g,
            const PeerOut& peers, cudaStream_t s) {
    const int BN = tile_n(g.N);
    const CUtensorMap mh = make_map(bt, g.K, g.N, ldt, static_cast<uint32_t>(BN));
    const CUtensorMap ml = make_map(bt + g.N * ldt, g.K, g.N, ldt, static_cast<uint32_t>(BN));
    // Output tensor maps for the TMA-store epilogue (local outputs only).
    CUtensorMap mc = ma, mc2 = ma;
    g.tma_store = 0;
    // (Measured in the GCN forward on B200, same build: layer-1 GEMM 0.46 ->
    // 0.385 ms, layer-2 0.132 -> 0.091 ms against the per-row stores.)
    // A TMA store writes whole 16-byte pieces of a row, also where the box
    // is clipped at the tensor's width: each stored width must be a multiple
    // of 4 floats -- its own, or rounded up where the caller's rows have room.
    const auto w4 = [&](int64_t w) { return g.pad_ok ? (w + 3) / 4 * 4 : w; };
    const int64_t w1 = w4(g.gap_lo ? g.gap_lo : std::min(g.N, g.nsplit)), w2 = w4(g.N - g.nsplit);
    if (peers.n == 0 && g.M <= INT32_MAX && aligned16(g.C, g.ldc) && w1 % 4 == 0 &&
        (g.nsplit >= g.N || (g.nsplit % 32 == 0 && aligned16(g.C2, g.ldc2) && w2 % 4 == 0))) {
        mc = make_map(g.C, w1, g.M, g.ldc, 32);  // boxes clip at C's (stored) width
        if (g.nsplit < g.N) mc2 = make_map(g.C2, w2, g.M, g.ldc2, 32);
        g.tma_store = 1;
    }
    if (use_persistent(g.vec != 0, g.K, ceil_div(g.M, BM)) && g.kb1 * BK >= g.K) {
        switch (BN) {
            case 16: launch_tcp<16>(ma, mh, ml, g, peers, s); break;
            case 32: launch_tcp<32>(ma, mh, ml, g, peers, s); break;
            case 48: launch_tcp<48>(ma, mh, ml, g, peers, s); break;
            case 64: launch_tcp<64>(ma, mh, ml, g, peers, s); break;
            case 96: launch_tcp<96>(ma, mh, ml, g, peers, s); break;
            case 128: launch_tcp<128>(ma, mh, ml, g, peers, s); break;
            default: launch_tcp<256>(ma, mh, ml, g, peers, s); break;
        }
        return;
    }
    switch (BN) {
        case 16: launch_tc<16>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        case 32: launch_tc<32>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        case 48: launch_tc<48>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        case 64: launch_tc<64>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        case 96: launch_tc<96>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        case 128: launch_tc<128>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
        default: launch_tc<256>(ma, ma2, mh, ml, mc, mc2, g, peers, s); break;
    }
}

}  // namespace

bool gemm_tc_supported(int64_t N, int64_t K, const float* A, int64_t lda) {
    return N >= 1 && N <= 256 && K >= 1 && lda % 4 == 0 && (reinterpret_cast<uintptr_t>(A) % 16) == 0;
}

void gemm_tc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
             int64_t ldc, const float* bias, int act, float alpha, cudaStream_t s, const PeerOut& peers,
             bool c_cols_padded, const float* row_scale) {
    if (M == 0 || N == 0) return;
    const int BN = tile_n(N);
    const int64_t Kp = (K + 3) / 4 * 4;
    Scratch<float> bt(static_cast<size_t>(2 * N * Kp), s);
    split_bt(B, ldb, K, N, Kp, Kp, bt.p, bt.p + N * Kp, s);
    const CUtensorMap ma = make_map(A, K, M, lda, BM);
    // 16-byte stores (the persistent kernel, and the per-tile one's peer
    // epilogue) when every output row starts 16-byte aligned and the stored
    // width is a multiple of 4 (N itself, or N padded when the caller's rows
    // have room: those columns receive act(0 + 0)).
    const int64_t n4 = (N + 3) / 4 * 4;
    bool vec = ldc % 4 == 0 && reinterpret_cast<uintptr_t>(C) % 16 == 0 &&
               (N % 4 == 0 || (c_cols_padded && ldc >= n4));
    for (int p = 0; p < peers.n; ++p) vec = vec && reinterpret_cast<uintptr_t>(peers.c[p]) % 16 == 0;
    (void)BN;
    TcArgs g{C, ldc, M, N, K, bias, act, alpha, vec ? n4 : N, vec ? 1 : 0, row_scale, nullptr, 0, N,
             static_cast<int>(ceil_div(K, BK)), 0};
    g.pad_ok = c_cols_padded && ldc >= n4;
    run_tc(ma, ma, bt.p, Kp, g, peers, s);
}

// C1 = A . B1 and C2 = A . B2 (K x N each) in one pass over A: the product
// with [B1 | B2] (2N <= 256 columns), its columns split in the epilogue.
void gemm_tc_pair(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B1, const float* B2,
                  int64_t ldb, float* C1, int64_t ldc1, float* C2, int64_t ldc2, cudaStream_t s,
                  bool c_cols_padded) {
    if (M == 0 || N == 0) return;
    // B2 starts at product column Ns.  Ns = N, unless N is not a multiple of
    // 32 and both outputs can take TMA stores: then Ns = round_up(N, 32),
    // columns [N, Ns) a zero gap, so the split falls on a 32-column box and
    // both outputs are stored by TMA boxes clipped at their widths (per-row
    // stores had taken the 232,965 x 128 x (41 + 41) product 0.26 ms).
    const bool aligned = aligned16(C1, ldc1) && aligned16(C2, ldc2);
    const int64_t N32 = (N + 31) / 32 * 32, n4 = (N + 3) / 4 * 4;
    const bool pad_ok = c_cols_padded && ldc1 >= n4 && ldc2 >= n4;
    const bool gap = N % 32 != 0 && aligned && (N % 4 == 0 || pad_ok) && M <= INT32_MAX && N32 + N <= 256;
    const int64_t Kp = (K + 3) / 4 * 4, Ns = gap ? N32 : N, N2 = Ns + N;
    Scratch<float> bt(static_cast<size_t>(2 * N2 * Kp), s);
    float* hi = bt.p;
    float* lo = bt.p + N2 * Kp;
    split_bt(B1, ldb, K, N, Kp, Kp, hi, lo, s);                     // rows [0, N) of B^T
    if (gap) {                                                      // rows [N, Ns): zero
        TG_CUDA(cudaMemsetAsync(hi + N * Kp, 0, static_cast<size_t>((Ns - N) * Kp) * sizeof(float), s));
        TG_CUDA(cudaMemsetAsync(lo + N * Kp, 0, static_cast<size_t>((Ns - N) * Kp) * sizeof(float), s));
    }
    split_bt(B2, ldb, K, N, Kp, Kp, hi + Ns * Kp, lo + Ns * Kp, s);  // rows [Ns, Ns + N)
    const CUtensorMap ma = make_map(A, K, M, lda, BM);
    // 16-byte stores (persistent kernel) when both outputs' rows are 16-byte
    // aligned and N % 4 == 0 (no vector straddles the split or the gap)
    const bool vec = aligned && N % 4 == 0;
    TcArgs g{C1, ldc1, M, N2, K, nullptr, TG_ACT_NONE, 0.0f, N2, vec ? 1 : 0, nullptr, C2, ldc2, Ns,
             static_cast<int>(ceil_div(K, BK)), 0};
    g.gap_lo = gap ? N : 0;
    g.pad_ok = pad_ok;
    run_tc(ma, ma, bt.p, Kp, g, PeerOut{}, s);
}

// C = act([A1 | A2] . [B1; B2] + bias): A1 M x K1, A2 M x K2, B1 K1 x N,
// B2 K2 x N; the concatenation never exists -- the producer switches tensor
// maps at k-block kb1 = ceil(K1 / BK) (A1's last block reads zeros past K1,
// and B1's rows are zero-padded to kb1 * BK).
void gemm_tc_cat(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1, int64_t K2, const float* A2,
                 int64_t lda2, const float* B1, int64_t ldb1, const float* B2, int64_t ldb2, float* C, int64_t ldc,
                 const float* bias, int act, float alpha, cudaStream_t s) {
    if (M == 0 || N == 0) return;
    const int kb1 = static_cast<int>(ceil_div(K1, BK));
    const int64_t K1p = static_cast<int64_t>(kb1) * BK, Kt = K1p + K2, Kp = (Kt + 3) / 4 * 4;
    Scratch<float> bt(static_cast<size_t>(2 * N * Kp), s);
    float* hi = bt.p;
    float* lo = bt.p + N * Kp;
    split_bt(B1, ldb1, K1, N, K1p, Kp, hi, lo, s);
    split_bt(B2, ldb2, K2, N, Kp - K1p, Kp, hi + K1p, lo + K1p, s);
    const CUtensorMap ma1 = make_map(A1, K1, M, lda1, BM);
    const CUtensorMap ma2 = make_map(A2, K2, M, lda2, BM);
    const TcArgs g{C, ldc, M, N, Kt, bias, act, alpha, N, 0, nullptr, nullptr, 0, N, kb1, 0};
    run_tc(ma1, ma2, bt.p, Kp, g, PeerOut{}, s);
}

// Reads and clears the tensor-core kernels' error word (synchronises `s`).
int gemm_tc_take_error(cudaStream_t s) {
    int h = 0;
    TG_CUDA(cudaStreamSynchronize(s));
    TG_CUDA(cudaMemcpyFromSymbol(&h, g_tc_error, sizeof(int)));
    if (h) {
        const int zero = 0;
        TG_CUDA(cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int)));
    }
    return h;
}

}  // namespace tg
