// ============================================================================
//  gemm.cu -- dense products on the hot path.
//
//  gemm_exact: C = A . B with every C[i][j] one fused multiply-add chain over
//  k = 0..K-1 in order -- the arithmetic of TinyGNN's matmul (i, k, j loop
//  with AVX2 FMA, src/ops.cpp:120-159) -- so results are bit-identical.
//  Register-tiled SIMT kernel: a CTA of 256 threads owns a BM x BN output
//  tile, stages BK-deep slabs of A (transposed) and B in shared memory,
//  double-buffered through registers, and each thread keeps a TM x TN
//  accumulator block.  The shapes on the path are tall-skinny
//  (N = 7..256), so BN is picked from N and A is read once.
//
//  The DUAL form interleaves two products per k (SAGE's fused dual GEMV,
//  src/layers.cpp:639-669).
// ============================================================================
#include <algorithm>
#include "launch.cuh"

namespace tg {

namespace {

struct GemmArgs {
    int64_t M, N, K;
    const float* A1; int64_t lda1;
    const float* A2; int64_t lda2;   // DUAL only
    const float* B1; const float* B2; int64_t ldb;
    float* C; int64_t ldc;
    const float* bias;
    int act; float alpha;
    int64_t n_fma_cols;  // DUAL: columns < this use the 8-wide body order
};

template <int BM, int BN, int BK, int TM, int TN, bool DUAL>
__global__ void __launch_bounds__(256) gemm_exact_kernel(const GemmArgs g) {
    static_assert((BM / TM) * (BN / TN) == 256, "256 threads");
    constexpr int NA = (BM * BK + 255) / 256;  // A elements per thread per slab
    constexpr int NB = (BK * BN + 255) / 256;  // B elements per thread per slab
    constexpr int NOPS = DUAL ? 2 : 1;

    __shared__ __align__(16) float As[NOPS][BK][BM];
    __shared__ __align__(16) float Bs[NOPS][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN);
    const int ty = tid / (BN / TN);
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;

    // Loader mapping: A slab is BM rows x BK k (k fastest), B slab BK x BN.
    float ra[NOPS][NA], rb[NOPS][NB];
    auto load_slab = [&](int64_t k0) {
#pragma unroll
        for (int o = 0; o < NOPS; ++o) {
            const float* A = o ? g.A2 : g.A1;
            const int64_t lda = o ? g.lda2 : g.lda1;
            const float* B = o ? g.B2 : g.B1;
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int e = tid + q * 256;
                const int r = e / BK, c = e % BK;
                const int64_t gm = m0 + r, gk = k0 + c;
                ra[o][q] = (e < BM * BK && gm < g.M && gk < g.K) ? __ldg(A + gm * lda + gk) : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int e = tid + q * 256;
                const int r = e / BN, c = e % BN;
                const int64_t gk = k0 + r, gn = n0 + c;
                rb[o][q] = (e < BK * BN && gk < g.K && gn < g.N) ? __ldg(B + gk * g.ldb + gn) : 0.0f;
            }
        }
    };
    auto store_slab = [&]() {
#pragma unroll
        for (int o = 0; o < NOPS; ++o) {
#pragma unroll
            for (int q = 0; q < NA; ++q) {
                const int e = tid + q * 256;
                if (e < BM * BK) As[o][e % BK][e / BK] = ra[o][q];
            }
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int e = tid + q * 256;
                if (e < BK * BN) Bs[o][e / BN][e % BN] = rb[o][q];
            }
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    bool body[TN];  // DUAL: column inside the reference's 8-wide body
#pragma unroll
    for (int j = 0; j < TN; ++j) body[j] = (n0 + tx * TN + j) < g.n_fma_cols;

    load_slab(0);
    for (int64_t k0 = 0; k0 < g.K; k0 += BK) {
        __syncthreads();
        store_slab();
        __syncthreads();
        if (k0 + BK < g.K) load_slab(k0 + BK);  // next slab in flight during compute
        const int kn = (g.K - k0 < BK) ? static_cast<int>(g.K - k0) : BK;
        for (int kk = 0; kk < kn; ++kk) {
            float a[NOPS][TM], b[NOPS][TN];
#pragma unroll
            for (int o = 0; o < NOPS; ++o) {
#pragma unroll
                for (int i = 0; i < TM; i += 4) {
                    const float4 t = *reinterpret_cast<const float4*>(&As[o][kk][ty * TM + i]);
                    a[o][i] = t.x; a[o][i + 1] = t.y; a[o][i + 2] = t.z; a[o][i + 3] = t.w;
                }
                if constexpr (TN % 4 == 0) {
#pragma unroll
                    for (int j = 0; j < TN; j += 4) {
                        const float4 t = *reinterpret_cast<const float4*>(&Bs[o][kk][tx * TN + j]);
                        b[o][j] = t.x; b[o][j + 1] = t.y; b[o][j + 2] = t.z; b[o][j + 3] = t.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < TN; ++j) b[o][j] = Bs[o][kk][tx * TN + j];
                }
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) {
                    if constexpr (DUAL) {
                        acc[i][j] = body[j]
                                        ? fmaf(a[1][i], b[1][j], fmaf(a[0][i], b[0][j], acc[i][j]))
                                        : __fadd_rn(acc[i][j], fmaf(a[0][i], b[0][j], __fmul_rn(a[1][i], b[1][j])));
                    } else {
                        acc[i][j] = fmaf(a[0][i], b[0][j], acc[i][j]);
                    }
                }
        }
    }

    // Epilogue: + bias (one rounding), activation, masked store.
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int64_t m = m0 + ty * TM + i;
        if (m >= g.M) break;
        float v[TN];
#pragma unroll
        for (int j = 0; j < TN; ++j) v[j] = acc[i][j];
        if (g.bias) {
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int64_t n = n0 + tx * TN + j;
                v[j] = __fadd_rn(v[j], n < g.N ? __ldg(g.bias + n) : 0.0f);
            }
        }
        act_v<TN>(v, g.act, g.alpha);
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int64_t n = n0 + tx * TN + j;
            if (n < g.N) g.C[m * g.ldc + n] = v[j];
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN, bool DUAL>
void launch_gemm(const GemmArgs& g, cudaStream_t s) {
    dim3 grid(static_cast<unsigned>(ceil_div(g.N, BN)), static_cast<unsigned>(ceil_div(g.M, BM)));
    launch("gemm_exact", gemm_exact_kernel<BM, BN, BK, TM, TN, DUAL>, grid, dim3(256), 0, s, g);
}

template <bool DUAL>
void dispatch_gemm(const GemmArgs& g, cudaStream_t s) {
    if (g.N <= 8) launch_gemm<256, 8, 8, 8, 1, DUAL>(g, s);
    else if (g.N <= 16) launch_gemm<256, 16, 8, 4, 4, DUAL>(g, s);
    else if (g.N <= 32) launch_gemm<128, 32, 8, 4, 4, DUAL>(g, s);
    else if (g.N <= 64) launch_gemm<128, 64, 8, 8, 4, DUAL>(g, s);
    else launch_gemm<128, 128, 8, 8, 8, DUAL>(g, s);
}

}  // namespace

void gemm_exact(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B,
                int64_t ldb, float* C, int64_t ldc, const float* bias, int act, float alpha,
                cudaStream_t s) {
    if (M == 0 || N == 0) return;
    // K == 0 runs no k step: C = act(0 + bias), like the zero-initialised
    // reference output.
    GemmArgs g{M, N, K, A, lda, nullptr, 0, B, nullptr, ldb, C, ldc, bias, act, alpha, 0};
    dispatch_gemm<false>(g, s);
}

bool gemm_tc_supported(int64_t N, int64_t K, const float* A, int64_t lda);
int gemm_tc_take_error(cudaStream_t s);
int gather_take_error(cudaStream_t s);
int peer_take_error(cudaStream_t s);
void gemm_tc(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
             int64_t ldc, const float* bias, int act, float alpha, cudaStream_t s, const PeerOut& peers = PeerOut{},
             bool c_cols_padded = false, const float* row_scale = nullptr);

void gemm_tc_pair(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B1, const float* B2,
                  int64_t ldb, float* C1, int64_t ldc1, float* C2, int64_t ldc2, cudaStream_t s,
                  bool c_cols_padded);
void gemm_tc_cat(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1, int64_t K2, const float* A2,
                 int64_t lda2, const float* B1, int64_t ldb1, const float* B2, int64_t ldb2, float* C, int64_t ldc,
                 const float* bias, int act, float alpha, cudaStream_t s);

// FAST: tensor cores (3xTF32) when the operands allow TMA; otherwise, and in
// EXACT mode, the k-sequential FMA kernel.
void gemm(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
          int64_t ldc, const float* bias, int act, float alpha, int mode, cudaStream_t s) {
    if ((mode & 0xff) == TG_MODE_FAST && gemm_tc_supported(N, K, A, lda))
        gemm_tc(M, N, K, A, lda, B, ldb, C, ldc, bias, act, alpha, s, PeerOut{}, (mode & TG_FLAG_C_COLS_PADDED) != 0);
    else
        gemm_exact(M, N, K, A, lda, B, ldb, C, ldc, bias, act, alpha, s);
}

namespace {
// C = act(rs[i] * C + bias), in place (the scaled GEMM without tensor cores).
__global__ void scale_rows_kernel(int64_t M, int64_t N, float* C, int64_t ldc, const float* rs, const float* bias,
                                  int act, float alpha) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < M * N; t += stride) {
        const int64_t i = t / N, j = t % N;
        float v = __fmul_rn(C[i * ldc + j], rs[i]);
        if (bias) v = __fadd_rn(v, bias[j]);
        C[i * ldc + j] = apply_act(act, v, alpha);
    }
}
}  // namespace

// C = act(diag(rs) . (A . B) + bias): the tensor-core epilogue scales each
// row before the bias; without tensor cores, the exact product then a pass.
void gemm_rowscale(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B, int64_t ldb,
                   float* C, int64_t ldc, const float* rs, const float* bias, int act, float alpha, int mode,
                   cudaStream_t s) {
    if (M == 0 || N == 0) return;
    if ((mode & 0xff) == TG_MODE_FAST && gemm_tc_supported(N, K, A, lda)) {
        gemm_tc(M, N, K, A, lda, B, ldb, C, ldc, bias, act, alpha, s, PeerOut{}, (mode & TG_FLAG_C_COLS_PADDED) != 0,
                rs);
        return;
    }
    gemm_exact(M, N, K, A, lda, B, ldb, C, ldc, nullptr, TG_ACT_NONE, 0.0f, s);
    const int64_t total = M * N;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(total, 256), 8 * num_sms()));
    launch("scale_rows", scale_rows_kernel, dim3(grid), dim3(256), 0, s, M, N, C, ldc, rs, bias, act, alpha);
}

// C1 = A . B1, C2 = A . B2: one tensor-core pass over A in FAST mode when
// [B1 | B2] fits one tile (2N <= 256), else two products.
void gemm_pair(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B1, const float* B2,
               int64_t ldb, float* C1, int64_t ldc1, float* C2, int64_t ldc2, int mode, cudaStream_t s) {
    if (M == 0 || N == 0) return;
    if ((mode & 0xff) == TG_MODE_FAST && gemm_tc_supported(2 * N, K, A, lda)) {
        gemm_tc_pair(M, N, K, A, lda, B1, B2, ldb, C1, ldc1, C2, ldc2, s, (mode & TG_FLAG_C_COLS_PADDED) != 0);
        return;
    }
    gemm(M, N, K, A, lda, B1, ldb, C1, ldc1, nullptr, TG_ACT_NONE, 0.0f, mode, s);
    gemm(M, N, K, A, lda, B2, ldb, C2, ldc2, nullptr, TG_ACT_NONE, 0.0f, mode, s);
}

namespace {
// C = act(C + T + bias) in place (the concatenated product without tensor cores).
__global__ void add_bias_act_kernel(int64_t M, int64_t N, float* C, int64_t ldc, const float* T, int64_t ldt,
                                    const float* bias, int act, float alpha) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < M * N; t += stride) {
        const int64_t i = t / N, j = t % N;
        float v = __fadd_rn(C[i * ldc + j], T[i * ldt + j]);
        if (bias) v = __fadd_rn(v, bias[j]);
        C[i * ldc + j] = apply_act(act, v, alpha);
    }
}
}  // namespace

// C = act([A1 | A2] . [B1; B2] + bias): FAST, one tensor-core pass with the
// concatenation done by the operand loads; otherwise two products and a sum.
void gemm_cat(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1, int64_t K2, const float* A2,
              int64_t lda2, const float* B1, int64_t ldb1, const float* B2, int64_t ldb2, float* C, int64_t ldc,
              const float* bias, int act, float alpha, int mode, cudaStream_t s) {
    if (M == 0 || N == 0) return;
    if ((mode & 0xff) == TG_MODE_FAST && gemm_tc_supported(N, K1, A1, lda1) && gemm_tc_supported(N, K2, A2, lda2)) {
        gemm_tc_cat(M, N, K1, A1, lda1, K2, A2, lda2, B1, ldb1, B2, ldb2, C, ldc, bias, act, alpha, s);
        return;
    }
    gemm(M, N, K1, A1, lda1, B1, ldb1, C, ldc, nullptr, TG_ACT_NONE, 0.0f, mode, s);
    Scratch<float> T(static_cast<size_t>(M * N), s);
    gemm(M, N, K2, A2, lda2, B2, ldb2, T.p, N, nullptr, TG_ACT_NONE, 0.0f, mode, s);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(ceil_div(M * N, 256), 8 * num_sms()));
    launch("add_bias_act", add_bias_act_kernel, dim3(grid), dim3(256), 0, s, M, N, C, ldc, T.p, N, bias, act, alpha);
}

void gemm_dual_exact(int64_t M, int64_t N, int64_t K, const float* A1, int64_t lda1,
                     const float* A2, int64_t lda2, const float* B1, const float* B2, int64_t ldb,
                     float* C, int64_t ldc, const float* bias, int act, float alpha,
                     cudaStream_t s) {
    if (M == 0 || N == 0) return;
    GemmArgs g{M, N, K, A1, lda1, A2, lda2, B1, B2, ldb, C, ldc, bias, act, alpha, (N / 8) * 8};
    dispatch_gemm<true>(g, s);
}

}  // namespace tg

using namespace tg;

extern "C" {

TG_API tg_status tg_gemm_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                             const float* B, int64_t ldb, float* C, int64_t ldc,
                             const float* bias, int32_t act, float alpha, int32_t mode,
                             void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K < 0) invalid("matmul: negative size");
        check_ld("matmul", "A", lda, K);
        check_ld("matmul", "B", ldb, N);
        check_ld("matmul", "C", ldc, N);
        check_ptr("matmul", "A", A, M > 0 && K > 0);
        check_ptr("matmul", "B", B, K > 0 && N > 0);
        check_ptr("matmul", "C", C, M > 0 && N > 0);
        gemm(M, N, K, A, lda, B, ldb, C, ldc, bias, act, alpha, mode, as_stream(stream));
    });
}

TG_API tg_status tg_gemm_rowscale_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
                                      const float* B, int64_t ldb, float* C, int64_t ldc,
                                      const float* row_scale, const float* bias, int32_t act, float alpha,
                                      int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K < 0) invalid("matmul: negative size");
        check_ld("matmul", "A", lda, K);
        check_ld("matmul", "B", ldb, N);
        check_ld("matmul", "C", ldc, N);
        check_ptr("matmul", "A", A, M > 0 && K > 0);
        check_ptr("matmul", "B", B, K > 0 && N > 0);
        check_ptr("matmul", "C", C, M > 0 && N > 0);
        check_ptr("matmul", "row_scale", row_scale, M > 0 && N > 0);
        gemm_rowscale(M, N, K, A, lda, B, ldb, C, ldc, row_scale, bias, act, alpha, mode, as_stream(stream));
    });
}

TG_API tg_status tg_gemm_pair_f32(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* B1,
                                  const float* B2, int64_t ldb, float* C1, int64_t ldc1, float* C2, int64_t ldc2,
                                  int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K < 0) invalid("matmul: negative size");
        check_ld("matmul", "A", lda, K);
        check_ld("matmul", "B", ldb, N);
        check_ld("matmul", "C1", ldc1, N);
        check_ld("matmul", "C2", ldc2, N);
        check_ptr("matmul", "A", A, M > 0 && K > 0);
        check_ptr("matmul", "B1/B2", B1 && B2 ? B1 : nullptr, K > 0 && N > 0);
        check_ptr("matmul", "C1/C2", C1 && C2 ? C1 : nullptr, M > 0 && N > 0);
        gemm_pair(M, N, K, A, lda, B1, B2, ldb, C1, ldc1, C2, ldc2, mode, as_stream(stream));
    });
}

TG_API tg_status tg_gemm_cat_f32(int64_t M, int64_t N, int64_t K1, const float* A1, int64_t lda1, int64_t K2,
                                 const float* A2, int64_t lda2, const float* B1, int64_t ldb1, const float* B2,
                                 int64_t ldb2, float* C, int64_t ldc, const float* bias, int32_t act, float alpha,
                                 int32_t mode, void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K1 < 0 || K2 < 0) invalid("matmul: negative size");
        check_ld("matmul", "A1", lda1, K1);
        check_ld("matmul", "A2", lda2, K2);
        check_ld("matmul", "B1", ldb1, N);
        check_ld("matmul", "B2", ldb2, N);
        check_ld("matmul", "C", ldc, N);
        check_ptr("matmul", "A1/B1", A1 && B1 ? A1 : nullptr, M > 0 && K1 > 0 && N > 0);
        check_ptr("matmul", "A2/B2", A2 && B2 ? A2 : nullptr, M > 0 && K2 > 0 && N > 0);
        check_ptr("matmul", "C", C, M > 0 && N > 0);
        gemm_cat(M, N, K1, A1, lda1, K2, A2, lda2, B1, ldb1, B2, ldb2, C, ldc, bias, act, alpha, mode,
                 as_stream(stream));
    });
}

TG_API tg_status tg_take_device_error(void* stream) {
    return guard([&] {
        require_device();
        const int code = gemm_tc_take_error(as_stream(stream));
        const int gcode = gather_take_error(as_stream(stream));
        const int pcode = peer_take_error(as_stream(stream));
        if (code)
            fail(TG_ERR_TIMEOUT, "a tensor-core GEMM pipeline wait ran out (stage code " + std::to_string(code) +
                                     "); its output is invalid");
        if (gcode)
            fail(TG_ERR_TIMEOUT, "a heavy-row gather pipeline wait ran out (code " + std::to_string(gcode) +
                                     "); its output is invalid");
        if (pcode)
            fail(TG_ERR_TIMEOUT, "tg_wait_flags: flag " + std::to_string(pcode - 20) +
                                     " did not reach its target in time (a peer's tiles are missing)");
    });
}

TG_API tg_status tg_gemm_dual_f32(int64_t M, int64_t N, int64_t K, const float* A1,
                                  int64_t lda1, const float* A2, int64_t lda2,
                                  const float* B1, const float* B2, int64_t ldb, float* C,
                                  int64_t ldc, const float* bias, int32_t act, float alpha,
                                  void* stream) {
    return guard([&] {
        require_device();
        if (M < 0 || N < 0 || K < 0) invalid("gemm_dual: negative size");
        check_ld("gemm_dual", "A1", lda1, K);
        check_ld("gemm_dual", "A2", lda2, K);
        check_ld("gemm_dual", "B", ldb, N);
        check_ld("gemm_dual", "C", ldc, N);
        gemm_dual_exact(M, N, K, A1, lda1, A2, lda2, B1, B2, ldb, C, ldc, bias, act, alpha,
                        as_stream(stream));
    });
}

}  // extern "C"
