// ============================================================================
//  tinygnn_b200/csrc/common.cuh -- shared helpers for the sm_100a kernels and
//  the C-ABI layer: error capture, activation functors, launch geometry.
// ============================================================================
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "tinygnn_b200.h"

namespace tg {

// ── Errors ──────────────────────────────────────────────────────────────────
// Internal code throws tg::Error; every extern "C" entry point converts it to
// a tg_status and stores the message for tg_last_error_message().
struct Error : std::runtime_error {
    tg_status status;
    Error(tg_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(tg_status s, const std::string& m) { throw Error(s, m); }
[[noreturn]] inline void invalid(const std::string& m) { fail(TG_ERR_INVALID_ARGUMENT, m); }

void set_last_error(const std::string& m);

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        fail(TG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                              cudaGetErrorString(e) + ")");
}
#define TG_CUDA(call) ::tg::cuda_check((call), #call)
#define TG_LAUNCH_CHECK(name) ::tg::cuda_check(cudaGetLastError(), name)

// Runs f and maps any exception to a status (the C-ABI boundary).
template <class F>
tg_status guard(F&& f) noexcept {
    try {
        f();
        return TG_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.status;
    } catch (const std::invalid_argument& e) {
        set_last_error(e.what());
        return TG_ERR_INVALID_ARGUMENT;
    } catch (const std::out_of_range& e) {
        set_last_error(e.what());
        return TG_ERR_OUT_OF_RANGE;
    } catch (const std::bad_alloc&) {
        set_last_error("out of host memory");
        return TG_ERR_RUNTIME;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return TG_ERR_RUNTIME;
    } catch (...) {
        set_last_error("unknown error");
        return TG_ERR_RUNTIME;
    }
}

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// ── Input CSR checks ─────────────────────────────────────────────────────
// Tensor::sparse_csr's checks (src/tensor.cpp:46-86) on device arrays --
// row_ptr non-decreasing, row_ptr[rows] == nnz, every column in [0, cols) --
// plus row_ptr[0] >= 0 (with the others, every row lies inside col_ind) and,
// when given, every row_order entry in [0, rows).  cols < 0: the columns are
// only compared, never used as addresses (no range check); nnz < 0: nnz is
// row_ptr[rows].  Throws invalid_argument with the reference's message.
// `words` (nullable) is device memory for the result (sizeof 32 bytes);
// without it the result goes to pool scratch.  Synchronises `s`.
void csr_validate(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp, const int32_t* ci, cudaStream_t s,
                  const int32_t* order = nullptr, void* words = nullptr);
constexpr size_t kCsrCheckWordsBytes = 32;

// The calling thread's tg_set_csr_checks setting (on unless turned off).
bool csr_checks_enabled();

// What every entry point that reads a caller's CSR runs first: the checks
// above, unless the caller turned them off for this thread.
inline void check_csr_input(int64_t rows, int64_t cols, int64_t nnz, const int32_t* rp, const int32_t* ci,
                            cudaStream_t s, const int32_t* order = nullptr, void* words = nullptr) {
    if (csr_checks_enabled() && (rows > 0 || nnz > 0)) csr_validate(rows, cols, nnz, rp, ci, s, order, words);
}

// Number of SMs of the current device (cached per device).
int num_sms();

// ── Peer outputs of a fused GEMM -> exchange ─────────────────────────────
// Up to kMaxPeers other GPUs' copies of an output (same offsets and leading
// dimension, mapped into this process), and for each of them the address of
// this rank's completion counter in that GPU's memory.
constexpr int kMaxPeers = 7;
struct PeerOut {
    float* c[kMaxPeers] = {};
    unsigned long long* flag[kMaxPeers] = {};
    int n = 0;
};

// ── Side stream ──────────────────────────────────────────────────────────
// A high-priority stream per (host thread, device) with two events, for
// kernels that run beside the caller's stream inside one call: record `fork`
// on the caller's stream, make the side stream wait for it, launch there,
// record `join`, and make the caller's stream wait for `join` before it
// continues -- the call stays ordered on the caller's stream (and captures
// into a CUDA graph as a fork/join).
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
SideStream& side_stream();

// ── Stream-ordered scratch ────────────────────────────────────────────────
// Scratch buffers come from the device's default memory pool with a high
// release threshold, so repeated calls reuse the same pages.
void* scratch_alloc(size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

template <class T>
struct Scratch {
    T* p = nullptr;
    cudaStream_t s = nullptr;
    Scratch(size_t n, cudaStream_t st) : s(st) {
        p = static_cast<T*>(scratch_alloc((n ? n : 1) * sizeof(T), st));
    }
    ~Scratch() {
        if (p) scratch_free(p, s);
    }
    Scratch(const Scratch&) = delete;
    Scratch& operator=(const Scratch&) = delete;
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ── Activations (reference src/ops.cpp:328-482) ──────────────────────────
// Device versions of the in-place activations; relu/leaky/elu/sigmoid keep the
// reference's branch structure so their results match it exactly apart from
// the last bits of exp/tanh.
__device__ __forceinline__ float apply_act(int act, float x, float alpha) {
    switch (act) {
        case TG_ACT_RELU:
            return x > 0.0f ? x : 0.0f;  // std::max(0.0f, x)
        case TG_ACT_LEAKY_RELU:
            return x >= 0.0f ? x : __fmul_rn(alpha, x);
        case TG_ACT_ELU:
            return x < 0.0f ? __fmul_rn(alpha, __fsub_rn(expf(x), 1.0f)) : x;
        case TG_ACT_SIGMOID:
            if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
            else {
                const float ex = expf(x);
                return __fdiv_rn(ex, __fadd_rn(1.0f, ex));
            }
        case TG_ACT_TANH:
            return tanhf(x);
        case TG_ACT_GELU: {
            const float inner = __fmul_rn(0.7978845608f, fmaf(__fmul_rn(__fmul_rn(0.044715f, x), x), x, x));
            return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
        }
        default:
            return x;
    }
}

// The activation of V values, the choice made once for all of them: an
// epilogue that called apply_act per element paid its switch (and the code
// of every activation) per value -- ~2k cycles per 16 columns in the
// tensor-core GEMM's epilogue.
template <int V>
__device__ __forceinline__ void act_v(float (&v)[V], int act, float alpha) {
    if (act == TG_ACT_NONE) return;
    if (act == TG_ACT_RELU) {
#pragma unroll
        for (int j = 0; j < V; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;  // apply_act's ReLU
        return;
    }
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = apply_act(act, v[j], alpha);
}

}  // namespace tg
