// api_internal.h -- context and weight objects behind the opaque handles of
// include/q35k.h (internal to libq35k).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace q35k {
struct GemvPeers;  // kernels.h
}

struct q35k_weight {
    int type = 0, n_in = 0, n_out = 0, nb = 0, n_pad = 0, device = 0;
    uint8_t* tiles = nullptr;  // 32-row chunk-major tiles (device_common.cuh)
    uint8_t* meta = nullptr;   // per-block GEMM metadata (gemm_tc.h)
    float* scale = nullptr;    // Q4_K / Q5_K: per-block drain scales of the exact GEMM
    size_t bytes = 0;
    bool fast_ok = true;       // every d and dmin finite: the fast mode may take it (launch_gemm_meta)
};

struct q35k_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::string err;

    // Device scratch, grown on demand and reused across calls.
    float* d_x = nullptr;
    size_t x_cap = 0;
    uint8_t* d_q8 = nullptr;  // planar Q8_K (the GEMV's input)
    size_t q8_cap = 0;
    uint8_t* d_q8raw = nullptr;  // BlockQ8K bytes (caller format)
    size_t q8raw_cap = 0;
    float* d_y = nullptr;
    size_t y_cap = 0;
    float* d_partial = nullptr;
    size_t partial_cap = 0;
    int* d_counters = nullptr;  // split-K arrival counters; zero between calls
    size_t counters_cap = 0;
    unsigned* d_err = nullptr;  // device error word (bounded waits that expired)
    unsigned* h_errw = nullptr;  // pinned host word the error word is read into at q35k_sync

    // Prefill GEMM scratch (gemm_tc.h): fp16 Q8_K operands, partial tiles and
    // arrival counters (zero between calls).
    void* d_xq = nullptr;
    size_t xq_cap = 0;
    void* d_xe = nullptr;
    size_t xe_cap = 0;
    float* d_xd = nullptr;
    size_t xd_cap = 0;
    float* d_gws = nullptr;
    size_t gws_cap = 0;
    int* d_gcnt = nullptr;
    size_t gcnt_cap = 0;
    unsigned* d_tmax = nullptr;  // fast-mode token maxima (zero between calls)
    size_t tmax_cap = 0;
    // Q4_K calls with at least this many tokens run on the tensor cores
    // (environment variable Q35K_GEMM_MIN_TOKENS overrides it at creation).
    int gemm_min_tokens = 16;
    // Q35K_GEMM_EXACT (default) or Q35K_GEMM_FAST (environment variable
    // Q35K_GEMM_MODE=fast at creation, or q35k_set_gemm_mode).
    int gemm_mode = 0;

    // Pinned host staging for the synchronous host-pointer calls.
    void* h_in = nullptr;
    size_t h_in_cap = 0;
    void* h_out = nullptr;
    size_t h_out_cap = 0;
    void* h_out_dev = nullptr;  // h_out's device address (mapped), set when h_out is allocated
    // While a host-pointer call runs: its mapped host error word, which the
    // GEMV launches of the call also set (GemvArgs::h_err); nullptr otherwise.
    unsigned* call_h_err = nullptr;

    ~q35k_ctx() {
        if (d_x) cudaFree(d_x);
        if (d_q8) cudaFree(d_q8);
        if (d_q8raw) cudaFree(d_q8raw);
        if (d_y) cudaFree(d_y);
        if (d_partial) cudaFree(d_partial);
        if (d_counters) cudaFree(d_counters);
        if (d_err) cudaFree(d_err);
        if (d_xq) cudaFree(d_xq);
        if (d_xe) cudaFree(d_xe);
        if (d_xd) cudaFree(d_xd);
        if (d_gws) cudaFree(d_gws);
        if (d_gcnt) cudaFree(d_gcnt);
        if (d_tmax) cudaFree(d_tmax);
        if (d_amax) cudaFree(d_amax);
        if (h_in) cudaFreeHost(h_in);
        if (h_out) cudaFreeHost(h_out);
        if (h_errw) cudaFreeHost(h_errw);
        if (stream) cudaStreamDestroy(stream);
    }

    int fail(int code, const char* fmt, ...);
    int cuda_fail(cudaError_t e, const char* what);
    int ensure_dev(void** p, size_t* cap, size_t bytes, bool zero);
    int ensure_host(void** p, size_t* cap, size_t bytes);
    int check_device_error();
    int on_device_error(unsigned word);
    // `pdl`: launch with programmatic stream serialization (the GEMV streams
    // weights before the preceding kernel finishes; its Q8_K reads wait).
    // `peers`: fused all-gather of a sharded decode call (kernels.h).
    // `argmax`: fused argmax keys per token (kernels.h); d_y may then be null.
    // `d_up`: quantize silu(x) * up (fused quantize or d_q8 == nullptr only).
    // `more_w` / `more_y`: n_more further weights of w's type and K in the
    // same launch, outputs [tokens][n_out] each (no peers or argmax then).
    int gemv(const q35k_weight* w, const uint8_t* d_q8, float* d_y, int tokens, cudaStream_t s, bool pdl = true,
             const float* d_x = nullptr, int ldy = 0, const q35k::GemvPeers* peers = nullptr,
             unsigned long long* argmax = nullptr, const float* d_up = nullptr,
             const q35k_weight* const* more_w = nullptr, float* const* more_y = nullptr, int n_more = 0);
    // Tensor-core prefill GEMM (Q4_K): quantize x (silu(x) * up with d_up),
    // then the GEMM.  prep == false: reuse the operands the previous call
    // prepared from the same x (same K and token count).
    int gemm(const q35k_weight* w, const float* d_x, float* d_y, int tokens, cudaStream_t s, int ldy = 0,
             const float* d_up = nullptr, bool prep = true);
    // Prefill calls that take the tensor-core GEMM: enough tokens and a type
    // the current mode supports (every K-quant type in both modes).
    bool uses_gemm(const q35k_weight* w, int tokens) const;
    bool gemm_fast(const q35k_weight* w) const;
    // Several weights of one K on one input (q35k_matmul_shared_dev).
    int matmul_shared(const q35k_weight* const* ws, int count, const float* d_x, float* const* d_ys, int tokens,
                      cudaStream_t s);
    // y[tokens][ldy] (columns below n_out) = x @ W^T on device pointers: the
    // dispatch behind q35k_matmul_dev (ldy = n_out) and the sharded calls.
    // With `peers` (sharded calls, fused all-gather) the call must take the
    // decode GEMV: tokens <= 8, else Q35K_ENOTSUP.
    // With `d_up` the input is silu(x) * up (q35k_matmul_silu_dev).
    int matmul_into(const q35k_weight* w, const float* d_x, float* d_y, int ldy, int tokens, cudaStream_t s,
                    const q35k::GemvPeers* peers = nullptr, unsigned long long* argmax = nullptr,
                    const float* d_up = nullptr);
    unsigned long long* d_amax = nullptr;  // fused-argmax keys
    size_t amax_cap = 0;
};
