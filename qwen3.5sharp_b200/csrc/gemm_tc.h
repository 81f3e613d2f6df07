// gemm_tc.h -- host interface of the tensor-core prefill GEMM (gemm_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace q35k {

struct TcGemmArgs {
    const uint8_t* tiles;  // uploaded weight tiles (32-row chunk-major layout)
    const uint8_t* meta;   // their GEMM metadata (launch_gemm_meta)
    const float* scale;    // the drain scale s of every (row, super-block), then the
                           // fast mode's row scales [n_pad]
    const float* xd;       // exact: Q8_K block scales [nb][m_pad]; fast: token scales [m_pad]
    float* y;              // [tokens][ldy], columns below n_out written
    int ldy;
    float* ws;             // partial tiles: [grid][2][tn tokens][128 rows]
    int* counters;         // [tiles][8][tn / 128] arrival counters, zero between launches
    unsigned* err;         // device error word
    int n_out, n_pad, tokens, m_pad, nb, tiles_t, grid;
    long long units;       // tiles * nb
    int tn;                // tokens per tile: 128, or 256 (fast mode, 256+ tokens)
    int type;              // TYPE_Q4_K, TYPE_Q5_K or TYPE_Q6_K
};

struct TcGemmPlan {
    int tn, m_pad, tiles_w, tiles_t, tiles, grid;
    long long units;
    size_t xq_bytes, xe_bytes, xd_bytes, ws_bytes, counters;
};

// Tokens per tile: 256 for fast-mode calls of at least 512 tokens (twice the
// work per MMA instruction and per dequantized weight tile; fewer tokens would
// leave too few tiles to share among the SMs), else 128.
int tc_gemm_tile_tokens(bool fast, int tokens);
TcGemmPlan plan_tc_gemm(int nb, int n_pad, int tokens, int num_sms, int tn);
// GEMM metadata of an uploaded weight: sizes and the kernels that fill it
// (the exact mode's drain scales, the fast mode's fp16 weight scales and its
// per-row normalisation 2^-e).  *unsafe (zeroed by the caller) is set when a
// block's d or dmin is not finite: such a weight's prefill keeps the exact
// arithmetic in the fast mode.
size_t gemm_meta_bytes(int type, int nb, int n_pad);
size_t gemm_scale_bytes(int type, int nb, int n_pad);
cudaError_t launch_gemm_meta(int type, const uint8_t* tiles, uint8_t* meta, float* scale, int nb, int n_pad,
                             unsigned* unsafe, cudaStream_t s);
// Whether the tensor-core GEMM takes this weight type in this mode: Q4_K,
// Q5_K and Q6_K in both modes (Q6_K's exact products sc * (q - 32) as two
// exact fp16 parts, two MMAs per K step).
bool tc_gemm_supports(int type, bool fast);
cudaError_t configure_tc_gemm();
// Q8_K quantization of x [tokens][k] into the GEMM's operands.  Exact mode:
// Xq [tokens][k] fp16 q values, Xe [tokens][k/256*16] fp16 block sums,
// Xd [k/256][m_pad] d.  Fast mode: Xq = fp16(2^e_t d q) with one power of two
// per token (1 for a token whose largest |x| is in [2^-4, 2^15), else the one
// that puts it in [2^13, 2^14)), Xd [m_pad] = 2^-e_t; tmax [tokens] is zero
// before and after the launches.  With `up` the rows quantized are
// silu(x) * up (ffn_down's input).
cudaError_t launch_gemm_prep(const float* x, int k, int tokens, int m_pad, void* xq, void* xe, float* xd,
                             unsigned* tmax, bool fast, cudaStream_t s, const float* up = nullptr);
// The GEMM; `pdl` lets it start while the preparation kernel finishes.
// Exact mode forms the reference's integer dots and scales them per
// super-block; fast mode multiplies fp16-rounded dequantized weights and
// activations with one fp32 accumulator per tile.
cudaError_t launch_tc_gemm(const TcGemmArgs& args, const void* xq, const void* xe, int k, bool fast, cudaStream_t s,
                           bool pdl);

}  // namespace q35k
