// kernels.h -- host-side launchers of the libq35k kernels (internal to the
// library; the public surface is include/q35k.h).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace q35k {

// Q8_K quantization of rows x [rows][k]: BlockQ8K bytes (planar_chunk == 0)
// or the planar layout in chunks of planar_chunk rows.  The kernel lets a
// dependent kernel launched with programmatic stream serialization start
// early (that kernel must wait on the grid dependency before reading q8).
// With `up` (laid out like x) the rows quantized are silu(x) * up (ffn_down's
// input, QuantizeQ8Kx4.Quantize4x8Silu).
// Planar chunks of ilv_rows or more rows (ilv_rows > 0; see q8_interleave_min_rows)
// get the word-interleaved qs plane.
cudaError_t launch_quantize_q8k(const float* x, uint8_t* q8, int k, int rows, int planar_chunk, cudaStream_t s,
                                const float* up = nullptr, int ilv_rows = 0);

// BlockQ8K rows -> planar layout in chunks of `chunk` rows.
cudaError_t launch_q8k_to_planar(const uint8_t* src, uint8_t* dst, int k, int rows, int chunk, cudaStream_t s,
                                 int ilv_rows);

// Bit-exact dequantization of `rows` GGUF rows of k values.
cudaError_t launch_dequantize(int type, const uint8_t* blocks, float* y, int k, int rows, cudaStream_t s);

// GGUF rows -> 32-row chunk-major tiles (layout in device_common.cuh).
cudaError_t launch_repack_tiles(int type, const uint8_t* rows_src, uint8_t* tiles, int nb, int n_out,
                                int n_pad, cudaStream_t s);

// Fused all-gather of a row-sharded decode call (csrc/shard.cu): besides its
// own y, the GEMV stores every output value into each peer's gather area
// (NVLink stores through IPC or peer pointers), at [token][row] with row
// stride ldp, as one 64-bit word (call number << 32 | value bits).  Each
// buffer holds two areas used on alternate calls: the call's number is
// *seq + 1 and its area (*seq + 1) & 1, where *seq counts this rank's
// completed fused calls (device memory, advanced by the gather kernel that
// follows the GEMV; read after the GEMV's grid-dependency wait).  n == 0: off.
constexpr int GEMV_MAX_PEERS = 7;
struct GemvPeers {
    unsigned long long* y[GEMV_MAX_PEERS];  // this rank's slice in peer k's gather area 0
    int n, ldp;
    size_t half;               // words from gather area 0 to area 1
    const unsigned* seq;
    // Optional phase timestamps of the call (%globaltimer, ns): [0] first CTA
    // start (atomicMin), [1] last CTA end (atomicMax); nullptr: off.
    unsigned long long* trace;
};

// Further weights of the same type and K sharing one launch and one set of
// activations (q/k/v, gate/up): matrix k's row groups start at row group
// g0[k] of the launch; its outputs go to y[k] with row stride ldy[k].
constexpr int GEMV_MAX_MATS = 4;
struct GemvMats {
    const uint8_t* tiles[GEMV_MAX_MATS - 1];
    float* y[GEMV_MAX_MATS - 1];
    int n_out[GEMV_MAX_MATS - 1], ldy[GEMV_MAX_MATS - 1], g0[GEMV_MAX_MATS - 1];
    int n;  // 0: one weight
};

struct GemvArgs {
    const uint8_t* tiles;  // uploaded weight tiles
    const uint8_t* q8;     // planar Q8_K of `tokens` rows (16-byte aligned), or
    const float* x;        // fp32 activations [tokens][ldx] to quantize in the
    int ldx;               //   GEMV itself (x != nullptr; see gemv_fuses_quantize)
    float* y;              // [tokens][ldy]
    int ldy;
    int n_out, nb, tokens;
    float* partial;     // pieces of row groups cut by a CTA boundary
    int* counters;      // one arrival counter per row group, zero between calls
    unsigned* err;      // device error word
    // Host-pointer calls: a word in mapped host memory that a CTA whose
    // bounded wait expired also sets (plain store), so the caller learns of it
    // after synchronizing without reading the device word back; nullptr: off.
    unsigned* h_err;
    int num_sms;
    GemvPeers peers;    // fused all-gather (peers.n == 0: off)
    // Fused argmax (vocab head): per token the 64-bit max of argmax_key(logit,
    // row) over all rows, combined with atomicMax; nullptr: off.  y may then
    // be nullptr (logits not written).
    unsigned long long* argmax;
    // ffn_down's input (fused quantize only): the GEMV quantizes silu(x) * up,
    // up laid out like x; nullptr: x itself.
    const float* up;
    GemvMats more;  // more weights in this launch (peers and argmax: one weight only)
};
// Row count the launch plans for: every matrix's rows, each padded to 32.
int gemv_plan_rows(const GemvArgs& a);

// Launch plan of the GEMV: one CTA per (row group, run of unit_blocks
// super-blocks); deterministic in (type, nb, n_out, tokens, sms).
// `partial_bytes` / `counters` size the split-K scratch it needs.
struct GemvPlan {
    int groups, n_pad, grid, splits, unit_blocks, warps, threads;
    // > 1: the splits of a row group form one thread-block cluster of this
    // size and are summed through distributed shared memory; 0: through the
    // partial-sum buffer and the arrival counters in global memory.
    int cluster;
    size_t smem_bytes, partial_bytes, counters;
    bool fits;
    // Run the kernel variant bounded at three 10-warp CTAs per SM (more
    // registers per thread): one or two tokens, at most 10 warps, and three
    // CTAs per SM already the limit (shared memory) or enough for the grid.
    bool three_per_sm;
};
GemvPlan plan_gemv(int type, int nb, int n_out, int tokens, int num_sms);
// Largest token count per GEMV launch for nb super-blocks per row (0: the
// row is too long to stage one token's activations).
int gemv_max_tokens(int nb);
cudaError_t launch_gemv(int type, const GemvArgs& a, cudaStream_t s, bool pdl);
// idx[t] = the row of keys[t] (fused argmax, see GemvArgs::argmax).
cudaError_t launch_argmax_index(unsigned long long* keys, int* idx, int tokens, cudaStream_t s);
// Whether the GEMV for this shape quantizes its own activations (small
// slices per CTA: decode) instead of reading planar Q8_K.
bool gemv_fuses_quantize(int type, int nb, int n_out, int tokens, int num_sms);

}  // namespace q35k
