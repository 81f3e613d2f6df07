// gemm_tc.cu -- prefill GEMM for Q4_K weights on the sm_100a tensor cores
// (tcgen05.mma, TMEM accumulators, tensor TMA).  Replaces the reference's
// Q4_K panel GEMM (Kernels/MulMatQ4K.cs:45-209, Kernels/GemmQ4K.cs:25-160,
// Kernels/GemmQ4K.Avx2.cs:39-217) for tokens >= the dispatch threshold.
//
// Arithmetic (the reference's, kept exact):
//   y[r][c] = sum_b (fp16(d_cb) * d8_rb) * S_b[r][c] - (fp16(dmin_cb) * d8_rb) * Mn_b[r][c]
// with S_b = sum_k q8[r][k] * sc_j(k) * q4[c][k] and Mn_b = sum_j m_j * bsum_j,
// both exact integers.  On the tensor cores:
//   * the activations are quantized to Q8_K exactly as the reference does
//     (warp_q8k_values); their q values, exact small integers, become the fp16
//     B operand Xq[r][k], and the 16 block sums of each super-block the fp16
//     operand Xe[r][16b + i];
//   * the weights become the fp16 A operand in TMEM: alpha * sc_j * q4 (exact:
//     at most 945 * 2^-e) for the 256 values of a super-block, plus 16 columns
//     beta * -m_{i/2} split into an fp16 high part and an fp16 low part
//     (hi + lo carries the fp32 product to ~2^-22), multiplied against Xe;
//   * with s = d / alpha and beta = dmin / s this gives, per super-block, one
//     fp32 accumulator  T_b = (d * S_b - dmin * Mn_b) / s ; the drain warps
//     read it from TMEM and add (d8_rb * s) * T_b into registers.
//   So every product of the reference is formed from exact integers and the
//   only differences are fp32 rounding (observed ~3e-7 of max |y|).
//   alpha = 2^-e with e chosen so that |beta * 63| <= 32768 (fp16 range);
//   a block with d == 0, or dmin/d beyond 2^23, uses s = dmin and scales the
//   weight values by d/dmin instead (fp16-rounded; such blocks carry no
//   measurable weight).
//
// Work decomposition: tiles of 128 weight rows (TMEM lanes, MMA M) x 128
// tokens (MMA N).  A unit is one (tile, super-block) pair; the persistent grid
// splits the units into equal contiguous ranges (stream-K), so every SM gets
// the same number of MMAs.  A tile cut by a range boundary is finished by
// whichever covering CTA arrives last (per drain warp, via a counter), which
// adds the pieces in CTA order: results are bit-identical run to run.
//
// Warp roles (640 threads, one CTA per SM):
//   warp 0      TMA: Xq, half a super-block (2 boxes of 64 K x 128 tokens,
//               128-byte swizzle) per stage
//   warp 1      TMEM allocation and the MMA issue (one thread)
//   warp 2      bulk copies: weight tiles + metadata + Xe (16 x 128, 32-byte
//               swizzle) per unit; the drain scales per unit
//   warps 4-11  weight producers, two groups: group h builds the A operand
//               of half h of every super-block (64 value columns in TMEM,
//               the 16-column min term in shared memory)
//   warps 12-19 drains: per super-block, accumulator -> registers, scaled by
//               the Q8_K and weight scales; then the tile's output
// TMEM: accumulators at columns 0 and 128 (double-buffered per super-block),
// A buffers of 64 value columns at 256 + 64 i.  Every mbarrier wait is bounded in time; on expiry
// the CTA sets the device error word, stops issuing work, waits (bounded) for
// its own copies and MMAs in flight, frees TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "device_common.cuh"
#include "gemm_tc.h"
#include "q8k_quant.cuh"
#include "tc_common.cuh"

namespace q35k {
namespace tcg {

constexpr int TM = 128;  // weight rows per tile
constexpr int Q4K_META_TILE = 5 * 512;  // GEMM metadata of one 32-row tile
// Uploaded 32-row tile and its GEMM metadata per weight type.  Q5_K shares
// Q4_K's header and so its metadata; Q6_K (fast mode only) keeps d * sc_s of
// its sixteen 16-value groups, two 512-byte chunks.
template <int TYPE> struct WFmt {
    static constexpr int TILE_BYTES = 32 * (TYPE == TYPE_Q4_K ? 144 : TYPE == TYPE_Q5_K ? 176 : 210);
    static constexpr int META_TILE = TYPE == TYPE_Q6_K ? 2 * 512 : 5 * 512;
};
constexpr int TN = 128;  // tokens per tile
// Five warpgroups of four warps; each warpgroup re-sizes its registers with
// setmaxnreg.  Registers are split between an SM's four sub-partitions, one
// warp of every warpgroup in each: 5 x 32 x 96 = 15360 <= 16384 at launch,
// and afterwards 128 x (ctrl + 2 prod + 2 drain) = 61440 = 640 x 96.  The
// exact mode's drain holds more state (per-super-block scaling), the fast
// mode's producers more (the fp16 dequantization): each split is the one
// ptxas fits without spills.
constexpr int THREADS = 640;
constexpr int LAUNCH_REGS = 96;
template <bool FAST, int TYPE = TYPE_Q4_K> struct RegSplit {
    // Q6_K's producers hold the most raw words (ql, qh, scales): 80 in both modes.
    static constexpr bool WIDE_PROD = FAST || TYPE == TYPE_Q6_K;
    static constexpr int CTRL = 32, PROD = WIDE_PROD ? 80 : 72, DRAIN = WIDE_PROD ? 144 : 152;
    static_assert(CTRL + 2 * PROD + 2 * DRAIN == 5 * LAUNCH_REGS, "split must use the launch registers exactly");
};
// Activation halves h = 0, 1 of every unit are loaded by warps WARP_TMA and
// WARP_TMA2: a warp that issues a TMA copy and then touches shared memory
// (its next barrier wait) stalls until that copy has landed, so one loader
// warp keeps one stage in flight at a time and two loaders double the rate.
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_WTMA = 2, WARP_TMA2 = 3, WARP_PROD0 = 4, WARP_DRAIN0 = 12, NUM_DRAIN = 8;
// Activation ring: half super-blocks (128 K x 128 tokens fp16 = two
// 128-byte-swizzled boxes of 64 K), released by the MMA.
constexpr int X_STAGES = 3;
constexpr int X_BOX_BYTES = 64 * 2 * TN;           // 16 KB
constexpr int X_STAGE_BYTES = 2 * X_BOX_BYTES;     // 32 KB
// Weight ring, one stage per unit: the unit's block-sum operand Xe (16 x 128
// fp16, 32-byte swizzle), the four 32-row weight tiles (4 x 4608 B) and their
// GEMM metadata (4 x 1536 B).  Released by the producers and the MMA.
constexpr int W_STAGES = 3;
constexpr int Q4K_TILE = 32 * 144;                 // one 32-row tile of the uploaded layout
constexpr int EXT_BOX_BYTES = 16 * 2 * TN;         // 4096
constexpr int W_EXT_OFF = 0;                       // 1024-aligned (swizzled TMA destination)
constexpr int W_TILE_OFF = EXT_BOX_BYTES;
constexpr int W_META_OFF = W_TILE_OFF + 4 * Q4K_TILE;
constexpr int W_STAGE_BYTES = W_META_OFF + 4 * Q4K_META_TILE;  // 32768 (32 KB)
static_assert(W_STAGE_BYTES % 1024 == 0, "weight stage alignment");
// Drain ring, one stage per unit: the drain scales s of the 128 rows and the
// 128 token scales d8.  Released by the drains.
constexpr int D_STAGES = 4;
constexpr int D_STAGE_BYTES = 2 * 128 * 4;
// A operand: 4 TMEM buffers of 64 value columns (one half super-block each;
// buffers 2 p + h belong to producer group h) and, for the min term, 4 shared
// memory tiles of 128 rows x 16 fp16 (32-byte swizzle, read by a
// shared-memory MMA).
constexpr int A_BUFS = 4;
constexpr int E_TILE_BYTES = 128 * 32;
constexpr int X_RING_BYTES = X_STAGES * X_STAGE_BYTES;
constexpr int W_RING_BYTES = W_STAGES * W_STAGE_BYTES;
constexpr int E_RING_BYTES = A_BUFS * E_TILE_BYTES;
constexpr int D_RING_BYTES = D_STAGES * D_STAGE_BYTES;
// TMEM: accumulators at columns 0 and 128; A buffers at 256 + 64 i.
constexpr int A_COL0 = 256;
constexpr int TMEM_COLS = 512;
constexpr int NUM_BARS = 2 * X_STAGES + 3 * W_STAGES + 2 * D_STAGES + 2 * A_BUFS + 4 + 1;
constexpr int BAR_BYTES = 512;
constexpr size_t SMEM_BYTES =
    1024 + (size_t)X_RING_BYTES + W_RING_BYTES + E_RING_BYTES + D_RING_BYTES + BAR_BYTES;
static_assert(NUM_BARS * 8 + 8 <= BAR_BYTES, "barrier area");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

// Geometry of one kernel instance.  TN = 128 (both modes) is the layout
// above.  TN = 256 (fast mode, 512 or more tokens): each MMA covers 256
// tokens, so every A operand the producers build and every control step of
// the MMA thread serves twice the work.  Its activation halves are 64 KB (two
// boxes of 64 K x 256 tokens), two stages; two weight stages without the Xe
// tile; one 256-column accumulator (the A buffers keep columns 256..511), so
// the next tile segment starts once the drains have read the last one.
// Q6_K in the exact mode: its products sc * (q - 32) need up to 12
// significant bits, so each half super-block's A operand is two exact fp16
// parts, sl * (q - 32) and 16 sh * (q - 32) with sc = 16 sh + sl (sl in
// [0, 15]), of 64 columns each, multiplied against the same activations and
// summed in the accumulator: two MMAs per K step, no min term (the -32 is
// applied to q itself).  Two A buffers of 128 columns then hold one unit.
template <bool FAST, int TNX, int TYPE = TYPE_Q4_K> struct Geo {
    static_assert(TNX == 128 || (FAST && TNX == 256), "tile width");
    static constexpr bool Q6X = TYPE == TYPE_Q6_K && !FAST;
    static constexpr bool MIN_TERM = !FAST && TYPE != TYPE_Q6_K;  // the exact mins MMA against Xe
    static constexpr int TILE_BYTES = WFmt<TYPE>::TILE_BYTES, META_TILE = WFmt<TYPE>::META_TILE;
    static constexpr int TN = TNX;
    static constexpr int X_STAGES = TNX == 128 ? 3 : 2;
    static constexpr int X_BOX_BYTES = 64 * 2 * TN;
    static constexpr int X_STAGE_BYTES = 2 * X_BOX_BYTES;
    // Fills on one activation barrier (x_full[f & 1][f % X_STAGES]) recur
    // every lcm(2, X_STAGES) fills.
    static constexpr int X_PHASE_FILLS = X_STAGES % 2 ? 2 * X_STAGES : X_STAGES;
    static constexpr int W_STAGES = TNX == 128 ? 3 : 2;
    static constexpr int EXT_BOX_BYTES = (TNX == 128 && !Q6X) ? 16 * 2 * TN : 0;
    static constexpr int W_EXT_OFF = 0;
    static constexpr int W_TILE_OFF = EXT_BOX_BYTES;
    static constexpr int W_META_OFF = W_TILE_OFF + 4 * TILE_BYTES;
    static constexpr int W_STAGE_BYTES = (W_META_OFF + 4 * META_TILE + 1023) / 1024 * 1024;
    static constexpr int D_STAGES = 4;
    static constexpr int D_STAGE_BYTES = 2 * 128 * 4;
    static constexpr int A_BUFS = Q6X ? 2 : 4;
    static constexpr int A_COLS = Q6X ? 128 : 64;  // TMEM columns of one A buffer
    static constexpr int E_TILE_BYTES = 128 * 32;
    static constexpr int X_RING_BYTES = X_STAGES * X_STAGE_BYTES;
    static constexpr int W_RING_BYTES = W_STAGES * W_STAGE_BYTES;
    static constexpr int E_RING_BYTES = (TNX == 128 && !Q6X) ? A_BUFS * E_TILE_BYTES : 0;
    static constexpr int D_RING_BYTES = TNX == 128 ? D_STAGES * D_STAGE_BYTES : 0;
    static constexpr int ACC_BUFS = 256 / TN;  // accumulators at columns 0 (and 128)
    static constexpr int A_COL0 = 256;
    static constexpr int TMEM_COLS = 512;
    static constexpr int PASSES = TN / 128;    // 64-token passes of one drain warp
    static constexpr int NUM_BARS = 3 * X_STAGES + 3 * W_STAGES + 2 * D_STAGES + 2 * A_BUFS + 4 + 1;
    static constexpr size_t SMEM_BYTES =
        1024 + (size_t)X_RING_BYTES + W_RING_BYTES + E_RING_BYTES + D_RING_BYTES + BAR_BYTES;
    static_assert(NUM_BARS * 8 + 8 <= BAR_BYTES, "barrier area");
    static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
    static_assert(W_STAGE_BYTES % 1024 == 0 && X_BOX_BYTES % 1024 == 0, "stage alignment");
};
static_assert(Geo<false, 128>::SMEM_BYTES == SMEM_BYTES && Geo<false, 128>::W_STAGE_BYTES == W_STAGE_BYTES,
              "TN = 128 keeps the layout above");

}  // namespace tcg

// ---------------------------------------------------------------------------
// Activation preparation: Q8_K quantization (bit-exact) -> fp16 Xq, Xe and the
// block scales d8 in Xd[b][m_pad] (zero for padded tokens).  One warp per
// (token, super-block).  Xq holds each aligned group of four K values in the
// order 0, 2, 1, 3; the MMA's K order only has to agree between its operands.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_xq_group(__half* row, int lane, const __half (&h)[8]) {
    const __half2 p0 = __halves2half2(h[0], h[2]);
    const __half2 p1 = __halves2half2(h[1], h[3]);
    const __half2 p2 = __halves2half2(h[4], h[6]);
    const __half2 p3 = __halves2half2(h[5], h[7]);
    uint2 v0, v1;
    v0.x = *reinterpret_cast<const uint32_t*>(&p0);
    v0.y = *reinterpret_cast<const uint32_t*>(&p1);
    v1.x = *reinterpret_cast<const uint32_t*>(&p2);
    v1.y = *reinterpret_cast<const uint32_t*>(&p3);
    reinterpret_cast<uint2*>(row)[lane] = v0;        // values 4l..4l+3
    reinterpret_cast<uint2*>(row + 128)[lane] = v1;  // values 128+4l..
}

__global__ void __launch_bounds__(256) gemm_prep_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                                       int k, int tokens, int m_pad, __half* __restrict__ xq,
                                                       __half* __restrict__ xe, float* __restrict__ xd) {
    griddep_launch_dependents();
    const int nb = k / QK;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= m_pad * nb) return;
    const int r = w / nb, b = w % nb;
    if (r >= tokens) {
        if (lane == 0) xd[(size_t)b * m_pad + r] = 0.f;
        return;
    }
    int q[8];
    const size_t off = (size_t)r * k + (size_t)b * QK;
    const float d = warp_q8k_values(x + off, lane, q, up ? up + off : nullptr);
    // The q values (exact small integers), in the K order of the weight
    // producers' nibble pairs.
    __half h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __int2half_rn(q[i]);
    store_xq_group(xq + (size_t)r * k + (size_t)b * QK, lane, h);
    int s0, s1;
    warp_q8k_bsums(pack_q4(q[0], q[1], q[2], q[3]), pack_q4(q[4], q[5], q[6], q[7]), s0, s1);
    if ((lane & 3) == 0) {
        __half* e = xe + (size_t)r * nb * 16 + (size_t)b * 16;
        e[lane >> 2] = __int2half_rn(s0);
        e[8 + (lane >> 2)] = __int2half_rn(s1);
    }
    if (lane == 0) xd[(size_t)b * m_pad + r] = d;
}

// Fast mode: Xq = fp16(2^e d q), the Q8_K-dequantized activations of a token
// times a power of two, and Xs[token] = 2^-e, which the GEMM's drain
// multiplies its outputs by (exact).  A token whose largest |x| lies in
// [2^FAST_TOKEN_LO, 2^FAST_TOKEN_HI) keeps e = 0: its fp16 values cannot
// overflow, and those that fall into the fp16 subnormals carry errors below
// 2^-21 of the token's largest value.  Any other token gets the e that puts
// its largest |x| in [2^13, 2^14).
constexpr int FAST_TOKEN_EXP = 14, FAST_TOKEN_LO = -4, FAST_TOKEN_HI = 15;

__device__ __forceinline__ int fast_token_exp(float tm) {
    int E = 0;
    if (tm > 0.f && isfinite(tm)) frexpf(tm, &E);
    // At most 120, so that 2^e and 2^-e stay normal floats (e >= -114 for
    // any finite maximum).
    return (E == 0 || (E > FAST_TOKEN_LO && E <= FAST_TOKEN_HI)) ? 0 : min(FAST_TOKEN_EXP - E, 120);
}

__device__ __forceinline__ void fast_quantize_store(const float (&v)[8], int lane, float scale,
                                                    __half* __restrict__ dst) {
    int q[8];
    const float d = warp_q8k_quantize(v, lane, q) * scale;
    __half h[8];
#pragma unroll
    for (int j = 0; j < 8; j++) h[j] = __float2half_rn(d * (float)q[j]);
    store_xq_group(dst, lane, h);
}

__device__ __forceinline__ float warp_abs_max(const float (&v)[8]) {
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) m = fmaxf(m, fabsf(v[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

// Two kernels: gemm_prep_fast_kernel, one warp per (token, super-block),
// stores the block with e = 0 and records its max |x| in tmax[token] (float
// bits, atomic max); gemm_token_scale_kernel, its programmatic dependent,
// writes Xs, clears tmax for the next call, and rewrites the rows of the
// tokens outside the range.  (A token's maximum is known only once all its
// blocks are read; storing with e = 0 first costs the common case nothing.)
__global__ void __launch_bounds__(256) gemm_prep_fast_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                                            int k, int tokens, __half* __restrict__ xq,
                                                            unsigned* __restrict__ tmax) {
    griddep_launch_dependents();
    const int nb = k / QK;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= tokens * nb) return;
    const int r = w / nb, b = w % nb;
    const size_t off = (size_t)r * k + (size_t)b * QK;
    float v[8];
    warp_q8k_load(x + off, lane, v, up ? up + off : nullptr);
    fast_quantize_store(v, lane, 1.f, xq + off);
    const float m = warp_abs_max(v);
    if (lane == 0) atomicMax(tmax + r, __float_as_uint(m));  // m >= 0: the bits order as the values
}

// FAST_SCALE_TOKENS tokens per CTA: few CTAs, so that while they wait for
// the preparation kernel they keep few SMs from the GEMM that follows.
constexpr int FAST_SCALE_TOKENS = 64;

__global__ void __launch_bounds__(256) gemm_token_scale_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ up, int k, int tokens,
                                                              int m_pad, __half* __restrict__ xq,
                                                              float* __restrict__ xs, unsigned* __restrict__ tmax) {
    griddep_launch_dependents();
    __shared__ int rescale[FAST_SCALE_TOKENS];
    __shared__ float scales[FAST_SCALE_TOKENS];
    __shared__ int n_rescale;
    const int r0 = blockIdx.x * FAST_SCALE_TOKENS;
    if (threadIdx.x == 0) n_rescale = 0;
    griddep_wait();  // the maxima and the e = 0 rows
    __syncthreads();
    if (threadIdx.x < FAST_SCALE_TOKENS && r0 + (int)threadIdx.x < m_pad) {
        const int r = r0 + threadIdx.x;
        if (r >= tokens) {
            xs[r] = 0.f;  // padded token
        } else {
            const float tm = __uint_as_float(tmax[r]);
            tmax[r] = 0u;
            const int e = fast_token_exp(tm);
            xs[r] = ldexpf(1.f, -e);
            if (e) {
                const int i = atomicAdd(&n_rescale, 1);
                rescale[i] = r;
                scales[i] = ldexpf(1.f, e);
            }
        }
    }
    __syncthreads();
    // Rows outside the range, one (token, super-block) per warp at a time.
    const int nb = k / QK, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int u = warp; u < n_rescale * nb; u += blockDim.x >> 5) {
        const int i = u / nb, b = u % nb;
        const size_t off = (size_t)rescale[i] * k + (size_t)b * QK;
        float v[8];
        warp_q8k_load(x + off, lane, v, up ? up + off : nullptr);
        fast_quantize_store(v, lane, scales[i], xq + off);
    }
}

// ---------------------------------------------------------------------------
// Device pieces of the GEMM.
// ---------------------------------------------------------------------------
namespace {

struct BlockScale {
    float s;      // the drain's multiplier of the accumulator (with d8)
    float alpha;  // weight-value scale (a power of two in the exact mode)
    float beta;   // min scale: dmin / s
};

// Scale choice of one Q4_K super-block from its first header word
// (fp16 d | fp16 dmin << 16).  Producer and drain call the same code.
__device__ __forceinline__ BlockScale q4k_block_scale(uint32_t hdr) {
    const float d = fp16_bits_to_float(hdr), dm = fp16_bits_to_float(hdr >> 16);
    BlockScale r;
    if (d != 0.f) {
        const float rho = __fdiv_rn(dm, d);
        float lim = fabsf(rho) * 63.f;
        int e = 0;
        while (e < 14 && lim > 32768.f) {
            lim *= 0.5f;
            e++;
        }
        if (!(lim > 32768.f)) {
            const float a = __int_as_float((127 - e) << 23);  // 2^-e
            r.s = d * __int_as_float((127 + e) << 23);
            r.alpha = a;
            r.beta = rho * a;
            return r;
        }
    }
    if (dm != 0.f) {
        r.s = dm;
        r.alpha = __fdiv_rn(d, dm);
        r.beta = 1.f;
    } else {
        r.s = 0.f;
        r.alpha = 0.f;
        r.beta = 0.f;
    }
    return r;
}

// Q4K.GetScaleMin (Kernels/Q4K.cs:7-18) on the 12 scale bytes held in three
// words (bytes 4..15 of the block).
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t w0, uint32_t w1, uint32_t w2, int& sc, int& m) {
    auto sb = [&](int i) -> int {
        const uint32_t w = i < 4 ? w0 : (i < 8 ? w1 : w2);
        return (int)((w >> (8 * (i & 3))) & 0xffu);
    };
    if (j < 4) {
        sc = sb(j) & 63;
        m = sb(j + 4) & 63;
    } else {
        sc = (sb(j + 4) & 0xF) | ((sb(j - 4) >> 6) << 4);
        m = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
    }
}

__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hadd2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// A small integer (|v| <= 2048) as both halves of an fp16 pair (exact).
__device__ __forceinline__ uint32_t h2_dup(int v) {
    const uint32_t u = __half_as_ushort(__int2half_rn(v));
    return u | (u << 16);
}
__device__ __forceinline__ int sext_byte(uint32_t w, int k) { return (int)(int8_t)(uint8_t)(w >> (8 * k)); }
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}


// Bounded wait; gives up when the CTA aborted or the time limit passed (the
// latter records DEV_ERR_TIMEOUT and raises the CTA's abort flag).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, unsigned* err, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_hint(bar, parity, 1000000u)) return true;
        if ((it & 7u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - start > tcg::WAIT_LIMIT_NS) {
                atomicOr(err, DEV_ERR_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Non-blocking test of two barrier phases in one go: both tests issue back
// to back and the thread waits once for the pair (a barrier test takes ~100
// cycles under load, and every cycle the MMA thread spends waiting is a
// bubble in the tensor pipe).
__device__ __forceinline__ bool test2(uint64_t* b0, uint32_t p0, uint64_t* b1, uint32_t p1) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred q0, q1;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q0, [%1], %2;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q1, [%3], %4;\n"
        "and.pred q0, q0, q1;\n"
        "selp.u32 %0, 1, 0, q0;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(b0)), "r"(p0), "r"(smem_u32(b1)), "r"(p1)
        : "memory");
    return ok != 0;
}
// One half super-block of the fast mode in a single instruction block: the
// eight 16-K MMAs (A in TMEM columns a_tmem + 8 t; B at the activation stage's
// descriptor, K steps t = 0..3 in the first 64-K box and 4..7 in the second,
// 16-byte units 2 t and BOX16 + 2 (t - 4)), the commit of `done`, and two
// non-blocking tests of the next half's input barriers.  The tests are issued
// before the MMAs and their result read after the commit, so their latency
// (~100 cycles under the kernel's shared-memory load) overlaps MMA issue
// instead of leaving the tensor pipe idle.
template <int BOX16>  // the second 64-K box of the stage, in 16-byte units
__device__ __forceinline__ bool mma_half_polled(uint32_t d_tmem, uint32_t a_tmem, uint64_t xdesc, uint32_t idesc,
                                                uint32_t accumulate, uint64_t* done, uint64_t* nb0, uint32_t np0,
                                                uint64_t* nb1, uint32_t np1) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred q0, q1, pa, pt;\n"
        ".reg .b64 bd;\n"
        ".reg .b32 at;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q0, [%8], %9;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q1, [%10], %11;\n"
        "setp.ne.b32 pa, %5, 0;\n"
        "setp.eq.b32 pt, %6, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, {%6, %6, %6, %6}, pa;\n"
        "add.u32 at, %2, 8;\n"
        "add.u64 bd, %3, 2;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 16;\n"
        "add.u64 bd, %3, 4;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 24;\n"
        "add.u64 bd, %3, 6;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 32;\n"
        "add.u64 bd, %3, %12;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 40;\n"
        "add.u64 bd, %3, %13;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 48;\n"
        "add.u64 bd, %3, %14;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 56;\n"
        "add.u64 bd, %3, %15;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n"
        "and.pred q0, q0, q1;\n"
        "selp.u32 %0, 1, 0, q0;\n"
        "}\n"
        : "=r"(ok)
        : "r"(d_tmem), "r"(a_tmem), "l"(xdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(smem_u32(done)),
          "r"(smem_u32(nb0)), "r"(np0), "r"(smem_u32(nb1)), "r"(np1), "n"(BOX16), "n"(BOX16 + 2), "n"(BOX16 + 4),
          "n"(BOX16 + 6)
        : "memory");
    return ok != 0;
}

// One half super-block of the exact Q6_K form in a single instruction block:
// for each of the eight 16-K steps, the MMAs of both A parts (TMEM columns
// a_tmem + 8 t and a_tmem + 64 + 8 t) against the step's activations (as in
// mma_half_polled), the commit of `done`, and the two non-blocking tests of
// the next half's input barriers.
template <int BOX16>
__device__ __forceinline__ bool mma_half_q6x(uint32_t d_tmem, uint32_t a_tmem, uint64_t xdesc, uint32_t idesc,
                                             uint32_t accumulate, uint64_t* done, uint64_t* nb0, uint32_t np0,
                                             uint64_t* nb1, uint32_t np1) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred q0, q1, pa, pt;\n"
        ".reg .b64 bd;\n"
        ".reg .b32 at;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q0, [%8], %9;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q1, [%10], %11;\n"
        "setp.ne.b32 pa, %5, 0;\n"
        "setp.eq.b32 pt, %6, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, {%6, %6, %6, %6}, pa;\n"
        "add.u32 at, %2, 64;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], %3, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 8;\n"
        "add.u64 bd, %3, 2;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 72;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 16;\n"
        "add.u64 bd, %3, 4;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 80;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 24;\n"
        "add.u64 bd, %3, 6;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 88;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 32;\n"
        "add.u64 bd, %3, %12;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 96;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 40;\n"
        "add.u64 bd, %3, %13;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 104;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 48;\n"
        "add.u64 bd, %3, %14;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 112;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 56;\n"
        "add.u64 bd, %3, %15;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 120;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n"
        "and.pred q0, q0, q1;\n"
        "selp.u32 %0, 1, 0, q0;\n"
        "}\n"
        : "=r"(ok)
        : "r"(d_tmem), "r"(a_tmem), "l"(xdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(smem_u32(done)),
          "r"(smem_u32(nb0)), "r"(np0), "r"(smem_u32(nb1)), "r"(np1), "n"(BOX16), "n"(BOX16 + 2), "n"(BOX16 + 4),
          "n"(BOX16 + 6)
        : "memory");
    return ok != 0;
}

// One half super-block of the exact Q4_K / Q5_K form in a single instruction
// block: the eight 16-K MMAs (as in mma_half_polled), the min-term MMA (A
// from the shared-memory tile at adesc_e, B = the block sums at bdesc_e), the
// commit of `done`, and the two non-blocking tests of the next half's input
// barriers.
template <int BOX16>
__device__ __forceinline__ bool mma_half_exact(uint32_t d_tmem, uint32_t a_tmem, uint64_t xdesc, uint32_t idesc,
                                               uint32_t accumulate, uint64_t adesc_e, uint64_t bdesc_e, uint64_t* done,
                                               uint64_t* nb0, uint32_t np0, uint64_t* nb1, uint32_t np1) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred q0, q1, pa, pt;\n"
        ".reg .b64 bd;\n"
        ".reg .b32 at;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q0, [%8], %9;\n"
        "mbarrier.test_wait.parity.shared::cta.b64 q1, [%10], %11;\n"
        "setp.ne.b32 pa, %5, 0;\n"
        "setp.eq.b32 pt, %6, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %3, %4, {%6, %6, %6, %6}, pa;\n"
        "add.u32 at, %2, 8;\n"
        "add.u64 bd, %3, 2;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 16;\n"
        "add.u64 bd, %3, 4;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 24;\n"
        "add.u64 bd, %3, 6;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 32;\n"
        "add.u64 bd, %3, %12;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 40;\n"
        "add.u64 bd, %3, %13;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 48;\n"
        "add.u64 bd, %3, %14;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "add.u32 at, %2, 56;\n"
        "add.u64 bd, %3, %15;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], [at], bd, %4, {%6, %6, %6, %6}, pt;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%1], %16, %17, %4, {%6, %6, %6, %6}, pt;\n"
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%7];\n"
        "and.pred q0, q0, q1;\n"
        "selp.u32 %0, 1, 0, q0;\n"
        "}\n"
        : "=r"(ok)
        : "r"(d_tmem), "r"(a_tmem), "l"(xdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(smem_u32(done)),
          "r"(smem_u32(nb0)), "r"(np0), "r"(smem_u32(nb1)), "r"(np1), "n"(BOX16), "n"(BOX16 + 2), "n"(BOX16 + 4),
          "n"(BOX16 + 6), "l"(adesc_e), "l"(bdesc_e)
        : "memory");
    return ok != 0;
}

// Wait for work already in flight (ignores the abort flag, still bounded).
__device__ __forceinline__ void wait_inflight(uint64_t* bar, uint32_t parity, unsigned* err) {
    const uint64_t start = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 63u) == 63u && globaltimer_ns() - start > tcg::WAIT_LIMIT_NS) {
            atomicOr(err, DEV_ERR_TIMEOUT);
            return;
        }
    }
}
// Warp-uniform wait: lane 0 polls, the verdict is broadcast.
__device__ __forceinline__ bool warp_wait_bar(uint64_t* bar, uint32_t parity, unsigned* err, volatile int* abort_flag,
                                              int lane) {
    int ok = 0;
    if (lane == 0) ok = wait_bar(bar, parity, err, abort_flag) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// (tile, super-block) of consecutive units without a division per step: the
// integer divisions a role would otherwise do per unit run on the XU pipe,
// which the whole CTA shares.
struct UnitPos {
    int t, b, tt, tw;  // tile, super-block, token tile, weight tile
    __device__ __forceinline__ void init(int u, int nb, int tiles_t) {
        t = u / nb;
        b = u - t * nb;
        tw = t / tiles_t;
        tt = t - tw * tiles_t;
    }
    __device__ __forceinline__ void next(int nb, int tiles_t) {
        if (++b == nb) {
            b = 0;
            ++t;
            if (++tt == tiles_t) {
                tt = 0;
                ++tw;
            }
        }
    }
};

// CTA whose unit range [c*U/G, (c+1)*U/G) contains unit u.
__device__ __forceinline__ int cta_of_unit(long long u, long long U, int G) {
    return (int)(((u + 1) * G + U - 1) / U) - 1;
}

}  // namespace

// ---------------------------------------------------------------------------
// Per-block GEMM metadata, computed once when a Q4_K weight is uploaded (the
// counterpart of the reference's load-time BlockQ4Kx8Meta,
// Kernels/RepackQ4K.cs:91-130).  For tile (g, b), chunk-major like the
// weight tile (16-byte chunk c of row r at c * 512 + r * 16):
//   chunk 0: fp16 alpha * sc_j, j = 0..7        (the A operand's sub-block scales)
//   chunk 1: fp16 high part of -beta * m_j, j = 0..7
//   chunk 2: fp16 low part of -beta * m_j
//   chunk 3: fp16 2^e d * sc_j                   (fast mode: the dequantized weight
//   chunk 4: fp16 2^e dmin * m_j                  2^e (q * (d sc_j) - dmin m_j) in fp16)
// and the drain's fp32 s of each row in s[(g nb + b) 32 + r] (q4k_block_scale).
//
// Fast mode normalises every weight row by a power of two 2^e (fast_row_scale:
// the row's largest |fp16 value| lands in [2^13, 2^14)), so its fp16 values
// neither overflow nor fall into the fp16 subnormals, whatever the row's d;
// the GEMM's drain multiplies the row's outputs by 2^-e (exact).  The passes:
// gemm_meta (exact-mode chunks, the row maxima), fast_row_scale (the maxima ->
// 2^-e in place), fast_meta (chunks 3 and 4).  A block with a non-finite d or
// dmin sets *unsafe and the weight's prefill keeps the exact arithmetic.
// One thread per (row, super-block).
// ---------------------------------------------------------------------------
constexpr int FAST_ROW_EXP = 14;  // a row's largest fast-mode |fp16 value| < 2^14

__device__ __forceinline__ void row_max_update(unsigned* row_max, int row, float v, unsigned* unsafe) {
    if (!isfinite(v)) {
        atomicOr(unsafe, 1u);
        return;
    }
    atomicMax(row_max + row, __float_as_uint(v));  // v >= 0: the bits order as the values
}

__global__ void __launch_bounds__(256) q4k_meta_kernel(const uint8_t* __restrict__ tiles, uint8_t* __restrict__ meta,
                                                      float* __restrict__ s_out, unsigned* __restrict__ row_max,
                                                      int n_pad, int nb, int tile_bytes, int qmax,
                                                      unsigned* __restrict__ unsafe) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)n_pad * nb) return;
    const int row = (int)(idx / nb), b = (int)(idx % nb);
    const int g = row >> 5, r = row & 31;
    const size_t tile = (size_t)g * nb + b;
    const uint4 hdr = *reinterpret_cast<const uint4*>(tiles + tile * tile_bytes + r * 16);  // Q4_K / Q5_K header
    const BlockScale bs = q4k_block_scale(hdr.x);
    const float d = fp16_bits_to_float(hdr.x), dm = fp16_bits_to_float(hdr.x >> 16);
    uint32_t sa[4], hi[4], lo[4];
    float vmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        uint16_t a2[2], h2[2], l2[2];
#pragma unroll
        for (int t = 0; t < 2; t++) {
            int sc, m;
            q4k_scale_min(j + t, hdr.y, hdr.z, hdr.w, sc, m);
            a2[t] = __half_as_ushort(__float2half_rn((float)sc * bs.alpha));
            const float v = -bs.beta * (float)m;
            const __half h = __float2half_rn(v);
            h2[t] = __half_as_ushort(h);
            l2[t] = __half_as_ushort(__float2half_rn(v - __half2float(h)));
            vmax = fmaxf(vmax, fabsf(d) * (float)(sc * qmax) + fabsf(dm) * (float)m);
        }
        sa[j / 2] = a2[0] | ((uint32_t)a2[1] << 16);
        hi[j / 2] = h2[0] | ((uint32_t)h2[1] << 16);
        lo[j / 2] = l2[0] | ((uint32_t)l2[1] << 16);
    }
    uint8_t* mt = meta + tile * tcg::Q4K_META_TILE + r * 16;
    *reinterpret_cast<uint4*>(mt) = make_uint4(sa[0], sa[1], sa[2], sa[3]);
    *reinterpret_cast<uint4*>(mt + 512) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(mt + 1024) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    s_out[tile * 32 + r] = bs.s;
    row_max_update(row_max, row, isfinite(d) && isfinite(dm) ? vmax : __int_as_float(0x7f800000), unsafe);
}

// Row maxima (float bits) -> the fast mode's row scales 2^-e in place, with
// e = FAST_ROW_EXP - E for a maximum in [2^(E-1), 2^E); 1 for an all-zero row.
__global__ void __launch_bounds__(256) fast_row_scale_kernel(float* __restrict__ rs, int n_pad) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= n_pad) return;
    const float vmax = rs[row];
    int E = 0;
    if (!(vmax > 0.f && isfinite(vmax))) {
        rs[row] = 1.f;
        return;
    }
    frexpf(vmax, &E);
    rs[row] = ldexpf(1.f, E - FAST_ROW_EXP);
}

__global__ void __launch_bounds__(256) q4k_fast_meta_kernel(const uint8_t* __restrict__ tiles,
                                                           uint8_t* __restrict__ meta, const float* __restrict__ rs,
                                                           int n_pad, int nb, int tile_bytes) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)n_pad * nb) return;
    const int row = (int)(idx / nb), b = (int)(idx % nb);
    const int g = row >> 5, r = row & 31;
    const size_t tile = (size_t)g * nb + b;
    const uint4 hdr = *reinterpret_cast<const uint4*>(tiles + tile * tile_bytes + r * 16);
    const float up = 1.f / rs[row];  // 2^e: exact
    const float d = fp16_bits_to_float(hdr.x) * up, dm = fp16_bits_to_float(hdr.x >> 16) * up;
    uint32_t fs[4], fm[4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
        uint16_t s2[2], m2[2];
#pragma unroll
        for (int t = 0; t < 2; t++) {
            int sc, m;
            q4k_scale_min(j + t, hdr.y, hdr.z, hdr.w, sc, m);
            s2[t] = __half_as_ushort(__float2half_rn(d * (float)sc));
            m2[t] = __half_as_ushort(__float2half_rn(dm * (float)m));
        }
        fs[j / 2] = s2[0] | ((uint32_t)s2[1] << 16);
        fm[j / 2] = m2[0] | ((uint32_t)m2[1] << 16);
    }
    uint8_t* mt = meta + tile * tcg::Q4K_META_TILE + r * 16;
    *reinterpret_cast<uint4*>(mt + 1536) = make_uint4(fs[0], fs[1], fs[2], fs[3]);
    *reinterpret_cast<uint4*>(mt + 2048) = make_uint4(fm[0], fm[1], fm[2], fm[3]);
}

// Q6_K metadata: for the fast mode fp16 2^e d * sc_s of the 16-value groups
// s = 0..7 (chunk 0) and 8..15 (chunk 1), one 16-byte slot per row as above
// (the producers form (q - 32) * (2^e d sc_s) with one fp16 rounding); for
// the exact mode the drain scale d of each row and super-block (the producers
// read the int8 scales from the tile itself).
__device__ __forceinline__ float q6k_group_scale(uint4 sv, int s) {
    const uint32_t w = s < 4 ? sv.x : s < 8 ? sv.y : s < 12 ? sv.z : sv.w;
    return (float)(int8_t)(w >> (8 * (s & 3)));
}

__global__ void __launch_bounds__(256) q6k_meta_kernel(const uint8_t* __restrict__ tiles, float* __restrict__ s_out,
                                                      unsigned* __restrict__ row_max, int n_pad, int nb,
                                                      unsigned* __restrict__ unsafe) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)n_pad * nb) return;
    const int row = (int)(idx / nb), b = (int)(idx % nb);
    const int g = row >> 5, r = row & 31;
    const size_t tile = (size_t)g * nb + b;
    const uint8_t* t = tiles + tile * tcg::WFmt<TYPE_Q6_K>::TILE_BYTES;
    const float d = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(t + Fmt<TYPE_Q6_K>::D_OFFSET + r * 2));
    s_out[tile * 32 + r] = d;
    const uint4 sv = *reinterpret_cast<const uint4*>(t + 12 * 512 + r * 16);
    float vmax = 0.f;
#pragma unroll
    for (int s = 0; s < 16; s++) vmax = fmaxf(vmax, fabsf(d * q6k_group_scale(sv, s)) * 32.f);
    row_max_update(row_max, row, isfinite(d) ? vmax : __int_as_float(0x7f800000), unsafe);
}

__global__ void __launch_bounds__(256) q6k_fast_meta_kernel(const uint8_t* __restrict__ tiles,
                                                           uint8_t* __restrict__ meta, const float* __restrict__ rs,
                                                           int n_pad, int nb) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)n_pad * nb) return;
    const int row = (int)(idx / nb), b = (int)(idx % nb);
    const int g = row >> 5, r = row & 31;
    const size_t tile = (size_t)g * nb + b;
    const uint8_t* t = tiles + tile * tcg::WFmt<TYPE_Q6_K>::TILE_BYTES;
    const float d = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(t + Fmt<TYPE_Q6_K>::D_OFFSET + r * 2)) *
                    (1.f / rs[row]);
    const uint4 sv = *reinterpret_cast<const uint4*>(t + 12 * 512 + r * 16);
    uint32_t ds[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
        ds[i] = __half_as_ushort(__float2half_rn(d * q6k_group_scale(sv, 2 * i))) |
                ((uint32_t)__half_as_ushort(__float2half_rn(d * q6k_group_scale(sv, 2 * i + 1))) << 16);
    uint8_t* mt = meta + tile * tcg::WFmt<TYPE_Q6_K>::META_TILE + r * 16;
    *reinterpret_cast<uint4*>(mt) = make_uint4(ds[0], ds[1], ds[2], ds[3]);
    *reinterpret_cast<uint4*>(mt + 512) = make_uint4(ds[4], ds[5], ds[6], ds[7]);
}

template <bool FAST, int TNX, int TYPE>
__global__ void __launch_bounds__(tcg::THREADS, 1)
    gemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_e,
                       const TcGemmArgs a) {
    using namespace tcg;
    using GG = Geo<FAST, TNX, TYPE>;
    constexpr int W_TILE = GG::TILE_BYTES, W_META = GG::META_TILE;
    constexpr int TN = GG::TN, X_STAGES = GG::X_STAGES, X_BOX_BYTES = GG::X_BOX_BYTES;
    constexpr int X_STAGE_BYTES = GG::X_STAGE_BYTES, X_PHASE_FILLS = GG::X_PHASE_FILLS;
    constexpr int W_STAGES = GG::W_STAGES, EXT_BOX_BYTES = GG::EXT_BOX_BYTES, W_EXT_OFF = GG::W_EXT_OFF;
    constexpr int W_TILE_OFF = GG::W_TILE_OFF, W_META_OFF = GG::W_META_OFF, W_STAGE_BYTES = GG::W_STAGE_BYTES;
    constexpr int D_STAGES = GG::D_STAGES, D_STAGE_BYTES = GG::D_STAGE_BYTES;
    constexpr int A_BUFS = GG::A_BUFS, E_TILE_BYTES = GG::E_TILE_BYTES;
    constexpr int X_RING_BYTES = GG::X_RING_BYTES, W_RING_BYTES = GG::W_RING_BYTES;
    constexpr int E_RING_BYTES = GG::E_RING_BYTES, D_RING_BYTES = GG::D_RING_BYTES;
    constexpr int ACC_BUFS = GG::ACC_BUFS, A_COL0 = GG::A_COL0, TMEM_COLS = GG::TMEM_COLS, PASSES = GG::PASSES;
    constexpr int A_COLS = GG::A_COLS;
    constexpr bool Q6X = GG::Q6X, MIN_TERM = GG::MIN_TERM;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* xring = smem;
    uint8_t* wring = xring + X_RING_BYTES;
    uint8_t* ering = wring + W_RING_BYTES;
    uint8_t* dring = ering + E_RING_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(dring + D_RING_BYTES);
    // x_full[h][slot] counts the fills of loader h only: fill f of slot
    // f % X_STAGES uses x_full[f & 1][f % X_STAGES], phase f / X_PHASE_FILLS,
    // so a barrier's next phase is always the same loader's next fill.
    // An activation stage is free once the MMAs of its fill completed, which
    // the A buffer's barrier of the same fill already tracks (a_empty): the
    // MMA issues one commit per half super-block.
    uint64_t* x_full = bars;                      // [2][X_STAGES] activation half stage landed
    uint64_t* w_full = x_full + 2 * X_STAGES;     // [W_STAGES] weight tiles + metadata landed
    uint64_t* e_full = w_full + W_STAGES;         // [W_STAGES] Xe landed
    uint64_t* w_empty = e_full + W_STAGES;        // [W_STAGES] producers read it (exact: and its MMAs completed)
    uint64_t* d_full = w_empty + W_STAGES;        // [D_STAGES] drain scales landed
    uint64_t* d_empty = d_full + D_STAGES;        // [D_STAGES] drains done with them
    uint64_t* a_full = d_empty + D_STAGES;        // [A_BUFS] A operand written (TMEM + min tile)
    uint64_t* a_empty = a_full + A_BUFS;          // [A_BUFS] its MMAs completed
    uint64_t* acc_full = a_empty + A_BUFS;        // [2]
    uint64_t* acc_empty = acc_full + 2;           // [2]
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const long long U = a.units;
    const int u0 = (int)((long long)blockIdx.x * U / G);
    const int u1 = (int)((long long)(blockIdx.x + 1) * U / G);
    const int n_units = u1 - u0;
    const int nb = a.nb;
    const int n_groups = a.n_pad / 32;

    if (threadIdx.x == 0) {
        for (int i = 0; i < X_STAGES; i++) {
            mbar_init(x_full + i, 1);
            mbar_init(x_full + X_STAGES + i, 1);
        }
        for (int i = 0; i < W_STAGES; i++) {
            mbar_init(w_full + i, 1);
            mbar_init(e_full + i, 1);
            // 8 producer warps (+ the MMA's commit in exact mode, whose
            // min-term MMA reads the stage's Xe tile)
            mbar_init(w_empty + i, MIN_TERM ? 9 : 8);
        }
        for (int i = 0; i < D_STAGES; i++) {
            mbar_init(d_full + i, 1);
            mbar_init(d_empty + i, NUM_DRAIN);
        }
        for (int i = 0; i < A_BUFS; i++) {
            mbar_init(a_full + i, 4);  // the 4 warps of the producer group
            mbar_init(a_empty + i, 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(acc_full + i, 1);
            mbar_init(acc_empty + i, NUM_DRAIN);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == WARP_MMA) {
        tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    const int wg = warp >> 2;
    if (wg == 0) {
        setmaxnreg_dec<RegSplit<FAST, TYPE>::CTRL>();
        if ((warp == WARP_TMA || warp == WARP_TMA2) && lane == 0) {
            // ---------------- activation halves ----------------
            // This warp loads half h of every unit: fills f = 2 i + h.
            griddep_wait();  // Xq comes from the preparation kernel
            const int h = warp == WARP_TMA ? 0 : 1;
            int issued = -1;
            UnitPos p;
            p.init(u0, nb, a.tiles_t);
            for (int i = 0; i < n_units; i++, p.next(nb, a.tiles_t)) {
                const int f = 2 * i + h;
                const int xs = f % X_STAGES;
                if (f >= X_STAGES) {  // the slot's previous fill g = f - X_STAGES was consumed
                    const int g = f - X_STAGES;
                    if (!wait_bar(a_empty + g % A_BUFS, (uint32_t)(g / A_BUFS) & 1u, a.err, abort_flag)) break;
                }
                uint64_t* full = x_full + h * X_STAGES + xs;
                mbar_arrive_expect_tx(full, X_STAGE_BYTES);
                uint8_t* dst = xring + xs * X_STAGE_BYTES;
                const int k0 = p.b * QK + 128 * h;
                tma_load_2d(dst, &tm_q, k0, p.tt * TN, full);
                tma_load_2d(dst + X_BOX_BYTES, &tm_q, k0 + 64, p.tt * TN, full);
                issued = f;
            }
            // Every copy this warp issued lands before the CTA exits.  Fill
            // f - X_STAGES was consumed before fill f was issued: with three
            // stages (the other loader's fill) this warp's last two fills can
            // be in flight, with two stages (its own) only its last.
            constexpr int BACK = X_STAGES % 2 ? 2 : 0;
            for (int f = issued - BACK; f <= issued; f += 2)
                if (f >= 0)
                    wait_inflight(x_full + h * X_STAGES + (f % X_STAGES), (uint32_t)(f / X_PHASE_FILLS) & 1u, a.err);
        } else if (warp == WARP_WTMA && lane == 0) {
            // ---------------- weight tiles, metadata, Xe; drain scales ----------------
            bool dep_done = false;
            int issued_w = 0, issued_d = 0;
            UnitPos p;
            p.init(u0, nb, a.tiles_t);
            for (int i = 0; i < n_units; i++, p.next(nb, a.tiles_t)) {
                const int b = p.b, tw = p.tw, tt = p.tt;
                int valid = 0;
                for (int q = 0; q < 4; q++) valid += (tw * 4 + q < n_groups) ? 1 : 0;
                const int ws = i % W_STAGES;
                if (!wait_bar(w_empty + ws, ((uint32_t)(i / W_STAGES) & 1u) ^ 1u, a.err, abort_flag)) break;
                uint8_t* dst = wring + ws * W_STAGE_BYTES;
                mbar_arrive_expect_tx(w_full + ws, (uint32_t)(valid * (W_TILE + W_META)));
                for (int q = 0; q < valid; q++) {
                    const size_t tile = (size_t)(tw * 4 + q) * nb + b;
                    bulk_g2s(dst + W_TILE_OFF + q * W_TILE, a.tiles + tile * W_TILE, W_TILE, w_full + ws);
                    bulk_g2s(dst + W_META_OFF + q * W_META, a.meta + tile * W_META, W_META,
                             w_full + ws);
                }
                issued_w = i + 1;
                if constexpr (FAST) continue;  // no min term, no per-super-block scales
                if (!dep_done) {
                    griddep_wait();  // Xe and d8 come from the preparation kernel
                    dep_done = true;
                }
                if constexpr (MIN_TERM) {
                    mbar_arrive_expect_tx(e_full + ws, EXT_BOX_BYTES);
                    tma_load_2d(dst + W_EXT_OFF, &tm_e, b * 16, tt * TN, e_full + ws);
                }
                const int ds = i % D_STAGES;
                if (!wait_bar(d_empty + ds, ((uint32_t)(i / D_STAGES) & 1u) ^ 1u, a.err, abort_flag)) break;
                uint8_t* dd = dring + ds * D_STAGE_BYTES;
                mbar_arrive_expect_tx(d_full + ds, (uint32_t)(valid * 128 + TN * 4));
                for (int q = 0; q < valid; q++)
                    bulk_g2s(dd + q * 128, a.scale + ((size_t)(tw * 4 + q) * nb + b) * 32, 128, d_full + ds);
                bulk_g2s(dd + 512, a.xd + (size_t)b * a.m_pad + tt * TN, TN * 4, d_full + ds);
                issued_d = i + 1;
            }
            for (int i = (issued_w > W_STAGES ? issued_w - W_STAGES : 0); i < issued_w; i++) {
                wait_inflight(w_full + (i % W_STAGES), (uint32_t)(i / W_STAGES) & 1u, a.err);
                if (MIN_TERM) wait_inflight(e_full + (i % W_STAGES), (uint32_t)(i / W_STAGES) & 1u, a.err);
            }
            for (int i = (issued_d > D_STAGES ? issued_d - D_STAGES : 0); i < issued_d; i++)
                wait_inflight(d_full + (i % D_STAGES), (uint32_t)(i / D_STAGES) & 1u, a.err);
        } else if (warp == WARP_MMA && lane == 0) {
            // ---------------- MMA issue ----------------
            // Exact mode: one accumulator per unit (drained per super-block).
            // Fast mode: one accumulator per tile segment (the run of units of
            // one tile this CTA computes), drained once.
            const uint32_t idesc = tc_idesc_f16_f32(TM, TN);
            // Inputs of fill f = 2 i + h: activation stage x_full[h][f % X_STAGES]
            // (phase f / X_PHASE_FILLS) and A buffer 2 (i & 1) + h (phase i / 2).
            auto x_bar = [&](int f) { return x_full + (f & 1) * X_STAGES + f % X_STAGES; };
            auto x_par = [&](int f) { return (uint32_t)(f / X_PHASE_FILLS) & 1u; };
            auto a_bar = [&](int f) { return a_full + f % A_BUFS; };
            auto a_par = [&](int f) { return (uint32_t)(f / A_BUFS) & 1u; };
            UnitPos p;
            p.init(u0, nb, a.tiles_t);
            int seg = 0;
            // The next half's inputs are tested (without blocking) in the middle
            // of the current half's MMAs; the thread blocks on them only when
            // they had not landed by then.
            bool ready = false;
            const int n_fills = 2 * n_units;
            for (int i = 0; i < n_units; i++, p.next(nb, a.tiles_t)) {
                const bool seg_start = (i == 0 || p.b == 0), seg_end = (p.b == nb - 1 || i == n_units - 1);
                const int acc_i = FAST ? seg : i;  // accumulator use
                const int accb = acc_i % ACC_BUFS;
                const int ws = i % W_STAGES;
                if ((!FAST || seg_start) &&
                    !wait_bar(acc_empty + accb, ((uint32_t)(acc_i / ACC_BUFS) & 1u) ^ 1u, a.err, abort_flag))
                    break;
                if (MIN_TERM && !wait_bar(e_full + ws, (uint32_t)(i / W_STAGES) & 1u, a.err, abort_flag)) break;
                const uint32_t d_tmem = tmem + (uint32_t)(accb * TN);
                bool ok = true;
                for (int h = 0; h < 2; h++) {
                    const int f = 2 * i + h;
                    if (!ready && !test2(x_bar(f), x_par(f), a_bar(f), a_par(f)) &&
                        !(wait_bar(x_bar(f), x_par(f), a.err, abort_flag) &&
                          wait_bar(a_bar(f), a_par(f), a.err, abort_flag))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const int xs = f % X_STAGES;
                    const int ab = f % A_BUFS;
                    // One descriptor per half; each 16-value K step is a
                    // constant offset of its start address (16-byte units).
                    const uint64_t xdesc = tc_smem_desc(smem_u32(xring + xs * X_STAGE_BYTES), 1024, 2);
                    const uint32_t a_tmem = tmem + (uint32_t)(A_COL0 + A_COLS * ab);
                    const bool fresh = FAST ? (seg_start && h == 0) : (h == 0);
                    if constexpr (FAST) {
                        // The last fill polls its own (landed) barriers: the
                        // result is not used.
                        const int fn = f + 1 < n_fills ? f + 1 : f;
                        ready = mma_half_polled<X_BOX_BYTES / 16>(d_tmem, a_tmem, xdesc, idesc, fresh ? 0u : 1u,
                                                                  a_empty + ab, x_bar(fn), x_par(fn), a_bar(fn),
                                                                  a_par(fn)) &&
                                f + 1 < n_fills;
                        continue;
                    }
                    if constexpr (Q6X) {
                        // Two exact parts of the A operand per K step, one B;
                        // the commit frees the A buffer and the activation stage.
                        const int fn = f + 1 < n_fills ? f + 1 : f;
                        ready = mma_half_q6x<X_BOX_BYTES / 16>(d_tmem, a_tmem, xdesc, idesc, fresh ? 0u : 1u,
                                                               a_empty + ab, x_bar(fn), x_par(fn), a_bar(fn),
                                                               a_par(fn)) &&
                                f + 1 < n_fills;
                        continue;
                    }
                    if constexpr (MIN_TERM) {
                        // The eight K steps, then the min term: 16 K from shared
                        // memory (A) against Xe; the commit frees the A buffer
                        // and the activation stage.
                        const uint64_t bext = tc_smem_desc(smem_u32(wring + ws * W_STAGE_BYTES + W_EXT_OFF), 256, 6);
                        const uint64_t aext = tc_smem_desc(smem_u32(ering + ab * E_TILE_BYTES), 256, 6);
                        const int fn = f + 1 < n_fills ? f + 1 : f;
                        ready = mma_half_exact<X_BOX_BYTES / 16>(d_tmem, a_tmem, xdesc, idesc, fresh ? 0u : 1u, aext,
                                                                 bext, a_empty + ab, x_bar(fn), x_par(fn), a_bar(fn),
                                                                 a_par(fn)) &&
                                f + 1 < n_fills;
                    }
                }
                if (!ok) break;
                if (MIN_TERM) tc_commit(w_empty + ws);
                if (!FAST || seg_end) tc_commit(acc_full + accb);
                if (seg_end) seg++;
            }
            // Every MMA issued by this thread completes before TMEM is freed.
            tc_commit(mma_done);
            wait_inflight(mma_done, 0, a.err);
        }
    } else if (warp < WARP_DRAIN0) {
        setmaxnreg_dec<RegSplit<FAST, TYPE>::PROD>();
        // ---------------- weight producers ----------------
        // Group h (4 warps, one per TMEM lane quadrant q) builds the A
        // operand of half h of every super-block: the 64 value columns of
        // rows 32q..32q+31 (Q6_K exact: two parts of 64) in TMEM buffer
        // (2 i + h) % A_BUFS, and the min-term tile (high part for h = 0, low
        // part for h = 1) in shared memory.  Each group owns its buffers, so
        // each barrier has one waiting group.
        const int h = (warp - WARP_PROD0) >> 2;
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int r = 32 * q + lane;  // row of the tile
        UnitPos p;
        p.init(u0, nb, a.tiles_t);
        for (int i = 0; i < n_units; i++, p.next(nb, a.tiles_t)) {
            const bool valid = p.tw * 4 + q < n_groups;
            const int ws = i % W_STAGES, fa = 2 * i + h, ab = fa % A_BUFS;
            if (!warp_wait_bar(w_full + ws, (uint32_t)(i / W_STAGES) & 1u, a.err, abort_flag, lane)) break;
            const uint8_t* stage = wring + ws * W_STAGE_BYTES;
            const uint8_t* tile = stage + W_TILE_OFF + q * W_TILE + lane * 16;
            const uint8_t* mt = stage + W_META_OFF + q * W_META + lane * 16;
            uint4 sa = make_uint4(0, 0, 0, 0), em = sa, w0 = sa, w1 = sa, w2 = sa, w3 = sa;
            uint4 x0 = sa, x1 = sa;  // Q5_K / Q6_K high bits
            if (valid) {
                if constexpr (TYPE == TYPE_Q6_K) {
                    // fast: d sc_s of the half's groups 8h..8h+7 (metadata);
                    // exact: the 16 int8 scales (tile chunk 12).  ql bytes
                    // 64h..64h+63 (chunks 4h..4h+3), qh bytes 32h..32h+31
                    // (chunks 8+2h, 9+2h)
                    sa = *reinterpret_cast<const uint4*>(Q6X ? tile + 12 * 512 : mt + h * 512);
                    w0 = *reinterpret_cast<const uint4*>(tile + (4 * h) * 512);
                    w1 = *reinterpret_cast<const uint4*>(tile + (4 * h + 1) * 512);
                    w2 = *reinterpret_cast<const uint4*>(tile + (4 * h + 2) * 512);
                    w3 = *reinterpret_cast<const uint4*>(tile + (4 * h + 3) * 512);
                    x0 = *reinterpret_cast<const uint4*>(tile + (8 + 2 * h) * 512);
                    x1 = *reinterpret_cast<const uint4*>(tile + (9 + 2 * h) * 512);
                } else {
                    // exact: alpha sc_j and the min-term part; fast: d sc_j and dmin m_j
                    sa = *reinterpret_cast<const uint4*>(mt + (FAST ? 3 : 0) * 512);
                    em = *reinterpret_cast<const uint4*>(mt + (FAST ? 4 : 1 + h) * 512);
                    // 64-value chunks c = 2h, 2h + 1 (tile chunks QS + 4h .. QS + 3 + 4h)
                    constexpr int QS = TYPE == TYPE_Q5_K ? 3 : 1;
                    w0 = *reinterpret_cast<const uint4*>(tile + (QS + 4 * h) * 512);
                    w1 = *reinterpret_cast<const uint4*>(tile + (QS + 1 + 4 * h) * 512);
                    w2 = *reinterpret_cast<const uint4*>(tile + (QS + 2 + 4 * h) * 512);
                    w3 = *reinterpret_cast<const uint4*>(tile + (QS + 3 + 4 * h) * 512);
                    if constexpr (TYPE == TYPE_Q5_K) {
                        // qh bytes 0..31 (chunks 1, 2): bit c of byte l is value 32c + l's fifth bit
                        x0 = *reinterpret_cast<const uint4*>(tile + 1 * 512);
                        x1 = *reinterpret_cast<const uint4*>(tile + 2 * 512);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(w_empty + ws);  // this warp is done with the stage
            if (!warp_wait_bar(a_empty + ab, ((uint32_t)(fa / A_BUFS) & 1u) ^ 1u, a.err, abort_flag, lane)) break;
            tc_fence_after();
            if constexpr (MIN_TERM) {
                // Min-term tile: row r holds 16 fp16 (both halves of pair j are
                // the value of sub-block j), 32-byte swizzle: 16-byte chunk c of
                // row r at (r / 8) * 256 + (r % 8) * 32 + ((c ^ ((r >> 2) & 1)) * 16).
                uint8_t* et = ering + ab * E_TILE_BYTES + (r >> 3) * 256 + (r & 7) * 32;
                const int sw = (r >> 2) & 1;
                const uint4 c0 = make_uint4(__byte_perm(em.x, 0u, 0x1010), __byte_perm(em.x, 0u, 0x3232),
                                            __byte_perm(em.y, 0u, 0x1010), __byte_perm(em.y, 0u, 0x3232));
                const uint4 c1 = make_uint4(__byte_perm(em.z, 0u, 0x1010), __byte_perm(em.z, 0u, 0x3232),
                                            __byte_perm(em.w, 0u, 0x1010), __byte_perm(em.w, 0u, 0x3232));
                *reinterpret_cast<uint4*>(et + (sw << 4)) = c0;
                *reinterpret_cast<uint4*>(et + ((sw ^ 1) << 4)) = c1;
            }
            const uint32_t a_col = tmem + lane_base + (uint32_t)(A_COL0 + A_COLS * ab);
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                // fp16 scales of sub-blocks 2c (low nibbles) and 2c + 1 (high
                // nibbles), c = 2h + cc: word c of sa (and em) holds both.
                const uint32_t sw = (h == 0) ? (cc == 0 ? sa.x : sa.y) : (cc == 0 ? sa.z : sa.w);
                const uint32_t s_lo = __byte_perm(sw, 0u, 0x1010), s_hi = __byte_perm(sw, 0u, 0x3232);
                const uint4 wa = cc ? w2 : w0, wb = cc ? w3 : w1;
                const uint32_t W[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                uint32_t v[32];
                if constexpr (TYPE == TYPE_Q6_K) {
                    // cc = 0: q1 = low nibbles of ql bytes l + qh bits 0-1 (values
                    // 128h + l), q2 = low nibbles of ql bytes 32 + l + qh bits 2-3
                    // (128h + 32 + l); cc = 1: the high nibbles with qh bits 4-5
                    // (q3, 128h + 64 + l) and 6-7 (q4, 128h + 96 + l).  fp16
                    // 1024 + q - 1056 = q - 32 exactly, times d sc_s (one rounding).
                    const uint32_t A[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    const uint32_t B[8] = {w2.x, w2.y, w2.z, w2.w, w3.x, w3.y, w3.z, w3.w};
                    const uint32_t H[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    const uint32_t S[4] = {sa.x, sa.y, sa.z, sa.w};
                    // Exact mode: part 0 (sl (q - 32)) is stored here, part 1
                    // (16 sh (q - 32)) by the common store below.
#pragma unroll 1
                    for (int part = Q6X ? 0 : 1; part < 2; part++) {
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        const uint32_t qa = cc ? (((A[w] >> 4) & 0x0F0F0F0Fu) | (H[w] & 0x30303030u))
                                               : ((A[w] & 0x0F0F0F0Fu) | ((H[w] << 4) & 0x30303030u));
                        const uint32_t qb = cc ? (((B[w] >> 4) & 0x0F0F0F0Fu) | ((H[w] >> 2) & 0x30303030u))
                                               : ((B[w] & 0x0F0F0F0Fu) | ((H[w] << 2) & 0x30303030u));
                        const int ga = 4 * cc + (w >> 2), gb = ga + 2;  // 16-value group within the half
                        uint32_t da, db;
                        if constexpr (Q6X) {
                            // sc = 16 sh + sl, sl in [0, 15]: the exact fp16
                            // factors sl (part 0) and 16 sh = sc - sl (part 1);
                            // the half's scales are bytes 8h..8h+7 (words 2h, 2h+1)
                            const uint32_t sw0 = h ? S[2] : S[0], sw1 = h ? S[3] : S[1];
                            const int sca = sext_byte(ga < 4 ? sw0 : sw1, ga & 3);
                            const int scb = sext_byte(gb < 4 ? sw0 : sw1, gb & 3);
                            da = h2_dup(part == 0 ? (sca & 15) : sca - (sca & 15));
                            db = h2_dup(part == 0 ? (scb & 15) : scb - (scb & 15));
                        } else {
                            da = __byte_perm(S[ga >> 1], 0u, (ga & 1) ? 0x3232 : 0x1010);
                            db = __byte_perm(S[gb >> 1], 0u, (gb & 1) ? 0x3232 : 0x1010);
                        }
                        const uint32_t a02 = hadd2_bits((qa & 0x003F003Fu) | 0x64006400u, 0xE420E420u);
                        const uint32_t a13 = hadd2_bits(((qa >> 8) & 0x003F003Fu) | 0x64006400u, 0xE420E420u);
                        const uint32_t b02 = hadd2_bits((qb & 0x003F003Fu) | 0x64006400u, 0xE420E420u);
                        const uint32_t b13 = hadd2_bits(((qb >> 8) & 0x003F003Fu) | 0x64006400u, 0xE420E420u);
                        v[2 * w] = hmul2_bits(a02, da);
                        v[2 * w + 1] = hmul2_bits(a13, da);
                        v[16 + 2 * w] = hmul2_bits(b02, db);
                        v[16 + 2 * w + 1] = hmul2_bits(b13, db);
                    }
                    if (Q6X && part == 0) tmem_st32(a_col + 32 * cc, v);
                    }
                } else if constexpr (TYPE == TYPE_Q5_K) {
                    // q = nibble + 16 * (bit 2c, or 2c + 1 for the high nibble, of
                    // qh byte l), c = 2h + cc; fp16 1024 + q is exact (q <= 31).
                    const uint32_t QH[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                    const int c = 2 * h + cc;
                    uint32_t n_lo, n_hi;
                    if constexpr (FAST) {
                        const uint32_t mw = (h == 0) ? (cc == 0 ? em.x : em.y) : (cc == 0 ? em.z : em.w);
                        n_lo = __byte_perm(mw, 0u, 0x1010) ^ 0x80008000u;  // -dmin m
                        n_hi = __byte_perm(mw, 0u, 0x3232) ^ 0x80008000u;
                    } else {
                        n_lo = hmul2_bits(s_lo, 0xE400E400u);  // -1024 s
                        n_hi = hmul2_bits(s_hi, 0xE400E400u);
                    }
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        const uint32_t lo = (W[w] & 0x0F0F0F0Fu) | (((QH[w] >> (2 * c)) & 0x01010101u) << 4);
                        const uint32_t hi = ((W[w] >> 4) & 0x0F0F0F0Fu) | (((QH[w] >> (2 * c + 1)) & 0x01010101u) << 4);
                        const uint32_t l02 = (lo & 0x001F001Fu) | 0x64006400u, l13 = ((lo >> 8) & 0x001F001Fu) | 0x64006400u;
                        const uint32_t h02 = (hi & 0x001F001Fu) | 0x64006400u, h13 = ((hi >> 8) & 0x001F001Fu) | 0x64006400u;
                        if constexpr (FAST) {
                            // w = q * (d sc) - dmin m, one fp16 rounding
                            v[2 * w] = hfma2_bits(hadd2_bits(l02, 0xE400E400u), s_lo, n_lo);
                            v[2 * w + 1] = hfma2_bits(hadd2_bits(l13, 0xE400E400u), s_lo, n_lo);
                            v[16 + 2 * w] = hfma2_bits(hadd2_bits(h02, 0xE400E400u), s_hi, n_hi);
                            v[16 + 2 * w + 1] = hfma2_bits(hadd2_bits(h13, 0xE400E400u), s_hi, n_hi);
                        } else {
                            // (1024 + q) s - 1024 s = q s exactly (q s <= 31 * 63 alpha)
                            v[2 * w] = hfma2_bits(l02, s_lo, n_lo);
                            v[2 * w + 1] = hfma2_bits(l13, s_lo, n_lo);
                            v[16 + 2 * w] = hfma2_bits(h02, s_hi, n_hi);
                            v[16 + 2 * w + 1] = hfma2_bits(h13, s_hi, n_hi);
                        }
                    }
                } else if constexpr (FAST) {
                    // w = q * (d sc) - dmin m, one fp16 rounding: q recovered
                    // exactly from the magic-number form, then one fma.
                    const uint32_t mw = (h == 0) ? (cc == 0 ? em.x : em.y) : (cc == 0 ? em.z : em.w);
                    const uint32_t nm_lo = __byte_perm(mw, 0u, 0x1010) ^ 0x80008000u;  // -dmin m
                    const uint32_t nm_hi = __byte_perm(mw, 0u, 0x3232) ^ 0x80008000u;
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        const uint32_t w8 = W[w] >> 8;
                        const uint32_t l02 = (W[w] & 0x000F000Fu) | 0x64006400u;
                        const uint32_t l13 = (w8 & 0x000F000Fu) | 0x64006400u;
                        const uint32_t h02 = (W[w] & 0x00F000F0u) | 0x64006400u;
                        const uint32_t h13 = (w8 & 0x00F000F0u) | 0x64006400u;
                        // (1024 + q) - 1024 = q; (1024 + 16 q) / 16 - 64 = q
                        const uint32_t q02 = hadd2_bits(l02, 0xE400E400u), q13 = hadd2_bits(l13, 0xE400E400u);
                        const uint32_t p02 = hfma2_bits(h02, 0x2C002C00u, 0xD400D400u);
                        const uint32_t p13 = hfma2_bits(h13, 0x2C002C00u, 0xD400D400u);
                        v[2 * w] = hfma2_bits(q02, s_lo, nm_lo);
                        v[2 * w + 1] = hfma2_bits(q13, s_lo, nm_lo);
                        v[16 + 2 * w] = hfma2_bits(p02, s_hi, nm_hi);
                        v[16 + 2 * w + 1] = hfma2_bits(p13, s_hi, nm_hi);
                    }
                } else {
                    // Low nibbles become fp16 1024 + q; high nibbles, masked in
                    // place, fp16 1024 + 16 q.  (1024 + q) s - 1024 s and
                    // (1024 + 16 q) s/16 - 64 s are q s exactly.
                    const uint32_t n_lo = hmul2_bits(s_lo, 0xE400E400u);   // -1024 s
                    const uint32_t s_h16 = hmul2_bits(s_hi, 0x2C002C00u);  // s / 16
                    const uint32_t n_hi = hmul2_bits(s_hi, 0xD400D400u);   // -64 s
#pragma unroll
                    for (int w = 0; w < 8; w++) {
                        // bytes l = 4w..4w+3: low nibbles are values 64c+l, high
                        // nibbles 64c+32+l.  One fp16 pair takes the nibbles of
                        // bytes 0 and 2, the other those of bytes 1 and 3: K order
                        // 0, 2, 1, 3, as in Xq.
                        const uint32_t w8 = W[w] >> 8;
                        const uint32_t l02 = (W[w] & 0x000F000Fu) | 0x64006400u;
                        const uint32_t l13 = (w8 & 0x000F000Fu) | 0x64006400u;
                        const uint32_t h02 = (W[w] & 0x00F000F0u) | 0x64006400u;
                        const uint32_t h13 = (w8 & 0x00F000F0u) | 0x64006400u;
                        v[2 * w] = hfma2_bits(l02, s_lo, n_lo);
                        v[2 * w + 1] = hfma2_bits(l13, s_lo, n_lo);
                        v[16 + 2 * w] = hfma2_bits(h02, s_h16, n_hi);
                        v[16 + 2 * w + 1] = hfma2_bits(h13, s_h16, n_hi);
                    }
                }
                tmem_st32(a_col + (Q6X ? 64 : 0) + 32 * cc, v);
            }
            tmem_st_wait();
            if (MIN_TERM) fence_proxy_async_smem();  // the min-term tile is read by the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full + ab);
        }
    } else {
        setmaxnreg_inc<RegSplit<FAST, TYPE>::DRAIN>();
        // ---------------- drains ----------------
        const int dw = warp - WARP_DRAIN0;
        const int q = warp & 3;    // lane quadrant = 32 weight rows of the tile
        const int th = dw >> 2;    // token half of the tile (TN / 2 tokens)
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        if constexpr (FAST) griddep_wait();  // the token scales come from the preparation kernel
        float out[64];
#pragma unroll
        for (int j = 0; j < 64; j++) out[j] = 0.f;
        int seg_b0 = 0, seg = 0;
        UnitPos p;
        p.init(u0, nb, a.tiles_t);
        for (int i = 0; i < n_units; i++, p.next(nb, a.tiles_t)) {
            const int t = p.t, b = p.b, tw = p.tw, tt = p.tt;
            if (i == 0 || b == 0) {
#pragma unroll
                for (int j = 0; j < 64; j++) out[j] = 0.f;
                seg_b0 = b;
            }
            const int g = tw * 4 + q;
            const int row = g * 32 + lane;
            if constexpr (!FAST) {
            const int ds = i % D_STAGES;
            const int accb = i & 1;
            if (!warp_wait_bar(d_full + ds, (uint32_t)(i / D_STAGES) & 1u, a.err, abort_flag, lane) ||
                !warp_wait_bar(acc_full + accb, (uint32_t)(i >> 1) & 1u, a.err, abort_flag, lane))
                break;
            tc_fence_after();
            const uint8_t* dstage = dring + ds * D_STAGE_BYTES;
            // Weight scale of this lane's row and the 64 token scales of this
            // warp's half, from the unit's drain stage.
            const float s = (g < n_groups) ? reinterpret_cast<const float*>(dstage)[q * 32 + lane] : 0.f;
            const float* dr = reinterpret_cast<const float*>(dstage + 512) + th * 64;
            const float2 ss = make_float2(s, s);
            uint32_t r0[32], r1[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(accb * TN + th * 64), r0);
            tmem_ld32(tmem + lane_base + (uint32_t)(accb * TN + th * 64 + 32), r1);
            tmem_ld_wait2(r0, r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + accb);  // the accumulator may be overwritten
#pragma unroll
            for (int j = 0; j < 64; j += 4) {
                // out += (d8 * s) * T, two tokens per packed instruction
                const float4 d4 = *reinterpret_cast<const float4*>(dr + j);
                const uint32_t* rr = j < 32 ? r0 + j : r1 + (j - 32);
                const float2 c0 = __fmul2_rn(make_float2(d4.x, d4.y), ss);
                const float2 c1 = __fmul2_rn(make_float2(d4.z, d4.w), ss);
                const float2 o0 = __ffma2_rn(c0, make_float2(__uint_as_float(rr[0]), __uint_as_float(rr[1])),
                                             make_float2(out[j], out[j + 1]));
                const float2 o1 = __ffma2_rn(c1, make_float2(__uint_as_float(rr[2]), __uint_as_float(rr[3])),
                                             make_float2(out[j + 2], out[j + 3]));
                out[j] = o0.x;
                out[j + 1] = o0.y;
                out[j + 2] = o1.x;
                out[j + 3] = o1.y;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty + ds);  // done with the unit's scales
            }

            if (b != nb - 1 && i != n_units - 1) continue;  // the tile's segment goes on
            int accb = 0;
            // Fast mode: the scales that undo the operands' normalisation, the
            // row's 2^-e_r and lane l's token scales 2^-e_t of tokens l and
            // 32 + l of each pass, loaded while the accumulator fills.
            float rsc = 0.f, ts_lo[PASSES], ts_hi[PASSES];
            if constexpr (FAST) {
                rsc = (g < n_groups) ? a.scale[(size_t)a.n_pad * a.nb + row] : 0.f;
#pragma unroll
                for (int pp = 0; pp < PASSES; pp++) {
                    const float* ts = a.xd + tt * TN + th * (TN / 2) + pp * 64;
                    ts_lo[pp] = ts[lane];
                    ts_hi[pp] = ts[32 + lane];
                }
                // One accumulator per tile segment: read it once, at the end.
                accb = seg % ACC_BUFS;
                if (!warp_wait_bar(acc_full + accb, (uint32_t)(seg / ACC_BUFS) & 1u, a.err, abort_flag, lane)) break;
                seg++;
                tc_fence_after();
            }
            // This warp's tokens of the tile: TN / 2 from th * TN / 2, in
            // passes of 64 (one pass for 128-token tiles).
            for (int pp = 0; pp < PASSES; pp++) {
            if constexpr (FAST) {
                const uint32_t col = (uint32_t)(accb * TN + th * (TN / 2) + pp * 64);
                uint32_t r0[32], r1[32];
                tmem_ld32(tmem + lane_base + col, r0);
                tmem_ld32(tmem + lane_base + col + 32, r1);
                tmem_ld_wait2(r0, r1);
                if (pp == PASSES - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acc_empty + accb);  // all of it read
                }
                // Undo the operands' normalisation: times the row scale 2^-e_r,
                // then the token scale 2^-e_t (each exact, barring underflow).
                const float tlo = pp ? ts_lo[PASSES - 1] : ts_lo[0];
                const float thi = pp ? ts_hi[PASSES - 1] : ts_hi[0];
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    out[j] = __uint_as_float(r0[j]) * rsc * __shfl_sync(0xffffffffu, tlo, j);
                    out[32 + j] = __uint_as_float(r1[j]) * rsc * __shfl_sync(0xffffffffu, thi, j);
                }
            }
            const int tok0 = tt * TN + th * (TN / 2) + pp * 64;
            if (seg_b0 == 0 && b == nb - 1) {
                // This CTA computed the whole tile.
                if (row < a.n_out) {
#pragma unroll
                    for (int j = 0; j < 64; j++)
                        if (tok0 + j < a.tokens) a.y[(size_t)(tok0 + j) * a.ldy + row] = out[j];
                }
                continue;
            }
            // A piece of a tile shared with neighbouring CTAs.
            const long long tu0 = (long long)t * nb;
            const int first = cta_of_unit(tu0, U, G), last = cta_of_unit(tu0 + nb - 1, U, G);
            const int me = blockIdx.x;
            int* const ctr = a.counters + ((size_t)t * NUM_DRAIN + dw) * PASSES + pp;
            if (last == first + 1) {
                // Two pieces.  CTA `last` computes its piece first (the start of
                // its range): it stores the piece into y and raises the tile's
                // flag.  CTA `first` computes its piece last (the end of its
                // range) and adds it onto y once the flag is up.  Each output is
                // one addition of the two pieces, whatever the timing.
                if (me == last) {
                    if (row < a.n_out) {
#pragma unroll
                        for (int j = 0; j < 64; j++)
                            if (tok0 + j < a.tokens) a.y[(size_t)(tok0 + j) * a.ldy + row] = out[j];
                    }
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) atomicExch(ctr, 1);
                } else {
                    int up = 0;
                    if (lane == 0) {
                        const uint64_t start = globaltimer_ns();
                        for (uint32_t it = 0;; ++it) {
                            if (ld_acquire_gpu(ctr) == 1) {
                                up = 1;
                                break;
                            }
                            if ((it & 63u) == 63u && globaltimer_ns() - start > WAIT_LIMIT_NS) {
                                atomicOr(a.err, DEV_ERR_TIMEOUT);
                                break;
                            }
                        }
                    }
                    up = __shfl_sync(0xffffffffu, up, 0);
                    if (!up) continue;
                    if (row < a.n_out) {
#pragma unroll
                        for (int j = 0; j < 64; j++)
                            if (tok0 + j < a.tokens) atomicAdd(a.y + (size_t)(tok0 + j) * a.ldy + row, out[j]);
                    }
                    if (lane == 0) *ctr = 0;  // ready for the next launch
                }
                continue;
            }
            // Three or more pieces: publish this one; the last of the covering
            // CTAs to arrive adds the pieces in CTA order.
            const int local = (th * (TN / 2) + pp * 64) * TM + q * 32 + lane;  // token-major piece of this warp
            // Slot 0 holds a CTA's first tile, slot 1 its last one.
            auto piece = [&](int cta) -> float* {
                const long long cu0 = (long long)cta * U / G;
                return a.ws + ((size_t)cta * 2 + ((cu0 / nb == t) ? 0 : 1)) * (TM * TN) + local;
            };
            float* mine = piece(me);
#pragma unroll
            for (int j = 0; j < 64; j++) __stcg(mine + j * TM, out[j]);
            __threadfence();
            __syncwarp();
            int is_last = 0;
            if (lane == 0) {
                const int old = atomicAdd(ctr, 1);
                is_last = (old == last - first) ? 1 : 0;
                if (is_last) *ctr = 0;  // ready for the next launch
            }
            is_last = __shfl_sync(0xffffffffu, is_last, 0);
            if (!is_last) continue;
            __threadfence();
            for (int cta = first; cta <= last; cta++) {
                const float* pc = piece(cta);
#pragma unroll
                for (int j = 0; j < 64; j++) {
                    const float v = __ldcg(pc + j * TM);
                    out[j] = (cta == first) ? v : out[j] + v;
                }
            }
            if (row < a.n_out) {
#pragma unroll
                for (int j = 0; j < 64; j++)
                    if (tok0 + j < a.tokens) a.y[(size_t)(tok0 + j) * a.ldy + row] = out[j];
            }
            }  // passes
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == WARP_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
size_t gemm_meta_bytes(int type, int nb, int n_pad) {
    const int per_tile = type == TYPE_Q6_K ? tcg::WFmt<TYPE_Q6_K>::META_TILE : tcg::Q4K_META_TILE;
    return (size_t)(n_pad / 32) * nb * per_tile;
}
size_t gemm_scale_bytes(int type, int nb, int n_pad) {
    (void)type;
    // The exact mode's drain scale of every (row, super-block), then the fast
    // mode's row scales 2^-e.
    return ((size_t)n_pad * nb + n_pad) * sizeof(float);
}

cudaError_t launch_gemm_meta(int type, const uint8_t* tiles, uint8_t* meta, float* scale, int nb, int n_pad,
                             unsigned* unsafe, cudaStream_t s) {
    const long long n = (long long)n_pad * nb;
    if (n == 0) return cudaSuccess;
    float* rs = scale + n;
    unsigned* row_max = reinterpret_cast<unsigned*>(rs);
    cudaError_t e = cudaMemsetAsync(row_max, 0, (size_t)n_pad * sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)((n + 255) / 256), row_grid = (unsigned)((n_pad + 255) / 256);
    switch (type) {
    case TYPE_Q4_K:
    case TYPE_Q5_K: {
        const int tile_bytes = type == TYPE_Q4_K ? tcg::WFmt<TYPE_Q4_K>::TILE_BYTES : tcg::WFmt<TYPE_Q5_K>::TILE_BYTES;
        const int qmax = type == TYPE_Q4_K ? 15 : 31;
        q4k_meta_kernel<<<grid, 256, 0, s>>>(tiles, meta, scale, row_max, n_pad, nb, tile_bytes, qmax, unsafe);
        fast_row_scale_kernel<<<row_grid, 256, 0, s>>>(rs, n_pad);
        q4k_fast_meta_kernel<<<grid, 256, 0, s>>>(tiles, meta, rs, n_pad, nb, tile_bytes);
        break;
    }
    case TYPE_Q6_K:
        q6k_meta_kernel<<<grid, 256, 0, s>>>(tiles, scale, row_max, n_pad, nb, unsafe);
        fast_row_scale_kernel<<<row_grid, 256, 0, s>>>(rs, n_pad);
        q6k_fast_meta_kernel<<<grid, 256, 0, s>>>(tiles, meta, rs, n_pad, nb);
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

bool tc_gemm_supports(int type, bool fast) {
    (void)fast;
    return type == TYPE_Q4_K || type == TYPE_Q5_K || type == TYPE_Q6_K;
}

int tc_gemm_tile_tokens(bool fast, int tokens) { return (fast && tokens >= 512) ? 256 : 128; }

TcGemmPlan plan_tc_gemm(int nb, int n_pad, int tokens, int num_sms, int tn) {
    TcGemmPlan p{};
    p.tn = tn == 256 ? 256 : 128;
    p.m_pad = (tokens + p.tn - 1) / p.tn * p.tn;
    p.tiles_w = (n_pad + tcg::TM - 1) / tcg::TM;
    p.tiles_t = p.m_pad / p.tn;
    p.tiles = p.tiles_w * p.tiles_t;
    p.units = (long long)p.tiles * nb;
    p.grid = (int)(p.units < num_sms ? p.units : num_sms);
    p.xq_bytes = (size_t)p.m_pad * nb * QK * 2;
    p.xe_bytes = (size_t)p.m_pad * nb * 16 * 2;
    p.xd_bytes = (size_t)p.m_pad * nb * 4;
    p.ws_bytes = (size_t)p.grid * 2 * tcg::TM * p.tn * 4;
    p.counters = (size_t)p.tiles * tcg::NUM_DRAIN * (p.tn / 128);
    return p;
}

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

bool encode_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                   uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

cudaError_t configure_tc_gemm() {
    // The warpgroups' setmaxnreg split draws on the registers the CTA is
    // launched with: each kernel must have been compiled to exactly
    // LAUNCH_REGS per thread, or a larger request would never be granted.
    using namespace tcg;
    const struct {
        const void* fn;
        size_t smem;
    } kernels[] = {
        {(const void*)gemm_q4k_tc_kernel<false, 128, TYPE_Q4_K>, Geo<false, 128, TYPE_Q4_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 128, TYPE_Q4_K>, Geo<true, 128, TYPE_Q4_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 256, TYPE_Q4_K>, Geo<true, 256, TYPE_Q4_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<false, 128, TYPE_Q5_K>, Geo<false, 128, TYPE_Q5_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 128, TYPE_Q5_K>, Geo<true, 128, TYPE_Q5_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 256, TYPE_Q5_K>, Geo<true, 256, TYPE_Q5_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<false, 128, TYPE_Q6_K>, Geo<false, 128, TYPE_Q6_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 128, TYPE_Q6_K>, Geo<true, 128, TYPE_Q6_K>::SMEM_BYTES},
        {(const void*)gemm_q4k_tc_kernel<true, 256, TYPE_Q6_K>, Geo<true, 256, TYPE_Q6_K>::SMEM_BYTES}};
    for (const auto& k : kernels) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, k.fn);
        if (e != cudaSuccess) return e;
        if (fa.numRegs != tcg::LAUNCH_REGS || fa.maxThreadsPerBlock < tcg::THREADS) return cudaErrorInvalidConfiguration;
        e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)k.smem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_gemm_prep(const float* x, int k, int tokens, int m_pad, void* xq, void* xe, float* xd,
                             unsigned* tmax, bool fast, cudaStream_t s, const float* up) {
    const int nb = k / QK;
    const long long warps = (long long)m_pad * nb;
    const int grid = (int)((warps + 7) / 8);
    if (!fast) {
        gemm_prep_kernel<<<grid, 256, 0, s>>>(x, up, k, tokens, m_pad, static_cast<__half*>(xq),
                                              static_cast<__half*>(xe), xd);
        return cudaGetLastError();
    }
    if (tokens > 0) {
        gemm_prep_fast_kernel<<<(int)(((long long)tokens * nb + 7) / 8), 256, 0, s>>>(
            x, up, k, tokens, static_cast<__half*>(xq), tmax);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((m_pad + FAST_SCALE_TOKENS - 1) / FAST_SCALE_TOKENS);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_token_scale_kernel, x, up, k, tokens, m_pad, static_cast<__half*>(xq), xd,
                              tmax);
}

template <int TYPE>
static cudaError_t launch_typed(cudaLaunchConfig_t& cfg, const TcGemmArgs& args, const CUtensorMap& tq,
                                const CUtensorMap& te, bool fast, bool wide) {
    using namespace tcg;
    if (wide) {
        cfg.dynamicSmemBytes = Geo<true, 256, TYPE>::SMEM_BYTES;
        return cudaLaunchKernelEx(&cfg, gemm_q4k_tc_kernel<true, 256, TYPE>, tq, te, args);
    }
    if (fast) {
        cfg.dynamicSmemBytes = Geo<true, 128, TYPE>::SMEM_BYTES;
        return cudaLaunchKernelEx(&cfg, gemm_q4k_tc_kernel<true, 128, TYPE>, tq, te, args);
    }
    cfg.dynamicSmemBytes = Geo<false, 128, TYPE>::SMEM_BYTES;
    return cudaLaunchKernelEx(&cfg, gemm_q4k_tc_kernel<false, 128, TYPE>, tq, te, args);
}

static cudaError_t launch_tc_instance(cudaLaunchConfig_t& cfg, const TcGemmArgs& args, const CUtensorMap& tq,
                                      const CUtensorMap& te, bool fast, bool wide) {
    switch (args.type) {
    case TYPE_Q4_K: return launch_typed<TYPE_Q4_K>(cfg, args, tq, te, fast, wide);
    case TYPE_Q5_K: return launch_typed<TYPE_Q5_K>(cfg, args, tq, te, fast, wide);
    case TYPE_Q6_K: return launch_typed<TYPE_Q6_K>(cfg, args, tq, te, fast, wide);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_tc_gemm(const TcGemmArgs& args, const void* xq, const void* xe, int k, bool fast, cudaStream_t s,
                           bool pdl) {
    CUtensorMap tq, te;
    const int nb = k / QK;
    const bool wide = fast && args.tn == 256;
    if (args.tn != 128 && !wide) return cudaErrorInvalidValue;
    if (!encode_2d_f16(&tq, xq, (uint64_t)k, (uint64_t)args.tokens, (uint64_t)k * 2, 64, (uint32_t)args.tn,
                       CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    if (fast) {
        te = tq;  // unused in fast mode
    } else if (!encode_2d_f16(&te, xe, (uint64_t)nb * 16, (uint64_t)args.tokens, (uint64_t)nb * 32, 16, tcg::TN,
                              CU_TENSOR_MAP_SWIZZLE_32B)) {
        return cudaErrorInvalidValue;
    }
    if (!tc_gemm_supports(args.type, fast)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(args.grid);
    cfg.blockDim = dim3(tcg::THREADS);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return launch_tc_instance(cfg, args, tq, te, fast, wide);
}

}  // namespace q35k
