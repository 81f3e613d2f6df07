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
//   warp 0      TMA: Xq (4 boxes of 64 K x 128 tokens, 128-byte swizzle) and
//               Xe (16 x 128, 32-byte swizzle) per unit into one of 3 stages
//   warp 1      TMEM allocation and the MMA issue (one thread)
//   warps 4-11  weight producers: the A operand of each half super-block,
//               in turn, in one of 3 TMEM buffers (64 value columns + 8 min
//               columns); two warps per TMEM lane quadrant
//   warps 12-19 drains: per super-block, accumulator -> registers, scaled by
//               the Q8_K and weight scales; then the tile's output
// TMEM: accumulators at columns 0 and 128 (double-buffered per super-block),
// A buffers of 64 value columns at 256 + 64 i and 8 min columns at 448 + 8 i.  Every mbarrier wait is bounded in time; on expiry
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
constexpr int TN = 128;  // tokens per tile
// Five warpgroups of four warps; each warpgroup re-sizes its registers with
// setmaxnreg.  Registers are split between an SM's four sub-partitions, one
// warp of every warpgroup in each: 5 x 32 x 96 = 15360 <= 16384 at launch,
// and afterwards 128 x (40 + 80 + 80 + 136 + 136) = 60416 <= 640 x 96.
constexpr int THREADS = 640;
constexpr int LAUNCH_REGS = 96;
constexpr int REGS_CTRL = 40, REGS_PROD = 80, REGS_DRAIN = 136;
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_PROD0 = 4, WARP_DRAIN0 = 12, NUM_DRAIN = 8;
constexpr int STAGES = 3;
constexpr int MAIN_BOX_BYTES = 64 * 2 * TN;                      // 64 fp16 K x 128 tokens
constexpr int EXT_BOX_BYTES = 16 * 2 * TN;                       // 16 fp16 K x 128 tokens
constexpr int STAGE_BYTES = 4 * MAIN_BOX_BYTES + EXT_BOX_BYTES;  // one super-block
// A buffers: 64 value columns at 256 + 64 i, 8 min columns at 448 + 8 i.
constexpr int A_BUFS = 3, A_COL0 = 256, E_COL0 = 448;
constexpr int TMEM_COLS = 512;
constexpr int Q4K_TILE = 32 * 144;  // one 32-row tile of the uploaded layout
constexpr int DR_BYTES = NUM_DRAIN * 64 * 4;  // per drain warp: the d8 of its 64 tokens
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 256 + DR_BYTES;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

}  // namespace tcg

// ---------------------------------------------------------------------------
// Activation preparation: Q8_K quantization (bit-exact) -> fp16 Xq, Xe and the
// block scales d8 in Xd[b][m_pad] (zero for padded tokens).  One warp per
// (token, super-block).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gemm_prep_kernel(const float* __restrict__ x, int k, int tokens, int m_pad,
                                                       __half* __restrict__ xq, __half* __restrict__ xe,
                                                       float* __restrict__ xd) {
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
    const float d = warp_q8k_values(x + (size_t)r * k + (size_t)b * QK, lane, q);
    __half* row = xq + (size_t)r * k + (size_t)b * QK;
    const __half2 p0 = __halves2half2(__int2half_rn(q[0]), __int2half_rn(q[1]));
    const __half2 p1 = __halves2half2(__int2half_rn(q[2]), __int2half_rn(q[3]));
    const __half2 p2 = __halves2half2(__int2half_rn(q[4]), __int2half_rn(q[5]));
    const __half2 p3 = __halves2half2(__int2half_rn(q[6]), __int2half_rn(q[7]));
    uint2 v0, v1;
    v0.x = *reinterpret_cast<const uint32_t*>(&p0);
    v0.y = *reinterpret_cast<const uint32_t*>(&p1);
    v1.x = *reinterpret_cast<const uint32_t*>(&p2);
    v1.y = *reinterpret_cast<const uint32_t*>(&p3);
    reinterpret_cast<uint2*>(row)[lane] = v0;        // values 4l..4l+3
    reinterpret_cast<uint2*>(row + 128)[lane] = v1;  // values 128+4l..
    int s0, s1;
    warp_q8k_bsums(q, s0, s1);
    if ((lane & 3) == 0) {
        __half* e = xe + (size_t)r * nb * 16 + (size_t)b * 16;
        e[lane >> 2] = __int2half_rn(s0);
        e[8 + (lane >> 2)] = __int2half_rn(s1);
    }
    if (lane == 0) xd[(size_t)b * m_pad + r] = d;
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
__device__ __forceinline__ uint32_t half2_bits(float v) {
    const __half h = __float2half_rn(v);
    const uint32_t u = __half_as_ushort(h);
    return u | (u << 16);
}

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Bounded wait; gives up when the CTA aborted or the time limit passed (the
// latter records DEV_ERR_TIMEOUT and raises the CTA's abort flag).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, unsigned* err, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - start > tcg::WAIT_LIMIT_NS) {
                atomicOr(err, DEV_ERR_TIMEOUT);
                *abort_flag = 1;
                return false;
            }
        }
    }
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

// CTA whose unit range [c*U/G, (c+1)*U/G) contains unit u.
__device__ __forceinline__ int cta_of_unit(long long u, long long U, int G) {
    return (int)(((u + 1) * G + U - 1) / U) - 1;
}

}  // namespace

__global__ void __launch_bounds__(tcg::THREADS, 1)
    gemm_q4k_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_e,
                       const TcGemmArgs a) {
    using namespace tcg;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* stages = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* b_full = bars;          // [STAGES]
    uint64_t* b_empty = bars + 3;     // [STAGES]
    uint64_t* a_full = bars + 6;      // [A_BUFS]
    uint64_t* a_empty = bars + 9;     // [A_BUFS]
    uint64_t* acc_full = bars + 12;   // [2]
    uint64_t* acc_empty = bars + 14;  // [2]
    uint64_t* mma_done = bars + 16;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* dr_smem = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const long long U = a.units;
    const int u0 = (int)((long long)blockIdx.x * U / G);
    const int u1 = (int)((long long)(blockIdx.x + 1) * U / G);
    const int n_units = u1 - u0;
    const int nb = a.nb;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(b_full + i, 1);
            mbar_init(b_empty + i, 1);
        }
        for (int i = 0; i < A_BUFS; i++) {
            mbar_init(a_full + i, 8);
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
      setmaxnreg_dec<REGS_CTRL>();
      if (warp == WARP_TMA) {
        // ---------------- activation loads ----------------
        if (lane == 0) {
            griddep_wait();  // Xq / Xe come from the preparation kernel
            int issued = 0;
            for (int i = 0; i < n_units; i++) {
                const int u = u0 + i, t = u / nb, b = u % nb, tt = t % a.tiles_t;
                const int st = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                if (!wait_bar(b_empty + st, ph ^ 1u, a.err, abort_flag)) break;
                mbar_arrive_expect_tx(b_full + st, STAGE_BYTES);
                uint8_t* dst = stages + st * STAGE_BYTES;
#pragma unroll
                for (int j = 0; j < 4; j++) tma_load_2d(dst + j * MAIN_BOX_BYTES, &tm_q, b * QK + 64 * j, tt * TN, b_full + st);
                tma_load_2d(dst + 4 * MAIN_BOX_BYTES, &tm_e, b * 16, tt * TN, b_full + st);
                issued = i + 1;
            }
            // Copies still in flight land before the CTA may exit.
            for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; i++)
                wait_inflight(b_full + (i % STAGES), (uint32_t)(i / STAGES) & 1u, a.err);
        }
      } else if (warp == WARP_MMA) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            const uint32_t idesc = tc_idesc_f16_f32(TM, TN);
            for (int i = 0; i < n_units; i++) {
                const int st = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                const int accb = i & 1;
                const uint32_t acc_ph = (uint32_t)(i >> 1) & 1u;
                if (!wait_bar(acc_empty + accb, acc_ph ^ 1u, a.err, abort_flag)) break;
                if (!wait_bar(b_full + st, ph, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t b_base = smem_u32(stages + st * STAGE_BYTES);
                const uint32_t d_tmem = tmem + (uint32_t)(accb * TN);
                bool ok = true;
                for (int h = 0; h < 2; h++) {
                    const int hs = 2 * i + h;
                    const int ab = hs % A_BUFS;
                    const uint32_t aph = (uint32_t)(hs / A_BUFS) & 1u;
                    if (!wait_bar(a_full + ab, aph, a.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem + (uint32_t)(A_COL0 + 64 * ab);
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const int kk = 8 * h + t;  // 16-value K step within the super-block
                        const uint64_t desc =
                            tc_smem_desc(b_base + (kk >> 2) * MAIN_BOX_BYTES + (kk & 3) * 32, 1024, 2);
                        tc_mma_f16_ts(d_tmem, a_tmem + 8 * t, desc, idesc, (h | t) != 0 ? 1u : 0u);
                    }
                    tc_mma_f16_ts(d_tmem, tmem + (uint32_t)(E_COL0 + 8 * ab),
                                  tc_smem_desc(b_base + 4 * MAIN_BOX_BYTES, 256, 6), idesc, 1u);
                    tc_commit(a_empty + ab);
                }
                if (!ok) break;
                tc_commit(b_empty + st);
                tc_commit(acc_full + accb);
            }
            // Every MMA issued by this thread completes before TMEM is freed.
            tc_commit(mma_done);
            wait_inflight(mma_done, 0, a.err);
        }
      }  // warps 2, 3: no role
    } else if (warp < WARP_DRAIN0) {
        setmaxnreg_dec<REGS_PROD>();
        // ---------------- weight producers ----------------
        // Every A buffer fill (one half super-block, in order) is built by all
        // eight producer warps: warp (q, part) writes the 32 value columns of
        // 64-value chunk 2h + part for lanes 32q..32q+31, and 4 of the 8 min
        // columns.  Each warp waits on every buffer phase in turn.
        const int q = warp & 3;                     // TMEM lane quadrant = 32-row group within the tile
        const int part = (warp - WARP_PROD0) >> 2;  // which 64-value chunk of the half
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int n_groups = a.n_pad / 32;
        const int n_fills = 2 * n_units;
        // Weight bytes of fill f: header chunk and the two 16-byte chunks of
        // qs holding 64-value chunk c = 2h + part (chunks 1 + 2c, 2 + 2c).
        auto load_fill = [&](int f, uint4& hdr, uint4& wa, uint4& wb) {
            const int u = u0 + (f >> 1), t = u / nb, b = u % nb, tw = t / a.tiles_t;
            const int g = tw * 4 + q;
            const int c = 2 * (f & 1) + part;
            if (g < n_groups) {
                const uint8_t* tile = a.tiles + ((size_t)g * nb + b) * Q4K_TILE + lane * 16;
                hdr = ldg16(tile);
                wa = ldg16(tile + (1 + 2 * c) * 512);
                wb = ldg16(tile + (2 + 2 * c) * 512);
            } else {
                hdr = wa = wb = make_uint4(0, 0, 0, 0);
            }
        };
        uint4 hdr, wa, wb;
        if (n_fills > 0) load_fill(0, hdr, wa, wb);
        for (int f = 0; f < n_fills; f++) {
            const int h = f & 1;
            const int ab = f % A_BUFS;
            const uint32_t aph = (uint32_t)(f / A_BUFS) & 1u;
            uint4 nhdr, nwa, nwb;
            if (f + 1 < n_fills) load_fill(f + 1, nhdr, nwa, nwb);
            if (!warp_wait_bar(a_empty + ab, aph ^ 1u, a.err, abort_flag, lane)) break;
            tc_fence_after();
            const BlockScale bs = q4k_block_scale(hdr.x);
            const uint32_t a_col = tmem + lane_base + (uint32_t)(A_COL0 + 64 * ab);
            const uint32_t e_col = tmem + lane_base + (uint32_t)(E_COL0 + 8 * ab);
            {
                const int c = 2 * h + part;  // 64-value chunk of the super-block
                int sc_lo, m_lo, sc_hi, m_hi;
                q4k_scale_min(2 * c, hdr.y, hdr.z, hdr.w, sc_lo, m_lo);
                q4k_scale_min(2 * c + 1, hdr.y, hdr.z, hdr.w, sc_hi, m_hi);
                const uint32_t s_lo = half2_bits((float)sc_lo * bs.alpha);
                const uint32_t n_lo = half2_bits(-1024.f * ((float)sc_lo * bs.alpha));
                const uint32_t s_hi = half2_bits((float)sc_hi * bs.alpha);
                const uint32_t n_hi = half2_bits(-1024.f * ((float)sc_hi * bs.alpha));
                const uint32_t W[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                uint32_t v[32];
#pragma unroll
                for (int w = 0; w < 8; w++) {
                    // bytes l = 4w..4w+3; low nibbles are values 64c+l, high nibbles 64c+32+l
                    const uint32_t t0 = __byte_perm(W[w], 0u, 0x4140);  // b0, b1 -> 16-bit lanes
                    const uint32_t t1 = __byte_perm(W[w], 0u, 0x4342);  // b2, b3
                    const uint32_t l0 = (t0 & 0x000F000Fu) | 0x64006400u;  // fp16 1024 + q
                    const uint32_t l1 = (t1 & 0x000F000Fu) | 0x64006400u;
                    const uint32_t h0 = ((t0 >> 4) & 0x000F000Fu) | 0x64006400u;
                    const uint32_t h1 = ((t1 >> 4) & 0x000F000Fu) | 0x64006400u;
                    // (1024 + q) * s - 1024 * s = q * s, exact in fp16
                    v[2 * w] = hfma2_bits(l0, s_lo, n_lo);
                    v[2 * w + 1] = hfma2_bits(l1, s_lo, n_lo);
                    v[16 + 2 * w] = hfma2_bits(h0, s_hi, n_hi);
                    v[16 + 2 * w + 1] = hfma2_bits(h1, s_hi, n_hi);
                }
                tmem_st32(a_col + 32 * part, v);
            }
            {
                // Min column j: -beta * m_j for the block sums 2j, 2j+1;
                // the fp16 high part in the first half of the super-block,
                // the low part in the second.  This warp writes j = 4 part..+3.
                uint32_t e[4];
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    int sc, m;
                    q4k_scale_min(4 * part + jj, hdr.y, hdr.z, hdr.w, sc, m);
                    const float v = -bs.beta * (float)m;
                    const float hi = __half2float(__float2half_rn(v));
                    e[jj] = half2_bits(h == 0 ? hi : v - hi);
                }
                tmem_st4(e_col + 4 * part, e);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full + ab);
            hdr = nhdr;
            wa = nwa;
            wb = nwb;
        }
    } else {
        setmaxnreg_inc<REGS_DRAIN>();
        // ---------------- drains ----------------
        const int dw = warp - WARP_DRAIN0;
        const int q = warp & 3;    // lane quadrant = 32 weight rows of the tile
        const int th = dw >> 2;    // 64-token half of the tile
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const int n_groups = a.n_pad / 32;
        griddep_wait();  // Xd comes from the preparation kernel
        float out[64];
#pragma unroll
        for (int j = 0; j < 64; j++) out[j] = 0.f;
        int seg_b0 = 0;
        for (int i = 0; i < n_units; i++) {
            const int u = u0 + i, t = u / nb, b = u % nb, tw = t / a.tiles_t, tt = t % a.tiles_t;
            if (i == 0 || b == 0) {
#pragma unroll
                for (int j = 0; j < 64; j++) out[j] = 0.f;
                seg_b0 = b;
            }
            const int g = tw * 4 + q;
            const int row = g * 32 + lane;
            float s = 0.f;
            if (g < n_groups) {
                const uint32_t hw =
                    __ldg(reinterpret_cast<const uint32_t*>(a.tiles + ((size_t)g * nb + b) * Q4K_TILE + lane * 16));
                s = q4k_block_scale(hw).s;
            }
            // This warp's 64 token scales, staged in shared memory (read back
            // as broadcasts) to keep registers for the accumulators.
            float* dr = dr_smem + dw * 64;
            {
                const float2 v = __ldg(reinterpret_cast<const float2*>(a.xd + (size_t)b * a.m_pad + tt * TN + th * 64) + lane);
                __syncwarp();
                reinterpret_cast<float2*>(dr)[lane] = v;
                __syncwarp();
            }
            const int accb = i & 1;
            const uint32_t acc_ph = (uint32_t)(i >> 1) & 1u;
            if (!warp_wait_bar(acc_full + accb, acc_ph, a.err, abort_flag, lane)) break;
            tc_fence_after();
#pragma unroll
            for (int hh = 0; hh < 4; hh++) {
                uint32_t r[16];
                tmem_ld16(tmem + lane_base + (uint32_t)(accb * TN + th * 64 + hh * 16), r);
                tmem_ld_wait(r);
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    const float4 d4 = *reinterpret_cast<const float4*>(dr + hh * 16 + j);
                    // out += (d8 * s) * T, two tokens per packed instruction
                    const float2 ss = make_float2(s, s);
                    const float2 c0 = fmul2(make_float2(d4.x, d4.y), ss);
                    const float2 c1 = fmul2(make_float2(d4.z, d4.w), ss);
                    const float2 o0 = ffma2(c0, make_float2(__uint_as_float(r[j + 0]), __uint_as_float(r[j + 1])),
                                            make_float2(out[hh * 16 + j + 0], out[hh * 16 + j + 1]));
                    const float2 o1 = ffma2(c1, make_float2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                                            make_float2(out[hh * 16 + j + 2], out[hh * 16 + j + 3]));
                    out[hh * 16 + j + 0] = o0.x;
                    out[hh * 16 + j + 1] = o0.y;
                    out[hh * 16 + j + 2] = o1.x;
                    out[hh * 16 + j + 3] = o1.y;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + accb);

            if (b != nb - 1 && i != n_units - 1) continue;  // the tile's segment goes on
            const int tok0 = tt * TN + th * 64;
            if (seg_b0 == 0 && b == nb - 1) {
                // This CTA computed the whole tile.
                if (row < a.n_out) {
#pragma unroll
                    for (int j = 0; j < 64; j++)
                        if (tok0 + j < a.tokens) a.y[(size_t)(tok0 + j) * a.n_out + row] = out[j];
                }
                continue;
            }
            // A piece of a tile shared with neighbouring CTAs: publish it; the
            // last of the covering CTAs to arrive adds the pieces in CTA order.
            const long long tu0 = (long long)t * nb;
            const int first = cta_of_unit(tu0, U, G), last = cta_of_unit(tu0 + nb - 1, U, G);
            const int me = blockIdx.x;
            const int local = (th * 64) * TM + q * 32 + lane;  // token-major piece of this warp
            auto slot_of = [&](int c) -> int {
                const long long cu0 = (long long)c * U / G;
                return (cu0 / nb == t) ? 0 : 1;
            };
            float* mine = a.ws + ((size_t)me * 2 + slot_of(me)) * (TM * TN) + local;
#pragma unroll
            for (int j = 0; j < 64; j++) __stcg(mine + j * TM, out[j]);
            __threadfence();
            __syncwarp();
            int is_last = 0;
            if (lane == 0) {
                int* ctr = a.counters + (size_t)t * NUM_DRAIN + dw;
                const int old = atomicAdd(ctr, 1);
                is_last = (old == last - first) ? 1 : 0;
                if (is_last) *ctr = 0;  // ready for the next launch
            }
            is_last = __shfl_sync(0xffffffffu, is_last, 0);
            if (!is_last) continue;
            __threadfence();
#pragma unroll
            for (int j = 0; j < 64; j++) {
                float v = 0.f;
                for (int c = first; c <= last; c++) {
                    const float x = (c == me) ? out[j]
                                              : __ldcg(a.ws + ((size_t)c * 2 + slot_of(c)) * (TM * TN) + local + j * TM);
                    v = (c == first) ? x : v + x;
                }
                if (row < a.n_out && tok0 + j < a.tokens) a.y[(size_t)(tok0 + j) * a.n_out + row] = v;
            }
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
TcGemmPlan plan_tc_gemm(int nb, int n_pad, int tokens, int num_sms) {
    TcGemmPlan p{};
    p.m_pad = (tokens + tcg::TN - 1) / tcg::TN * tcg::TN;
    p.tiles_w = (n_pad + tcg::TM - 1) / tcg::TM;
    p.tiles_t = p.m_pad / tcg::TN;
    p.tiles = p.tiles_w * p.tiles_t;
    p.units = (long long)p.tiles * nb;
    p.grid = (int)(p.units < num_sms ? p.units : num_sms);
    p.xq_bytes = (size_t)p.m_pad * nb * QK * 2;
    p.xe_bytes = (size_t)p.m_pad * nb * 16 * 2;
    p.xd_bytes = (size_t)p.m_pad * nb * 4;
    p.ws_bytes = (size_t)p.grid * 2 * tcg::TM * tcg::TN * 4;
    p.counters = (size_t)p.tiles * tcg::NUM_DRAIN;
    p.smem_bytes = tcg::SMEM_BYTES;
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
    // launched with: the kernel must have been compiled to exactly
    // LAUNCH_REGS per thread, or a larger request would never be granted.
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, gemm_q4k_tc_kernel);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != tcg::LAUNCH_REGS || fa.maxThreadsPerBlock < tcg::THREADS) return cudaErrorInvalidConfiguration;
    return cudaFuncSetAttribute(gemm_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)tcg::SMEM_BYTES);
}

cudaError_t launch_gemm_prep(const float* x, int k, int tokens, int m_pad, void* xq, void* xe, float* xd,
                             cudaStream_t s) {
    const int nb = k / QK;
    const long long warps = (long long)m_pad * nb;
    const int grid = (int)((warps + 7) / 8);
    gemm_prep_kernel<<<grid, 256, 0, s>>>(x, k, tokens, m_pad, static_cast<__half*>(xq), static_cast<__half*>(xe),
                                          xd);
    return cudaGetLastError();
}

cudaError_t launch_tc_gemm(const TcGemmArgs& args, const void* xq, const void* xe, int k, cudaStream_t s, bool pdl) {
    CUtensorMap tq, te;
    const int nb = k / QK;
    if (!encode_2d_f16(&tq, xq, (uint64_t)k, (uint64_t)args.tokens, (uint64_t)k * 2, 64, tcg::TN,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d_f16(&te, xe, (uint64_t)nb * 16, (uint64_t)args.tokens, (uint64_t)nb * 32, 16, tcg::TN,
                       CU_TENSOR_MAP_SWIZZLE_32B))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(args.grid);
    cfg.blockDim = dim3(tcg::THREADS);
    cfg.dynamicSmemBytes = tcg::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_q4k_tc_kernel, tq, te, args);
}

}  // namespace q35k
