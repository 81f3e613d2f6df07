// gemv_dot.cuh -- per-tile K-quant x Q8_K dot products of the decode GEMV:
// lane r of a warp decodes row r of a 32-row tile (chunk-major layout, see
// device_common.cuh) against staged Q8_K activations, for M tokens at once.
//
// Integer dots (dp4a, dp2a) into exact int32 per super-block, scaled in fp32
// once per block: acc += (d_w*d_x)*S - (dmin_w*d_x)*Mn
// (VecDotQ4K.DotScalar, Kernels/VecDotQ4K.cs:42-61; Q5K.Dot,
// Kernels/Q5K.cs:62-83; the Q6_K bias form of Q6K.DotAvx2,
// Kernels/Q6K.cs:105-108,159).
#pragma once

#include "device_common.cuh"

#include <cuda_fp16.h>

namespace q35k {

// dp4a with unsigned a bytes (0..255) and signed b bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Sign-extend byte k of w.
__device__ __forceinline__ int sext_byte(uint32_t w, int k) { return (int)(int8_t)(uint8_t)(w >> (8 * k)); }
__device__ __forceinline__ int byte_of(uint32_t w, int k) { return (w >> (8 * k)) & 0xff; }

// Q4_K / Q5_K header: fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins,
// unpacked as Q4K.UnpackScales (Kernels/Q4K.cs:20-33).
struct KHeader {
    float d, dmin;
    uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};
__device__ __forceinline__ KHeader unpack_header(uint4 h) {
    KHeader k;
    k.d = fp16_bits_to_float(h.x);
    k.dmin = fp16_bits_to_float(h.x >> 16);
    const uint32_t u0 = h.y, u1 = h.z, u2 = h.w;
    k.sc_lo = u0 & 0x3f3f3f3fu;
    k.sc_hi = (u2 & 0x0f0f0f0fu) | (((u0 >> 6) & 0x03030303u) << 4);
    k.mn_lo = u1 & 0x3f3f3f3fu;
    k.mn_hi = ((u2 >> 4) & 0x0f0f0f0fu) | (((u1 >> 6) & 0x03030303u) << 4);
    return k;
}
__device__ __forceinline__ int k_scale(const KHeader& k, int j) { return byte_of(j < 4 ? k.sc_lo : k.sc_hi, j & 3); }

// Staged planar Q8_K activations in block-major order (device_common.cuh):
// block t of token m at qs + (t*rows + m)*256, d[t*rows4 + m],
// bsums + (t*rows + m)*16.
struct Q8Smem {
    const int8_t* qs;
    const float* d;
    const int16_t* bs;
    int rows, rows4;
    __device__ __forceinline__ const int8_t* q(int m, int t) const { return qs + (t * rows + m) * QK; }
    __device__ __forceinline__ float dx(int m, int t) const { return d[t * rows4 + m]; }
    __device__ __forceinline__ const int16_t* bsums(int m, int t) const { return bs + (t * rows + m) * 16; }
};

template <int TYPE, int M>
__device__ __forceinline__ void block_dot_k45(const uint8_t* __restrict__ tile, int r, const Q8Smem& q8, int b,
                                              float* acc) {
    const KHeader hd = unpack_header(*reinterpret_cast<const uint4*>(tile + r * 16));
    uint32_t qh[8];
    if (TYPE == TYPE_Q5_K) {
        const uint4 h0 = *reinterpret_cast<const uint4*>(tile + 1 * 512 + r * 16);
        const uint4 h1 = *reinterpret_cast<const uint4*>(tile + 2 * 512 + r * 16);
        qh[0] = h0.x; qh[1] = h0.y; qh[2] = h0.z; qh[3] = h0.w;
        qh[4] = h1.x; qh[5] = h1.y; qh[6] = h1.z; qh[7] = h1.w;
    }
    constexpr int QS_CHUNK = (TYPE == TYPE_Q5_K) ? 3 : 1;
    int S[M];
#pragma unroll
    for (int m = 0; m < M; m++) S[m] = 0;
#pragma unroll
    for (int gg = 0; gg < 4; gg++) {
        const uint4 c0 = *reinterpret_cast<const uint4*>(tile + (QS_CHUNK + 2 * gg) * 512 + r * 16);
        const uint4 c1 = *reinterpret_cast<const uint4*>(tile + (QS_CHUNK + 1 + 2 * gg) * 512 + r * 16);
        const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        // lo: low nibbles; hi16: high nibbles left in place (16 x value), so
        // no shift is needed; the 16 is divided out exactly after the dots.
        uint32_t lo[8], hi16[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            lo[i] = w[i] & 0x0f0f0f0fu;
            hi16[i] = w[i] & 0xf0f0f0f0u;
            if (TYPE == TYPE_Q5_K) {
                lo[i] |= ((qh[i] >> (2 * gg)) & 0x01010101u) << 4;
                hi16[i] = (hi16[i] >> 4) | (((qh[i] >> (2 * gg + 1)) & 0x01010101u) << 4);
            }
        }
        const int scl = k_scale(hd, 2 * gg), sch = k_scale(hd, 2 * gg + 1);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4* qv = reinterpret_cast<const int4*>(q8.q(m, b) + 64 * gg);
            const int4 a0 = qv[0], a1 = qv[1], a2 = qv[2], a3 = qv[3];
            int sl0 = dp4a_us(lo[0], a0.x, 0), sl1 = dp4a_us(lo[1], a0.y, 0);
            sl0 = dp4a_us(lo[2], a0.z, sl0); sl1 = dp4a_us(lo[3], a0.w, sl1);
            sl0 = dp4a_us(lo[4], a1.x, sl0); sl1 = dp4a_us(lo[5], a1.y, sl1);
            sl0 = dp4a_us(lo[6], a1.z, sl0); sl1 = dp4a_us(lo[7], a1.w, sl1);
            int sh0 = dp4a_us(hi16[0], a2.x, 0), sh1 = dp4a_us(hi16[1], a2.y, 0);
            sh0 = dp4a_us(hi16[2], a2.z, sh0); sh1 = dp4a_us(hi16[3], a2.w, sh1);
            sh0 = dp4a_us(hi16[4], a3.x, sh0); sh1 = dp4a_us(hi16[5], a3.y, sh1);
            sh0 = dp4a_us(hi16[6], a3.z, sh0); sh1 = dp4a_us(hi16[7], a3.w, sh1);
            const int sh = (TYPE == TYPE_Q5_K) ? (sh0 + sh1) : ((sh0 + sh1) >> 4);
            S[m] += scl * (sl0 + sl1) + sch * sh;
        }
    }
    // Mins: sum_j m_j * (bsums[2j] + bsums[2j+1]) with dp2a against [m_j, m_j]
    // byte pairs (6-bit mins are non-negative bytes).
    const uint32_t mp0 = __byte_perm(hd.mn_lo, 0u, 0x1100u), mp1 = __byte_perm(hd.mn_lo, 0u, 0x3322u);
    const uint32_t mp2 = __byte_perm(hd.mn_hi, 0u, 0x1100u), mp3 = __byte_perm(hd.mn_hi, 0u, 0x3322u);
#pragma unroll
    for (int m = 0; m < M; m++) {
        const int4 b0 = *reinterpret_cast<const int4*>(q8.bsums(m, b));
        const int4 b1 = *reinterpret_cast<const int4*>(q8.bsums(m, b) + 8);
        int mn = __dp2a_lo(b0.x, (int)mp0, 0);
        mn = __dp2a_hi(b0.y, (int)mp0, mn);
        mn = __dp2a_lo(b0.z, (int)mp1, mn);
        mn = __dp2a_hi(b0.w, (int)mp1, mn);
        mn = __dp2a_lo(b1.x, (int)mp2, mn);
        mn = __dp2a_hi(b1.y, (int)mp2, mn);
        mn = __dp2a_lo(b1.z, (int)mp3, mn);
        mn = __dp2a_hi(b1.w, (int)mp3, mn);
        const float dx = q8.dx(m, b);
        acc[m] = fmaf(hd.d * dx, (float)S[m], acc[m]);
        acc[m] = fmaf(-(hd.dmin * dx), (float)mn, acc[m]);
    }
}

template <int M>
__device__ __forceinline__ void block_dot_q6k(const uint8_t* __restrict__ tile, int r, const Q8Smem& q8, int b,
                                              float* acc) {
    const float d = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(tile + Fmt<TYPE_Q6_K>::D_OFFSET + r * 2));
    const uint4 scv = *reinterpret_cast<const uint4*>(tile + 12 * 512 + r * 16);
    const uint32_t s4[4] = {scv.x, scv.y, scv.z, scv.w};
    int S[M];
#pragma unroll
    for (int m = 0; m < M; m++) S[m] = 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int lg = 0; lg < 2; lg++) {
            const uint4 A = *reinterpret_cast<const uint4*>(tile + (4 * h + lg) * 512 + r * 16);
            const uint4 B = *reinterpret_cast<const uint4*>(tile + (4 * h + 2 + lg) * 512 + r * 16);
            const uint4 H = *reinterpret_cast<const uint4*>(tile + (8 + 2 * h + lg) * 512 + r * 16);
            const uint32_t a[4] = {A.x, A.y, A.z, A.w};
            const uint32_t bq[4] = {B.x, B.y, B.z, B.w};
            const uint32_t hh[4] = {H.x, H.y, H.z, H.w};
            int q1[4], q2[4], q3[4], q4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                q1[i] = (int)((a[i] & 0x0f0f0f0fu) | ((hh[i] << 4) & 0x30303030u));
                q2[i] = (int)((bq[i] & 0x0f0f0f0fu) | ((hh[i] << 2) & 0x30303030u));
                q3[i] = (int)(((a[i] >> 4) & 0x0f0f0f0fu) | (hh[i] & 0x30303030u));
                q4[i] = (int)(((bq[i] >> 4) & 0x0f0f0f0fu) | ((hh[i] >> 2) & 0x30303030u));
            }
            // 16-value sub-block scales 8h+lg, +2, +4, +6 (signed bytes).
            const int s1 = sext_byte(s4[2 * h], lg), s2 = sext_byte(s4[2 * h], 2 + lg);
            const int s3 = sext_byte(s4[2 * h + 1], lg), s4v = sext_byte(s4[2 * h + 1], 2 + lg);
#pragma unroll
            for (int m = 0; m < M; m++) {
                const int8_t* base = q8.q(m, b) + 128 * h + 16 * lg;
                const int4 x1 = *reinterpret_cast<const int4*>(base);
                const int4 x2 = *reinterpret_cast<const int4*>(base + 32);
                const int4 x3 = *reinterpret_cast<const int4*>(base + 64);
                const int4 x4 = *reinterpret_cast<const int4*>(base + 96);
                int d1 = dp4a(q1[0], x1.x, 0); d1 = dp4a(q1[1], x1.y, d1); d1 = dp4a(q1[2], x1.z, d1); d1 = dp4a(q1[3], x1.w, d1);
                int d2 = dp4a(q2[0], x2.x, 0); d2 = dp4a(q2[1], x2.y, d2); d2 = dp4a(q2[2], x2.z, d2); d2 = dp4a(q2[3], x2.w, d2);
                int d3 = dp4a(q3[0], x3.x, 0); d3 = dp4a(q3[1], x3.y, d3); d3 = dp4a(q3[2], x3.z, d3); d3 = dp4a(q3[3], x3.w, d3);
                int d4 = dp4a(q4[0], x4.x, 0); d4 = dp4a(q4[1], x4.y, d4); d4 = dp4a(q4[2], x4.z, d4); d4 = dp4a(q4[3], x4.w, d4);
                S[m] += s1 * d1 + s2 * d2 + s3 * d3 + s4v * d4;
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        // -32 bias folded through the Q8_K block sums (Kernels/Q6K.cs:105-108):
        // sum_j sc_j * bsums_j with dp2a (int16 bsums x signed-byte scales).
        const int4 b0 = *reinterpret_cast<const int4*>(q8.bsums(m, b));
        const int4 b1 = *reinterpret_cast<const int4*>(q8.bsums(m, b) + 8);
        int bias = __dp2a_lo(b0.x, (int)s4[0], 0);
        bias = __dp2a_hi(b0.y, (int)s4[0], bias);
        bias = __dp2a_lo(b0.z, (int)s4[1], bias);
        bias = __dp2a_hi(b0.w, (int)s4[1], bias);
        bias = __dp2a_lo(b1.x, (int)s4[2], bias);
        bias = __dp2a_hi(b1.y, (int)s4[2], bias);
        bias = __dp2a_lo(b1.z, (int)s4[3], bias);
        bias = __dp2a_hi(b1.w, (int)s4[3], bias);
        acc[m] = fmaf(d * q8.dx(m, b), (float)(S[m] - 32 * bias), acc[m]);
    }
}

// ---------------------------------------------------------------------------
// Tensor-core form for 3..8 tokens (6..8 for Q6_K; q8_interleave_min_rows)
// (legacy mma.sync: the weights' decode, not the MACs, bounds this
// HBM-streaming kernel, so the point is fewer instructions per weight, not
// tcgen05 throughput).  Its cost per tile does not depend on the token count
// (an mma always spans 8 token columns), while the dp4a form's grows with it.  A warp computes its
// 32-row tile as two m16 halves x 8 token columns.  Lane (g = lane/4,
// c = lane%4) supplies rows g, g+8 of a half and token g of the B operand:
//   * integer dots per sub-block: mma m16n8k32 u8 x s8 (Q4_K/Q5_K, 32-value
//     sub-blocks) or m16n8k16 (Q6_K, 16-value sub-blocks), A = the unpacked
//     quants, B = Q8_K words read from the word-interleaved planar qs
//     (device_common.cuh): in every 16-value group the lane takes values
//     4c..4c+3, so each operand word is one 32-bit load for both sides;
//   * exact int32 S per (row, token, block) = sum of sc_j x D_j;
//   * the mins (Q4_K/Q5_K) or the -32 bias (Q6_K) sum_k coef[row][k] *
//     bsums[token][k] as one m16n8k16 f16 mma per half: coefficients
//     (<= 63, or |sc| <= 128) and block sums (|bsum| <= 2032) are exact in
//     fp16 and every partial sum stays below 2^24, so the fp32 result is exact;
//   * acc += (d*dx)*S - (dmin*dx)*Mn in fp32, as the dp4a form.
// Result fragment (both mma shapes): D[0] = (row g, token 2c), D[1] = (g,
// 2c+1), D[2] = (g+8, 2c), D[3] = (g+8, 2c+1).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void imma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
__device__ __forceinline__ void hmma_k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
// Two small integers (|v| < 2048) as an fp16 pair (exact).
__device__ __forceinline__ uint32_t half2_of(int lo, int hi) {
    const __half2 h = __halves2half2(__int2half_rn(lo), __int2half_rn(hi));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Per-block operands shared by both halves of a tile: the B words of token g
// (zero for g >= M), its block sums as fp16 pairs for the coefficient mma and
// the d of tokens 2c, 2c+1.
template <int M>
struct MmaB {
    uint32_t w[16];  // B word of 16-value group s, values 4c..4c+3
    uint32_t bs0, bs1;
    float dx0, dx1;
    __device__ __forceinline__ void load(const Q8Smem& q8, int b, int g, int c) {
        const uint32_t* qs = reinterpret_cast<const uint32_t*>(q8.qs + (size_t)b * M * QK);
#pragma unroll
        for (int s = 0; s < 16; s++) w[s] = g < M ? qs[(4 * s + c) * M + g] : 0u;
        if (g < M) {
            const int16_t* bs = q8.bsums(g, b);
            const uint32_t p0 = *reinterpret_cast<const uint32_t*>(bs + 2 * c);
            const uint32_t p1 = *reinterpret_cast<const uint32_t*>(bs + 8 + 2 * c);
            bs0 = half2_of((int)(int16_t)(p0 & 0xffffu), (int)(int16_t)(p0 >> 16));
            bs1 = half2_of((int)(int16_t)(p1 & 0xffffu), (int)(int16_t)(p1 >> 16));
        } else {
            bs0 = bs1 = 0u;
        }
        dx0 = 2 * c < M ? q8.dx(2 * c, b) : 0.f;
        dx1 = 2 * c + 1 < M ? q8.dx(2 * c + 1, b) : 0.f;
    }
};

// acc[i][j] (row g + 8i of the half, token 2c + j) += (d_i dx_j) S - (dmin_i dx_j) cf
// (Q4_K/Q5_K), or (d_i dx_j) (S - 32 cf) with Q6_BIAS (cf = the bias sums).
template <bool Q6_BIAS>
__device__ __forceinline__ void mma_epilogue(float (&acc)[2][2], const int (&S)[4], const float (&cf)[4], float d0,
                                             float d1, float m0, float m1, float dx0, float dx1) {
    const float dx[2] = {dx0, dx1};
    const float dd[2] = {d0, d1}, dm[2] = {m0, m1};
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int k = 2 * i + j;
            if (Q6_BIAS) {
                acc[i][j] = fmaf(dd[i] * dx[j], (float)(S[k] - 32 * (int)cf[k]), acc[i][j]);
            } else {
                acc[i][j] = fmaf(dd[i] * dx[j], (float)S[k], acc[i][j]);
                acc[i][j] = fmaf(-(dm[i] * dx[j]), cf[k], acc[i][j]);
            }
        }
}

template <int TYPE, int M>
__device__ __forceinline__ void half_dot_k45(const uint8_t* __restrict__ tile, int r0, int c, const MmaB<M>& B,
                                             float (&acc)[2][2]) {
    const int r1 = r0 + 8;
    const KHeader h0 = unpack_header(*reinterpret_cast<const uint4*>(tile + r0 * 16));
    const KHeader h1 = unpack_header(*reinterpret_cast<const uint4*>(tile + r1 * 16));
    constexpr int QS_CHUNK = (TYPE == TYPE_Q5_K) ? 3 : 1;
    uint32_t qh00 = 0, qh01 = 0, qh10 = 0, qh11 = 0;  // qh bytes 4c.. and 16+4c.. of rows r0, r1
    if (TYPE == TYPE_Q5_K) {
        qh00 = *reinterpret_cast<const uint32_t*>(tile + 1 * 512 + r0 * 16 + 4 * c);
        qh01 = *reinterpret_cast<const uint32_t*>(tile + 2 * 512 + r0 * 16 + 4 * c);
        qh10 = *reinterpret_cast<const uint32_t*>(tile + 1 * 512 + r1 * 16 + 4 * c);
        qh11 = *reinterpret_cast<const uint32_t*>(tile + 2 * 512 + r1 * 16 + 4 * c);
    }
    int S[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < 4; p++) {
        // qs bytes 32p + 4c.. (chunk QS_CHUNK + 2p) and 32p + 16 + 4c.. (next chunk)
        const uint32_t w00 = *reinterpret_cast<const uint32_t*>(tile + (QS_CHUNK + 2 * p) * 512 + r0 * 16 + 4 * c);
        const uint32_t w01 = *reinterpret_cast<const uint32_t*>(tile + (QS_CHUNK + 2 * p + 1) * 512 + r0 * 16 + 4 * c);
        const uint32_t w10 = *reinterpret_cast<const uint32_t*>(tile + (QS_CHUNK + 2 * p) * 512 + r1 * 16 + 4 * c);
        const uint32_t w11 = *reinterpret_cast<const uint32_t*>(tile + (QS_CHUNK + 2 * p + 1) * 512 + r1 * 16 + 4 * c);
        uint32_t lo00 = w00 & 0x0f0f0f0fu, lo01 = w01 & 0x0f0f0f0fu, lo10 = w10 & 0x0f0f0f0fu, lo11 = w11 & 0x0f0f0f0fu;
        uint32_t hi00, hi01, hi10, hi11;
        if (TYPE == TYPE_Q5_K) {
            lo00 |= ((qh00 >> (2 * p)) & 0x01010101u) << 4;
            lo01 |= ((qh01 >> (2 * p)) & 0x01010101u) << 4;
            lo10 |= ((qh10 >> (2 * p)) & 0x01010101u) << 4;
            lo11 |= ((qh11 >> (2 * p)) & 0x01010101u) << 4;
            hi00 = ((w00 >> 4) & 0x0f0f0f0fu) | (((qh00 >> (2 * p + 1)) & 0x01010101u) << 4);
            hi01 = ((w01 >> 4) & 0x0f0f0f0fu) | (((qh01 >> (2 * p + 1)) & 0x01010101u) << 4);
            hi10 = ((w10 >> 4) & 0x0f0f0f0fu) | (((qh10 >> (2 * p + 1)) & 0x01010101u) << 4);
            hi11 = ((w11 >> 4) & 0x0f0f0f0fu) | (((qh11 >> (2 * p + 1)) & 0x01010101u) << 4);
        } else {
            // high nibbles left in place: 16 x the value, divided out below
            hi00 = w00 & 0xf0f0f0f0u;
            hi01 = w01 & 0xf0f0f0f0u;
            hi10 = w10 & 0xf0f0f0f0u;
            hi11 = w11 & 0xf0f0f0f0u;
        }
        int dl[4], dh[4];
        imma_k32(dl, lo00, lo10, lo01, lo11, B.w[4 * p], B.w[4 * p + 1]);
        imma_k32(dh, hi00, hi10, hi01, hi11, B.w[4 * p + 2], B.w[4 * p + 3]);
        const int sl0 = k_scale(h0, 2 * p), sh0 = k_scale(h0, 2 * p + 1);
        const int sl1 = k_scale(h1, 2 * p), sh1 = k_scale(h1, 2 * p + 1);
        if (TYPE == TYPE_Q5_K) {
            S[0] += sl0 * dl[0] + sh0 * dh[0];
            S[1] += sl0 * dl[1] + sh0 * dh[1];
            S[2] += sl1 * dl[2] + sh1 * dh[2];
            S[3] += sl1 * dl[3] + sh1 * dh[3];
        } else {
            // in units of 1/16: |16 S| <= 16 * 256*63*15*127 < 2^31
            S[0] += 16 * sl0 * dl[0] + sh0 * dh[0];
            S[1] += 16 * sl0 * dl[1] + sh0 * dh[1];
            S[2] += 16 * sl1 * dl[2] + sh1 * dh[2];
            S[3] += 16 * sl1 * dl[3] + sh1 * dh[3];
        }
    }
    if (TYPE != TYPE_Q5_K)
#pragma unroll
        for (int k = 0; k < 4; k++) S[k] >>= 4;  // exact: every term is a multiple of 16
    // Mins: A[row][k] = m_{k/2}; the lane supplies k = 2c, 2c+1 (m_c) and 8+2c, 9+2c (m_{4+c}).
    const int mc0 = byte_of(h0.mn_lo, c), mc4_0 = byte_of(h0.mn_hi, c);
    const int mc1 = byte_of(h1.mn_lo, c), mc4_1 = byte_of(h1.mn_hi, c);
    float mn[4];
    hmma_k16(mn, half2_of(mc0, mc0), half2_of(mc1, mc1), half2_of(mc4_0, mc4_0), half2_of(mc4_1, mc4_1), B.bs0,
             B.bs1);
    mma_epilogue<false>(acc, S, mn, h0.d, h1.d, h0.dmin, h1.dmin, B.dx0, B.dx1);
}

template <int M>
__device__ __forceinline__ void half_dot_q6k(const uint8_t* __restrict__ tile, int r0, int c, const MmaB<M>& B,
                                             float (&acc)[2][2]) {
    const int r1 = r0 + 8;
    const float d0 = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(tile + Fmt<TYPE_Q6_K>::D_OFFSET + r0 * 2));
    const float d1 = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(tile + Fmt<TYPE_Q6_K>::D_OFFSET + r1 * 2));
    const uint4 sv0 = *reinterpret_cast<const uint4*>(tile + 12 * 512 + r0 * 16);
    const uint4 sv1 = *reinterpret_cast<const uint4*>(tile + 12 * 512 + r1 * 16);
    const uint32_t s0[4] = {sv0.x, sv0.y, sv0.z, sv0.w}, s1[4] = {sv1.x, sv1.y, sv1.z, sv1.w};
    int S[4] = {0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int lg = 0; lg < 2; lg++) {
            uint32_t q[2][4];  // [row][quarter]: values 128h + 32*quarter + 16lg + 4c..+3
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int r = rr ? r1 : r0;
                const uint32_t a = *reinterpret_cast<const uint32_t*>(tile + (4 * h + lg) * 512 + r * 16 + 4 * c);
                const uint32_t bq = *reinterpret_cast<const uint32_t*>(tile + (4 * h + 2 + lg) * 512 + r * 16 + 4 * c);
                const uint32_t hh = *reinterpret_cast<const uint32_t*>(tile + (8 + 2 * h + lg) * 512 + r * 16 + 4 * c);
                q[rr][0] = (a & 0x0f0f0f0fu) | ((hh << 4) & 0x30303030u);
                q[rr][1] = (bq & 0x0f0f0f0fu) | ((hh << 2) & 0x30303030u);
                q[rr][2] = ((a >> 4) & 0x0f0f0f0fu) | (hh & 0x30303030u);
                q[rr][3] = ((bq >> 4) & 0x0f0f0f0fu) | ((hh >> 2) & 0x30303030u);
            }
#pragma unroll
            for (int qq = 0; qq < 4; qq++) {
                const int s = 8 * h + 2 * qq + lg;  // 16-value group
                int dq[4];
                imma_k16(dq, q[0][qq], q[1][qq], B.w[s]);
                const int sc0 = sext_byte(s0[s >> 2], s & 3), sc1 = sext_byte(s1[s >> 2], s & 3);
                S[0] += sc0 * dq[0];
                S[1] += sc0 * dq[1];
                S[2] += sc1 * dq[2];
                S[3] += sc1 * dq[3];
            }
        }
    }
    // -32 bias: sum_s sc_s * bsums_s; the lane supplies s = 2c, 2c+1 and 8+2c, 9+2c.
    const int w0 = c >> 1, b0 = 2 * (c & 1);
    float bias[4];
    hmma_k16(bias, half2_of(sext_byte(s0[w0], b0), sext_byte(s0[w0], b0 + 1)),
             half2_of(sext_byte(s1[w0], b0), sext_byte(s1[w0], b0 + 1)),
             half2_of(sext_byte(s0[2 + w0], b0), sext_byte(s0[2 + w0], b0 + 1)),
             half2_of(sext_byte(s1[2 + w0], b0), sext_byte(s1[2 + w0], b0 + 1)), B.bs0, B.bs1);
    mma_epilogue<true>(acc, S, bias, d0, d1, 0.f, 0.f, B.dx0, B.dx1);
}

// One 32-row tile (one super-block) for 3..8 tokens; acc[half][i][j] = row
// 16*half + g + 8i, token 2c + j.
template <int TYPE, int M>
__device__ __forceinline__ void tile_dot_mma(const uint8_t* tile, int lane, const MmaB<M>& B,
                                             float (&acc)[2][2][2]) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
        if (TYPE == TYPE_Q6_K)
            half_dot_q6k<M>(tile, 16 * hf + g, c, B, acc[hf]);
        else
            half_dot_k45<TYPE, M>(tile, 16 * hf + g, c, B, acc[hf]);
    }
}

template <int TYPE, int M>
__device__ __forceinline__ void tile_dot(const uint8_t* tile, int lane, const Q8Smem& q8, int b, float* acc) {
    if (TYPE == TYPE_Q6_K)
        block_dot_q6k<M>(tile, lane, q8, b, acc);
    else
        block_dot_k45<TYPE, M>(tile, lane, q8, b, acc);
}


}  // namespace q35k
