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

template <int TYPE, int M>
__device__ __forceinline__ void tile_dot(const uint8_t* tile, int lane, const Q8Smem& q8, int b, float* acc) {
    if (TYPE == TYPE_Q6_K)
        block_dot_q6k<M>(tile, lane, q8, b, acc);
    else
        block_dot_k45<TYPE, M>(tile, lane, q8, b, acc);
}


}  // namespace q35k
