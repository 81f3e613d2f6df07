// q8k_quant.cuh -- bit-exact Q8_K quantization of one 256-value super-block
// by one warp, shared by the standalone quantizer and the GEMV's fused
// prologue (both must produce the same bytes).
//
// Follows Q8K.QuantizeRow + Q8K.ScaleBlock (Kernels/Q8K.cs:12-146):
//   amax = max |x|; max = the first element (lowest index) with |x| == amax,
//   sign kept; iscale = -127/max; d = 1/iscale (a true reciprocal);
//   q = clamp(round_half_even(x * iscale), -127, 127); bsums = sums of 16.
//   amax == 0 -> an all-zero block (d = 0).
// Every fp32 operation is an explicitly rounded intrinsic (__fdiv_rn,
// __fmul_rn, __float2int_rn), so nvcc cannot contract or reassociate it; each
// mirrors one separately rounded C# operation of the reference.
// Lane l owns values 4l..4l+3 and 128+4l..128+4l+3 (two coalesced float4s).
#pragma once

#include "device_common.cuh"

namespace q35k {

struct Q8Out {
    uint32_t* d;        // the block's d word
    uint32_t* qs;       // 64 words of qs: word w (values 4w..4w+3) at qs[w * qs_stride]
    int16_t* bs;        // 16 bsums
    int qs_stride = 1;  // > 1: the words of several rows interleaved (planar chunks of >= 3 rows)
};

// The quantization itself: returns d (the same value on every lane) and this
// lane's eight q values (q[0..3] = values 4l..4l+3, q[4..7] = 128+4l..+3).
// An all-zero block gives d = 0 and q = 0.  src: 256 floats, 16-byte aligned.
// With `up` (ffn_down's input): the block quantized is silu(src) * up, SiLU
// as g / (1 + exp(-g)) in fp32 (Ops.SiLUMul, Qwen35Sharp.Model/Ops.cs:624-675).
__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

// This lane's eight values of the block (silu(src) * up with `up`).
__device__ __forceinline__ void warp_q8k_load(const float* __restrict__ src, int lane, float (&v)[8],
                                              const float* __restrict__ up = nullptr) {
    float4 v0 = __ldg(reinterpret_cast<const float4*>(src) + lane);
    float4 v1 = __ldg(reinterpret_cast<const float4*>(src + 128) + lane);
    if (up) {
        const float4 u0 = __ldg(reinterpret_cast<const float4*>(up) + lane);
        const float4 u1 = __ldg(reinterpret_cast<const float4*>(up + 128) + lane);
        v0 = make_float4(silu_mul(v0.x, u0.x), silu_mul(v0.y, u0.y), silu_mul(v0.z, u0.z), silu_mul(v0.w, u0.w));
        v1 = make_float4(silu_mul(v1.x, u1.x), silu_mul(v1.y, u1.y), silu_mul(v1.z, u1.z), silu_mul(v1.w, u1.w));
    }
    v[0] = v0.x, v[1] = v0.y, v[2] = v0.z, v[3] = v0.w;
    v[4] = v1.x, v[5] = v1.y, v[6] = v1.z, v[7] = v1.w;
}

// The quantization of values loaded by warp_q8k_load.
__device__ __forceinline__ float warp_q8k_quantize(const float (&v)[8], int lane, int (&q)[8]) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
    // fmaxf drops NaNs, so every lane's amax is a non-negative number, whose
    // bit pattern orders like its value: one integer max over the warp.
    amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(amax)));

    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = 0;
        return 0.f;
    }
    // First index whose |x| equals amax, and its signed value.  Every index
    // of the low half (4*lane + i, i < 4) precedes every index of the high
    // half (128 + 4*lane + i - 4), and within a half lanes go in index
    // order: the first hit is the lowest lane's first hit in the low half if
    // any lane has one, else the lowest lane's first hit in the high half.
    float vlo = 0.f, vhi = 0.f;
    bool hlo = false, hhi = false;
#pragma unroll
    for (int i = 3; i >= 0; i--)
        if (fabsf(v[i]) == amax) hlo = true, vlo = v[i];
#pragma unroll
    for (int i = 7; i >= 4; i--)
        if (fabsf(v[i]) == amax) hhi = true, vhi = v[i];
    const unsigned mlo = __ballot_sync(0xffffffffu, hlo), mhi = __ballot_sync(0xffffffffu, hhi);
    const float val = __shfl_sync(0xffffffffu, mlo ? vlo : vhi, __ffs(mlo ? mlo : mhi) - 1);
    const float iscale = __fdiv_rn(-127.f, val);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int t = __float2int_rn(__fmul_rn(v[i], iscale));
        q[i] = min(127, max(-127, t));
    }
    return __fdiv_rn(1.f, iscale);
}

__device__ __forceinline__ float warp_q8k_values(const float* __restrict__ src, int lane, int (&q)[8],
                                                 const float* __restrict__ up = nullptr) {
    float v[8];
    warp_q8k_load(src, lane, v, up);
    return warp_q8k_quantize(v, lane, q);
}

// The four q values (each in [-127, 127]) as the bytes of one word, lowest first.
__device__ __forceinline__ uint32_t pack_q4(int a, int b, int c, int d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// Sums of 16 of the packed values: s0 = bsums[lane/4] and s1 = bsums[8 + lane/4],
// valid on lanes with lane % 4 == 0.
__device__ __forceinline__ void warp_q8k_bsums(uint32_t w0, uint32_t w1, int& s0, int& s1) {
    s0 = __dp4a((int)w0, 0x01010101, 0);
    s1 = __dp4a((int)w1, 0x01010101, 0);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
}

// src: 256 floats, 16-byte aligned.  Writes d, qs, bsums through `out`.
__device__ __forceinline__ void warp_quantize_q8k_block(const float* __restrict__ src, const Q8Out& out, int lane,
                                                        const float* __restrict__ up = nullptr) {
    int q[8];
    const float d = warp_q8k_values(src, lane, q, up);
    if (lane == 0) *out.d = __float_as_uint(d);
    const uint32_t w0 = pack_q4(q[0], q[1], q[2], q[3]);
    const uint32_t w1 = pack_q4(q[4], q[5], q[6], q[7]);
    out.qs[lane * out.qs_stride] = w0;
    out.qs[(32 + lane) * out.qs_stride] = w1;
    int s0, s1;
    warp_q8k_bsums(w0, w1, s0, s1);
    if ((lane & 3) == 0) {
        out.bs[lane >> 2] = static_cast<int16_t>(s0);
        out.bs[8 + (lane >> 2)] = static_cast<int16_t>(s1);
    }
}

}  // namespace q35k
