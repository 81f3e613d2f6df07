// gemv.cu -- decode GEMV (1..8 tokens) for Q4_K / Q5_K / Q6_K weights.
//
// Memory-bound design (no tensor cores):
//   * a CTA owns one 32-row group and a contiguous range of super-blocks
//     (split-K when the matrix is too small to fill the GPU);
//   * one thread issues every weight tile of the CTA as a 1-D bulk async copy
//     (cp.async.bulk, no multicast) into shared memory at once, one mbarrier
//     per tile, so the whole unit is in flight while compute starts on the
//     first tile;
//   * lane r of each warp decodes row r of a tile: the chunk-major tile layout
//     makes every 16-byte load a contiguous 512-byte line per warp, and all
//     lanes read the same Q8_K activation words (shared-memory broadcast);
//   * integer dots with dp4a into exact int32 per super-block, scaled in fp32
//     once per block: acc += (d_w*d_x)*S - (dmin_w*d_x)*Mn
//     (VecDotQ4K.DotScalar, Kernels/VecDotQ4K.cs:42-61; Q5K.Dot,
//     Kernels/Q5K.cs:62-83; Q6K.DotAvx2's bias form, Kernels/Q6K.cs:105-108,159);
//   * warps split the tiles, reduce through shared memory; split-K partials
//     are combined by the last-arriving CTA of a row group in fixed order
//     (deterministic), which also resets the group's counter.
#include "device_common.cuh"
#include "kernels.h"

#include <algorithm>

namespace q35k {

constexpr int GEMV_WARPS = 4;
constexpr int GEMV_MAX_TOKENS = 8;
constexpr int GEMV_TARGET_UNIT_BYTES = 72 * 1024;

__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct SmemLayout {
    int bars, flags, tiles, q8s, q8d, q8b, red, total;
};

// Dynamic shared memory of one GEMV CTA (all offsets 16-byte aligned):
// mbarriers | 2 int flags | weight tiles | Q8_K qs | Q8_K d | Q8_K bsums |
// cross-warp reduction buffer.
__host__ __device__ inline SmemLayout gemv_smem_layout(int tile_bytes, int bps, int m) {
    SmemLayout L;
    L.bars = 0;
    L.flags = 8 * bps;
    L.tiles = align_up(L.flags + 8, 128);
    L.q8s = L.tiles + bps * tile_bytes;
    L.q8d = L.q8s + m * bps * QK;
    L.q8b = L.q8d + align_up(m * bps * 4, 16);
    L.red = L.q8b + align_up(m * bps * 32, 16);
    L.total = L.red + GEMV_WARPS * m * 32 * 4;
    return L;
}

__device__ __forceinline__ int byte_of(uint32_t w, int k) { return (w >> (8 * k)) & 0xff; }
__device__ __forceinline__ int sbyte_of(uint32_t w, int k) { return (int)(int8_t)((w >> (8 * k)) & 0xff); }

// Q4_K / Q5_K header: fp16 d, fp16 dmin, 12 bytes of 6-bit scales/mins.
// Unpacked as Q4K.UnpackScales (Kernels/Q4K.cs:20-33).
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
__device__ __forceinline__ int k_scale(const KHeader& k, int j) {
    return byte_of(j < 4 ? k.sc_lo : k.sc_hi, j & 3);
}
__device__ __forceinline__ int k_min(const KHeader& k, int j) { return byte_of(j < 4 ? k.mn_lo : k.mn_hi, j & 3); }

// Sum_j mins_j * (bsums[2j] + bsums[2j+1]) from the 16 int16 bsums.
__device__ __forceinline__ int mins_dot(const KHeader& k, const int16_t* bs) {
    const int4 b0 = *reinterpret_cast<const int4*>(bs);
    const int4 b1 = *reinterpret_cast<const int4*>(bs + 8);
    const uint32_t w[8] = {(uint32_t)b0.x, (uint32_t)b0.y, (uint32_t)b0.z, (uint32_t)b0.w,
                           (uint32_t)b1.x, (uint32_t)b1.y, (uint32_t)b1.z, (uint32_t)b1.w};
    int mn = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int pair = (int)(int16_t)(w[j] & 0xffffu) + (int)(int16_t)(w[j] >> 16);
        mn += k_min(k, j) * pair;
    }
    return mn;
}

template <int TYPE, int M>
__device__ __forceinline__ void block_dot_k45(const uint8_t* __restrict__ tile, int r, const int8_t* q8s,
                                              const float* q8d, const int16_t* q8b, int t, int bps, float* acc) {
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
        int lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t l = w[i] & 0x0f0f0f0fu;
            uint32_t h = (w[i] >> 4) & 0x0f0f0f0fu;
            if (TYPE == TYPE_Q5_K) {
                l |= ((qh[i] >> (2 * gg)) & 0x01010101u) << 4;
                h |= ((qh[i] >> (2 * gg + 1)) & 0x01010101u) << 4;
            }
            lo[i] = (int)l;
            hi[i] = (int)h;
        }
        const int scl = k_scale(hd, 2 * gg), sch = k_scale(hd, 2 * gg + 1);
#pragma unroll
        for (int m = 0; m < M; m++) {
            const int4* qv = reinterpret_cast<const int4*>(q8s + (m * bps + t) * QK + 64 * gg);
            const int4 a0 = qv[0], a1 = qv[1], a2 = qv[2], a3 = qv[3];
            int sl = dp4a(lo[0], a0.x, 0);
            sl = dp4a(lo[1], a0.y, sl); sl = dp4a(lo[2], a0.z, sl); sl = dp4a(lo[3], a0.w, sl);
            sl = dp4a(lo[4], a1.x, sl); sl = dp4a(lo[5], a1.y, sl); sl = dp4a(lo[6], a1.z, sl);
            sl = dp4a(lo[7], a1.w, sl);
            int sh = dp4a(hi[0], a2.x, 0);
            sh = dp4a(hi[1], a2.y, sh); sh = dp4a(hi[2], a2.z, sh); sh = dp4a(hi[3], a2.w, sh);
            sh = dp4a(hi[4], a3.x, sh); sh = dp4a(hi[5], a3.y, sh); sh = dp4a(hi[6], a3.z, sh);
            sh = dp4a(hi[7], a3.w, sh);
            S[m] += scl * sl + sch * sh;
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        const int Mn = mins_dot(hd, q8b + (m * bps + t) * 16);
        const float dx = q8d[m * bps + t];
        acc[m] = fmaf(hd.d * dx, (float)S[m], acc[m]);
        acc[m] = fmaf(-(hd.dmin * dx), (float)Mn, acc[m]);
    }
}

template <int M>
__device__ __forceinline__ void block_dot_q6k(const uint8_t* __restrict__ tile, int r, const int8_t* q8s,
                                              const float* q8d, const int16_t* q8b, int t, int bps, float* acc) {
    const float d = fp16_bits_to_float(*reinterpret_cast<const uint16_t*>(tile + Fmt<TYPE_Q6_K>::D_OFFSET + r * 2));
    const uint4 scv = *reinterpret_cast<const uint4*>(tile + 12 * 512 + r * 16);
    int sc[16];
    {
        const uint32_t s4[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
        for (int j = 0; j < 16; j++) sc[j] = sbyte_of(s4[j >> 2], j & 3);
    }
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
            const uint32_t b[4] = {B.x, B.y, B.z, B.w};
            const uint32_t hh[4] = {H.x, H.y, H.z, H.w};
            int q1[4], q2[4], q3[4], q4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                q1[i] = (int)((a[i] & 0x0f0f0f0fu) | ((hh[i] << 4) & 0x30303030u));
                q2[i] = (int)((b[i] & 0x0f0f0f0fu) | ((hh[i] << 2) & 0x30303030u));
                q3[i] = (int)(((a[i] >> 4) & 0x0f0f0f0fu) | (hh[i] & 0x30303030u));
                q4[i] = (int)(((b[i] >> 4) & 0x0f0f0f0fu) | ((hh[i] >> 2) & 0x30303030u));
            }
            const int s1 = sc[8 * h + lg], s2 = sc[8 * h + 2 + lg], s3 = sc[8 * h + 4 + lg], s4 = sc[8 * h + 6 + lg];
#pragma unroll
            for (int m = 0; m < M; m++) {
                const int8_t* base = q8s + (m * bps + t) * QK + 128 * h + 16 * lg;
                const int4 x1 = *reinterpret_cast<const int4*>(base);
                const int4 x2 = *reinterpret_cast<const int4*>(base + 32);
                const int4 x3 = *reinterpret_cast<const int4*>(base + 64);
                const int4 x4 = *reinterpret_cast<const int4*>(base + 96);
                int d1 = dp4a(q1[0], x1.x, 0); d1 = dp4a(q1[1], x1.y, d1); d1 = dp4a(q1[2], x1.z, d1); d1 = dp4a(q1[3], x1.w, d1);
                int d2 = dp4a(q2[0], x2.x, 0); d2 = dp4a(q2[1], x2.y, d2); d2 = dp4a(q2[2], x2.z, d2); d2 = dp4a(q2[3], x2.w, d2);
                int d3 = dp4a(q3[0], x3.x, 0); d3 = dp4a(q3[1], x3.y, d3); d3 = dp4a(q3[2], x3.z, d3); d3 = dp4a(q3[3], x3.w, d3);
                int d4 = dp4a(q4[0], x4.x, 0); d4 = dp4a(q4[1], x4.y, d4); d4 = dp4a(q4[2], x4.z, d4); d4 = dp4a(q4[3], x4.w, d4);
                S[m] += s1 * d1 + s2 * d2 + s3 * d3 + s4 * d4;
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        // -32 bias folded through the Q8_K block sums (Kernels/Q6K.cs:105-108).
        const int4 b0 = *reinterpret_cast<const int4*>(q8b + (m * bps + t) * 16);
        const int4 b1 = *reinterpret_cast<const int4*>(q8b + (m * bps + t) * 16 + 8);
        const uint32_t w[8] = {(uint32_t)b0.x, (uint32_t)b0.y, (uint32_t)b0.z, (uint32_t)b0.w,
                               (uint32_t)b1.x, (uint32_t)b1.y, (uint32_t)b1.z, (uint32_t)b1.w};
        int bias = 0;
#pragma unroll
        for (int j = 0; j < 8; j++)
            bias += sc[2 * j] * (int)(int16_t)(w[j] & 0xffffu) + sc[2 * j + 1] * (int)(int16_t)(w[j] >> 16);
        const float dx = q8d[m * bps + t];
        acc[m] = fmaf(d * dx, (float)(S[m] - 32 * bias), acc[m]);
    }
}

template <int TYPE, int M>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_kernel(GemvArgs a, int splits, int bps, int n_pad) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TILE = Fmt<TYPE>::TILE;
    const SmemLayout L = gemv_smem_layout(TILE, bps, M);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
    uint8_t* wt = smem + L.tiles;
    int8_t* q8s = reinterpret_cast<int8_t*>(smem + L.q8s);
    float* q8d = reinterpret_cast<float*>(smem + L.q8d);
    int16_t* q8b = reinterpret_cast<int16_t*>(smem + L.q8b);
    float* red = reinterpret_cast<float*>(smem + L.red);
    int& s_last = reinterpret_cast<int*>(smem + L.flags)[0];
    int& s_timeout = reinterpret_cast<int*>(smem + L.flags)[1];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.x / splits, s = blockIdx.x % splits;
    const int b0 = s * bps;
    const int kr = min(bps, a.nb - b0);

    if (tid == 0) {
        s_timeout = 0;
        for (int t = 0; t < kr; t++) mbar_init(&bars[t], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        const uint8_t* src = a.tiles + ((size_t)g * a.nb + b0) * TILE;
        for (int t = 0; t < kr; t++) {
            mbar_arrive_expect_tx(&bars[t], TILE);
            bulk_g2s(wt + t * TILE, src + (size_t)t * TILE, TILE, &bars[t]);
        }
    }
    // Stage the K-range of the Q8_K activations: 73 words per block
    // (word 0 = d, 1..64 = qs, 65..72 = bsums).
    for (int idx = tid; idx < M * kr * 73; idx += blockDim.x) {
        const int m = idx / (kr * 73), rem = idx % (kr * 73), t = rem / 73, w = rem % 73;
        const uint32_t v = __ldg(reinterpret_cast<const uint32_t*>(a.q8 + ((size_t)m * a.nb + b0 + t) * Q8K_BYTES) + w);
        if (w == 0)
            q8d[m * bps + t] = __uint_as_float(v);
        else if (w <= 64)
            reinterpret_cast<uint32_t*>(q8s + (m * bps + t) * QK)[w - 1] = v;
        else
            reinterpret_cast<uint32_t*>(q8b + (m * bps + t) * 16)[w - 65] = v;
    }
    __syncthreads();

    float acc[M];
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = 0.f;
    for (int t = warp; t < kr; t += GEMV_WARPS) {
        if (!mbar_wait_bounded(&bars[t], 0, a.err)) {
            s_timeout = 1;
            break;
        }
        if (TYPE == TYPE_Q6_K)
            block_dot_q6k<M>(wt + t * TILE, lane, q8s, q8d, q8b, t, bps, acc);
        else
            block_dot_k45<TYPE, M>(wt + t * TILE, lane, q8s, q8d, q8b, t, bps, acc);
    }
#pragma unroll
    for (int m = 0; m < M; m++) red[(warp * M + m) * 32 + lane] = acc[m];
    __syncthreads();

    const int row = g * TILE_ROWS + lane;
    if (warp == 0) {
#pragma unroll
        for (int m = 0; m < M; m++) {
            float v = red[m * 32 + lane];
#pragma unroll
            for (int w = 1; w < GEMV_WARPS; w++) v += red[(w * M + m) * 32 + lane];
            if (splits == 1) {
                if (row < a.n_out) a.y[(size_t)m * a.ldy + row] = v;
            } else {
                a.partial[((size_t)s * M + m) * n_pad + row] = v;
            }
        }
    }
    if (splits > 1) {
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = (atomicAdd(&a.counters[g], 1) == splits - 1);
        __syncthreads();
        if (s_last && warp == 0) {
            __threadfence();
#pragma unroll
            for (int m = 0; m < M; m++) {
                float v = 0.f;
                for (int k = 0; k < splits; k++) v += __ldcg(&a.partial[((size_t)k * M + m) * n_pad + row]);
                if (row < a.n_out) a.y[(size_t)m * a.ldy + row] = v;
            }
            if (lane == 0) a.counters[g] = 0;
        }
    }
    if (s_timeout) {
        // Give the copies still in flight a bounded chance to land before the
        // CTA's shared memory is released.
        __syncthreads();
        if (tid == 0)
            for (int t = 0; t < kr; t++) mbar_wait_bounded(&bars[t], 0, a.err, 100000000ull);
    }
}

GemvPlan plan_gemv(int type, int nb, int n_out, int tokens, int num_sms) {
    GemvPlan p{};
    const int tile = TILE_ROWS * block_bytes(type);
    p.groups = (n_out + TILE_ROWS - 1) / TILE_ROWS;
    p.n_pad = p.groups * TILE_ROWS;
    const int bps_max = std::max(1, std::min(nb, GEMV_TARGET_UNIT_BYTES / tile));
    int splits = (nb + bps_max - 1) / bps_max;
    while ((long)p.groups * splits < 2L * num_sms && splits < nb) splits++;
    p.bps = (nb + splits - 1) / splits;
    p.splits = (nb + p.bps - 1) / p.bps;
    const int m = std::min(std::max(tokens, 1), GEMV_MAX_TOKENS);
    p.smem_bytes = (size_t)gemv_smem_layout(tile, p.bps, m).total;
    p.partial_bytes = p.splits > 1 ? (size_t)p.splits * GEMV_MAX_TOKENS * p.n_pad * sizeof(float) : 0;
    p.counters = (size_t)p.groups;
    return p;
}

// Opt-in shared memory for every instantiation on the current device
// (called once per context).
constexpr int GEMV_MAX_SMEM = 227 * 1024;

template <int TYPE, int M>
static void configure_typed() {
    cudaFuncSetAttribute(gemv_kernel<TYPE, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
}

template <int TYPE>
static void configure_all_m() {
    configure_typed<TYPE, 1>();
    configure_typed<TYPE, 2>();
    configure_typed<TYPE, 3>();
    configure_typed<TYPE, 4>();
    configure_typed<TYPE, 5>();
    configure_typed<TYPE, 6>();
    configure_typed<TYPE, 7>();
    configure_typed<TYPE, 8>();
}

void configure_gemv_kernels() {
    configure_all_m<TYPE_Q4_K>();
    configure_all_m<TYPE_Q5_K>();
    configure_all_m<TYPE_Q6_K>();
}

template <int TYPE, int M>
static cudaError_t launch_typed(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
    if (p.smem_bytes > (size_t)GEMV_MAX_SMEM) return cudaErrorInvalidConfiguration;
    const unsigned grid = (unsigned)p.groups * (unsigned)p.splits;
    gemv_kernel<TYPE, M><<<grid, GEMV_WARPS * 32, p.smem_bytes, s>>>(a, p.splits, p.bps, p.n_pad);
    return cudaGetLastError();
}

template <int TYPE>
static cudaError_t launch_m(const GemvArgs& a, const GemvPlan& p, cudaStream_t s) {
    switch (a.tokens) {
    case 1: return launch_typed<TYPE, 1>(a, p, s);
    case 2: return launch_typed<TYPE, 2>(a, p, s);
    case 3: return launch_typed<TYPE, 3>(a, p, s);
    case 4: return launch_typed<TYPE, 4>(a, p, s);
    case 5: return launch_typed<TYPE, 5>(a, p, s);
    case 6: return launch_typed<TYPE, 6>(a, p, s);
    case 7: return launch_typed<TYPE, 7>(a, p, s);
    case 8: return launch_typed<TYPE, 8>(a, p, s);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(int type, const GemvArgs& a, cudaStream_t s) {
    const GemvPlan p = plan_gemv(type, a.nb, a.n_out, a.tokens, a.num_sms);
    switch (type) {
    case TYPE_Q4_K: return launch_m<TYPE_Q4_K>(a, p, s);
    case TYPE_Q5_K: return launch_m<TYPE_Q5_K>(a, p, s);
    case TYPE_Q6_K: return launch_m<TYPE_Q6_K>(a, p, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace q35k
