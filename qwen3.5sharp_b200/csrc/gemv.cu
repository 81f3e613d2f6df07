// gemv.cu -- decode GEMV (1..8 tokens) for Q4_K / Q5_K / Q6_K weights.
//
// HBM-streaming design (no tensor cores; the kernel is bound by the weight
// stream):
//   * persistent: one CTA per SM; the weight matrix is a flat sequence of
//     tiles (32 rows x 1 super-block, see device_common.cuh) in row-group
//     order and every CTA owns one contiguous, equal share of it (stream-K),
//     so the load is balanced to one tile whatever the shape;
//   * tile c of the share belongs to warp c % NW; every warp prefetches its
//     own tiles into its own K shared-memory stages with 1-D bulk async copies
//     (cp.async.bulk, no multicast) and refills a stage the moment it has
//     consumed it, so NW*K tiles stay in flight per SM with no producer warp,
//     no empty barriers and no cross-warp waits (one full mbarrier per stage,
//     one consumer, phases in order);
//   * lane r of a warp decodes row r of its tile; the chunk-major tile layout
//     makes every 16-byte load a contiguous 512-byte line per warp, and all
//     lanes read the same Q8_K words (shared-memory broadcast);
//   * integer dots (dp4a, dp2a) into exact int32 per super-block, scaled in
//     fp32 once per block: acc += (d_w*d_x)*S - (dmin_w*d_x)*Mn
//     (VecDotQ4K.DotScalar, Kernels/VecDotQ4K.cs:42-61; Q5K.Dot,
//     Kernels/Q5K.cs:62-83; the Q6_K bias form of Q6K.DotAvx2,
//     Kernels/Q6K.cs:105-108,159);
//   * a row group's warp partials meet in a small ring of shared-memory
//     slots, where the last warp to arrive adds them in tile order; a row
//     group cut by a CTA boundary is finished by whichever CTA arrives last,
//     summing the pieces in CTA order and resetting the group's arrival
//     counter.  Every sum has a fixed order, so results are deterministic;
//   * the Q8_K activations arrive in a planar layout (qs | d | bsums) that the
//     CTA stages with three bulk copies; with programmatic dependent launch
//     the weight prefetch starts before the producing kernel ends and only
//     the activation copy waits for it.
#include "device_common.cuh"
#include "kernels.h"

#include <algorithm>

namespace q35k {

constexpr int GEMV_MAX_TOKENS = 8;
constexpr int GEMV_SMEM_LIMIT = 227 * 1024;
constexpr int GEMV_MAX_STAGES = 48;           // consumer warps x stages per warp
constexpr int GEMV_RING_BUDGET = 180 * 1024;  // weight bytes in flight per SM (upper bound)
constexpr int GEMV_Q8_LIMIT = 96 * 1024;      // staged Q8_K activations per CTA

// Consumer warps: more for few tokens (fewer registers per thread).
__host__ __device__ constexpr int gemv_consumers(int m) { return m <= 2 ? 12 : 8; }

__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct SmemLayout {
    int full, q8bar, slot_cnt, slot_owner, ring, q8, slots, total;
};

// Slots for row-group partial sums (row group g uses slot g % nslot); each
// holds min(nb, NW) warp partials.  Slot ownership passes from row group g to
// g + nslot once g has been summed, so a warp running ahead waits rather than
// overwrite; ceil(S/nb)+2 slots keep such waits rare.
__host__ __device__ constexpr int gemv_nslot(int stages, int nb) { return (stages + nb - 1) / nb + 2; }
constexpr int GEMV_MAX_SLOTS = GEMV_MAX_STAGES + 2;

// Dynamic shared memory of one GEMV CTA (16-byte aligned regions):
// full mbarriers | activation mbarrier | slot counters | slot owners |
// weight stages | planar Q8_K (qs | d | bsums) | row-group partial slots.
__host__ __device__ inline SmemLayout gemv_smem_layout(int tile_bytes, int stages, int m, int nb, int nw) {
    SmemLayout L;
    L.full = 0;
    L.q8bar = 8 * GEMV_MAX_STAGES;
    L.slot_cnt = L.q8bar + 16;
    L.slot_owner = L.slot_cnt + 4 * GEMV_MAX_SLOTS;
    L.ring = align_up(L.slot_owner + 4 * GEMV_MAX_SLOTS, 128);
    L.q8 = L.ring + stages * tile_bytes;
    L.slots = L.q8 + align_up((int)q8_planar(m, nb).bytes, 16);
    const int e = nb < nw ? nb : nw;
    L.total = L.slots + (stages ? gemv_nslot(stages, nb) : 0) * e * m * 32 * 4;
    return L;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
template <int NTHREADS>
__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(NTHREADS) : "memory");
}
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

// Staged planar Q8_K activations: qs[m][nb][256], d[m][nb], bsums[m][nb][16].
struct Q8Smem {
    const int8_t* qs;
    const float* d;
    const int16_t* bs;
    int nb;
    __device__ __forceinline__ const int8_t* q(int m, int b) const { return qs + (m * nb + b) * QK; }
    __device__ __forceinline__ float dx(int m, int b) const { return d[m * nb + b]; }
    __device__ __forceinline__ const int16_t* bsums(int m, int b) const { return bs + (m * nb + b) * 16; }
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

// Which CTA owns tile T when `tiles` tiles are split evenly over `grid` CTAs
// (CTA i owns [tiles*i/grid, tiles*(i+1)/grid)).
__device__ __forceinline__ int tile_owner(long T, long tiles, int grid) {
    return (int)(((T + 1) * (long)grid - 1) / tiles);
}

template <int TYPE, int M>
__global__ void __launch_bounds__(gemv_consumers(M) * 32, 1) gemv_kernel(GemvArgs a, GemvPlan p) {
    constexpr int NW = gemv_consumers(M);
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TILE = Fmt<TYPE>::TILE;
    const int K = p.stages / NW;  // stages per warp
    const SmemLayout L = gemv_smem_layout(TILE, p.stages, M, a.nb, NW);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* q8bar = reinterpret_cast<uint64_t*>(smem + L.q8bar);
    int* slot_cnt = reinterpret_cast<int*>(smem + L.slot_cnt);
    volatile int* slot_owner = reinterpret_cast<volatile int*>(smem + L.slot_owner);
    uint8_t* ring = smem + L.ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.nb;
    const long tiles = (long)p.groups * nb;
    const long T0 = tiles * blockIdx.x / gridDim.x;
    const long T1 = tiles * (blockIdx.x + 1) / gridDim.x;
    const int n_tiles = (int)(T1 - T0);
    const int nslot = gemv_nslot(p.stages, nb);
    const long g_first = T0 / nb;

    if (tid == 0) {
        for (int i = 0; i < p.stages; i++) mbar_init(&full[i], 1);
        mbar_init(q8bar, 1);
        fence_mbar_init();
    }
    for (int i = tid; i < nslot; i += NW * 32) {
        slot_cnt[i] = 0;
        // the first row group of this CTA that maps to slot i
        slot_owner[i] = (int)(g_first + ((i - (int)(g_first % nslot)) + nslot) % nslot);
    }
    __syncthreads();

    // This warp's tiles are c = warp + NW*i; tile i lives in stage warp*K + i%K.
    uint8_t* my_ring = ring + (size_t)warp * K * TILE;
    uint64_t* my_full = full + warp * K;
    auto prefetch = [&](int i) {
        const int c = warp + NW * i;
        if (c < n_tiles) {
            const int k = i % K;
            mbar_arrive_expect_tx(&my_full[k], TILE);
            bulk_g2s(my_ring + (size_t)k * TILE, a.tiles + (size_t)(T0 + c) * TILE, TILE, &my_full[k]);
        }
    };
    // Weights first: they do not depend on the preceding kernel.
    if (lane == 0)
        for (int i = 0; i < K; i++) prefetch(i);

    // Then the activations, once the producing kernel has completed.
    const Q8Planar pl = q8_planar(M, nb);
    uint8_t* q8smem = smem + L.q8;
    if (tid == 0) {
        griddep_wait();
        const uint32_t qs_bytes = (uint32_t)(pl.d - pl.qs);
        const uint32_t d_bytes = (uint32_t)(pl.bs - pl.d);
        const uint32_t bs_bytes = (uint32_t)(pl.bytes - pl.bs);
        mbar_arrive_expect_tx(q8bar, qs_bytes + d_bytes + bs_bytes);
        bulk_g2s(q8smem + pl.qs, a.q8 + pl.qs, qs_bytes, q8bar);
        bulk_g2s(q8smem + pl.d, a.q8 + pl.d, d_bytes, q8bar);
        bulk_g2s(q8smem + pl.bs, a.q8 + pl.bs, bs_bytes, q8bar);
    }
    bool ok = mbar_wait_bounded(q8bar, 0, a.err);
    const Q8Smem q8{reinterpret_cast<const int8_t*>(q8smem + pl.qs), reinterpret_cast<const float*>(q8smem + pl.d),
                    reinterpret_cast<const int16_t*>(q8smem + pl.bs), nb};
    const int E = min(nb, NW);
    float* slots = reinterpret_cast<float*>(smem + L.slots);

    // Final value of row group g's rows: whole groups store y; a group cut by
    // a CTA boundary publishes this CTA's piece and the last piece to arrive
    // sums all pieces in CTA order.
    auto finish = [&](long g, const float* v) {
        const int row = (int)g * TILE_ROWS + lane;
        const bool whole = g * nb >= T0 && (g + 1) * nb <= T1;
        if (whole) {
            if (row < a.n_out)
#pragma unroll
                for (int m = 0; m < M; m++) a.y[(size_t)m * a.ldy + row] = v[m];
            return;
        }
        const int first = tile_owner(g * nb, tiles, gridDim.x);
        const int pieces = tile_owner((g + 1) * nb - 1, tiles, gridDim.x) - first + 1;
        const int piece = (int)blockIdx.x - first;
        float* part = a.partial + (size_t)g * p.max_pieces * M * 32;
#pragma unroll
        for (int m = 0; m < M; m++) part[((size_t)piece * M + m) * 32 + lane] = v[m];
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&a.counters[g], 1) == pieces - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence();
#pragma unroll
            for (int m = 0; m < M; m++) {
                float s = 0.f;
                for (int k = 0; k < pieces; k++) s += __ldcg(&part[((size_t)k * M + m) * 32 + lane]);
                if (row < a.n_out) a.y[(size_t)m * a.ldy + row] = s;
            }
            if (lane == 0) a.counters[g] = 0;
        }
    };
    // This warp has done its last tile of row group g: add its partial to the
    // group's slot; the last warp of the group sums the slot in tile order.
    auto flush = [&](long g, const float* acc) {
        const int a0 = (int)(max(T0, g * nb) - T0);
        const int touched = min(NW, (int)(min(T1, (g + 1) * nb) - T0) - a0);
        const int slot = (int)(g % nslot);
        if (touched == 1) {
            // One warp holds the whole (piece of the) row group: no slot.  The
            // first row group still hands its slot on to g + nslot.
            if (g == g_first && lane == 0) slot_owner[slot] = (int)(g + nslot);
            finish(g, acc);
            return;
        }
        if (lane == 0) {
            // Wait (bounded) until row group g owns the slot.
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t it = 0; slot_owner[slot] != (int)g; it++) {
                if ((it & 1023u) == 1023u && globaltimer_ns() - t0 > 2000000000ull) {
                    atomicOr(a.err, DEV_ERR_TIMEOUT);
                    break;
                }
            }
            __threadfence_block();
        }
        __syncwarp();
        const int e = (warp - a0 % NW + NW) % NW;
        float* sl = slots + (size_t)slot * E * M * 32;
#pragma unroll
        for (int m = 0; m < M; m++) sl[(e * M + m) * 32 + lane] = acc[m];
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&slot_cnt[slot], 1) == touched - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            float v[M];
#pragma unroll
            for (int m = 0; m < M; m++) {
                v[m] = 0.f;
                for (int k = 0; k < touched; k++) v[m] += sl[(k * M + m) * 32 + lane];
            }
            __syncwarp();
            if (lane == 0) {
                slot_cnt[slot] = 0;
                __threadfence_block();
                slot_owner[slot] = (int)(g + nslot);  // hand the slot on
            }
            finish(g, v);
        }
    };

    int c = warp;
    long g = (T0 + c) / nb;
    int b = (int)(T0 + c - g * nb);
    int k = 0;        // stage of tile i (i % K)
    uint32_t ph = 0;  // its phase ((i / K) & 1)
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = 0.f;
    for (int i = 0; c < n_tiles; i++) {
        if (ok && !mbar_wait_bounded(&my_full[k], ph, a.err)) ok = false;
        if (ok) tile_dot<TYPE, M>(my_ring + (size_t)k * TILE, lane, q8, b, acc);
        __syncwarp();
        // The stage is consumed: refill it with this warp's tile i + K.
        if (lane == 0 && ok) prefetch(i + K);
        // Advance by NW tiles.
        const int cn = c + NW;
        int bn = b + NW;
        long gn = g;
        while (bn >= nb) {
            bn -= nb;
            gn++;
        }
        if (cn >= n_tiles || gn != g) {
            flush(g, acc);
#pragma unroll
            for (int m = 0; m < M; m++) acc[m] = 0.f;
        }
        c = cn;
        b = bn;
        g = gn;
        if (++k == K) {
            k = 0;
            ph ^= 1u;
        }
    }
    if (!ok) {
        // A wait gave up: give this warp's copies in flight a bounded chance
        // to land before the CTA's shared memory is released.
        __syncwarp();
        if (lane == 0)
            for (int s = 0; s < K; s++) mbar_wait_bounded(&my_full[s], ph ^ (s < k ? 1u : 0u), a.err, 100000000ull);
    }
}

GemvPlan plan_gemv(int type, int nb, int n_out, int tokens, int num_sms) {
    GemvPlan p{};
    const int tile = TILE_ROWS * block_bytes(type);
    const int m = std::min(std::max(tokens, 1), GEMV_MAX_TOKENS);
    p.groups = (n_out + TILE_ROWS - 1) / TILE_ROWS;
    p.n_pad = p.groups * TILE_ROWS;
    const long tiles = (long)p.groups * nb;
    p.grid = (int)std::min<long>(tiles, num_sms);
    // Stages: NW x K (K = 4, 3, 2 or 1 per warp) -- the largest ring that fits
    // next to the activations and the partial slots, within the in-flight budget.
    const int nw = gemv_consumers(m);
    p.stages = nw;
    for (int k = 4; k >= 1; k--) {
        const int s = nw * k;
        if (s * tile <= GEMV_RING_BUDGET && gemv_smem_layout(tile, s, m, nb, nw).total <= GEMV_SMEM_LIMIT) {
            p.stages = s;
            break;
        }
    }
    p.smem_bytes = (size_t)gemv_smem_layout(tile, p.stages, m, nb, nw).total;
    // A row group spans at most this many CTAs.
    const long per_cta = std::max<long>(1, tiles / p.grid);
    p.max_pieces = (int)std::min<long>(p.grid, (nb + per_cta - 1) / per_cta + 1);
    p.partial_bytes = (size_t)p.groups * p.max_pieces * GEMV_MAX_TOKENS * 32 * sizeof(float);
    p.counters = (size_t)p.groups;
    p.fits = (long)q8_planar(m, nb).bytes <= GEMV_Q8_LIMIT && p.smem_bytes <= (size_t)GEMV_SMEM_LIMIT;
    p.threads = nw * 32;
    return p;
}

int gemv_max_tokens(int nb) {
    // Tokens per launch so that the staged Q8_K activations fit.
    int m = GEMV_MAX_TOKENS;
    while (m > 0 && q8_planar(m, nb).bytes > (size_t)GEMV_Q8_LIMIT) m--;
    return m;
}

// Opt-in shared memory for every instantiation on the current device
// (called once per context).
template <int TYPE, int M>
static void configure_typed() {
    cudaFuncSetAttribute(gemv_kernel<TYPE, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_SMEM_LIMIT);
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
static cudaError_t launch_typed(const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
    if (!p.fits) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.grid);
    cfg.blockDim = dim3((unsigned)p.threads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<TYPE, M>, a, p);
}

template <int TYPE>
static cudaError_t launch_m(const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
    switch (a.tokens) {
    case 1: return launch_typed<TYPE, 1>(a, p, s, pdl);
    case 2: return launch_typed<TYPE, 2>(a, p, s, pdl);
    case 3: return launch_typed<TYPE, 3>(a, p, s, pdl);
    case 4: return launch_typed<TYPE, 4>(a, p, s, pdl);
    case 5: return launch_typed<TYPE, 5>(a, p, s, pdl);
    case 6: return launch_typed<TYPE, 6>(a, p, s, pdl);
    case 7: return launch_typed<TYPE, 7>(a, p, s, pdl);
    case 8: return launch_typed<TYPE, 8>(a, p, s, pdl);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(int type, const GemvArgs& a, cudaStream_t s, bool pdl) {
    const GemvPlan p = plan_gemv(type, a.nb, a.n_out, a.tokens, a.num_sms);
    switch (type) {
    case TYPE_Q4_K: return launch_m<TYPE_Q4_K>(a, p, s, pdl);
    case TYPE_Q5_K: return launch_m<TYPE_Q5_K>(a, p, s, pdl);
    case TYPE_Q6_K: return launch_m<TYPE_Q6_K>(a, p, s, pdl);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace q35k
