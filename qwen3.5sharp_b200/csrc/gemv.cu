// gemv.cu -- decode GEMV (1..8 tokens) for Q4_K / Q5_K / Q6_K weights.
//
// HBM-streaming design (no tensor cores; the kernel is bound by the weight
// stream):
//   * persistent: one CTA per SM; the weight matrix is a flat sequence of
//     tiles (32 rows x 1 super-block, see device_common.cuh) in row-group
//     order and every CTA owns one contiguous, equal share of it (stream-K),
//     so the load is balanced to one tile whatever the shape;
//   * one producer lane streams the CTA's tiles through a power-of-two ring
//     of shared-memory stages with 1-D bulk async copies (cp.async.bulk, no
//     multicast), one full/empty mbarrier pair per stage;
//   * each consumer warp owns whole row groups (lane r = row r), so no
//     cross-warp reduction or barrier sits in the main loop: the producer
//     interleaves the tiles of the row groups the warps are working on
//     ("rounds" of up to NW row groups, tile t of every row group in turn);
//   * the chunk-major tile layout makes every 16-byte load a contiguous
//     512-byte line per warp; all lanes read the same Q8_K words
//     (shared-memory broadcast);
//   * integer dots (dp4a, dp2a) into exact int32 per super-block, scaled in
//     fp32 once per block: acc += (d_w*d_x)*S - (dmin_w*d_x)*Mn
//     (VecDotQ4K.DotScalar, Kernels/VecDotQ4K.cs:42-61; Q5K.Dot,
//     Kernels/Q5K.cs:62-83; the Q6_K bias form of Q6K.DotAvx2,
//     Kernels/Q6K.cs:105-108,159);
//   * a row group cut by a CTA boundary is finished by whichever CTA arrives
//     last, summing the pieces in CTA order (deterministic) and resetting the
//     group's arrival counter for the next call;
//   * the activation quantizer runs as the preceding kernel; with
//     programmatic dependent launch the weight stream starts before it ends
//     and only the consumers wait for its Q8_K output.
#include "device_common.cuh"
#include "kernels.h"

#include <algorithm>

namespace q35k {

constexpr int GEMV_MAX_TOKENS = 8;
constexpr int GEMV_SMEM_LIMIT = 227 * 1024;
constexpr int GEMV_MAX_STAGES = 48;                // consumer warps x stages per warp
constexpr int GEMV_RING_BUDGET = 180 * 1024;       // weight bytes in flight per SM (upper bound)
constexpr int GEMV_Q8_LIMIT = 96 * 1024;  // staged Q8_K activations per CTA

// Consumer warps: more for few tokens (fewer registers per thread).
__host__ __device__ constexpr int gemv_consumers(int m) { return m <= 2 ? 12 : 8; }

__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct SmemLayout {
    int full, empty, ring, q8s, q8d, q8b, total;
};

// Dynamic shared memory of one GEMV CTA (16-byte aligned regions):
// full mbarriers | empty mbarriers | weight ring | Q8_K qs | Q8_K d | Q8_K bsums.
__host__ __device__ inline SmemLayout gemv_smem_layout(int tile_bytes, int stages, int m, int nb) {
    SmemLayout L;
    L.full = 0;
    L.empty = 8 * GEMV_MAX_STAGES;
    L.ring = 16 * GEMV_MAX_STAGES;
    L.q8s = L.ring + stages * tile_bytes;
    L.q8d = L.q8s + m * nb * QK;
    L.q8b = L.q8d + align_up(m * nb * 4, 16);
    L.total = L.q8b + align_up(m * nb * 32, 16);
    return L;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
template <int NTHREADS>
__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(NTHREADS) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Staged Q8_K activations: qs[m][nb][256], d[m][nb], bsums[m][nb][16].
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

// Which CTA owns tile T when `tiles` tiles are split evenly over `grid` CTAs
// (CTA i owns [tiles*i/grid, tiles*(i+1)/grid)).
__device__ __forceinline__ int tile_owner(long T, long tiles, int grid) {
    return (int)(((T + 1) * (long)grid - 1) / tiles);
}

// The CTA's share [T0, T1) of the tile sequence as work items, in issue order:
//   head  : a partial first row group (tiles tb..te-1), warp 0;
//   rounds: full row groups, NW at a time; in round r the j-th row group goes
//           to warp (j + hoff) % NW and tile t of it sits at ring position
//           base_r + t * nj + j;
//   tail  : a partial last row group, the next warp in rotation.
struct Share {
    long g_head;
    int head_tb, head_te;  // head piece (head_te > head_tb if present)
    long g_full0;          // first full row group
    int nfull;             // number of full row groups
    long g_tail;
    int tail_te;           // tail piece tiles 0..tail_te-1 (tail_te > 0 if present)
    int hoff;              // 1 if a head piece exists
};

__device__ __forceinline__ Share make_share(long T0, long T1, int nb) {
    Share s{};
    const long gA = T0 / nb, gZ = (T1 - 1) / nb;
    const int ta = (int)(T0 - gA * nb);       // first tile inside gA
    const int tz = (int)(T1 - gZ * nb);       // tiles of gZ inside the share
    if (gA == gZ) {
        if (ta == 0 && tz == nb) {
            s.g_full0 = gA;
            s.nfull = 1;
        } else {
            s.g_head = gA;
            s.head_tb = ta;
            s.head_te = tz;
        }
    } else {
        long f0 = gA, f1 = gZ + 1;  // full row groups [f0, f1)
        if (ta != 0) {
            s.g_head = gA;
            s.head_tb = ta;
            s.head_te = nb;
            f0 = gA + 1;
        }
        if (tz != nb) {
            s.g_tail = gZ;
            s.tail_te = tz;
            f1 = gZ;
        }
        s.g_full0 = f0;
        s.nfull = (int)(f1 - f0);
    }
    s.hoff = s.head_te > s.head_tb ? 1 : 0;
    return s;
}

template <int TYPE, int M>
__device__ __forceinline__ void tile_dot(const uint8_t* tile, int lane, const Q8Smem& q8, int b, float* acc) {
    if (TYPE == TYPE_Q6_K)
        block_dot_q6k<M>(tile, lane, q8, b, acc);
    else
        block_dot_k45<TYPE, M>(tile, lane, q8, b, acc);
}

template <int TYPE, int M>
__global__ void __launch_bounds__((gemv_consumers(M) + 1) * 32, 1) gemv_kernel(GemvArgs a, GemvPlan p) {
    constexpr int NW = gemv_consumers(M);
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TILE = Fmt<TYPE>::TILE;
    const SmemLayout L = gemv_smem_layout(TILE, p.stages, M, a.nb);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
    uint8_t* ring = smem + L.ring;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = a.nb;
    const long tiles = (long)p.groups * nb;
    const long T0 = tiles * blockIdx.x / gridDim.x;
    const long T1 = tiles * (blockIdx.x + 1) / gridDim.x;
    // Each consumer warp owns a private run of 2^wlog stages and consumes it
    // in order (the single-consumer pipeline that mbarrier phase parity
    // needs); its i-th tile lands in stage warp*2^wlog + i % 2^wlog.
    const int wlog = p.warp_stage_log2, wmask = (1 << wlog) - 1;
    const Share sh = make_share(T0, T1, nb);
    const int head_len = sh.head_te - sh.head_tb;

    if (tid == 0) {
        for (int i = 0; i < NW << wlog; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == NW) {
        // ---------------- producer: issue tiles round by round ----------------
        // Tile t of the j-th row group of round R goes to warp w = (j + hoff)
        // % NW as that warp's tile number i = (head tiles of w) + R*nb + t.
        if (lane != 0) return;
        bool ok = true;
        auto issue = [&](long T, int w, int i) {
            const int st = (w << wlog) + (i & wmask);
            if (i > wmask) ok = ok && mbar_wait_bounded(&empty[st], (uint32_t)(((i >> wlog) - 1) & 1), a.err);
            if (ok) {
                mbar_arrive_expect_tx(&full[st], TILE);
                bulk_g2s(ring + (size_t)st * TILE, a.tiles + (size_t)T * TILE, TILE, &full[st]);
            }
        };
        for (int t = sh.head_tb; t < sh.head_te && ok; t++) issue(sh.g_head * nb + t, 0, t - sh.head_tb);
        int R = 0;
        for (int r0 = 0; r0 < sh.nfull && ok; r0 += NW, R++) {
            const int nj = min(NW, sh.nfull - r0);
            for (int t = 0; t < nb && ok; t++)
                for (int j = 0; j < nj; j++) {
                    const int w = (j + sh.hoff) % NW;
                    issue((sh.g_full0 + r0 + j) * nb + t, w, (w == 0 ? head_len : 0) + R * nb + t);
                }
        }
        if (sh.tail_te > 0) {
            const int w = (sh.hoff + sh.nfull) % NW;
            const int i0 = (w == 0 ? head_len : 0) + (sh.nfull / NW) * nb;
            for (int t = 0; t < sh.tail_te && ok; t++) issue(sh.g_tail * nb + t, w, i0 + t);
        }
        return;
    }

    // ---------------- consumers ----------------
    griddep_wait();  // the Q8_K activations come from the preceding kernel
    int8_t* q8s = reinterpret_cast<int8_t*>(smem + L.q8s);
    float* q8d = reinterpret_cast<float*>(smem + L.q8d);
    int16_t* q8b = reinterpret_cast<int16_t*>(smem + L.q8b);
    // 73 words per BlockQ8K: word 0 = d, 1..64 = qs, 65..72 = bsums.
    for (int idx = tid; idx < M * nb * 73; idx += NW * 32) {
        const int mb = idx / 73, w = idx % 73;
        const uint32_t v = __ldg(reinterpret_cast<const uint32_t*>(a.q8 + (size_t)mb * Q8K_BYTES) + w);
        if (w == 0)
            q8d[mb] = __uint_as_float(v);
        else if (w <= 64)
            reinterpret_cast<uint32_t*>(q8s + mb * QK)[w - 1] = v;
        else
            reinterpret_cast<uint32_t*>(q8b + mb * 16)[w - 65] = v;
    }
    consumer_bar<NW * 32>();
    const Q8Smem q8{q8s, q8d, q8b, nb};

    bool ok = true;
    int i_tile = 0;  // this warp's tile counter (its private stages, in order)
    // Process the warp's next tile: super-block b of its current row group.
    auto consume = [&](int b, float* acc) {
        const int st = (warp << wlog) + (i_tile & wmask);
        if (ok && !mbar_wait_bounded(&full[st], (uint32_t)((i_tile >> wlog) & 1), a.err)) ok = false;
        if (ok) tile_dot<TYPE, M>(ring + (size_t)st * TILE, lane, q8, b, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        i_tile++;
    };
    auto store_whole = [&](long g, const float* acc) {
        const int row = (int)g * TILE_ROWS + lane;
        if (row < a.n_out)
#pragma unroll
            for (int m = 0; m < M; m++) a.y[(size_t)m * a.ldy + row] = acc[m];
    };
    // A row group cut by a CTA boundary: publish this CTA's piece; the last
    // piece to arrive sums all pieces in CTA order and stores y.
    auto store_piece = [&](long g, const float* acc) {
        const int row = (int)g * TILE_ROWS + lane;
        const int first = tile_owner(g * nb, tiles, gridDim.x);
        const int pieces = tile_owner((g + 1) * nb - 1, tiles, gridDim.x) - first + 1;
        const int piece = (int)blockIdx.x - first;
        float* part = a.partial + (size_t)g * p.max_pieces * M * 32;
#pragma unroll
        for (int m = 0; m < M; m++) part[((size_t)piece * M + m) * 32 + lane] = acc[m];
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

    if (head_len > 0 && warp == 0) {
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; m++) acc[m] = 0.f;
        for (int t = sh.head_tb; t < sh.head_te; t++) consume(t, acc);
        store_piece(sh.g_head, acc);
    }
    for (int r0 = 0; r0 < sh.nfull; r0 += NW) {
        const int nj = min(NW, sh.nfull - r0);
        const int j = (warp - sh.hoff + NW) % NW;
        if (j < nj) {
            float acc[M];
#pragma unroll
            for (int m = 0; m < M; m++) acc[m] = 0.f;
            for (int t = 0; t < nb; t++) consume(t, acc);
            store_whole(sh.g_full0 + r0 + j, acc);
        }
    }
    if (sh.tail_te > 0 && warp == (sh.hoff + sh.nfull) % NW) {
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; m++) acc[m] = 0.f;
        for (int t = 0; t < sh.tail_te; t++) consume(t, acc);
        store_piece(sh.g_tail, acc);
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
    // Stages per consumer warp: the largest power of two (<= 4) whose ring
    // fits next to the staged activations and within the in-flight budget.
    const int nw = gemv_consumers(m);
    const int room = std::min(GEMV_SMEM_LIMIT - gemv_smem_layout(tile, 0, m, nb).total, GEMV_RING_BUDGET);
    p.warp_stage_log2 = 0;
    while (p.warp_stage_log2 < 2 && nw * (2 << p.warp_stage_log2) * tile <= room) p.warp_stage_log2++;
    p.stages = nw << p.warp_stage_log2;
    p.smem_bytes = (size_t)gemv_smem_layout(tile, p.stages, m, nb).total;
    // A row group spans at most this many CTAs.
    const long per_cta = std::max<long>(1, tiles / p.grid);
    p.max_pieces = (int)std::min<long>(p.grid, (nb + per_cta - 1) / per_cta + 1);
    p.partial_bytes = (size_t)p.groups * p.max_pieces * GEMV_MAX_TOKENS * 32 * sizeof(float);
    p.counters = (size_t)p.groups;
    p.fits = (long)m * nb * Q8K_BYTES <= GEMV_Q8_LIMIT && p.smem_bytes <= (size_t)GEMV_SMEM_LIMIT;
    p.threads = (gemv_consumers(m) + 1) * 32;
    return p;
}

int gemv_max_tokens(int nb) {
    // Tokens per launch so that the staged Q8_K activations fit.
    const int m = GEMV_Q8_LIMIT / (nb * Q8K_BYTES);
    return std::max(0, std::min(GEMV_MAX_TOKENS, m));
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
