// gemv.cu -- decode GEMV (1..8 tokens) for Q4_K / Q5_K / Q6_K weights.
//
// HBM-streaming design (no tensor cores; the kernel is bound by the weight
// stream):
//   * one CTA per work unit = (32-row group, run of U super-blocks); many
//     small CTAs per SM, so the hardware scheduler balances the load across
//     SMs (a faster SM simply takes more units) and there is no tail;
//   * thread 0 issues every weight tile of the unit as a 1-D bulk async copy
//     (cp.async.bulk, no multicast) at CTA start, one mbarrier per tile, and
//     -- with programmatic dependent launch -- before waiting for the kernel
//     that produces the activations; then three more bulk copies stage the
//     unit's K-range of the planar Q8_K activations;
//   * warp w takes tiles w, w+W, ... of the unit; lane r decodes row r (the
//     chunk-major tile layout makes every 16-byte load a contiguous 512-byte
//     line per warp) and all lanes read the same Q8_K words (shared-memory
//     broadcast); integer dots live in gemv_dot.cuh;
//   * the warps' partial sums are added in warp order; the units of a row
//     group split along K (2..8 of them) are one thread-block cluster, whose
//     first CTA sums the pieces in K order through distributed shared memory;
//     a row group split further is finished by whichever unit arrives last,
//     summing the pieces in K order through global memory and resetting the
//     group's arrival counter.  Every sum has a fixed order, so results are
//     deterministic.
#include "device_common.cuh"
#include "gemv_dot.cuh"
#include "kernels.h"
#include "q8k_quant.cuh"

#include <algorithm>

namespace q35k {

constexpr int GEMV_MAX_TOKENS = 8;
constexpr int GEMV_MAX_WARPS = 20;        // one warp per tile of a whole-row unit
constexpr int GEMV_SPLIT_WARPS = 10;      // warps of a split-K unit
constexpr int GEMV_FUSED_MAX_TOKENS = 2;  // token counts with a fused-quantize variant
// The fused quantizer writes the plain planar layout; the mma token counts take the
// tensor-core dots over the word-interleaved one.
static_assert(GEMV_FUSED_MAX_TOKENS < q8_interleave_min_rows(TYPE_Q4_K) &&
                  GEMV_FUSED_MAX_TOKENS < q8_interleave_min_rows(TYPE_Q6_K),
              "fused GEMV layouts");
// Unit sizes of the launch plan (compile-time; the defaults are the measured best).
#ifndef Q35K_GEMV_UNIT_KB
#define Q35K_GEMV_UNIT_KB 72
#endif
#ifndef Q35K_GEMV_ROW_KB
#define Q35K_GEMV_ROW_KB 96
#endif
constexpr int GEMV_UNIT_BYTES = Q35K_GEMV_UNIT_KB * 1024;  // weight bytes per split-K work unit (target)
constexpr int GEMV_ROW_BYTES = Q35K_GEMV_ROW_KB * 1024;    // largest whole-row unit
constexpr int GEMV_SMEM_LIMIT = 227 * 1024;
constexpr int GEMV_MAX_CLUSTER = 8;  // portable thread-block cluster size

__host__ __device__ constexpr int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct SmemLayout {
    int bars, flags, tiles, q8, red, total;
};

// Dynamic shared memory of one GEMV CTA (16-byte aligned regions):
// U+1 mbarriers | flags | U weight tiles | planar Q8_K of U blocks | W*M*32
// partial sums.
__host__ __device__ inline SmemLayout gemv_smem_layout(int type, int tile_bytes, int units, int m, int warps) {
    SmemLayout L;
    const int rows4 = (m + 3) / 4 * 4;
    L.bars = 0;
    L.flags = 8 * (units + 1);
    L.tiles = align_up(L.flags + 16, 128);
    L.q8 = L.tiles + units * tile_bytes;
    // The mma token counts read their activations from global memory (L2), not staged.
    L.red = L.q8 + (m >= q8_interleave_min_rows(type) ? 0 : units * (m * QK + rows4 * 4 + m * 32));
    L.total = L.red + warps * m * 32 * 4;
    return L;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Barrier over every thread of the thread-block cluster (release / acquire at
// cluster scope: shared-memory writes before it are visible to the cluster's
// CTAs after it).
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The float at the same shared-memory offset as `p` in the cluster's CTA `rank`.
__device__ __forceinline__ float ld_cluster_f32(const float* p, int rank) {
    uint32_t addr;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(smem_u32(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Order-preserving key of (logit, row) for the fused argmax: the largest key
// is the reference's ArgMax (Qwen35Sharp.Cli/Program.cs:127-140) -- the first
// row holding the largest logit under a strict '>' scan from row 0.  -0 and +0
// compare equal; a NaN at row 0 keeps row 0 (the scan's start value), a NaN
// elsewhere is never taken.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    uint32_t o;
    if (v != v) {
        o = row == 0 ? 0xffffffffu : 0u;
    } else {
        const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
        o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return ((unsigned long long)o << 32) | (0xffffffffu - (uint32_t)row);
}

// Warp-wide max of a 64-bit key; lane 0 folds it into *dst.
__device__ __forceinline__ void warp_argmax_commit(unsigned long long key, unsigned long long* dst, int lane) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if (lane == 0) atomicMax(dst, key);
}

// FUSED: quantize this CTA's K-range of the fp32 activations (a.x) to Q8_K in
// shared memory (q8k_quant.cuh, the same bytes as the standalone quantizer)
// while the weight tiles are in flight, instead of staging planar Q8_K from
// a.q8 -- one kernel per call, used when that slice is small (decode).
// SPLIT: the launch splits row groups along K (several units per row group);
// whole-row launches run an instantiation without the split-K code.
template <int TYPE, int M, bool FUSED, bool SPLIT>
__device__ __forceinline__ void decode_body(const GemvArgs& a, const GemvPlan& p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TILE = Fmt<TYPE>::TILE;
    const int U = p.unit_blocks, W = p.warps, nb = a.nb;
    const SmemLayout L = gemv_smem_layout(TYPE, TILE, U, M, W);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);  // [0, kr): tiles, [kr]: activations
    uint8_t* tiles = smem + L.tiles;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.x / p.splits, s = blockIdx.x % p.splits;
    const int b0 = s * U;
    // The matrix this row group belongs to (several weights per launch).
    const uint8_t* wtiles = a.tiles;
    float* y = a.y;
    int n_out = a.n_out, ldy = a.ldy, gl = g;
#pragma unroll
    for (int k = 0; k < GEMV_MAX_MATS - 1; k++)
        if (k < a.more.n && g >= a.more.g0[k]) {
            wtiles = a.more.tiles[k];
            y = a.more.y[k];
            n_out = a.more.n_out[k];
            ldy = a.more.ldy[k];
            gl = g - a.more.g0[k];
        }
    const int kr = min(U, nb - b0);

    if (tid == 0) {
        for (int t = 0; t <= kr; t++) mbar_init(&bars[t], 1);
        fence_mbar_init();
        if (a.peers.trace) atomicMin(a.peers.trace, (unsigned long long)globaltimer_ns());
    }
    __syncthreads();
    const Q8Planar pl = q8_planar(M, nb);
    uint8_t* q8s = smem + L.q8;
    const int qs_bytes = kr * M * QK, d_bytes = kr * pl.rows4 * 4, bs_bytes = kr * M * 32;
    if (tid == 0) {
        // Weights first: they do not depend on the preceding kernel.
        const uint8_t* src = wtiles + ((size_t)gl * nb + b0) * TILE;
        for (int t = 0; t < kr; t++) {
            mbar_arrive_expect_tx(&bars[t], TILE);
            bulk_g2s(tiles + (size_t)t * TILE, src + (size_t)t * TILE, TILE, &bars[t]);
        }
        if (!FUSED && M < q8_interleave_min_rows(TYPE)) {
            // Then the activations, once the producing kernel has completed.
            griddep_wait();
            mbar_arrive_expect_tx(&bars[kr], qs_bytes + d_bytes + bs_bytes);
            bulk_g2s(q8s, a.q8 + pl.qs + (size_t)b0 * M * QK, qs_bytes, &bars[kr]);
            bulk_g2s(q8s + qs_bytes, a.q8 + pl.d + (size_t)b0 * pl.rows4 * 4, d_bytes, &bars[kr]);
            bulk_g2s(q8s + qs_bytes + d_bytes, a.q8 + pl.bs + (size_t)b0 * M * 32, bs_bytes, &bars[kr]);
        }
    }
    // The next kernel in the stream may start streaming its own weights on
    // SMs this grid frees; it reads activations and writes results only
    // after its own griddepcontrol.wait, i.e. after this grid completed.
    // Fused all-gather: the kernel after this one (the gather) reads the call
    // counter when it starts, so it may start only once every CTA has passed
    // the wait for the kernel before (the previous call's gather, which
    // advanced the counter): the trigger then follows that wait.
    if (a.peers.n == 0) asm volatile("griddepcontrol.launch_dependents;");
    // mma token counts: the unit's K-range of the planar Q8_K in global memory (each
    // warp loads its B operand words directly; L2 serves the CTAs of a K-range).
    constexpr bool Q8_GLOBAL = M >= q8_interleave_min_rows(TYPE);
    const Q8Smem q8 = Q8_GLOBAL
        ? Q8Smem{reinterpret_cast<const int8_t*>(a.q8 + pl.qs + (size_t)b0 * M * QK),
                 reinterpret_cast<const float*>(a.q8 + pl.d + (size_t)b0 * pl.rows4 * 4),
                 reinterpret_cast<const int16_t*>(a.q8 + pl.bs + (size_t)b0 * M * 32), M, pl.rows4}
        : Q8Smem{reinterpret_cast<const int8_t*>(q8s), reinterpret_cast<const float*>(q8s + qs_bytes),
                 reinterpret_cast<const int16_t*>(q8s + qs_bytes + d_bytes), M, pl.rows4};
    bool ok = true;
    if (FUSED) {
        griddep_wait();  // x comes from the preceding kernel
        // Each warp quantizes the blocks of the tiles it decodes (all tokens),
        // so it depends on no other warp.
        for (int t = warp; t < kr; t += W)
#pragma unroll
            for (int m = 0; m < M; m++) {
                Q8Out out;
                out.d = reinterpret_cast<uint32_t*>(q8s + qs_bytes) + t * pl.rows4 + m;
                out.qs = reinterpret_cast<uint32_t*>(q8s + (size_t)(t * M + m) * QK);
                out.bs = reinterpret_cast<int16_t*>(q8s + qs_bytes + d_bytes) + (t * M + m) * 16;
                const size_t off = (size_t)m * a.ldx + (size_t)(b0 + t) * QK;
                warp_quantize_q8k_block(a.x + off, out, lane, a.up ? a.up + off : nullptr);
            }
        __syncwarp();
    } else if (Q8_GLOBAL) {
        griddep_wait();  // q8 comes from the preceding kernel
    } else {
        ok = mbar_wait_bounded(&bars[kr], 0, a.err);
    }
    if (a.peers.n) asm volatile("griddepcontrol.launch_dependents;");

    float* red = reinterpret_cast<float*>(smem + L.red);
    if constexpr (M >= q8_interleave_min_rows(TYPE)) {
        // Tensor-core dots (gemv_dot.cuh); the staged qs plane is word-interleaved.
        // A warp's B operands come from L2: each tile's are loaded before
        // its weight tile is awaited, and the next tile's during this one's
        // decode, so their latency hides behind the weight stream.
        float acc[2][2][2] = {};
        const int g = lane >> 2, c = lane & 3;
        MmaB<M> B;
        if (warp < kr) B.load(q8, warp, g, c);
        for (int t = warp; ok && t < kr; t += W) {
            MmaB<M> Bn;
            if (t + W < kr) Bn.load(q8, t + W, g, c);
            if (!mbar_wait_bounded(&bars[t], 0, a.err)) {
                ok = false;
                break;
            }
            tile_dot_mma<TYPE, M>(tiles + (size_t)t * TILE, lane, B, acc);
            B = Bn;
        }
#pragma unroll
        for (int hf = 0; hf < 2; hf++)
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 2; j++)
                    if (2 * c + j < M) red[(warp * M + 2 * c + j) * 32 + 16 * hf + 8 * i + g] = acc[hf][i][j];
    } else {
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; m++) acc[m] = 0.f;
        for (int t = warp; ok && t < kr; t += W) {
            if (!mbar_wait_bounded(&bars[t], 0, a.err)) {
                ok = false;
                break;
            }
            tile_dot<TYPE, M>(tiles + (size_t)t * TILE, lane, q8, t, acc);
        }
#pragma unroll
        for (int m = 0; m < M; m++) red[(warp * M + m) * 32 + lane] = acc[m];
    }
    __syncthreads();

    if (warp == 0) {
        const int row = gl * TILE_ROWS + lane;
        // Fused all-gather: this call's number and its gather area in the
        // peers' buffers.  Each value goes out as one 64-bit store of (call
        // number, value bits), so a peer knows it has arrived without a
        // fence or a flag.
        const unsigned ep = a.peers.n ? *a.peers.seq + 1u : 0u;
        const size_t poff = (size_t)(ep & 1u) * a.peers.half;
        const int ldp = a.peers.ldp;
        auto to_peers = [&](size_t off, float v) {
            const unsigned long long word = ((unsigned long long)ep << 32) | __float_as_uint(v);
            for (int k = 0; k < a.peers.n; k++) st_relaxed_sys_u64(a.peers.y[k] + poff + off, word);
        };
        float v[M];
#pragma unroll
        for (int m = 0; m < M; m++) {
            v[m] = red[m * 32 + lane];
            for (int w = 1; w < W; w++) v[m] += red[(w * M + m) * 32 + lane];
        }
        if constexpr (!SPLIT) {
            if (row < n_out && y)
#pragma unroll
                for (int m = 0; m < M; m++) {
                    y[(size_t)m * ldy + row] = v[m];
                    to_peers((size_t)m * ldp + row, v[m]);
                }
            if (a.argmax)
#pragma unroll
                for (int m = 0; m < M; m++)
                    warp_argmax_commit(row < n_out ? argmax_key(v[m], row) : 0ull, a.argmax + m, lane);
        } else if (p.cluster > 1) {
            // The row group's K-ranges form one thread-block cluster: this
            // piece stays in this CTA's shared memory (each lane overwrites
            // only the entries it has just read), and the cluster's first
            // CTA sums the pieces in K order below.
#pragma unroll
            for (int m = 0; m < M; m++) red[m * 32 + lane] = v[m];
        } else {
            // Publish this K-range's piece; the last piece to arrive sums all
            // pieces in K order and resets the row group's counter.
            float* part = a.partial + (size_t)g * p.splits * M * 32;
#pragma unroll
            for (int m = 0; m < M; m++) part[((size_t)s * M + m) * 32 + lane] = v[m];
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(&a.counters[g], 1) == p.splits - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
#pragma unroll
                for (int m = 0; m < M; m++) {
                    float sum = 0.f;
                    for (int k = 0; k < p.splits; k++) sum += __ldcg(&part[((size_t)k * M + m) * 32 + lane]);
                    if (row < n_out && y) {
                        y[(size_t)m * ldy + row] = sum;
                        to_peers((size_t)m * ldp + row, sum);
                    }
                    if (a.argmax) warp_argmax_commit(row < n_out ? argmax_key(sum, row) : 0ull, a.argmax + m, lane);
                }
                if (lane == 0) a.counters[g] = 0;
            }
        }
    }
    if constexpr (SPLIT) {
        if (p.cluster > 1) {
            cluster_barrier();  // every piece is in its CTA's shared memory
            if (warp == 0 && s == 0) {
                const int row = gl * TILE_ROWS + lane;
                const unsigned ep = a.peers.n ? *a.peers.seq + 1u : 0u;
                const size_t poff = (size_t)(ep & 1u) * a.peers.half;
                // The same additions, in the same order, as the global-memory
                // path: bit-identical results either way.
#pragma unroll
                for (int m = 0; m < M; m++) {
                    float sum = 0.f;
                    sum += red[m * 32 + lane];
                    for (int k = 1; k < p.splits; k++) sum += ld_cluster_f32(&red[m * 32 + lane], k);
                    if (row < n_out && y) {
                        y[(size_t)m * ldy + row] = sum;
                        const unsigned long long word = ((unsigned long long)ep << 32) | __float_as_uint(sum);
                        for (int k = 0; k < a.peers.n; k++)
                            st_relaxed_sys_u64(a.peers.y[k] + poff + (size_t)m * a.peers.ldp + row, word);
                    }
                    if (a.argmax) warp_argmax_commit(row < n_out ? argmax_key(sum, row) : 0ull, a.argmax + m, lane);
                }
            }
            cluster_barrier();  // the first CTA has read every piece: the CTAs may exit
        }
    }
    if (a.peers.trace && tid == 0) atomicMax(a.peers.trace + 1, (unsigned long long)globaltimer_ns());
    // Any warp whose wait gave up reports it to the host-pointer caller too.
    if (!ok && lane == 0 && a.h_err) *reinterpret_cast<volatile unsigned*>(a.h_err) = DEV_ERR_TIMEOUT;
    if (!ok && tid == 0) {
        // A wait gave up: give the copies in flight a bounded chance to land
        // before the CTA's shared memory is released.
        for (int t = 0; t < kr + ((FUSED || Q8_GLOBAL) ? 0 : 1); t++)
            mbar_wait_bounded(&bars[t], 0, a.err, 100000000ull);
    }
}

// The kernels.  q35k_decode_kernel takes every launch plan (up to 20 warps).
// One- and two-token launches of at most GEMV_SPLIT_WARPS warps (whole rows of
// up to 10 tiles, split-K units) whose grid fits three CTAs per SM, or whose
// shared memory allows no more, run q35k_decode_kernel_10w instead, whose
// bounds (three 10-warp CTAs per SM) let the compiler keep more of the decode
// in registers.
template <int TYPE, int M, bool FUSED, bool SPLIT>
__global__ void __launch_bounds__(GEMV_MAX_WARPS * 32) q35k_decode_kernel(GemvArgs a, GemvPlan p) {
    decode_body<TYPE, M, FUSED, SPLIT>(a, p);
}

template <int TYPE, int M, bool FUSED, bool SPLIT>
__global__ void __launch_bounds__(GEMV_SPLIT_WARPS * 32, 3) q35k_decode_kernel_10w(GemvArgs a, GemvPlan p) {
    decode_body<TYPE, M, FUSED, SPLIT>(a, p);
}

// Q4_K whole rows of 11..20 tiles at one or two tokens: 20-warp CTAs bounded at
// two per SM (48 registers; without the bound the two-token form takes 53-56
// and only one CTA fits an SM).
template <int TYPE, int M, bool FUSED>
__global__ void __launch_bounds__(GEMV_MAX_WARPS * 32, 2) q35k_decode_kernel_20w(GemvArgs a, GemvPlan p) {
    decode_body<TYPE, M, FUSED, false>(a, p);
}

GemvPlan plan_gemv(int type, int nb, int n_out, int tokens, int num_sms) {
    GemvPlan p{};
    const int tile = TILE_ROWS * block_bytes(type);
    const int m = std::min(std::max(tokens, 1), GEMV_MAX_TOKENS);
    p.groups = (n_out + TILE_ROWS - 1) / TILE_ROWS;
    p.n_pad = p.groups * TILE_ROWS;
    // A whole row group per CTA, one warp per tile, when it is at most
    // GEMV_MAX_WARPS tiles and GEMV_ROW_BYTES and there are enough row
    // groups to fill the SMs: no split-K fix-up, and every tile decoded in
    // parallel.  Otherwise units of up to ~GEMV_UNIT_BYTES over
    // GEMV_SPLIT_WARPS warps; split K further only while there are fewer
    // units than SMs.
    int u, max_warps;
    if (nb <= GEMV_MAX_WARPS && nb * tile <= GEMV_ROW_BYTES && p.groups >= num_sms) {
        u = nb;
        // mma token counts: 10 warps (two tiles each at 20 tiles), so that two CTAs
        // share an SM and one's copies overlap the other's decode.
        max_warps = m >= q8_interleave_min_rows(type) ? GEMV_SPLIT_WARPS : GEMV_MAX_WARPS;
    } else {
        u = std::max(1, std::min(nb, GEMV_UNIT_BYTES / tile));
        int splits = (nb + u - 1) / u;
        while (splits < nb && (long)p.groups * splits < num_sms) splits++;
        u = (nb + splits - 1) / splits;
        max_warps = GEMV_SPLIT_WARPS;
    }
    // The activations of one unit must fit next to its tiles.
    while (u > 1 && gemv_smem_layout(type, tile, u, m, std::min(u, max_warps)).total > GEMV_SMEM_LIMIT) u--;
    p.unit_blocks = u;
    p.splits = (nb + u - 1) / u;
    p.warps = std::min(u, max_warps);
    p.grid = p.groups * p.splits;
    p.smem_bytes = (size_t)gemv_smem_layout(type, tile, u, m, p.warps).total;
    // Splits of a row group that fit one portable cluster are reduced through
    // distributed shared memory.
    p.cluster = (p.splits > 1 && p.splits <= GEMV_MAX_CLUSTER) ? p.splits : 0;
    p.partial_bytes = p.splits > 1 ? (size_t)p.groups * p.splits * GEMV_MAX_TOKENS * 32 * sizeof(float) : 0;
    p.counters = (size_t)p.groups;
    p.fits = p.smem_bytes <= (size_t)GEMV_SMEM_LIMIT;
    p.threads = p.warps * 32;
    // Shared memory per SM: 228 KB, 1 KB of it reserved per CTA.
    const long smem_fit = 233472L / ((long)p.smem_bytes + 1024);
    p.three_per_sm = m <= GEMV_FUSED_MAX_TOKENS && p.warps <= GEMV_SPLIT_WARPS &&
                     (smem_fit <= 3 || (long)p.grid <= 3L * num_sms);
    return p;
}

int gemv_max_tokens(int nb) {
    // The staged activations are only the unit's K-range, so every token
    // count up to 8 fits for any nb.
    (void)nb;
    return GEMV_MAX_TOKENS;
}

// Opt-in shared memory for every instantiation on the current device
// (called once per context).
template <int TYPE, int M, bool FUSED>
static void configure_fused() {
    cudaFuncSetAttribute(q35k_decode_kernel<TYPE, M, FUSED, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GEMV_SMEM_LIMIT);
    cudaFuncSetAttribute(q35k_decode_kernel<TYPE, M, FUSED, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         GEMV_SMEM_LIMIT);
    if constexpr (M <= GEMV_FUSED_MAX_TOKENS) {
        cudaFuncSetAttribute(q35k_decode_kernel_10w<TYPE, M, FUSED, false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_SMEM_LIMIT);
        cudaFuncSetAttribute(q35k_decode_kernel_10w<TYPE, M, FUSED, true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_SMEM_LIMIT);
        if constexpr (TYPE == TYPE_Q4_K)
            cudaFuncSetAttribute(q35k_decode_kernel_20w<TYPE, M, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GEMV_SMEM_LIMIT);
    }
}

template <int TYPE, int M>
static void configure_typed() {
    configure_fused<TYPE, M, false>();
    if (M <= GEMV_FUSED_MAX_TOKENS) configure_fused<TYPE, M, M <= GEMV_FUSED_MAX_TOKENS>();
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

// Whole-row units (one unit per row group) run an instantiation without the
// split-K code; plans with three_per_sm the kernel with the larger register
// budget (a plan that would fit four CTAs per SM and needs them keeps the
// other); Q4_K whole rows of more than 10 warps at one or two tokens the
// 20-warp kernel bounded at two CTAs per SM.
template <int TYPE, int M, bool FUSED, bool SPLIT>
static cudaError_t launch_variant(cudaLaunchConfig_t& cfg, const GemvArgs& a, const GemvPlan& p) {
    if constexpr (M <= GEMV_FUSED_MAX_TOKENS)
        if (p.three_per_sm) return cudaLaunchKernelEx(&cfg, q35k_decode_kernel_10w<TYPE, M, FUSED, SPLIT>, a, p);
    if constexpr (M <= GEMV_FUSED_MAX_TOKENS && !SPLIT && TYPE == TYPE_Q4_K)
        if (p.warps > GEMV_SPLIT_WARPS) return cudaLaunchKernelEx(&cfg, q35k_decode_kernel_20w<TYPE, M, FUSED>, a, p);
    return cudaLaunchKernelEx(&cfg, q35k_decode_kernel<TYPE, M, FUSED, SPLIT>, a, p);
}

template <int TYPE, int M, bool FUSED>
static cudaError_t launch_split(cudaLaunchConfig_t& cfg, const GemvArgs& a, const GemvPlan& p) {
    return p.splits > 1 ? launch_variant<TYPE, M, FUSED, true>(cfg, a, p) : launch_variant<TYPE, M, FUSED, false>(cfg, a, p);
}

template <int TYPE, int M>
static cudaError_t launch_typed(const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
    if (!p.fits) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.grid);
    cfg.blockDim = dim3((unsigned)p.threads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int n = 0;
    if (pdl) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (p.cluster > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = (unsigned)p.cluster;
        attr[n].val.clusterDim.y = 1;
        attr[n++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    // The fused variant exists for small token counts only.
    constexpr bool F = M <= GEMV_FUSED_MAX_TOKENS;
    if (a.x != nullptr && !F) return cudaErrorInvalidValue;
    return a.x != nullptr ? launch_split<TYPE, M, F>(cfg, a, p) : launch_split<TYPE, M, false>(cfg, a, p);
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

bool gemv_fuses_quantize(int type, int nb, int n_out, int tokens, int num_sms) {
    if (tokens > GEMV_FUSED_MAX_TOKENS) return false;
    const GemvPlan p = plan_gemv(type, nb, n_out, tokens, num_sms);
    // Each warp quantizes at most two super-blocks of the unit's K-range.
    return tokens * p.unit_blocks <= 2 * p.warps;
}

// Row index of each token's fused-argmax key; the key is then cleared for the
// next call (the GEMV folds its outputs into it with atomicMax, after its own
// grid-dependency wait, i.e. after this kernel completed).  Launched with
// programmatic dependent launch: the next call's GEMV may start streaming its
// weights while this kernel waits for the one before it.
__global__ void argmax_index_kernel(unsigned long long* __restrict__ keys, int* __restrict__ idx, int tokens) {
    asm volatile("griddepcontrol.launch_dependents;");
    griddep_wait();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < tokens) {
        idx[t] = (int)(0xffffffffu - (uint32_t)(keys[t] & 0xffffffffull));
        keys[t] = 0ull;
    }
}

cudaError_t launch_argmax_index(unsigned long long* keys, int* idx, int tokens, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((tokens + 127) / 128));
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, argmax_index_kernel, keys, idx, tokens);
}

int gemv_plan_rows(const GemvArgs& a) {
    if (a.more.n <= 0) return a.n_out;
    const int k = a.more.n - 1;
    return a.more.g0[k] * TILE_ROWS + a.more.n_out[k];
}

cudaError_t launch_gemv(int type, const GemvArgs& a, cudaStream_t s, bool pdl) {
    if (a.more.n < 0 || a.more.n > GEMV_MAX_MATS - 1) return cudaErrorInvalidValue;
    const GemvPlan p = plan_gemv(type, a.nb, gemv_plan_rows(a), a.tokens, a.num_sms);
    switch (type) {
    case TYPE_Q4_K: return launch_m<TYPE_Q4_K>(a, p, s, pdl);
    case TYPE_Q5_K: return launch_m<TYPE_Q5_K>(a, p, s, pdl);
    case TYPE_Q6_K: return launch_m<TYPE_Q6_K>(a, p, s, pdl);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace q35k
