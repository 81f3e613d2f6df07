// device_common.cuh -- constants, tile layout and sm_100a PTX helpers shared
// by the libq35k kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q35k {

constexpr int QK = 256;
constexpr int Q8K_BYTES = 292;  // f32 d | s8 qs[256] | s16 bsums[16]
constexpr int TYPE_Q4_K = 12, TYPE_Q5_K = 13, TYPE_Q6_K = 14;

// Device error word bits (read back by the host after a call).
constexpr unsigned DEV_ERR_TIMEOUT = 1u;

// Rows per tile: one warp lane per weight row.
constexpr int TILE_ROWS = 32;

// ---------------------------------------------------------------------------
// HBM tile layout of an uploaded weight.
//
// Rows are grouped 32 at a time (padded with zero blocks to a multiple of 32).
// Tile (g, b) holds super-block b of rows 32g..32g+31 and sits at byte offset
// (g * nb + b) * TILE_BYTES, so the tiles of one row group are contiguous in
// K.  Inside a tile the block bytes are stored chunk-major: 16-byte chunk c of
// row r is at c * 512 + r * 16.  A warp whose lane r decodes row r therefore
// reads each chunk as one contiguous, bank-conflict-free 512-byte line.
// Q6_K blocks (210 B = 13 chunks + 2 bytes) keep their trailing fp16 d in a
// 64-byte row-indexed tail at 13 * 512.  The block bytes are unchanged; only
// their placement differs from the GGUF rows, so a tile is exactly
// 32 * block_bytes bytes.
// ---------------------------------------------------------------------------
template <int TYPE> struct Fmt;
template <> struct Fmt<TYPE_Q4_K> {
    static constexpr int BLOCK = 144, CHUNKS = 9, TILE = 32 * 144;
};
template <> struct Fmt<TYPE_Q5_K> {
    static constexpr int BLOCK = 176, CHUNKS = 11, TILE = 32 * 176;
};
template <> struct Fmt<TYPE_Q6_K> {
    static constexpr int BLOCK = 210, CHUNKS = 13, TILE = 32 * 210;
    static constexpr int D_OFFSET = 13 * 512;
};

__host__ __device__ inline int block_bytes(int type) {
    return type == TYPE_Q4_K ? 144 : type == TYPE_Q5_K ? 176 : type == TYPE_Q6_K ? 210 : 0;
}

// ---------------------------------------------------------------------------
// Planar Q8_K activations, the GEMV's input layout: the same values as
// BlockQ8K (Kernels/BlockLayout.cs:41-46) split into three planes, block-major
// so that the super-blocks [b0, b0+n) of all rows are one contiguous,
// 16-byte aligned range per plane (three bulk copies stage a K-range):
//   qs [nb][rows][256] int8 | d [nb][rows4] f32 (rows4 = rows rounded up
//   to 4) | bsums [nb][rows][16] int16.
// Tokens are grouped in chunks of `chunk` rows (one GEMV launch each); chunk
// j starts at j * q8_planar(chunk, nb).bytes and its planes are sized by its
// own row count.  In a chunk of q8_interleave_min_rows(type) or more rows the
// qs plane is word-interleaved instead, [nb][64][rows] 32-bit words (word w =
// values 4w..4w+3): the layout in which the tensor-core GEMV (gemv_dot.cuh)
// reads its B fragments, one coalesced 32-bit load per lane.  The mma form's
// cost per tile does not depend on the token count while the dp4a form's
// grows with it; on B200 the mma form wins from 3 tokens for Q4_K / Q5_K and
// from 6 for Q6_K (whose dp4a decode is cheaper per token).
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int q8_interleave_min_rows(int type) { return type == TYPE_Q6_K ? 6 : 3; }
struct Q8Planar {
    size_t qs, d, bs, bytes;
    int rows, rows4;
};
__host__ __device__ inline Q8Planar q8_planar(int rows, int nb) {
    Q8Planar p;
    p.rows = rows;
    p.rows4 = (rows + 3) / 4 * 4;
    p.qs = 0;
    p.d = (size_t)nb * rows * QK;
    p.bs = p.d + (size_t)nb * p.rows4 * 4;
    p.bytes = p.bs + (size_t)nb * rows * 32;
    return p;
}
// Total bytes of `rows` tokens stored in chunks of `chunk`.
__host__ __device__ inline size_t q8_planar_total(int rows, int nb, int chunk) {
    const int full = rows / chunk, rem = rows % chunk;
    return (size_t)full * q8_planar(chunk, nb).bytes + (rem ? q8_planar(rem, nb).bytes : 0);
}

// ---------------------------------------------------------------------------
// PTX helpers (mbarrier + bulk async copy, sm_90+ / sm_100a).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared, completion counted on `bar` (no multicast).
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps in the barrier unit (up to `hint_ns`) instead of spinning on the
// issue slots that the working warps of its sub-partition need.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Relaxed system-scope 64-bit access (values exchanged between GPUs; an
// aligned 64-bit access is single-copy atomic).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase.  Gives up after `limit_ns` of wall time,
// records DEV_ERR_TIMEOUT in *err and returns false: no device wait here can
// spin forever.  The waiting warp sleeps in the barrier unit between tests
// (suspend-time hint) rather than spending issue slots that the decoding
// warps of its SM sub-partition need.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 1000000u)) return true;
        if (globaltimer_ns() - start > limit_ns) {
            atomicOr(err, DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float fp16_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

}  // namespace q35k
