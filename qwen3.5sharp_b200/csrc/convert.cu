// convert.cu -- Q8_K activation quantization, bit-exact dequantization and the
// upload-time tile repack.
//
// Bit-exactness: every fp32 operation below is an explicitly rounded
// intrinsic (__fdiv_rn, __fmul_rn, __fsub_rn, __float2int_rn), so nvcc cannot
// contract or reassociate it; each mirrors one separately rounded C#
// operation of the reference (RyuJIT emits no FMA on these paths).
#include "device_common.cuh"
#include "kernels.h"
#include "q8k_quant.cuh"

namespace q35k {

// Launch with programmatic stream serialization: the kernel may become
// resident while the kernel before it in the stream drains (it waits on the
// grid dependency before touching memory), and lets its own dependent start.
template <typename... P, typename... A>
static cudaError_t launch_dependent(void (*kernel)(P...), int grid, int block, cudaStream_t s, A... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);
}

// ---------------------------------------------------------------------------
// Q8_K quantization: one warp per 256-value super-block (q8k_quant.cuh).
// Output goes either to BlockQ8K blocks (chunk == 0) or to the planar layout
// (device_common.cuh) in chunks of `chunk` rows.
// ---------------------------------------------------------------------------
__device__ __forceinline__ Q8Out q8_out(uint8_t* q8, int row, int b, int nb, int rows, int chunk, int ilv_rows) {
    Q8Out o;
    if (chunk == 0) {
        uint8_t* blk = q8 + ((size_t)row * nb + b) * Q8K_BYTES;
        o.d = reinterpret_cast<uint32_t*>(blk);
        o.qs = reinterpret_cast<uint32_t*>(blk + 4);
        o.bs = reinterpret_cast<int16_t*>(blk + 260);
    } else {
        const int j = row / chunk, rr = row % chunk;
        const int mj = min(chunk, rows - j * chunk);
        uint8_t* base = q8 + (size_t)j * q8_planar(chunk, nb).bytes;
        const Q8Planar pl = q8_planar(mj, nb);
        const size_t blk = (size_t)b * mj + rr;  // block-major
        o.d = reinterpret_cast<uint32_t*>(base + pl.d) + (size_t)b * pl.rows4 + rr;
        if (ilv_rows > 0 && mj >= ilv_rows) {
            // word w of row rr at word w * mj + rr of the block's qs
            o.qs = reinterpret_cast<uint32_t*>(base + pl.qs + (size_t)b * mj * QK) + rr;
            o.qs_stride = mj;
        } else {
            o.qs = reinterpret_cast<uint32_t*>(base + pl.qs + blk * QK);
        }
        o.bs = reinterpret_cast<int16_t*>(base + pl.bs + blk * 32);
    }
    return o;
}

__global__ void __launch_bounds__(256) quantize_q8k_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                                           uint8_t* __restrict__ q8, int nb, int total_blocks, int rows,
                                                           int chunk, int ilv_rows) {
    // A GEMV launched after this kernel with programmatic stream
    // serialization may start now: it streams weights first and waits on the
    // grid dependency (full completion of this grid) before reading q8.
    asm volatile("griddepcontrol.launch_dependents;");
    // This kernel is itself launched as a programmatic dependent: x comes
    // from the kernel before it, and q8 may still be read by it (the
    // previous call's GEMV).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= total_blocks) return;
    const int row = warp / nb, b = warp % nb;
    const size_t off = (size_t)row * nb * QK + (size_t)b * QK;
    warp_quantize_q8k_block(x + off, q8_out(q8, row, b, nb, rows, chunk, ilv_rows), lane, up ? up + off : nullptr);
}

cudaError_t launch_quantize_q8k(const float* x, uint8_t* q8, int k, int rows, int planar_chunk, cudaStream_t s,
                                const float* up, int ilv_rows) {
    const int nb = k / QK;
    const int total = nb * rows;
    if (total == 0) return cudaSuccess;
    const int warps_per_cta = 8;
    return launch_dependent(quantize_q8k_kernel, (total + warps_per_cta - 1) / warps_per_cta, warps_per_cta * 32, s,
                            x, up, q8, nb, total, rows, planar_chunk, ilv_rows);
}

// BlockQ8K rows (a caller's pre-quantized activations) -> the planar layout,
// one warp per block: word 0 = d, 1..64 = qs, 65..72 = bsums.
__global__ void __launch_bounds__(256) q8k_to_planar_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                            int nb, int total_blocks, int rows, int chunk,
                                                            int ilv_rows) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // dst may still be read by the kernel before
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= total_blocks) return;
    const uint32_t* in = reinterpret_cast<const uint32_t*>(src + (size_t)warp * Q8K_BYTES);
    const Q8Out out = q8_out(dst, warp / nb, warp % nb, nb, rows, chunk, ilv_rows);
    if (lane == 0) *out.d = __ldg(in);
    out.qs[lane * out.qs_stride] = __ldg(in + 1 + lane);
    out.qs[(32 + lane) * out.qs_stride] = __ldg(in + 33 + lane);
    if (lane < 8) reinterpret_cast<uint32_t*>(out.bs)[lane] = __ldg(in + 65 + lane);
}

cudaError_t launch_q8k_to_planar(const uint8_t* src, uint8_t* dst, int k, int rows, int chunk, cudaStream_t s,
                                 int ilv_rows) {
    const int nb = k / QK;
    const int total = nb * rows;
    if (total == 0) return cudaSuccess;
    const int warps_per_cta = 8;
    return launch_dependent(q8k_to_planar_kernel, (total + warps_per_cta - 1) / warps_per_cta, warps_per_cta * 32, s,
                            src, dst, nb, total, rows, chunk, ilv_rows);
}

// ---------------------------------------------------------------------------
// Dequantization: one CTA of 256 threads per super-block, thread l -> value l.
// Q4K.DequantizeRow (Kernels/Q4K.cs:35-60), Q5K.DequantizeRow
// (Kernels/Q5K.cs:5-35), Q6K.DequantizeRow (Kernels/Q6K.cs:9-39).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, int& sc, int& m) {
    // Q4K.GetScaleMin (Kernels/Q4K.cs:7-18).
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__global__ void __launch_bounds__(256) dequant_kernel(int type, const uint8_t* __restrict__ blocks,
                                                      float* __restrict__ y) {
    const int blk = blockIdx.x;
    const int l = threadIdx.x;
    const int bb = block_bytes(type);
    const uint8_t* b = blocks + (size_t)blk * bb;
    float out;
    if (type == TYPE_Q6_K) {
        // value l: half h = l/128, within-half position p, quarter qq = p/32, l32 = p%32
        const int h = l >> 7, p = l & 127, qq = p >> 5, l32 = p & 31;
        const uint8_t* ql = b + 64 * h;
        const uint8_t* qh = b + 128 + 32 * h;
        const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + 8 * h;
        const float d = fp16_bits_to_float(b[208] | (b[209] << 8));
        const int lo_src = (qq & 1) ? ql[l32 + 32] : ql[l32];
        const int nib = (qq < 2) ? (lo_src & 0xF) : (lo_src >> 4);
        const int hb = (qh[l32] >> (2 * qq)) & 3;
        const int q = nib | (hb << 4);
        const int is = l32 / 16 + 2 * qq;
        out = __fmul_rn(__fmul_rn(d, (float)sc[is]), (float)(q - 32));
    } else {
        const float d = fp16_bits_to_float(b[0] | (b[1] << 8));
        const float dmin = fp16_bits_to_float(b[2] | (b[3] << 8));
        const int c = l >> 6, hi = (l >> 5) & 1, l32 = l & 31;
        int sc, m;
        scale_min_k4(2 * c + hi, b + 4, sc, m);
        int q;
        if (type == TYPE_Q4_K) {
            const uint8_t byte = b[16 + 32 * c + l32];
            q = hi ? (byte >> 4) : (byte & 0xF);
        } else {
            const uint8_t byte = b[48 + 32 * c + l32];
            const uint8_t h = b[16 + l32];
            q = (hi ? (byte >> 4) : (byte & 0xF)) + (((h >> (2 * c + hi)) & 1) ? 16 : 0);
        }
        const float d1 = __fmul_rn(d, (float)sc);
        const float m1 = __fmul_rn(dmin, (float)m);
        out = __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    y[(size_t)blk * QK + l] = out;
}

cudaError_t launch_dequantize(int type, const uint8_t* blocks, float* y, int k, int rows, cudaStream_t s) {
    const long total = (long)(k / QK) * rows;
    if (total == 0) return cudaSuccess;
    dequant_kernel<<<(unsigned)total, 256, 0, s>>>(type, blocks, y);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Upload-time repack: GGUF rows -> 32-row chunk-major tiles.  One thread per
// (row, block, 16-byte chunk); rows >= n_out become zero blocks (d = 0, so
// they contribute nothing and their outputs are never stored).
// ---------------------------------------------------------------------------
__global__ void repack_tiles_kernel(int type, const uint8_t* __restrict__ src, uint8_t* __restrict__ tiles, int nb,
                                    int n_out, int n_pad) {
    const int bb = block_bytes(type);
    const int chunks = (bb + 15) / 16;  // 9, 11, 14 (Q6_K: 13 full + tail)
    const long tid = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long total = (long)n_pad * nb * chunks;
    if (tid >= total) return;
    const int c = (int)(tid % chunks);
    const long rb = tid / chunks;
    const int b = (int)(rb % nb);
    const int row = (int)(rb / nb);
    const int g = row / TILE_ROWS, r = row % TILE_ROWS;
    uint8_t* tile = tiles + ((size_t)g * nb + b) * (size_t)(TILE_ROWS * bb);
    const uint8_t* blk = src + ((size_t)row * nb + b) * bb;
    const bool live = row < n_out;
    if (type == TYPE_Q6_K && c == 13) {
        uint8_t* dst = tile + 13 * 512 + r * 2;
        dst[0] = live ? blk[208] : 0;
        dst[1] = live ? blk[209] : 0;
        return;
    }
    uint8_t* dst = tile + c * 512 + r * 16;
#pragma unroll
    for (int i = 0; i < 16; i++) dst[i] = live ? blk[c * 16 + i] : 0;
}

cudaError_t launch_repack_tiles(int type, const uint8_t* rows_src, uint8_t* tiles, int nb, int n_out, int n_pad,
                                cudaStream_t s) {
    const int bb = block_bytes(type);
    const int chunks = (bb + 15) / 16;
    const long total = (long)n_pad * nb * chunks;
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    repack_tiles_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, s>>>(type, rows_src, tiles, nb,
                                                                                        n_out, n_pad);
    return cudaGetLastError();
}

}  // namespace q35k
