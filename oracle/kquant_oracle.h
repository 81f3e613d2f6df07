/*
 * kquant_oracle.h -- CPU restatement of the Qwen35Sharp K-quant matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libq35k) links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker / the timed CPU reference.
 *
 * PARITY UNPINNED: the reference (DracoUnion/Qwen3.5Sharp) is managed C#
 * (.NET 10) and cannot be built or run here (no dotnet SDK), and its test
 * project holds no golden vectors or known-answer tests for Q4_K/Q5_K/Q6_K.
 * This restatement is cross-checked instead against (a) an independent
 * pure-Python restatement of the same C# formulas, (b) hand-derived
 * known-answer blocks, and (c) its own scalar-vs-AVX2 pairing, the pattern the
 * reference's own tests use.
 *
 * Two layers are restated:
 *   - semantics:   the scalar C# methods (DotScalar, Q5K.Dot, GemmScalar, ...)
 *   - execution:   the AVX2 instruction sequences the reference actually runs
 *                  (VecDotQ4K.DotAvx2, Q6K.DotAvx2/DotAvx2x4,
 *                  GemmQ4K.GemmAvx2Tile, QuantizeQ8Kx4.Quantize4x8Avx2),
 *                  threaded with the reference's static row partition.  This
 *                  layer is the timed CPU baseline.
 * Every function cites the reference file:line it follows (paths relative to
 * src/Qwen35Sharp.Kernels/ unless stated otherwise).
 */
#ifndef KQUANT_ORACLE_H
#define KQUANT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type codes (src/Qwen35Sharp.Gguf/GgmlTensorType.cs). */
enum { OQ_Q4_K = 12, OQ_Q5_K = 13, OQ_Q6_K = 14 };

/* Block sizes (BlockLayout.cs:8-29). */
enum {
    OQ_QK = 256,
    OQ_Q4K_BYTES = 144,
    OQ_Q5K_BYTES = 176,
    OQ_Q6K_BYTES = 210,
    OQ_Q8K_BYTES = 292,
    OQ_Q4KX8_BYTES = 1152,
    OQ_Q4KX8_META_BYTES = 448,
    OQ_Q8KX4_BYTES = 1168
};

/* fp16 <-> fp32 (HalfBits.ToSingle / FromSingle, BlockLayout.cs:166-168). */
float oq_fp16_to_f32(uint16_t h);
uint16_t oq_f32_to_fp16(float f);

int oq_block_bytes(int type);

/* Q8_K activation quantizer, Q8K.QuantizeRow (Q8K.cs:12-77) with ScaleBlock
 * (Q8K.cs:83-146).  `_scalar` follows the non-AVX branches, `_avx2` the AVX2
 * branches; both must produce identical bytes. */
void oq_quantize_q8k_scalar(const float* x, void* y, int k);
void oq_quantize_q8k_avx2(const float* x, void* y, int k);

/* Dequantize one row of k values (Q4K.cs:35-60, Q5K.cs:5-35, Q6K.cs:9-39). */
int oq_dequantize(int type, const void* blocks, float* y, int k);

/* Row dot products against one Q8_K row.
 *   semantic: VecDotQ4K.DotScalar (VecDotQ4K.cs:16-65), Q5K.Dot (Q5K.cs:37-87),
 *             Q6K.DotScalar (Q6K.cs:44-85)
 *   executed: VecDotQ4K.DotAvx2 (VecDotQ4K.cs:67-126), Q5K.Dot (scalar only),
 *             Q6K.DotAvx2 (Q6K.cs:87-167) */
float oq_dot_scalar(int type, const void* w, const void* q8, int n);
float oq_dot_avx2(int type, const void* w, const void* q8, int n);

/* Q6K.DotAvx2x4 (Q6K.cs:172-248): one weight row against four Q8_K rows. */
void oq_dot_q6k_avx2x4(const void* w, const void* y0, const void* y1,
                       const void* y2, const void* y3, int n, float* dst);

/* Q8_Kx4 quantizer, QuantizeQ8Kx4.Quantize4x8Avx2 (QuantizeQ8Kx4.cs:108-144,
 * FillBsums :191-203).  x holds 4 rows of k floats. */
void oq_quantize_q8kx4(const float* x, void* y, int k);

/* Load-time Q4_K panel repack (RepackQ4K.cs:5-85) and meta sidecar
 * (RepackQ4K.cs:91-130).  nOut must be a multiple of 8. */
void oq_repack_q4kx8(const void* src, void* dst, int nIn, int nOut);
void oq_build_meta_q4kx8(const void* src, void* dst, int nIn, int nOut);

/* Q4_K x Q8_K panel GEMM semantics (GemmQ4K.GemmScalar, GemmQ4K.cs:25-106),
 * restated on row-major blocks: dst[t*ldc + c] for t<rows (rows%4==0),
 * c<cols (cols%8==0).  q8 holds `rows` Q8_K rows (same q/d as Q8_Kx4). */
void oq_gemm_q4k_semantic(const void* w, const void* q8, float* dst, int ldc,
                          int nIn, int rows, int cols);

/* ---- Reference dispatch (threaded, static partition) ------------------- */

/* A prepared weight: raw row-major blocks plus, for Q4_K, the load-time panel
 * and meta (Qwen35Model.LoadWeights, Model/Qwen35Model.cs:463-565). */
typedef struct oq_weight oq_weight;
oq_weight* oq_weight_prepare(int type, const void* blocks, int nIn, int nOut);
void oq_weight_release(oq_weight* w);

/* Linear / DecodeLinear (Model/Qwen35Model.Decode.cs:22-87):
 *   Q4_K: tokens==1 -> MulMatQ4K.Gemv, else MulMatQ4K.Gemm (MulMatQ4K.cs:12-127)
 *   Q5_K: Q5K.Gemm = per-token Gemv (Q5K.cs:89-118)
 *   Q6_K: Q6K.Gemm (Q6K.cs:317-413)
 * threads = worker count of the CpuThreadPool (CpuThreadPool.cs:46-92). */
int oq_matmul(const oq_weight* w, const float* x, float* y, int tokens, int threads);

/* GemvPrequant (Decode.cs:89-112) for each of `tokens` Q8_K rows. */
int oq_matmul_q8k(const oq_weight* w, const void* q8k, float* y, int tokens, int threads);

/* Scalar semantics of the same dispatch, single thread (the parity target
 * that is independent of the AVX2 summation order). */
int oq_matmul_semantic(const oq_weight* w, const float* x, float* y, int tokens);

#ifdef __cplusplus
}
#endif
#endif
