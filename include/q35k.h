/*
 * q35k.h -- C ABI of libq35k, the B200 (sm_100a) implementation of the
 * Qwen35Sharp quantized y = x @ W^T path for GGUF Q4_K, Q5_K and Q6_K weights.
 *
 * Each entry point replaces one reference kernel entry point the model
 * forward pass calls (reference paths are relative to the DracoUnion/
 * Qwen3.5Sharp tree; "Kernels/" = src/Qwen35Sharp.Kernels/, "Model/" =
 * src/Qwen35Sharp.Model/).  The C# P/Invoke declarations a maintainer adds
 * next to those entry points ship as bindings/Q35k.cs.
 *
 * Conventions (mirroring the reference's, Model/Qwen35Model.Decode.cs:13-112):
 *   - Matrices are row-major: x is [tokens][n_in] fp32, y is [tokens][n_out]
 *     fp32; weights are GGUF rows of n_in/256 super-blocks (dim0 innermost).
 *   - n_in must be a multiple of 256 (Model/Qwen35Model.cs:480-481).
 *   - Host-pointer calls are synchronous: y is complete on return.  The
 *     `_dev` variants take device pointers and a cudaStream_t (as void*) and
 *     are asynchronous on that stream.
 *   - One context per caller thread.  Calls on one context must not overlap
 *     on the GPU (the context's split-K scratch is shared), exactly as the
 *     reference's CpuThreadPool/ScratchArena pair is not re-entrant.
 *   - Every call returns a status; q35k_last_error() describes the last
 *     failure.  The C# shim maps statuses to the exception types the
 *     reference throws (the comments on the Q35K_E* codes below).
 *   - There is no CPU fallback: a context cannot be created without an
 *     sm_100 device.
 */
#ifndef Q35K_H
#define Q35K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define Q35K_OK 0
#define Q35K_EINVAL 1   /* bad argument           -> ArgumentException */
#define Q35K_ENOTSUP 2  /* unsupported type/shape -> NotSupportedException */
#define Q35K_ENOMEM 3   /* device/host allocation -> InsufficientMemoryException */
#define Q35K_ECUDA 4    /* CUDA runtime error     -> InvalidOperationException */
#define Q35K_ETIMEOUT 5 /* a bounded device wait expired -> TimeoutException */
#define Q35K_ENCCL 6    /* NCCL error             -> InvalidOperationException */
#define Q35K_EDATA 7    /* malformed/truncated GGUF -> InvalidDataException */
#define Q35K_EIO 8      /* file cannot be opened/mapped -> IOException */

/* GGML tensor type codes (src/Qwen35Sharp.Gguf/GgmlTensorType.cs). */
#define Q35K_TYPE_Q4_K 12
#define Q35K_TYPE_Q5_K 13
#define Q35K_TYPE_Q6_K 14

/* Wire sizes (Kernels/BlockLayout.cs:8-29). */
#define Q35K_QK 256
#define Q35K_Q4K_BYTES 144
#define Q35K_Q5K_BYTES 176
#define Q35K_Q6K_BYTES 210
#define Q35K_Q8K_BYTES 292

typedef struct q35k_ctx q35k_ctx;
typedef struct q35k_weight q35k_weight;

/* ---- Context ----------------------------------------------------------- */

/* Create a context on CUDA device `device` (must be sm_100).  Replaces the
 * reference's per-model CpuThreadPool + ScratchArena pair
 * (Kernels/CpuThreadPool.cs:25-44, Kernels/ScratchArena.cs:7-47). */
int q35k_create(int device, q35k_ctx** out);
int q35k_destroy(q35k_ctx* ctx);
/* Message of the last failure on this context (never NULL). */
const char* q35k_last_error(const q35k_ctx* ctx);
/* Library version string. */
const char* q35k_version(void);
/* Wait for the context's stream and report any device-side error word
 * (a bounded wait that expired inside a kernel). */
int q35k_sync(q35k_ctx* ctx);

/* ---- Weights (Model/Qwen35Model.cs:463-565, LoadWeights) --------------- */

/* Upload n_out rows of GGUF blocks of type ggml_type from host memory, once
 * per tensor; the handle owns the device copy (re-laid out for the kernels;
 * the block bytes are unchanged).  Replaces the load-time copy + repack
 * (Model/Qwen35Model.cs:498-524, Kernels/RepackQ4K.cs:71-130). */
int q35k_weight_upload(q35k_ctx* ctx, int ggml_type, const void* blocks, int n_in, int n_out,
                       q35k_weight** out);
int q35k_weight_free(q35k_ctx* ctx, q35k_weight* w);
int q35k_weight_info(const q35k_weight* w, int* ggml_type, int* n_in, int* n_out, size_t* device_bytes);

/* ---- Matmul ------------------------------------------------------------ */

/* y[tokens][n_out] = x[tokens][n_in] @ W^T with the reference's arithmetic:
 * x rows are quantized to Q8_K, per-super-block integer dots are scaled by the
 * fp16 block scales.  Host pointers, synchronous.  Replaces
 *   Linear       (Model/Qwen35Model.Decode.cs:22-52)  -> MulMatQ4K.Gemm
 *                (Kernels/MulMatQ4K.cs:45-127), Q5K.Gemm (Kernels/Q5K.cs:114-118),
 *                Q6K.Gemm (Kernels/Q6K.cs:317-353);
 *   DecodeLinear (Model/Qwen35Model.Decode.cs:59-87)  -> MulMatQ4K.Gemv
 *                (Kernels/MulMatQ4K.cs:12-26), Q5K.Gemv (Kernels/Q5K.cs:89-95),
 *                Q6K.Gemv (Kernels/Q6K.cs:301-315). */
int q35k_matmul(q35k_ctx* ctx, const q35k_weight* w, const float* x, float* y, int tokens);

/* Same with `tokens` caller-quantized Q8_K rows (BlockQ8K, 292 bytes per 256
 * values, Kernels/BlockLayout.cs:41-46).  Replaces GemvPrequant
 * (Model/Qwen35Model.Decode.cs:89-112) -> MulMatQ4K.GemvPrequant
 * (Kernels/MulMatQ4K.cs:28-43), Q5K.GemvPrequant (Kernels/Q5K.cs:97-112),
 * Q6K.GemvPrequant (Kernels/Q6K.cs:415-430). */
int q35k_matmul_q8k(q35k_ctx* ctx, const q35k_weight* w, const void* q8k, float* y, int tokens);

/* Page-lock a caller's host buffer (cudaHostRegister, mapped and portable) so
 * that the host-pointer calls use it in place: q35k_matmul copies x straight
 * from it and -- for decode calls -- has the GEMV store y over the bus
 * straight into it, instead of staging both through the context's pinned
 * buffers (one host memcpy of y per call saved).  No counterpart in the
 * reference, whose model keeps persistent input and output buffers
 * (NativeBuffer, Kernels/NativeBuffer.cs:5-35; the ScratchArena slots); those
 * are the buffers to register, once, at load.  Buffers that are already
 * page-locked (pinned allocations) are used in place without registering.
 * Unregister before freeing the memory.  Q35K_EINVAL if the range is already
 * registered, Q35K_ENOMEM if the pages cannot be locked. */
int q35k_host_register(q35k_ctx* ctx, void* ptr, size_t bytes);
int q35k_host_unregister(q35k_ctx* ctx, void* ptr);

/* Device-pointer variants of the two calls above, asynchronous on `stream`
 * (a cudaStream_t; NULL = the context's own stream). */
int q35k_matmul_dev(q35k_ctx* ctx, const q35k_weight* w, const float* d_x, float* d_y, int tokens,
                    void* stream);
int q35k_matmul_q8k_dev(q35k_ctx* ctx, const q35k_weight* w, const void* d_q8k, float* d_y, int tokens,
                        void* stream);

/* Vocab head + ArgMax (Qwen35Sharp.Cli/Program.cs:127-140, after the logits
 * of Qwen35Model.cs:280-290): idx[t] = the first row holding the largest
 * logit of token t (strict '>' scan from row 0; a NaN at row 0 keeps row 0,
 * later NaNs are never taken), computed in the GEMV's epilogue so the logits
 * need not be written (d_y may be NULL; if given, the logits are written too).
 * Runs the decode GEMV for any token count.  The host variant is synchronous
 * and writes no logits. */
int q35k_matmul_argmax(q35k_ctx* ctx, const q35k_weight* w, const float* x, int* idx, int tokens);
int q35k_matmul_argmax_dev(q35k_ctx* ctx, const q35k_weight* w, const float* d_x, float* d_y, int* d_idx, int tokens,
                           void* stream);

/* Up to Q35K_MAX_SHARED weights with the same nIn applied to one input, with
 * one quantization of it: ys[i] [tokens][nOut_i] = x @ ws[i]^T.  Replaces
 * MulMatPanel.QuantizeAndGemm (Kernels/MulMatPanel.cs:27-54, up to three
 * panel GEMMs on one Q8_Kx4 panel) and the decode pattern of one
 * Q8K.QuantizeRow feeding GemvPrequant per weight: DecodeGateUp
 * (Model/Qwen35Model.Decode.cs:254-265, ffn_gate / ffn_up) and DecodeAttention
 * (Model/Qwen35Model.Decode.cs:286-292, attn_q / attn_k / attn_v).  Decode
 * weights of one type run in one GEMV launch.  ws and ys are host arrays of
 * `count` entries (ys of device pointers in the _dev variant). */
#define Q35K_MAX_SHARED 4
int q35k_matmul_shared(q35k_ctx* ctx, const q35k_weight* const* ws, int count, const float* x, float* const* ys,
                       int tokens);
int q35k_matmul_shared_dev(q35k_ctx* ctx, const q35k_weight* const* ws, int count, const float* d_x,
                           float* const* d_ys, int tokens, void* stream);

/* ffn_down on SiLU(gate) * up: y = (silu(gate) . up) @ W^T, gate and up
 * [tokens][nIn], silu(g) = g / (1 + exp(-g)).  The product is formed inside
 * the Q8_K quantization of the call (no intermediate written).  Replaces
 * MulMatPanel.SiluQuantizeAndGemm (Kernels/MulMatPanel.cs:57-79, with
 * QuantizeQ8Kx4.Quantize4x8Silu, Kernels/QuantizeQ8Kx4.cs:24-35) and the
 * decode sequence Ops.SiLUMul (Model/Ops.cs:624-675) + DecodeLinear(ffn_down)
 * (Model/Qwen35Model.Decode.cs:248-249). */
int q35k_matmul_silu(q35k_ctx* ctx, const q35k_weight* w, const float* gate, const float* up, float* y, int tokens);
int q35k_matmul_silu_dev(q35k_ctx* ctx, const q35k_weight* w, const float* d_gate, const float* d_up, float* d_y,
                         int tokens, void* stream);

/* Arithmetic of the tensor-core prefill GEMM (tokens >= 16).  No
 * counterpart in the reference, which has one arithmetic:
 *   Q35K_GEMM_EXACT (default): the reference's -- Q8_K activations, exact
 *     products, fp32 scaling per super-block (results within fp32 rounding
 *     of the reference's).  Every type runs on the tensor cores; Q6_K, whose
 *     sc * (q - 32) needs 12 significant bits, as two exact fp16 parts
 *     (sc = 16 sh + sl) and two MMAs per K step;
 *   Q35K_GEMM_FAST: fp16-rounded dequantized weights times fp16-rounded
 *     dequantized Q8_K activations, one fp32 accumulator per tile (2-4.5e-4
 *     of max |y| from the reference's results, whatever the scales: each
 *     weight row, and each token whose largest |x| is outside [2^-4, 2^15),
 *     is normalised by a power of two before the rounding); faster.  A
 *     weight with an infinite or NaN block scale (flagged at upload) keeps
 *     the exact path. */
#define Q35K_GEMM_EXACT 0
#define Q35K_GEMM_FAST 1
int q35k_set_gemm_mode(q35k_ctx* ctx, int mode);

/* ---- Utilities ---------------------------------------------------------- */

/* Q8K.QuantizeRow (Kernels/Q8K.cs:12-77) on `rows` rows of k floats:
 * bit-exact BlockQ8K bytes (rows * k/256 * 292). */
int q35k_quantize_q8k(q35k_ctx* ctx, const float* x, void* q8k, int k, int rows);
int q35k_quantize_q8k_dev(q35k_ctx* ctx, const float* d_x, void* d_q8k, int k, int rows, void* stream);
/* The same on silu(gate) * up, the product formed inside the quantizer:
 * QuantizeQ8Kx4.Quantize4x8Silu (Kernels/QuantizeQ8Kx4.cs:24-35) in the
 * BlockQ8K layout (the quantization of q35k_matmul_silu). */
int q35k_quantize_q8k_silu(q35k_ctx* ctx, const float* gate, const float* up, void* q8k, int k, int rows);
int q35k_quantize_q8k_silu_dev(q35k_ctx* ctx, const float* d_gate, const float* d_up, void* d_q8k, int k, int rows,
                               void* stream);

/* Q4K/Q5K/Q6K.DequantizeRow (Kernels/Q4K.cs:35-60, Kernels/Q5K.cs:5-35,
 * Kernels/Q6K.cs:9-39) on `rows` rows of k values: bit-exact fp32. */
int q35k_dequantize(q35k_ctx* ctx, int ggml_type, const void* blocks, float* y, int k, int rows);
int q35k_dequantize_dev(q35k_ctx* ctx, int ggml_type, const void* d_blocks, float* d_y, int k, int rows,
                        void* stream);

/* ---- Row-sharded matmul over the GPUs of one node ------------------------
 *
 * The reference splits output rows between the workers of its CpuThreadPool
 * (Kernels/MulMatQ4K.cs:31-36, Kernels/CpuThreadPool.cs:46-92); here a group
 * of GPUs ("ranks") each holds rows [r * n_shard, (r + 1) * n_shard) of a
 * weight (n_shard = ceil(n_out / ranks); the last rank may hold fewer), computes its slice
 * of y, and the slices are all-gathered over NVLink so that every rank holds
 * the full y. */
typedef struct q35k_shard q35k_shard;
typedef struct q35k_sharded_weight q35k_sharded_weight;
#define Q35K_GATHER_NCCL 0 /* NCCL all-gather (any group) */
#define Q35K_GATHER_PEER 1 /* peer copies over NVLink (all ranks in one process) */
/* Fused into the decode GEMV: each rank stores its slice straight into every
 * peer's buffer over NVLink and raises a flag there; a bounded wait replaces
 * the collective.  Calls of at most Q35K_STATIC_MAX_TOKENS tokens and groups
 * of at most 8 ranks; other calls fall back to the NCCL gather (the peer
 * copies in a process without NCCL).  Calls of one group must not overlap. */
#define Q35K_GATHER_FUSED 2
#define Q35K_NCCL_ID_BYTES 128

/* One process driving `ndev` GPUs (NCCL communicators from ncclCommInitAll). */
int q35k_shard_create(int ndev, const int* devices, q35k_shard** out);
/* One process per GPU: rank `rank` of `nranks` on `device`; every rank
 * passes the same id, made by one of them with q35k_nccl_unique_id and
 * shared by the caller's own means. */
int q35k_nccl_unique_id(void* id_out /* Q35K_NCCL_ID_BYTES */);
int q35k_shard_create_rank(int nranks, int rank, const void* nccl_id, int device, q35k_shard** out);
int q35k_shard_destroy(q35k_shard* s);
const char* q35k_shard_last_error(const q35k_shard* s);
int q35k_shard_info(const q35k_shard* s, int* nranks, int* first_rank, int* local_devices);
int q35k_shard_sync(q35k_shard* s);
/* Upload the local ranks' rows of a full GGUF weight (n_out rows, host). */
int q35k_shard_weight_upload(q35k_shard* s, int ggml_type, const void* blocks, int n_in, int n_out,
                             q35k_sharded_weight** out);
int q35k_shard_weight_free(q35k_shard* s, q35k_sharded_weight* w);
/* y = x @ W^T with x replicated on every local device (d_x[i]) and the full
 * y [tokens][n_out] written to every local device (d_y[i]); asynchronous on
 * streams[i] (cudaStream_t of local device i; NULL array or entry = the
 * group's own streams, which q35k_shard_sync waits for). */
int q35k_shard_matmul_dev(q35k_shard* s, const q35k_sharded_weight* w, const float* const* d_x, float* const* d_y,
                          int tokens, int gather_mode, void* const* streams);
/* Host pointers, synchronous: x [tokens][n_in] in, full y out. */
int q35k_shard_matmul(q35k_shard* s, const q35k_sharded_weight* w, const float* x, float* y, int tokens,
                      int gather_mode);
/* Bound of the fused gather's wait for the peers' flags (default 2000 ms).
 * A rank that does not take part in a fused call makes the other ranks'
 * waits run out: their call reports Q35K_ETIMEOUT at q35k_shard_sync (the
 * reference's synchronous exceptions, Model/Qwen35Model.Decode.cs:18-85,
 * become a TimeoutException) instead of hanging. */
int q35k_shard_set_wait_limit(q35k_shard* s, int milliseconds);
/* Collective: after a Q35K_ETIMEOUT, every rank of the group calls this
 * before its next call.  It waits for the rank's kernels, clears its error
 * state and the fused gather's flags and call counters, and (one process per
 * GPU) returns once every rank has done so. */
int q35k_shard_reset(q35k_shard* s);
/* Diagnostics of the fused gather: with tracing on, each fused call records
 * on every local device the %globaltimer (ns) of six phases -- GEMV first
 * CTA start, GEMV last CTA end, gather kernel start, every peer value of the
 * call arrived, the GEMV's completion seen by the gather kernel, gather
 * kernel end -- which q35k_shard_trace copies out for local device `local`
 * (after the call; it synchronizes that device). */
int q35k_shard_set_trace(q35k_shard* s, int on);
int q35k_shard_trace(q35k_shard* s, int local, uint64_t* out6);

/* ---- Allocation-free decode matmul --------------------------------------
 *
 * No counterpart in the reference.  For callers that must not have a library
 * allocate device memory during a call: a host whose device memory is all
 * handed out by its own arena, or a latency-critical decode loop in which a
 * cudaMalloc/cudaFree (which synchronize the device) would stall the
 * pipeline.  q35k_matmul_dev grows its context's scratch with cudaMalloc on
 * demand; this entry point instead keeps all of its scratch in one fixed
 * array of Q35K_STATIC_SCRATCH_BYTES that every GPU loading libq35k holds
 * until the process exits, and allocates nothing.
 *
 * Same result as q35k_matmul_dev for tokens <= Q35K_STATIC_MAX_TOKENS:
 * d_y[tokens][n_out] = d_x[tokens][n_in] @ W^T, asynchronous on `stream` (a
 * cudaStream_t; NULL = the legacy default stream).  The weight's device must
 * be the current device.  Shapes whose scratch would not fit the array, or
 * more tokens, return Q35K_EINVAL; q35k_last_error(NULL) says why.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture.
 *   - All calls share the array and it keeps the previous call's contents:
 *     each call clears the counters it relies on before its kernels run, and
 *     calls that overlap on the GPU (other streams, other host threads) race
 *     on the array -- do not issue them.
 *   - A bounded device wait that expires inside this call's kernels is not
 *     reported (use q35k_matmul_dev + q35k_sync to observe those).
 *   - The resolved address belongs to the device's primary context: do not
 *     reset it (cudaDeviceReset, or a library that resets the primary
 *     context) between calls, or later calls would write through a stale
 *     address. */
#define Q35K_STATIC_MAX_TOKENS 8
#define Q35K_STATIC_SCRATCH_BYTES (8u << 20)
int q35k_matmul_static_dev(const q35k_weight* w, const float* d_x, float* d_y, int tokens, void* stream);

/* ---- GGUF ingestion ------------------------------------------------------ */

/* A GGUF v2/v3 file, memory-mapped read-only with its metadata and tensor
 * table parsed at open: Qwen35Sharp.Gguf/GgufFile.cs (constructor :27-60,
 * Parse :110-172).  Malformed or truncated files give Q35K_EDATA (the
 * reference's InvalidDataException / EndOfStreamException), versions other
 * than 2 and 3 Q35K_ENOTSUP, a file that cannot be opened Q35K_EIO; the
 * message is in q35k_last_error(NULL).  Host only: no GPU is needed. */
typedef struct q35k_gguf q35k_gguf;
int q35k_gguf_open(const char* path, q35k_gguf** out);
int q35k_gguf_close(q35k_gguf* g);
/* Version, tensor count, general.alignment (default 32) and the file offset
 * of the aligned data section (GgufFile.DataBase). */
int q35k_gguf_info(const q35k_gguf* g, int* version, int* n_tensors, uint32_t* alignment, uint64_t* data_offset);
/* Index of the tensor `name` (the last one of that name), or -1. */
int q35k_gguf_find(const q35k_gguf* g, const char* name);
/* Tensor `index` in file order: name (valid until close), ggml type, dim
 * count and dims (GGUF order, dim 0 innermost; unused dims reported as 1),
 * offset from the data section (GgufTensorInfo, GgufTensorInfo.cs). */
int q35k_gguf_tensor(const q35k_gguf* g, int index, const char** name, int* type, int* n_dims, int64_t* dims4,
                     uint64_t* offset);
/* Host pointer to `bytes` bytes of tensor `index` in the mapping
 * (Q35K_EDATA if they run past the end of the file). */
int q35k_gguf_tensor_data(const q35k_gguf* g, int index, size_t bytes, const void** data);
/* Metadata scalars (GgufFile.GetInt32/GetUint32/GetFloat32/GetString,
 * GgufFile.cs:62-99): integers of any width (bool is not an integer), floats
 * (integers coerced), strings (valid until close); arrays report their
 * element type and length.  Q35K_EINVAL when the key is missing or of
 * another kind. */
int q35k_gguf_get_int(const q35k_gguf* g, const char* key, int64_t* value);
int q35k_gguf_get_float(const q35k_gguf* g, const char* key, double* value);
int q35k_gguf_get_string(const q35k_gguf* g, const char* key, const char** value);
int q35k_gguf_get_array(const q35k_gguf* g, const char* key, int* elem_type, uint64_t* count);
/* Upload the Q4_K/Q5_K/Q6_K tensor `name` straight from the mapping, as
 * LoadWeights does for each quantized tensor (Model/Qwen35Model.cs:463-565):
 * nIn = dims[0], nOut = dims[1]; a stack of matrices (experts) or nIn not a
 * multiple of 256 gives Q35K_ENOTSUP, another type Q35K_ENOTSUP. */
int q35k_weight_upload_gguf(q35k_ctx* ctx, const q35k_gguf* g, const char* name, q35k_weight** out);

#ifdef __cplusplus
}
#endif
#endif
