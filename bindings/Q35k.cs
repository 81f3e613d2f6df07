// Q35k.cs -- P/Invoke binding of libq35k (include/q35k.h) for the Qwen35Sharp
// kernels project.  Drop this file into src/Qwen35Sharp.Kernels/ (namespace
// Flygon.Kernels, AllowUnsafeBlocks as the project already sets) and put
// libq35k.so on the native loader path.  Every C entry point of the header
// has one declaration here with the same argument order; handles are nint,
// device pointers and CUDA streams are nint as well, host buffers are the
// pointer types the reference kernels already take (BlockQ8K*, float*).
//
// Status codes map to the exceptions the replaced C# kernels throw
// (Q35k.Check / CheckShard); the entry points that replace a reference
// kernel are named in the comments, with the reference file and lines.
using System.Runtime.InteropServices;

namespace Flygon.Kernels;

public static unsafe partial class Q35k
{
    const string Lib = "q35k";

    public const int Ok = 0, EInval = 1, ENotSup = 2, ENoMem = 3, ECuda = 4, ETimeout = 5, ENccl = 6, EData = 7, EIo = 8;
    public const int TypeQ4K = 12, TypeQ5K = 13, TypeQ6K = 14;
    public const int GemmExact = 0, GemmFast = 1;
    public const int GatherNccl = 0, GatherPeer = 1, GatherFused = 2;
    public const int MaxShared = 4, NcclIdBytes = 128, StaticMaxTokens = 8;

    // ---- Context (CpuThreadPool + ScratchArena, Kernels/CpuThreadPool.cs:25-44) ----
    [LibraryImport(Lib)] public static partial int q35k_create(int device, out nint ctx);
    [LibraryImport(Lib)] public static partial int q35k_destroy(nint ctx);
    [LibraryImport(Lib)] public static partial nint q35k_last_error(nint ctx);
    [LibraryImport(Lib)] public static partial nint q35k_version();
    [LibraryImport(Lib)] public static partial int q35k_sync(nint ctx);

    // ---- Weights (LoadWeights, Model/Qwen35Model.cs:463-565) ----
    [LibraryImport(Lib)] public static partial int q35k_weight_upload(nint ctx, int ggmlType, void* blocks, int nIn, int nOut,
                                                                       out nint weight);
    [LibraryImport(Lib)] public static partial int q35k_weight_free(nint ctx, nint weight);
    [LibraryImport(Lib)] public static partial int q35k_weight_info(nint weight, out int ggmlType, out int nIn, out int nOut,
                                                                     out nuint deviceBytes);

    // ---- Matmul: Linear / DecodeLinear (Model/Qwen35Model.Decode.cs:22-87) ->
    //      MulMatQ4K.Gemv/Gemm, Q5K.Gemv/Gemm, Q6K.Gemv/Gemm ----
    [LibraryImport(Lib)] public static partial int q35k_matmul(nint ctx, nint w, float* x, float* y, int tokens);
    // GemvPrequant (Model/Qwen35Model.Decode.cs:89-112)
    [LibraryImport(Lib)] public static partial int q35k_matmul_q8k(nint ctx, nint w, BlockQ8K* x, float* y, int tokens);
    // Persistent NativeBuffer inputs/outputs used in place by the calls above.
    [LibraryImport(Lib)] public static partial int q35k_host_register(nint ctx, void* ptr, nuint bytes);
    [LibraryImport(Lib)] public static partial int q35k_host_unregister(nint ctx, void* ptr);
    [LibraryImport(Lib)] public static partial int q35k_matmul_dev(nint ctx, nint w, nint dX, nint dY, int tokens, nint stream);
    [LibraryImport(Lib)] public static partial int q35k_matmul_q8k_dev(nint ctx, nint w, nint dQ8k, nint dY, int tokens,
                                                                        nint stream);
    // Vocab head + ArgMax (Qwen35Sharp.Cli/Program.cs:127-140)
    [LibraryImport(Lib)] public static partial int q35k_matmul_argmax(nint ctx, nint w, float* x, int* idx, int tokens);
    [LibraryImport(Lib)] public static partial int q35k_matmul_argmax_dev(nint ctx, nint w, nint dX, nint dY, nint dIdx,
                                                                           int tokens, nint stream);
    // One quantized input, several weights (DecodeGateUp / DecodeAttention,
    // Model/Qwen35Model.Decode.cs:254-292; MulMatPanel.QuantizeAndGemm)
    [LibraryImport(Lib)] public static partial int q35k_matmul_shared(nint ctx, nint* ws, int count, float* x, float** ys,
                                                                       int tokens);
    [LibraryImport(Lib)] public static partial int q35k_matmul_shared_dev(nint ctx, nint* ws, int count, nint dX, nint* dYs,
                                                                           int tokens, nint stream);
    // ffn_down on SiLU(gate) * up (Ops.SiLUMul + DecodeLinear; MulMatPanel.SiluQuantizeAndGemm)
    [LibraryImport(Lib)] public static partial int q35k_matmul_silu(nint ctx, nint w, float* gate, float* up, float* y,
                                                                     int tokens);
    [LibraryImport(Lib)] public static partial int q35k_matmul_silu_dev(nint ctx, nint w, nint dGate, nint dUp, nint dY,
                                                                         int tokens, nint stream);
    [LibraryImport(Lib)] public static partial int q35k_set_gemm_mode(nint ctx, int mode);

    // ---- Utilities: Q8K.QuantizeRow (Kernels/Q8K.cs:12-77), *.DequantizeRow ----
    [LibraryImport(Lib)] public static partial int q35k_quantize_q8k(nint ctx, float* x, BlockQ8K* q8, int k, int rows);
    [LibraryImport(Lib)] public static partial int q35k_quantize_q8k_dev(nint ctx, nint dX, nint dQ8k, int k, int rows,
                                                                          nint stream);
    [LibraryImport(Lib)] public static partial int q35k_quantize_q8k_silu(nint ctx, float* gate, float* up, BlockQ8K* q8,
                                                                           int k, int rows);
    [LibraryImport(Lib)] public static partial int q35k_quantize_q8k_silu_dev(nint ctx, nint dGate, nint dUp, nint dQ8k,
                                                                               int k, int rows, nint stream);
    [LibraryImport(Lib)] public static partial int q35k_dequantize(nint ctx, int ggmlType, void* blocks, float* y, int k,
                                                                    int rows);
    [LibraryImport(Lib)] public static partial int q35k_dequantize_dev(nint ctx, int ggmlType, nint dBlocks, nint dY, int k,
                                                                        int rows, nint stream);

    // ---- Row-sharded matmul over the GPUs of one node (the CpuThreadPool row
    //      split of Kernels/MulMatQ4K.cs:31-36, over GPUs) ----
    [LibraryImport(Lib)] public static partial int q35k_shard_create(int ndev, int* devices, out nint shard);
    [LibraryImport(Lib)] public static partial int q35k_nccl_unique_id(byte* id128);
    [LibraryImport(Lib)] public static partial int q35k_shard_create_rank(int nranks, int rank, byte* id128, int device,
                                                                           out nint shard);
    [LibraryImport(Lib)] public static partial int q35k_shard_destroy(nint shard);
    [LibraryImport(Lib)] public static partial nint q35k_shard_last_error(nint shard);
    [LibraryImport(Lib)] public static partial int q35k_shard_info(nint shard, out int nranks, out int firstRank,
                                                                    out int localDevices);
    [LibraryImport(Lib)] public static partial int q35k_shard_sync(nint shard);
    [LibraryImport(Lib)] public static partial int q35k_shard_weight_upload(nint shard, int ggmlType, void* blocks, int nIn,
                                                                             int nOut, out nint weight);
    [LibraryImport(Lib)] public static partial int q35k_shard_weight_free(nint shard, nint weight);
    [LibraryImport(Lib)] public static partial int q35k_shard_matmul_dev(nint shard, nint w, nint* dX, nint* dY, int tokens,
                                                                          int gatherMode, nint* streams);
    [LibraryImport(Lib)] public static partial int q35k_shard_matmul(nint shard, nint w, float* x, float* y, int tokens,
                                                                      int gatherMode);
    [LibraryImport(Lib)] public static partial int q35k_shard_set_wait_limit(nint shard, int milliseconds);
    [LibraryImport(Lib)] public static partial int q35k_shard_reset(nint shard);
    [LibraryImport(Lib)] public static partial int q35k_shard_set_trace(nint shard, int on);
    [LibraryImport(Lib)] public static partial int q35k_shard_trace(nint shard, int local, ulong* out6);

    // ---- Decode matmul that allocates no device memory ----
    [LibraryImport(Lib)] public static partial int q35k_matmul_static_dev(nint w, nint dX, nint dY, int tokens, nint stream);

    // ---- GGUF ingestion (Qwen35Sharp.Gguf/GgufFile.cs:27-172) ----
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_open(string path, out nint gguf);
    [LibraryImport(Lib)] public static partial int q35k_gguf_close(nint gguf);
    [LibraryImport(Lib)] public static partial int q35k_gguf_info(nint gguf, out int version, out int nTensors,
                                                                   out uint alignment, out ulong dataOffset);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_find(nint gguf, string name);
    [LibraryImport(Lib)] public static partial int q35k_gguf_tensor(nint gguf, int index, out nint name, out int type,
                                                                     out int nDims, long* dims4, out ulong offset);
    [LibraryImport(Lib)] public static partial int q35k_gguf_tensor_data(nint gguf, int index, nuint bytes, out nint data);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_get_int(nint gguf, string key, out long value);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_get_float(nint gguf, string key, out double value);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_get_string(nint gguf, string key, out nint value);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_gguf_get_array(nint gguf, string key, out int elemType, out ulong count);
    [LibraryImport(Lib, StringMarshalling = StringMarshalling.Utf8)]
    public static partial int q35k_weight_upload_gguf(nint ctx, nint gguf, string name, out nint weight);

    /// Throws the exception the replaced C# kernel would have thrown for a
    /// non-zero status of a context call (ctx == 0: calls without a context).
    public static void Check(nint ctx, int status)
    {
        if (status != Ok) throw ToException(status, Marshal.PtrToStringUTF8(q35k_last_error(ctx)));
    }

    /// The same for the row-sharded calls.
    public static void CheckShard(nint shard, int status)
    {
        if (status != Ok) throw ToException(status, Marshal.PtrToStringUTF8(q35k_shard_last_error(shard)));
    }

    static Exception ToException(int status, string? msg)
    {
        msg ??= "q35k error " + status;
        return status switch
        {
            EInval => new ArgumentException(msg),
            ENotSup => new NotSupportedException(msg),
            ENoMem => new InsufficientMemoryException(msg),
            ETimeout => new TimeoutException(msg),       // a bounded device wait expired
            EData => new InvalidDataException(msg),      // malformed or truncated GGUF
            EIo => new IOException(msg),                 // GGUF file cannot be opened or mapped
            _ => new InvalidOperationException(msg),     // ECuda, ENccl
        };
    }
}
