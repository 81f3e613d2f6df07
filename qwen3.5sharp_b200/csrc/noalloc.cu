// noalloc.cu -- q35k_matmul_static_dev: the decode matmul without any device
// allocation.
//
// The regular entry points keep their scratch (split-K partial sums, arrival
// counters, planar Q8_K activations) in context buffers that grow with
// cudaMalloc on demand.  Some callers cannot allow that on their hot path:
// a host that hands all device memory to its own arena and never lets a
// library allocate, or a latency-critical decode loop where cudaMalloc /
// cudaFree would synchronize the device and stall it.  This entry point runs
// the same kernels with its scratch in one fixed-size, file-scope device
// array instead.  The caller still provides the (already uploaded) weight,
// the input x and the output y.
//
// Rules, stated where a caller sees them (include/q35k.h):
//   * The array holds NOALLOC_SCRATCH_BYTES on every GPU that loads this
//     library, from load until the process exits.
//   * Host code cannot use the array's name as a device address: on its first
//     call on a device (with that device current) the entry point resolves
//     the address once with cudaGetSymbolAddress and caches it.  Make that
//     first call before any stream capture.
//   * All calls share the one array and it keeps the previous call's
//     contents: each call clears the arrival counters it uses before its
//     kernels run.  Calls that overlap on the GPU (two streams, or two host
//     threads) race on the array and must not be issued.
//   * The cached address belongs to the device's primary context: a
//     cudaDeviceReset (or another library resetting the primary context)
//     between calls leaves it dangling, so the context must not be reset
//     while this entry point is in use.
#include "../../include/q35k.h"
#include "api_internal.h"
#include "device_common.cuh"
#include "kernels.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

namespace q35k {

constexpr size_t NOALLOC_SCRATCH_BYTES = Q35K_STATIC_SCRATCH_BYTES;  // 8 MiB per device
constexpr int NOALLOC_MAX_DEVICES = 64;

// The scratch: [error word | counters | partial sums | planar Q8_K].
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

static void* g_scratch_addr[NOALLOC_MAX_DEVICES];
static std::mutex g_scratch_mu;

void set_thread_error(const std::string& msg);  // api.cu

// Device address of the scratch array on the current device (resolved once).
static int scratch_address(int device, unsigned char** out) {
    if (device < 0 || device >= NOALLOC_MAX_DEVICES) {
        set_thread_error("q35k_matmul_static_dev: device index out of range");
        return Q35K_EINVAL;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            set_thread_error(std::string("q35k_matmul_static_dev: cudaGetSymbolAddress failed: ") +
                             cudaGetErrorString(e));
            return Q35K_ECUDA;
        }
        g_scratch_addr[device] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[device]);
    return Q35K_OK;
}

}  // namespace q35k

using namespace q35k;

extern "C" int q35k_matmul_static_dev(const q35k_weight* w, const float* d_x, float* d_y, int tokens,
                                      void* stream) {
    if (!w || !d_x || !d_y) {
        set_thread_error("q35k_matmul_static_dev: NULL weight, input or output");
        return Q35K_EINVAL;
    }
    if (tokens < 1 || tokens > Q35K_STATIC_MAX_TOKENS) {
        set_thread_error("q35k_matmul_static_dev: tokens must be 1.." + std::to_string(Q35K_STATIC_MAX_TOKENS));
        return Q35K_EINVAL;
    }
    if ((uintptr_t)d_x % 16 || (uintptr_t)d_y % 4) {
        set_thread_error("q35k_matmul_static_dev: x must be 16-byte and y 4-byte aligned");
        return Q35K_EINVAL;
    }
    int cur = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e != cudaSuccess || cur != w->device) {
        set_thread_error("q35k_matmul_static_dev: the weight's device must be the current device");
        return Q35K_EINVAL;
    }
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cur)) != cudaSuccess) {
        set_thread_error(std::string("q35k_matmul_static_dev: ") + cudaGetErrorString(e));
        return Q35K_ECUDA;
    }
    const GemvPlan p = plan_gemv(w->type, w->nb, w->n_out, tokens, sms);
    const bool fused = gemv_fuses_quantize(w->type, w->nb, w->n_out, tokens, sms);

    // Carve the scratch: error word, counters, partial sums, planar Q8_K.
    if (!p.fits) {
        set_thread_error("q35k_matmul_static_dev: the decode GEMV has no shared-memory plan for this shape");
        return Q35K_ENOTSUP;
    }
    // The kernel indexes the split-K partial sums as [groups][splits][tokens][32]
    // floats (the context path sizes them for 8 tokens, as it reuses them).
    const size_t err_bytes = 256;
    const size_t cnt_bytes = (p.counters * sizeof(int) + 255) / 256 * 256;
    const size_t part_raw = p.splits > 1 ? (size_t)p.groups * p.splits * tokens * 32 * sizeof(float) : 0;
    const size_t part_bytes = (part_raw + 255) / 256 * 256;
    const size_t q8_bytes = fused ? 0 : (q8_planar(tokens, w->nb).bytes + 255) / 256 * 256;
    const size_t need = err_bytes + cnt_bytes + part_bytes + q8_bytes;
    if (need > NOALLOC_SCRATCH_BYTES) {
        char buf[256];
        snprintf(buf, sizeof buf,
                 "q35k_matmul_static_dev: this shape needs %zu bytes of scratch; the static array holds %zu "
                 "(use q35k_matmul_dev)",
                 need, NOALLOC_SCRATCH_BYTES);
        set_thread_error(buf);
        return Q35K_EINVAL;
    }
    unsigned char* base = nullptr;
    int rc = scratch_address(cur, &base);
    if (rc != Q35K_OK) return rc;
    unsigned* d_err = reinterpret_cast<unsigned*>(base);
    int* counters = reinterpret_cast<int*>(base + err_bytes);
    float* partial = reinterpret_cast<float*>(base + err_bytes + cnt_bytes);
    uint8_t* q8 = base + err_bytes + cnt_bytes + part_bytes;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The array keeps the last call's contents: clear what must start at zero.
    e = cudaMemsetAsync(base, 0, err_bytes + cnt_bytes, s);
    if (e == cudaSuccess && !fused)
        e = launch_quantize_q8k(d_x, q8, w->n_in, tokens, tokens, s, nullptr, q8_interleave_min_rows(w->type));
    if (e == cudaSuccess) {
        GemvArgs a{};
        a.tiles = w->tiles;
        if (fused) {
            a.x = d_x;
            a.ldx = w->n_in;
        } else {
            a.q8 = q8;
        }
        a.y = d_y;
        a.ldy = w->n_out;
        a.n_out = w->n_out;
        a.nb = w->nb;
        a.tokens = tokens;
        a.partial = partial;
        a.counters = counters;
        a.err = d_err;
        a.num_sms = sms;
        e = launch_gemv(w->type, a, s, /*pdl=*/!fused);
    }
    if (e != cudaSuccess) {
        set_thread_error(std::string("q35k_matmul_static_dev: launch failed: ") + cudaGetErrorString(e));
        return Q35K_ECUDA;
    }
    return Q35K_OK;
}
