// api.cu -- the C ABI of libq35k (include/q35k.h): contexts, weight upload,
// matmul dispatch, utilities.  All compute runs in the CUDA kernels of this
// library; there is no CPU fallback.
#include "../../include/q35k.h"
#include "device_common.cuh"
#include "gemm_tc.h"
#include "kernels.h"
#include "api_internal.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

using namespace q35k;

namespace q35k {
void configure_gemv_kernels();
}

int q35k_ctx::fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    err = buf;
    return code;
}

int q35k_ctx::cuda_fail(cudaError_t e, const char* what) {
    return fail(Q35K_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int q35k_ctx::ensure_dev(void** p, size_t* cap, size_t bytes, bool zero) {
    if (bytes <= *cap) return Q35K_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t want = std::max(bytes, (size_t)256);
    cudaError_t e = cudaMalloc(p, want);
    if (e != cudaSuccess) {
        *p = nullptr;
        cudaGetLastError();
        return fail(Q35K_ENOMEM, "cudaMalloc(%zu) failed: %s", want, cudaGetErrorString(e));
    }
    if (zero) {
        e = cudaMemset(*p, 0, want);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset");
    }
    *cap = want;
    return Q35K_OK;
}

int q35k_ctx::ensure_host(void** p, size_t* cap, size_t bytes) {
    if (bytes <= *cap) return Q35K_OK;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    if (p == &h_out) h_out_dev = nullptr;
    size_t want = std::max(bytes, (size_t)4096);
    cudaError_t e = cudaMallocHost(p, want);
    if (e != cudaSuccess) {
        *p = nullptr;
        cudaGetLastError();
        return fail(Q35K_ENOMEM, "cudaMallocHost(%zu) failed: %s", want, cudaGetErrorString(e));
    }
    *cap = want;
    if (p == &h_out && (cudaHostGetDevicePointer(&h_out_dev, h_out, 0) != cudaSuccess || !h_out_dev)) {
        cudaGetLastError();
        h_out_dev = nullptr;
    }
    return Q35K_OK;
}

int q35k_ctx::check_device_error() {
    // A pinned destination: one direct DMA instead of a staged pageable copy.
    cudaError_t e = cudaMemcpyAsync(h_errw, d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    const unsigned word = *reinterpret_cast<volatile unsigned*>(h_errw);
    if (word) return on_device_error(word);
    return Q35K_OK;
}

int q35k_ctx::on_device_error(unsigned word) {
    // Reset the error word and the split-K arrival counters (a CTA that gave
    // up may have left a counter non-zero).
    cudaMemset(d_err, 0, sizeof(unsigned));
    if (d_counters) cudaMemset(d_counters, 0, counters_cap);
    if (d_gcnt) cudaMemset(d_gcnt, 0, gcnt_cap);
    cudaDeviceSynchronize();
    return fail(Q35K_ETIMEOUT, "a bounded device wait expired inside a kernel (error word 0x%x)", word);
}

static bool valid_type(int t) { return t == Q35K_TYPE_Q4_K || t == Q35K_TYPE_Q5_K || t == Q35K_TYPE_Q6_K; }

static thread_local std::string g_create_error;

namespace q35k {
// Errors of calls that have no context: reported by q35k_last_error(NULL).
void set_thread_error(const std::string& msg) { g_create_error = msg; }
}  // namespace q35k

extern "C" {

const char* q35k_version(void) { return "q35k 0.1 (sm_100a)"; }

int q35k_create(int device, q35k_ctx** out) {
    if (!out) return Q35K_EINVAL;
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        g_create_error = "no CUDA device is visible (libq35k has no CPU fallback)";
        cudaGetLastError();
        return Q35K_ECUDA;
    }
    if (device < 0 || device >= count) {
        g_create_error = "device index out of range";
        return Q35K_EINVAL;
    }
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) {
        g_create_error = cudaGetErrorString(e);
        return Q35K_ECUDA;
    }
    if (prop.major != 10) {
        g_create_error = "libq35k is built for sm_100a (B200); device is sm_" + std::to_string(prop.major) +
                         std::to_string(prop.minor);
        return Q35K_ENOTSUP;
    }
    if ((e = cudaSetDevice(device)) != cudaSuccess) {
        g_create_error = cudaGetErrorString(e);
        return Q35K_ECUDA;
    }
    q35k_ctx* c = new (std::nothrow) q35k_ctx();
    if (!c) return Q35K_ENOMEM;
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaMalloc(&c->d_err, sizeof(unsigned))) != cudaSuccess ||
        (e = cudaMemset(c->d_err, 0, sizeof(unsigned))) != cudaSuccess ||
        (e = cudaHostAlloc(reinterpret_cast<void**>(&c->h_errw), 64, cudaHostAllocDefault)) != cudaSuccess) {
        g_create_error = cudaGetErrorString(e);
        delete c;
        return Q35K_ECUDA;
    }
    configure_gemv_kernels();
    if ((e = configure_tc_gemm()) != cudaSuccess) {
        g_create_error = std::string("GEMM configuration: ") + cudaGetErrorString(e);
        delete c;
        return Q35K_ECUDA;
    }
    if (const char* v = getenv("Q35K_GEMM_MIN_TOKENS")) c->gemm_min_tokens = std::max(1, atoi(v));
    if (const char* v = getenv("Q35K_GEMM_MODE")) c->gemm_mode = (strcmp(v, "fast") == 0) ? Q35K_GEMM_FAST : Q35K_GEMM_EXACT;
    if ((e = cudaGetLastError()) != cudaSuccess) {
        g_create_error = std::string("kernel configuration: ") + cudaGetErrorString(e);
        delete c;
        return Q35K_ECUDA;
    }
    *out = c;
    return Q35K_OK;
}

int q35k_destroy(q35k_ctx* c) {
    if (!c) return Q35K_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    delete c;
    return Q35K_OK;
}

const char* q35k_last_error(const q35k_ctx* c) {
    if (!c) return g_create_error.c_str();
    return c->err.c_str();
}

int q35k_set_gemm_mode(q35k_ctx* c, int mode) {
    if (!c) return Q35K_EINVAL;
    if (mode != Q35K_GEMM_EXACT && mode != Q35K_GEMM_FAST) return c->fail(Q35K_EINVAL, "unknown GEMM mode %d", mode);
    c->gemm_mode = mode;
    return Q35K_OK;
}

int q35k_sync(q35k_ctx* c) {
    if (!c) return Q35K_EINVAL;
    cudaSetDevice(c->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return c->cuda_fail(e, "cudaDeviceSynchronize");
    return c->check_device_error();
}

int q35k_weight_upload(q35k_ctx* c, int type, const void* blocks, int n_in, int n_out, q35k_weight** out) {
    if (!c || !out) return Q35K_EINVAL;
    *out = nullptr;
    if (!valid_type(type)) return c->fail(Q35K_ENOTSUP, "ggml type %d is not a K-quant weight (12, 13, 14)", type);
    if (!blocks) return c->fail(Q35K_EINVAL, "blocks is NULL");
    if (n_in <= 0 || n_in % QK != 0) return c->fail(Q35K_ENOTSUP, "nIn=%d is not a multiple of 256", n_in);
    if (n_out <= 0) return c->fail(Q35K_EINVAL, "nOut must be positive");
    cudaSetDevice(c->device);
    const int nb = n_in / QK, bb = block_bytes(type);
    const int n_pad = (n_out + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS;
    const size_t raw_bytes = (size_t)n_out * nb * bb;
    const size_t tile_bytes = (size_t)n_pad * nb * bb;
    q35k_weight* w = new (std::nothrow) q35k_weight();
    if (!w) return Q35K_ENOMEM;
    w->type = type;
    w->n_in = n_in;
    w->n_out = n_out;
    w->nb = nb;
    w->n_pad = n_pad;
    w->device = c->device;
    w->bytes = tile_bytes;
    uint8_t* raw = nullptr;
    cudaError_t e = cudaMalloc(&w->tiles, tile_bytes);
    // The staged GGUF rows, then a word the metadata kernel flags non-finite block scales in.
    const size_t flag_off = (raw_bytes + 15) / 16 * 16;
    if (e == cudaSuccess) e = cudaMalloc(&raw, flag_off + 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (w->tiles) cudaFree(w->tiles);
        delete w;
        return c->fail(Q35K_ENOMEM, "weight upload: cudaMalloc(%zu) failed", tile_bytes + raw_bytes);
    }
    {
        // The prefill GEMM's per-block metadata, computed once here.
        const size_t mb = gemm_meta_bytes(type, nb, n_pad), sb = gemm_scale_bytes(type, nb, n_pad);
        if ((e = cudaMalloc(&w->meta, mb + sb)) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(w->tiles);
            cudaFree(raw);
            delete w;
            return c->fail(Q35K_ENOMEM, "weight upload: cudaMalloc(%zu) failed", mb + sb);
        }
        w->scale = sb ? reinterpret_cast<float*>(w->meta + mb) : nullptr;
        w->bytes += mb + sb;
    }
    e = cudaMemcpyAsync(raw, blocks, raw_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_repack_tiles(type, raw, w->tiles, nb, n_out, n_pad, c->stream);
    unsigned* d_unsafe = reinterpret_cast<unsigned*>(raw + flag_off);
    unsigned unsafe = 0;
    if (e == cudaSuccess) e = cudaMemsetAsync(d_unsafe, 0, sizeof(unsigned), c->stream);
    if (e == cudaSuccess)
        e = launch_gemm_meta(type, w->tiles, w->meta, w->scale, nb, n_pad, d_unsafe, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&unsafe, d_unsafe, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    w->fast_ok = unsafe == 0;
    cudaFree(raw);
    if (e != cudaSuccess) {
        cudaFree(w->tiles);
        if (w->meta) cudaFree(w->meta);
        delete w;
        return c->cuda_fail(e, "weight upload");
    }
    *out = w;
    return Q35K_OK;
}

int q35k_weight_free(q35k_ctx* c, q35k_weight* w) {
    if (!w) return Q35K_OK;
    if (c) cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    cudaFree(w->tiles);
    if (w->meta) cudaFree(w->meta);
    delete w;
    return Q35K_OK;
}

int q35k_weight_info(const q35k_weight* w, int* type, int* n_in, int* n_out, size_t* device_bytes) {
    if (!w) return Q35K_EINVAL;
    if (type) *type = w->type;
    if (n_in) *n_in = w->n_in;
    if (n_out) *n_out = w->n_out;
    if (device_bytes) *device_bytes = w->bytes;
    return Q35K_OK;
}

}  // extern "C"

// Tokens per GEMV launch for this weight (0: rows too long for the GEMV).
static int gemv_chunk(const q35k_weight* w) { return gemv_max_tokens(w->nb); }

// Launch the GEMV for `tokens` rows of planar Q8_K (in chunks of
// gemv_chunk(w) rows) already on the device.
int q35k_ctx::gemv(const q35k_weight* w, const uint8_t* d_q8, float* d_y, int tokens, cudaStream_t s, bool pdl,
                   const float* d_x, int ldy, const q35k::GemvPeers* peers, unsigned long long* argmax,
                   const float* d_up, const q35k_weight* const* more_w, float* const* more_y, int n_more) {
    if (ldy <= 0) ldy = w->n_out;
    const int chunk = gemv_chunk(w);
    if (chunk <= 0) return fail(Q35K_ENOTSUP, "nIn=%d is too long for the decode GEMV", w->n_in);
    if (n_more < 0 || n_more > GEMV_MAX_MATS - 1) return fail(Q35K_EINVAL, "too many weights for one GEMV launch");
    GemvMats more{};
    int groups = (w->n_out + TILE_ROWS - 1) / TILE_ROWS;
    for (int k = 0; k < n_more; k++) {
        const q35k_weight* m = more_w[k];
        if (m->type != w->type || m->nb != w->nb) return fail(Q35K_EINVAL, "weights of one GEMV launch differ in type or nIn");
        more.tiles[k] = m->tiles;
        more.n_out[k] = m->n_out;
        more.ldy[k] = m->n_out;
        more.g0[k] = groups;
        groups += (m->n_out + TILE_ROWS - 1) / TILE_ROWS;
    }
    more.n = n_more;
    GemvArgs probe{};
    probe.n_out = w->n_out;
    probe.more = more;
    const GemvPlan p = plan_gemv(w->type, w->nb, gemv_plan_rows(probe), chunk, num_sms);
    int rc;
    if ((rc = ensure_dev((void**)&d_partial, &partial_cap, p.partial_bytes, false)) != Q35K_OK) return rc;
    if ((rc = ensure_dev((void**)&d_counters, &counters_cap, p.counters * sizeof(int), true)) != Q35K_OK) return rc;
    const size_t chunk_stride = q8_planar(chunk, w->nb).bytes;
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        GemvArgs a{};
        a.tiles = w->tiles;
        if (d_x) {
            a.x = d_x + (size_t)t0 * w->n_in;
            a.ldx = w->n_in;
        } else {
            a.q8 = d_q8 + (size_t)(t0 / chunk) * chunk_stride;
        }
        a.y = d_y ? d_y + (size_t)t0 * ldy : nullptr;
        a.argmax = argmax ? argmax + t0 : nullptr;
        a.up = d_x && d_up ? d_up + (size_t)t0 * w->n_in : nullptr;
        a.more = more;
        for (int k = 0; k < n_more; k++) a.more.y[k] = more_y[k] + (size_t)t0 * more.ldy[k];
        a.ldy = ldy;
        a.n_out = w->n_out;
        a.nb = w->nb;
        a.tokens = std::min(chunk, tokens - t0);
        a.partial = d_partial;
        a.counters = d_counters;
        a.err = d_err;
        a.h_err = call_h_err;
        a.num_sms = num_sms;
        if (peers) a.peers = *peers;  // one launch: tokens <= chunk (checked by the caller)
        cudaError_t e = launch_gemv(w->type, a, s, pdl && t0 == 0);
        if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
    }
    return Q35K_OK;
}

bool q35k_ctx::uses_gemm(const q35k_weight* w, int tokens) const {
    return tokens >= gemm_min_tokens && tc_gemm_supports(w->type, gemm_fast(w));
}

// Fast-mode arithmetic for this weight: the mode is fast and its block
// scales are finite (else the exact form, or the GEMV).
bool q35k_ctx::gemm_fast(const q35k_weight* w) const { return gemm_mode == Q35K_GEMM_FAST && w->fast_ok; }

int q35k_ctx::gemm(const q35k_weight* w, const float* d_x, float* d_y, int tokens, cudaStream_t s, int ldy,
                   const float* d_up, bool prep) {
    if (ldy <= 0) ldy = w->n_out;
    const bool fast = gemm_fast(w);
    const TcGemmPlan p = plan_tc_gemm(w->nb, w->n_pad, tokens, num_sms, tc_gemm_tile_tokens(fast, tokens));
    int rc;
    if ((rc = ensure_dev(&d_xq, &xq_cap, p.xq_bytes, false)) != Q35K_OK) return rc;
    if ((rc = ensure_dev(&d_xe, &xe_cap, p.xe_bytes, false)) != Q35K_OK) return rc;
    if ((rc = ensure_dev((void**)&d_xd, &xd_cap, p.xd_bytes, false)) != Q35K_OK) return rc;
    if ((rc = ensure_dev((void**)&d_gws, &gws_cap, p.ws_bytes, false)) != Q35K_OK) return rc;
    if ((rc = ensure_dev((void**)&d_gcnt, &gcnt_cap, p.counters * sizeof(int), true)) != Q35K_OK) return rc;
    if (fast && (rc = ensure_dev((void**)&d_tmax, &tmax_cap, (size_t)p.m_pad * sizeof(unsigned), true)) != Q35K_OK)
        return rc;
    cudaError_t e;
    if (prep) {
        e = launch_gemm_prep(d_x, w->n_in, tokens, p.m_pad, d_xq, d_xe, d_xd, d_tmax, fast, s, d_up);
        if (e != cudaSuccess) return cuda_fail(e, "GEMM activation launch");
    }
    TcGemmArgs a{};
    a.tiles = w->tiles;
    a.meta = w->meta;
    a.scale = w->scale;
    a.xd = d_xd;
    a.y = d_y;
    a.ldy = ldy;
    a.ws = d_gws;
    a.counters = d_gcnt;
    a.err = d_err;
    a.n_out = w->n_out;
    a.n_pad = w->n_pad;
    a.tokens = tokens;
    a.m_pad = p.m_pad;
    a.nb = w->nb;
    a.tiles_t = p.tiles_t;
    a.grid = p.grid;
    a.units = p.units;
    a.tn = p.tn;
    a.type = w->type;
    e = launch_tc_gemm(a, d_xq, d_xe, w->n_in, fast, s, true);
    if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
    return Q35K_OK;
}

int q35k_ctx::matmul_into(const q35k_weight* w, const float* d_x, float* d_y, int ldy, int tokens, cudaStream_t s,
                          const q35k::GemvPeers* peers, unsigned long long* argmax, const float* d_up) {
    const int chunk = gemv_chunk(w);
    if (peers && (chunk <= 0 || tokens > chunk))
        return fail(Q35K_ENOTSUP, "the fused all-gather takes decode calls of at most %d tokens", chunk);
    // Prefill: the tensor-core GEMM (the fused gather and argmax are GEMV epilogues).
    if (!peers && !argmax && uses_gemm(w, tokens))
        return gemm(w, d_x, d_y, tokens, s, ldy, d_up);
    if (chunk <= 0) return fail(Q35K_ENOTSUP, "nIn=%d is too long for the decode GEMV", w->n_in);
    // Decode: the GEMV quantizes its own slices of x (one kernel per call).
    if (tokens <= chunk && gemv_fuses_quantize(w->type, w->nb, w->n_out, tokens, num_sms))
        return gemv(w, nullptr, d_y, tokens, s, true, d_x, ldy, peers, argmax, d_up);
    int rc;
    if ((rc = ensure_dev((void**)&d_q8, &q8_cap, q8_planar_total(tokens, w->nb, chunk), false)) != Q35K_OK) return rc;
    cudaError_t e = launch_quantize_q8k(d_x, d_q8, w->n_in, tokens, chunk, s, d_up, q8_interleave_min_rows(w->type));
    if (e != cudaSuccess) return cuda_fail(e, "Q8_K quantize launch");
    return gemv(w, d_q8, d_y, tokens, s, true, nullptr, ldy, peers, argmax);
}

// One input, several weights of one K.  Prefill GEMM weights share one
// activation preparation; the GEMV weights of each type run in one launch,
// quantizing their own slices of x (decode) or reading one shared planar
// Q8_K of x.
int q35k_ctx::matmul_shared(const q35k_weight* const* ws, int count, const float* d_x, float* const* d_ys, int tokens,
                            cudaStream_t s) {
    const q35k_weight* w0 = ws[0];
    const int chunk = gemv_chunk(w0);
    int prepped = -1;  // arithmetic of the prepared GEMM operands (0 exact, 1 fast), -1: none
    int quantized = 0;  // layout threshold of the planar Q8_K in d_q8 (q8_interleave_min_rows), 0: none
    int rc;
    for (int i = 0; i < count; i++) {
        const q35k_weight* w = ws[i];
        if (uses_gemm(w, tokens)) {
            const int f = gemm_fast(w) ? 1 : 0;
            if ((rc = gemm(w, d_x, d_ys[i], tokens, s, 0, nullptr, prepped != f)) != Q35K_OK) return rc;
            prepped = f;
        }
    }
    if (chunk <= 0) return fail(Q35K_ENOTSUP, "nIn=%d is too long for the decode GEMV", w0->n_in);
    static const int types[] = {Q35K_TYPE_Q4_K, Q35K_TYPE_Q5_K, Q35K_TYPE_Q6_K};
    for (int type : types) {
        const q35k_weight* lw[GEMV_MAX_MATS];
        float* ly[GEMV_MAX_MATS];
        int n = 0, rows = 0;
        for (int i = 0; i < count; i++) {
            const q35k_weight* w = ws[i];
            if (w->type != type || uses_gemm(w, tokens)) continue;
            lw[n] = w;
            ly[n++] = d_ys[i];
            rows += (w->n_out + TILE_ROWS - 1) / TILE_ROWS * TILE_ROWS;
        }
        if (n == 0) continue;
        if (tokens <= chunk && gemv_fuses_quantize(type, w0->nb, rows, tokens, num_sms)) {
            rc = gemv(lw[0], nullptr, ly[0], tokens, s, true, d_x, 0, nullptr, nullptr, nullptr, lw + 1, ly + 1, n - 1);
        } else {
            // One quantization serves every type with the same planar layout
            // (Q4_K and Q5_K; Q6_K interleaves from more tokens).
            const int ilv = q8_interleave_min_rows(type);
            if (quantized != ilv) {
                if ((rc = ensure_dev((void**)&d_q8, &q8_cap, q8_planar_total(tokens, w0->nb, chunk), false)) != Q35K_OK)
                    return rc;
                cudaError_t e = launch_quantize_q8k(d_x, d_q8, w0->n_in, tokens, chunk, s, nullptr, ilv);
                if (e != cudaSuccess) return cuda_fail(e, "Q8_K quantize launch");
                quantized = ilv;
            }
            rc = gemv(lw[0], d_q8, ly[0], tokens, s, true, nullptr, 0, nullptr, nullptr, nullptr, lw + 1, ly + 1, n - 1);
        }
        if (rc != Q35K_OK) return rc;
    }
    return Q35K_OK;
}

static int check_matmul_args(q35k_ctx* c, const q35k_weight* w, const void* x, const void* y, int tokens) {
    if (!c) return Q35K_EINVAL;
    if (!w) return c->fail(Q35K_EINVAL, "weight handle is NULL");
    if (!x || !y) return c->fail(Q35K_EINVAL, "input/output pointer is NULL");
    if (tokens <= 0) return c->fail(Q35K_EINVAL, "tokens must be positive");
    if (w->device != c->device) return c->fail(Q35K_EINVAL, "weight lives on device %d, context on %d", w->device, c->device);
    return Q35K_OK;
}

static cudaStream_t pick(q35k_ctx* c, void* stream) { return stream ? (cudaStream_t)stream : c->stream; }

// Page-locked host ranges registered with q35k_host_register (process-wide,
// as the registration is): base, length and device alias.
namespace {
struct HostRange {
    const char* base;
    size_t bytes;
    char* dev;
};
std::mutex g_ranges_mu;
std::vector<HostRange> g_ranges;
}  // namespace

// Device address of a caller's host buffer [p, p + bytes) when it is
// page-locked and mapped into the device's address space as one contiguous
// range (registered with q35k_host_register, or allocated pinned by the
// caller); nullptr for pageable memory.  Host-pointer calls then read x and
// write y in place instead of staging them through the context's buffers.
static void* host_alias(const void* p, size_t bytes) {
    if (!p || bytes == 0) return nullptr;
    const char* cp = static_cast<const char*>(p);
    {
        std::lock_guard<std::mutex> lock(g_ranges_mu);
        for (const HostRange& r : g_ranges)
            if (cp >= r.base && cp + bytes <= r.base + r.bytes) return r.dev + (cp - r.base);
    }
    cudaPointerAttributes a0, a1;
    if (cudaPointerGetAttributes(&a0, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a0.type != cudaMemoryTypeHost || !a0.devicePointer) return nullptr;
    if (cudaPointerGetAttributes(&a1, cp + bytes - 1) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a1.type != cudaMemoryTypeHost || static_cast<char*>(a1.devicePointer) != static_cast<char*>(a0.devicePointer) + (bytes - 1))
        return nullptr;
    return a0.devicePointer;
}

// x of a host-pointer decode call crosses the bus in this kernel (mapped host
// memory -> device) rather than by a copy-engine transfer: the GEMV launched
// after it with programmatic dependent launch starts streaming its weights
// while x is still in flight, and reads x only after this grid completed.
__global__ void q35k_stage_in_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t n) {
    asm volatile("griddepcontrol.launch_dependents;");
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if ((((uintptr_t)src | (uintptr_t)dst) & 15) == 0 && n % 4 == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        float4* d4 = reinterpret_cast<float4*>(dst);
        for (size_t i = i0; i < n / 4; i += stride) d4[i] = s4[i];
    } else {
        for (size_t i = i0; i < n; i += stride) dst[i] = src[i];
    }
}

// The device error word of a host-pointer call, read out into mapped host
// memory once the kernels before it have completed (no copy-engine transfer
// on the call's critical path).
__global__ void q35k_err_out_kernel(const unsigned* __restrict__ d_err, unsigned* h_err) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    *reinterpret_cast<volatile unsigned*>(h_err) = *reinterpret_cast<const volatile unsigned*>(d_err);
}

template <typename... P, typename... A>
static cudaError_t launch_k(void (*kernel)(P...), int grid, int block, cudaStream_t st, bool pdl, A... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);
}

// Inputs of at most this many bytes go through q35k_stage_in_kernel; larger
// ones (prefill) through the copy engines.
constexpr size_t STAGE_KERNEL_MAX_BYTES = 256 * 1024;

// Device buffers handed in by the caller: the quantizer reads x as float4,
// the GEMV reads Q8_K blocks and writes y as 32-bit words.
static int check_alignment(q35k_ctx* c, const void* x, size_t x_align, const void* y, size_t y_align) {
    if ((uintptr_t)x % x_align) return c->fail(Q35K_EINVAL, "input pointer must be %zu-byte aligned", x_align);
    if ((uintptr_t)y % y_align) return c->fail(Q35K_EINVAL, "output pointer must be %zu-byte aligned", y_align);
    return Q35K_OK;
}

extern "C" {

int q35k_matmul_q8k_dev(q35k_ctx* c, const q35k_weight* w, const void* d_q8k, float* d_y, int tokens, void* stream) {
    int rc = check_matmul_args(c, w, d_q8k, d_y, tokens);
    if (rc) return rc;
    if ((rc = check_alignment(c, d_q8k, 4, d_y, 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    cudaStream_t s = pick(c, stream);
    const int chunk = gemv_chunk(w);
    if (chunk <= 0) return c->fail(Q35K_ENOTSUP, "nIn=%d is too long for the decode GEMV", w->n_in);
    // The caller's BlockQ8K rows -> the GEMV's planar layout.
    if ((rc = c->ensure_dev((void**)&c->d_q8, &c->q8_cap, q8_planar_total(tokens, w->nb, chunk), false)) != Q35K_OK)
        return rc;
    cudaError_t e = launch_q8k_to_planar((const uint8_t*)d_q8k, c->d_q8, w->n_in, tokens, chunk, s,
                                         q8_interleave_min_rows(w->type));
    if (e != cudaSuccess) return c->cuda_fail(e, "Q8_K repack launch");
    return c->gemv(w, c->d_q8, d_y, tokens, s);
}

int q35k_matmul_dev(q35k_ctx* c, const q35k_weight* w, const float* d_x, float* d_y, int tokens, void* stream) {
    int rc = check_matmul_args(c, w, d_x, d_y, tokens);
    if (rc) return rc;
    if ((rc = check_alignment(c, d_x, 16, d_y, 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    return c->matmul_into(w, d_x, d_y, w->n_out, tokens, pick(c, stream));
}

int q35k_matmul(q35k_ctx* c, const q35k_weight* w, const float* x, float* y, int tokens) {
    int rc = check_matmul_args(c, w, x, y, tokens);
    if (rc) return rc;
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)tokens * w->n_in * sizeof(float);
    const size_t out_bytes = (size_t)tokens * w->n_out * sizeof(float);
    const bool gemm = c->uses_gemm(w, tokens);
    // Page-locked caller buffers (q35k_host_register) are used in place: x is
    // read straight from it and y written straight into it.  Pageable ones go
    // through the context's pinned staging buffers.
    const float* x_alias = static_cast<const float*>(host_alias(x, in_bytes));
    float* y_alias = static_cast<float*>(host_alias(y, out_bytes));
    if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, in_bytes, false)) != Q35K_OK) return rc;
    if (gemm && (rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return rc;
    if (!x_alias && (rc = c->ensure_host(&c->h_in, &c->h_in_cap, in_bytes)) != Q35K_OK) return rc;
    // Staging for y (pageable callers) and, after it, the mapped error word.
    const size_t stage_y = y_alias ? 0 : out_bytes;
    if ((rc = c->ensure_host(&c->h_out, &c->h_out_cap, stage_y + 64)) != Q35K_OK) return rc;
    volatile unsigned* h_err = reinterpret_cast<volatile unsigned*>(static_cast<char*>(c->h_out) + stage_y);
    *h_err = 0;
    char* const h_out_dev = static_cast<char*>(c->h_out_dev);
    if (!h_out_dev) return c->fail(Q35K_ECUDA, "the pinned staging buffer is not mapped into the device's address space");
    unsigned* const h_err_dev = reinterpret_cast<unsigned*>(h_out_dev + stage_y);
    if (!x_alias) {
        std::memcpy(c->h_in, x, in_bytes);
        void* dp = nullptr;
        if (cudaHostGetDevicePointer(&dp, c->h_in, 0) == cudaSuccess) x_alias = static_cast<const float*>(dp);
        cudaGetLastError();
    }
    cudaError_t e;
    if (x_alias && in_bytes <= STAGE_KERNEL_MAX_BYTES) {
        const size_t n = in_bytes / sizeof(float);
        const int grid = (int)std::min<size_t>((n / 4 + 255) / 256, 16);
        e = launch_k(q35k_stage_in_kernel, std::max(grid, 1), 256, c->stream, false, x_alias, c->d_x, n);
    } else {
        e = cudaMemcpyAsync(c->d_x, x_alias ? x : static_cast<const float*>(c->h_in), in_bytes,
                            cudaMemcpyHostToDevice, c->stream);
    }
    if (e != cudaSuccess) return c->cuda_fail(e, "H2D transfer of x");
    // Decode calls: the GEMV stores y over the bus straight into host memory
    // (the caller's page-locked y, or the mapped staging buffer), so the
    // transfer overlaps the kernel and no copy follows it.  Prefill calls
    // (tensor-core GEMM, whose tiles would cross the bus piece by piece) copy
    // y back afterwards.
    float* d_out = c->d_y;
    if (!gemm) d_out = y_alias ? y_alias : reinterpret_cast<float*>(h_out_dev);
    // Decode calls: the GEMV launches set the mapped error word themselves
    // when a wait expires; prefill calls read the device word out after the
    // GEMM and the copy of y.
    c->call_h_err = gemm ? nullptr : h_err_dev;
    rc = q35k_matmul_dev(c, w, c->d_x, d_out, tokens, c->stream);
    c->call_h_err = nullptr;
    if (rc != Q35K_OK) return rc;
    e = gemm ? cudaMemcpyAsync(y_alias ? y : c->h_out, c->d_y, out_bytes, cudaMemcpyDeviceToHost, c->stream)
             : cudaSuccess;
    if (e == cudaSuccess && gemm)
        e = launch_k(q35k_err_out_kernel, 1, 1, c->stream, false, (const unsigned*)c->d_err, h_err_dev);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "matmul");
    if (*h_err) return c->on_device_error(*h_err);
    if (!y_alias) std::memcpy(y, c->h_out, out_bytes);
    return Q35K_OK;
}

int q35k_host_register(q35k_ctx* c, void* p, size_t bytes) {
    if (!c) return Q35K_EINVAL;
    if (!p || bytes == 0) return c->fail(Q35K_EINVAL, "host_register: NULL pointer or zero size");
    cudaSetDevice(c->device);
    cudaError_t e = cudaHostRegister(p, bytes, cudaHostRegisterPortable | cudaHostRegisterMapped);
    if (e == cudaErrorHostMemoryAlreadyRegistered) {
        cudaGetLastError();
        return c->fail(Q35K_EINVAL, "host_register: the range is already page-locked");
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return c->fail(Q35K_ENOMEM, "host_register: cudaHostRegister(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
    void* dev = nullptr;
    if ((e = cudaHostGetDevicePointer(&dev, p, 0)) != cudaSuccess || !dev) {
        cudaGetLastError();
        cudaHostUnregister(p);
        return c->fail(Q35K_ECUDA, "host_register: no device address for the range: %s", cudaGetErrorString(e));
    }
    std::lock_guard<std::mutex> lock(g_ranges_mu);
    g_ranges.push_back(HostRange{static_cast<const char*>(p), bytes, static_cast<char*>(dev)});
    return Q35K_OK;
}

int q35k_host_unregister(q35k_ctx* c, void* p) {
    if (!c) return Q35K_EINVAL;
    if (!p) return c->fail(Q35K_EINVAL, "host_unregister: NULL pointer");
    cudaSetDevice(c->device);
    {
        std::lock_guard<std::mutex> lock(g_ranges_mu);
        for (size_t i = 0; i < g_ranges.size(); i++)
            if (g_ranges[i].base == p) {
                g_ranges.erase(g_ranges.begin() + (long)i);
                break;
            }
    }
    const cudaError_t e = cudaHostUnregister(p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return c->fail(Q35K_EINVAL, "host_unregister: %s", cudaGetErrorString(e));
    }
    return Q35K_OK;
}

int q35k_matmul_argmax_dev(q35k_ctx* c, const q35k_weight* w, const float* d_x, float* d_y, int* d_idx, int tokens,
                           void* stream) {
    int rc = check_matmul_args(c, w, d_x, d_idx, tokens);
    if (rc) return rc;
    if ((rc = check_alignment(c, d_x, 16, d_y, 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    const cudaStream_t s = pick(c, stream);
    // The keys are zeroed when allocated and cleared again by the index
    // kernel of every call, so no reset precedes the GEMV (which then starts
    // with programmatic dependent launch like any other decode call).
    if ((rc = c->ensure_dev((void**)&c->d_amax, &c->amax_cap, (size_t)tokens * sizeof(unsigned long long), true)) !=
        Q35K_OK)
        return rc;
    if ((rc = c->matmul_into(w, d_x, d_y, w->n_out, tokens, s, nullptr, c->d_amax)) != Q35K_OK) return rc;
    cudaError_t e = launch_argmax_index(c->d_amax, d_idx, tokens, s);
    if (e != cudaSuccess) return c->cuda_fail(e, "argmax index launch");
    return Q35K_OK;
}

int q35k_matmul_argmax(q35k_ctx* c, const q35k_weight* w, const float* x, int* idx, int tokens) {
    int rc = check_matmul_args(c, w, x, idx, tokens);
    if (rc) return rc;
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)tokens * w->n_in * sizeof(float);
    const size_t out_bytes = (size_t)tokens * sizeof(int);
    if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, in_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_in, &c->h_in_cap, in_bytes)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_out, &c->h_out_cap, out_bytes + 64)) != Q35K_OK) return rc;
    std::memcpy(c->h_in, x, in_bytes);
    cudaError_t e = cudaMemcpyAsync(c->d_x, c->h_in, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "H2D copy of x");
    int* d_idx = reinterpret_cast<int*>(c->d_y);
    if ((rc = q35k_matmul_argmax_dev(c, w, c->d_x, nullptr, d_idx, tokens, c->stream)) != Q35K_OK) return rc;
    unsigned* h_err = (unsigned*)((char*)c->h_out + out_bytes);
    e = cudaMemcpyAsync(c->h_out, d_idx, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "matmul_argmax");
    if (*h_err) return c->on_device_error(*h_err);
    std::memcpy(idx, c->h_out, out_bytes);
    return Q35K_OK;
}

static int check_shared_args(q35k_ctx* c, const q35k_weight* const* ws, int count, const void* x,
                             const void* const* ys, int tokens) {
    if (!c) return Q35K_EINVAL;
    if (!ws || !ys) return c->fail(Q35K_EINVAL, "weight or output array is NULL");
    if (count < 1 || count > Q35K_MAX_SHARED)
        return c->fail(Q35K_EINVAL, "count must be 1..%d (got %d)", Q35K_MAX_SHARED, count);
    for (int i = 0; i < count; i++) {
        int rc = check_matmul_args(c, ws[i], x, ys[i], tokens);
        if (rc) return rc;
        if (ws[i]->n_in != ws[0]->n_in)
            return c->fail(Q35K_EINVAL, "weights of one shared call differ in nIn (%d vs %d)", ws[i]->n_in, ws[0]->n_in);
    }
    return Q35K_OK;
}

int q35k_matmul_shared_dev(q35k_ctx* c, const q35k_weight* const* ws, int count, const float* d_x, float* const* d_ys,
                           int tokens, void* stream) {
    int rc = check_shared_args(c, ws, count, d_x, (const void* const*)d_ys, tokens);
    if (rc) return rc;
    for (int i = 0; i < count; i++)
        if ((rc = check_alignment(c, d_x, 16, d_ys[i], 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    return c->matmul_shared(ws, count, d_x, d_ys, tokens, pick(c, stream));
}

int q35k_matmul_shared(q35k_ctx* c, const q35k_weight* const* ws, int count, const float* x, float* const* ys,
                       int tokens) {
    int rc = check_shared_args(c, ws, count, x, (const void* const*)ys, tokens);
    if (rc) return rc;
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)tokens * ws[0]->n_in * sizeof(float);
    size_t out_bytes = 0, off[Q35K_MAX_SHARED];
    for (int i = 0; i < count; i++) {
        off[i] = out_bytes;
        out_bytes += ((size_t)tokens * ws[i]->n_out * sizeof(float) + 15) / 16 * 16;
    }
    if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, in_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_in, &c->h_in_cap, in_bytes)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_out, &c->h_out_cap, out_bytes + 64)) != Q35K_OK) return rc;
    std::memcpy(c->h_in, x, in_bytes);
    cudaError_t e = cudaMemcpyAsync(c->d_x, c->h_in, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "H2D copy of x");
    float* d_ys[Q35K_MAX_SHARED];
    for (int i = 0; i < count; i++) d_ys[i] = (float*)((char*)c->d_y + off[i]);
    if ((rc = c->matmul_shared(ws, count, c->d_x, d_ys, tokens, c->stream)) != Q35K_OK) return rc;
    unsigned* h_err = (unsigned*)((char*)c->h_out + out_bytes);
    e = cudaMemcpyAsync(c->h_out, c->d_y, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "matmul_shared");
    if (*h_err) return c->on_device_error(*h_err);
    for (int i = 0; i < count; i++)
        std::memcpy(ys[i], (char*)c->h_out + off[i], (size_t)tokens * ws[i]->n_out * sizeof(float));
    return Q35K_OK;
}

int q35k_matmul_silu_dev(q35k_ctx* c, const q35k_weight* w, const float* d_gate, const float* d_up, float* d_y,
                         int tokens, void* stream) {
    int rc = check_matmul_args(c, w, d_gate, d_y, tokens);
    if (rc) return rc;
    if (!d_up) return c->fail(Q35K_EINVAL, "up pointer is NULL");
    if ((rc = check_alignment(c, d_gate, 16, d_y, 4)) != Q35K_OK) return rc;
    if ((rc = check_alignment(c, d_up, 16, d_y, 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    return c->matmul_into(w, d_gate, d_y, w->n_out, tokens, pick(c, stream), nullptr, nullptr, d_up);
}

int q35k_matmul_silu(q35k_ctx* c, const q35k_weight* w, const float* gate, const float* up, float* y, int tokens) {
    int rc = check_matmul_args(c, w, gate, y, tokens);
    if (rc) return rc;
    if (!up) return c->fail(Q35K_EINVAL, "up pointer is NULL");
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)tokens * w->n_in * sizeof(float);
    const size_t out_bytes = (size_t)tokens * w->n_out * sizeof(float);
    if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, 2 * in_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_in, &c->h_in_cap, 2 * in_bytes)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_out, &c->h_out_cap, out_bytes + 64)) != Q35K_OK) return rc;
    std::memcpy(c->h_in, gate, in_bytes);
    std::memcpy((char*)c->h_in + in_bytes, up, in_bytes);
    cudaError_t e = cudaMemcpyAsync(c->d_x, c->h_in, 2 * in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "H2D copy of gate and up");
    const float* d_up = (const float*)((const char*)c->d_x + in_bytes);
    if ((rc = q35k_matmul_silu_dev(c, w, c->d_x, d_up, c->d_y, tokens, c->stream)) != Q35K_OK) return rc;
    unsigned* h_err = (unsigned*)((char*)c->h_out + out_bytes);
    e = cudaMemcpyAsync(c->h_out, c->d_y, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "matmul_silu");
    if (*h_err) return c->on_device_error(*h_err);
    std::memcpy(y, c->h_out, out_bytes);
    return Q35K_OK;
}

int q35k_matmul_q8k(q35k_ctx* c, const q35k_weight* w, const void* q8k, float* y, int tokens) {
    int rc = check_matmul_args(c, w, q8k, y, tokens);
    if (rc) return rc;
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)tokens * w->nb * Q8K_BYTES;
    const size_t out_bytes = (size_t)tokens * w->n_out * sizeof(float);
    if ((rc = c->ensure_dev((void**)&c->d_q8raw, &c->q8raw_cap, in_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_in, &c->h_in_cap, in_bytes)) != Q35K_OK) return rc;
    if ((rc = c->ensure_host(&c->h_out, &c->h_out_cap, out_bytes + 64)) != Q35K_OK) return rc;
    std::memcpy(c->h_in, q8k, in_bytes);
    cudaError_t e = cudaMemcpyAsync(c->d_q8raw, c->h_in, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "H2D copy of q8k");
    if ((rc = q35k_matmul_q8k_dev(c, w, c->d_q8raw, c->d_y, tokens, c->stream)) != Q35K_OK) return rc;
    unsigned* h_err = (unsigned*)((char*)c->h_out + out_bytes);
    e = cudaMemcpyAsync(c->h_out, c->d_y, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_err, c->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return c->cuda_fail(e, "matmul_q8k");
    if (*h_err) return c->on_device_error(*h_err);
    std::memcpy(y, c->h_out, out_bytes);
    return Q35K_OK;
}

// Q8_K rows of x, or of silu(x) * up (up != nullptr).
static int quantize_dev(q35k_ctx* c, const float* d_x, const float* d_up, void* d_q8k, int k, int rows, void* stream) {
    if (!c) return Q35K_EINVAL;
    if (!d_x || !d_q8k) return c->fail(Q35K_EINVAL, "NULL pointer");
    if (k <= 0 || k % QK) return c->fail(Q35K_EINVAL, "k=%d is not a multiple of 256", k);
    if (rows <= 0) return c->fail(Q35K_EINVAL, "rows must be positive");
    int rc = check_alignment(c, d_x, 16, d_q8k, 4);
    if (rc) return rc;
    if (d_up && (rc = check_alignment(c, d_up, 16, d_q8k, 4)) != Q35K_OK) return rc;
    cudaSetDevice(c->device);
    cudaError_t e = launch_quantize_q8k(d_x, (uint8_t*)d_q8k, k, rows, 0, pick(c, stream), d_up);
    return e == cudaSuccess ? Q35K_OK : c->cuda_fail(e, "Q8_K quantize launch");
}

static int quantize_host(q35k_ctx* c, const float* x, const float* up, void* q8k, int k, int rows) {
    if (!c) return Q35K_EINVAL;
    if (!x || !q8k) return c->fail(Q35K_EINVAL, "NULL pointer");
    if (k <= 0 || k % QK) return c->fail(Q35K_EINVAL, "k=%d is not a multiple of 256", k);
    if (rows <= 0) return c->fail(Q35K_EINVAL, "rows must be positive");
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)rows * k * sizeof(float);
    const size_t out_bytes = (size_t)rows * (k / QK) * Q8K_BYTES;
    const int n_in = up ? 2 : 1;
    int rc;
    if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, n_in * in_bytes, false)) != Q35K_OK) return rc;
    if ((rc = c->ensure_dev((void**)&c->d_q8raw, &c->q8raw_cap, out_bytes, false)) != Q35K_OK) return rc;
    const float* d_up = up ? (const float*)((const char*)c->d_x + in_bytes) : nullptr;
    cudaError_t e = cudaMemcpyAsync(c->d_x, x, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && up) e = cudaMemcpyAsync((void*)d_up, up, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_quantize_q8k(c->d_x, c->d_q8raw, k, rows, 0, c->stream, d_up);
    if (e == cudaSuccess) e = cudaMemcpyAsync(q8k, c->d_q8raw, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    return e == cudaSuccess ? Q35K_OK : c->cuda_fail(e, "quantize_q8k");
}

int q35k_quantize_q8k_dev(q35k_ctx* c, const float* d_x, void* d_q8k, int k, int rows, void* stream) {
    return quantize_dev(c, d_x, nullptr, d_q8k, k, rows, stream);
}
int q35k_quantize_q8k(q35k_ctx* c, const float* x, void* q8k, int k, int rows) {
    return quantize_host(c, x, nullptr, q8k, k, rows);
}
int q35k_quantize_q8k_silu_dev(q35k_ctx* c, const float* d_gate, const float* d_up, void* d_q8k, int k, int rows,
                               void* stream) {
    if (c && !d_up) return c->fail(Q35K_EINVAL, "NULL pointer");
    return quantize_dev(c, d_gate, d_up, d_q8k, k, rows, stream);
}
int q35k_quantize_q8k_silu(q35k_ctx* c, const float* gate, const float* up, void* q8k, int k, int rows) {
    if (c && !up) return c->fail(Q35K_EINVAL, "NULL pointer");
    return quantize_host(c, gate, up, q8k, k, rows);
}

int q35k_dequantize_dev(q35k_ctx* c, int type, const void* d_blocks, float* d_y, int k, int rows, void* stream) {
    if (!c) return Q35K_EINVAL;
    if (!valid_type(type)) return c->fail(Q35K_ENOTSUP, "ggml type %d is not a K-quant type", type);
    if (!d_blocks || !d_y) return c->fail(Q35K_EINVAL, "NULL pointer");
    if (k <= 0 || k % QK) return c->fail(Q35K_EINVAL, "k=%d is not a multiple of 256", k);
    if (rows <= 0) return c->fail(Q35K_EINVAL, "rows must be positive");
    int rc = check_alignment(c, d_blocks, 1, d_y, 4);
    if (rc) return rc;
    cudaSetDevice(c->device);
    cudaError_t e = launch_dequantize(type, (const uint8_t*)d_blocks, d_y, k, rows, pick(c, stream));
    return e == cudaSuccess ? Q35K_OK : c->cuda_fail(e, "dequantize launch");
}

int q35k_dequantize(q35k_ctx* c, int type, const void* blocks, float* y, int k, int rows) {
    if (!c) return Q35K_EINVAL;
    if (!valid_type(type)) return c->fail(Q35K_ENOTSUP, "ggml type %d is not a K-quant type", type);
    if (!blocks || !y) return c->fail(Q35K_EINVAL, "NULL pointer");
    if (k <= 0 || k % QK) return c->fail(Q35K_EINVAL, "k=%d is not a multiple of 256", k);
    if (rows <= 0) return c->fail(Q35K_EINVAL, "rows must be positive");
    cudaSetDevice(c->device);
    const size_t in_bytes = (size_t)rows * (k / QK) * block_bytes(type);
    const size_t out_bytes = (size_t)rows * k * sizeof(float);
    void* d_in = nullptr;
    float* d_out = nullptr;
    cudaError_t e = cudaMalloc(&d_in, in_bytes);
    if (e == cudaSuccess) e = cudaMalloc((void**)&d_out, out_bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d_in);
        return c->fail(Q35K_ENOMEM, "dequantize: cudaMalloc failed");
    }
    e = cudaMemcpyAsync(d_in, blocks, in_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_dequantize(type, (const uint8_t*)d_in, d_out, k, rows, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(y, d_out, out_bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d_in);
    cudaFree(d_out);
    return e == cudaSuccess ? Q35K_OK : c->cuda_fail(e, "dequantize");
}

}  // extern "C"
