// shard.cu -- row-sharded matmul over several GPUs of one node: each rank
// holds rows [r * n_shard, (r + 1) * n_shard) of the weight, computes its
// slice of y with the single-GPU kernels, and the slices are all-gathered
// over NVLink (NCCL, or peer copies) so that every rank ends with the full y.
//
// The reference splits output rows between the workers of its thread pool
// the same way (Kernels/MulMatQ4K.cs:31-36); here the workers are GPUs.
// Two ways to build a group:
//   * q35k_shard_create: one process drives all GPUs (ncclCommInitAll);
//   * q35k_shard_create_rank: one process per GPU (ncclCommInitRank with an
//     id from q35k_nccl_unique_id shared by the caller).
// NCCL is loaded at run time (libnccl.so.2); without it only the peer-copy
// and fused gathers of a single-process group are available.
//
// Fused gather (Q35K_GATHER_FUSED, decode calls of at most 8 tokens): every
// rank owns a "symmetric" buffer -- a header (the rank's call counter) and
// two gather areas [nranks][tokens][n_shard] of 64-bit words used on
// alternate calls -- that every other rank can store into (CUDA IPC mappings
// exchanged once over NCCL, or peer pointers in one process).  The GEMV
// writes its rows straight into the caller's y and stores each of them into
// every peer's area as one 64-bit word (call number << 32 | value bits), so
// the receiver knows a value has arrived from the word itself: there is no
// fence, flag or separate publish step.  The gather kernel after the GEMV
// starts while the GEMV's last CTAs still run, waits (bounded in time) for
// each peer word of this call and copies the values into y.  The call
// counter lives in device memory and is advanced by that kernel once its own
// GEMV has completed, so a call's kernel arguments do not change from call
// to call (the call can be captured in a CUDA graph).  Alternate areas keep
// a peer's next call from overwriting a slice this rank is still reading:
// that call's stores come after the peer's own gather of the call in
// between, which needed this rank's words of that call.
#include "../../include/q35k.h"
#include "api_internal.h"
#include "device_common.cuh"
#include "kernels.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <new>
#include <string>
#include <vector>

namespace q35k {
void set_thread_error(const std::string& msg);  // api.cu

namespace {

// ---- NCCL, resolved at run time ----
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.why = std::string("libnccl.so.2 could not be loaded: ") + dlerror();
            return;
        }
        bool all = true;
        auto get = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn) all = false;
        };
        get(api.GetUniqueId, "ncclGetUniqueId");
        get(api.CommInitRank, "ncclCommInitRank");
        get(api.CommInitAll, "ncclCommInitAll");
        get(api.CommDestroy, "ncclCommDestroy");
        get(api.AllGather, "ncclAllGather");
        get(api.GroupStart, "ncclGroupStart");
        get(api.GroupEnd, "ncclGroupEnd");
        get(api.GetErrorString, "ncclGetErrorString");
        api.ok = all;
        if (!all) api.why = "libnccl.so.2 lacks an expected entry point";
    });
    return api;
}

// Rows per rank: an equal share (the last rank may hold fewer).  Every rank
// lays out its own rows in tiles, so a shard may start at any row; when the
// ranks hold equal shares a single-token y is gathered in place.
int shard_rows(int n_out, int nranks) { return (n_out + nranks - 1) / nranks; }

// y[t][r * n_shard + j] = g[r][t][j] for the columns below n_out.
// Launched with programmatic dependent launch in the fused gather: the next
// call's GEMV may start streaming its weights at once (it reads x and stores
// into the other gather areas only after its own griddepcontrol.wait), and
// this kernel reads the gather area only after the kernel before it (the
// flag wait) has completed.
__global__ void gather_permute_kernel(const float* __restrict__ g, float* __restrict__ y, int nranks, int tokens,
                                      int n_shard, int n_out) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const long long total = (long long)tokens * n_out;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / n_out), c = (int)(i % n_out);
        const int r = c / n_shard, j = c - r * n_shard;
        y[i] = g[((size_t)r * tokens + t) * n_shard + j];
    }
}

// Symmetric buffer header (u32 words): this rank's count of completed fused
// calls at HDR_SEQ, the gather kernel's arrival counter at HDR_DONE, and
// 64-bit phase timestamps from byte HDR_TRACE (tracing only).  The gather
// areas start at SYM_HDR.
constexpr size_t SYM_HDR = 256;
constexpr int SYM_MAX_RANKS = 32;
constexpr int HDR_SEQ = 32, HDR_DONE = 33;
constexpr size_t HDR_TRACE = 192;  // 8 slots of u64
constexpr int TRACE_SLOTS = 6;

struct GatherArgs {
    int peer_rank[GEMV_MAX_PEERS];
    unsigned* hdr;                        // this rank's buffer header
    const unsigned long long* area;       // this rank's gather area 0, [nranks][tokens][n_shard] words
    float* y;                             // [tokens][ldy]
    size_t half;                          // words from area 0 to area 1
    int n_peers, tokens, n_shard, n_out, ldy;
    unsigned* err;
    unsigned long long* trace;            // phase timestamps (nullptr: off)
    unsigned long long limit_ns;          // bound of the wait for a peer's words
};

// After this rank's GEMV (launched with programmatic dependent launch; it may
// start while the GEMV's last CTAs run, which is safe because this kernel
// reads only the peers' words, and because the GEMV lets it start only once
// the previous call's gather has completed, so the call counter it reads is
// current).  A wait that runs out sets DEV_ERR_TIMEOUT and skips the rest;
// the host then reports Q35K_ETIMEOUT and the group must be reset
// (q35k_shard_reset) before its next fused call.
__global__ void __launch_bounds__(256) q35k_shard_gather_kernel(GatherArgs g) {
    asm volatile("griddepcontrol.launch_dependents;");
    const unsigned ep = *reinterpret_cast<volatile const unsigned*>(g.hdr + HDR_SEQ) + 1u;
    const int tid = threadIdx.x;
    if (g.trace && tid == 0) atomicMin(g.trace + 2, (unsigned long long)globaltimer_ns());
    const unsigned long long* area = g.area + (size_t)(ep & 1u) * g.half;
    const int nthreads = gridDim.x * blockDim.x, me = blockIdx.x * blockDim.x + tid;
    bool good = true;
    const uint64_t t0 = globaltimer_ns();
    for (int k = 0; good && k < g.n_peers; k++) {
        const int r = g.peer_rank[k];
        const int rows = min(g.n_shard, g.n_out - r * g.n_shard);
        for (int t = 0; good && t < g.tokens; t++) {
            const unsigned long long* src = area + ((size_t)r * g.tokens + t) * g.n_shard;
            float* dst = g.y + (size_t)t * g.ldy + (size_t)r * g.n_shard;
            for (int j = me; j < rows; j += nthreads) {
                unsigned long long v = ld_relaxed_sys_u64(src + j);
                for (uint32_t it = 0; (unsigned)(v >> 32) != ep; ++it) {
                    if ((it & 63u) == 63u && globaltimer_ns() - t0 > g.limit_ns) {
                        atomicOr(g.err, DEV_ERR_TIMEOUT);
                        good = false;
                        break;
                    }
                    __nanosleep(64);
                    v = ld_relaxed_sys_u64(src + j);
                }
                if (!good) break;
                dst[j] = __uint_as_float((unsigned)v);
            }
        }
    }
    if (g.trace) atomicMax(g.trace + 3, (unsigned long long)globaltimer_ns());
    // The last CTA to finish advances this rank's call counter -- after this
    // rank's GEMV has completed (it reads the counter) -- for the next call's
    // kernels, which read it after their own grid-dependency wait.
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(g.hdr + HDR_DONE, 1u) == gridDim.x - 1) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            if (g.trace) atomicMax(g.trace + 4, (unsigned long long)globaltimer_ns());
            *reinterpret_cast<volatile unsigned*>(g.hdr + HDR_DONE) = 0u;
            *reinterpret_cast<volatile unsigned*>(g.hdr + HDR_SEQ) = ep;
        }
        if (g.trace) atomicMax(g.trace + 5, (unsigned long long)globaltimer_ns());
    }
}

}  // namespace
}  // namespace q35k

using namespace q35k;

struct q35k_shard {
    int nranks = 0;               // ranks in the group
    int first_rank = 0;           // rank of local device 0
    std::vector<int> devices;     // local devices (all of them, or this process's one)
    std::vector<q35k_ctx*> ctxs;  // one context per local device
    std::vector<ncclComm_t> comms;
    std::vector<float*> gbuf;     // per local device: [nranks][tokens][n_shard]
    std::vector<size_t> gcap;
    std::vector<cudaEvent_t> done;     // per local device: its slice is in every peer's gather buffer
    std::vector<cudaEvent_t> free_ev;  // per local device: its gather buffer has been read out
    std::vector<char> used;
    // Fused gather: per local device its symmetric buffer, and every rank's
    // buffer as that device addresses it ([local][rank]; opened through IPC
    // where sym_ipc is set).
    std::vector<uint8_t*> sym;
    std::vector<std::vector<uint8_t*>> sym_view;
    std::vector<std::vector<char>> sym_ipc;
    size_t sym_area = 0;  // bytes of one gather area
    unsigned long long wait_limit_ns = 2000000000ull;  // bound of the fused gather's flag wait
    bool trace = false;   // record phase timestamps of fused calls
    std::string err;

    int fail(int code, const std::string& msg) {
        err = msg;
        return code;
    }
    int nccl_fail(ncclResult_t r, const char* what) {
        return fail(Q35K_ENCCL, std::string(what) + ": " + nccl().GetErrorString(r));
    }
};

struct q35k_sharded_weight {
    int type = 0, n_in = 0, n_out = 0, n_shard = 0;
    std::vector<q35k_weight*> parts;  // per local device: its rows
};

// Close this process's IPC views of peers' symmetric buffers and free its own.
static void free_sym(q35k_shard* s) {
    for (size_t i = 0; i < s->sym.size(); i++) {
        cudaSetDevice(s->devices[i]);
        for (size_t j = 0; j < s->sym_view[i].size(); j++)
            if (s->sym_ipc[i][j] && s->sym_view[i][j]) cudaIpcCloseMemHandle(s->sym_view[i][j]);
        if (s->sym[i]) cudaFree(s->sym[i]);
    }
    s->sym.clear();
    s->sym_view.clear();
    s->sym_ipc.clear();
    s->sym_area = 0;
}

static void destroy_shard(q35k_shard* s) {
    for (size_t i = 0; i < s->devices.size(); i++) {
        cudaSetDevice(s->devices[i]);
        cudaDeviceSynchronize();
    }
    free_sym(s);
    for (size_t i = 0; i < s->devices.size(); i++) {
        cudaSetDevice(s->devices[i]);
        cudaDeviceSynchronize();
        if (i < s->gbuf.size() && s->gbuf[i]) cudaFree(s->gbuf[i]);
        if (i < s->done.size() && s->done[i]) cudaEventDestroy(s->done[i]);
        if (i < s->free_ev.size() && s->free_ev[i]) cudaEventDestroy(s->free_ev[i]);
    }
    for (ncclComm_t c : s->comms)
        if (c) nccl().CommDestroy(c);
    for (q35k_ctx* c : s->ctxs) q35k_destroy(c);
    delete s;
}

static int init_local(q35k_shard* s) {
    for (int d : s->devices) {
        q35k_ctx* c = nullptr;
        const int rc = q35k_create(d, &c);
        if (rc != Q35K_OK) return s->fail(rc, std::string("context on device ") + std::to_string(d) + ": " +
                                                  q35k_last_error(nullptr));
        s->ctxs.push_back(c);
        cudaEvent_t ev, fe;
        cudaSetDevice(d);
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&fe, cudaEventDisableTiming) != cudaSuccess)
            return s->fail(Q35K_ECUDA, "cudaEventCreate failed");
        s->done.push_back(ev);
        s->free_ev.push_back(fe);
    }
    s->used.assign(s->devices.size(), 0);
    s->gbuf.assign(s->devices.size(), nullptr);
    s->gcap.assign(s->devices.size(), 0);
    return Q35K_OK;
}

// One process per GPU: all-gather `bytes` host bytes from every rank (NCCL
// on the group's stream, through a device staging buffer); also a barrier.
static int allgather_host(q35k_shard* s, const void* mine, void* all, size_t bytes) {
    cudaSetDevice(s->devices[0]);
    uint8_t* d = nullptr;
    if (cudaMalloc(&d, bytes * s->nranks) != cudaSuccess) {
        cudaGetLastError();
        return s->fail(Q35K_ENOMEM, "staging buffer for the handle exchange");
    }
    cudaStream_t st = s->ctxs[0]->stream;
    int rc = Q35K_OK;
    if (cudaMemcpyAsync(d + bytes * s->first_rank, mine, bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
        rc = s->fail(Q35K_ECUDA, "handle exchange copy");
    } else {
        const ncclResult_t r = nccl().AllGather(d + bytes * s->first_rank, d, bytes, ncclUint8, s->comms[0], st);
        if (r != ncclSuccess) rc = s->nccl_fail(r, "ncclAllGather (handle exchange)");
        else if (cudaMemcpyAsync(all, d, bytes * s->nranks, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                 cudaStreamSynchronize(st) != cudaSuccess)
            rc = s->fail(Q35K_ECUDA, "handle exchange copy back");
    }
    cudaFree(d);
    return rc;
}

// Collective: make every rank's symmetric buffer hold gather areas of at
// least `area` bytes, and map every peer's buffer.
static int ensure_sym(q35k_shard* s, size_t area) {
    if (!s->sym.empty() && area <= s->sym_area) return Q35K_OK;
    const int nloc = (int)s->devices.size();
    const bool one_process = nloc == s->nranks;
    if (!one_process && (s->comms.empty() || nloc != 1))
        return s->fail(Q35K_ENOTSUP, "the fused gather of a rank group needs NCCL for its handle exchange");
    if (s->nranks > SYM_MAX_RANKS) return s->fail(Q35K_ENOTSUP, "too many ranks for the fused gather");
    // Every store into the old buffers has landed: this rank's last fused call
    // waited for all peers' flags, which they raise after their stores.
    for (int i = 0; i < nloc; i++) {
        cudaSetDevice(s->devices[i]);
        if (cudaDeviceSynchronize() != cudaSuccess) return s->fail(Q35K_ECUDA, "synchronize before the gather buffers grow");
    }
    if (!s->sym.empty() && !one_process) {
        // Peers close their views of the old buffers before any rank frees its own.
        for (size_t j = 0; j < s->sym_view[0].size(); j++)
            if (s->sym_ipc[0][j] && s->sym_view[0][j]) cudaIpcCloseMemHandle(s->sym_view[0][j]);
        s->sym_ipc[0].assign(s->nranks, 0);
        char dummy = 0;
        std::vector<char> all(s->nranks);
        const int rc = allgather_host(s, &dummy, all.data(), 1);
        if (rc != Q35K_OK) return rc;
    }
    free_sym(s);
    const size_t bytes = SYM_HDR + 2 * area;
    s->sym.assign(nloc, nullptr);
    s->sym_view.assign(nloc, std::vector<uint8_t*>(s->nranks, nullptr));
    s->sym_ipc.assign(nloc, std::vector<char>(s->nranks, 0));
    for (int i = 0; i < nloc; i++) {
        cudaSetDevice(s->devices[i]);
        if (cudaMalloc(&s->sym[i], bytes) != cudaSuccess || cudaMemset(s->sym[i], 0, bytes) != cudaSuccess ||
            cudaDeviceSynchronize() != cudaSuccess) {
            cudaGetLastError();
            free_sym(s);
            return s->fail(Q35K_ENOMEM, "symmetric gather buffer allocation failed");
        }
    }
    if (one_process) {
        for (int i = 0; i < nloc; i++) {
            cudaSetDevice(s->devices[i]);
            for (int j = 0; j < nloc; j++) {
                s->sym_view[i][j] = s->sym[j];
                if (j == i) continue;
                int can = 0;
                cudaDeviceCanAccessPeer(&can, s->devices[i], s->devices[j]);
                if (!can) {
                    free_sym(s);
                    return s->fail(Q35K_ENOTSUP, "devices without peer access: no fused gather");
                }
                const cudaError_t e = cudaDeviceEnablePeerAccess(s->devices[j], 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                    free_sym(s);
                    return s->fail(Q35K_ECUDA, std::string("peer access: ") + cudaGetErrorString(e));
                }
                cudaGetLastError();
            }
        }
    } else {
        cudaSetDevice(s->devices[0]);
        cudaIpcMemHandle_t h;
        if (cudaIpcGetMemHandle(&h, s->sym[0]) != cudaSuccess) {
            cudaGetLastError();
            free_sym(s);
            return s->fail(Q35K_ECUDA, "cudaIpcGetMemHandle failed");
        }
        std::vector<cudaIpcMemHandle_t> all(s->nranks);
        int rc = allgather_host(s, &h, all.data(), sizeof h);
        if (rc != Q35K_OK) {
            free_sym(s);
            return rc;
        }
        for (int j = 0; j < s->nranks; j++) {
            if (j == s->first_rank) {
                s->sym_view[0][j] = s->sym[0];
                continue;
            }
            void* v = nullptr;
            const cudaError_t e = cudaIpcOpenMemHandle(&v, all[j], cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                cudaGetLastError();
                free_sym(s);
                return s->fail(Q35K_ECUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
            }
            s->sym_view[0][j] = static_cast<uint8_t*>(v);
            s->sym_ipc[0][j] = 1;
        }
        // Every rank has zeroed its buffer before any peer can store into it:
        // the exchange above completed on all ranks first.
    }
    s->sym_area = area;
    return Q35K_OK;
}

// Launch with programmatic stream serialization (the kernel starts while the
// previous one drains and orders itself with griddepcontrol.wait).
template <typename... P, typename... A>
static cudaError_t launch_pdl(void (*kernel)(P...), int grid, int block, cudaStream_t st, A... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((unsigned)block);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<P>(args)...);
}

// The fused-gather call (see the file comment); multi-rank groups only.
static int shard_matmul_fused(q35k_shard* s, const q35k_sharded_weight* w, const float* const* d_x,
                              float* const* d_y, int tokens, const std::function<cudaStream_t(int)>& stream_of) {
    const int nloc = (int)s->devices.size();
    const size_t slot = (size_t)tokens * w->n_shard;  // words per rank
    // Areas sized for the largest decode call of this weight (8 tokens), so
    // that the collective growth happens once.
    const size_t area = (size_t)s->nranks * 8 * w->n_shard * sizeof(unsigned long long);
    int rc = ensure_sym(s, area);
    if (rc != Q35K_OK) return rc;
    for (int i = 0; i < nloc; i++) {
        q35k_ctx* c = s->ctxs[i];
        cudaSetDevice(s->devices[i]);
        const cudaStream_t st = stream_of(i);
        const int rank = s->first_rank + i;
        unsigned* hdr = reinterpret_cast<unsigned*>(s->sym[i]);
        unsigned long long* trace =
            s->trace ? reinterpret_cast<unsigned long long*>(s->sym[i] + HDR_TRACE) : nullptr;
        GemvPeers pr{};
        GatherArgs g{};
        for (int j = 0; j < s->nranks; j++) {
            if (j == rank) continue;
            uint8_t* v = s->sym_view[i][j];
            pr.y[pr.n++] = reinterpret_cast<unsigned long long*>(v + SYM_HDR) + (size_t)rank * slot;
            g.peer_rank[g.n_peers++] = j;
        }
        pr.ldp = w->n_shard;
        pr.half = s->sym_area / sizeof(unsigned long long);
        pr.seq = hdr + HDR_SEQ;
        pr.trace = trace;
        if (trace) {
            // slots 0 and 2 take a minimum, the others a maximum
            cudaMemsetAsync(trace, 0, TRACE_SLOTS * sizeof(unsigned long long), st);
            cudaMemsetAsync(trace, 0xff, sizeof(unsigned long long), st);
            cudaMemsetAsync(trace + 2, 0xff, sizeof(unsigned long long), st);
        }
        if (w->parts[i]) {
            // This rank's rows go straight to their columns of y.
            rc = c->matmul_into(w->parts[i], d_x[i], d_y[i] + (size_t)rank * w->n_shard, w->n_out, tokens, st, &pr);
            if (rc != Q35K_OK) return s->fail(rc, c->err);
        }
        g.hdr = hdr;
        g.area = reinterpret_cast<const unsigned long long*>(s->sym[i] + SYM_HDR);
        g.y = d_y[i];
        g.half = pr.half;
        g.tokens = tokens;
        g.n_shard = w->n_shard;
        g.n_out = w->n_out;
        g.ldy = w->n_out;
        g.err = c->d_err;
        g.trace = trace;
        g.limit_ns = s->wait_limit_ns;
        const long long total = (long long)g.n_peers * slot;
        const int grid = (int)std::max(1LL, std::min<long long>((total + 1023) / 1024, 148));
        cudaError_t e = launch_pdl(q35k_shard_gather_kernel, grid, 256, st, g);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return s->fail(Q35K_ECUDA, std::string("fused gather: ") + cudaGetErrorString(e));
    }
    return Q35K_OK;
}

extern "C" {

int q35k_nccl_unique_id(void* id_out) {
    if (!id_out) return Q35K_EINVAL;
    const NcclApi& n = nccl();
    if (!n.ok) {
        set_thread_error(n.why);
        return Q35K_ENOTSUP;
    }
    ncclUniqueId id;
    const ncclResult_t r = n.GetUniqueId(&id);
    if (r != ncclSuccess) {
        set_thread_error(std::string("ncclGetUniqueId: ") + n.GetErrorString(r));
        return Q35K_ENCCL;
    }
    std::memcpy(id_out, &id, sizeof id);
    return Q35K_OK;
}

int q35k_shard_create(int ndev, const int* devices, q35k_shard** out) {
    if (!out || ndev < 1 || !devices) return Q35K_EINVAL;
    *out = nullptr;
    q35k_shard* s = new (std::nothrow) q35k_shard();
    if (!s) return Q35K_ENOMEM;
    s->nranks = ndev;
    s->devices.assign(devices, devices + ndev);
    int rc = init_local(s);
    if (rc == Q35K_OK && ndev > 1) {
        const NcclApi& n = nccl();
        if (n.ok) {
            s->comms.assign(ndev, nullptr);
            const ncclResult_t r = n.CommInitAll(s->comms.data(), ndev, devices);
            if (r != ncclSuccess) {
                s->comms.clear();
                rc = s->nccl_fail(r, "ncclCommInitAll");
            }
        }
        // Without NCCL the group still works with the peer-copy gather.
    }
    if (rc != Q35K_OK) {
        set_thread_error(s->err);
        destroy_shard(s);
        return rc;
    }
    *out = s;
    return Q35K_OK;
}

int q35k_shard_create_rank(int nranks, int rank, const void* nccl_id, int device, q35k_shard** out) {
    if (!out || nranks < 1 || rank < 0 || rank >= nranks || (nranks > 1 && !nccl_id)) return Q35K_EINVAL;
    *out = nullptr;
    q35k_shard* s = new (std::nothrow) q35k_shard();
    if (!s) return Q35K_ENOMEM;
    s->nranks = nranks;
    s->first_rank = rank;
    s->devices.push_back(device);
    int rc = init_local(s);
    if (rc == Q35K_OK && nranks > 1) {
        const NcclApi& n = nccl();
        if (!n.ok) {
            rc = s->fail(Q35K_ENOTSUP, n.why);
        } else {
            ncclUniqueId id;
            std::memcpy(&id, nccl_id, sizeof id);
            ncclComm_t c = nullptr;
            cudaSetDevice(device);
            const ncclResult_t r = n.CommInitRank(&c, nranks, id, rank);
            if (r != ncclSuccess) rc = s->nccl_fail(r, "ncclCommInitRank");
            else s->comms.push_back(c);
        }
    }
    if (rc != Q35K_OK) {
        set_thread_error(s->err);
        destroy_shard(s);
        return rc;
    }
    *out = s;
    return Q35K_OK;
}

int q35k_shard_destroy(q35k_shard* s) {
    if (s) destroy_shard(s);
    return Q35K_OK;
}

const char* q35k_shard_last_error(const q35k_shard* s) { return s ? s->err.c_str() : q35k_last_error(nullptr); }

int q35k_shard_weight_upload(q35k_shard* s, int ggml_type, const void* blocks, int n_in, int n_out,
                             q35k_sharded_weight** out) {
    if (!s || !out || !blocks || n_in <= 0 || n_out <= 0) return Q35K_EINVAL;
    *out = nullptr;
    if (n_in % QK) return s->fail(Q35K_ENOTSUP, "nIn is not a multiple of 256");
    const int bb = block_bytes(ggml_type);
    if (!bb) return s->fail(Q35K_ENOTSUP, "not a K-quant weight type");
    q35k_sharded_weight* w = new (std::nothrow) q35k_sharded_weight();
    if (!w) return Q35K_ENOMEM;
    w->type = ggml_type;
    w->n_in = n_in;
    w->n_out = n_out;
    w->n_shard = shard_rows(n_out, s->nranks);
    const size_t row_bytes = (size_t)(n_in / QK) * bb;
    for (size_t i = 0; i < s->devices.size(); i++) {
        const int rank = s->first_rank + (int)i;
        const int r0 = std::min(n_out, rank * w->n_shard), r1 = std::min(n_out, r0 + w->n_shard);
        q35k_weight* part = nullptr;
        if (r1 > r0) {
            const int rc = q35k_weight_upload(s->ctxs[i], ggml_type, static_cast<const uint8_t*>(blocks) + r0 * row_bytes,
                                              n_in, r1 - r0, &part);
            if (rc != Q35K_OK) {
                s->err = q35k_last_error(s->ctxs[i]);
                for (size_t k = 0; k < w->parts.size(); k++) q35k_weight_free(s->ctxs[k], w->parts[k]);
                delete w;
                return rc;
            }
        }
        w->parts.push_back(part);
    }
    *out = w;
    return Q35K_OK;
}

int q35k_shard_weight_free(q35k_shard* s, q35k_sharded_weight* w) {
    if (!w) return Q35K_OK;
    for (size_t i = 0; i < w->parts.size(); i++)
        if (w->parts[i]) q35k_weight_free(s ? s->ctxs[i] : nullptr, w->parts[i]);
    delete w;
    return Q35K_OK;
}

int q35k_shard_matmul_dev(q35k_shard* s, const q35k_sharded_weight* w, const float* const* d_x, float* const* d_y,
                          int tokens, int gather_mode, void* const* streams) {
    if (!s || !w || !d_x || !d_y || tokens <= 0) return Q35K_EINVAL;
    auto stream_of = [&](int i) -> cudaStream_t {
        return (streams && streams[i]) ? static_cast<cudaStream_t>(streams[i]) : s->ctxs[i]->stream;
    };
    if (gather_mode != Q35K_GATHER_NCCL && gather_mode != Q35K_GATHER_PEER && gather_mode != Q35K_GATHER_FUSED)
        return s->fail(Q35K_EINVAL, "gather_mode must be Q35K_GATHER_NCCL, Q35K_GATHER_PEER or Q35K_GATHER_FUSED");
    const int nloc = (int)s->devices.size();
    const bool multi = s->nranks > 1;
    if (gather_mode == Q35K_GATHER_FUSED) {
        if (multi && tokens <= Q35K_STATIC_MAX_TOKENS && s->nranks - 1 <= GEMV_MAX_PEERS)
            return shard_matmul_fused(s, w, d_x, d_y, tokens, stream_of);
        // Prefill-sized calls (and single-rank groups) take the other gathers.
        gather_mode = (nloc == s->nranks || s->comms.empty()) ? Q35K_GATHER_PEER : Q35K_GATHER_NCCL;
        if (multi && gather_mode == Q35K_GATHER_PEER && nloc != s->nranks)
            return s->fail(Q35K_ENOTSUP, "no NCCL for this rank group's gather");
    }
    if (multi && gather_mode == Q35K_GATHER_NCCL && s->comms.empty())
        return s->fail(Q35K_ENOTSUP, std::string("NCCL gather unavailable: ") + nccl().why);
    if (multi && gather_mode == Q35K_GATHER_PEER && nloc != s->nranks)
        return s->fail(Q35K_ENOTSUP, "the peer-copy gather needs all ranks in this process");
    const size_t slot = (size_t)tokens * w->n_shard;  // floats per rank
    // The output is its own gather buffer when the slices are contiguous in y.
    const bool direct = tokens == 1 && w->n_out == s->nranks * w->n_shard;
    for (int i = 0; i < nloc; i++) {
        q35k_ctx* c = s->ctxs[i];
        cudaSetDevice(s->devices[i]);
        float* g = d_y[i];
        if (!direct) {
            const size_t need = slot * s->nranks * sizeof(float);
            if (need > s->gcap[i]) {
                if (s->gbuf[i]) cudaFree(s->gbuf[i]);
                s->gbuf[i] = nullptr;
                s->gcap[i] = 0;
                if (cudaMalloc(&s->gbuf[i], need) != cudaSuccess) {
                    cudaGetLastError();
                    return s->fail(Q35K_ENOMEM, "gather buffer allocation failed");
                }
                s->gcap[i] = need;
            }
            g = s->gbuf[i];
        }
        const int rank = s->first_rank + i;
        float* mine = g + (size_t)rank * slot;
        if (multi && gather_mode == Q35K_GATHER_PEER) {
            // Peers may still read this buffer from the previous call.
            for (int j = 0; j < nloc; j++)
                if (j != i && s->used[j]) cudaStreamWaitEvent(stream_of(i), s->free_ev[j], 0);
        }
        if (w->parts[i]) {
            // Slot layout [tokens][n_shard]; this rank's rows fill the first
            // columns (the last rank may hold fewer).
            const int rc = c->matmul_into(w->parts[i], d_x[i], mine, w->n_shard, tokens, stream_of(i));
            if (rc != Q35K_OK) return s->fail(rc, c->err);
        } else {
            cudaMemsetAsync(mine, 0, slot * sizeof(float), stream_of(i));
        }
    }
    if (multi) {
        if (gather_mode == Q35K_GATHER_NCCL) {
            const NcclApi& n = nccl();
            n.GroupStart();
            for (int i = 0; i < nloc; i++) {
                cudaSetDevice(s->devices[i]);
                float* g = direct ? d_y[i] : s->gbuf[i];
                const ncclResult_t r = n.AllGather(g + (size_t)(s->first_rank + i) * slot, g, slot, ncclFloat32,
                                                   s->comms[i], stream_of(i));
                if (r != ncclSuccess) {
                    n.GroupEnd();
                    return s->nccl_fail(r, "ncclAllGather");
                }
            }
            const ncclResult_t r = n.GroupEnd();
            if (r != ncclSuccess) return s->nccl_fail(r, "ncclGroupEnd");
        } else {
            // Each device pushes its slice into every peer's buffer (copy
            // engines over NVLink), then the peers wait for all pushes.
            for (int i = 0; i < nloc; i++) {
                cudaSetDevice(s->devices[i]);
                const float* src = (direct ? d_y[i] : s->gbuf[i]) + (size_t)i * slot;
                for (int j = 0; j < nloc; j++) {
                    if (j == i) continue;
                    float* dst = (direct ? d_y[j] : s->gbuf[j]) + (size_t)i * slot;
                    const cudaError_t e = cudaMemcpyPeerAsync(dst, s->devices[j], src, s->devices[i],
                                                              slot * sizeof(float), stream_of(i));
                    if (e != cudaSuccess) return s->fail(Q35K_ECUDA, std::string("peer copy: ") + cudaGetErrorString(e));
                }
                cudaEventRecord(s->done[i], stream_of(i));
            }
            for (int j = 0; j < nloc; j++) {
                cudaSetDevice(s->devices[j]);
                for (int i = 0; i < nloc; i++)
                    if (i != j) cudaStreamWaitEvent(stream_of(j), s->done[i], 0);
            }
        }
    }
    if (!direct) {
        for (int i = 0; i < nloc; i++) {
            cudaSetDevice(s->devices[i]);
            const long long total = (long long)tokens * w->n_out;
            const int grid = (int)std::min<long long>((total + 255) / 256, 4096);
            gather_permute_kernel<<<grid, 256, 0, stream_of(i)>>>(s->gbuf[i], d_y[i], s->nranks, tokens,
                                                                       w->n_shard, w->n_out);
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return s->fail(Q35K_ECUDA, std::string("gather permute: ") + cudaGetErrorString(e));
        }
    }
    if (multi && gather_mode == Q35K_GATHER_PEER) {
        for (int i = 0; i < nloc; i++) {
            cudaSetDevice(s->devices[i]);
            cudaEventRecord(s->free_ev[i], stream_of(i));
            s->used[i] = 1;
        }
    }
    return Q35K_OK;
}

int q35k_shard_sync(q35k_shard* s) {
    if (!s) return Q35K_EINVAL;
    for (q35k_ctx* c : s->ctxs) {
        const int rc = q35k_sync(c);
        if (rc != Q35K_OK) return s->fail(rc, q35k_last_error(c));
    }
    return Q35K_OK;
}

int q35k_shard_set_wait_limit(q35k_shard* s, int milliseconds) {
    if (!s) return Q35K_EINVAL;
    if (milliseconds < 1 || milliseconds > 600000) return s->fail(Q35K_EINVAL, "wait limit must be 1..600000 ms");
    s->wait_limit_ns = (unsigned long long)milliseconds * 1000000ull;
    return Q35K_OK;
}

int q35k_shard_reset(q35k_shard* s) {
    if (!s) return Q35K_EINVAL;
    // 1. No kernel of this process is in flight after the synchronization
    //    (every device wait is bounded).  2. One process per GPU: a barrier,
    //    so no rank's kernel can still store a flag into this rank's buffer.
    //    3. The fused gather's flags and call counters restart from zero.
    //    4. A second barrier: no rank starts its next call before every rank
    //    has cleared its buffer.
    const bool multi_process = (int)s->devices.size() != s->nranks && !s->comms.empty();
    for (size_t i = 0; i < s->devices.size(); i++) {
        cudaSetDevice(s->devices[i]);
        cudaDeviceSynchronize();
        cudaGetLastError();
    }
    char mine = 1;
    std::vector<char> all(s->nranks);
    if (multi_process) {
        const int rc = allgather_host(s, &mine, all.data(), 1);
        if (rc != Q35K_OK) return rc;
    }
    for (size_t i = 0; i < s->devices.size(); i++) {
        cudaSetDevice(s->devices[i]);
        q35k_ctx* c = s->ctxs[i];
        if (cudaMemset(c->d_err, 0, sizeof(unsigned)) != cudaSuccess ||
            (c->d_counters && cudaMemset(c->d_counters, 0, c->counters_cap) != cudaSuccess) ||
            (c->d_gcnt && cudaMemset(c->d_gcnt, 0, c->gcnt_cap) != cudaSuccess) ||
            (i < s->sym.size() && s->sym[i] && cudaMemset(s->sym[i], 0, SYM_HDR + 2 * s->sym_area) != cudaSuccess) ||
            cudaDeviceSynchronize() != cudaSuccess)
            return s->fail(Q35K_ECUDA, "shard reset: clearing the device state failed");
    }
    if (multi_process) {
        const int rc = allgather_host(s, &mine, all.data(), 1);
        if (rc != Q35K_OK) return rc;
    }
    return Q35K_OK;
}

int q35k_shard_set_trace(q35k_shard* s, int on) {
    if (!s) return Q35K_EINVAL;
    s->trace = on != 0;
    return Q35K_OK;
}

int q35k_shard_trace(q35k_shard* s, int local, uint64_t* out) {
    if (!s || !out) return Q35K_EINVAL;
    if (local < 0 || local >= (int)s->devices.size()) return s->fail(Q35K_EINVAL, "local device index out of range");
    if (!s->trace || (size_t)local >= s->sym.size() || !s->sym[local])
        return s->fail(Q35K_EINVAL, "no traced fused call on this group (q35k_shard_set_trace)");
    cudaSetDevice(s->devices[local]);
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(out, s->sym[local] + HDR_TRACE, TRACE_SLOTS * sizeof(uint64_t), cudaMemcpyDeviceToHost) != cudaSuccess)
        return s->fail(Q35K_ECUDA, "reading the trace failed");
    return Q35K_OK;
}

int q35k_shard_matmul(q35k_shard* s, const q35k_sharded_weight* w, const float* x, float* y, int tokens,
                      int gather_mode) {
    if (!s || !w || !x || !y || tokens <= 0) return Q35K_EINVAL;
    const int nloc = (int)s->devices.size();
    const size_t in_bytes = (size_t)tokens * w->n_in * sizeof(float);
    const size_t out_bytes = (size_t)tokens * w->n_out * sizeof(float);
    std::vector<const float*> dx(nloc);
    std::vector<float*> dy(nloc);
    for (int i = 0; i < nloc; i++) {
        q35k_ctx* c = s->ctxs[i];
        cudaSetDevice(s->devices[i]);
        int rc;
        if ((rc = c->ensure_dev((void**)&c->d_x, &c->x_cap, in_bytes, false)) != Q35K_OK ||
            (rc = c->ensure_host(&c->h_in, &c->h_in_cap, in_bytes)) != Q35K_OK)
            return s->fail(rc, c->err);
        std::memcpy(c->h_in, x, in_bytes);
        if (cudaMemcpyAsync(c->d_x, c->h_in, in_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
            return s->fail(Q35K_ECUDA, "H2D copy of x");
        dx[i] = c->d_x;
    }
    // The full y lands on every device; this process reads it from its first.
    for (int i = 0; i < nloc; i++) {
        q35k_ctx* c = s->ctxs[i];
        cudaSetDevice(s->devices[i]);
        int rc;
        if ((rc = c->ensure_dev((void**)&c->d_y, &c->y_cap, out_bytes, false)) != Q35K_OK) return s->fail(rc, c->err);
        dy[i] = c->d_y;
    }
    int rc = q35k_shard_matmul_dev(s, w, dx.data(), dy.data(), tokens, gather_mode, nullptr);
    if (rc != Q35K_OK) return rc;
    q35k_ctx* c0 = s->ctxs[0];
    cudaSetDevice(s->devices[0]);
    if ((rc = c0->ensure_host(&c0->h_out, &c0->h_out_cap, out_bytes)) != Q35K_OK) return s->fail(rc, c0->err);
    if (cudaMemcpyAsync(c0->h_out, c0->d_y, out_bytes, cudaMemcpyDeviceToHost, c0->stream) != cudaSuccess)
        return s->fail(Q35K_ECUDA, "D2H copy of y");
    if ((rc = q35k_shard_sync(s)) != Q35K_OK) return rc;
    std::memcpy(y, c0->h_out, out_bytes);
    return Q35K_OK;
}

int q35k_shard_info(const q35k_shard* s, int* nranks, int* first_rank, int* local_devices) {
    if (!s) return Q35K_EINVAL;
    if (nranks) *nranks = s->nranks;
    if (first_rank) *first_rank = s->first_rank;
    if (local_devices) *local_devices = (int)s->devices.size();
    return Q35K_OK;
}

}  // extern "C"
