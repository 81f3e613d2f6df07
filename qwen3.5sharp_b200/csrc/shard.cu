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
// gather of a single-process group is available.
#include "../../include/q35k.h"
#include "api_internal.h"
#include "device_common.cuh"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
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
__global__ void gather_permute_kernel(const float* __restrict__ g, float* __restrict__ y, int nranks, int tokens,
                                      int n_shard, int n_out) {
    const long long total = (long long)tokens * n_out;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / n_out), c = (int)(i % n_out);
        const int r = c / n_shard, j = c - r * n_shard;
        y[i] = g[((size_t)r * tokens + t) * n_shard + j];
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

static void destroy_shard(q35k_shard* s) {
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
    if (gather_mode != Q35K_GATHER_NCCL && gather_mode != Q35K_GATHER_PEER)
        return s->fail(Q35K_EINVAL, "gather_mode must be Q35K_GATHER_NCCL or Q35K_GATHER_PEER");
    const int nloc = (int)s->devices.size();
    const bool multi = s->nranks > 1;
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
