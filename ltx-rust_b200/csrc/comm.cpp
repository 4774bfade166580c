// Tensor-parallel communicator of a context: NCCL, loaded at run time.
//
// The library does not link NCCL: a process that never splits a model across
// GPUs needs no NCCL at all, and a process that already has one (PyTorch
// loads its own libnccl.so.2) must use that same copy rather than a second
// one.  So the first call that needs NCCL dlopens "libnccl.so.2", preferring
// the copy already mapped into the process (RTLD_NOLOAD), and resolves the
// handful of entry points below.  nccl.h supplies only the types.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "internal.hpp"

namespace ltx {

namespace {

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    const char *(*get_error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!h) {
            api.why = std::string("cannot load libnccl.so.2: ") + (dlerror() ? dlerror() : "not found");
            return;
        }
        auto sym = [&](const char *name) { return dlsym(h, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(sym("ncclCommGetAsyncError"));
        api.get_error_string = reinterpret_cast<decltype(api.get_error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_abort && api.all_reduce &&
                 api.all_gather && api.comm_get_async_error && api.get_error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an expected entry point";
    });
    return api;
}

const char *nccl_str(ncclResult_t r) { return nccl().get_error_string ? nccl().get_error_string(r) : "?"; }

}  // namespace

int comm_after(ltx_ctx *ctx) {
    if (!ctx->comm_stream) return LTX_OK;
    LTX_CUDA_TRY(ctx, cudaEventRecord(ctx->comm_ev[0], ctx->stream));
    LTX_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->comm_stream, ctx->comm_ev[0], 0));
    return LTX_OK;
}

int comm_join(ltx_ctx *ctx) {
    if (!ctx->comm_stream) return LTX_OK;
    LTX_CUDA_TRY(ctx, cudaEventRecord(ctx->comm_ev[1], ctx->comm_stream));
    LTX_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->stream, ctx->comm_ev[1], 0));
    return LTX_OK;
}

static int allreduce_on_comm(ltx_ctx *ctx, void *buf, size_t count, ncclDataType_t dt, const char *what) {
    if (ctx->tp_size <= 1 || count == 0) return LTX_OK;
    ncclResult_t r = nccl().all_reduce(buf, buf, count, dt, ncclSum, static_cast<ncclComm_t>(ctx->comm),
                                       ctx->comm_stream ? ctx->comm_stream : ctx->stream);
    if (r != ncclSuccess) return fail(ctx, LTX_ERR_NCCL, "allreduce of %zu %s: %s", count, what, nccl_str(r));
    return LTX_OK;
}

int allreduce_sum_bf16_async(ltx_ctx *ctx, void *buf, size_t count) {
    return allreduce_on_comm(ctx, buf, count, ncclBfloat16, "bf16");
}

int allreduce_sum(ltx_ctx *ctx, float *buf, size_t count) {
    if (ctx->tp_size <= 1 || count == 0) return LTX_OK;
    if (int rc = comm_after(ctx)) return rc;
    if (int rc = allreduce_on_comm(ctx, buf, count, ncclFloat32, "floats")) return rc;
    return comm_join(ctx);
}

int allreduce_sum_bf16(ltx_ctx *ctx, void *buf, size_t count) {
    if (ctx->tp_size <= 1 || count == 0) return LTX_OK;
    if (int rc = comm_after(ctx)) return rc;
    if (int rc = allreduce_on_comm(ctx, buf, count, ncclBfloat16, "bf16")) return rc;
    return comm_join(ctx);
}

int cfg_allgather(ltx_ctx *ctx, float *buf, size_t count) {
    if (!ctx->cfg_comm || count == 0) return LTX_OK;
    ncclResult_t r = nccl().all_gather(buf + (size_t)ctx->cfg_rank * count, buf, count, ncclFloat32,
                                       static_cast<ncclComm_t>(ctx->cfg_comm), ctx->stream);
    if (r != ncclSuccess) return fail(ctx, LTX_ERR_NCCL, "CFG all-gather of %zu floats: %s", count, nccl_str(r));
    return LTX_OK;
}

// ── peer memory of the tensor-parallel ranks ────────────────────────────────

namespace {

size_t up256(size_t b) { return (b + 255) & ~size_t(255); }

// Every rank's `n` bytes, in rank order, over the communicator (through the
// context's scratch; returns once the bytes are on the host).
int allgather_host_bytes(ltx_ctx *ctx, const void *mine, size_t n, std::vector<char> &all) {
    const int R = ctx->tp_size;
    if (int rc = ensure_scratch(ctx, up256(n * R))) return rc;
    char *d = static_cast<char *>(ctx->scratch);
    LTX_CUDA_TRY(ctx, cudaMemcpyAsync(d + (size_t)ctx->tp_rank * n, mine, n, cudaMemcpyHostToDevice, ctx->stream));
    if (int rc = comm_after(ctx)) return rc;
    ncclResult_t r = nccl().all_gather(d + (size_t)ctx->tp_rank * n, d, n, ncclUint8, static_cast<ncclComm_t>(ctx->comm),
                                       ctx->comm_stream ? ctx->comm_stream : ctx->stream);
    if (r != ncclSuccess) return fail(ctx, LTX_ERR_NCCL, "all-gather of %zu bytes: %s", n, nccl_str(r));
    if (int rc = comm_join(ctx)) return rc;
    all.resize(n * R);
    LTX_CUDA_TRY(ctx, cudaMemcpyAsync(all.data(), d, n * R, cudaMemcpyDeviceToHost, ctx->stream));
    LTX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return LTX_OK;
}

void unmap_peers(TpPeerMem &pm) {
    for (int r = 0; r < kMaxTpPeers; ++r) {
        if (pm.peer[r] && pm.peer[r] != pm.base) cudaIpcCloseMemHandle(pm.peer[r]);
        pm.peer[r] = nullptr;
    }
}

}  // namespace

void tp_peer_release(ltx_ctx *ctx) {
    TpPeerMem &pm = ctx->pm;
    unmap_peers(pm);
    if (pm.base) cudaFree(pm.base);
    const uint32_t epoch = pm.epoch, gepoch = pm.gepoch, bepoch = pm.bepoch;
    pm = TpPeerMem{};
    pm.epoch = epoch;
    pm.gepoch = gepoch;
    pm.bepoch = bepoch;
}

int tp_peer_ensure(ltx_ctx *ctx, int64_t rows, int64_t D, bool *on) {
    *on = false;
    TpPeerMem &pm = ctx->pm;
    const int n = ctx->tp_size;
    if (!ctx->comm || n < 2 || n > kMaxTpPeers || pm.state == -1) return LTX_OK;
    if (pm.state == 1 && rows <= pm.rows_cap && D == pm.D) {
        *on = true;
        return LTX_OK;
    }
    // (Re)allocation, collective: every rank gets here at the same call.
    // Nothing may still write into the old memory when it goes: each rank
    // drains its work, then all unmap, then all free.
    std::vector<char> sync;
    const char one = 1;
    if (pm.base) {
        LTX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        if (int rc = allgather_host_bytes(ctx, &one, 1, sync)) return rc;
        unmap_peers(pm);
        if (int rc = allgather_host_bytes(ctx, &one, 1, sync)) return rc;
        tp_peer_release(ctx);
    }
    const char *env = getenv("LTX_TP_EXCHANGE");
    bool ok = !(env && strcmp(env, "nccl") == 0);
    TpPeerMem nm;
    nm.epoch = pm.epoch;
    nm.gepoch = pm.gepoch;
    nm.bepoch = pm.bepoch;
    nm.rows_cap = rows;
    nm.D = D;
    nm.tiles_cap = ((rows + 127) / 128) * ((D + 127) / 128);   // any tile width >= 128
    size_t off = up256((size_t)rows * D * 4);
    nm.recv_off = off;
    off += up256((size_t)(n - 1) * rows * D * 2);
    nm.tstamp_off = off;
    off += up256((size_t)(n - 1) * nm.tiles_cap * 4 * 4);
    nm.dstamp_off = off;
    off += 256;
    nm.count_off = off;
    off += 256;
    nm.mblocks_cap = (rows + 127) / 128;
    nm.xn_off = off;
    off += up256((size_t)rows * D * 2);
    nm.gstamp_off = off;
    off += up256((size_t)(n - 1) * nm.mblocks_cap * 4);
    nm.gcount_off = off;
    off += up256((size_t)nm.mblocks_cap * 4);
    nm.bytes = off;
    cudaIpcMemHandle_t h{};
    if (ok && cudaMalloc(reinterpret_cast<void **>(&nm.base), nm.bytes) != cudaSuccess) {
        cudaGetLastError();
        nm.base = nullptr;
        ok = false;
    }
    if (ok && (cudaMemsetAsync(nm.base, 0, nm.bytes, ctx->stream) != cudaSuccess ||
               cudaIpcGetMemHandle(&h, nm.base) != cudaSuccess)) {
        cudaGetLastError();
        ok = false;
    }
    std::vector<char> handles;
    if (int rc = allgather_host_bytes(ctx, &h, sizeof h, handles)) {
        if (nm.base) cudaFree(nm.base);
        return rc;
    }
    nm.peer[ctx->tp_rank] = nm.base;
    for (int r = 0; r < n && ok; ++r) {
        if (r == ctx->tp_rank) continue;
        cudaIpcMemHandle_t hr;
        memcpy(&hr, handles.data() + (size_t)r * sizeof hr, sizeof hr);
        void *mapped = nullptr;
        if (cudaIpcOpenMemHandle(&mapped, hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else {
            nm.peer[r] = static_cast<char *>(mapped);
        }
    }
    // the ranks vote: the fused path runs only if every rank mapped every peer
    const char mine = ok ? 1 : 0;
    std::vector<char> votes;
    if (int rc = allgather_host_bytes(ctx, &mine, 1, votes)) {
        unmap_peers(nm);
        if (nm.base) cudaFree(nm.base);
        return rc;
    }
    bool all_ok = true;
    for (char v : votes) all_ok = all_ok && v == 1;
    if (!all_ok) {
        unmap_peers(nm);
        if (nm.base) cudaFree(nm.base);
        pm = TpPeerMem{};
        pm.epoch = nm.epoch;
        pm.gepoch = nm.gepoch;
        pm.bepoch = nm.bepoch;
        pm.state = -1;
        return LTX_OK;
    }
    nm.state = 1;
    pm = nm;
    *on = true;
    return LTX_OK;
}

void comm_release(ltx_ctx *ctx, bool abort) {
    if (ctx->pm.base && ctx->comm && !abort) {
        // Every rank stops using the others' memory before any of it goes:
        // drain, unmap, then free (an exporter must not free before the
        // importers have unmapped).
        cudaStreamSynchronize(ctx->stream);
        std::vector<char> sync;
        const char one = 1;
        if (allgather_host_bytes(ctx, &one, 1, sync) == LTX_OK) {
            unmap_peers(ctx->pm);
            allgather_host_bytes(ctx, &one, 1, sync);
        }
    }
    tp_peer_release(ctx);
    if (ctx->cfg_comm) {
        if (abort)
            nccl().comm_abort(static_cast<ncclComm_t>(ctx->cfg_comm));
        else
            nccl().comm_destroy(static_cast<ncclComm_t>(ctx->cfg_comm));
        ctx->cfg_comm = nullptr;
        ctx->cfg_rank = 0;
    }
    if (!ctx->comm) return;
    const NcclApi &api = nccl();
    if (abort) {
        api.comm_abort(static_cast<ncclComm_t>(ctx->comm));
    } else {
        if (ctx->comm_stream) cudaStreamSynchronize(ctx->comm_stream);
        api.comm_destroy(static_cast<ncclComm_t>(ctx->comm));
    }
    ctx->comm = nullptr;
    ctx->tp_size = 1;
    ctx->tp_rank = 0;
    // Neither call blocks: resources of work still in flight (an aborted
    // collective's kernels) are released once it completes.
    if (ctx->comm_stream) cudaStreamDestroy(ctx->comm_stream);
    ctx->comm_stream = nullptr;
    for (cudaEvent_t &e : ctx->comm_ev)
        if (e) cudaEventDestroy(e), e = nullptr;
}

}  // namespace ltx

extern "C" int ltx_comm_unique_id(uint8_t *id_out, size_t len) {
    if (!id_out || len < LTX_COMM_ID_BYTES) return ltx::host_fail(LTX_ERR_INVALID_ARG, "id buffer shorter than 128 bytes");
    const auto &api = ltx::nccl();
    if (!api.ok) return ltx::host_fail(LTX_ERR_NCCL, "%s", api.why.c_str());
    ncclUniqueId id;
    ncclResult_t r = api.get_unique_id(&id);
    if (r != ncclSuccess) return ltx::host_fail(LTX_ERR_NCCL, "ncclGetUniqueId: %s", ltx::nccl_str(r));
    static_assert(sizeof(id.internal) == LTX_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, id.internal, LTX_COMM_ID_BYTES);
    return LTX_OK;
}

extern "C" int ltx_ctx_init_comm(ltx_ctx *ctx, const uint8_t *id, size_t len, int32_t nranks, int32_t rank) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!id || len < LTX_COMM_ID_BYTES || nranks < 1 || rank < 0 || rank >= nranks)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_ctx_init_comm: bad id, rank %d or size %d", rank, nranks);
    if (ctx->comm) return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "context already has a communicator");
    if (nranks == 1) return LTX_OK;
    const auto &api = ltx::nccl();
    if (!api.ok) return ltx::fail(ctx, LTX_ERR_NCCL, "%s", api.why.c_str());
    cudaSetDevice(ctx->device);
    ncclUniqueId uid;
    memcpy(uid.internal, id, LTX_COMM_ID_BYTES);
    ncclComm_t comm = nullptr;
    ncclResult_t r = api.comm_init_rank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return ltx::fail(ctx, LTX_ERR_NCCL, "ncclCommInitRank: %s", ltx::nccl_str(r));
    ctx->comm = comm;
    ctx->tp_size = nranks;
    ctx->tp_rank = rank;
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);   // hi: the greatest priority (numerically lowest)
    if (cudaStreamCreateWithPriority(&ctx->comm_stream, cudaStreamNonBlocking, hi) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->comm_ev[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->comm_ev[1], cudaEventDisableTiming) != cudaSuccess) {
        ltx::comm_release(ctx, false);
        return ltx::fail(ctx, LTX_ERR_CUDA, "ltx_ctx_init_comm: cannot create the communicator's stream");
    }
    return LTX_OK;
}

extern "C" int ltx_ctx_init_cfg_comm(ltx_ctx *ctx, const uint8_t *id, size_t len, int32_t cfg_rank) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!id || len < LTX_COMM_ID_BYTES || cfg_rank < 0 || cfg_rank > 1)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_ctx_init_cfg_comm: bad id or CFG rank %d", cfg_rank);
    if (ctx->cfg_comm) return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "context already has a CFG pair");
    const auto &api = ltx::nccl();
    if (!api.ok) return ltx::fail(ctx, LTX_ERR_NCCL, "%s", api.why.c_str());
    cudaSetDevice(ctx->device);
    ncclUniqueId uid;
    memcpy(uid.internal, id, LTX_COMM_ID_BYTES);
    ncclComm_t comm = nullptr;
    ncclResult_t r = api.comm_init_rank(&comm, 2, uid, cfg_rank);
    if (r != ncclSuccess) return ltx::fail(ctx, LTX_ERR_NCCL, "ncclCommInitRank (CFG pair): %s", ltx::nccl_str(r));
    ctx->cfg_comm = comm;
    ctx->cfg_rank = cfg_rank;
    return LTX_OK;
}

extern "C" int ltx_ctx_tp_exchange(const ltx_ctx *ctx) {
    if (!ctx || !ctx->comm || ctx->tp_size < 2) return 0;
    return ctx->pm.state == 1 ? 1 : ctx->pm.state == -1 ? 2 : 0;
}

extern "C" int ltx_ctx_comm_check(ltx_ctx *ctx) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    for (void *c : {ctx->comm, ctx->cfg_comm}) {
        if (!c) continue;
        ncclResult_t async = ncclSuccess;
        ncclResult_t r = ltx::nccl().comm_get_async_error(static_cast<ncclComm_t>(c), &async);
        if (r != ncclSuccess || async != ncclSuccess)
            return ltx::fail(ctx, LTX_ERR_NCCL, "communicator error: %s", ltx::nccl_str(r != ncclSuccess ? r : async));
    }
    return LTX_OK;
}

extern "C" void ltx_ctx_abort_comm(ltx_ctx *ctx) {
    if (ctx) ltx::comm_release(ctx, true);
}
