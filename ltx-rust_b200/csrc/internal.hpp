// Host-side internals shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ltx_b200.h"

namespace ltx {
// Tensor-parallel peer memory: one cudaMalloc per rank, mapped into every
// other rank of the communicator (CUDA IPC over NVLink), laid out alike on
// every rank so one offset names the same object everywhere:
//   x      f32  [rows_cap][D]                 the replicated residual stream
//   recv   bf16 [tp-1][rows_cap][D]           partial products other ranks pushed
//   tstamp u32  [tp-1][tiles_cap][4]          per-tile, per-warp arrival stamps
//   dstamp u32  [tp-1]                        "all my pushes landed" stamps
//          (+128 bytes: u32 [tp-1] rank-barrier stamps)
//   count  u32                                CTAs of the current launch done
//   xn     bf16 [rows_cap][D]                 normalised rows, gathered from their owners
//   gstamp u32  [tp-1][mblocks_cap]           per-M-block "my rows of xn landed" stamps
//   gcount u32  [mblocks_cap]                 norm blocks done per M-block (current launch)
// Stamps hold the launch epoch that wrote them; epochs only grow, so nothing
// is ever reset between launches.
constexpr int kMaxTpPeers = 8;
struct TpPeerMem {
    char *base = nullptr;            // this rank's allocation
    size_t bytes = 0;
    int64_t rows_cap = 0, D = 0, tiles_cap = 0;
    size_t recv_off = 0, tstamp_off = 0, dstamp_off = 0, count_off = 0;
    size_t xn_off = 0, gstamp_off = 0, gcount_off = 0;
    int64_t mblocks_cap = 0;
    uint32_t gepoch = 0;             // gathers of normalised rows so far (same sequence on every rank)
    uint32_t bepoch = 0;             // rank barriers so far
    char *peer[kMaxTpPeers] = {};    // every rank's allocation as mapped here (own = base)
    uint32_t epoch = 0;              // fused launches so far (the same sequence on every rank)
    int state = 0;                   // 0 not set up, 1 on, -1 off (the NCCL path runs)
};
}  // namespace ltx

struct ltx_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    std::string last_error;
    // Device word that kernels set when a bounded wait gives up (a code, 0 = fine).
    int *timeout_flag = nullptr;
    int sm_count = 0;
    // Scratch buffer grown on demand and reused by later calls on this context.
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    // Forward/step workspace (activations), grown on demand and reused.
    void *work = nullptr;
    size_t work_bytes = 0;
    // Pinned host staging for the small per-call uploads (timestep index),
    // so they do not serialise the host with the stream.
    void *pinned = nullptr;
    size_t pinned_bytes = 0;
    cudaEvent_t upload_done = nullptr;
    // Tensor-parallel communicator (an ncclComm_t), or null: one GPU.
    void *comm = nullptr;
    int tp_size = 1, tp_rank = 0;
    // Every collective of the communicator runs on comm_stream (one issue
    // order for NCCL), ordered against the context's stream by events.
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t comm_ev[2] = {nullptr, nullptr};   // [0]: stream -> comm, [1]: comm -> stream
    // CTAs of the persistent GEMMs (0 = one per SM).  Lowered while
    // collectives run beside them, so NCCL's kernels find free SMs.
    int gemm_sms = 0;
    // CFG-parallel pair (an ncclComm_t over 2 ranks), or null: this context
    // runs both passes of the CFG batch.  With it, cfg_rank 0 computes the
    // conditional pass and 1 the unconditional one, and the two velocities
    // are all-gathered once per step.
    void *cfg_comm = nullptr;
    int cfg_rank = 0;
    // Peer memory of the tensor-parallel ranks (fused projection + exchange).
    ltx::TpPeerMem pm;
};

namespace ltx {

inline int fail(ltx_ctx *ctx, int code, const char *fmt, ...) {
    if (ctx) {
        char buf[1024];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

inline int cuda_fail(ltx_ctx *ctx, cudaError_t e, const char *what) {
    return fail(ctx, LTX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Makes sure ctx->scratch holds at least `bytes`; returns a status.
int ensure_scratch(ltx_ctx *ctx, size_t bytes);
// Copies host bytes to the device through the context's pinned staging
// buffer (waits for the previous upload from that buffer to finish first).
int upload(ltx_ctx *ctx, void *dst_dev, const void *src_host, size_t bytes);

// Sum-allreduce of `count` floats in place over the context's communicator
// (a no-op without one), ordered after the work enqueued so far on the
// context's stream and before any work enqueued on it later.
int allreduce_sum(ltx_ctx *ctx, float *buf, size_t count);
int allreduce_sum_bf16(ltx_ctx *ctx, void *buf, size_t count);
// The pieces of that ordering, for callers that overlap a collective with
// compute: comm_after makes the comm stream wait for the context stream's
// work so far; allreduce_sum_bf16_async enqueues on the comm stream only;
// comm_join makes the context stream wait for the comm stream's work so far.
int comm_after(ltx_ctx *ctx);
int allreduce_sum_bf16_async(ltx_ctx *ctx, void *buf, size_t count);
int comm_join(ltx_ctx *ctx);
// Destroys (or aborts) the context's communicator.
void comm_release(ltx_ctx *ctx, bool abort);
// All-gather of `count` floats per rank over the CFG pair, on the context's
// stream: rank r's block goes to buf + r*count; the rank's own block is
// already in place.
int cfg_allgather(ltx_ctx *ctx, float *buf, size_t count);

// Tensor-parallel peer memory for `rows` x D residual rows (collective over
// the communicator when it (re)allocates; every rank calls it with the same
// shape).  *on = false when the fused path is off: one rank, more than
// kMaxTpPeers ranks, LTX_TP_EXCHANGE=nccl in the environment, or a rank that
// could not map its peers' memory (the ranks vote, so all agree).
int tp_peer_ensure(ltx_ctx *ctx, int64_t rows, int64_t D, bool *on);
void tp_peer_release(ltx_ctx *ctx);

// Message of the last failed host-only call (no context) on this thread.
inline std::string &host_error() {
    static thread_local std::string msg;
    return msg;
}
inline int host_fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    host_error() = buf;
    return code;
}

inline size_t dtype_size(int dt) {
    switch (dt) {
    case LTX_F32: return 4;
    case LTX_F16:
    case LTX_BF16: return 2;
    case LTX_F8_E4M3:
    case LTX_F8_E5M2: return 1;
    default: return 0;
    }
}

}  // namespace ltx

#define LTX_CUDA_TRY(ctx, call)                                          \
    do {                                                                 \
        cudaError_t _e = (call);                                         \
        if (_e != cudaSuccess) return ltx::cuda_fail((ctx), _e, #call);  \
    } while (0)
