// ltx_ctx: device, stream, last-error text, device timeout flag, scratch.
#include <algorithm>
#include <cstring>
#include <new>

#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

int ensure_scratch(ltx_ctx *ctx, size_t bytes) {
    if (ctx->scratch_bytes >= bytes) return LTX_OK;
    if (ctx->scratch) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->scratch, bytes);
    if (e != cudaSuccess) return fail(ctx, LTX_ERR_OOM, "scratch allocation of %zu bytes: %s", bytes, cudaGetErrorString(e));
    ctx->scratch_bytes = bytes;
    return LTX_OK;
}

int upload(ltx_ctx *ctx, void *dst_dev, const void *src_host, size_t bytes) {
    if (bytes == 0) return LTX_OK;
    // The staging buffer is reused: the previous upload must have left it.
    LTX_CUDA_TRY(ctx, cudaEventSynchronize(ctx->upload_done));
    if (ctx->pinned_bytes < bytes) {
        if (ctx->pinned) cudaFreeHost(ctx->pinned);
        ctx->pinned = nullptr;
        ctx->pinned_bytes = 0;
        const size_t want = std::max<size_t>(bytes, 1 << 20);
        if (cudaHostAlloc(&ctx->pinned, want, cudaHostAllocDefault) != cudaSuccess)
            return fail(ctx, LTX_ERR_OOM, "pinned staging of %zu bytes", want);
        ctx->pinned_bytes = want;
    }
    memcpy(ctx->pinned, src_host, bytes);
    LTX_CUDA_TRY(ctx, cudaMemcpyAsync(dst_dev, ctx->pinned, bytes, cudaMemcpyHostToDevice, ctx->stream));
    LTX_CUDA_TRY(ctx, cudaEventRecord(ctx->upload_done, ctx->stream));
    return LTX_OK;
}

}  // namespace ltx

extern "C" int ltx_ctx_create(int device, void *stream, ltx_ctx **out) {
    if (!out) return LTX_ERR_INVALID_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LTX_ERR_CUDA;
    ltx_ctx *ctx = new (std::nothrow) ltx_ctx();
    if (!ctx) return LTX_ERR_OOM;
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete ctx;
        return LTX_ERR_CUDA;
    }
    cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    // The caller's stream; NULL is the CUDA default (legacy) stream, which is
    // also what PyTorch and most hosts enqueue on by default.
    ctx->stream = static_cast<cudaStream_t>(stream);
    if (cudaEventCreateWithFlags(&ctx->upload_done, cudaEventDisableTiming) != cudaSuccess ||
        cudaMalloc(&ctx->timeout_flag, sizeof(int)) != cudaSuccess ||
        cudaMemsetAsync(ctx->timeout_flag, 0, sizeof(int), ctx->stream) != cudaSuccess) {
        if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
        return LTX_ERR_CUDA;
    }
    *out = ctx;
    return LTX_OK;
}

extern "C" void ltx_ctx_destroy(ltx_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ltx::comm_release(ctx, false);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->work) cudaFree(ctx->work);
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    if (ctx->upload_done) cudaEventDestroy(ctx->upload_done);
    if (ctx->timeout_flag) cudaFree(ctx->timeout_flag);
    if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

extern "C" const char *ltx_last_error(const ltx_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

extern "C" const char *ltx_host_last_error(void) { return ltx::host_error().c_str(); }

extern "C" void *ltx_ctx_stream(const ltx_ctx *ctx) { return ctx ? static_cast<void *>(ctx->stream) : nullptr; }

extern "C" int ltx_ctx_synchronize(ltx_ctx *ctx) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return ltx::cuda_fail(ctx, e, "cudaStreamSynchronize");
    int flag = 0;
    e = cudaMemcpy(&flag, ctx->timeout_flag, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return ltx::cuda_fail(ctx, e, "reading the timeout flag");
    if (flag) {
        cudaMemset(ctx->timeout_flag, 0, sizeof(int));
        if (flag == ltx::kErrTooManyTimesteps)
            return ltx::fail(ctx, LTX_ERR_UNSUPPORTED,
                             "a forward had more than %d distinct timesteps on the device (pass them from the host: "
                             "ltx_denoise_step's mask_host)", ltx::kMaxDistinctTs);
        return ltx::fail(ctx, LTX_ERR_TIMEOUT, "a device-side wait gave up (code %d)", flag);
    }
    return LTX_OK;
}
