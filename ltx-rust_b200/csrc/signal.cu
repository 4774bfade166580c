// Device-side signalling with bounded waits: one stream (or one GPU, through a
// peer pointer) sets a 32-bit flag, another stream's work waits for it
// without a host round trip.  No reference counterpart (the reference runs
// one device, host-ordered); it is the primitive the multi-stream and
// multi-GPU paths order work with, and the way a lost peer is detected: a wait
// gives up after its limit, records a code in the context's timeout flag
// (ltx_ctx_synchronize then returns LTX_ERR_TIMEOUT) and returns, so the
// context stays usable.
#include "device_common.cuh"
#include "internal.hpp"

namespace {

constexpr int kWaitFlagCode = 0x5157;   // "wait flag" code in the context's timeout flag

__global__ void wait_flag_kernel(const int *flag, int expect, uint64_t limit_ns, int *timeout_flag) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint64_t t0 = ltx::global_ns();
    unsigned sleep_ns = 32;
    for (;;) {
        int v;
        asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v == expect) return;
        if (ltx::global_ns() - t0 > limit_ns) {
            atomicExch(timeout_flag, kWaitFlagCode);
            return;
        }
        __nanosleep(sleep_ns);
        if (sleep_ns < 4096) sleep_ns *= 2;
    }
}

__global__ void set_flag_kernel(int *flag, int value) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

}  // namespace

extern "C" int ltx_wait_flag(ltx_ctx *ctx, const int32_t *flag_dev, int32_t expect, uint32_t timeout_ms) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!flag_dev || ((uintptr_t)flag_dev & 3))
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_wait_flag: null or unaligned flag");
    const uint64_t limit_ms = timeout_ms == 0 || timeout_ms > 2000 ? 2000 : timeout_ms;
    wait_flag_kernel<<<1, 32, 0, ctx->stream>>>(flag_dev, expect, limit_ms * 1000000ull, ctx->timeout_flag);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_wait_flag");
}

extern "C" int ltx_set_flag(ltx_ctx *ctx, int32_t *flag_dev, int32_t value) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!flag_dev || ((uintptr_t)flag_dev & 3))
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_set_flag: null or unaligned flag");
    set_flag_kernel<<<1, 32, 0, ctx->stream>>>(flag_dev, value);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_set_flag");
}
