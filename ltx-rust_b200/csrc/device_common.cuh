// Device helpers shared by the kernels: exact dtype decoders, bounded waits,
// and the sm_100a PTX wrappers (mbarrier, TMA, tcgen05) the tensor-core
// kernels are built from.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ltx_b200.h"

namespace ltx {

// ── exact decoders ──────────────────────────────────────────────────────────

// float8_e4m3fn -> f32, exact (crates/ltx-weights/src/fp8.rs:90-120).
// The 7 magnitude bits are placed in the f32 exponent/mantissa field and
// rescaled by 2^120, which lands normals and subnormals exactly (f32 keeps
// denormals here: the library is built without flush-to-zero).
__device__ __forceinline__ float dec_e4m3(uint32_t b) {
    const uint32_t em = b & 0x7Fu;
    float v = __uint_as_float(em << 20) * 0x1p120f;
    v = __uint_as_float(__float_as_uint(v) | ((b & 0x80u) << 24));
    return em == 0x7Fu ? __uint_as_float(0x7FC00000u) : v;
}

// float8_e5m2 -> f32, exact, with IEEE inf/NaN (fp8.rs:127-158).
__device__ __forceinline__ float dec_e5m2(uint32_t b) {
    const uint32_t em = b & 0x7Fu;
    float v = __uint_as_float(em << 21) * 0x1p112f;
    if ((em >> 2) == 31u) v = (em & 3u) ? __uint_as_float(0x7FC00000u) : __uint_as_float(0x7F800000u);
    return __uint_as_float(__float_as_uint(v) | ((b & 0x80u) << 24));
}

__device__ __forceinline__ float dec_bf16(uint32_t h) { return __uint_as_float(h << 16); }
__device__ __forceinline__ float dec_f16(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// Element `i` of an array of dtype `dt`, decoded exactly to f32.
__device__ __forceinline__ float load_as_f32(const void *p, int dt, int64_t i) {
    switch (dt) {
    case LTX_F32: return static_cast<const float *>(p)[i];
    case LTX_F16: return dec_f16(static_cast<const uint16_t *>(p)[i]);
    case LTX_BF16: return dec_bf16(static_cast<const uint16_t *>(p)[i]);
    case LTX_F8_E4M3: return dec_e4m3(static_cast<const uint8_t *>(p)[i]);
    default: return dec_e5m2(static_cast<const uint8_t *>(p)[i]);
    }
}

// ── bounded waits ───────────────────────────────────────────────────────────

// Every spin in this library stops after this many nanoseconds, records a
// code in the context's timeout flag and lets the kernel wind down.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// System-scope acquire load / release store of a 32-bit stamp (a word another
// GPU writes or reads over NVLink).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Stamps hold launch epochs that only grow: "reached" tolerates wrap-around.
__device__ __forceinline__ bool stamp_reached(uint32_t stamp, uint32_t epoch) { return (int32_t)(stamp - epoch) >= 0; }

// ── shared-memory barriers (mbarrier) ───────────────────────────────────────

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar`; returns false (and raises `flag`) when
// the wait exceeds kWaitLimitNs.  Once `*aborted` is set the caller's role
// stops waiting at once, so a stuck CTA winds down in bounded time.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *flag, int code, bool *aborted) {
    if (*aborted) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kWaitLimitNs) {
            if (flag) atomicExch(flag, code);
            *aborted = true;
            return false;
        }
    }
    return true;
}

// mbar_wait by every lane of a warp with one outcome for the whole warp: it
// fails (and aborts every lane) if any lane's wait failed.  Use it before
// warp-collective instructions (tcgen05.ld/st .sync.aligned), which must not
// be reached by part of a warp.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, int *flag, int code, bool *aborted) {
    const bool ok = mbar_wait(bar, parity, flag, code, aborted);
    if (__all_sync(0xffffffffu, ok)) return true;
    *aborted = true;
    return false;
}

// ── TMA ─────────────────────────────────────────────────────────────────────

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ── tcgen05 (5th-gen tensor cores, TMEM accumulators) ───────────────────────

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/f16 in, f32 accumulate).
__device__ __forceinline__ void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f8f6f4 (both operands e4m3,
// K = 32 per instruction: one 128-byte swizzle row holds 128 of them).
__device__ __forceinline__ void umma_f8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrives once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Instruction descriptor for kind::f16 with f32 accumulation, both operands
// K-major unless b_mn_major (bit layout: PTX ISA "Instruction descriptor").
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool b_mn_major = false) {
    return (1u << 4)                                   // D format f32
           | ((bf16 ? 1u : 0u) << 7)                  // A format
           | ((bf16 ? 1u : 0u) << 10)                 // B format
           | ((b_mn_major ? 1u : 0u) << 16)           // B major
           | ((uint32_t)(N >> 3) << 17)               // N / 8
           | ((uint32_t)(M >> 4) << 24);              // M / 16
}

// Instruction descriptor for kind::f8f6f4 with f32 accumulation: A and B both
// e4m3 (format code 0), K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
    return (1u << 4)                                   // D format f32
           | (0u << 7) | (0u << 10)                   // A, B format e4m3
           | ((uint32_t)(N >> 3) << 17)               // N / 8
           | ((uint32_t)(M >> 4) << 24);              // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm100 version 1.
// lbo/sbo are byte strides (multiples of 16).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;   // version
    d |= 2ull << 61;   // SWIZZLE_128B
    return d;
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets row
// (warp's lane quarter)*32 + t, columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
        "elect.sync rx|px, %1;\n\t"
        "selp.u32 %0, 1, 0, px;\n\t}"
        : "=r"(pred)
        : "r"(0xFFFFFFFFu));
    return pred != 0;
}

}  // namespace ltx
