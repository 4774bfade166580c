// K1: FP8 (or f32/f16/bf16) dequant + stacked LoRA merge, bit-exact with
// ltx-weights WeightStore::read (crates/ltx-weights/src/store.rs:479-521)
// and LowRankDelta::add_to (store.rs:767-793).
//
// Two kernels:
//   dequant_only  — no LoRA delta: a streaming, HBM-bound decode + scale +
//                   convert, 16 input elements per thread per step.
//   dequant_merge — with deltas: each element runs the reference's sequential
//                   f32 FMA chain (rank FMAs per delta, r ascending).  That is
//                   FP32-pipe-bound, not HBM-bound: 64 FMAs per element at
//                   rank 64.  The CTA stages coeff*B (rows x r) and A
//                   (r x cols) in shared memory and each thread keeps an
//                   8 x 8 register tile of scalar IEEE fma.rn chains, so the
//                   rounding of every element is the reference's.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {
namespace {

struct DeltaDev {
    const void *a;
    const void *b;
    int rank;
    int a_dt;
    int b_dt;
    float coeff;
};

struct MergeParams {
    const void *w;
    int w_dt;
    int fp8_scaled;   // FP8 tensor with a `_scale` sibling
    float scale;
    int64_t rows, cols;
    int n_deltas;
    DeltaDev d[LTX_MAX_DELTAS];
    void *dst;
    int dst_bf16;
    int dst_aligned16;  // dst is 16-byte aligned: vector stores allowed
    int *timeout_flag;  // where a bounded wait records that it gave up (null: nowhere)
};

__device__ __forceinline__ float base_value(const MergeParams &p, int64_t idx) {
    float v = load_as_f32(p.w, p.w_dt, idx);
    // store.rs:506: scale.mul_add(v, 0.0) — also turns -0.0 into +0.0.
    return p.fp8_scaled ? __fmaf_rn(p.scale, v, 0.0f) : v;
}

__device__ __forceinline__ void store_out(const MergeParams &p, int64_t idx, float v) {
    if (p.dst_bf16)
        static_cast<__nv_bfloat16 *>(p.dst)[idx] = __float2bfloat16_rn(v);
    else
        static_cast<float *>(p.dst)[idx] = v;
}

// ── no-delta path: HBM-bound streaming kernel ────────────────────────────────

// Four FP8 bytes (byte j = element j) -> f32, exact: the hardware converts
// e4m3/e5m2 pairs to f16 (both formats are subsets of f16, NaN stays NaN,
// e5m2 infinities stay infinite), and f16 -> f32 is exact.
template <int WDT>
__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float *f) {
    uint32_t h01, h23;
    if constexpr (WDT == LTX_F8_E4M3)
        asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
            "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
            : "=r"(h01), "=r"(h23) : "r"(w));
    else
        asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
            "cvt.rn.f16x2.e5m2x2 %0, lo;\n\tcvt.rn.f16x2.e5m2x2 %1, hi;\n\t}"
            : "=r"(h01), "=r"(h23) : "r"(w));
    f[0] = __half2float(__ushort_as_half((unsigned short)(h01 & 0xFFFFu)));
    f[1] = __half2float(__ushort_as_half((unsigned short)(h01 >> 16)));
    f[2] = __half2float(__ushort_as_half((unsigned short)(h23 & 0xFFFFu)));
    f[3] = __half2float(__ushort_as_half((unsigned short)(h23 >> 16)));
}

// 16 input elements (one 16-byte FP8 load) -> decode, scale, convert, store.
template <int WDT, bool OUT_BF16>
__device__ __forceinline__ void dequant16(const MergeParams &p, int64_t v, uint4 raw) {
    float f[16];
    if constexpr (WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) {
        fp8x4_to_f32<WDT>(raw.x, f);
        fp8x4_to_f32<WDT>(raw.y, f + 4);
        fp8x4_to_f32<WDT>(raw.z, f + 8);
        fp8x4_to_f32<WDT>(raw.w, f + 12);
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = load_as_f32(p.w, WDT, v * 16 + j);
    }
    if (p.fp8_scaled) {
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = __fmaf_rn(p.scale, f[j], 0.0f);
    }
    if constexpr (OUT_BF16) {
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
            o[j] = *reinterpret_cast<uint32_t *>(&h);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(p.dst) + v * 2;
        __stcs(dst, make_uint4(o[0], o[1], o[2], o[3]));
        __stcs(dst + 1, make_uint4(o[4], o[5], o[6], o[7]));
    } else {
        float4 *dst = reinterpret_cast<float4 *>(p.dst) + v * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) __stcs(dst + j, make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]));
    }
}

// Each thread takes kDqUnroll 16-element vectors a grid-stride apart and
// issues all their loads before decoding any, so a wave of CTAs keeps the
// whole input of a 4096 x 4096 weight in flight; the launch sizes the grid
// for one such round where it fits.
constexpr int kDqUnroll = 4;

template <int WDT, bool OUT_BF16>
__global__ void __launch_bounds__(256) dequant_only_kernel(MergeParams p, int64_t n) {
    const int64_t n16 = n / 16;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.w);
    for (; v < n16; v += kDqUnroll * stride) {
        uint4 raw[kDqUnroll];
        if constexpr (WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) {
#pragma unroll
            for (int u = 0; u < kDqUnroll; ++u)
                if (v + u * stride < n16) raw[u] = __ldcs(src + v + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kDqUnroll; ++u)
            if (v + u * stride < n16) dequant16<WDT, OUT_BF16>(p, v + u * stride, raw[u]);
    }
    // tail (n not a multiple of 16)
    for (int64_t i = n16 * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        store_out(p, i, base_value(p, i));
}

// Streaming through shared memory with bulk copies: each CTA walks chunks of
// kBulkElems elements (grid-stride).  Thread 0 keeps kBulkStages chunk loads
// in flight (cp.async.bulk global -> shared, completion counted on an
// mbarrier); every thread decodes its 32 elements of the chunk from shared
// memory into an output buffer there, and thread 0 writes the buffer back
// with one bulk store.  A few large copies in flight per SM keep HBM busy
// with far fewer instructions per byte than per-thread 16-byte loads.
constexpr int kBulkElems = 8192, kBulkStages = 4;

__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_store(void *gdst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
                 "r"(bytes)
                 : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }

template <bool OUT_BF16>
constexpr size_t bulk_smem_bytes() {
    return (size_t)kBulkStages * kBulkElems * (1 + (OUT_BF16 ? 2 : 4)) + 64;
}

template <int WDT, bool OUT_BF16>
__global__ void __launch_bounds__(256) dequant_bulk_kernel(MergeParams p, int64_t nchunks, int *timeout_flag) {
    constexpr int OUT_ES = OUT_BF16 ? 2 : 4;
    constexpr uint32_t IN_BYTES = kBulkElems, OUT_BYTES = kBulkElems * OUT_ES;
    static_assert(kBulkElems == 32 * 256, "one chunk is 32 elements per thread");
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char *in = smem;                              // [stages][IN_BYTES]
    unsigned char *out = smem + kBulkStages * IN_BYTES;    // [stages][OUT_BYTES]
    uint64_t *full = reinterpret_cast<uint64_t *>(out + kBulkStages * OUT_BYTES);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    // Launched as a programmatic dependent of the previous kernel on the
    // stream: the set-up above overlaps that kernel's tail; no global memory
    // is touched before it has completed.  The next such launch (another
    // weight's dequant) may likewise start setting up as this one's CTAs drain.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    __syncthreads();
    const int64_t first = blockIdx.x, step = gridDim.x;
    const int64_t mine = first < nchunks ? (nchunks - 1 - first) / step + 1 : 0;   // this CTA's chunks
    int64_t issued = 0;
    auto issue = [&](int64_t i) {   // thread 0: the load of this CTA's i-th chunk
        const int s = (int)(i % kBulkStages);
        mbar_arrive_expect_tx(&full[s], IN_BYTES);
        bulk_load(in + s * IN_BYTES, static_cast<const uint8_t *>(p.w) + (first + i * step) * IN_BYTES, IN_BYTES,
                  &full[s]);
        issued = i + 1;
    };
    if (tid == 0)
        for (int64_t i = 0; i < mine && i < kBulkStages; ++i) issue(i);
    bool aborted = false;
    int64_t i = 0;
    for (; i < mine; ++i) {
        const int s = (int)(i % kBulkStages);
        const uint32_t ph = (uint32_t)((i / kBulkStages) & 1);
        if (tid == 0) bulk_wait_read<kBulkStages - 1>();   // the store that last used out[s] has read it
        // every thread's wait has one outcome for the block (bounded)
        if (!__syncthreads_and(mbar_wait(&full[s], ph, timeout_flag, 120, &aborted))) break;
        const uint4 *src = reinterpret_cast<const uint4 *>(in + s * IN_BYTES) + tid * 2;
        const uint4 r0 = src[0], r1 = src[1];
        const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        float f[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) fp8x4_to_f32<WDT>(w[j], f + 4 * j);
        if (p.fp8_scaled) {
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __fmaf_rn(p.scale, f[j], 0.0f);
        }
        if constexpr (OUT_BF16) {
            uint4 *dst = reinterpret_cast<uint4 *>(out + s * OUT_BYTES) + tid * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(f[8 * q + 2 * e], f[8 * q + 2 * e + 1]);
                    o[e] = *reinterpret_cast<uint32_t *>(&h);
                }
                dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        } else {
            float4 *dst = reinterpret_cast<float4 *>(out + s * OUT_BYTES) + tid * 8;
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the bulk store
        __syncthreads();
        if (tid == 0) {
            bulk_store(static_cast<unsigned char *>(p.dst) + (first + i * step) * OUT_BYTES, out + s * OUT_BYTES,
                       OUT_BYTES);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            if (i + kBulkStages < mine) issue(i + kBulkStages);   // in[s] is free: every thread has read it
        }
    }
    if (tid == 0) {
        // loads an abort left unconsumed land (bounded waits) before the CTA
        // exits, and every store completes
        bool quiet = false;
        for (int64_t j = i; j < issued; ++j)
            mbar_wait(&full[j % kBulkStages], (uint32_t)((j / kBulkStages) & 1), nullptr, 0, &quiet);
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
}

__global__ void dequant_only_scalar_kernel(MergeParams p, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_out(p, i, base_value(p, i));
}

// ── delta path: FP32-FMA-bound tiled kernel ──────────────────────────────────
//
// All deltas' (c, a) pairs form ONE chain: for delta d, rank step r,
// v = fma(coeff_d * B_d[o][r], A_d[r][i], v).  A pre-pass writes the chain as
// f32 into scratch — a32[k][cols_p] and c32[k][rows_p] (c transposed so a
// CTA's rows are contiguous for each k) — zero-padded to the tile grid, so
// the main kernel stages it with unconditional 16-byte cp.async copies.

constexpr int kWarps = 8;       // 2 (rows) x 4 (columns) warps
constexpr int kTileRows = 128;  // per warp 64 rows; per lane 8 rows (2 x 4)
constexpr int kTileCols = 128;  // per warp 32 columns; per lane 8 columns (2 x 4)
constexpr int kRChunk = 32;     // chain steps per stage

// Thread -> element map of the 128 x 128 tile.  Lanes form 8 row groups x 4
// column groups, so per chain step a warp's shared loads are one contiguous
// 128-byte piece of coeff*B (2 float4) and one 64-byte piece of A (2 float4):
// one LSU wavefront each.
//   rows: wr*64 + 32*j + 4*lr + e   (j < 2, e < 4; register row 4j + e)
//   cols: wc*32 + 16*k + 4*lc + e   (k < 2, e < 4)
// Each element's chain runs as scalar IEEE fma.rn (on this B200 scalar FFMA
// measured 122 FMA/clk/SM against 103-111 for packed FFMA2, and needs no
// duplicated operand pairs).
struct MergeSmem {
    float a[2][kRChunk][kTileCols];    // A chain rows       32 KB
    float c[2][kRChunk][kTileRows];    // coeff*B            32 KB
    uint8_t w8[kTileRows][kTileCols];  // FP8 base tile, 16-byte chunks swizzled by (row >> 2) & 7  16 KB
};   // 80 KB: two CTAs per SM (registers allow two)

struct ChainMap {
    int n;                      // deltas
    int start[LTX_MAX_DELTAS];  // first chain index of each delta
};

// One chain step k per grid row (blockIdx.y): x < cols_p writes A's row,
// the next rows_p x write coeff*B's column.
__global__ void merge_prepass_kernel(MergeParams p, ChainMap cm, float *a32, float *c32, int64_t cols_p,
                                     int64_t rows_p) {
    const int k = blockIdx.y;
    int d = 0;
#pragma unroll
    for (int i = 1; i < LTX_MAX_DELTAS; ++i) d += (i < cm.n && k >= cm.start[i]);
    const DeltaDev dl = p.d[d];
    const int r = k - cm.start[d];
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t x = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; x < cols_p + rows_p; x += stride) {
        if (x < cols_p) {
            a32[(int64_t)k * cols_p + x] = x < p.cols ? load_as_f32(dl.a, dl.a_dt, (int64_t)r * p.cols + x) : 0.f;
        } else {
            const int64_t o = x - cols_p;
            // store.rs:786: coeff = self.scale * b_value (one f32 rounding)
            c32[(int64_t)k * rows_p + o] = o < p.rows ? __fmul_rn(dl.coeff, load_as_f32(dl.b, dl.b_dt, o * dl.rank + r)) : 0.f;
        }
    }
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int WDT>
__device__ __forceinline__ float base_t(const MergeParams &p, int64_t idx) {
    float v = load_as_f32(p.w, WDT, idx);
    return p.fp8_scaled ? __fmaf_rn(p.scale, v, 0.0f) : v;
}

// One 128 x 128 tile at (row0, col0).  FULL: the common case, specialised
// without the ragged paths — an FP8 base staged whole (base_vec), a chain of
// whole 32-step chunks, every row and column inside the tensor, a 16-byte
// aligned output.
template <int WDT, bool OUT_BF16, bool FULL>
__device__ __forceinline__ void merge_tile(const MergeParams &p, MergeSmem &s, const float *__restrict__ a32,
                                           const float *__restrict__ c32, int ktot, int64_t cols_p, int64_t rows_p,
                                           int base_vec, int64_t row0, int64_t col0) {
    constexpr int TCW = kTileCols;
    constexpr int NCG = 2;   // 16-column groups per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wr = warp >> 2, wc = warp & 3, lr = lane >> 2, lc = lane & 3;
    const int trow = wr * 64 + 4 * lr;         // + 32j + e
    const int tcol = wc * 32 + 4 * lc;   // + 16k + e
    const int nchunks = (ktot + kRChunk - 1) / kRChunk;

    auto issue = [&](int chunk, int buf) {
        const int k0 = chunk * kRChunk;
        for (int q = threadIdx.x; q < kRChunk * TCW / 4; q += blockDim.x) {
            const int r = q / (TCW / 4), c4 = q % (TCW / 4);
            const int k = FULL ? k0 + r : min(k0 + r, ktot - 1);   // rows past the chain end are never read
            cp_async16(&s.a[buf][r][c4 * 4], a32 + (int64_t)k * cols_p + col0 + c4 * 4);
        }
        for (int q = threadIdx.x; q < kRChunk * kTileRows / 4; q += blockDim.x) {
            const int r = q / (kTileRows / 4), c4 = q % (kTileRows / 4);
            const int k = FULL ? k0 + r : min(k0 + r, ktot - 1);
            cp_async16(&s.c[buf][r][c4 * 4], c32 + (int64_t)k * rows_p + row0 + c4 * 4);
        }
    };
    // Group 0: the FP8 base tile (full, aligned tiles only) and chain chunk 0.
    if (FULL || base_vec) {
        for (int q = threadIdx.x; q < kTileRows * TCW / 16; q += blockDim.x) {
            const int rr = q / (TCW / 16), c16 = q % (TCW / 16);
            cp_async16(&s.w8[rr][(c16 ^ ((rr >> 2) & 7)) * 16],
                       static_cast<const uint8_t *>(p.w) + (row0 + rr) * p.cols + col0 + c16 * 16);
        }
    }
    issue(0, 0);
    cp_async_commit();

    float acc[8][4 * NCG];   // [row 4j + e][column 4k + e']
    if (FULL || base_vec) {
        // FP8 only: decode the staged base tile.
        cp_async_wait<0>();
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int rr = trow + 32 * (i >> 2) + (i & 3);
#pragma unroll
            for (int k = 0; k < NCG; ++k) {
                const int cc = tcol + 16 * k;
                const uint32_t w4 =
                    *reinterpret_cast<const uint32_t *>(&s.w8[rr][(((cc >> 4) ^ ((rr >> 2) & 7)) << 4) | (cc & 15)]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t b = (w4 >> (8 * e)) & 0xFFu;
                    float x = WDT == LTX_F8_E4M3 ? dec_e4m3(b) : dec_e5m2(b);
                    if (p.fp8_scaled) x = __fmaf_rn(p.scale, x, 0.0f);
                    acc[i][4 * k + e] = x;
                }
            }
        }
    } else if constexpr (!FULL) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t r = row0 + trow + 32 * (i >> 2) + (i & 3);
#pragma unroll
            for (int k = 0; k < NCG; ++k) {
                const int64_t c = col0 + tcol + 16 * k;
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    acc[i][4 * k + e] = (r < p.rows && c + e < p.cols) ? base_t<WDT>(p, r * p.cols + c + e) : 0.f;
            }
        }
    }

    for (int ch = 0; ch < nchunks; ++ch) {
        const int buf = ch & 1;
        if (!FULL && !base_vec) {
            if (ch + 1 < nchunks) {
                issue(ch + 1, buf ^ 1);
                cp_async_commit();
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
        } else {
            cp_async_wait<0>();   // chunk ch (the only group in flight) has landed
        }
        // One barrier per chunk: past it every thread's copies of chunk ch have
        // landed and every thread has finished chunk ch-1, so the other buffer
        // can be refilled with chunk ch+1 under this chunk's FMAs.
        __syncthreads();
        if ((FULL || base_vec) && ch + 1 < nchunks) {
            issue(ch + 1, buf ^ 1);
            cp_async_commit();
        }
        const int nr = FULL ? kRChunk : min(kRChunk, ktot - ch * kRChunk);
        // Chain step r for this thread's 8 x 4*NCG elements: v = fma(c_row, a_col, v).
        auto step = [&](int r) {
            float av[4 * NCG], cv[8];
#pragma unroll
            for (int k = 0; k < NCG; ++k) {
                const float4 a4 = *reinterpret_cast<const float4 *>(&s.a[buf][r][tcol + 16 * k]);
                av[4 * k] = a4.x, av[4 * k + 1] = a4.y, av[4 * k + 2] = a4.z, av[4 * k + 3] = a4.w;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float4 c4 = *reinterpret_cast<const float4 *>(&s.c[buf][r][trow + 32 * j]);
                cv[4 * j] = c4.x, cv[4 * j + 1] = c4.y, cv[4 * j + 2] = c4.z, cv[4 * j + 3] = c4.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int q = 0; q < 4 * NCG; ++q) acc[i][q] = __fmaf_rn(cv[i], av[q], acc[i][q]);
        };
        if (nr == kRChunk) {
#pragma unroll 2
            for (int r = 0; r < kRChunk; ++r) step(r);
        } else {
            for (int r = 0; r < nr; ++r) step(r);
        }
        if (!FULL && !base_vec) __syncthreads();   // buffer `buf` is refilled at the top of the next chunk
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t r = row0 + trow + 32 * (i >> 2) + (i & 3);
        if (!FULL && r >= p.rows) continue;
#pragma unroll
        for (int k = 0; k < NCG; ++k) {
            const int64_t c = col0 + tcol + 16 * k;
            const int64_t base = r * p.cols + c;
            const float *v = &acc[i][4 * k];
            if (FULL || (p.dst_aligned16 && c + 4 <= p.cols && (base & 3) == 0)) {
                if constexpr (OUT_BF16) {
                    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
                    __stcs(reinterpret_cast<uint2 *>(static_cast<__nv_bfloat16 *>(p.dst) + base),
                           make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1)));
                } else {
                    __stcs(reinterpret_cast<float4 *>(static_cast<float *>(p.dst) + base),
                           make_float4(v[0], v[1], v[2], v[3]));
                }
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (c + e < p.cols) store_out(p, base + e, v[e]);
            }
        }
    }
}

template <int WDT, bool OUT_BF16, bool FULL>
__global__ void __launch_bounds__(kWarps * 32, 2)
    dequant_merge_kernel(MergeParams p, const float *__restrict__ a32, const float *__restrict__ c32, int ktot,
                         int64_t cols_p, int64_t rows_p, int base_vec, int tiles_x) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    MergeSmem &s = *reinterpret_cast<MergeSmem *>(smem_raw);
    const int t = blockIdx.x;
    merge_tile<WDT, OUT_BF16, FULL>(p, s, a32, c32, ktot, cols_p, rows_p, base_vec, (int64_t)(t / tiles_x) * kTileRows,
                                    (int64_t)(t % tiles_x) * kTileCols);
}

// Bytes of chain scratch the delta path needs for this call (0 without deltas).
size_t merge_scratch_bytes(const MergeParams &p) {
    if (p.n_deltas == 0) return 0;
    int64_t ktot = 0;
    for (int d = 0; d < p.n_deltas; ++d) ktot += p.d[d].rank;
    const int64_t cols_p = (p.cols + kTileCols - 1) / kTileCols * kTileCols;
    const int64_t rows_p = (p.rows + kTileRows - 1) / kTileRows * kTileRows;
    return (size_t)(ktot * (cols_p + rows_p)) * sizeof(float);
}

template <int WDT>
cudaError_t launch_merge(const MergeParams &p, cudaStream_t st, int sms, void *scratch) {
    const size_t smem = sizeof(MergeSmem);
    const int64_t n = p.rows * p.cols;
    if (p.n_deltas == 0) {
        const bool vec = ((WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) ? ((uintptr_t)p.w % 16 == 0) : true) &&
                         ((uintptr_t)p.dst % 16 == 0);
        if (!vec) {
            dequant_only_scalar_kernel<<<sms * 4, 256, 0, st>>>(p, n);
            return cudaGetLastError();
        }
        // one unrolled round per thread where it fits in one wave of resident CTAs
        if ((WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) && n % kBulkElems == 0) {
            const int64_t nchunks = n / kBulkElems;
            auto k = p.dst_bf16 ? dequant_bulk_kernel<WDT, true> : dequant_bulk_kernel<WDT, false>;
            const size_t bsm = p.dst_bf16 ? bulk_smem_bytes<true>() : bulk_smem_bytes<false>();
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm);
            if (e != cudaSuccess) return e;
            const int per_sm = p.dst_bf16 ? 2 : 1;   // CTAs that fit one SM's shared memory
            const int grid = (int)std::min<int64_t>(nchunks, (int64_t)sms * per_sm);
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(grid);
            cfg.blockDim = dim3(256);
            cfg.dynamicSmemBytes = bsm;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            return cudaLaunchKernelEx(&cfg, k, p, nchunks, p.timeout_flag);
        }
        static int per_sm[2][2] = {{0, 0}, {0, 0}};   // [e5m2][bf16 out], filled once
        int &resident = per_sm[WDT == LTX_F8_E5M2][p.dst_bf16 ? 1 : 0];
        if (!resident) {
            int nb = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &nb, p.dst_bf16 ? dequant_only_kernel<WDT, true> : dequant_only_kernel<WDT, false>, 256, 0);
            resident = std::max(nb, 1);
        }
        const int64_t work = (n / 16 + kDqUnroll - 1) / kDqUnroll + 1;   // threads for one unrolled round
        const int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)sms * resident);
        if (p.dst_bf16)
            dequant_only_kernel<WDT, true><<<grid, 256, 0, st>>>(p, n);
        else
            dequant_only_kernel<WDT, false><<<grid, 256, 0, st>>>(p, n);
        return cudaGetLastError();
    }
    // Chain scratch: a32[ktot][cols_p] + c32[ktot][rows_p], f32, zero padded.
    ChainMap cm{};
    cm.n = p.n_deltas;
    int ktot = 0;
    for (int d = 0; d < p.n_deltas; ++d) {
        cm.start[d] = ktot;
        ktot += p.d[d].rank;
    }
    const int64_t cols_p = (p.cols + kTileCols - 1) / kTileCols * kTileCols;
    const int64_t rows_p = (p.rows + kTileRows - 1) / kTileRows * kTileRows;
    float *a32 = static_cast<float *>(scratch);
    float *c32 = a32 + (int64_t)ktot * cols_p;
    const int base_vec = (WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) && p.cols % kTileCols == 0 &&
                         p.rows % kTileRows == 0 && (uintptr_t)p.w % 16 == 0;
    if (ktot > 65535) return cudaErrorInvalidConfiguration;   // one grid row per chain step
    {
        const int64_t gx = std::min<int64_t>((cols_p + rows_p + 255) / 256, std::max<int64_t>(1, 8 * sms / ktot));
        merge_prepass_kernel<<<dim3((unsigned)gx, (unsigned)ktot), 256, 0, st>>>(p, cm, a32, c32, cols_p, rows_p);
    }
    const int64_t tiles_x = cols_p / kTileCols, ntiles = tiles_x * (rows_p / kTileRows);
    if (ntiles > INT32_MAX) return cudaErrorInvalidConfiguration;
    const bool full = base_vec && ktot % kRChunk == 0 && p.dst_aligned16;
    auto launch = [&](auto k) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<(unsigned)ntiles, kWarps * 32, smem, st>>>(p, a32, c32, ktot, cols_p, rows_p, base_vec, (int)tiles_x);
        return cudaSuccess;
    };
    cudaError_t e;
    if (p.dst_bf16)
        e = full ? launch(dequant_merge_kernel<WDT, true, true>) : launch(dequant_merge_kernel<WDT, true, false>);
    else
        e = full ? launch(dequant_merge_kernel<WDT, false, true>) : launch(dequant_merge_kernel<WDT, false, false>);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace

// rows * cols without int64 overflow, and small enough (2^48 elements) that
// every byte count derived from it stays in range.
static bool merge_shape_fits(int64_t rows, int64_t cols) {
    constexpr int64_t kMaxElements = int64_t(1) << 48;
    return rows == 0 || cols == 0 || rows <= kMaxElements / cols;
}

// Validates and enqueues one dequant(+merge) on `stream`.
int dequant_merge(ltx_ctx *ctx, cudaStream_t stream, const void *w, int w_dt, int has_scale, float scale, int64_t rows,
                  int64_t cols, const ltx_lora_delta *deltas, int n_deltas, void *dst, int dst_dt) {
    if (!w || !dst) return fail(ctx, LTX_ERR_INVALID_ARG, "dequant_merge: null pointer");
    if (rows < 0 || cols < 0) return fail(ctx, LTX_ERR_SHAPE, "dequant_merge: negative shape");
    if (!merge_shape_fits(rows, cols))
        return fail(ctx, LTX_ERR_SHAPE, "dequant_merge: %lld x %lld elements exceed 2^48", (long long)rows,
                    (long long)cols);
    if (w_dt < LTX_F32 || w_dt > LTX_F8_E5M2) return fail(ctx, LTX_ERR_DTYPE, "dequant_merge: bad weight dtype %d", w_dt);
    if (dst_dt != LTX_F32 && dst_dt != LTX_BF16)
        return fail(ctx, LTX_ERR_DTYPE, "dequant_merge: output dtype must be F32 or BF16");
    if (n_deltas < 0 || n_deltas > LTX_MAX_DELTAS || (n_deltas > 0 && !deltas))
        return fail(ctx, LTX_ERR_INVALID_ARG, "dequant_merge: bad delta count %d", n_deltas);
    if (rows * cols == 0) return LTX_OK;
    MergeParams p{};
    p.timeout_flag = ctx->timeout_flag;
    p.w = w;
    p.w_dt = w_dt;
    p.fp8_scaled = (w_dt == LTX_F8_E4M3 || w_dt == LTX_F8_E5M2) && has_scale;
    p.scale = scale;
    p.rows = rows;
    p.cols = cols;
    p.n_deltas = n_deltas;
    for (int i = 0; i < n_deltas; ++i) {
        const ltx_lora_delta &d = deltas[i];
        if (!d.a_dev || !d.b_dev || d.rank <= 0)
            return fail(ctx, LTX_ERR_SHAPE, "dequant_merge: delta %d has rank %d or a null factor", i, d.rank);
        if (d.a_dtype < LTX_F32 || d.a_dtype > LTX_F8_E5M2 || d.b_dtype < LTX_F32 || d.b_dtype > LTX_F8_E5M2)
            return fail(ctx, LTX_ERR_DTYPE, "dequant_merge: delta %d has an unsupported dtype", i);
        p.d[i] = DeltaDev{d.a_dev, d.b_dev, d.rank, d.a_dtype, d.b_dtype, d.coeff};
    }
    p.dst = dst;
    p.dst_bf16 = dst_dt == LTX_BF16;
    p.dst_aligned16 = ((uintptr_t)dst % 16) == 0;
    const size_t need = merge_scratch_bytes(p);
    if (need) {
        int rc = ensure_scratch(ctx, need);
        if (rc != LTX_OK) return rc;
    }
    cudaError_t e;
    switch (w_dt) {
    case LTX_F32: e = launch_merge<LTX_F32>(p, stream, ctx->sm_count, ctx->scratch); break;
    case LTX_F16: e = launch_merge<LTX_F16>(p, stream, ctx->sm_count, ctx->scratch); break;
    case LTX_BF16: e = launch_merge<LTX_BF16>(p, stream, ctx->sm_count, ctx->scratch); break;
    case LTX_F8_E4M3: e = launch_merge<LTX_F8_E4M3>(p, stream, ctx->sm_count, ctx->scratch); break;
    default: e = launch_merge<LTX_F8_E5M2>(p, stream, ctx->sm_count, ctx->scratch); break;
    }
    if (e != cudaSuccess) return cuda_fail(ctx, e, "dequant_merge launch");
    return LTX_OK;
}

}  // namespace ltx

extern "C" float ltx_lora_coeff(float strength, float alpha, int32_t rank) {
    // store.rs:615: strength.mul_add(alpha / rank as f32, 0.0)
    return fmaf(strength, alpha / (float)rank, 0.0f);
}

extern "C" int ltx_dequant_merge(ltx_ctx *ctx, const void *w_dev, int32_t w_dtype, int32_t has_scale, float scale,
                                 int64_t out_features, int64_t in_features, const ltx_lora_delta *deltas,
                                 int32_t n_deltas, void *dst_dev, int32_t dst_dtype) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    return ltx::dequant_merge(ctx, ctx->stream, w_dev, w_dtype, has_scale, scale, out_features, in_features, deltas,
                              n_deltas, dst_dev, dst_dtype);
}

// ── allocation-free entry point ──────────────────────────────────────────────
//
// For callers that cannot call cudaMalloc: code running inside a memory pool
// or a host framework that owns every device allocation, or a process that
// must not allocate after start-up (a real-time pipeline, or a sandbox whose
// device allocator is closed).  Those callers bring their own input and output
// buffers; the only extra device memory the merge needs is its chain scratch
// (all stacked LoRA deltas' A rows and coeff*B columns as f32, zero-padded to
// the tile grid), which here lives in one fixed file-scope device array
// instead of a cudaMalloc'd buffer.
//
//   * Size: kNoAllocScratchBytes (16 MiB) on every GPU that loads this
//     library, held until the process exits.  A call needs
//       4 * (sum of ranks) * (round_up(in, 128) + round_up(out, 128)) bytes;
//     rank 64 fits every weight of the 22B DiT (the largest, the 24576 x 4096
//     adaLN projection, needs 7.3 MB).  Larger calls are rejected with
//     LTX_ERR_UNSUPPORTED before anything is enqueued.
//   * Sharing: every call on a device uses the same array.  The kernels write
//     every scratch element they later read, so nothing has to start at zero,
//     but two calls whose work overlaps on the GPU (different streams, or the
//     same array used from two host threads with no ordering) race on it.
//   * Set-up: the first call on each device resolves the array's device
//     address with cudaGetSymbolAddress (with that device current) and caches
//     it.  Make that first call before any stream capture.  The cached address
//     belongs to the device's primary context: after cudaDeviceReset (which
//     destroys that context and the array with it) this entry point must not
//     be called again in the process.
namespace ltx {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_merge_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_addr[kMaxDevices] = {};

void set_err(char *buf, size_t len, const char *fmt, ...) {
    if (!buf || !len) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, len, fmt, ap);
    va_end(ap);
}

}  // namespace
}  // namespace ltx

extern "C" int ltx_dequant_merge_noalloc(void *stream, const void *w_dev, int32_t w_dtype, int32_t has_scale,
                                         float scale, int64_t out_features, int64_t in_features,
                                         const ltx_lora_delta *deltas, int32_t n_deltas, void *dst_dev,
                                         int32_t dst_dtype, char *errbuf, size_t errbuf_len) {
    using namespace ltx;
    if (errbuf && errbuf_len) errbuf[0] = 0;
    if (!w_dev || !dst_dev) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: null pointer");
        return LTX_ERR_INVALID_ARG;
    }
    if (out_features < 0 || in_features < 0) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: negative shape");
        return LTX_ERR_SHAPE;
    }
    if (!merge_shape_fits(out_features, in_features)) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: %lld x %lld elements exceed 2^48",
                (long long)out_features, (long long)in_features);
        return LTX_ERR_SHAPE;
    }
    if (w_dtype < LTX_F32 || w_dtype > LTX_F8_E5M2) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: bad weight dtype %d", w_dtype);
        return LTX_ERR_DTYPE;
    }
    if (dst_dtype != LTX_F32 && dst_dtype != LTX_BF16) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: output dtype must be F32 or BF16");
        return LTX_ERR_DTYPE;
    }
    if (n_deltas < 0 || n_deltas > LTX_MAX_DELTAS || (n_deltas > 0 && !deltas)) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: bad delta count %d", n_deltas);
        return LTX_ERR_INVALID_ARG;
    }
    if (out_features * in_features == 0) return LTX_OK;
    MergeParams p{};
    p.w = w_dev;
    p.w_dt = w_dtype;
    p.fp8_scaled = (w_dtype == LTX_F8_E4M3 || w_dtype == LTX_F8_E5M2) && has_scale;
    p.scale = scale;
    p.rows = out_features;
    p.cols = in_features;
    p.n_deltas = n_deltas;
    for (int i = 0; i < n_deltas; ++i) {
        const ltx_lora_delta &d = deltas[i];
        if (!d.a_dev || !d.b_dev || d.rank <= 0) {
            set_err(errbuf, errbuf_len, "dequant_merge_noalloc: delta %d has rank %d or a null factor", i, d.rank);
            return LTX_ERR_SHAPE;
        }
        if (d.a_dtype < LTX_F32 || d.a_dtype > LTX_F8_E5M2 || d.b_dtype < LTX_F32 || d.b_dtype > LTX_F8_E5M2) {
            set_err(errbuf, errbuf_len, "dequant_merge_noalloc: delta %d has an unsupported dtype", i);
            return LTX_ERR_DTYPE;
        }
        p.d[i] = DeltaDev{d.a_dev, d.b_dev, d.rank, d.a_dtype, d.b_dtype, d.coeff};
    }
    p.dst = dst_dev;
    p.dst_bf16 = dst_dtype == LTX_BF16;
    p.dst_aligned16 = ((uintptr_t)dst_dev % 16) == 0;
    const size_t need = merge_scratch_bytes(p);
    if (need > kNoAllocScratchBytes) {
        set_err(errbuf, errbuf_len,
                "dequant_merge_noalloc: this merge needs %zu bytes of scratch; the allocation-free entry point has "
                "%zu (4 * total rank * (round_up(in,128) + round_up(out,128)))",
                need, kNoAllocScratchBytes);
        return LTX_ERR_UNSUPPORTED;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: no usable current device");
        return LTX_ERR_CUDA;
    }
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            // A host-side stand-in names the array here; the device address
            // comes from the runtime, with `dev` current.
            e = cudaGetSymbolAddress(&g_scratch_addr[dev], g_merge_scratch);
            if (e != cudaSuccess) {
                g_scratch_addr[dev] = nullptr;
                set_err(errbuf, errbuf_len, "dequant_merge_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
                return LTX_ERR_CUDA;
            }
        }
        scratch = g_scratch_addr[dev];
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc: %s", cudaGetErrorString(e));
        return LTX_ERR_CUDA;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (w_dtype) {
    case LTX_F32: e = launch_merge<LTX_F32>(p, st, sms, scratch); break;
    case LTX_F16: e = launch_merge<LTX_F16>(p, st, sms, scratch); break;
    case LTX_BF16: e = launch_merge<LTX_BF16>(p, st, sms, scratch); break;
    case LTX_F8_E4M3: e = launch_merge<LTX_F8_E4M3>(p, st, sms, scratch); break;
    default: e = launch_merge<LTX_F8_E5M2>(p, st, sms, scratch); break;
    }
    if (e != cudaSuccess) {
        set_err(errbuf, errbuf_len, "dequant_merge_noalloc launch: %s", cudaGetErrorString(e));
        return LTX_ERR_CUDA;
    }
    return LTX_OK;
}
