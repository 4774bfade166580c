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
//                   (r x cols) in shared memory and each thread keeps a
//                   16 x 8 register tile, issuing packed FFMA2 (two
//                   independent IEEE fma.rn per instruction), so the
//                   rounding of every element is the reference's.
#include "device_common.cuh"
#include "internal.hpp"

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

template <int WDT, bool OUT_BF16>
__global__ void __launch_bounds__(256) dequant_only_kernel(MergeParams p, int64_t n) {
    const int64_t n16 = n / 16;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n16; v += stride) {
        float f[16];
        if constexpr (WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p.w) + v);
            const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t byte = (w4[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                f[j] = WDT == LTX_F8_E4M3 ? dec_e4m3(byte) : dec_e5m2(byte);
            }
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
    // tail (n not a multiple of 16)
    for (int64_t i = n16 * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        store_out(p, i, base_value(p, i));
}

__global__ void dequant_only_scalar_kernel(MergeParams p, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_out(p, i, base_value(p, i));
}

// ── delta path: FP32-FMA-bound tiled kernel ──────────────────────────────────

constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 16;
constexpr int kTileRows = kWarps * kRowsPerWarp;  // 128
constexpr int kTileCols = 256;                     // 32 lanes x 8 columns
constexpr int kRChunk = 32;                        // rank steps staged per pass

struct MergeSmem {
    float a[kRChunk][kTileCols];        // A[r][col], decoded          32 KB
    float c[kRChunk][kTileRows];        // coeff * B[row][r]            16 KB
};

template <int WDT, bool OUT_BF16>
__global__ void __launch_bounds__(kWarps * 32, 1) dequant_merge_kernel(MergeParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    MergeSmem &s = *reinterpret_cast<MergeSmem *>(smem_raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.y * kTileRows;
    const int64_t col0 = (int64_t)blockIdx.x * kTileCols;
    const int64_t my_row = row0 + warp * kRowsPerWarp;
    const int64_t my_col = col0 + lane * 8;
    const bool full_cols = my_col + 8 <= p.cols;

    // acc[i][j/2] holds columns (2j, 2j+1) of row i as a float2 for FFMA2.
    float2 acc[kRowsPerWarp][4];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int64_t r = my_row + i;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float x0 = 0.f, x1 = 0.f;
            if (r < p.rows) {
                const int64_t base = r * p.cols + my_col + 2 * j;
                if (full_cols || my_col + 2 * j < p.cols) x0 = base_value(p, base);
                if (full_cols || my_col + 2 * j + 1 < p.cols) x1 = base_value(p, base + 1);
            }
            acc[i][j] = make_float2(x0, x1);
        }
    }

    for (int d = 0; d < p.n_deltas; ++d) {
        const DeltaDev dl = p.d[d];
        for (int rc = 0; rc < dl.rank; rc += kRChunk) {
            const int nr = min(kRChunk, dl.rank - rc);
            __syncthreads();
            // Stage A[rc .. rc+nr)[col0 .. col0+256) and coeff*B[row0 .. +128)[rc .. rc+nr).
            for (int idx = threadIdx.x; idx < kRChunk * kTileCols; idx += blockDim.x) {
                const int r = idx / kTileCols, cc = idx % kTileCols;
                const int64_t gc = col0 + cc;
                s.a[r][cc] = (r < nr && gc < p.cols) ? load_as_f32(dl.a, dl.a_dt, (int64_t)(rc + r) * p.cols + gc) : 0.f;
            }
            for (int idx = threadIdx.x; idx < kRChunk * kTileRows; idx += blockDim.x) {
                const int rr = idx % kTileRows, r = idx / kTileRows;
                const int64_t gr = row0 + rr;
                // store.rs:786: coeff = self.scale * b_value (one f32 rounding)
                s.c[r][rr] = (r < nr && gr < p.rows)
                                 ? __fmul_rn(dl.coeff, load_as_f32(dl.b, dl.b_dt, gr * dl.rank + rc + r))
                                 : 0.f;
            }
            __syncthreads();
            for (int r = 0; r < nr; ++r) {
                const float4 a0 = *reinterpret_cast<const float4 *>(&s.a[r][lane * 8]);
                const float4 a1 = *reinterpret_cast<const float4 *>(&s.a[r][lane * 8 + 4]);
                const float2 av[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                                      make_float2(a1.z, a1.w)};
                float cv[kRowsPerWarp];
#pragma unroll
                for (int q = 0; q < kRowsPerWarp / 4; ++q) {
                    const float4 c4 = *reinterpret_cast<const float4 *>(&s.c[r][warp * kRowsPerWarp + 4 * q]);
                    cv[4 * q] = c4.x;
                    cv[4 * q + 1] = c4.y;
                    cv[4 * q + 2] = c4.z;
                    cv[4 * q + 3] = c4.w;
                }
#pragma unroll
                for (int i = 0; i < kRowsPerWarp; ++i) {
                    const float2 c2 = make_float2(cv[i], cv[i]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = __ffma2_rn(c2, av[j], acc[i][j]);
                }
            }
        }
    }

#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int64_t r = my_row + i;
        if (r >= p.rows) continue;
        const int64_t base = r * p.cols + my_col;
        if (p.dst_aligned16 && full_cols && ((base & 7) == 0)) {
            if constexpr (OUT_BF16) {
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(acc[i][j].x, acc[i][j].y);
                    o[j] = *reinterpret_cast<uint32_t *>(&h);
                }
                __stcs(reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.dst) + base),
                       make_uint4(o[0], o[1], o[2], o[3]));
            } else {
                float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.dst) + base);
                __stcs(dst, make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y));
                __stcs(dst + 1, make_float4(acc[i][2].x, acc[i][2].y, acc[i][3].x, acc[i][3].y));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (my_col + 2 * j < p.cols) store_out(p, base + 2 * j, acc[i][j].x);
                if (my_col + 2 * j + 1 < p.cols) store_out(p, base + 2 * j + 1, acc[i][j].y);
            }
        }
    }
}

template <int WDT>
cudaError_t launch_merge(const MergeParams &p, cudaStream_t st, int sms) {
    const size_t smem = sizeof(MergeSmem);
    const int64_t n = p.rows * p.cols;
    if (p.n_deltas == 0) {
        const bool vec = ((WDT == LTX_F8_E4M3 || WDT == LTX_F8_E5M2) ? ((uintptr_t)p.w % 16 == 0) : true) &&
                         ((uintptr_t)p.dst % 16 == 0);
        if (!vec) {
            dequant_only_scalar_kernel<<<sms * 4, 256, 0, st>>>(p, n);
            return cudaGetLastError();
        }
        const int64_t work = n / 16 + 1;
        const int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)sms * 8);
        if (p.dst_bf16)
            dequant_only_kernel<WDT, true><<<grid, 256, 0, st>>>(p, n);
        else
            dequant_only_kernel<WDT, false><<<grid, 256, 0, st>>>(p, n);
        return cudaGetLastError();
    }
    dim3 grid((unsigned)((p.cols + kTileCols - 1) / kTileCols), (unsigned)((p.rows + kTileRows - 1) / kTileRows));
    if (p.dst_bf16) {
        auto k = dequant_merge_kernel<WDT, true>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kWarps * 32, smem, st>>>(p);
    } else {
        auto k = dequant_merge_kernel<WDT, false>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<grid, kWarps * 32, smem, st>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace

// Validates and enqueues one dequant(+merge) on `stream`.
int dequant_merge(ltx_ctx *ctx, cudaStream_t stream, const void *w, int w_dt, int has_scale, float scale, int64_t rows,
                  int64_t cols, const ltx_lora_delta *deltas, int n_deltas, void *dst, int dst_dt) {
    if (!w || !dst) return fail(ctx, LTX_ERR_INVALID_ARG, "dequant_merge: null pointer");
    if (rows < 0 || cols < 0) return fail(ctx, LTX_ERR_SHAPE, "dequant_merge: negative shape");
    if (w_dt < LTX_F32 || w_dt > LTX_F8_E5M2) return fail(ctx, LTX_ERR_DTYPE, "dequant_merge: bad weight dtype %d", w_dt);
    if (dst_dt != LTX_F32 && dst_dt != LTX_BF16)
        return fail(ctx, LTX_ERR_DTYPE, "dequant_merge: output dtype must be F32 or BF16");
    if (n_deltas < 0 || n_deltas > LTX_MAX_DELTAS || (n_deltas > 0 && !deltas))
        return fail(ctx, LTX_ERR_INVALID_ARG, "dequant_merge: bad delta count %d", n_deltas);
    if (rows * cols == 0) return LTX_OK;
    MergeParams p{};
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
    cudaError_t e;
    switch (w_dt) {
    case LTX_F32: e = launch_merge<LTX_F32>(p, stream, ctx->sm_count); break;
    case LTX_F16: e = launch_merge<LTX_F16>(p, stream, ctx->sm_count); break;
    case LTX_BF16: e = launch_merge<LTX_BF16>(p, stream, ctx->sm_count); break;
    case LTX_F8_E4M3: e = launch_merge<LTX_F8_E4M3>(p, stream, ctx->sm_count); break;
    default: e = launch_merge<LTX_F8_E5M2>(p, stream, ctx->sm_count); break;
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
