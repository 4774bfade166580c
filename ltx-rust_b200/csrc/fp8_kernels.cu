// Producers of the FP8 (e4m3) GEMM operands for the model's FP8 path:
// every projection input is quantised per row (token) with scale
// amax(row) / 448, which the GEMM epilogue multiplies back.  HBM-bound
// streaming kernels; each writes 1 byte per element plus one f32 per row.
//   norm_mod_e4m3          RMSNorm / adaLN modulate (norm.rs:23-53,
//                          block.rs:131-132, :150-151) straight to e4m3
//   quantize_rows_e4m3     bf16 rows (attention output, GELU output, context)
//   bf16_to_f32, scale_pad_bf16    load-time helpers for the LoRA factors
#include <cuda_fp8.h>

#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

namespace {

constexpr float kE4M3Max = 448.0f;

__device__ __forceinline__ float warp_max_all(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_add_all(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// four floats -> four e4m3 bytes (round to nearest even, saturating)
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return lo | (hi << 16);
}

// norm_mod (same modes as norm_mod_kernel) for D = 4096, two warps per row,
// then e4m3 with the row's scale: out[row] = q, scale[row] = amax / 448.
__global__ void __launch_bounds__(256) norm_mod_e4m3_kernel(const float *x, int64_t ldx, int rows, float eps, int mode,
                                                            const float *tab, int tab_coeff, const int *idx,
                                                            int k_shift, uint8_t *out, int64_t ldo, float *scale) {
    constexpr int D = 4096, SPLIT = 2, NV = D / 128 / SPLIT, RPB = 8 / SPLIT;
    __shared__ float part[3][8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rib = warp / SPLIT, piece = warp % SPLIT;
    const int row = blockIdx.x * RPB + rib;
    const bool live = row < rows;
    const int col0 = piece * (D / SPLIT);
    float4 v[NV];
    if (live) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)row * ldx + col0);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    } else {
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean = 0.f;
    if (mode == 2) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        s = warp_add_all(s);
        if (lane == 0) part[0][warp] = s;
        __syncthreads();
        mean = (part[0][rib * SPLIT] + part[0][rib * SPLIT + 1]) / (float)D;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_add_all(ss);
    if (lane == 0) part[1][warp] = ss;
    __syncthreads();
    const float denom = sqrtf((part[1][rib * SPLIT] + part[1][rib * SPLIT + 1]) / (float)D + eps);
    const float4 *sh = nullptr, *sc = nullptr;
    if (mode != 0 && live) {
        const int u = idx ? idx[row] : 0;
        const float *shift = tab + ((int64_t)u * tab_coeff + k_shift) * D + col0;
        sh = reinterpret_cast<const float4 *>(shift);
        sc = reinterpret_cast<const float4 *>(shift + D);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float a = v[i].x / denom, b = v[i].y / denom, c = v[i].z / denom, d = v[i].w / denom;
        if (mode != 0 && live) {
            const float4 s4 = __ldg(sc + lane + 32 * i), h4 = __ldg(sh + lane + 32 * i);
            a = a * (s4.x + 1.0f) + h4.x;
            b = b * (s4.y + 1.0f) + h4.y;
            c = c * (s4.z + 1.0f) + h4.z;
            d = d * (s4.w + 1.0f) + h4.w;
        }
        v[i] = make_float4(a, b, c, d);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(a), fabsf(b)), fmaxf(fabsf(c), fabsf(d))));
    }
    amax = warp_max_all(amax);
    if (lane == 0) part[2][warp] = amax;
    __syncthreads();
    if (!live) return;
    amax = fmaxf(part[2][rib * SPLIT], part[2][rib * SPLIT + 1]);
    const float s = amax > 0.f ? amax / kE4M3Max : 1.0f;
    const float inv = amax > 0.f ? kE4M3Max / amax : 0.0f;
    uint32_t *o = reinterpret_cast<uint32_t *>(out + (int64_t)row * ldo + col0);
#pragma unroll
    for (int i = 0; i < NV; ++i) o[lane + 32 * i] = pack_e4m3x4(v[i].x * inv, v[i].y * inv, v[i].z * inv, v[i].w * inv);
    if (piece == 0 && lane == 0) scale[row] = s;
}

// One block per row of `cols` bf16 values (cols % 8 == 0): pass 1 the row's
// amax, pass 2 (from L1/L2) the e4m3 bytes.
__global__ void __launch_bounds__(256) quantize_rows_e4m3_kernel(const __nv_bfloat16 *in, int64_t ldi, int rows,
                                                                 int cols, uint8_t *out, int64_t ldo, float *scale) {
    __shared__ float red[8];
    const int row = blockIdx.x;
    if (row >= rows) return;
    const uint4 *ir = reinterpret_cast<const uint4 *>(in + (int64_t)row * ldi);
    const int n8 = cols / 8;
    float amax = 0.f;
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
        const uint4 u = ir[i];
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h[q]);
            amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    amax = warp_max_all(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) amax = fmaxf(amax, red[w]);
    const float inv = amax > 0.f ? kE4M3Max / amax : 0.0f;
    uint2 *orow = reinterpret_cast<uint2 *>(out + (int64_t)row * ldo);
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
        const uint4 u = ir[i];
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
        const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
        const float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
        orow[i] = make_uint2(pack_e4m3x4(f0.x * inv, f0.y * inv, f1.x * inv, f1.y * inv),
                             pack_e4m3x4(f2.x * inv, f2.y * inv, f3.x * inv, f3.y * inv));
    }
    if (threadIdx.x == 0) scale[row] = amax > 0.f ? amax / kE4M3Max : 1.0f;
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16 *in, int64_t n, float *out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __bfloat162float(in[i]);
}

// out[r][c] = bf16(in[r][c] * mul) for c < cols_in, 0 for cols_in <= c < cols_out
__global__ void scale_pad_bf16_kernel(const __nv_bfloat16 *in, int rows, int cols_in, int cols_out, float mul,
                                      __nv_bfloat16 *out) {
    const int64_t n = (int64_t)rows * cols_out;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / cols_out), c = (int)(i % cols_out);
        out[i] = c < cols_in ? __float2bfloat16_rn(__bfloat162float(in[(int64_t)r * cols_in + c]) * mul)
                             : __float2bfloat16_rn(0.f);
    }
}

int blocks_for(int64_t n, int sms) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
}

}  // namespace

cudaError_t norm_mod_e4m3(cudaStream_t st, const float *x, int64_t ldx, int rows, int D, float eps, int mode,
                          const float *tab, int tab_coeff, const int *idx, int k_shift, uint8_t *out, int64_t ldo,
                          float *scale) {
    if (rows <= 0) return cudaSuccess;
    if (D != 4096 || ldx % 4 || ldo % 4 || ((uintptr_t)x & 15) || ((uintptr_t)out & 3) ||
        (tab && ((uintptr_t)tab & 15)))
        return cudaErrorInvalidValue;
    norm_mod_e4m3_kernel<<<(rows + 3) / 4, 256, 0, st>>>(x, ldx, rows, eps, mode, tab, tab_coeff, idx, k_shift, out,
                                                         ldo, scale);
    return cudaGetLastError();
}

cudaError_t quantize_rows_e4m3(cudaStream_t st, const __nv_bfloat16 *in, int64_t ldi, int rows, int cols, uint8_t *out,
                               int64_t ldo, float *scale) {
    if (rows <= 0) return cudaSuccess;
    if (cols % 8 || ldi % 8 || ldo % 8 || ((uintptr_t)in & 15) || ((uintptr_t)out & 7)) return cudaErrorInvalidValue;
    quantize_rows_e4m3_kernel<<<rows, 256, 0, st>>>(in, ldi, rows, cols, out, ldo, scale);
    return cudaGetLastError();
}

cudaError_t bf16_to_f32(cudaStream_t st, int sms, const __nv_bfloat16 *in, int64_t n, float *out) {
    if (n <= 0) return cudaSuccess;
    bf16_to_f32_kernel<<<blocks_for(n, sms), 256, 0, st>>>(in, n, out);
    return cudaGetLastError();
}

cudaError_t scale_pad_bf16(cudaStream_t st, int sms, const __nv_bfloat16 *in, int rows, int cols_in, int cols_out,
                           float mul, __nv_bfloat16 *out) {
    if ((int64_t)rows * cols_out <= 0) return cudaSuccess;
    scale_pad_bf16_kernel<<<blocks_for((int64_t)rows * cols_out, sms), 256, 0, st>>>(in, rows, cols_in, cols_out, mul,
                                                                                     out);
    return cudaGetLastError();
}

}  // namespace ltx

extern "C" int ltx_quantize_rows_e4m3(ltx_ctx *ctx, const void *in_dev, int64_t ldi, int32_t rows, int32_t cols,
                                      void *out_dev, int64_t ldo, float *scale_dev) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!in_dev || !out_dev || !scale_dev || rows < 0 || cols < 0)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_quantize_rows_e4m3: bad arguments");
    cudaError_t e = ltx::quantize_rows_e4m3(ctx->stream, static_cast<const __nv_bfloat16 *>(in_dev), ldi, rows, cols,
                                            static_cast<uint8_t *>(out_dev), ldo, scale_dev);
    if (e == cudaErrorInvalidValue)
        return ltx::fail(ctx, LTX_ERR_SHAPE, "ltx_quantize_rows_e4m3: cols and leading dimensions must be multiples of 8, "
                         "16-byte aligned input");
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_quantize_rows_e4m3");
}
