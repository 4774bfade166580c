// Kernels of the tensor-parallel forward: a model split over ranks by heads
// (attention) and hidden units (FFN).  Each rank holds D/n of every Q/K row,
// so the Q/K RMSNorm over the full inner dimension (Attention::forward,
// crates/ltx-dit/src/attention.rs:137-195; RmsNorm_gamma over all D) runs in
// two halves around a sum-allreduce of per-row sums of squares; and each
// row-split output projection's partial product (bf16) is summed across
// ranks before the bias, gate and residual add that the single-GPU GEMM epilogue
// fuses.  All three are HBM-bound streaming kernels.
#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

namespace {

// out[seg * rows + row] = sum_c x_seg[row][c]^2 over cols, for seg < nseg
// (segment seg starts seg_stride elements after the previous one).  One warp
// per row, 16-byte loads when aligned.
__global__ void __launch_bounds__(256) sumsq_rows_kernel(const __nv_bfloat16 *x, int64_t ld, int rows, int cols,
                                                         int nseg, int64_t seg_stride, float *out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows * nseg) return;
    const int seg = warp / rows, row = warp % rows;
    const __nv_bfloat16 *xr = x + (int64_t)seg * seg_stride + (int64_t)row * ld;
    float ss = 0.f;
    if ((cols & 7) == 0 && ((uintptr_t)xr & 15) == 0) {
        for (int c = lane * 8; c < cols; c += 256) {
            const uint4 u = *reinterpret_cast<const uint4 *>(xr + c);
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float2 f = __bfloat1622float2(h[q]);
                ss = fmaf(f.x, f.x, ss);
                ss = fmaf(f.y, f.y, ss);
            }
        }
    } else {
        for (int c = lane; c < cols; c += 32) {
            const float v = __bfloat162float(xr[c]);
            ss = fmaf(v, v, ss);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) out[warp] = ss;
}

// x[row][c] = x / sqrt(ss[row] / D + eps) * gamma[c], then RoPE with the
// tables of the global heads head0.. (split: [rows][D/2]; interleaved:
// [rows][D]).  One block per row; cols = local width (heads * d).
__global__ void __launch_bounds__(256) norm_apply_rope_kernel(__nv_bfloat16 *x, int64_t ld, int rows, int cols, int D,
                                                              int d, int head0, float eps, const float *gamma,
                                                              const float *ss, const float *cos_t,
                                                              const float *sin_t, int interleaved) {
    extern __shared__ float row_s[];
    const int row = blockIdx.x;
    if (row >= rows) return;
    __nv_bfloat16 *xr = x + (int64_t)row * ld;
    const float denom = sqrtf(ss[row] / (float)D + eps);
    for (int c = threadIdx.x; c < cols; c += blockDim.x) row_s[c] = __bfloat162float(xr[c]) / denom * gamma[c];
    __syncthreads();
    if (!cos_t) {
        for (int c = threadIdx.x; c < cols; c += blockDim.x) xr[c] = __float2bfloat16_rn(row_s[c]);
        return;
    }
    if (!interleaved) {
        const int half = d / 2, width = cols / 2;
        const float *cr = cos_t + (int64_t)row * (D / 2) + (int64_t)head0 * half;
        const float *sr = sin_t + (int64_t)row * (D / 2) + (int64_t)head0 * half;
        for (int i = threadIdx.x; i < width; i += blockDim.x) {
            const int h = i / half, j = i % half;
            const float x1 = row_s[h * d + j], x2 = row_s[h * d + half + j];
            const float c = cr[i], s = sr[i];
            xr[h * d + j] = __float2bfloat16_rn(c * x1 - s * x2);
            xr[h * d + half + j] = __float2bfloat16_rn(s * x1 + c * x2);
        }
    } else {
        const float *cr = cos_t + (int64_t)row * D + (int64_t)head0 * d;
        const float *sr = sin_t + (int64_t)row * D + (int64_t)head0 * d;
        for (int c = threadIdx.x; c < cols; c += blockDim.x) {
            const float rot = (c & 1) ? row_s[c - 1] : -row_s[c + 1];
            xr[c] = __float2bfloat16_rn(row_s[c] * cr[c] + rot * sr[c]);
        }
    }
}

// The same for head dim 128 with split RoPE (or none), one warp per row and
// 16-byte accesses: per iteration the warp takes 4 heads, lane group k (8
// lanes) the pairs 8k'..8k'+7 of its head (x1 at j, x2 at j + 64).  Without
// RoPE each lane takes 8 consecutive columns.  Same arithmetic per element.
__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float *f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
        f[2 * e] = t.x;
        f[2 * e + 1] = t.y;
    }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float *f) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
        w[e] = *reinterpret_cast<const uint32_t *>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}
__global__ void __launch_bounds__(256) norm_apply_rope_d128_kernel(__nv_bfloat16 *x, int64_t ld, int rows, int cols,
                                                                   int D, int head0, float eps, const float *gamma,
                                                                   const float *ss, const float *cos_t,
                                                                   const float *sin_t) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row >= rows) return;
    __nv_bfloat16 *xr = x + (int64_t)row * ld;
    const float denom = sqrtf(ss[row] / (float)D + eps);
    if (!cos_t) {
        for (int c = lane * 8; c < cols; c += 256) {
            float f[8], g[8];
            bf16x8_to_f32(*reinterpret_cast<const uint4 *>(xr + c), f);
            *reinterpret_cast<float4 *>(g) = __ldg(reinterpret_cast<const float4 *>(gamma + c));
            *reinterpret_cast<float4 *>(g + 4) = __ldg(reinterpret_cast<const float4 *>(gamma + c + 4));
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] / denom * g[e];
            *reinterpret_cast<uint4 *>(xr + c) = f32_to_bf16x8(f);
        }
        return;
    }
    const float *cr = cos_t + (int64_t)row * (D / 2) + (int64_t)head0 * 64;
    const float *sr = sin_t + (int64_t)row * (D / 2) + (int64_t)head0 * 64;
    const int k = lane & 7;
    for (int h = lane >> 3; h < cols / 128; h += 4) {
        const int c1 = h * 128 + 8 * k, c2 = c1 + 64, t = h * 64 + 8 * k;
        float x1[8], x2[8], g1[8], g2[8], cs[8], sn[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4 *>(xr + c1), x1);
        bf16x8_to_f32(*reinterpret_cast<const uint4 *>(xr + c2), x2);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            *reinterpret_cast<float4 *>(g1 + 4 * q) = __ldg(reinterpret_cast<const float4 *>(gamma + c1 + 4 * q));
            *reinterpret_cast<float4 *>(g2 + 4 * q) = __ldg(reinterpret_cast<const float4 *>(gamma + c2 + 4 * q));
            *reinterpret_cast<float4 *>(cs + 4 * q) = *reinterpret_cast<const float4 *>(cr + t + 4 * q);
            *reinterpret_cast<float4 *>(sn + 4 * q) = *reinterpret_cast<const float4 *>(sr + t + 4 * q);
        }
        float o1[8], o2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float a = x1[e] / denom * g1[e], b = x2[e] / denom * g2[e];
            o1[e] = cs[e] * a - sn[e] * b;
            o2[e] = sn[e] * a + cs[e] * b;
        }
        *reinterpret_cast<uint4 *>(xr + c1) = f32_to_bf16x8(o1);
        *reinterpret_cast<uint4 *>(xr + c2) = f32_to_bf16x8(o2);
    }
}

// x[row][c] += (p[row][c] + bias[c]) * gate[idx[row]][c]: the single-GPU
// EPI_RESID epilogue, applied after the partial products (bf16) were summed.
__global__ void __launch_bounds__(256) resid_add_kernel(float *x, const __nv_bfloat16 *p, int rows, int D,
                                                        const float *bias, const float *gate, const int *gidx,
                                                        int64_t ld_gate) {
    const int64_t n4 = (int64_t)rows * D / 4;
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = v * 4;
        const int row = (int)(i / D), col = (int)(i % D);
        float4 xv = reinterpret_cast<float4 *>(x)[v];
        const uint2 pu = reinterpret_cast<const uint2 *>(p)[v];
        const float2 p01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&pu.x));
        const float2 p23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&pu.y));
        const float4 pv = make_float4(p01.x, p01.y, p23.x, p23.y);
        float b[4] = {0.f, 0.f, 0.f, 0.f}, g[4] = {1.f, 1.f, 1.f, 1.f};
        if (bias) {
            const float4 b4 = *reinterpret_cast<const float4 *>(bias + col);
            b[0] = b4.x; b[1] = b4.y; b[2] = b4.z; b[3] = b4.w;
        }
        if (gate) {
            const float *gr = gate + (int64_t)(gidx ? gidx[row] : 0) * ld_gate + col;
            g[0] = gr[0]; g[1] = gr[1]; g[2] = gr[2]; g[3] = gr[3];
        }
        xv.x += (pv.x + b[0]) * g[0];
        xv.y += (pv.y + b[1]) * g[1];
        xv.z += (pv.z + b[2]) * g[2];
        xv.w += (pv.w + b[3]) * g[3];
        reinterpret_cast<float4 *>(x)[v] = xv;
    }
}

int grid_cap(int64_t work_items, int per_block, int sms) {
    const int64_t b = (work_items + per_block - 1) / per_block;
    return (int)std::max<int64_t>(1, std::min<int64_t>(b, (int64_t)sms * 16));
}

}  // namespace

cudaError_t tp_sumsq_rows(cudaStream_t st, const __nv_bfloat16 *x, int64_t ld, int rows, int cols, int nseg,
                          int64_t seg_stride, float *out) {
    const int64_t warps = (int64_t)rows * nseg;
    if (warps == 0) return cudaSuccess;
    sumsq_rows_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(x, ld, rows, cols, nseg, seg_stride, out);
    return cudaGetLastError();
}

cudaError_t tp_norm_apply_rope(cudaStream_t st, __nv_bfloat16 *x, int64_t ld, int rows, int cols, int D, int d,
                               int head0, float eps, const float *gamma, const float *ss, const float *cos_t,
                               const float *sin_t, bool interleaved) {
    if (rows == 0) return cudaSuccess;
    const bool aligned = ld % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)gamma & 15) == 0 &&
                         (!cos_t || (((uintptr_t)cos_t & 15) == 0 && ((uintptr_t)sin_t & 15) == 0 && D % 8 == 0));
    if (d == 128 && !interleaved && cols % 512 == 0 && aligned) {
        norm_apply_rope_d128_kernel<<<(rows + 7) / 8, 256, 0, st>>>(x, ld, rows, cols, D, head0, eps, gamma, ss, cos_t,
                                                                    sin_t);
        return cudaGetLastError();
    }
    const size_t smem = (size_t)cols * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(norm_apply_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    norm_apply_rope_kernel<<<rows, 256, smem, st>>>(x, ld, rows, cols, D, d, head0, eps, gamma, ss, cos_t, sin_t,
                                                    interleaved ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t tp_resid_add(cudaStream_t st, int sms, float *x, const __nv_bfloat16 *p, int rows, int D,
                         const float *bias, const float *gate, const int *gidx, int64_t ld_gate) {
    if (rows == 0) return cudaSuccess;
    if (D % 4) return cudaErrorInvalidValue;
    resid_add_kernel<<<grid_cap((int64_t)rows * D / 4, 256, sms), 256, 0, st>>>(x, p, rows, D, bias, gate, gidx,
                                                                                 ld_gate);
    return cudaGetLastError();
}

}  // namespace ltx
