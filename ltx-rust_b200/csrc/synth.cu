// Synthetic checkpoint generation on the device: seeded N(0, std) weights,
// quantised to float8_e4m3fn with a per-tensor scale amax/448 — the layout of
// an FP8 LTX checkpoint — so random-init models go through the same
// dequant+merge path as real ones.  Counter-based (hash) RNG: the bytes
// depend only on (seed, stream id, element index), never on the grid.
#include <cuda_fp8.h>

#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Standard normal for element i of stream (seed, sid), Box-Muller on two 32-bit uniforms.
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t sid, uint64_t i) {
    const uint64_t h = splitmix64(seed ^ splitmix64(sid * 0x632BE59BD9B4E019ull + i));
    const float u1 = ((uint32_t)(h >> 40) + 1) * (1.0f / 16777217.0f);   // (0, 1]
    const float u2 = (uint32_t)(h & 0xFFFFFF) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void fill_normal_kernel(float *out, int64_t n, uint64_t seed, uint64_t sid, float mean, float std) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = mean + std * normal_at(seed, sid, (uint64_t)i);
}

__global__ void fill_normal_bf16_kernel(__nv_bfloat16 *out, int64_t n, uint64_t seed, uint64_t sid, float std) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2bfloat16_rn(std * normal_at(seed, sid, (uint64_t)i));
}

__global__ void absmax_kernel(const float *x, int64_t n, unsigned int *amax_bits) {
    float m = 0.f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));   // non-negative floats order as uints
}

// q = e4m3(x / scale), scale = amax / 448 (round to nearest even, saturating).
__global__ void quantize_e4m3_kernel(const float *x, int64_t n, const unsigned int *amax_bits, uint8_t *q,
                                     float *scale_out) {
    const float scale = __uint_as_float(*amax_bits) / 448.0f;
    const float inv = scale > 0.f ? 1.0f / scale : 0.f;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        q[i] = (uint8_t)__nv_cvt_float_to_fp8(x[i] * inv, __NV_SATFINITE, __NV_E4M3);
}

int grid_of(int64_t n, int sms) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8)); }

}  // namespace

cudaError_t synth_normal_f32(cudaStream_t st, int sms, float *out, int64_t n, uint64_t seed, uint64_t sid, float mean,
                             float std) {
    fill_normal_kernel<<<grid_of(n, sms), 256, 0, st>>>(out, n, seed, sid, mean, std);
    return cudaGetLastError();
}

cudaError_t synth_normal_bf16(cudaStream_t st, int sms, __nv_bfloat16 *out, int64_t n, uint64_t seed, uint64_t sid,
                              float std) {
    fill_normal_bf16_kernel<<<grid_of(n, sms), 256, 0, st>>>(out, n, seed, sid, std);
    return cudaGetLastError();
}

// f32 scratch [n] -> FP8 bytes + device scale (amax/448).  `work` holds one unsigned int.
cudaError_t synth_quantize_fp8(cudaStream_t st, int sms, const float *x, int64_t n, uint8_t *q, float *scale_dev,
                               unsigned int *work) {
    cudaError_t e = cudaMemsetAsync(work, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    absmax_kernel<<<grid_of(n, sms), 256, 0, st>>>(x, n, work);
    quantize_e4m3_kernel<<<grid_of(n, sms), 256, 0, st>>>(x, n, work, q, scale_dev);
    return cudaGetLastError();
}

}  // namespace ltx
