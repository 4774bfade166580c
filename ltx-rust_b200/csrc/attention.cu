// K3: flash attention forward on the 5th-generation tensor cores.
//
// Replaces sdp_attention (crates/ltx-dit/src/attention.rs:228-242), which
// materialises softmax(Q K^T * scale) V as a full [B, H, Tq, Tk] f32 matrix;
// here the scores live only in TMEM.  Head dim 128, bf16 Q/K/V, f32
// accumulation, non-causal, optional key padding mask for a ragged last tile.
//
// One CTA per (batch, head, 128-query tile), 6 warps:
//   warp 0   TMA: Q once, then K_j / V_j into a 2-stage ring (3-D tensor
//            maps {H*128, T, B}, so a tile never reads the next batch).
//   warp 1   one thread issues tcgen05.mma:
//              S_j  = Q K_j^T        -> TMEM S[j%2]   (A,B K-major)
//              PV_j = P_j V_j        -> TMEM PV[j%2]  (A = P from smem,
//                                                      B = V_j MN-major)
//            QK_{j+1} is issued before PV_j, so the tensor core computes the
//            next scores while the softmax warps work on the current ones.
//   warps 2-9  two threads per query row (warps w and w+4 share a TMEM lane
//            quadrant; each takes 64 of the 128 score / output columns):
//            row max exchanged through shared memory (named barrier), exp2
//            two-at-a-time (ex2.approx.f16x2), P_j (bf16) written to smem in
//            the 128B-swizzled K-major layout the MMA reads (each half-thread
//            writes one whole 64-key swizzle atom), O half kept in registers
//            and updated with PV_{j-1} one tile late (O = O*exp2(m_o - m) + PV).
// All waits are bounded (2 s) and report LTX_ERR_TIMEOUT through the flag.
#include <cuda.h>

#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

struct AttnParams {
    int B, H, Tq, Tk;
    float scale_log2;      // softmax scale * log2(e)
    __nv_bfloat16 *out;    // [B*Tq, ldo]
    int64_t ldo;
    int *timeout_flag;
};

namespace {

constexpr int D = 128;
constexpr int BQ = 128, BKV = 128;
constexpr int KV_STAGES = 2;
constexpr int kThreads = 320;
constexpr int kSoftmaxWarps = 8;
constexpr int TILE_BYTES = 128 * D * 2;   // 32 KB: 128 rows x 128 bf16 (two 64-col swizzle atoms)
constexpr int HALF_BYTES = 128 * 64 * 2;  // 16 KB: one atom column block

struct AttnSmemLayout {
    static constexpr int Q = 0;
    static constexpr int P = Q + TILE_BYTES;
    static constexpr int K = P + TILE_BYTES;
    static constexpr int V = K + KV_STAGES * TILE_BYTES;
    static constexpr int BAR = V + KV_STAGES * TILE_BYTES;
    static constexpr int RED = BAR + 256;                   // [2 parity][2 half][128 rows] f32
    static constexpr int BYTES = RED + 2 * 2 * 128 * 4;
};
constexpr size_t kAttnSmem = AttnSmemLayout::BYTES + 1024;

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const void *tmap, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// exp2 of two values with one MUFU op: f32 -> f16x2 -> ex2.approx.f16x2 -> f32.
// (P is rounded to bf16 for the MMA afterwards, so the f16 step costs nothing.)
__device__ __forceinline__ float2 ex2x2(float a, float b) {
    uint32_t in, out;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(in) : "f"(b), "f"(a));
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(out) : "r"(in));
    __half2 h = *reinterpret_cast<__half2 *>(&out);
    return __half22float2(h);
}

__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// VF16: V (and so P) are f16; otherwise bf16.  Q and K are always bf16.
template <bool VF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *sQ = smem + AttnSmemLayout::Q;
    unsigned char *sP = smem + AttnSmemLayout::P;
    unsigned char *sK = smem + AttnSmemLayout::K;
    unsigned char *sV = smem + AttnSmemLayout::V;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AttnSmemLayout::BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *k_full = bars + 1;            // [KV_STAGES]
    uint64_t *v_full = bars + 3;            // [KV_STAGES]
    uint64_t *kv_empty = bars + 5;          // [KV_STAGES]
    uint64_t *s_full = bars + 7;            // [2]
    uint64_t *s_empty = bars + 9;           // [2]
    uint64_t *p_full = bars + 11;
    uint64_t *p_empty = bars + 12;
    uint64_t *pv_full = bars + 13;          // [2]
    uint64_t *pv_empty = bars + 15;         // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 17);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q_tiles = (p.Tq + BQ - 1) / BQ;
    const int qt = blockIdx.x % q_tiles;
    const int h = (blockIdx.x / q_tiles) % p.H;
    const int b = blockIdx.x / (q_tiles * p.H);
    const int n_kv = (p.Tk + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KV_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_empty[i], kSoftmaxWarps);
            mbar_init(&pv_full[i], 1);
            mbar_init(&pv_empty[i], kSoftmaxWarps);
        }
        mbar_init(p_full, kSoftmaxWarps);
        mbar_init(p_empty, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool aborted = false;

    if (warp == 0) {
        if (elect_one()) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(q_full, TILE_BYTES);
            tma_load_3d(sQ, &tmQ, q_full, h * D, qt * BQ, b);
            tma_load_3d(sQ + HALF_BYTES, &tmQ, q_full, h * D + 64, qt * BQ, b);
            int issued = 0;
            for (int j = 0; j < n_kv && !aborted; ++j, ++issued) {
                const int s = j % KV_STAGES;
                const uint32_t ph = (j / KV_STAGES) & 1;
                if (!mbar_wait(&kv_empty[s], ph ^ 1, p.timeout_flag, 201, &aborted)) break;
                unsigned char *k_dst = sK + s * TILE_BYTES, *v_dst = sV + s * TILE_BYTES;
                mbar_arrive_expect_tx(&k_full[s], TILE_BYTES);
                tma_load_3d(k_dst, &tmK, &k_full[s], h * D, j * BKV, b);
                tma_load_3d(k_dst + HALF_BYTES, &tmK, &k_full[s], h * D + 64, j * BKV, b);
                mbar_arrive_expect_tx(&v_full[s], TILE_BYTES);
                tma_load_3d(v_dst, &tmV, &v_full[s], h * D, j * BKV, b);
                tma_load_3d(v_dst + HALF_BYTES, &tmV, &v_full[s], h * D + 64, j * BKV, b);
            }
            // Wait for every copy this thread started before the CTA can exit.
            bool a2 = false;
            mbar_wait(q_full, 0, nullptr, 0, &a2);
            for (int j = issued > KV_STAGES ? issued - KV_STAGES : 0; j < issued; ++j) {
                mbar_wait(&k_full[j % KV_STAGES], (j / KV_STAGES) & 1, nullptr, 0, &a2);
                mbar_wait(&v_full[j % KV_STAGES], (j / KV_STAGES) & 1, nullptr, 0, &a2);
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc_qk = idesc_f16(BQ, BKV, true, false);
            constexpr uint32_t idesc_pv = idesc_f16(BQ, D, !VF16, true);   // B = V, MN-major
            const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
            auto issue_pv = [&](int j) -> bool {
                const int s = j % KV_STAGES;
                if (!mbar_wait(p_full, j & 1, p.timeout_flag, 202, &aborted)) return false;
                if (!mbar_wait(&v_full[s], (j / KV_STAGES) & 1, p.timeout_flag, 203, &aborted)) return false;
                if (!mbar_wait(&pv_empty[j & 1], ((j >> 1) & 1) ^ 1, p.timeout_flag, 204, &aborted)) return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV + s * TILE_BYTES);
                const uint32_t d_tmem = tmem + 256 + (j & 1) * 128;
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk) {
                    const uint64_t ad = sdesc_sw128(p_addr + (kk >> 2) * HALF_BYTES + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, HALF_BYTES, 1024);
                    umma_f16_ss(d_tmem, ad, bd, idesc_pv, kk ? 1u : 0u);
                }
                umma_commit(&pv_full[j & 1]);
                umma_commit(&kv_empty[s]);
                umma_commit(p_empty);
                return true;
            };
            if (mbar_wait(q_full, 0, p.timeout_flag, 205, &aborted)) {
                for (int j = 0; j < n_kv; ++j) {
                    const int s = j % KV_STAGES;
                    if (!mbar_wait(&k_full[s], (j / KV_STAGES) & 1, p.timeout_flag, 206, &aborted)) break;
                    if (!mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, p.timeout_flag, 207, &aborted)) break;
                    tc_fence_after();
                    const uint32_t k_addr = smem_u32(sK + s * TILE_BYTES);
                    const uint32_t d_tmem = tmem + (j & 1) * 128;
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                        umma_f16_ss(d_tmem, sdesc_sw128(q_addr + off, 16, 1024), sdesc_sw128(k_addr + off, 16, 1024),
                                    idesc_qk, kk ? 1u : 0u);
                    }
                    umma_commit(&s_full[j & 1]);
                    if (j > 0 && !issue_pv(j - 1)) break;
                }
                if (!aborted) issue_pv(n_kv - 1);
            }
        }
    } else {
        // Softmax / output warps 2..9: row quad*32 + lane, column half `hf` (64 of 128).
        const int quad = warp & 3;
        const int hf = (warp - 2) >> 2;
        const int row_in_tile = quad * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        float *red = reinterpret_cast<float *>(smem + AttnSmemLayout::RED);   // [2][2][128]
        float2 o[D / 4];   // this thread's 64 output columns as pairs
#pragma unroll
        for (int c = 0; c < D / 4; ++c) o[c] = make_float2(0.f, 0.f);
        float m = -INFINITY, l = 0.f, m_o = -INFINITY;
        float m_hist[2] = {-INFINITY, -INFINITY};   // max used for P_j, by j % 2
        // P smem: row r, 16-byte chunk c of atom a at a*16K + r*128 + ((c ^ (r&7)) * 16).
        // This thread writes atom `hf` of its row (keys hf*64 .. hf*64+63).
        unsigned char *p_row = sP + hf * HALF_BYTES + row_in_tile * 128;
        const int sw = row_in_tile & 7;

        auto fold_pv = [&](int j) -> bool {
            if (!mbar_wait(&pv_full[j & 1], (j >> 1) & 1, p.timeout_flag, 208, &aborted)) return false;
            tc_fence_after();
            const float mj = m_hist[j & 1];
            const float alpha = ex2(m_o - mj);   // 0 on the first fold (m_o = -inf)
            const float2 a2 = make_float2(alpha, alpha);
            m_o = mj;
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tmem + lane_base + 256 + (j & 1) * 128 + hf * 64, r0);
            tmem_ld_32x32b_x32(tmem + lane_base + 256 + (j & 1) * 128 + hf * 64 + 32, r1);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                o[e] = __ffma2_rn(o[e], a2, make_float2(__uint_as_float(r0[2 * e]), __uint_as_float(r0[2 * e + 1])));
                o[16 + e] = __ffma2_rn(o[16 + e], a2, make_float2(__uint_as_float(r1[2 * e]), __uint_as_float(r1[2 * e + 1])));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pv_empty[j & 1]);
            return true;
        };

        // Every softmax thread calls softmax_bar() exactly n_kv + 1 times, also
        // after a timed-out wait (it then skips the work, not the barrier), so
        // the named barrier can never be left waiting.
        const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
        for (int j = 0; j < n_kv; ++j) {
            const bool live = mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.timeout_flag, 209, &aborted);
            const int kv0 = j * BKV + hf * 64;
            const bool ragged = kv0 + 64 > p.Tk;   // only the last tile can be
            float sv[64];
            float mx = -INFINITY;
            if (live) {
                tc_fence_after();
                const uint32_t s_tmem = tmem + lane_base + (j & 1) * 128 + hf * 64;
                uint32_t r0[32], r1[32];
                tmem_ld_32x32b_x32(s_tmem, r0);
                tmem_ld_32x32b_x32(s_tmem + 32, r1);
                tmem_ld_wait();
                // the scores are in registers: hand the TMEM buffer back to the MMA warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[j & 1]);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    sv[e] = __uint_as_float(r0[e]);
                    sv[32 + e] = __uint_as_float(r1[e]);
                }
                if (ragged) {
#pragma unroll
                    for (int e = 0; e < 64; ++e)
                        if (kv0 + e >= p.Tk) sv[e] = -INFINITY;
                }
#pragma unroll
                for (int e = 0; e < 64; ++e) mx = fmaxf(mx, sv[e]);
                mx *= p.scale_log2;   // scale > 0: max(s * scale) = scale * max(s)
            }
            float *rj = red + (j & 1) * 256;
            rj[hf * 128 + row_in_tile] = mx;
            softmax_bar();
            if (!live || aborted) continue;
            mx = fmaxf(rj[row_in_tile], rj[128 + row_in_tile]);
            const float m_new = fmaxf(m, mx);
            const float corr = ex2(m - m_new);
            m = m_new;
            m_hist[j & 1] = m_new;
            // P_j overwrites P_{j-1}: wait until PV_{j-1} has read it.
            if (j > 0 && !mbar_wait(p_empty, (j - 1) & 1, p.timeout_flag, 210, &aborted)) continue;
            // P = exp2(s * scale - m): two per MUFU op (ex2.approx.f16x2), partial row sum in f32.
            const float2 nm2 = make_float2(-m_new, -m_new);
            float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int q = 0; q < 8; ++q) {   // 8 chunks of 8 keys = one 16-byte smem store each
                uint32_t pk[4];
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const int e = q * 8 + 2 * t;
                    const float2 x = __ffma2_rn(make_float2(sv[e], sv[e + 1]), sl2, nm2);
                    uint32_t in, out;
                    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(in) : "f"(x.y), "f"(x.x));
                    asm("ex2.approx.f16x2 %0, %1;" : "=r"(out) : "r"(in));
                    const float2 pf = __half22float2(*reinterpret_cast<__half2 *>(&out));
                    sum2 = __fadd2_rn(sum2, pf);
                    if constexpr (VF16) {
                        pk[t] = out;
                    } else {
                        __nv_bfloat162 hv = __floats2bfloat162_rn(pf.x, pf.y);
                        pk[t] = *reinterpret_cast<uint32_t *>(&hv);
                    }
                }
                *reinterpret_cast<uint4 *>(p_row + ((q ^ sw) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            l = l * corr + (sum2.x + sum2.y);
            fence_proxy_async_smem();   // P (generic-proxy writes) -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            if (j > 0) fold_pv(j - 1);
        }
        if (!aborted) fold_pv(n_kv - 1);
        // combine the two partial row sums in the buffer the last max exchange did not use
        float *rl = red + (n_kv & 1) * 256;
        rl[hf * 128 + row_in_tile] = l;
        softmax_bar();
        const float l_row = rl[row_in_tile] + rl[128 + row_in_tile];
        if (!aborted) {
            const int q_row = qt * BQ + row_in_tile;
            if (q_row < p.Tq) {
                const float inv = 1.f / l_row;
                __nv_bfloat16 *dst = p.out + ((int64_t)b * p.Tq + q_row) * p.ldo + h * D + hf * 64;
#pragma unroll
                for (int c = 0; c < D / 4; c += 4) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        __nv_bfloat162 hv = __floats2bfloat162_rn(o[c + e].x * inv, o[c + e].y * inv);
                        w[e] = *reinterpret_cast<uint32_t *>(&hv);
                    }
                    *reinterpret_cast<uint4 *>(dst + 2 * c) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn_attn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// [B, T, cols] bf16 view: base pointer, row stride ld (elements), box {64, 128, 1}.
bool make_tmap_3d(CUtensorMap *m, const void *ptr, int B, int T, int cols, int64_t ld, bool f16 = false) {
    EncodeTiledFn fn = encode_fn_attn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(ld * 2 * T)};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr),
              dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// out[b*Tq + t, h*128 + c] = softmax_k(q.k * scale) v for every batch b, head h.
// q/k/v: bf16, token-major with leading dimensions (elements); head h occupies
// columns [h*128, h*128+128).  Requirements: head_dim 128, ld % 8 == 0,
// 16-byte aligned bases.
int attention_fwd(ltx_ctx *ctx, cudaStream_t st, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v,
                  int64_t ldv, int B, int H, int Tq, int Tk, float scale, void *out, int64_t ldo, bool v_f16) {
    if (!q || !k || !v || !out) return fail(ctx, LTX_ERR_INVALID_ARG, "attention: null pointer");
    if (B <= 0 || H <= 0 || Tq <= 0 || Tk <= 0) return fail(ctx, LTX_ERR_SHAPE, "attention: empty shape");
    if (ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8 || ((uintptr_t)q & 15) || ((uintptr_t)k & 15) || ((uintptr_t)v & 15) ||
        ((uintptr_t)out & 15))
        return fail(ctx, LTX_ERR_SHAPE, "attention: rows must be 16-byte aligned");
    CUtensorMap tq, tk, tv;
    if (!make_tmap_3d(&tq, q, B, Tq, H * D, ldq) || !make_tmap_3d(&tk, k, B, Tk, H * D, ldk) ||
        !make_tmap_3d(&tv, v, B, Tk, H * D, ldv, v_f16))
        return fail(ctx, LTX_ERR_CUDA, "attention: cuTensorMapEncodeTiled failed");
    AttnParams p{B, H, Tq, Tk, scale * 1.4426950408889634f, static_cast<__nv_bfloat16 *>(out), ldo, ctx->timeout_flag};
    auto kern = v_f16 ? attn_fwd_kernel<true> : attn_fwd_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmem);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention smem attribute");
    const int grid = B * H * ((Tq + BQ - 1) / BQ);
    kern<<<grid, kThreads, kAttnSmem, st>>>(tq, tk, tv, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention launch");
    return LTX_OK;
}

}  // namespace ltx

extern "C" int ltx_attention_fwd(ltx_ctx *ctx, const void *q_dev, int64_t ldq, const void *k_dev, int64_t ldk,
                                 const void *v_dev, int64_t ldv, int32_t v_dtype, int32_t batch, int32_t heads,
                                 int32_t tq, int32_t tk, int32_t head_dim, float scale, void *out_dev, int64_t ldo) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (head_dim != 128) return ltx::fail(ctx, LTX_ERR_UNSUPPORTED, "attention: head_dim %d (only 128)", head_dim);
    if (v_dtype != LTX_BF16 && v_dtype != LTX_F16) return ltx::fail(ctx, LTX_ERR_DTYPE, "attention: V must be BF16 or F16");
    return ltx::attention_fwd(ctx, ctx->stream, q_dev, ldq, k_dev, ldk, v_dev, ldv, batch, heads, tq, tk, scale,
                              out_dev, ldo, v_dtype == LTX_F16);
}
