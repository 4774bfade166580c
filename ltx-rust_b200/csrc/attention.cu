// K3: flash attention forward on the 5th-generation tensor cores.
//
// Replaces sdp_attention (crates/ltx-dit/src/attention.rs:228-242), which
// materialises softmax(Q K^T * scale) V as a full [B, H, Tq, Tk] f32 matrix;
// here the scores live only in TMEM.  Head dim 128, bf16 Q/K, bf16 or f16 V,
// f32 accumulation, non-causal, key padding mask for a ragged last tile.
//
// One CTA per (batch, head, 256 queries) = two 128-row query tiles A and B
// that share every K/V tile (half the L2->SM traffic of one tile per CTA).
// 10 warps:
//   warp 0     TMA: Q_A and Q_B once, then K_0, V_0, K_1, V_1, ... through a
//              3-slot ring of 32 KB tiles (3-D tensor maps {H*128, T, B}, so
//              a tile never reads the next batch).
//   warp 1     one thread issues tcgen05.mma in the order
//                QK_A(0) QK_B(0) | QK_A(j+1) PV_A(j) QK_B(j+1) PV_B(j) ...
//              S_X = Q_X K_j^T -> TMEM S_X; O_X += P_X V_j -> TMEM O_X
//              (P from smem, V as an MN-major B operand).  QK_t(j+1) goes
//              out as soon as tile t's softmax has read S_t(j) into registers
//              (s_free), PV_t(j) once P_t(j) is in smem (p_full): the next
//              scores are computed under the current exp/P work, and tile A's
//              softmax runs under tile B's MMAs and vice versa.
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: one query row per
//              thread; the row's 128 scores are read from TMEM into
//              registers, max and exp2 (two per MUFU op, ex2.approx.f16x2),
//              P (f16 or bf16) written to smem in the 128B-swizzled K-major
//              layout.  O stays in TMEM; it is rescaled in place (tcgen05.ld/
//              st) only when a row max grows by more than kRescaleLog2 over
//              the max P is taken against.  Before P_t(j) is written or O_t
//              rescaled, the softmax waits for PV_t(j-1) (pv_done).
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
constexpr int kRing = 3;                  // K/V tile slots
constexpr int kThreads = 320;
constexpr int TILE_BYTES = 128 * D * 2;   // 32 KB: 128 rows x 128 16-bit values (two 64-col swizzle atoms)
constexpr int HALF_BYTES = 128 * 64 * 2;  // 16 KB: one atom column block
constexpr float kRescaleLog2 = 8.0f;      // O is rescaled when a row max grows by more than 2^8

struct AttnSmemLayout {
    static constexpr int Q = 0;                         // Q_A, Q_B
    static constexpr int P = Q + 2 * TILE_BYTES;        // P_A, P_B
    static constexpr int RING = P + 2 * TILE_BYTES;     // kRing K/V slots
    static constexpr int BAR = RING + kRing * TILE_BYTES;
    static constexpr int BYTES = BAR + 256;
};
constexpr size_t kAttnSmem = AttnSmemLayout::BYTES + 1024;
static_assert(kAttnSmem <= 232448, "attention smem exceeds the per-CTA limit");

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

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also names the 32 destination registers of an earlier
// tcgen05.ld as read-write operands, so no use of them can be scheduled before
// the wait (the loads land asynchronously).
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]),
          "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
          "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
        :
        : "memory");
}

// VF16: V (and so P) are f16; otherwise bf16.  Q and K are always bf16.
template <bool VF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *sQ = smem + AttnSmemLayout::Q;
    unsigned char *sP = smem + AttnSmemLayout::P;
    unsigned char *sRing = smem + AttnSmemLayout::RING;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AttnSmemLayout::BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *slot_full = bars + 1;         // [kRing]
    uint64_t *slot_empty = bars + 4;        // [kRing]
    uint64_t *s_full = bars + 7;            // [2]  tile A, B
    uint64_t *p_full = bars + 9;            // [2]
    uint64_t *pv_done = bars + 11;          // [2]
    uint64_t *s_free = bars + 13;           // [2]  S_t read into registers by all 4 softmax warps
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 15);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q_tiles = (p.Tq + 2 * BQ - 1) / (2 * BQ);
    const int qt = blockIdx.x % q_tiles;
    const int h = (blockIdx.x / q_tiles) % p.H;
    const int b = blockIdx.x / (q_tiles * p.H);
    const int n_kv = (p.Tk + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kRing; ++s) {
            mbar_init(&slot_full[s], 1);
            mbar_init(&slot_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 4);
            mbar_init(&pv_done[i], 1);
            mbar_init(&s_free[i], 4);
        }
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;   // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
    bool aborted = false;

    if (warp == 0) {
        if (elect_one()) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
            for (int t = 0; t < 2; ++t) {
                tma_load_3d(sQ + t * TILE_BYTES, &tmQ, q_full, h * D, qt * 2 * BQ + t * BQ, b);
                tma_load_3d(sQ + t * TILE_BYTES + HALF_BYTES, &tmQ, q_full, h * D + 64, qt * 2 * BQ + t * BQ, b);
            }
            // load sequence: s = 2j -> K_j, s = 2j + 1 -> V_j, slot s % kRing
            int issued = 0;
            for (int s = 0; s < 2 * n_kv && !aborted; ++s, ++issued) {
                const int slot = s % kRing;
                if (!mbar_wait(&slot_empty[slot], ((s / kRing) & 1) ^ 1, p.timeout_flag, 201, &aborted)) break;
                unsigned char *dst = sRing + slot * TILE_BYTES;
                const void *tm = (s & 1) ? &tmV : &tmK;
                const int j = s >> 1;
                mbar_arrive_expect_tx(&slot_full[slot], TILE_BYTES);
                tma_load_3d(dst, tm, &slot_full[slot], h * D, j * BKV, b);
                tma_load_3d(dst + HALF_BYTES, tm, &slot_full[slot], h * D + 64, j * BKV, b);
            }
            // Wait for every copy this thread started before the CTA can exit.
            bool a2 = false;
            mbar_wait(q_full, 0, nullptr, 0, &a2);
            for (int s = issued > kRing ? issued - kRing : 0; s < issued; ++s)
                mbar_wait(&slot_full[s % kRing], (s / kRing) & 1, nullptr, 0, &a2);
        }
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc_qk = idesc_f16(BQ, BKV, true, false);
            constexpr uint32_t idesc_pv = idesc_f16(BQ, D, !VF16, true);   // B = V, MN-major
            const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
            auto slot_of = [](int s) { return s % kRing; };
            auto wait_slot = [&](int s, int code) {
                return mbar_wait(&slot_full[slot_of(s)], (s / kRing) & 1, p.timeout_flag, code, &aborted);
            };
            auto issue_qk = [&](int t, int j) {   // S_t = Q_t K_j^T
                const uint32_t k_addr = smem_u32(sRing + slot_of(2 * j) * TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
                    umma_f16_ss(tmem + t * 128, sdesc_sw128(q_addr + t * TILE_BYTES + off, 16, 1024),
                                sdesc_sw128(k_addr + off, 16, 1024), idesc_qk, kk ? 1u : 0u);
                }
                umma_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {   // O_t (+)= P_t V_j
                const uint32_t v_addr = smem_u32(sRing + slot_of(2 * j + 1) * TILE_BYTES);
                const uint32_t pa = p_addr + t * TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk) {
                    const uint64_t ad = sdesc_sw128(pa + (kk >> 2) * HALF_BYTES + (kk & 3) * 32, 16, 1024);
                    const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, HALF_BYTES, 1024);
                    umma_f16_ss(tmem + 256 + t * 128, ad, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&pv_done[t]);
            };
            bool ok = mbar_wait(q_full, 0, p.timeout_flag, 205, &aborted) && wait_slot(0, 206);
            if (ok) {
                tc_fence_after();
                issue_qk(0, 0);
                issue_qk(1, 0);
                umma_commit(&slot_empty[slot_of(0)]);   // K_0 read by both
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                // Per tile: QK_t(j+1) as soon as the softmax has read S_t(j) into
                // registers (s_free), then PV_t(j) once P_t(j) is in smem (p_full):
                // the next scores are computed under the current tile's exp/P work.
                if (!wait_slot(2 * j + 1, 207)) break;
                const bool next = j + 1 < n_kv;
                if (next && !wait_slot(2 * j + 2, 208)) break;
                for (int t = 0; t < 2; ++t) {
                    if (next) {
                        if (!mbar_wait(&s_free[t], j & 1, p.timeout_flag, 213 + t, &aborted)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        issue_qk(t, j + 1);
                    }
                    if (!mbar_wait(&p_full[t], j & 1, p.timeout_flag, 209 + t, &aborted)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(t, j);
                }
                if (!ok) break;
                umma_commit(&slot_empty[slot_of(2 * j + 1)]);        // V_j read by both PVs
                if (next) umma_commit(&slot_empty[slot_of(2 * j + 2)]);   // K_{j+1} read by both QKs
            }
        }
    } else {
        // Softmax warps: tile t = 0 (warps 2-5) or 1 (warps 6-9), row quad*32 + lane.
        const int t = (warp - 2) >> 2;
        const int quad = warp & 3;
        const int row_in_tile = quad * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t s_tmem = tmem + lane_base + t * 128;
        const uint32_t o_tmem = tmem + lane_base + 256 + t * 128;
        unsigned char *p_row = sP + t * TILE_BYTES + row_in_tile * 128;
        const int sw = row_in_tile & 7;
        const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
        float m_ref = -INFINITY;   // the max P is taken against
        float l = 0.f;
        for (int j = 0; j < n_kv && !aborted; ++j) {
            // warp-uniform outcome: the tcgen05.ld/st below are warp-collective
            if (!warp_wait(&s_full[t], j & 1, p.timeout_flag, 211, &aborted)) break;
            tc_fence_after();
            const int kv0 = j * BKV;
            const bool ragged = kv0 + BKV > p.Tk;   // only the last tile can be
            // pass 1: the row max over the 128 scores, all four 32-column TMEM
            // loads in flight together (one wait), 8 independent partial maxima.
            // Keys 64..127 stay in registers (rh) for pass 2.
            uint32_t rh[2][32];
            float mx;
            {
                uint32_t r01[2][32];
                tmem_ld_32x32b_x32(s_tmem + 0, r01[0]);
                tmem_ld_32x32b_x32(s_tmem + 32, r01[1]);
                tmem_ld_32x32b_x32(s_tmem + 64, rh[0]);
                tmem_ld_32x32b_x32(s_tmem + 96, rh[1]);
                tmem_ld_wait_regs(r01[0]);
                tmem_ld_wait_regs(r01[1]);
                tmem_ld_wait_regs(rh[0]);
                tmem_ld_wait_regs(rh[1]);
                if (ragged) {
#pragma unroll
                    for (int e = 0; e < 64; ++e) {
                        if (kv0 + e >= p.Tk) r01[e >> 5][e & 31] = __float_as_uint(-INFINITY);
                        if (kv0 + 64 + e >= p.Tk) rh[e >> 5][e & 31] = __float_as_uint(-INFINITY);
                    }
                }
                float m8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) m8[u] = -INFINITY;
#pragma unroll
                for (int e = 0; e < 64; ++e) {
                    m8[e & 7] = fmaxf(m8[e & 7], __uint_as_float(r01[e >> 5][e & 31]));
                    m8[(e + 4) & 7] = fmaxf(m8[(e + 4) & 7], __uint_as_float(rh[e >> 5][e & 31]));
                }
                mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            }
            mx *= p.scale_log2;   // scale > 0: max(s * scale) = scale * max(s)
            // The rows of one warp decide together: tcgen05.ld/st are
            // warp-collective (.sync.aligned), so the O rescale runs for the
            // whole warp when any of its rows needs it; a row that does not
            // keeps its reference (alpha = 1).
            const bool grow = mx > m_ref + kRescaleLog2;
            // P_t and O_t belong to PV_t(j-1) until it completes (it is issued
            // after QK_t(j), so S_t(j) being ready does not imply it).
            if (j > 0 && !warp_wait(&pv_done[t], (j - 1) & 1, p.timeout_flag, 215, &aborted)) break;
            if (__any_sync(0xffffffffu, grow)) {
                // O_t and l are relative to m_ref; move them to mx (P.V of the
                // previous tile has completed: waited for above).
                const float alpha = grow ? ex2(m_ref - mx) : 1.0f;   // 0 when m_ref = -inf
                if (j > 0) {
                    const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t o[32];
                        tmem_ld_32x32b_x32(o_tmem + c * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            const float2 v = __fmul2_rn(make_float2(__uint_as_float(o[2 * e]), __uint_as_float(o[2 * e + 1])), a2);
                            o[2 * e] = __float_as_uint(v.x);
                            o[2 * e + 1] = __float_as_uint(v.y);
                        }
                        tmem_st_32x32b_x32(o_tmem + c * 32, o);
                    }
                    tmem_st_wait();
                }
                l *= alpha;
                if (grow) m_ref = mx;
            }
            // pass 2: P = exp2(s * scale - m_ref) (<= 2^kRescaleLog2), two per MUFU op; row sum in f32.
            // Keys 0..63 are re-read from TMEM while keys 64..127 (kept in
            // registers) are turned into P; once the re-read lands S_t is free.
            const float2 nm2 = make_float2(-m_ref, -m_ref);
            float2 sum2 = make_float2(0.f, 0.f);
            auto p_half = [&](uint32_t (&r)[2][32], int hf) {
                unsigned char *atom = p_row + hf * HALF_BYTES;
#pragma unroll
                for (int q = 0; q < 8; ++q) {      // 16-byte chunk q of the atom row: keys hf*64 + 8q ..
                    uint32_t pk[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = q * 8 + 2 * u;
                        const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[e >> 5][e & 31]),
                                                                __uint_as_float(r[e >> 5][(e & 31) + 1])), sl2, nm2);
                        uint32_t in, out;
                        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(in) : "f"(x.y), "f"(x.x));
                        asm("ex2.approx.f16x2 %0, %1;" : "=r"(out) : "r"(in));
                        const float2 pf = __half22float2(*reinterpret_cast<__half2 *>(&out));
                        sum2 = __fadd2_rn(sum2, pf);
                        if constexpr (VF16) {
                            pk[u] = out;
                        } else {
                            __nv_bfloat162 hv = __floats2bfloat162_rn(pf.x, pf.y);
                            pk[u] = *reinterpret_cast<uint32_t *>(&hv);
                        }
                    }
                    *reinterpret_cast<uint4 *>(atom + ((q ^ sw) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
            };
            {
                uint32_t r0[2][32];
                tmem_ld_32x32b_x32(s_tmem + 0, r0[0]);
                tmem_ld_32x32b_x32(s_tmem + 32, r0[1]);
                p_half(rh, 1);
                tmem_ld_wait_regs(r0[0]);
                tmem_ld_wait_regs(r0[1]);
                // S_t is in registers: the MMA warp may overwrite it with QK_t(j+1)
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[t]);
                if (ragged) {
#pragma unroll
                    for (int e = 0; e < 64; ++e)
                        if (kv0 + e >= p.Tk) r0[e >> 5][e & 31] = __float_as_uint(-INFINITY);
                }
                p_half(r0, 0);
            }
            l += sum2.x + sum2.y;
            tc_fence_before();
            fence_proxy_async_smem();   // P (generic-proxy writes) -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        // O_t is final once the last P.V has completed.
        if (!aborted && warp_wait(&pv_done[t], (n_kv - 1) & 1, p.timeout_flag, 212, &aborted)) {
            tc_fence_after();
            const int q_row = qt * 2 * BQ + t * BQ + row_in_tile;
            const float inv = 1.f / l;
            __nv_bfloat16 *dst = p.out + ((int64_t)b * p.Tq + q_row) * p.ldo + h * D;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(o_tmem + c * 32, r);
                tmem_ld_wait();
                if (q_row < p.Tq) {
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(r[g * 8 + 2 * e]) * inv,
                                                                      __uint_as_float(r[g * 8 + 2 * e + 1]) * inv);
                            w[e] = *reinterpret_cast<uint32_t *>(&hv);
                        }
                        *reinterpret_cast<uint4 *>(dst + c * 32 + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
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
    const int grid = B * H * ((Tq + 2 * BQ - 1) / (2 * BQ));
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
