// K3: flash attention forward on the 5th-generation tensor cores.
//
// Replaces sdp_attention (crates/ltx-dit/src/attention.rs:228-242), which
// materialises softmax(Q K^T * scale) V as a full [B, H, Tq, Tk] f32 matrix;
// here the scores live only in TMEM.  Head dim 128, bf16 Q/K, bf16 or f16 V,
// f32 accumulation, non-causal, key padding mask for a ragged last tile.
//
// One CTA per (batch, head, 256 queries) = two 128-row query tiles A and B
// that share every K/V tile (half the L2->SM traffic of one tile per CTA).
// TMEM (512 columns): S_A, S_B (128 f32 columns each) and O_A, O_B.  P_t is
// written back into the upper half of S_t's columns as packed 16-bit pairs,
// and the P.V MMA reads its A operand from there: P never touches shared
// memory (no P stores or proxy fence in the softmax, and the 64 KB a shared
// P buffer would take go to a deeper K/V ring).
// 10 warps:
//   warp 0     TMA: Q_A and Q_B once, then K_0, V_0, K_1, V_1, ... through a
//              5-slot ring of 32 KB tiles (3-D tensor maps {H*128, T, B}, so
//              a tile never reads the next batch).
//   warp 1     one thread issues tcgen05.mma in the order
//                QK_A(0) QK_B(0) | PV_A(j) QK_A(j+1) PV_B(j) QK_B(j+1) ...
//              S_t = Q_t K_j^T -> TMEM S_t; O_t += P_t V_j -> TMEM O_t (P_t
//              from TMEM, V as an MN-major B operand from shared memory).
//              PV_t(j) goes out once the softmax has stored P_t(j) (p_full);
//              QK_t(j+1), which overwrites S_t/P_t, follows it in the same
//              in-order MMA stream.  Tile A's softmax runs under tile B's
//              MMAs and vice versa.
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: one query row per
//              thread; the row's 128 scores are read from TMEM into
//              registers, max, then exp2 in f32 (three quarters on the
//              MUFU, a quarter by a polynomial on the FMA pipe), P (f16 or
//              bf16) stored to TMEM with tcgen05.st.  O stays in
//              TMEM; it is rescaled in place (tcgen05.ld/st) only when a row
//              max grows by more than kRescaleLog2 over the max P is taken
//              against.  S_t(j) being ready (s_full, committed after
//              QK_t(j)) implies PV_t(j-1) completed, so O_t is stable then.
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
constexpr int kRing = 5;                  // K/V tile slots
constexpr int kThreads = 320;
constexpr int TILE_BYTES = 128 * D * 2;   // 32 KB: 128 rows x 128 16-bit values (two 64-col swizzle atoms)
constexpr int HALF_BYTES = 128 * 64 * 2;  // 16 KB: one atom column block
constexpr float kRescaleLog2 = 8.0f;      // O is rescaled when a row max grows by more than 2^8
// P pairs (of the 16 per 32-key chunk) whose exp2 runs on the FMA pipe
// (exp2_fma2) instead of the MUFU: bit u set = pair u.  One MUFU ex2 costs
// 6 cycles per warp per SM sub-partition (measured), so 128 per row per K/V
// tile make the MUFU as busy as the tensor core; a quarter of them on the
// FMA pipe measured fastest (12.5% and 31% were slower).
constexpr uint32_t kEmuPairs = 0x1111u;

struct AttnSmemLayout {
    static constexpr int Q = 0;                         // Q_A, Q_B
    static constexpr int RING = Q + 2 * TILE_BYTES;     // kRing K/V slots
    static constexpr int BAR = RING + kRing * TILE_BYTES;
    static constexpr int BYTES = BAR + 256;
};
static_assert((8 + 2 * kRing) * 8 <= 256, "attention barriers exceed their smem block");
constexpr size_t kAttnSmem = AttnSmemLayout::BYTES + 1024;
static_assert(kAttnSmem <= 232448, "attention smem exceeds the per-CTA limit");

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const void *tmap, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 2^x on the FMA pipe, two at a time: 2^x = 2^n * 2^f with n = rint(x)
// (Cody-Waite range reduction through the 1.5 * 2^23 rounding constant, whose
// sum with x carries n in its low mantissa bits) and f = x - n in [-0.5, 0.5];
// 2^f by the cubic c0 + f (c1 + f (c2 + f c3)), coefficients fitted here as
// the minimax (Lawson-weighted least squares) relative-error polynomial on
// [-0.5, 0.5]: max relative error 7.7e-5, below f16's half ulp (2.4e-4).
// 2^n is added into the exponent field.  x is clamped at -30 first: 2^-30
// rounds to 0 in f16, and the exponent add stays in range.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
    constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
    constexpr float c0 = 0x1.fff682p-1f, c1 = 0x1.62f1e0p-1f, c2 = 0x1.f0e03ap-3f, c3 = 0x1.c46242p-5f;
    x = make_float2(fmaxf(x.x, -30.f), fmaxf(x.y, -30.f));
    const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
    float2 q = __ffma2_rn(make_float2(c3, c3), f, make_float2(c2, c2));
    q = __ffma2_rn(q, f, make_float2(c1, c1));
    q = __ffma2_rn(q, f, make_float2(c0, c0));
    return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
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
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
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
    unsigned char *sRing = smem + AttnSmemLayout::RING;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AttnSmemLayout::BAR);
    uint64_t *q_full = bars + 0;
    uint64_t *slot_full = bars + 1;                 // [kRing]
    uint64_t *slot_empty = bars + 1 + kRing;        // [kRing]
    uint64_t *s_full = bars + 1 + 2 * kRing;        // [2]  tile A, B: QK_t(j) (and every earlier MMA) done
    uint64_t *p_full = bars + 3 + 2 * kRing;        // [2]  P_t(j) stored by all 4 softmax warps
    uint64_t *pv_done = bars + 5 + 2 * kRing;       // [2]  the last PV_t: O_t final
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 7 + 2 * kRing);

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
            constexpr uint32_t idesc_pv = idesc_f16(BQ, D, !VF16, true);   // A = P (TMEM), B = V, MN-major
            const uint32_t q_addr = smem_u32(sQ);
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
            auto issue_pv = [&](int t, int j) {   // O_t (+)= P_t V_j; P_t: TMEM columns 64..127 of S_t
                const uint32_t v_addr = smem_u32(sRing + slot_of(2 * j + 1) * TILE_BYTES);
#pragma unroll
                for (int kk = 0; kk < BKV / 16; ++kk) {   // 16 keys = 8 packed columns per MMA
                    const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, HALF_BYTES, 1024);
                    umma_f16_ts(tmem + 256 + t * 128, tmem + t * 128 + 64 + kk * 8, bd, idesc_pv,
                                (j > 0 || kk > 0) ? 1u : 0u);
                }
            };
            bool ok = mbar_wait(q_full, 0, p.timeout_flag, 205, &aborted) && wait_slot(0, 206);
            if (ok) {
                tc_fence_after();
                issue_qk(0, 0);
                issue_qk(1, 0);
                umma_commit(&slot_empty[slot_of(0)]);   // K_0 read by both
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                // Per tile: PV_t(j) once the softmax has stored P_t(j) (p_full),
                // then QK_t(j+1) into the same columns: MMAs of one thread run
                // in issue order, so P_t(j) is read before S_t(j+1) lands.
                if (!wait_slot(2 * j + 1, 207)) break;
                const bool next = j + 1 < n_kv;
                if (next && !wait_slot(2 * j + 2, 208)) break;
                for (int t = 0; t < 2; ++t) {
                    if (!mbar_wait(&p_full[t], j & 1, p.timeout_flag, 209 + t, &aborted)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(t, j);
                    if (next)
                        issue_qk(t, j + 1);
                    else
                        umma_commit(&pv_done[t]);
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
            if (__any_sync(0xffffffffu, grow)) {
                // O_t and l are relative to m_ref; move them to mx (PV_t(j-1)
                // was issued before QK_t(j), whose completion was waited for).
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
            // pass 2: P = exp2(s * scale - m_ref) (<= 2^kRescaleLog2) in f32; row sum of the f32 values.
            // P is stored as packed 16-bit pairs (key 2c in the low half of
            // column c) into columns 64..127 of S_t: keys 0..63 -> 64..95,
            // keys 64..127 -> 96..127.  Keys 64..127 are already in registers
            // (rh); keys 0..63 are re-read from columns 0..63, which no P
            // store touches.
            const float2 nm2 = make_float2(-m_ref, -m_ref);
            float2 sum2 = make_float2(0.f, 0.f);
            auto p_store = [&](const uint32_t (&r)[32], uint32_t col) {   // 32 keys -> 16 columns
                uint32_t pk[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[2 * u]), __uint_as_float(r[2 * u + 1])),
                                                sl2, nm2);
                    const float2 pf = ((kEmuPairs >> u) & 1u) ? exp2_fma2(x) : make_float2(ex2(x.x), ex2(x.y));
                    sum2 = __fadd2_rn(sum2, pf);
                    if constexpr (VF16) {
                        uint32_t out;
                        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(pf.y), "f"(pf.x));
                        pk[u] = out;
                    } else {
                        __nv_bfloat162 hv = __floats2bfloat162_rn(pf.x, pf.y);
                        pk[u] = *reinterpret_cast<uint32_t *>(&hv);
                    }
                }
                tmem_st_32x32b_x16(s_tmem + col, pk);
            };
            {
                uint32_t r0[2][32];
                tmem_ld_32x32b_x32(s_tmem + 0, r0[0]);
                tmem_ld_32x32b_x32(s_tmem + 32, r0[1]);
                p_store(rh[0], 96);
                p_store(rh[1], 112);
                tmem_ld_wait_regs(r0[0]);
                tmem_ld_wait_regs(r0[1]);
                if (ragged) {
#pragma unroll
                    for (int e = 0; e < 64; ++e)
                        if (kv0 + e >= p.Tk) r0[e >> 5][e & 31] = __float_as_uint(-INFINITY);
                }
                p_store(r0[0], 64);
                p_store(r0[1], 80);
            }
            l += sum2.x + sum2.y;
            tmem_st_wait();             // P_t(j) in TMEM ...
            tc_fence_before();          // ... and ordered before the arrive for the MMA thread
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
        }
        // O_t is final once the last P.V has completed.
        if (!aborted && warp_wait(&pv_done[t], 0, p.timeout_flag, 212, &aborted)) {   // one commit per tile
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
