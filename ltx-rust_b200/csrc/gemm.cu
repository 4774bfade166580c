// K2: C[M,N] = A[M,K] . W[N,K]^T on the 5th-generation tensor cores, with
// the DiT's linear-layer epilogues fused.  Replaces Burn `Linear::forward`
// for every projection of the block (crates/ltx-dit/src/attention.rs:150-152,
// :194, feed_forward.rs:38-42, model.rs:187, :254, adaln.rs:84-88, :130-142).
//
// Design (sm_100a, one CTA per SM, persistent):
//   warp 0      TMA producer: 128x64 A tile + BNx64 W tile per stage,
//               128-byte swizzle, STAGES-deep ring of mbarriers.
//   warp 1      one thread issues tcgen05.mma (M=128, N=BN, K=16) x 4 per
//               stage into a TMEM accumulator; tcgen05.commit frees the stage.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (one row per
//               thread), fused bias / GELU(tanh) / gated residual, store.
//   Two TMEM accumulators (2 x BN columns) let the epilogue of tile i run
//   under the mainloop of tile i+1.  Tiles are walked in groups of M-blocks
//   whose A panel fits ~48 MB of L2, so W is streamed once per group.
// Each CTA loads its own tiles from local HBM; no load is shared across a cluster.
#include <cuda.h>

#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

enum GemmEpilogue : int {
    EPI_BF16 = 0,        // out_bf16 = acc + bias
    EPI_GELU_BF16 = 1,   // out_bf16 = gelu_tanh(acc + bias)
    EPI_F32 = 2,         // out_f32 = acc + bias
    EPI_RESID = 3,       // x_f32 += (acc + bias) * gate[gidx[row]][col]   (gate optional)
    EPI_TP_RESID = 4,    // EPI_RESID with acc summed over the tensor-parallel ranks (gemm_tp_resid)
};

struct GemmParams {
    int M, N, K;
    const float *a_scale;   // FP8 operands: per-row scale of A [M] (null = 1)
    float w_scale;          // FP8 operands: per-tensor scale of W
    const float *bias;      // [N] or null
    void *out;              // bf16 / f32 [M, ldo]
    int64_t ldo;
    const float *gate;      // [U, ld_gate] or null (EPI_RESID)
    const int *gate_idx;    // [M] row -> gate row (EPI_RESID, null = row 0)
    int64_t ld_gate;
    int *timeout_flag;
    int f16_from_col;       // EPI_BF16: columns >= this are written as f16 (N = none)
    int group_m;            // M-blocks walked together (their A panel stays in L2)
    int k2_blocks;          // FP8 only: bf16 K-blocks of 64 appended to every tile
                            // (A2 [M, 64*k2] . B2 [N, 64*k2]^T, same accumulator)
    const float *w_col_scale;   // FP8 only: per-column weight scale [N] (null = w_scale)
    int resid_tma;          // EPI_RESID: the residual moves by TMA through shared memory (tmX)
    int m_rot;              // M-blocks are walked from this one on, wrapping (0: natural order)
    // A rows gathered from other ranks (TpGather): the producer waits for the
    // owner's stamp of an M-block before loading its A tiles (ag_stamp null: no wait)
    const uint32_t *ag_stamp;
    uint32_t ag_epoch;
    int ag_n, ag_me, ag_mcap;
    int tp_bcast;           // EPI_TP_RESID: 1 = write finished rows into every other rank's x too
    // EPI_TP_RESID: this rank, the ranks, this launch's epoch and the peer
    // memory (every rank's base as mapped here; the offsets of ltx::TpPeerMem)
    int tp_rank, tp_size;
    uint32_t epoch;
    int64_t rows_cap, tiles_cap;
    size_t recv_off, tstamp_off, dstamp_off, count_off;
    char *peer[kMaxTpPeers];
};

namespace {

constexpr int BM = 128;
constexpr size_t kGroupPanelBytes = 48u << 20;   // A panel kept in L2 while W streams past it
constexpr int kThreads = 192;
// EPI_RESID staging: two 128-row x 32-column f32 chunks of the residual,
// 128-byte swizzled, filled and drained by TMA.
constexpr int kXChunkBytes = BM * 32 * 4;
constexpr int kXStageBytes = 2 * kXChunkBytes;
// EPI_TP_RESID staging: per epilogue warp, its 32 rows x 32 columns of f32.
constexpr int kTpStageBytes = 4 * 32 * 32 * 4;

// F8: e4m3 operands (kind::f8f6f4), 128 elements of K per stage; otherwise
// bf16 (kind::f16), 64 per stage.  Either way a stage row is one 128-byte
// swizzle row, so the tile bytes, the descriptors and the 4 MMAs per stage
// (K = 32 e4m3 or 16 bf16 each, +32 bytes apart) are the same.
template <int BN, bool F8 = false>
struct GemmCfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int BKE = F8 ? 128 : 64;   // K elements per stage
    static constexpr int A_BYTES = BM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = 2 * BN;  // power of two >= 32
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
};

__device__ __forceinline__ float gelu_tanh(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))  (feed_forward.rs:31-32)
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(u));
}

// Tile t -> (M-block, N-block): groups of group_m M-blocks, M fastest inside a
// group, so the ~148 tiles in flight share a few W panels and one A panel, and
// W is streamed from DRAM once per group.
// m_rot rotates the M-block order (the tensor-parallel exchange walks the
// other ranks' rows first and its own last).
__device__ __forceinline__ void tile_coords(int t, int m_blocks, int n_blocks, int group_m, int m_rot, int &mb,
                                            int &nb) {
    const int per_group = group_m * n_blocks;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int gm = min(group_m, m_blocks - first_m);
    const int r = t - g * per_group;
    mb = first_m + r % gm + m_rot;
    if (mb >= m_blocks) mb -= m_blocks;
    nb = r / gm;
}

// Tensor-parallel row ownership: rank r owns M-blocks [lo(r), lo(r+1)),
// lo(r) = r * m_blocks / n.
__host__ __device__ __forceinline__ int tp_lo(int r, int m_blocks, int n) { return (int)((int64_t)r * m_blocks / n); }
__device__ __forceinline__ int tp_owner(int mb, int m_blocks, int n) {
    int o = 0;
    while (o + 1 < n && mb >= tp_lo(o + 1, m_blocks, n)) ++o;
    return o;
}

__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int BN, int EPI, bool F8>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                const __grid_constant__ CUtensorMap tmX, GemmParams p) {
    using C = GemmCfg<BN, F8>;
    constexpr int XS = EPI == EPI_RESID ? kXStageBytes : EPI == EPI_TP_RESID ? kTpStageBytes : 0;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char *sA = smem;
    unsigned char *sB = smem + C::STAGES * C::A_BYTES;
    float *xs = reinterpret_cast<float *>(smem + C::STAGES * C::STAGE_BYTES);   // EPI_RESID staging (XS bytes)
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES + XS);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *xfull = tempty + 2;   // [2] residual chunk landed (EPI_RESID with resid_tma)
    uint64_t *xdone = xfull + 2;    // [2] the 128 epilogue threads have written it back
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xdone + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_blocks = (p.M + BM - 1) / BM, n_blocks = (p.N + BN - 1) / BN;
    const int num_tiles = m_blocks * n_blocks;
    const int k_blocks = (p.K + C::BKE - 1) / C::BKE;
    const int k2_blocks = F8 ? p.k2_blocks : 0;
    const int k_total = k_blocks + k2_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
            mbar_init(&xfull[a], 1);
            mbar_init(&xdone[a], 128);
        }
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    bool aborted = false;

    if (warp == 0) {
        if (elect_one()) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            if (k2_blocks) {
                tma_prefetch_desc(&tmA2);
                tma_prefetch_desc(&tmB2);
            }
            uint32_t it = 0;
            int ag_ready = -1;   // the last M-block whose gathered rows are known to be here
            for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x) {
                int mb, nb;
                tile_coords(t, m_blocks, n_blocks, p.group_m, p.m_rot, mb, nb);
                if (p.ag_stamp && mb != ag_ready) {
                    const int o = tp_owner(mb, m_blocks, p.ag_n);
                    if (o != p.ag_me) {
                        const uint32_t *f = p.ag_stamp + (int64_t)(o < p.ag_me ? o : o - 1) * p.ag_mcap + mb;
                        const uint64_t t0 = global_ns();
                        while (!stamp_reached(ld_acquire_sys(f), p.ag_epoch)) {
                            if (global_ns() - t0 > kWaitLimitNs) {
                                atomicExch(p.timeout_flag, 110);
                                aborted = true;
                                break;
                            }
                            __nanosleep(64);
                        }
                        if (aborted) break;
                        // rows another GPU wrote (generic proxy), read next by TMA (async proxy)
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                    }
                    ag_ready = mb;
                }
                for (int kb = 0; kb < k_total; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, p.timeout_flag, 101, &aborted)) break;
                    mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                    if (kb < k_blocks) {
                        tma_load_2d(sA + s * C::A_BYTES, &tmA, &full[s], kb * C::BKE, mb * BM);
                        tma_load_2d(sB + s * C::B_BYTES, &tmB, &full[s], kb * C::BKE, nb * BN);
                    } else {   // appended bf16 block: 64 elements = one 128-byte row
                        tma_load_2d(sA + s * C::A_BYTES, &tmA2, &full[s], (kb - k_blocks) * 64, mb * BM);
                        tma_load_2d(sB + s * C::B_BYTES, &tmB2, &full[s], (kb - k_blocks) * 64, nb * BN);
                    }
                }
            }
            if (aborted) {
                // Let the copies already issued land before the CTA exits.
                bool a2 = false;
                for (uint32_t j = it > (uint32_t)C::STAGES ? it - C::STAGES : 0; j < it; ++j)
                    mbar_wait(&full[j % C::STAGES], (j / C::STAGES) & 1, nullptr, 0, &a2);
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = F8 ? idesc_e4m3(BM, BN) : idesc_f16(BM, BN, true);
            constexpr uint32_t idesc_bf16 = idesc_f16(BM, BN, true);
            uint32_t it = 0, tile_i = 0;
            for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tile_i) {
                const uint32_t acc = tile_i & 1, aph = (tile_i >> 1) & 1;
                if (!mbar_wait(&tempty[acc], aph ^ 1, p.timeout_flag, 102, &aborted)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < k_total; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t ph = (it / C::STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, p.timeout_flag, 103, &aborted)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
                    const bool main_k = kb < k_blocks;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sdesc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(b_addr + kk * 32, 16, 1024);
                        if constexpr (F8) {
                            if (main_k)
                                umma_f8_ss(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
                            else   // appended bf16 block: both operands bf16 (kind::f16)
                                umma_f16_ss(d_tmem, ad, bd, idesc_bf16, 1u);
                        } else {
                            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
                        }
                    }
                    umma_commit(&empty[s]);
                }
                if (aborted) break;
                umma_commit(&tfull[acc]);
            }
        }
    } else if (EPI == EPI_RESID && p.resid_tma) {
        // Residual epilogue through shared memory: per 32-column chunk, one
        // elected thread TMA-loads x[128 rows][32 cols] into a staging buffer
        // (the next chunk's load is in flight while this one is processed),
        // every thread updates its row there, and the elected thread TMA-stores
        // the chunk back.  Global traffic moves in whole lines instead of one
        // 16-byte piece of 32 different rows per instruction.
        const int quad = warp & 3;
        const int erow = quad * 32 + lane;   // row within the tile (TMEM lane)
        const bool elected = warp == 2 && lane == 0;
        uint32_t u = 0;                       // staging uses so far: buffer u & 1, phase (u >> 1) & 1
        uint32_t issued = 0;                  // uses whose load the elected thread has started
        auto load_chunk = [&](uint32_t uu, int mb, int nb, int c) {   // elected thread only
            bulk_wait_read0();                // earlier stores have finished reading their buffers
            issued = uu + 1;
            const int b = uu & 1;
            mbar_arrive_expect_tx(&xfull[b], kXChunkBytes);
            tma_load_2d(xs + b * (kXChunkBytes / 4), &tmX, &xfull[b], nb * BN + c * 32, mb * BM);
        };
        uint32_t tile_i = 0;
        for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tile_i) {
            int mb, nb;
            tile_coords(t, m_blocks, n_blocks, p.group_m, p.m_rot, mb, nb);
            const uint32_t acc = tile_i & 1, aph = (tile_i >> 1) & 1;
            if (elected) load_chunk(u, mb, nb, 0);   // under this tile's mainloop
            __syncwarp();
            if (!warp_wait(&tfull[acc], aph, p.timeout_flag, 104, &aborted)) break;
            tc_fence_after();
            const int row = mb * BM + erow;
            const bool row_ok = row < p.M;
            const float *gate_row = nullptr;
            if (p.gate) gate_row = p.gate + (int64_t)(p.gate_idx && row_ok ? p.gate_idx[row] : 0) * p.ld_gate;
            const float sa = F8 && p.a_scale && row_ok ? __ldg(p.a_scale + row) : 1.0f;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c, ++u) {
                if (elected && c + 1 < BN / 32) load_chunk(u + 1, mb, nb, c + 1);
                __syncwarp();
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
                tmem_ld_wait();
                const int b = u & 1;
                const uint32_t ph = (u >> 1) & 1;
                if (!warp_wait(&xfull[b], ph, p.timeout_flag, 106, &aborted)) break;
                const int col0 = nb * BN + c * 32;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                if constexpr (F8) {
                    // acc is in units of (row scale x weight scale)
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] *= sa * (p.w_col_scale ? (col0 + j < p.N ? __ldg(p.w_col_scale + col0 + j) : 0.f)
                                                    : p.w_scale);
                }
                if (p.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
                }
                // row erow of the 128-byte swizzled chunk: 16-byte piece q sits at q ^ (erow % 8)
                float4 *xr = reinterpret_cast<float4 *>(xs + b * (kXChunkBytes / 4) + erow * 32);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int pos = q ^ (erow & 7);
                    float4 x = xr[pos];
                    float g[4] = {1.f, 1.f, 1.f, 1.f};
                    if (gate_row) {
                        if (col0 + 4 * q + 4 <= p.N) {
                            const float4 g4 = __ldg(reinterpret_cast<const float4 *>(gate_row + col0 + 4 * q));
                            g[0] = g4.x; g[1] = g4.y; g[2] = g4.z; g[3] = g4.w;
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) g[e] = col0 + 4 * q + e < p.N ? gate_row[col0 + 4 * q + e] : 0.f;
                        }
                    }
                    x.x += v[4 * q] * g[0];
                    x.y += v[4 * q + 1] * g[1];
                    x.z += v[4 * q + 2] * g[2];
                    x.w += v[4 * q + 3] * g[3];
                    xr[pos] = x;
                }
                fence_proxy_async_smem();   // the writes above, visible to the TMA store
                mbar_arrive(&xdone[b]);
                if (elected) {
                    if (mbar_wait(&xdone[b], ph, p.timeout_flag, 107, &aborted)) {
                        tma_store_2d(&tmX, xs + b * (kXChunkBytes / 4), col0, mb * BM);
                        bulk_commit();
                    }
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        if (elected) {
            // Before the CTA exits: loads an abort left unconsumed have landed
            // (bounded waits), and every store has completed.
            bool quiet = false;
            for (uint32_t uu = u; uu < issued; ++uu) mbar_wait(&xfull[uu & 1], (uu >> 1) & 1, nullptr, 0, &quiet);
            bulk_wait_all();
        }
    } else if (EPI == EPI_TP_RESID) {
        // Row-split projection of a model split over n ranks, with the sum over
        // ranks fused in: every rank computes a partial product of every tile.
        // Rank r owns the rows of M-blocks [lo(r), lo(r+1)) and walks them last.
        //  - a tile it does not own: the partial goes, as bf16, straight into
        //    the owner's receive area over NVLink (its slot among the owner's
        //    n-1 sources), then a per-warp stamp (this launch's epoch) tells the
        //    owner those 32 rows have landed;
        //  - a tile it owns: once the other ranks' stamps for these rows are in
        //    (bounded wait), acc + their partials (in slot order) + bias, gated,
        //    update the residual x here and in every other rank's x, so the
        //    replicas stay identical bit for bit.
        // Each warp moves its 32 rows through shared memory so that global
        // and NVLink traffic is row-contiguous (8 lanes per 128-byte row).
        const int quad = warp & 3;
        float *stg = xs + quad * 32 * 32;
        const int n = p.tp_size, me = p.tp_rank;
        float *x_loc = static_cast<float *>(p.out);
        uint32_t tile_i = 0;
        for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tile_i) {
            int mb, nb;
            tile_coords(t, m_blocks, n_blocks, p.group_m, p.m_rot, mb, nb);
            const uint32_t acc = tile_i & 1, aph = (tile_i >> 1) & 1;
            if (!warp_wait(&tfull[acc], aph, p.timeout_flag, 104, &aborted)) break;
            tc_fence_after();
            const int owner = tp_owner(mb, m_blocks, n);
            const int64_t tile = (int64_t)mb * n_blocks + nb;
            const int row_base = mb * BM + quad * 32;
            if (owner == me) {
                bool ok = true;
                const uint32_t *ts = reinterpret_cast<const uint32_t *>(p.peer[me] + p.tstamp_off);
                const uint64_t t0 = global_ns();
                for (int sl = 0; sl < n - 1 && ok; ++sl) {
                    const uint32_t *f = ts + ((int64_t)sl * p.tiles_cap + tile) * 4 + quad;
                    while (!stamp_reached(ld_acquire_sys(f), p.epoch)) {
                        if (global_ns() - t0 > kWaitLimitNs) {
                            ok = false;
                            break;
                        }
                        __nanosleep(32);
                    }
                }
                if (!__all_sync(0xffffffffu, ok)) {
                    if (lane == 0) atomicExch(p.timeout_flag, 108);
                    aborted = true;
                    break;
                }
            }
            const int slot = me < owner ? me : me - 1;   // this rank among the owner's sources
            const int q = lane & 7;
            // owned rows: lane l holds the gate table row of this warp's row l
            const int gidx_lane =
                owner == me && p.gate && p.gate_idx && row_base + lane < p.M ? p.gate_idx[row_base + lane] : 0;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
                tmem_ld_wait();
                // lane = row: 16-byte piece j of the row sits at j ^ (row % 8)
                float4 *srow = reinterpret_cast<float4 *>(stg + lane * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    srow[j ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                       __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                __syncwarp();
                const int col = nb * BN + c * 32 + 4 * q;
                // lane -> rows i*4 + lane/8 (i < 8) of this warp's 32, columns col..col+3
                float4 v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int rl = i * 4 + (lane >> 3);
                    v[i] = reinterpret_cast<const float4 *>(stg + rl * 32)[q ^ (rl & 7)];
                }
                if (owner == me) {
                    // every load of the chunk is issued before the first use
                    float4 xv[8], g[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rl = i * 4 + (lane >> 3);
                        const int row = row_base + rl;
                        const int gi = __shfl_sync(0xffffffffu, gidx_lane, rl);
                        xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                        g[i] = make_float4(1.f, 1.f, 1.f, 1.f);
                        if (row < p.M) {
                            xv[i] = *reinterpret_cast<const float4 *>(x_loc + (int64_t)row * p.ldo + col);
                            if (p.gate)
                                g[i] = __ldg(reinterpret_cast<const float4 *>(p.gate + (int64_t)gi * p.ld_gate + col));
                        }
                    }
                    const __nv_bfloat16 *rcv = reinterpret_cast<const __nv_bfloat16 *>(p.peer[me] + p.recv_off);
                    for (int sl = 0; sl < n - 1; ++sl) {   // partials added in slot (rank) order
                        uint2 u[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int row = row_base + i * 4 + (lane >> 3);
                            u[i] = row < p.M ? __ldcg(reinterpret_cast<const uint2 *>(
                                                   rcv + ((int64_t)sl * p.rows_cap + row) * p.N + col))
                                             : make_uint2(0u, 0u);
                        }
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u[i].x));
                            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u[i].y));
                            v[i].x += a.x;
                            v[i].y += a.y;
                            v[i].z += b.x;
                            v[i].w += b.y;
                        }
                    }
                    const float4 b4 =
                        p.bias ? __ldg(reinterpret_cast<const float4 *>(p.bias + col)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int row = row_base + i * 4 + (lane >> 3);
                        if (row >= p.M) continue;
                        if (p.bias) {
                            v[i].x += b4.x;
                            v[i].y += b4.y;
                            v[i].z += b4.z;
                            v[i].w += b4.w;
                        }
                        float4 x = xv[i];
                        x.x += v[i].x * g[i].x;
                        x.y += v[i].y * g[i].y;
                        x.z += v[i].z * g[i].z;
                        x.w += v[i].w * g[i].w;
                        const int64_t xo = (int64_t)row * p.ldo + col;
                        *reinterpret_cast<float4 *>(x_loc + xo) = x;
                        if (p.tp_bcast)
                            for (int pr = 0; pr < n; ++pr)
                                if (pr != me) *reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.peer[pr]) + xo) = x;
                    }
                } else {
                    __nv_bfloat16 *dst0 = reinterpret_cast<__nv_bfloat16 *>(p.peer[owner] + p.recv_off) +
                                          (int64_t)slot * p.rows_cap * p.N + col;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int row = row_base + i * 4 + (lane >> 3);
                        if (row >= p.M) continue;
                        const __nv_bfloat162 lo2 = __floats2bfloat162_rn(v[i].x, v[i].y),
                                             hi2 = __floats2bfloat162_rn(v[i].z, v[i].w);
                        *reinterpret_cast<uint2 *>(dst0 + (int64_t)row * p.N) =
                            make_uint2(*reinterpret_cast<const uint32_t *>(&lo2), *reinterpret_cast<const uint32_t *>(&hi2));
                    }
                }
                __syncwarp();
            }
            if (owner != me) {
                __threadfence_system();   // these rows' pushes, before their stamp
                __syncwarp();
                if (lane == 0)
                    st_release_sys(reinterpret_cast<uint32_t *>(p.peer[owner] + p.tstamp_off) +
                                       ((int64_t)slot * p.tiles_cap + tile) * 4 + quad,
                                   p.epoch);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
        __threadfence_system();   // every push of this warp, before the CTA reports done
    } else {
        // Epilogue warps 2..5 own TMEM lane quadrant (warp % 4).
        const int quad = warp & 3;
        uint32_t tile_i = 0;
        for (int t = blockIdx.x; t < num_tiles && !aborted; t += gridDim.x, ++tile_i) {
            int mb, nb;
            tile_coords(t, m_blocks, n_blocks, p.group_m, p.m_rot, mb, nb);
            const uint32_t acc = tile_i & 1, aph = (tile_i >> 1) & 1;
            // warp-uniform outcome: the tcgen05.ld below are warp-collective
            if (!warp_wait(&tfull[acc], aph, p.timeout_flag, 104, &aborted)) break;
            tc_fence_after();
            const int row = mb * BM + quad * 32 + lane;
            const bool row_ok = row < p.M;
            const float *gate_row = nullptr;
            if (EPI == EPI_RESID && p.gate) gate_row = p.gate + (int64_t)(p.gate_idx && row_ok ? p.gate_idx[row] : 0) * p.ld_gate;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + c * 32, r);
                tmem_ld_wait();
                const int col0 = nb * BN + c * 32;
                if (!row_ok || col0 >= p.N) continue;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                const bool full_cols = col0 + 32 <= p.N;
                if constexpr (F8) {
                    // acc is in units of (row scale x weight scale)
                    const float sa = p.a_scale ? __ldg(p.a_scale + row) : 1.0f;
                    if (p.w_col_scale) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            v[j] *= sa * ((full_cols || col0 + j < p.N) ? __ldg(p.w_col_scale + col0 + j) : 0.f);
                    } else {
                        const float sc = sa * p.w_scale;
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] *= sc;
                    }
                }
                if (p.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (full_cols || col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
                }
                if constexpr (EPI == EPI_BF16 || EPI == EPI_GELU_BF16) {
                    if constexpr (EPI == EPI_GELU_BF16) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
                    }
                    __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + (int64_t)row * p.ldo + col0;
                    // 32-column chunks never straddle f16_from_col (a multiple of 32 when used).
                    const bool as_f16 = EPI == EPI_BF16 && col0 >= p.f16_from_col;
                    if (full_cols && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                if (as_f16) {
                                    __half2 h = __floats2half2_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
                                    w[e] = *reinterpret_cast<uint32_t *>(&h);
                                } else {
                                    __nv_bfloat162 h = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
                                    w[e] = *reinterpret_cast<uint32_t *>(&h);
                                }
                            }
                            *reinterpret_cast<uint4 *>(o + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.N) {
                                if (as_f16)
                                    reinterpret_cast<__half *>(o)[j] = __float2half_rn(v[j]);
                                else
                                    o[j] = __float2bfloat16_rn(v[j]);
                            }
                    }
                } else if constexpr (EPI == EPI_F32) {
                    float *o = static_cast<float *>(p.out) + (int64_t)row * p.ldo + col0;
                    if (full_cols && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            *reinterpret_cast<float4 *>(o + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.N) o[j] = v[j];
                    }
                } else {  // EPI_RESID
                    float *o = static_cast<float *>(p.out) + (int64_t)row * p.ldo + col0;
                    if (full_cols && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float4 x = *reinterpret_cast<float4 *>(o + 4 * q);
                            float g[4] = {1.f, 1.f, 1.f, 1.f};
                            if (gate_row) {
                                const float4 g4 = __ldg(reinterpret_cast<const float4 *>(gate_row + col0 + 4 * q));
                                g[0] = g4.x; g[1] = g4.y; g[2] = g4.z; g[3] = g4.w;
                            }
                            x.x += v[4 * q] * g[0];
                            x.y += v[4 * q + 1] * g[1];
                            x.z += v[4 * q + 2] * g[2];
                            x.w += v[4 * q + 3] * g[3];
                            *reinterpret_cast<float4 *>(o + 4 * q) = x;
                        }
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < p.N) o[j] += v[j] * (gate_row ? gate_row[col0 + j] : 1.f);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
    if constexpr (EPI == EPI_TP_RESID) {
        // The last CTA to finish tells every other rank that all of this
        // rank's pushes of this launch have landed (its done stamp there).
        if (threadIdx.x == 0) {
            __threadfence_system();
            uint32_t *count = reinterpret_cast<uint32_t *>(p.peer[p.tp_rank] + p.count_off);
            if (atomicAdd(count, 1u) + 1 == gridDim.x) {
                atomicExch(count, 0u);
                __threadfence_system();
                for (int pr = 0; pr < p.tp_size; ++pr)
                    if (pr != p.tp_rank)
                        st_release_sys(reinterpret_cast<uint32_t *>(p.peer[pr] + p.dstamp_off) +
                                           (p.tp_rank < pr ? p.tp_rank : p.tp_rank - 1),
                                       p.epoch);
            }
        }
    }
}

// Rank barrier on the stream: stamps `epoch` into every other rank's slot for
// this rank, then waits (bounded; code 111) for every other rank's stamp here.
struct TpBarrierArgs {
    uint32_t *peer_bstamp[kMaxTpPeers];   // every rank's barrier stamps [n-1]
    int n, me;
    uint32_t epoch;
    int *timeout_flag;
};
__global__ void tp_barrier_kernel(TpBarrierArgs a) {
    const int s = threadIdx.x;
    if (blockIdx.x != 0) return;
    if (s < a.n && s != a.me) st_release_sys(a.peer_bstamp[s] + (a.me < s ? a.me : a.me - 1), a.epoch);
    if (s >= a.n - 1) return;
    const uint32_t *own = a.peer_bstamp[a.me] + s;
    const uint64_t t0 = global_ns();
    while (!stamp_reached(ld_acquire_sys(own), a.epoch)) {
        if (global_ns() - t0 > kWaitLimitNs) {
            atomicExch(a.timeout_flag, 111);
            return;
        }
        __nanosleep(64);
    }
}

// Holds the stream until every other rank's fused projection of this epoch
// has finished pushing into this rank's memory (bounded; code 109 on timeout).
__global__ void tp_wait_kernel(const uint32_t *dstamp, int slots, uint32_t epoch, int *timeout_flag) {
    const int s = threadIdx.x;
    if (blockIdx.x != 0 || s >= slots) return;
    const uint64_t t0 = global_ns();
    while (!stamp_reached(ld_acquire_sys(dstamp + s), epoch)) {
        if (global_ns() - t0 > kWaitLimitNs) {
            atomicExch(timeout_flag, 109);
            return;
        }
        __nanosleep(64);
    }
}

// ── host side ────────────────────────────────────────────────────────────────

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 2-D row-major [rows, cols] of 1- or 2-byte elements with leading dimension
// ld (elements); the box is one 128-byte swizzle row wide: {128 / es, box_rows}.
bool make_tmap_2d(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, int es) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / es), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, es == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr),
              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D row-major f32 [rows, cols] with leading dimension ld (elements), box
// {box_cols, box_rows}, 128-byte swizzle (box_cols * 4 must be 128).
bool make_tmap_f32(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                   int box_cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || box_cols * 4 != 128) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr ? const_cast<void *>(ptr) : nullptr, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI, bool F8>
cudaError_t launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &ta2, const CUtensorMap &tb2,
                        const CUtensorMap &tx, const GemmParams &p, int sms, cudaStream_t st) {
    using C = GemmCfg<BN, F8>;
    constexpr size_t smem =
        C::SMEM + (EPI == EPI_RESID ? kXStageBytes : EPI == EPI_TP_RESID ? kTpStageBytes : 0);
    static_assert(smem <= 232448, "GEMM shared memory exceeds the per-CTA limit");
    auto k = gemm_kernel<BN, EPI, F8>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    const int grid = std::min(tiles, sms);
    if constexpr (EPI == EPI_TP_RESID) {
        // Its CTAs wait on other GPUs' CTAs, which wait on this GPU's: every CTA
        // must be resident at once, which a cooperative launch guarantees (or refuses).
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, k, ta, tb, ta2, tb2, tx, p);
    }
    k<<<grid, kThreads, smem, st>>>(ta, tb, ta2, tb2, tx, p);
    return cudaGetLastError();
}

template <int BN, bool F8>
cudaError_t dispatch_epi(int epi, const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &ta2,
                         const CUtensorMap &tb2, const CUtensorMap &tx, const GemmParams &p, int sms, cudaStream_t st) {
    switch (epi) {
    case EPI_BF16: return launch_gemm<BN, EPI_BF16, F8>(ta, tb, ta2, tb2, tx, p, sms, st);
    case EPI_GELU_BF16: return launch_gemm<BN, EPI_GELU_BF16, F8>(ta, tb, ta2, tb2, tx, p, sms, st);
    case EPI_F32: return launch_gemm<BN, EPI_F32, F8>(ta, tb, ta2, tb2, tx, p, sms, st);
    default: return launch_gemm<BN, EPI_RESID, F8>(ta, tb, ta2, tb2, tx, p, sms, st);
    }
}

// Shared by the bf16 and e4m3 entry points: es = element bytes (2 or 1).
// e4m3 only: `lr` appends k2 bf16 K-elements (A2 [M, k2] . B2 [N, k2]^T).
int gemm_any(ltx_ctx *ctx, cudaStream_t st, int es, const void *A, int64_t lda, const float *a_scale, const void *W,
             int64_t ldw, float w_scale, int M, int N, int K, int epi, const float *bias, void *out, int64_t ldo,
             const float *gate, const int *gate_idx, int64_t ld_gate, int f16_from_col, const GemmLowRank *lr = nullptr,
             const float *w_col_scale = nullptr, const TpGather *ag = nullptr) {
    if (!A || !W || !out) return fail(ctx, LTX_ERR_INVALID_ARG, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return fail(ctx, LTX_ERR_SHAPE, "gemm: empty shape %d x %d x %d", M, N, K);
    const int align = 16 / es;   // elements per 16 bytes (TMA strides and the innermost coordinate)
    if (lda % align || ldw % align || lda < K || ldw < K || ((uintptr_t)A & 15) || ((uintptr_t)W & 15))
        return fail(ctx, LTX_ERR_SHAPE, "gemm: operands need 16-byte aligned rows (lda %lld ldw %lld)", (long long)lda,
                    (long long)ldw);
    if (epi < EPI_BF16 || epi > EPI_RESID) return fail(ctx, LTX_ERR_INVALID_ARG, "gemm: bad epilogue %d", epi);
    if (epi == EPI_RESID && gate && (((uintptr_t)gate & 15) || ld_gate % 4))
        return fail(ctx, LTX_ERR_SHAPE, "gemm: gate rows must be 16-byte aligned (ld_gate %lld)", (long long)ld_gate);
    const int BN = N <= 128 ? 128 : 256;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, M, K, lda, BM, es) || !make_tmap_2d(&tb, W, N, K, ldw, BN, es))
        return fail(ctx, LTX_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed");
    CUtensorMap ta2 = ta, tb2 = tb;   // unused unless a low-rank block is appended
    int k2_blocks = 0;
    if (lr && lr->k2 > 0) {
        if (es != 1 || lr->k2 % 64 || !lr->a2 || !lr->b2 || lr->lda2 % 8 || lr->ldb2 % 8 || lr->lda2 < lr->k2 ||
            lr->ldb2 < lr->k2 || ((uintptr_t)lr->a2 & 15) || ((uintptr_t)lr->b2 & 15))
            return fail(ctx, LTX_ERR_SHAPE, "gemm: appended bf16 block needs e4m3 operands and k2 a multiple of 64");
        if (!make_tmap_2d(&ta2, lr->a2, M, lr->k2, lr->lda2, BM, 2) || !make_tmap_2d(&tb2, lr->b2, N, lr->k2, lr->ldb2, BN, 2))
            return fail(ctx, LTX_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (appended block)");
        k2_blocks = lr->k2 / 64;
    }
    if (f16_from_col < 0 || f16_from_col > N) f16_from_col = N;
    if (f16_from_col < N && (epi != EPI_BF16 || f16_from_col % 32))
        return fail(ctx, LTX_ERR_INVALID_ARG, "gemm: f16 columns need the bf16 epilogue and a multiple of 32");
    // as many M-blocks per group as keep their A panel within ~48 MB of L2
    const int m_blocks = (M + BM - 1) / BM;
    const size_t panel = (size_t)BM * K * es;
    // A weight that fits in that budget itself stays in L2 whatever the order:
    // then the N-blocks of one M-block run back to back (group_m = 1) and
    // every A panel is read from DRAM once.
    const size_t w_bytes = (size_t)N * K * es;
    const int group_m = w_bytes <= kGroupPanelBytes
                            ? 1
                            : (int)std::max<size_t>(1, std::min<size_t>((size_t)m_blocks, kGroupPanelBytes / panel));
    GemmParams p{M,   N,    K,        a_scale, w_scale,           bias,         out,     ldo,       gate,
                 gate_idx, ld_gate, ctx->timeout_flag, f16_from_col, group_m, k2_blocks, w_col_scale};
    if (ag && ag->stamp && ag->n > 1) {
        // gathered A rows: this rank's own rows first, the others' as they arrive
        p.ag_stamp = ag->stamp;
        p.ag_epoch = ag->epoch;
        p.ag_n = ag->n;
        p.ag_me = ag->me;
        p.ag_mcap = ag->mcap;
        if (m_blocks > ag->mcap) return fail(ctx, LTX_ERR_SHAPE, "gemm: more M-blocks than the gather stamps");
        p.m_rot = tp_lo(ag->me, m_blocks, ag->n);
    }
    // EPI_RESID: the residual x [M, ldo] f32 as a TMA map with 128 x 32 boxes
    // (rows 16-byte aligned); otherwise the epilogue updates it with plain loads.
    CUtensorMap tx = ta;
    if (epi == EPI_RESID && ((uintptr_t)out & 15) == 0 && ldo % 4 == 0 && ldo >= N) {
        if (!make_tmap_f32(&tx, out, M, N, ldo, BM, 32))
            return fail(ctx, LTX_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (residual)");
        p.resid_tma = 1;
    }
    cudaError_t e;
    const int sms = ctx->gemm_sms > 0 ? std::min(ctx->gemm_sms, ctx->sm_count) : ctx->sm_count;
    if (es == 1)
        e = BN == 128 ? dispatch_epi<128, true>(epi, ta, tb, ta2, tb2, tx, p, sms, st)
                      : dispatch_epi<256, true>(epi, ta, tb, ta2, tb2, tx, p, sms, st);
    else
        e = BN == 128 ? dispatch_epi<128, false>(epi, ta, tb, ta2, tb2, tx, p, sms, st)
                      : dispatch_epi<256, false>(epi, ta, tb, ta2, tb2, tx, p, sms, st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gemm launch");
    return LTX_OK;
}

}  // namespace

// x += (sum over ranks of A_r . W_r^T + bias) * gate on every rank of the
// communicator, in one launch per rank plus a wait: the row-split projection
// of a model split over ranks with the reduction and the replication of the
// result fused into the GEMM's epilogue (EPI_TP_RESID), moving over NVLink
// into the peer memory of ctx->pm (x is its residual).  Collective: every
// rank enqueues the same sequence of these calls with the same shapes.
int gemm_tp_resid(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const void *W, int64_t ldw, int M, int N,
                  int K, const float *bias, const float *gate, const int *gate_idx, int64_t ld_gate, bool bcast) {
    TpPeerMem &pm = ctx->pm;
    const int n = ctx->tp_size;
    constexpr int BN = 256;
    if (pm.state != 1 || n < 2 || n > kMaxTpPeers)
        return fail(ctx, LTX_ERR_INVALID_ARG, "gemm_tp_resid: no peer memory");
    if (!A || !W || M <= 0 || K <= 0 || N != pm.D || N % BN || M > pm.rows_cap)
        return fail(ctx, LTX_ERR_SHAPE, "gemm_tp_resid: %d x %d x %d does not fit the peer memory (%lld x %lld)", M, N,
                    K, (long long)pm.rows_cap, (long long)pm.D);
    if (lda % 8 || ldw % 8 || lda < K || ldw < K || ((uintptr_t)A & 15) || ((uintptr_t)W & 15) ||
        ((uintptr_t)bias & 15) || ((uintptr_t)gate & 15) || (gate && ld_gate % 4))
        return fail(ctx, LTX_ERR_SHAPE, "gemm_tp_resid: operands need 16-byte aligned rows");
    const int m_blocks = (M + BM - 1) / BM, n_blocks = N / BN;
    if ((int64_t)m_blocks * n_blocks > pm.tiles_cap) return fail(ctx, LTX_ERR_SHAPE, "gemm_tp_resid: too many tiles");
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, M, K, lda, BM, 2) || !make_tmap_2d(&tb, W, N, K, ldw, BN, 2))
        return fail(ctx, LTX_ERR_CUDA, "gemm_tp_resid: cuTensorMapEncodeTiled failed");
    const size_t panel = (size_t)BM * K * 2, w_bytes = (size_t)N * K * 2;
    const int group_m = w_bytes <= kGroupPanelBytes
                            ? 1
                            : (int)std::max<size_t>(1, std::min<size_t>((size_t)m_blocks, kGroupPanelBytes / panel));
    GemmParams p{M, N, K, nullptr, 1.0f, bias, pm.base, pm.D, gate, gate_idx, ld_gate, ctx->timeout_flag, N, group_m};
    p.m_rot = tp_lo(ctx->tp_rank + 1, m_blocks, n) % m_blocks;   // the other ranks' rows first, this rank's last
    p.tp_rank = ctx->tp_rank;
    p.tp_size = n;
    p.tp_bcast = bcast ? 1 : 0;
    p.epoch = ++pm.epoch;
    p.rows_cap = pm.rows_cap;
    p.tiles_cap = pm.tiles_cap;
    p.recv_off = pm.recv_off;
    p.tstamp_off = pm.tstamp_off;
    p.dstamp_off = pm.dstamp_off;
    p.count_off = pm.count_off;
    for (int r = 0; r < n; ++r) p.peer[r] = pm.peer[r];
    cudaError_t e = launch_gemm<BN, EPI_TP_RESID, false>(ta, tb, ta, tb, ta, p, ctx->sm_count, st);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "gemm_tp_resid launch");
    tp_wait_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const uint32_t *>(pm.base + pm.dstamp_off), n - 1, p.epoch,
                                     ctx->timeout_flag);
    e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : cuda_fail(ctx, e, "tp wait launch");
}

// Every rank of the communicator reaches this point of its stream before any
// goes on (so the ranks' peer memory may be rewritten after it).  Collective.
int tp_peer_barrier(ltx_ctx *ctx, cudaStream_t st) {
    TpPeerMem &pm = ctx->pm;
    const int n = ctx->tp_size;
    if (pm.state != 1 || n < 2) return LTX_OK;
    TpBarrierArgs a{};
    for (int q = 0; q < n; ++q) a.peer_bstamp[q] = reinterpret_cast<uint32_t *>(pm.peer[q] + pm.dstamp_off + 128);
    a.n = n;
    a.me = ctx->tp_rank;
    a.epoch = ++pm.bepoch;
    a.timeout_flag = ctx->timeout_flag;
    tp_barrier_kernel<<<1, 32, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : cuda_fail(ctx, e, "tp barrier launch");
}

// Enqueues out = epilogue(A[M,K] . W[N,K]^T).  A and W are bf16 row-major
// with leading dimensions lda/ldw (elements, multiples of 8, 16-byte aligned bases).
int gemm_bf16(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const void *W, int64_t ldw, int M, int N,
              int K, int epi, const float *bias, void *out, int64_t ldo, const float *gate, const int *gate_idx,
              int64_t ld_gate, int f16_from_col, const TpGather *ag) {
    return gemm_any(ctx, st, 2, A, lda, nullptr, W, ldw, 1.0f, M, N, K, epi, bias, out, ldo, gate, gate_idx, ld_gate,
                    f16_from_col, nullptr, nullptr, ag);
}

// The same with e4m3 A and W (leading dimensions multiples of 16): the
// accumulator is multiplied by a_scale[row] * w_scale before the epilogue.
int gemm_e4m3(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const float *a_scale, const void *W,
              int64_t ldw, float w_scale, int M, int N, int K, int epi, const float *bias, void *out, int64_t ldo,
              const float *gate, const int *gate_idx, int64_t ld_gate, int f16_from_col, const GemmLowRank *lr,
              const float *w_col_scale) {
    return gemm_any(ctx, st, 1, A, lda, a_scale, W, ldw, w_scale, M, N, K, epi, bias, out, ldo, gate, gate_idx, ld_gate,
                    f16_from_col, lr, w_col_scale);
}

}  // namespace ltx

extern "C" int ltx_gemm_bf16(ltx_ctx *ctx, const void *a_dev, int64_t lda, const void *w_dev, int64_t ldw, int32_t m,
                             int32_t n, int32_t k, int32_t epilogue, const float *bias_dev, void *out_dev, int64_t ldo,
                             const float *gate_dev, const int32_t *gate_idx_dev, int64_t ld_gate) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    return ltx::gemm_bf16(ctx, ctx->stream, a_dev, lda, w_dev, ldw, m, n, k, epilogue, bias_dev, out_dev, ldo, gate_dev,
                          gate_idx_dev, ld_gate, n);
}

extern "C" int ltx_gemm_e4m3(ltx_ctx *ctx, const void *a_dev, int64_t lda, const float *a_scale_dev, const void *w_dev,
                             int64_t ldw, float w_scale, const float *w_col_scale_dev, int32_t m, int32_t n, int32_t k,
                             int32_t epilogue, const float *bias_dev, void *out_dev, int64_t ldo, const float *gate_dev,
                             const int32_t *gate_idx_dev, int64_t ld_gate, const void *a2_dev, int64_t lda2,
                             const void *b2_dev, int64_t ldb2, int32_t k2) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    const ltx::GemmLowRank lr{a2_dev, lda2, b2_dev, ldb2, k2};
    return ltx::gemm_e4m3(ctx, ctx->stream, a_dev, lda, a_scale_dev, w_dev, ldw, w_scale, m, n, k, epilogue, bias_dev,
                          out_dev, ldo, gate_dev, gate_idx_dev, ld_gate, n, k2 > 0 ? &lr : nullptr, w_col_scale_dev);
}
