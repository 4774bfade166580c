// ltx_model_*: the ltx-dit VideoTransformer seam (crates/ltx-dit/src/model.rs:57-255,
// load.rs:47-396, block.rs:118-236, config.rs:56-231) and the ltx-sampler step
// (guidance.rs:102-166, loop_.rs:37-65) on the B200 kernels.
//
// Layout in HBM (D = inner dim, rows = batch * tokens):
//   weights   bf16 [out, in] (PyTorch layout, the GEMM's W[N,K]); Q|K|V of the
//             self-attention fused into one [3D, D] matrix, K|V of the
//             cross-attention into [2D, Dc]; biases, norms, tables f32.
//   residual  x f32 [rows, D]; GEMM inputs bf16; attention reads q/k/v as
//             column slices of the fused projection output (no copies).
//   modulation tables  [L][U][coeff][D] f32 for the U distinct timesteps.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <set>
#include <new>
#include <string>
#include <vector>

#include "kernels.hpp"
#include "store.hpp"

namespace ltx {

cudaError_t synth_normal_f32(cudaStream_t st, int sms, float *out, int64_t n, uint64_t seed, uint64_t sid, float mean,
                             float std);
cudaError_t synth_normal_bf16(cudaStream_t st, int sms, __nv_bfloat16 *out, int64_t n, uint64_t seed, uint64_t sid,
                              float std);
cudaError_t synth_quantize_fp8(cudaStream_t st, int sms, const float *x, int64_t n, uint8_t *q, float *scale_dev,
                               unsigned int *work);

struct DitConfig {
    int heads = 32, head_dim = 128, in_ch = 128, out_ch = 128, layers = 28, cross_dim = 4096;
    float eps = 1e-6f;
    double theta = 10000.0;
    int max_pos[3] = {20, 2048, 2048};
    int ts_mult = 1000;
    bool use_mid = true, interleaved = false;
    bool gated = false, cross_adaln = false, prompt_adaln = true, ff_bias = false, kf_abs_pos = false;
    // "gemm_precision": "e4m3" runs all block projections as native FP8 GEMMs
    // (exact FP8 base weights + unmerged LoRA), "e4m3_ffn" only the two FFN
    // projections; default "bf16" (merged weights).  fp8 = any of them.
    bool fp8 = false, fp8_attn = false, fp8_ffn = false;
    // "offload_blocks": n > 0 keeps the blocks in host memory with n on the
    // device at a time (OffloadMode::Stream { n_blocks: n }); 0 = Resident
    int offload_blocks = 0;
    int inner() const { return heads * head_dim; }
    int coeff() const { return cross_adaln ? 9 : 6; }
};

// DiTConfig::from_json + validate (config.rs:56-231).  Accepts the bare
// transformer object or {"transformer": {...}}.
static int parse_config(ltx_ctx *ctx, const std::string &text, DitConfig &c) {
    Json root;
    if (!parse_json(text, root) || root.kind != Json::Obj) return fail(ctx, LTX_ERR_FORMAT, "config JSON parse error");
    const Json *j = root.get("transformer");
    if (!j || j->kind != Json::Obj) j = &root;
    auto num = [&](const char *k, auto &dst) {
        const Json *v = j->get(k);
        if (v && v->kind == Json::Num) dst = static_cast<std::remove_reference_t<decltype(dst)>>(v->num);
    };
    auto flag = [&](const char *k, bool &dst) {
        const Json *v = j->get(k);
        if (v && v->kind == Json::Bool) dst = v->b;
    };
    num("num_attention_heads", c.heads);
    num("attention_head_dim", c.head_dim);
    num("in_channels", c.in_ch);
    num("out_channels", c.out_ch);
    num("num_layers", c.layers);
    num("cross_attention_dim", c.cross_dim);
    num("norm_eps", c.eps);
    num("positional_embedding_theta", c.theta);
    num("timestep_scale_multiplier", c.ts_mult);
    if (const Json *mp = j->get("positional_embedding_max_pos"); mp && mp->kind == Json::Arr && mp->arr.size() == 3)
        for (int i = 0; i < 3; ++i) c.max_pos[i] = (int)mp->arr[i].num;
    flag("use_middle_indices_grid", c.use_mid);
    if (const Json *rt = j->get("rope_type"); rt && rt->kind == Json::Str) c.interleaved = rt->str == "interleaved";
    flag("apply_gated_attention", c.gated);
    flag("cross_attention_adaln", c.cross_adaln);
    flag("use_prompt_adaln_single", c.prompt_adaln);
    flag("ff_bias", c.ff_bias);
    flag("use_keyframes_abs_pos_embedding", c.kf_abs_pos);
    for (const Json *o : {static_cast<const Json *>(&root), j}) {   // this build's own key: top level or beside the transformer's
        const Json *gp = o->get("gemm_precision");
        if (gp && gp->kind == Json::Str) {
            if (gp->str == "e4m3")
                c.fp8 = c.fp8_attn = c.fp8_ffn = true;
            else if (gp->str == "e4m3_ffn")
                c.fp8 = c.fp8_ffn = true;
            else if (gp->str != "bf16")
                return fail(ctx, LTX_ERR_CONFIG, "gemm_precision must be \"bf16\", \"e4m3\" or \"e4m3_ffn\"");
        }
    }
    for (const Json *o : {static_cast<const Json *>(&root), j}) {
        const Json *ob = o->get("offload_blocks");
        if (ob && ob->kind == Json::Num) c.offload_blocks = (int)ob->num;
    }
    if (c.offload_blocks < 0) return fail(ctx, LTX_ERR_CONFIG, "offload_blocks must be >= 0");
    // validate (config.rs:188-231)
    if (c.heads <= 0) return fail(ctx, LTX_ERR_CONFIG, "num_attention_heads must be > 0");
    if (c.head_dim % 2) return fail(ctx, LTX_ERR_CONFIG, "attention_head_dim must be even for RoPE");
    if (c.inner() < 6) return fail(ctx, LTX_ERR_CONFIG, "inner_dim %d must be at least 6", c.inner());
    if ((c.inner() / 2) % c.heads) return fail(ctx, LTX_ERR_CONFIG, "inner_dim / 2 must be divisible by num_attention_heads");
    if (c.cross_adaln && c.prompt_adaln)
        return fail(ctx, LTX_ERR_CONFIG, "use_prompt_adaln_single with cross_attention_adaln is not wired in this core");
    if (c.kf_abs_pos) return fail(ctx, LTX_ERR_CONFIG, "use_keyframes_abs_pos_embedding is not wired in this core");
    if (c.layers < 0 || c.in_ch <= 0 || c.out_ch <= 0 || c.cross_dim <= 0)
        return fail(ctx, LTX_ERR_CONFIG, "bad dimensions in config");
    if (c.inner() % 8 || c.in_ch % 8 || c.cross_dim % 8)
        return fail(ctx, LTX_ERR_UNSUPPORTED, "inner_dim, in_channels and cross_attention_dim must be multiples of 8");
    if (c.fp8 && (c.inner() != 4096 || c.head_dim != 128 || c.gated || c.cross_adaln || c.cross_dim % 16 ||
                  c.interleaved))
        return fail(ctx, LTX_ERR_UNSUPPORTED,
                    "gemm_precision e4m3 needs the 22B block layout: inner dim 4096 (32 x 128 heads), split RoPE, no "
                    "gated attention or cross-attention adaLN, cross dim %% 16 == 0");
    return LTX_OK;
}

// One projection of the FP8 path: the exact e4m3 base weight with its
// per-tensor scale, and the LoRA kept factored: A quantised per tensor
// (rank padded to 64 with zero rows) and B2 = coeff * B / sw in bf16, which
// the GEMM adds in the same accumulator (x.A^T / sx) . B2^T.
struct LinF8 {
    uint8_t *w = nullptr;   // [out, in]
    float sw = 1.f;
    uint8_t *a = nullptr;   // [r64, in]
    float sa = 1.f;
    __nv_bfloat16 *b2 = nullptr;   // [out, r64]
    int r64 = 0;            // 0 = no LoRA
};

struct BlockW {
    LinF8 fqkv, fo, fq2, fkv2, fo2, fff1, fff2;   // FP8 path (gemm_precision e4m3)
    __nv_bfloat16 *qkv, *o, *q2, *kv2, *o2, *ff1, *ff2, *g1, *g2;
    float *qkv_b, *o_b, *q2_b, *kv2_b, *o2_b, *ff1_b, *ff2_b, *g1_b, *g2_b;
    float *qn, *kn, *qn2, *kn2, *sst, *pst;
};

}  // namespace ltx

struct ltx_model {
    int device = 0;
    ltx::DitConfig cfg;
    // tensor-parallel shard: this model holds rank tr of tp (heads and FFN
    // hidden units split; everything else replicated)
    int tp = 1, tr = 0;
    int lora_r64 = 0;   // FP8 path: LoRA rank padded to 64 (the factored term's K)
    // OffloadMode::Stream (crates/ltx-dit/src/offload.rs:43-56): the blocks'
    // weights live in pinned host memory (blocks[l] views into it) and at most
    // offload_n of them are on the device, in slots[], uploaded on copy_stream
    // just before use.  offload_n = 0: every block resident in the arena.
    int offload_n = 0;
    size_t block_bytes = 0;
    void *host_blocks = nullptr;
    std::vector<ltx::BlockW> slots;
    std::vector<char *> slot_base;
    cudaStream_t copy_stream = nullptr;
    std::vector<cudaEvent_t> copied, freed;   // per slot: upload done / block computed
    void *arena = nullptr;
    size_t arena_bytes = 0;
    __nv_bfloat16 *patch_w = nullptr, *out_w = nullptr;
    float *patch_b = nullptr, *out_b = nullptr, *sst_out = nullptr;
    float *t1_w = nullptr, *t1_b = nullptr, *t2_w = nullptr, *t2_b = nullptr, *lin_w = nullptr, *lin_b = nullptr;
    float *rope_freq = nullptr;   // [grid]
    float *sin_freq = nullptr;    // [128]
    float **sst_list = nullptr;   // device array of L pointers
    int rope_grid = 0;
    std::vector<ltx::BlockW> blocks;
};

namespace ltx {

// ── arena layout ─────────────────────────────────────────────────────────────

struct Arena {
    size_t off = 0;
    char *base = nullptr;
    template <class T>
    T *take(int64_t n) {
        off = (off + 255) & ~size_t(255);
        T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
        off += (size_t)std::max<int64_t>(n, 1) * sizeof(T);
        return p;
    }
};

// Assigns every weight a slice of one allocation (sizing pass when a.base == null).
// One block's projection weights, biases and norms (everything of a block
// except its modulation tables), laid out from the arena's current offset.
// With offload the same layout is used for the host image of every block and
// for each device slot.
static void layout_block(const ltx_model *m, BlockW &b, Arena &a) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim;
    // this rank's share of the split dimensions
    const int64_t Dl = D / m->tp, Fl = 4 * D / m->tp, Hl = c.heads / m->tp;
    const int r64 = m->lora_r64;
    auto f8 = [&](LinF8 &L, int64_t out, int64_t in) {
        L.w = a.take<uint8_t>(out * in);
        L.r64 = r64;
        if (r64) {
            L.a = a.take<uint8_t>((int64_t)r64 * in);
            L.b2 = a.take<__nv_bfloat16>(out * r64);
        }
    };
    // FP8 path: e4m3 weights + factored LoRA instead of merged bf16 (tp = 1)
    if (c.fp8_attn) {
        f8(b.fqkv, 3 * D, D);
        f8(b.fo, D, D);
        f8(b.fq2, D, D);
        f8(b.fkv2, 2 * D, Dc);
        f8(b.fo2, D, D);
    }
    if (c.fp8_ffn) {
        f8(b.fff1, 4 * D, D);
        f8(b.fff2, D, 4 * D);
    }
    b.qkv = c.fp8_attn ? nullptr : a.take<__nv_bfloat16>(3 * Dl * D);
    b.qkv_b = a.take<float>(3 * Dl);
    b.qn = a.take<float>(Dl);
    b.kn = a.take<float>(Dl);
    b.o = c.fp8_attn ? nullptr : a.take<__nv_bfloat16>(D * Dl);
    b.o_b = a.take<float>(D);
    b.q2 = c.fp8_attn ? nullptr : a.take<__nv_bfloat16>(Dl * D);
    b.q2_b = a.take<float>(Dl);
    b.kv2 = c.fp8_attn ? nullptr : a.take<__nv_bfloat16>(2 * Dl * Dc);
    b.kv2_b = a.take<float>(2 * Dl);
    b.qn2 = a.take<float>(Dl);
    b.kn2 = a.take<float>(Dl);
    b.o2 = c.fp8_attn ? nullptr : a.take<__nv_bfloat16>(D * Dl);
    b.o2_b = a.take<float>(D);
    b.ff1 = c.fp8_ffn ? nullptr : a.take<__nv_bfloat16>(Fl * D);
    b.ff1_b = c.ff_bias ? a.take<float>(Fl) : nullptr;
    b.ff2 = c.fp8_ffn ? nullptr : a.take<__nv_bfloat16>(D * Fl);
    b.ff2_b = c.ff_bias ? a.take<float>(D) : nullptr;
    b.g1 = c.gated ? a.take<__nv_bfloat16>(Hl * D) : nullptr;
    b.g1_b = c.gated ? a.take<float>(Hl) : nullptr;
    b.g2 = c.gated ? a.take<__nv_bfloat16>(Hl * D) : nullptr;
    b.g2_b = c.gated ? a.take<float>(Hl) : nullptr;
}

// Bytes of one block's image (layout_block from offset 0, 256-aligned).
static size_t block_bytes(const ltx_model *m) {
    Arena a;
    BlockW b{};
    layout_block(m, b, a);
    return (a.off + 255) & ~size_t(255);
}

// Assigns every resident weight a slice of the device arena (sizing pass when
// a.base == null): the head, the adaLN tables, every block's modulation
// tables, and either all blocks (resident) or the offload slots.
static void layout(ltx_model *m, Arena &a) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), K = c.coeff();
    m->patch_w = a.take<__nv_bfloat16>(D * c.in_ch);
    m->patch_b = a.take<float>(D);
    m->t1_w = a.take<float>(D * 256);
    m->t1_b = a.take<float>(D);
    m->t2_w = a.take<float>(D * D);
    m->t2_b = a.take<float>(D);
    m->lin_w = a.take<float>(K * D * D);
    m->lin_b = a.take<float>(K * D);
    m->sst_out = a.take<float>(2 * D);
    m->out_w = a.take<__nv_bfloat16>(c.out_ch * D);
    m->out_b = a.take<float>(c.out_ch);
    m->rope_grid = (int)(D / 6);
    m->rope_freq = a.take<float>(m->rope_grid);
    m->sin_freq = a.take<float>(128);
    m->sst_list = a.take<float *>(c.layers);
    m->blocks.resize(c.layers);
    for (auto &b : m->blocks) {   // modulation tables stay resident (adaLN reads all layers at once)
        b.sst = a.take<float>(K * D);
        b.pst = c.cross_adaln ? a.take<float>(2 * D) : nullptr;
    }
    if (m->offload_n > 0) {
        m->slots.resize(m->offload_n);
        m->slot_base.clear();
        for (auto &sv : m->slots) {
            const size_t start = (a.off + 255) & ~size_t(255);
            Arena one;
            one.base = a.base ? a.base + start : nullptr;
            layout_block(m, sv, one);
            if (a.base) m->slot_base.push_back(a.base + start);
            a.off = start + m->block_bytes;
        }
    } else {
        for (auto &b : m->blocks) layout_block(m, b, a);
    }
}

// Frees everything a model owns (device arena, offload image, stream, events).
static void free_model(ltx_model *m) {
    if (!m) return;
    if (m->arena) cudaFree(m->arena);
    if (m->host_blocks) cudaFreeHost(m->host_blocks);
    for (auto ev : m->copied)
        if (ev) cudaEventDestroy(ev);
    for (auto ev : m->freed)
        if (ev) cudaEventDestroy(ev);
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    delete m;
}

static int alloc_model(ltx_ctx *ctx, const DitConfig &cfg, ltx_model *&m, int lora_rank = 0) {
    if (cfg.fp8 && ctx->tp_size > 1)
        return fail(ctx, LTX_ERR_UNSUPPORTED, "gemm_precision e4m3 runs on one GPU (no tensor-parallel split)");
    m = new (std::nothrow) ltx_model();
    if (!m) return LTX_ERR_OOM;
    m->device = ctx->device;
    m->cfg = cfg;
    m->tp = ctx->tp_size;
    m->tr = ctx->tp_rank;
    m->lora_r64 = cfg.fp8 && lora_rank > 0 ? (lora_rank + 63) / 64 * 64 : 0;
    m->offload_n = cfg.offload_blocks > 0 && cfg.offload_blocks < cfg.layers ? cfg.offload_blocks : 0;
    if (m->offload_n) m->block_bytes = block_bytes(m);
    if (m->tp > 1 && (cfg.heads % m->tp || (cfg.inner() / m->tp) % 8)) {
        const int tp = m->tp;
        delete m;
        m = nullptr;
        return fail(ctx, LTX_ERR_UNSUPPORTED, "%d heads of width %d do not split over %d ranks", cfg.heads,
                    cfg.head_dim, tp);
    }
    Arena sizing;
    layout(m, sizing);
    m->arena_bytes = sizing.off + 256;
    cudaError_t e = cudaMalloc(&m->arena, m->arena_bytes);
    if (e != cudaSuccess) {
        delete m;
        m = nullptr;
        return fail(ctx, LTX_ERR_OOM, "model weights: %zu bytes: %s", sizing.off, cudaGetErrorString(e));
    }
    cudaMemsetAsync(m->arena, 0, m->arena_bytes, ctx->stream);
    Arena real;
    real.base = static_cast<char *>(m->arena);
    layout(m, real);
    if (m->offload_n) {
        // pinned host image of every block (zeroed: absent biases stay 0), slots, copy stream, events
        const size_t host_bytes = m->block_bytes * (size_t)cfg.layers;
        e = cudaHostAlloc(&m->host_blocks, host_bytes, cudaHostAllocDefault);
        if (e != cudaSuccess) {
            m->host_blocks = nullptr;
            const int rc = fail(ctx, LTX_ERR_OOM, "offloaded blocks: %zu bytes of pinned host memory: %s", host_bytes,
                                cudaGetErrorString(e));
            free_model(m);
            m = nullptr;
            return rc;
        }
        memset(m->host_blocks, 0, host_bytes);
        for (int l = 0; l < cfg.layers; ++l) {
            Arena one;
            one.base = static_cast<char *>(m->host_blocks) + (size_t)l * m->block_bytes;
            layout_block(m, m->blocks[l], one);
        }
        m->copied.resize(m->offload_n);
        m->freed.resize(m->offload_n);
        bool ok = cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking) == cudaSuccess;
        for (int i = 0; ok && i < m->offload_n; ++i)
            ok = cudaEventCreateWithFlags(&m->copied[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&m->freed[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            free_model(m);
            m = nullptr;
            return fail(ctx, LTX_ERR_CUDA, "offload stream/events");
        }
    }
    // host-computed tables: RoPE frequency grid (rope.rs:311-322, f64 -> f32) and
    // the sinusoid frequencies exp(-ln(1e4) * i / 128) in f32 (adaln.rs:43-59).
    std::vector<float> grid(m->rope_grid), sf(128);
    for (int i = 0; i < m->rope_grid; ++i) {
        double v = m->rope_grid == 1 ? cfg.theta * M_PI / 2.0
                                     : std::pow(cfg.theta, (double)i / (double)(m->rope_grid - 1)) * M_PI / 2.0;
        grid[i] = (float)v;
    }
    const float log10k = std::log(10000.0f);
    for (int i = 0; i < 128; ++i) sf[i] = std::exp(-log10k * (float)i / 128.0f);
    std::vector<float *> ssts;
    for (auto &b : m->blocks) ssts.push_back(b.sst);
    if (m->rope_grid) cudaMemcpyAsync(m->rope_freq, grid.data(), grid.size() * 4, cudaMemcpyHostToDevice, ctx->stream);
    cudaMemcpyAsync(m->sin_freq, sf.data(), 128 * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (!ssts.empty())
        cudaMemcpyAsync(m->sst_list, ssts.data(), ssts.size() * sizeof(float *), cudaMemcpyHostToDevice, ctx->stream);
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "model table upload");
    return LTX_OK;
}

// ── tensor-parallel slices ───────────────────────────────────────────────────

// Which part of a full row-major [R, C] tensor a rank keeps.  ROWS: the rows
// form `nseg` equal blocks (the fused Q|K|V or K|V projections) and the rank
// keeps its 1/n of every block; COLS: it keeps its 1/n of the columns.
struct Split {
    enum Kind { ALL, ROWS, COLS } kind = ALL;
    int nseg = 1;
};
static const Split kAll{Split::ALL, 1}, kRows{Split::ROWS, 1}, kCols{Split::COLS, 1};

static cudaError_t slice_to(cudaStream_t st, void *dst, const void *full, int64_t R, int64_t C, size_t es, Split sp,
                            int n, int r) {
    const char *src = static_cast<const char *>(full);
    char *d = static_cast<char *>(dst);
    if (sp.kind == Split::ALL || n == 1)
        return cudaMemcpyAsync(dst, full, (size_t)(R * C) * es, cudaMemcpyDeviceToDevice, st);
    if (sp.kind == Split::ROWS) {
        const int64_t blk = R / sp.nseg, part = blk / n;
        for (int s = 0; s < sp.nseg; ++s) {
            cudaError_t e = cudaMemcpyAsync(d + (size_t)(s * part * C) * es, src + (size_t)((s * blk + r * part) * C) * es,
                                            (size_t)(part * C) * es, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    const int64_t part = C / n;
    return cudaMemcpy2DAsync(d, (size_t)part * es, src + (size_t)(r * part) * es, (size_t)C * es, (size_t)part * es,
                             (size_t)R, cudaMemcpyDeviceToDevice, st);
}

// ── loading from a weight store (load.rs:47-396) ─────────────────────────────

struct Loader {
    ltx_store *st;
    ltx_ctx *ctx;
    int n = 1, r = 0;
    void *tmp = nullptr;      // full-tensor staging for sharded reads (n > 1)
    int shape_check(const std::string &key, std::vector<int64_t> want) {
        auto it = st->entries.find(key);
        if (it == st->entries.end()) return fail(ctx, LTX_ERR_MISSING_KEY, "missing key: \"%s\"", key.c_str());
        if (it->second.shape != want) {
            std::string got, exp;
            for (auto d : it->second.shape) got += std::to_string(d) + ",";
            for (auto d : want) exp += std::to_string(d) + ",";
            return fail(ctx, LTX_ERR_SHAPE, "invalid tensor data for key \"%s\": shape mismatch: expected [%s] got [%s]",
                        key.c_str(), exp.c_str(), got.c_str());
        }
        return LTX_OK;
    }
    // reads the full tensor `key` (checked against `shape`) and keeps this
    // rank's `sp` part of it in dst
    int req(const std::string &key, std::vector<int64_t> shape, void *dst, int dt, Split sp = kAll) {
        int rc = shape_check(key, shape);
        if (rc) return rc;
        if (n == 1 || sp.kind == Split::ALL) return store_read_device(st, key, dt, dst, numel(shape));
        rc = store_read_device(st, key, dt, tmp, numel(shape));
        if (rc) return rc;
        const int64_t R = shape[0];
        int64_t C = 1;
        for (size_t i = 1; i < shape.size(); ++i) C *= shape[i];
        LTX_CUDA_TRY(ctx, slice_to(ctx->stream, dst, tmp, R, C, dtype_size(dt), sp, n, r));
        return LTX_OK;
    }
    // optional tensor (bias): absent -> left zero, returns whether present
    int opt(const std::string &key, std::vector<int64_t> shape, void *dst, int dt, Split sp = kAll,
            bool *present = nullptr) {
        if (!st->entries.count(key)) {
            if (present) *present = false;
            return LTX_OK;
        }
        if (present) *present = true;
        return req(key, shape, dst, dt, sp);
    }
};

#define TRY(x)                   \
    do {                         \
        int _rc = (x);           \
        if (_rc) return _rc;     \
    } while (0)

// With offload, a block is written into device slot 0 (plus its resident
// modulation tables) and then copied to its host image.  The slot is zeroed
// first, so a weight the store lacks (an optional bias) reads 0 as it does in
// the zeroed resident arena, not the previous block's value.
static BlockW staging_view(ltx_model *m, ltx_ctx *ctx, int l) {
    cudaMemsetAsync(m->slot_base[0], 0, m->block_bytes, ctx->stream);
    BlockW b = m->slots[0];
    b.sst = m->blocks[l].sst;
    b.pst = m->blocks[l].pst;
    return b;
}

// The per-tensor FP8 scales are host values of the block's LinF8 records,
// not part of its device image: copied from the staging view to block l's
// record at load, and from there into the slot's view at each use.
static void copy_scales(BlockW &dst, const BlockW &src) {
    LinF8 BlockW::*const f8[] = {&BlockW::fqkv, &BlockW::fo, &BlockW::fq2, &BlockW::fkv2,
                                 &BlockW::fo2,  &BlockW::fff1, &BlockW::fff2};
    for (auto f : f8) {
        (dst.*f).sw = (src.*f).sw;
        (dst.*f).sa = (src.*f).sa;
    }
}

// Copies staged block l (slot 0) to its host image and keeps its FP8 scales.
static int stash_block(ltx_model *m, ltx_ctx *ctx, int l, const BlockW &stage) {
    LTX_CUDA_TRY(ctx, cudaMemcpyAsync(static_cast<char *>(m->host_blocks) + (size_t)l * m->block_bytes,
                                      m->slot_base[0], m->block_bytes, cudaMemcpyDeviceToHost, ctx->stream));
    LTX_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));   // slot 0 is reused by the next block
    copy_scales(m->blocks[l], stage);
    return LTX_OK;
}

static int load_weights_into(ltx_model *m, Loader &L) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, F = 4 * D, H = c.heads, K = c.coeff();
    const int64_t Dl = D / m->tp;
    TRY(L.req("patchify_proj.weight", {D, c.in_ch}, m->patch_w, LTX_BF16));
    TRY(L.opt("patchify_proj.bias", {D}, m->patch_b, LTX_F32));
    TRY(L.req("adaln_single.emb.timestep_embedder.linear_1.weight", {D, 256}, m->t1_w, LTX_F32));
    TRY(L.opt("adaln_single.emb.timestep_embedder.linear_1.bias", {D}, m->t1_b, LTX_F32));
    TRY(L.req("adaln_single.emb.timestep_embedder.linear_2.weight", {D, D}, m->t2_w, LTX_F32));
    TRY(L.opt("adaln_single.emb.timestep_embedder.linear_2.bias", {D}, m->t2_b, LTX_F32));
    TRY(L.req("adaln_single.linear.weight", {K * D, D}, m->lin_w, LTX_F32));
    TRY(L.opt("adaln_single.linear.bias", {K * D}, m->lin_b, LTX_F32));
    TRY(L.req("scale_shift_table", {2, D}, m->sst_out, LTX_F32));
    TRY(L.req("proj_out.weight", {c.out_ch, D}, m->out_w, LTX_BF16));
    TRY(L.opt("proj_out.bias", {c.out_ch}, m->out_b, LTX_F32));
    for (int i = 0; i < c.layers; ++i) {
        BlockW stage = m->offload_n ? staging_view(m, L.ctx, i) : BlockW{};
        BlockW &b = m->offload_n ? stage : m->blocks[i];
        const std::string p = "transformer_blocks." + std::to_string(i) + ".";
        const std::string a1 = p + "attn1.", a2 = p + "attn2.";
        TRY(L.req(a1 + "to_q.weight", {D, D}, b.qkv, LTX_BF16, kRows));
        TRY(L.req(a1 + "to_k.weight", {D, D}, b.qkv + Dl * D, LTX_BF16, kRows));
        TRY(L.req(a1 + "to_v.weight", {D, D}, b.qkv + 2 * Dl * D, LTX_BF16, kRows));
        TRY(L.opt(a1 + "to_q.bias", {D}, b.qkv_b, LTX_F32, kRows));
        TRY(L.opt(a1 + "to_k.bias", {D}, b.qkv_b + Dl, LTX_F32, kRows));
        TRY(L.opt(a1 + "to_v.bias", {D}, b.qkv_b + 2 * Dl, LTX_F32, kRows));
        TRY(L.req(a1 + "q_norm.weight", {D}, b.qn, LTX_F32, kRows));
        TRY(L.req(a1 + "k_norm.weight", {D}, b.kn, LTX_F32, kRows));
        TRY(L.req(a1 + "to_out.0.weight", {D, D}, b.o, LTX_BF16, kCols));
        TRY(L.opt(a1 + "to_out.0.bias", {D}, b.o_b, LTX_F32));
        TRY(L.req(a2 + "to_q.weight", {D, D}, b.q2, LTX_BF16, kRows));
        TRY(L.opt(a2 + "to_q.bias", {D}, b.q2_b, LTX_F32, kRows));
        TRY(L.req(a2 + "to_k.weight", {D, Dc}, b.kv2, LTX_BF16, kRows));
        TRY(L.req(a2 + "to_v.weight", {D, Dc}, b.kv2 + Dl * Dc, LTX_BF16, kRows));
        TRY(L.opt(a2 + "to_k.bias", {D}, b.kv2_b, LTX_F32, kRows));
        TRY(L.opt(a2 + "to_v.bias", {D}, b.kv2_b + Dl, LTX_F32, kRows));
        TRY(L.req(a2 + "q_norm.weight", {D}, b.qn2, LTX_F32, kRows));
        TRY(L.req(a2 + "k_norm.weight", {D}, b.kn2, LTX_F32, kRows));
        TRY(L.req(a2 + "to_out.0.weight", {D, D}, b.o2, LTX_BF16, kCols));
        TRY(L.opt(a2 + "to_out.0.bias", {D}, b.o2_b, LTX_F32));
        if (c.gated) {
            TRY(L.req(a1 + "to_gate_logits.weight", {H, D}, b.g1, LTX_BF16, kRows));
            TRY(L.opt(a1 + "to_gate_logits.bias", {H}, b.g1_b, LTX_F32, kRows));
            TRY(L.req(a2 + "to_gate_logits.weight", {H, D}, b.g2, LTX_BF16, kRows));
            TRY(L.opt(a2 + "to_gate_logits.bias", {H}, b.g2_b, LTX_F32, kRows));
        }
        TRY(L.req(p + "ff.net.0.proj.weight", {F, D}, b.ff1, LTX_BF16, kRows));
        TRY(L.req(p + "ff.net.2.weight", {D, F}, b.ff2, LTX_BF16, kCols));
        if (c.ff_bias) {
            TRY(L.opt(p + "ff.net.0.proj.bias", {F}, b.ff1_b, LTX_F32, kRows));
            TRY(L.opt(p + "ff.net.2.bias", {D}, b.ff2_b, LTX_F32));
        }
        TRY(L.req(p + "scale_shift_table", {K, D}, b.sst, LTX_F32));
        if (c.cross_adaln) TRY(L.req(p + "prompt_scale_shift_table", {2, D}, b.pst, LTX_F32));
        if (m->offload_n) TRY(stash_block(m, L.ctx, i, b));
    }
    return LTX_OK;
}

static int load_weights(ltx_model *m, ltx_store *st, ltx_ctx *ctx) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner();
    Loader L{st, ctx, m->tp, m->tr};
    if (m->tp > 1) {
        // the largest split tensor, as f32: [4D, D] or [D, cross_dim]
        const size_t big = (size_t)std::max<int64_t>(4 * D * D, D * c.cross_dim) * 4;
        cudaError_t e = cudaMalloc(&L.tmp, big);
        if (e != cudaSuccess) return fail(ctx, LTX_ERR_OOM, "shard staging of %zu bytes: %s", big, cudaGetErrorString(e));
    }
    int rc = load_weights_into(m, L);
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (L.tmp) cudaFree(L.tmp);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(ctx, e, "model load");
    return LTX_OK;
}

// ── synthetic FP8 + LoRA checkpoint on the device ────────────────────────────

struct Synth {
    ltx_ctx *ctx;
    uint64_t seed;
    int rank;
    float strength;
    int n = 1, r = 0;            // tensor-parallel shard kept
    uint64_t sid = 1;
    float *f32 = nullptr;        // [max numel]
    uint8_t *q8 = nullptr;       // [max numel]
    __nv_bfloat16 *la = nullptr, *lb = nullptr;
    float *scale_dev = nullptr;
    unsigned int *work = nullptr;
    void *full = nullptr;        // full merged tensor before slicing (n > 1)
    // W ~ N(0, 0.02) -> e4m3 with scale amax/448; LoRA A [r, in], B [out, r]
    // bf16 ~ N(0, 0.01), alpha = rank; merged through ltx_dequant_merge.  The
    // whole tensor is always generated (same random stream and FP8 scale on
    // every shard count), then this rank's part is kept.
    int linear(void *dst, int64_t out, int64_t in, int dst_dt, Split sp = kAll) {
        const int64_t n_el = out * in;
        cudaStream_t st = ctx->stream;
        LTX_CUDA_TRY(ctx, synth_normal_f32(st, ctx->sm_count, f32, n_el, seed, sid++, 0.f, 0.02f));
        LTX_CUDA_TRY(ctx, synth_quantize_fp8(st, ctx->sm_count, f32, n_el, q8, scale_dev, work));
        float scale = 0.f;
        LTX_CUDA_TRY(ctx, cudaMemcpyAsync(&scale, scale_dev, 4, cudaMemcpyDeviceToHost, st));
        LTX_CUDA_TRY(ctx, cudaStreamSynchronize(st));
        ltx_lora_delta d{};
        int nd = 0;
        if (rank > 0) {
            LTX_CUDA_TRY(ctx, synth_normal_bf16(st, ctx->sm_count, la, rank * in, seed, sid++, 0.01f));
            LTX_CUDA_TRY(ctx, synth_normal_bf16(st, ctx->sm_count, lb, out * rank, seed, sid++, 0.01f));
            d = ltx_lora_delta{la, lb, rank, LTX_BF16, LTX_BF16, ltx_lora_coeff(strength, (float)rank, rank)};
            nd = 1;
        }
        const bool sliced = n > 1 && sp.kind != Split::ALL;
        const int rc = dequant_merge(ctx, st, q8, LTX_F8_E4M3, 1, scale, out, in, &d, nd, sliced ? full : dst, dst_dt);
        if (rc || !sliced) return rc;
        LTX_CUDA_TRY(ctx, slice_to(st, dst, full, out, in, dtype_size(dst_dt), sp, n, r));
        return LTX_OK;
    }
    // The FP8 path's copy of `linear`: the same random stream (the same base
    // bytes, scale and LoRA factors), kept unmerged (LinF8).
    int linear_f8(LinF8 &L, int64_t out, int64_t in) {
        const int64_t n_el = out * in;
        cudaStream_t st = ctx->stream;
        LTX_CUDA_TRY(ctx, synth_normal_f32(st, ctx->sm_count, f32, n_el, seed, sid++, 0.f, 0.02f));
        LTX_CUDA_TRY(ctx, synth_quantize_fp8(st, ctx->sm_count, f32, n_el, q8, scale_dev, work));
        float scale = 0.f;
        LTX_CUDA_TRY(ctx, cudaMemcpyAsync(&scale, scale_dev, 4, cudaMemcpyDeviceToHost, st));
        LTX_CUDA_TRY(ctx, cudaStreamSynchronize(st));
        LTX_CUDA_TRY(ctx, cudaMemcpyAsync(L.w, q8, (size_t)n_el, cudaMemcpyDeviceToDevice, st));
        L.sw = scale;
        if (rank > 0) {
            LTX_CUDA_TRY(ctx, synth_normal_bf16(st, ctx->sm_count, la, rank * in, seed, sid++, 0.01f));
            LTX_CUDA_TRY(ctx, synth_normal_bf16(st, ctx->sm_count, lb, out * rank, seed, sid++, 0.01f));
            const float coeff = ltx_lora_coeff(strength, (float)rank, rank);
            // A per tensor to e4m3 (rows rank..r64 stay zero), B2 = coeff * B / sw
            LTX_CUDA_TRY(ctx, bf16_to_f32(st, ctx->sm_count, la, (int64_t)rank * in, f32));
            LTX_CUDA_TRY(ctx, synth_quantize_fp8(st, ctx->sm_count, f32, (int64_t)rank * in, L.a, scale_dev, work));
            float sa = 0.f;
            LTX_CUDA_TRY(ctx, cudaMemcpyAsync(&sa, scale_dev, 4, cudaMemcpyDeviceToHost, st));
            LTX_CUDA_TRY(ctx, cudaStreamSynchronize(st));
            L.sa = sa;
            LTX_CUDA_TRY(ctx, scale_pad_bf16(st, ctx->sm_count, lb, (int)out, rank, L.r64, coeff / scale, L.b2));
        }
        return LTX_OK;
    }
    int vec(float *dst, int64_t n_el, float mean, float std, Split sp = kAll) {
        const bool sliced = n > 1 && sp.kind != Split::ALL;
        LTX_CUDA_TRY(ctx, synth_normal_f32(ctx->stream, ctx->sm_count, sliced ? static_cast<float *>(full) : dst, n_el,
                                           seed, sid++, mean, std));
        if (sliced) LTX_CUDA_TRY(ctx, slice_to(ctx->stream, dst, full, n_el, 1, 4, sp, n, r));
        return LTX_OK;
    }
};

static int init_random(ltx_model *m, ltx_ctx *ctx, uint64_t seed, int rank, float strength) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, F = 4 * D, H = c.heads, K = c.coeff();
    const int64_t maxn = std::max<int64_t>({F * D, K * D * D, 2 * D * Dc, 3 * D * D});
    Synth s{ctx, seed, rank, strength, m->tp, m->tr};
    // scratch: f32 weight [maxn] | fp8 [maxn] | LoRA A [rank*max_in] | LoRA B [max_out*rank] | scale | amax
    //          | full merged tensor [maxn] (sharded models only)
    const int64_t max_in = std::max<int64_t>({F, Dc, D, 256, (int64_t)c.in_ch});
    const int64_t max_out = std::max<int64_t>({K * D, F, 3 * D, 2 * D, (int64_t)c.out_ch});
    Arena sz;
    sz.take<float>(maxn);
    sz.take<uint8_t>(maxn);
    sz.take<__nv_bfloat16>((int64_t)rank * max_in);
    sz.take<__nv_bfloat16>(max_out * rank);
    sz.take<float>(1);
    sz.take<unsigned int>(1);
    if (m->tp > 1) sz.take<float>(maxn);
    void *buf = nullptr;
    if (cudaMalloc(&buf, sz.off + 256) != cudaSuccess) return fail(ctx, LTX_ERR_OOM, "synthetic init scratch");
    Arena ar;
    ar.base = static_cast<char *>(buf);
    s.f32 = ar.take<float>(maxn);
    s.q8 = ar.take<uint8_t>(maxn);
    s.la = ar.take<__nv_bfloat16>((int64_t)rank * max_in);
    s.lb = ar.take<__nv_bfloat16>(max_out * rank);
    s.scale_dev = ar.take<float>(1);
    s.work = ar.take<unsigned int>(1);
    if (m->tp > 1) s.full = ar.take<float>(maxn);
    const Split qkv3{Split::ROWS, 3}, kv2{Split::ROWS, 2};
    int rc = [&]() -> int {
        TRY(s.linear(m->patch_w, D, c.in_ch, LTX_BF16));
        TRY(s.linear(m->t1_w, D, 256, LTX_F32));
        TRY(s.linear(m->t2_w, D, D, LTX_F32));
        TRY(s.linear(m->lin_w, K * D, D, LTX_F32));
        TRY(s.vec(m->sst_out, 2 * D, 0.f, 0.02f));
        TRY(s.linear(m->out_w, c.out_ch, D, LTX_BF16));
        for (int li = 0; li < c.layers; ++li) {
            BlockW stage = m->offload_n ? staging_view(m, ctx, li) : BlockW{};
            BlockW &b = m->offload_n ? stage : m->blocks[li];
            // the same random stream in either precision (same order of draws)
            if (c.fp8_attn) {
                TRY(s.linear_f8(b.fqkv, 3 * D, D));
                TRY(s.linear_f8(b.fo, D, D));
                TRY(s.linear_f8(b.fq2, D, D));
                TRY(s.linear_f8(b.fkv2, 2 * D, Dc));
                TRY(s.linear_f8(b.fo2, D, D));
            } else {
                TRY(s.linear(b.qkv, 3 * D, D, LTX_BF16, qkv3));
                TRY(s.linear(b.o, D, D, LTX_BF16, kCols));
                TRY(s.linear(b.q2, D, D, LTX_BF16, kRows));
                TRY(s.linear(b.kv2, 2 * D, Dc, LTX_BF16, kv2));
                TRY(s.linear(b.o2, D, D, LTX_BF16, kCols));
            }
            if (c.fp8_ffn) {
                TRY(s.linear_f8(b.fff1, F, D));
                TRY(s.linear_f8(b.fff2, D, F));
            } else {
                TRY(s.linear(b.ff1, F, D, LTX_BF16, kRows));
                TRY(s.linear(b.ff2, D, F, LTX_BF16, kCols));
            }
            TRY(s.vec(b.qn, D, 1.f, 0.02f, kRows));
            TRY(s.vec(b.kn, D, 1.f, 0.02f, kRows));
            TRY(s.vec(b.qn2, D, 1.f, 0.02f, kRows));
            TRY(s.vec(b.kn2, D, 1.f, 0.02f, kRows));
            TRY(s.vec(b.sst, K * D, 0.f, 0.02f));
            if (b.pst) TRY(s.vec(b.pst, 2 * D, 0.f, 0.02f));
            if (b.g1) {
                TRY(s.linear(b.g1, H, D, LTX_BF16, kRows));
                TRY(s.linear(b.g2, H, D, LTX_BF16, kRows));
            }
            if (m->offload_n) TRY(stash_block(m, ctx, li, b));
        }
        return LTX_OK;
    }();
    cudaStreamSynchronize(ctx->stream);
    cudaFree(buf);
    return rc;
}

// ── forward (model.rs:169-255, block.rs:118-236) ─────────────────────────────

struct Work {
    float *x, *out32, *tok_t, *mod, *emb, *h1, *sinus, *tab, *otab, *cos, *sin, *glog;
    __nv_bfloat16 *xn, *qkv, *att, *q2, *kv2, *ctxb, *ffh, *latb;
    int *idx;
    float *ts_u;
    double *partial;
    __nv_bfloat16 *part;   // tensor-parallel: summed partial projections (bf16)
    float *ss;             // tensor-parallel: Q/K sums of squares
    // FP8 path: e4m3 projection inputs with per-row scales, the factored-LoRA
    // operand (x.A^T / sx), and the quantised context (once per forward)
    uint8_t *xq, *cq;
    float *sx, *scq;
    __nv_bfloat16 *xa, *xac;
    size_t bytes;
};

// Forward workspace for `rows` latent rows and `crow` context rows on a model
// split over `tp` ranks (tp = 1: whole model).
static Work carve_work(char *base, const DitConfig &c, int64_t rows, int64_t crow, int U, int L, int tp,
                       int r64 = 0) {
    Arena a;
    a.base = base;
    const int64_t D = c.inner(), Dc = c.cross_dim, K = c.coeff();
    const int64_t Dl = D / tp, Fl = 4 * D / tp, Hl = c.heads / tp;
    Work w{};
    w.x = a.take<float>(rows * D);
    w.out32 = a.take<float>(rows * std::max(c.out_ch, 1));
    w.tok_t = a.take<float>(rows);
    w.ts_u = a.take<float>(U);
    w.idx = a.take<int>(rows);
    w.sinus = a.take<float>(U * 256);
    w.h1 = a.take<float>(U * D);
    w.emb = a.take<float>(U * D);
    w.mod = a.take<float>(U * K * D);
    w.tab = a.take<float>((int64_t)L * U * K * D);
    w.otab = a.take<float>(U * 2 * D);
    const int width = c.interleaved ? (int)D : (int)(D / 2);
    w.cos = a.take<float>(rows * width);
    w.sin = a.take<float>(rows * width);
    w.glog = a.take<float>(rows * Hl);
    w.xn = a.take<__nv_bfloat16>(rows * D);
    w.qkv = a.take<__nv_bfloat16>(rows * 3 * Dl);
    w.att = a.take<__nv_bfloat16>(rows * Dl);
    w.q2 = w.qkv;   // cross-attention reuses the self-attention projection buffer
    w.kv2 = a.take<__nv_bfloat16>(crow * 2 * Dl);
    w.ctxb = a.take<__nv_bfloat16>(crow * Dc);
    w.ffh = a.take<__nv_bfloat16>(rows * Fl);
    w.latb = a.take<__nv_bfloat16>(rows * std::max(c.in_ch, 8));
    w.partial = a.take<double>((int64_t)cfg_scratch_bytes() / 8);
    w.part = tp > 1 ? a.take<__nv_bfloat16>(rows * D) : nullptr;
    w.ss = tp > 1 ? a.take<float>(2 * rows + crow) : nullptr;
    if (c.fp8) {
        w.xq = a.take<uint8_t>(rows * 4 * D);
        w.sx = a.take<float>(rows);
        w.cq = a.take<uint8_t>(crow * Dc);
        w.scq = a.take<float>(crow);
        w.xa = a.take<__nv_bfloat16>(rows * std::max(r64, 1));
        w.xac = a.take<__nv_bfloat16>(crow * std::max(r64, 1));
    }
    w.bytes = a.off + 256;
    return w;
}

static int ensure_work(ltx_ctx *ctx, size_t bytes) {
    if (ctx->work_bytes >= bytes) return LTX_OK;
    cudaStreamSynchronize(ctx->stream);
    if (ctx->work) cudaFree(ctx->work);
    ctx->work = nullptr;
    ctx->work_bytes = 0;
    cudaError_t e = cudaMalloc(&ctx->work, bytes);
    if (e != cudaSuccess) return fail(ctx, LTX_ERR_OOM, "forward workspace of %zu bytes: %s", bytes, cudaGetErrorString(e));
    ctx->work_bytes = bytes;
    return LTX_OK;
}

#define CU(x)                                                        \
    do {                                                             \
        cudaError_t _e = (x);                                        \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, #x);        \
    } while (0)

// Distinct per-token timesteps: idx[token] into ts_u (the adaLN path runs on
// these only; model.rs:196-206 runs it per token, with the same result).
static int unique_timesteps(const std::vector<float> &ts, std::vector<float> &uniq, std::vector<int> &idx) {
    std::map<uint32_t, int> pos;
    idx.resize(ts.size());
    for (size_t i = 0; i < ts.size(); ++i) {
        uint32_t bits;
        memcpy(&bits, &ts[i], 4);
        auto it = pos.find(bits);
        if (it == pos.end()) {
            it = pos.emplace(bits, (int)uniq.size()).first;
            uniq.push_back(ts[i]);
        }
        idx[i] = it->second;
    }
    return (int)uniq.size();
}

// One block run on TransformerBlock::forward's own inputs (block.rs:118-126)
// instead of the whole model: the residual x in place, the per-token
// modulation `timestep` [rows, K*D] and the RoPE tables in the reference's
// layout (split: cos, sin (B, H, T, d/2); interleaved: (B, 1, T, D)).
struct BlockSeam {
    int index;
    float *x;
    const float *mod;
    const float *pe_cos, *pe_sin;
};

// The full forward on device buffers.  `ts_host` are the per-token timesteps
// (B*T, host copy) used to build the distinct-timestep index.
// pos_shared: every batch row has the same positions (the CFG halves of a
// denoise step), so the RoPE tables are built for T rows instead of B*T.
// seam: run only block seam->index on the caller's block inputs (no patch
// embedding, adaLN, RoPE table build or output head).
// ts_dev: the per-token timesteps on the device instead (ts_host empty): they
// are deduplicated there into kMaxDistinctTs tables, with no host round trip.
static int forward_impl(ltx_model *m, ltx_ctx *ctx, const float *latent, const std::vector<float> &ts_host,
                        const float *positions, const float *context, int B, int T, int S, float *out,
                        const Work *given = nullptr, Work *work_out = nullptr, bool pos_shared = false,
                        const BlockSeam *seam = nullptr, const float *ts_dev = nullptr) {
    const DitConfig &c = m->cfg;
    if (ctx->tp_size != m->tp || ctx->tp_rank != m->tr)
        return fail(ctx, LTX_ERR_INVALID_ARG, "model shard %d of %d run on a context of rank %d of %d", m->tr, m->tp,
                    ctx->tp_rank, ctx->tp_size);
    const int64_t D = c.inner(), Dc = c.cross_dim, H = c.heads, d = c.head_dim, K = c.coeff();
    const int64_t rows = (int64_t)B * T, crow = (int64_t)B * S;
    cudaStream_t st = ctx->stream;
    const int sms = ctx->sm_count;
    // Split over ranks: the residual lives in the ranks' shared peer memory,
    // where the fused row-split projections update every rank's copy.  Set up
    // first (it is collective and uses the scratch buffer).
    bool peer_x = false;
    if (m->tp > 1 && !seam) TRY(tp_peer_ensure(ctx, rows, D, &peer_x));
    std::vector<float> uniq;
    std::vector<int> idx;
    const int U = seam ? 1 : ts_dev ? kMaxDistinctTs : unique_timesteps(ts_host, uniq, idx);
    Work w;
    float *seam_tab = nullptr;   // seam: per-token tables [rows][K][D]
    if (seam) {
        const size_t wb = carve_work(nullptr, c, rows, crow, 1, 1, m->tp, m->lora_r64).bytes;
        TRY(ensure_work(ctx, wb + (size_t)rows * K * D * sizeof(float) + 256));
        w = carve_work(static_cast<char *>(ctx->work), c, rows, crow, 1, 1, m->tp, m->lora_r64);
        seam_tab = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(ctx->work) + wb + 255) & ~uintptr_t(255));
        w.x = seam->x;
    } else if (given) {
        w = *given;
    } else {
        Work sizing = carve_work(nullptr, c, rows, crow, U, c.layers, m->tp, m->lora_r64);
        TRY(ensure_work(ctx, sizing.bytes));
        w = carve_work(static_cast<char *>(ctx->work), c, rows, crow, U, c.layers, m->tp, m->lora_r64);
    }
    // Sequence-parallel norms on top (D 4096, the vectorised norm kernel): each
    // rank keeps only its own rows of x current (M-blocks [lo(r), lo(r+1)),
    // lo(r) = r * blocks / n), normalises those and sends them into every
    // rank's copy of the normalised rows, which the next GEMMs gather.
    // On by default from 4 ranks (measured 4.8% faster at 4, the same at 2);
    // LTX_TP_SEQ_NORMS=1 / =0 in every rank's environment forces it on / off.
    const char *sp_env = getenv("LTX_TP_SEQ_NORMS");
    const bool sp_want = sp_env && *sp_env ? strcmp(sp_env, "1") == 0 : ctx->tp_size >= 4;
    const bool sp = peer_x && D == 4096 && sp_want;
    if (peer_x) w.x = reinterpret_cast<float *>(ctx->pm.base);
    if (sp) w.xn = reinterpret_cast<__nv_bfloat16 *>(ctx->pm.base + ctx->pm.xn_off);
    if (work_out) *work_out = w;
    if (!seam && ts_dev) {
        CU(timestep_set(st, ts_dev, rows, U, w.ts_u, w.idx, ctx->timeout_flag, kErrTooManyTimesteps));
    } else if (!seam) {
        // one pinned upload: distinct timesteps then the per-token index
        std::vector<char> blob((size_t)U * 4 + (size_t)rows * 4);
        memcpy(blob.data(), uniq.data(), (size_t)U * 4);
        memcpy(blob.data() + (size_t)U * 4, idx.data(), (size_t)rows * 4);
        TRY(ensure_scratch(ctx, blob.size()));
        TRY(upload(ctx, ctx->scratch, blob.data(), blob.size()));
        CU(cudaMemcpyAsync(w.ts_u, ctx->scratch, (size_t)U * 4, cudaMemcpyDeviceToDevice, st));
        CU(cudaMemcpyAsync(w.idx, static_cast<char *>(ctx->scratch) + (size_t)U * 4, (size_t)rows * 4,
                           cudaMemcpyDeviceToDevice, st));
    }

    const int width = c.interleaved ? (int)D : (int)(D / 2);
    // The fused Q/K kernel (D 4096, head dim 128, split RoPE, one GPU) indexes
    // the RoPE table by row % tab_rows, so rows that share positions share
    // table rows.
    const bool fused_qk = m->tp == 1 && D == 4096 && d == 128 && !c.interleaved;
    const int tab_b = fused_qk && pos_shared && !seam ? 1 : B;
    if (!seam) {
        // patch embedding (model.rs:187): f32 latent -> bf16 -> tensor-core GEMM, f32 out
        CU(f32_to_bf16(st, sms, latent, rows * c.in_ch, w.latb));
        TRY(gemm_bf16(ctx, st, w.latb, c.in_ch, m->patch_w, c.in_ch, (int)rows, (int)D, c.in_ch, LTX_EPI_F32,
                      m->patch_b, w.x, D, nullptr, nullptr, 0));
        // adaLN-single on the distinct timesteps (adaln.rs:130-142), f32 throughout
        CU(sinusoid(st, w.ts_u, U, (float)c.ts_mult, m->sin_freq, w.sinus));
        CU(small_linear(st, w.sinus, U, 256, m->t1_w, m->t1_b, (int)D, false, w.h1));
        CU(small_linear(st, w.h1, U, (int)D, m->t2_w, m->t2_b, (int)D, true, w.emb));
        CU(small_linear(st, w.emb, U, (int)D, m->lin_w, m->lin_b, (int)(K * D), true, w.mod));
        CU(ada_tables(st, sms, m->sst_list, c.layers, (int)K, w.mod, m->sst_out, w.emb, U, (int)D, w.tab, w.otab));
        // RoPE tables (rope.rs:46-167), built once per forward, read by every block's Q/K norm
        const float mp[3] = {(float)c.max_pos[0], (float)c.max_pos[1], (float)c.max_pos[2]};
        CU(rope_table(st, sms, positions, tab_b, T, m->rope_freq, m->rope_grid, mp, c.use_mid, c.interleaved, width,
                      w.cos, w.sin));
    } else {
        // the caller's per-token modulation plus this block's table (ada_values)
        CU(seam_tables(st, sms, m->blocks[seam->index].sst, seam->mod, rows, (int)(K * D), seam_tab, w.idx));
        if (c.interleaved) {
            CU(cudaMemcpyAsync(w.cos, seam->pe_cos, (size_t)rows * D * 4, cudaMemcpyDeviceToDevice, st));
            CU(cudaMemcpyAsync(w.sin, seam->pe_sin, (size_t)rows * D * 4, cudaMemcpyDeviceToDevice, st));
        } else {
            CU(pe_rows(st, sms, seam->pe_cos, seam->pe_sin, B, (int)H, T, (int)(d / 2), w.cos, w.sin));
        }
    }
    if (!c.cross_adaln) CU(f32_to_bf16(st, sms, context, crow * Dc, w.ctxb));

    // Tensor-parallel split: this rank runs heads [tr*Hl, (tr+1)*Hl) and FFN
    // units [tr*Fl, (tr+1)*Fl); everything else is replicated.  tp = 1 is the
    // whole model.
    const int tp = m->tp;
    const int64_t Dl = D / tp, Hl = H / tp, Fl = 4 * D / tp, head0 = (int64_t)m->tr * Hl;
    const float scale = 1.0f / sqrtf((float)d);
    auto attend = [&](const __nv_bfloat16 *q, int64_t ldq, const __nv_bfloat16 *k, int64_t ldk, const __nv_bfloat16 *v,
                      int64_t ldv, int Tk) -> int {
        if (d == 128) return attention_fwd(ctx, st, q, ldq, k, ldk, v, ldv, B, (int)Hl, T, Tk, scale, w.att, Dl, true);
        CU(attention_generic(st, q, ldq, k, ldk, v, ldv, B, (int)Hl, T, Tk, (int)d, scale, w.att, Dl));
        return LTX_OK;
    };
    // x += (A . W^T + bias) * gate: fused into the GEMM epilogue on one GPU;
    // split over ranks, the partial products are summed first: inside the
    // GEMM over NVLink peer memory (gemm_tp_resid) when the ranks share it,
    // else by NCCL.  The NCCL path runs the rows in kSlabs token slabs: slab
    // i's sum-allreduce and residual add run on the communicator's stream
    // while the GEMM computes slab i+1 on SMs left free for the collective;
    // the context stream joins after the last slab.
    auto project_residual = [&](const __nv_bfloat16 *a, int64_t lda, const __nv_bfloat16 *wt, int64_t kdim,
                                const float *bias, const float *gate) -> int {
        const int *gidx = gate ? w.idx : nullptr;
        if (tp == 1)
            return gemm_bf16(ctx, st, a, lda, wt, kdim, (int)rows, (int)D, (int)kdim, LTX_EPI_RESID, bias, w.x, D, gate,
                             gidx, K * D);
        // the sum over ranks fused into the GEMM, over NVLink peer memory (the
        // finished rows also go to every rank unless the norms are sequence-parallel)
        if (peer_x && D % 256 == 0)
            return gemm_tp_resid(ctx, st, a, lda, wt, kdim, (int)rows, (int)D, (int)kdim, bias, gate, gidx, K * D, !sp);
        // otherwise NCCL:
        constexpr int kSlabs = 4, kCommSms = 16;
        const int64_t slab = rows >= 16 * 128 ? (rows + kSlabs * 128 - 1) / (kSlabs * 128) * 128 : rows;
        struct GemmSmsGuard {   // restores the GEMM grid on every exit
            ltx_ctx *c;
            ~GemmSmsGuard() { c->gemm_sms = 0; }
        } guard{ctx};
        if (slab < rows) ctx->gemm_sms = ctx->sm_count - kCommSms;
        for (int64_t r0 = 0; r0 < rows; r0 += slab) {
            const int m = (int)std::min<int64_t>(slab, rows - r0);
            // the partial products travel as bf16: half the bytes of the allreduce
            TRY(gemm_bf16(ctx, st, a + r0 * lda, lda, wt, kdim, m, (int)D, (int)kdim, LTX_EPI_BF16, nullptr,
                          w.part + r0 * D, D, nullptr, nullptr, 0));
            TRY(comm_after(ctx));
            TRY(allreduce_sum_bf16_async(ctx, w.part + r0 * D, (size_t)m * D));
            CU(tp_resid_add(ctx->comm_stream ? ctx->comm_stream : st, sms, w.x + r0 * D, w.part + r0 * D, m, (int)D,
                            bias, gate, gidx ? gidx + r0 : nullptr, K * D));
        }
        return comm_join(ctx);
    };
    // x -> w.xn = mod(norm(x)) in `mode`: every row, or with sequence-parallel
    // norms this rank's rows, also written into every other rank's w.xn; the
    // GEMMs that read w.xn next gather the other ranks' rows (agp).
    TpGather ag{};
    const TpGather *agp = sp ? &ag : nullptr;
    auto norm_x = [&](int mode, const float *tabp, int coeff, int k_shift) -> int {
        if (!sp) {
            CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, mode, tabp, coeff, w.idx, k_shift, w.xn, D));
            return LTX_OK;
        }
        TpPeerMem &pm = ctx->pm;
        const int n = ctx->tp_size, me = ctx->tp_rank;
        const int64_t mblk = (rows + 127) / 128;
        const int64_t r0 = (int64_t)me * mblk / n * 128;
        const int64_t r1 = std::min<int64_t>(rows, (int64_t)(me + 1) * mblk / n * 128);
        TpNormPush push{};
        push.n = n;
        push.me = me;
        push.mcap = (int)pm.mblocks_cap;
        push.row0 = (int)r0;
        push.epoch = ++pm.gepoch;
        for (int q = 0; q < n; ++q) {
            push.peer_out[q] = pm.peer[q] + pm.xn_off + (size_t)r0 * D * 2;
            push.peer_stamp[q] = reinterpret_cast<uint32_t *>(pm.peer[q] + pm.gstamp_off);
        }
        push.count = reinterpret_cast<uint32_t *>(pm.base + pm.gcount_off);
        if (r1 > r0)
            CU(norm_mod_push(st, w.x + r0 * D, D, (int)(r1 - r0), c.eps, mode, tabp, coeff, w.idx ? w.idx + r0 : nullptr,
                             k_shift, w.xn + r0 * D, D, push));
        ag = TpGather{reinterpret_cast<const uint32_t *>(pm.base + pm.gstamp_off), pm.gepoch, n, me, (int)pm.mblocks_cap};
        return LTX_OK;
    };
    // RMSNorm(gamma) over the full inner dimension of `nseg` projections that
    // each hold Dl columns per row here (+ RoPE with the tables when given)
    auto norm_split = [&](__nv_bfloat16 *buf, int64_t ld, int nrows, const float *gamma, float *ss, bool rope) -> int {
        CU(tp_norm_apply_rope(st, buf, ld, nrows, (int)Dl, (int)D, (int)d, (int)head0, c.eps, gamma, ss,
                              rope ? w.cos : nullptr, rope ? w.sin : nullptr, c.interleaved));
        return LTX_OK;
    };
    // FP8 path: one projection = e4m3 GEMM of the row-quantised input with the
    // exact FP8 base weight, plus the factored LoRA term in the same
    // accumulator (xa = xq . A_q^T * sa = (x . A^T) / sx, then xa . B2^T).
    auto lin_f8 = [&](const LinF8 &Lw, const uint8_t *xq, int64_t ldx, const float *sx, __nv_bfloat16 *xa, int M, int N,
                      int Kd, int epi, const float *bias, void *out, int64_t ldo, const float *gate, int f16col) -> int {
        GemmLowRank lr{};
        const GemmLowRank *plr = nullptr;
        if (Lw.r64 > 0) {
            TRY(gemm_e4m3(ctx, st, xq, ldx, nullptr, Lw.a, Kd, Lw.sa, M, Lw.r64, Kd, LTX_EPI_BF16, nullptr, xa, Lw.r64,
                          nullptr, nullptr, 0));
            lr = GemmLowRank{xa, Lw.r64, Lw.b2, Lw.r64, Lw.r64};
            plr = &lr;
        }
        return gemm_e4m3(ctx, st, xq, ldx, sx, Lw.w, Kd, Lw.sw, M, N, Kd, epi, bias, out, ldo, gate,
                         gate ? w.idx : nullptr, K * D, f16col, plr);
    };
    if (c.fp8_attn) CU(quantize_rows_e4m3(st, w.ctxb, Dc, (int)crow, (int)Dc, w.cq, Dc, w.scq));
    auto attn_f8 = [&](const BlockW &b, const float *tab) -> int {
        // self-attention
        CU(norm_mod_e4m3(st, w.x, D, (int)rows, (int)D, c.eps, 1, tab, (int)K, w.idx, 0, w.xq, D, w.sx));
        TRY(lin_f8(b.fqkv, w.xq, D, w.sx, w.xa, (int)rows, (int)(3 * D), (int)D, LTX_EPI_BF16, b.qkv_b, w.qkv, 3 * D,
                   nullptr, (int)(2 * D)));
        cudaError_t qe = cudaSuccess;
        if (!qk_norm_rope_fused(st, w.qkv, w.qkv + D, 3 * D, (int)rows, (int)D, c.eps, b.qn, b.kn, w.cos, w.sin,
                                tab_b * T, &qe))
            return fail(ctx, LTX_ERR_UNSUPPORTED, "fused Q/K norm: unexpected layout");
        CU(qe);
        TRY(attend(w.qkv, 3 * D, w.qkv + D, 3 * D, w.qkv + 2 * D, 3 * D, T));
        CU(quantize_rows_e4m3(st, w.att, D, (int)rows, (int)D, w.xq, D, w.sx));
        TRY(lin_f8(b.fo, w.xq, D, w.sx, w.xa, (int)rows, (int)D, (int)D, LTX_EPI_RESID, b.o_b, w.x, D, tab + 2 * D,
                   (int)D));
        // cross-attention
        CU(norm_mod_e4m3(st, w.x, D, (int)rows, (int)D, c.eps, 0, nullptr, 0, nullptr, 0, w.xq, D, w.sx));
        TRY(lin_f8(b.fq2, w.xq, D, w.sx, w.xa, (int)rows, (int)D, (int)D, LTX_EPI_BF16, b.q2_b, w.q2, D, nullptr,
                   (int)D));
        TRY(lin_f8(b.fkv2, w.cq, Dc, w.scq, w.xac, (int)crow, (int)(2 * D), (int)Dc, LTX_EPI_BF16, b.kv2_b, w.kv2,
                   2 * D, nullptr, (int)D));
        CU(qk_norm_rope(st, w.q2, D, (int)rows, (int)D, (int)H, c.eps, b.qn2, nullptr, nullptr, false));
        CU(qk_norm_rope(st, w.kv2, 2 * D, (int)crow, (int)D, (int)H, c.eps, b.kn2, nullptr, nullptr, false));
        TRY(attend(w.q2, D, w.kv2, 2 * D, w.kv2 + D, 2 * D, S));
        CU(quantize_rows_e4m3(st, w.att, D, (int)rows, (int)D, w.xq, D, w.sx));
        TRY(lin_f8(b.fo2, w.xq, D, w.sx, w.xa, (int)rows, (int)D, (int)D, LTX_EPI_RESID, b.o2_b, w.x, D, nullptr,
                   (int)D));
        return LTX_OK;
    };
    auto ffn_f8 = [&](const BlockW &b, const float *tab) -> int {
        CU(norm_mod_e4m3(st, w.x, D, (int)rows, (int)D, c.eps, 1, tab, (int)K, w.idx, 3, w.xq, D, w.sx));
        TRY(lin_f8(b.fff1, w.xq, D, w.sx, w.xa, (int)rows, (int)(4 * D), (int)D, LTX_EPI_GELU_BF16, b.ff1_b, w.ffh,
                   4 * D, nullptr, (int)(4 * D)));
        CU(quantize_rows_e4m3(st, w.ffh, 4 * D, (int)rows, (int)(4 * D), w.xq, 4 * D, w.sx));
        TRY(lin_f8(b.fff2, w.xq, 4 * D, w.sx, w.xa, (int)rows, (int)D, (int)(4 * D), LTX_EPI_RESID, b.ff2_b, w.x, D,
                   tab + 5 * D, (int)D));
        return LTX_OK;
    };
    // OffloadMode::Stream: block l's weights are uploaded into slot l % n on
    // the copy stream once the block that used that slot before (l - n) has
    // been computed; the compute stream waits for the upload.
    const int n_off = m->offload_n;
    auto prefetch = [&](int l) -> int {
        const int slot = l % n_off;
        CU(cudaStreamWaitEvent(m->copy_stream, m->freed[slot], 0));
        CU(cudaMemcpyAsync(m->slot_base[slot], static_cast<char *>(m->host_blocks) + (size_t)l * m->block_bytes,
                           m->block_bytes, cudaMemcpyHostToDevice, m->copy_stream));
        CU(cudaEventRecord(m->copied[slot], m->copy_stream));
        return LTX_OK;
    };
    for (int l = 0; n_off && !seam && l < std::min(n_off, c.layers); ++l) TRY(prefetch(l));
    // one block: x updated in place on the compute stream
    auto block_body = [&](const BlockW &b, const float *tab) -> int {
        if (c.fp8_attn && c.fp8_ffn) {
            TRY(attn_f8(b, tab));
            TRY(ffn_f8(b, tab));
            return LTX_OK;
        }
        // self-attention: x += attn(mod(rms(x))) * gate_msa
        TRY(norm_x(1, tab, (int)K, 0));
        // V columns come out as f16: the attention keeps P in f16 for the P.V MMA
        const int vcol = d == 128 ? (int)(2 * Dl) : (int)(3 * Dl);
        TRY(gemm_bf16(ctx, st, w.xn, D, b.qkv, D, (int)rows, (int)(3 * Dl), (int)D, LTX_EPI_BF16, b.qkv_b, w.qkv,
                      3 * Dl, nullptr, nullptr, 0, vcol, agp));
        if (tp > 1) {
            CU(tp_sumsq_rows(st, w.qkv, 3 * Dl, (int)rows, (int)Dl, 2, Dl, w.ss));
            TRY(allreduce_sum(ctx, w.ss, (size_t)2 * rows));
            TRY(norm_split(w.qkv, 3 * Dl, (int)rows, b.qn, w.ss, true));
            TRY(norm_split(w.qkv + Dl, 3 * Dl, (int)rows, b.kn, w.ss + rows, true));
        } else if (fused_qk) {
            cudaError_t qe = cudaSuccess;
            if (!qk_norm_rope_fused(st, w.qkv, w.qkv + D, 3 * D, (int)rows, (int)D, c.eps, b.qn, b.kn, w.cos, w.sin,
                                    tab_b * T, &qe))
                return fail(ctx, LTX_ERR_UNSUPPORTED, "fused Q/K norm: unexpected layout");
            CU(qe);
        } else {
            CU(qk_norm_rope(st, w.qkv, 3 * D, (int)rows, (int)D, (int)H, c.eps, b.qn, w.cos, w.sin, c.interleaved));
            CU(qk_norm_rope(st, w.qkv + D, 3 * D, (int)rows, (int)D, (int)H, c.eps, b.kn, w.cos, w.sin, c.interleaved));
        }
        TRY(attend(w.qkv, 3 * Dl, w.qkv + Dl, 3 * Dl, w.qkv + 2 * Dl, 3 * Dl, T));
        if (c.gated) {
            TRY(gemm_bf16(ctx, st, w.xn, D, b.g1, D, (int)rows, (int)Hl, (int)D, LTX_EPI_F32, b.g1_b, w.glog, Hl,
                          nullptr, nullptr, 0, 1 << 30, agp));
            CU(head_gate(st, sms, w.att, Dl, w.glog, Hl, (int)rows, (int)Hl, (int)d));
        }
        TRY(project_residual(w.att, Dl, b.o, Dl, b.o_b, tab + 2 * D));
        // cross-attention: x += attn(rms(x), ctx)   [flag path: modulated q, gated, modulated ctx]
        if (c.cross_adaln)
            TRY(norm_x(1, tab, (int)K, 6));
        else
            TRY(norm_x(0, nullptr, 0, 0));
        TRY(gemm_bf16(ctx, st, w.xn, D, b.q2, D, (int)rows, (int)Dl, (int)D, LTX_EPI_BF16, b.q2_b, w.q2, Dl, nullptr,
                      nullptr, 0, 1 << 30, agp));
        if (c.cross_adaln) CU(ctx_mod(st, sms, context, crow * Dc, (int)Dc, b.pst, w.ctxb));
        TRY(gemm_bf16(ctx, st, w.ctxb, Dc, b.kv2, Dc, (int)crow, (int)(2 * Dl), (int)Dc, LTX_EPI_BF16, b.kv2_b, w.kv2,
                      2 * Dl, nullptr, nullptr, 0, d == 128 ? (int)Dl : (int)(2 * Dl)));
        if (tp > 1) {
            CU(tp_sumsq_rows(st, w.q2, Dl, (int)rows, (int)Dl, 1, 0, w.ss));
            CU(tp_sumsq_rows(st, w.kv2, 2 * Dl, (int)crow, (int)Dl, 1, 0, w.ss + rows));
            TRY(allreduce_sum(ctx, w.ss, (size_t)(rows + crow)));
            TRY(norm_split(w.q2, Dl, (int)rows, b.qn2, w.ss, false));
            TRY(norm_split(w.kv2, 2 * Dl, (int)crow, b.kn2, w.ss + rows, false));
        } else {
            CU(qk_norm_rope(st, w.q2, D, (int)rows, (int)D, (int)H, c.eps, b.qn2, nullptr, nullptr, false));
            CU(qk_norm_rope(st, w.kv2, 2 * D, (int)crow, (int)D, (int)H, c.eps, b.kn2, nullptr, nullptr, false));
        }
        TRY(attend(w.q2, Dl, w.kv2, 2 * Dl, w.kv2 + Dl, 2 * Dl, S));
        if (c.gated) {
            TRY(gemm_bf16(ctx, st, w.xn, D, b.g2, D, (int)rows, (int)Hl, (int)D, LTX_EPI_F32, b.g2_b, w.glog, Hl,
                          nullptr, nullptr, 0, 1 << 30, agp));
            CU(head_gate(st, sms, w.att, Dl, w.glog, Hl, (int)rows, (int)Hl, (int)d));
        }
        TRY(project_residual(w.att, Dl, b.o2, Dl, b.o2_b, c.cross_adaln ? tab + 8 * D : nullptr));
        // feed-forward: x += ff(mod(rms(x))) * gate_mlp
        if (c.fp8_ffn) {
            TRY(ffn_f8(b, tab));
            return LTX_OK;
        }
        TRY(norm_x(1, tab, (int)K, 3));
        TRY(gemm_bf16(ctx, st, w.xn, D, b.ff1, D, (int)rows, (int)Fl, (int)D, LTX_EPI_GELU_BF16, b.ff1_b, w.ffh, Fl,
                      nullptr, nullptr, 0, 1 << 30, agp));
        TRY(project_residual(w.ffh, Fl, b.ff2, Fl, b.ff2_b, tab + 5 * D));
        return LTX_OK;
    };
    if (seam) return block_body(m->blocks[seam->index], seam_tab);
    for (int l = 0; l < c.layers; ++l) {
        BlockW bv = m->blocks[l];
        if (n_off) {
            const int slot = l % n_off;
            CU(cudaStreamWaitEvent(st, m->copied[slot], 0));
            bv = m->slots[slot];
            bv.sst = m->blocks[l].sst;
            bv.pst = m->blocks[l].pst;
            copy_scales(bv, m->blocks[l]);
        }
        TRY(block_body(bv, w.tab + (int64_t)l * U * K * D));
        if (n_off) {   // the slot is free once this block's kernels ran; refill it with block l + n
            CU(cudaEventRecord(m->freed[l % n_off], st));
            if (l + n_off < c.layers) TRY(prefetch(l + n_off));
        }
    }
    // output head: LN(x) * (1 + scale) + shift -> proj_out (model.rs:237-254)
    TRY(norm_x(2, w.otab, 2, 0));
    TRY(gemm_bf16(ctx, st, w.xn, D, m->out_w, D, (int)rows, c.out_ch, (int)D, LTX_EPI_F32, m->out_b, out, c.out_ch,
                  nullptr, nullptr, 0, 1 << 30, agp));
    // the next forward's first norm rewrites every rank's gathered rows: no
    // rank may get there while another still reads them here
    if (sp) TRY(tp_peer_barrier(ctx, st));
    return LTX_OK;
}

}  // namespace ltx

using namespace ltx;

extern "C" int ltx_model_load(ltx_ctx *ctx, ltx_store *st, const char *config_json, ltx_model **out) {
    if (!ctx || !st || !out) return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_model_load: null argument") : LTX_ERR_INVALID_ARG;
    *out = nullptr;
    std::string cj;
    if (config_json) {
        cj = config_json;
    } else {
        auto it = st->metadata.find("config");
        if (it == st->metadata.end()) return fail(ctx, LTX_ERR_MISSING_CONFIG, "checkpoint metadata has no \"config\" field");
        cj = it->second;
    }
    DitConfig cfg;
    TRY(parse_config(ctx, cj, cfg));
    if (cfg.fp8)
        return fail(ctx, LTX_ERR_UNSUPPORTED, "gemm_precision e4m3 is built for synthetic models (ltx_model_init_random)");
    ltx_model *m = nullptr;
    TRY(alloc_model(ctx, cfg, m));
    int rc = load_weights(m, st, ctx);
    if (rc) {
        free_model(m);
        return rc;
    }
    *out = m;
    return LTX_OK;
}

extern "C" int ltx_model_init_random(ltx_ctx *ctx, const char *config_json, uint64_t seed, int32_t lora_rank,
                                     float lora_strength, ltx_model **out) {
    if (!ctx || !config_json || !out || lora_rank < 0)
        return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_model_init_random: bad arguments") : LTX_ERR_INVALID_ARG;
    *out = nullptr;
    DitConfig cfg;
    TRY(parse_config(ctx, config_json, cfg));
    ltx_model *m = nullptr;
    TRY(alloc_model(ctx, cfg, m, lora_rank));
    int rc = init_random(m, ctx, seed, lora_rank, lora_strength);
    if (rc) {
        free_model(m);
        return rc;
    }
    *out = m;
    return LTX_OK;
}

extern "C" void ltx_model_destroy(ltx_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    // The model's own copy stream (streamed offload); work on the callers'
    // streams is theirs to finish first (ltx_ctx_synchronize).
    if (m->copy_stream) cudaStreamSynchronize(m->copy_stream);
    free_model(m);
}

extern "C" int64_t ltx_model_weight_bytes(const ltx_model *m) { return m ? (int64_t)m->arena_bytes : 0; }

extern "C" int ltx_model_forward(ltx_model *m, ltx_ctx *ctx, const float *latent_dev, const float *timesteps_dev,
                                 const float *positions_dev, const float *context_dev, int32_t batch, int32_t tokens,
                                 int32_t context_tokens, float *out_dev) {
    if (!m || !ctx || !latent_dev || !timesteps_dev || !positions_dev || !context_dev || !out_dev)
        return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_model_forward: null argument") : LTX_ERR_INVALID_ARG;
    if (batch <= 0 || tokens <= 0 || context_tokens <= 0)
        return fail(ctx, LTX_ERR_SHAPE, "ltx_model_forward: empty batch/tokens/context");
    return forward_impl(m, ctx, latent_dev, {}, positions_dev, context_dev, batch, tokens, context_tokens, out_dev,
                        nullptr, nullptr, false, nullptr, timesteps_dev);
}

extern "C" int ltx_block_forward(ltx_model *m, ltx_ctx *ctx, int32_t block_index, float *x_dev,
                                 const float *context_dev, const float *timestep_dev, const float *pe_cos_dev,
                                 const float *pe_sin_dev, int32_t batch, int32_t tokens, int32_t context_tokens) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!m || !x_dev || !context_dev || !timestep_dev || !pe_cos_dev || !pe_sin_dev)
        return fail(ctx, LTX_ERR_INVALID_ARG, "ltx_block_forward: null argument");
    if (block_index < 0 || block_index >= m->cfg.layers)
        return fail(ctx, LTX_ERR_INVALID_ARG, "ltx_block_forward: block %d of %d", block_index, m->cfg.layers);
    if (batch <= 0 || tokens <= 0 || context_tokens <= 0)
        return fail(ctx, LTX_ERR_SHAPE, "ltx_block_forward: empty batch/tokens/context");
    if (m->offload_n)
        return fail(ctx, LTX_ERR_UNSUPPORTED, "ltx_block_forward: the model keeps its blocks in host memory "
                                              "(offload_blocks); run it through ltx_model_forward");
    const BlockSeam seam{block_index, x_dev, timestep_dev, pe_cos_dev, pe_sin_dev};
    return forward_impl(m, ctx, nullptr, {}, nullptr, context_dev, batch, tokens, context_tokens, nullptr, nullptr,
                        nullptr, false, &seam);
}

// GuidedDenoiser::apply's combine (guidance.rs:149-165) + post_process and
// euler_step (loop_.rs:37-65) on x0 predictions from any denoiser.
extern "C" int ltx_cfg_euler_step(ltx_ctx *ctx, const float *cond_x0_dev, const float *uncond_x0_dev,
                                  float *latent_dev, const float *clean_dev, const float *mask_dev, int32_t tokens,
                                  int32_t channels, float sigma, float sigma_next, float cfg_scale,
                                  float rescale_scale) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!cond_x0_dev || !latent_dev || !clean_dev || !mask_dev)
        return fail(ctx, LTX_ERR_INVALID_ARG, "ltx_cfg_euler_step: null argument");
    if (tokens < 0 || channels <= 0) return fail(ctx, LTX_ERR_SHAPE, "ltx_cfg_euler_step: bad shape");
    if (!std::isfinite(sigma) || sigma <= 0.f) return fail(ctx, LTX_ERR_SIGMA, "invalid sigma %g", (double)sigma);
    if (!std::isfinite(sigma_next) || sigma_next < 0.f)
        return fail(ctx, LTX_ERR_SIGMA, "invalid next sigma %g", (double)sigma_next);
    const bool use_cfg = std::fabs(cfg_scale - 1.0f) > 1e-5f;   // needs_uncond (guidance.rs:58-60)
    if (use_cfg && !uncond_x0_dev)
        return fail(ctx, LTX_ERR_NEGATIVE_CONTEXT, "cfg_scale != 1 needs the unconditional prediction");
    if (tokens == 0) return LTX_OK;
    TRY(ensure_scratch(ctx, cfg_scratch_bytes()));
    CU(cfg_euler(ctx->stream, ctx->sm_count, latent_dev, cond_x0_dev, use_cfg ? uncond_x0_dev : cond_x0_dev, nullptr,
                 mask_dev, clean_dev, tokens, channels, cfg_scale, rescale_scale, use_cfg,
                 static_cast<double *>(ctx->scratch), sigma, sigma_next));
    return LTX_OK;
}

namespace ltx {

// Step buffers ahead of the forward's workspace in ctx->work, so that their
// offsets do not depend on the forward's sizing: the batch-2 latent copy, the
// velocity output, and the batch-2 positions and contexts.
struct StepBufs {
    float *lat2, *vel, *pos2, *ctx2;
    size_t bytes;
};

static StepBufs carve_step(char *base, const DitConfig &c, int B, int T, int S) {
    Arena a;
    a.base = base;
    StepBufs b{};
    b.lat2 = a.take<float>((int64_t)B * T * c.in_ch);
    b.vel = a.take<float>((int64_t)2 * T * c.out_ch);   // both CFG passes (a pair rank gathers the other's)
    b.pos2 = a.take<float>((int64_t)B * 3 * T * 2);
    b.ctx2 = a.take<float>((int64_t)B * S * c.cross_dim);
    b.bytes = (a.off + 255) & ~size_t(255);
    return b;
}

// Bytes of ctx->work one step needs with U distinct timesteps.
static size_t step_work_bytes(const ltx_model *m, int B, int T, int S, int U) {
    const DitConfig &c = m->cfg;
    return carve_step(nullptr, c, B, T, S).bytes +
           carve_work(nullptr, c, (int64_t)B * T, (int64_t)B * S, U, c.layers, m->tp, m->lora_r64).bytes;
}

// Copies positions and the cond/uncond contexts into the batch-2 layout.
static int stage_static(ltx_ctx *ctx, const StepBufs &sb, const float *positions_dev, const float *cc,
                        const float *cu, int B, int T, int S, int64_t Dc) {
    cudaStream_t st = ctx->stream;
    for (int b = 0; b < B; ++b) {
        CU(cudaMemcpyAsync(sb.pos2 + (int64_t)b * 3 * T * 2, positions_dev, (size_t)3 * T * 2 * 4,
                           cudaMemcpyDeviceToDevice, st));
        CU(cudaMemcpyAsync(sb.ctx2 + (int64_t)b * S * Dc, b == 0 ? cc : cu, (size_t)S * Dc * 4,
                           cudaMemcpyDeviceToDevice, st));
    }
    return LTX_OK;
}

// Rows of the CFG batch this context's forward computes: both passes (2),
// one when CFG is off, or one when the context is half of a CFG pair.
static int forward_batch(const ltx_ctx *ctx, bool use_cfg) { return use_cfg && !ctx->cfg_comm ? 2 : 1; }

// Positions and the context(s) of this context's forward into the step
// buffers: cond then uncond, or the pair rank's own (0: cond, 1: uncond).
static int stage_for_step(ltx_ctx *ctx, const StepBufs &sb, const float *positions_dev, const float *cc,
                          const float *cu, bool use_cfg, int T, int S, int64_t Dc) {
    if (use_cfg && ctx->cfg_comm)
        return stage_static(ctx, sb, positions_dev, ctx->cfg_rank == 0 ? cc : cu, nullptr, 1, T, S, Dc);
    return stage_static(ctx, sb, positions_dev, cc, cu, forward_batch(ctx, use_cfg), T, S, Dc);
}

// One Euler step of euler_denoising_loop (loop_.rs:93-149) with GuidedDenoiser::apply
// (guidance.rs:102-166): the cond and uncond passes run as ONE batch-2 forward,
// then the CFG/rescale combine, post_process and the Euler update in one kernel.
// On a CFG pair each rank runs its own pass (batch 1) and the two velocities
// are all-gathered before the update, which every rank then computes from the
// same inputs.  Arguments are validated by the callers.  static_ready:
// positions/contexts are already in the step buffers (the loop stages them once).
static int denoise_step_core(ltx_model *m, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                             const float *mask_host, const float *mask_dev, const float *positions_dev,
                             const float *cc, const float *cu, int T, int S, float sigma, float sigma_next,
                             float cfg_scale, float rescale_scale, bool static_ready) {
    const DitConfig &c = m->cfg;
    const bool use_cfg = std::fabs(cfg_scale - 1.0f) > 1e-5f;   // needs_uncond (guidance.rs:58-60)
    const bool pair = use_cfg && ctx->cfg_comm;                 // this rank runs one pass of the CFG batch
    const int B = forward_batch(ctx, use_cfg), C = c.in_ch;
    cudaStream_t st = ctx->stream;
    // per-token timesteps = mask * sigma (guidance.rs:114), each CFG row:
    // on the host when the caller has the mask there, else on the device
    std::vector<float> ts;
    int U = kMaxDistinctTs;
    if (mask_host) {
        ts.resize((size_t)B * T);
        for (int b = 0; b < B; ++b)
            for (int t = 0; t < T; ++t) ts[(size_t)b * T + t] = mask_host[t] * sigma;
        std::vector<float> uq;
        std::vector<int> ix;
        U = unique_timesteps(ts, uq, ix);
    }
    TRY(ensure_work(ctx, step_work_bytes(m, B, T, S, U)));   // grow-only: a no-op inside a loop
    char *base = static_cast<char *>(ctx->work);
    const StepBufs sb = carve_step(base, c, B, T, S);
    Work w = carve_work(base + sb.bytes, c, (int64_t)B * T, (int64_t)B * S, U, c.layers, m->tp, m->lora_r64);
    if (!static_ready) TRY(stage_for_step(ctx, sb, positions_dev, cc, cu, use_cfg, T, S, c.cross_dim));
    for (int b = 0; b < B; ++b)
        CU(cudaMemcpyAsync(sb.lat2 + (int64_t)b * T * C, latent_dev, (size_t)T * C * 4, cudaMemcpyDeviceToDevice, st));
    // a pair rank's velocity goes to its own slot: cond [0, T*C), uncond [T*C, 2*T*C)
    float *vel = pair ? sb.vel + (int64_t)ctx->cfg_rank * T * C : sb.vel;
    if (mask_host) {
        TRY(forward_impl(m, ctx, sb.lat2, ts, sb.pos2, sb.ctx2, B, T, S, vel, &w, nullptr, true));
        // per-token t for the velocity -> x0 adapter: x0 = x - t * v
        TRY(upload(ctx, w.tok_t, ts.data(), (size_t)T * 4));
    } else {
        CU(mask_timesteps(st, ctx->sm_count, mask_dev, sigma, T, B, w.tok_t));
        TRY(forward_impl(m, ctx, sb.lat2, {}, sb.pos2, sb.ctx2, B, T, S, vel, &w, nullptr, true, nullptr, w.tok_t));
    }
    if (pair) TRY(cfg_allgather(ctx, sb.vel, (size_t)T * C));
    CU(cfg_euler(st, ctx->sm_count, latent_dev, sb.vel, use_cfg ? sb.vel + (int64_t)T * C : sb.vel, w.tok_t, mask_dev,
                 clean_dev, T, C, cfg_scale, rescale_scale, use_cfg, w.partial, sigma, sigma_next));
    return LTX_OK;
}

// Validation shared by the step and the loop entry points.
static int check_step_args(ltx_model *m, ltx_ctx *ctx, const void *latent_dev, const void *clean_dev,
                           const void *mask_dev, const void *positions_dev, const void *cc, const void *cu,
                           int32_t tokens, int32_t context_tokens, float cfg_scale, const char *who) {
    if (!m || !latent_dev || !clean_dev || !mask_dev || !positions_dev || !cc)
        return fail(ctx, LTX_ERR_INVALID_ARG, "%s: null argument", who);
    if (tokens <= 0 || context_tokens <= 0) return fail(ctx, LTX_ERR_SHAPE, "%s: empty tokens/context", who);
    if (std::fabs(cfg_scale - 1.0f) > 1e-5f && !cu)
        return fail(ctx, LTX_ERR_NEGATIVE_CONTEXT, "cfg_scale != 1 needs a negative context");
    if (m->cfg.in_ch != m->cfg.out_ch) return fail(ctx, LTX_ERR_CONFIG, "denoising needs in_channels == out_channels");
    return LTX_OK;
}

}  // namespace ltx

extern "C" int ltx_denoise_step(ltx_model *m, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                                const float *mask_host, const float *mask_dev, const float *positions_dev,
                                const float *ctx_cond_dev, const float *ctx_uncond_dev, int32_t tokens,
                                int32_t context_tokens, float sigma, float sigma_next, float cfg_scale,
                                float rescale_scale) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    TRY(check_step_args(m, ctx, latent_dev, clean_dev, mask_dev, positions_dev, ctx_cond_dev, ctx_uncond_dev, tokens,
                        context_tokens, cfg_scale, "ltx_denoise_step"));
    if (!std::isfinite(sigma) || sigma <= 0.f) return fail(ctx, LTX_ERR_SIGMA, "invalid sigma %g", (double)sigma);
    if (!std::isfinite(sigma_next) || sigma_next < 0.f)
        return fail(ctx, LTX_ERR_SIGMA, "invalid next sigma %g", (double)sigma_next);
    return denoise_step_core(m, ctx, latent_dev, clean_dev, mask_host, mask_dev, positions_dev, ctx_cond_dev,
                             ctx_uncond_dev, tokens, context_tokens, sigma, sigma_next, cfg_scale, rescale_scale, false);
}

// euler_denoising_loop (loop_.rs:93-149) + clear_conditioning (loop_.rs:162-185)
// on the device: every step is enqueued without a host round trip; the
// positions and contexts are staged once, the workspace is sized once for the
// whole schedule.
extern "C" int ltx_denoise_loop(ltx_model *m, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                                const float *mask_host, const float *mask_dev, const float *positions_dev,
                                const float *ctx_cond_dev, const float *ctx_uncond_dev, int32_t tokens,
                                int32_t context_tokens, const float *sigmas_host, int32_t n_sigmas, float cfg_scale,
                                float rescale_scale, int32_t target_tokens, float *out_dev) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    TRY(check_step_args(m, ctx, latent_dev, clean_dev, mask_dev, positions_dev, ctx_cond_dev, ctx_uncond_dev, tokens,
                        context_tokens, cfg_scale, "ltx_denoise_loop"));
    if (!sigmas_host || n_sigmas < 2)
        return fail(ctx, LTX_ERR_SCHEDULE, "schedule has %d sigmas; need at least 2", sigmas_host ? n_sigmas : 0);
    // the reference checks each pair as it reaches it and returns no state on
    // error, so checking every pair first gives the same result
    for (int i = 0; i + 1 < n_sigmas; ++i) {
        const float s = sigmas_host[i], sn = sigmas_host[i + 1];
        if (!std::isfinite(s) || s <= 0.f) return fail(ctx, LTX_ERR_SIGMA, "step %d: invalid sigma %g", i, (double)s);
        if (!std::isfinite(sn) || sn < 0.f)
            return fail(ctx, LTX_ERR_SIGMA, "step %d: invalid sigma %g", i + 1, (double)sn);
    }
    if (target_tokens < 0 || target_tokens > tokens)
        return fail(ctx, LTX_ERR_TARGET_TOKENS, "target token count %d exceeds the state's %d tokens", target_tokens,
                    tokens);
    const DitConfig &c = m->cfg;
    const bool use_cfg = std::fabs(cfg_scale - 1.0f) > 1e-5f;
    const int B = forward_batch(ctx, use_cfg), T = tokens, S = context_tokens;
    // distinct mask values bound the distinct timesteps of every step (the
    // device path sizes for kMaxDistinctTs)
    int U = kMaxDistinctTs;
    if (mask_host) {
        std::set<uint32_t> mvals;
        for (int t = 0; t < T; ++t) {
            uint32_t bits;
            memcpy(&bits, &mask_host[t], 4);
            mvals.insert(bits);
        }
        U = (int)mvals.size();
    }
    TRY(ensure_work(ctx, step_work_bytes(m, B, T, S, U)));
    const StepBufs sb = carve_step(static_cast<char *>(ctx->work), c, B, T, S);
    TRY(stage_for_step(ctx, sb, positions_dev, ctx_cond_dev, ctx_uncond_dev, use_cfg, T, S, c.cross_dim));
    for (int i = 0; i + 1 < n_sigmas; ++i)
        TRY(denoise_step_core(m, ctx, latent_dev, clean_dev, mask_host, mask_dev, positions_dev, ctx_cond_dev,
                              ctx_uncond_dev, T, S, sigmas_host[i], sigmas_host[i + 1], cfg_scale, rescale_scale, true));
    if (out_dev && target_tokens > 0)
        CU(cudaMemcpyAsync(out_dev, latent_dev, (size_t)target_tokens * c.in_ch * 4, cudaMemcpyDeviceToDevice,
                           ctx->stream));
    return LTX_OK;
}
