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
#include <cstring>
#include <map>
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
    return LTX_OK;
}

struct BlockW {
    __nv_bfloat16 *qkv, *o, *q2, *kv2, *o2, *ff1, *ff2, *g1, *g2;
    float *qkv_b, *o_b, *q2_b, *kv2_b, *o2_b, *ff1_b, *ff2_b, *g1_b, *g2_b;
    float *qn, *kn, *qn2, *kn2, *sst, *pst;
};

}  // namespace ltx

struct ltx_model {
    int device = 0;
    ltx::DitConfig cfg;
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
static void layout(ltx_model *m, Arena &a) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, F = 4 * D, H = c.heads, K = c.coeff();
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
    for (auto &b : m->blocks) {
        b.qkv = a.take<__nv_bfloat16>(3 * D * D);
        b.qkv_b = a.take<float>(3 * D);
        b.qn = a.take<float>(D);
        b.kn = a.take<float>(D);
        b.o = a.take<__nv_bfloat16>(D * D);
        b.o_b = a.take<float>(D);
        b.q2 = a.take<__nv_bfloat16>(D * D);
        b.q2_b = a.take<float>(D);
        b.kv2 = a.take<__nv_bfloat16>(2 * D * Dc);
        b.kv2_b = a.take<float>(2 * D);
        b.qn2 = a.take<float>(D);
        b.kn2 = a.take<float>(D);
        b.o2 = a.take<__nv_bfloat16>(D * D);
        b.o2_b = a.take<float>(D);
        b.ff1 = a.take<__nv_bfloat16>(F * D);
        b.ff1_b = c.ff_bias ? a.take<float>(F) : nullptr;
        b.ff2 = a.take<__nv_bfloat16>(D * F);
        b.ff2_b = c.ff_bias ? a.take<float>(D) : nullptr;
        b.sst = a.take<float>(K * D);
        b.pst = c.cross_adaln ? a.take<float>(2 * D) : nullptr;
        b.g1 = c.gated ? a.take<__nv_bfloat16>(H * D) : nullptr;
        b.g1_b = c.gated ? a.take<float>(H) : nullptr;
        b.g2 = c.gated ? a.take<__nv_bfloat16>(H * D) : nullptr;
        b.g2_b = c.gated ? a.take<float>(H) : nullptr;
    }
}

static int alloc_model(ltx_ctx *ctx, const DitConfig &cfg, ltx_model *&m) {
    m = new (std::nothrow) ltx_model();
    if (!m) return LTX_ERR_OOM;
    m->device = ctx->device;
    m->cfg = cfg;
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

// ── loading from a weight store (load.rs:47-396) ─────────────────────────────

struct Loader {
    ltx_store *st;
    ltx_ctx *ctx;
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
    int req(const std::string &key, std::vector<int64_t> shape, void *dst, int dt) {
        int rc = shape_check(key, shape);
        if (rc) return rc;
        return store_read_device(st, key, dt, dst, numel(shape));
    }
    // optional tensor (bias): absent -> left zero, returns whether present
    int opt(const std::string &key, std::vector<int64_t> shape, void *dst, int dt, bool *present = nullptr) {
        if (!st->entries.count(key)) {
            if (present) *present = false;
            return LTX_OK;
        }
        if (present) *present = true;
        return req(key, shape, dst, dt);
    }
};

#define TRY(x)                   \
    do {                         \
        int _rc = (x);           \
        if (_rc) return _rc;     \
    } while (0)

static int load_weights(ltx_model *m, ltx_store *st, ltx_ctx *ctx) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, F = 4 * D, H = c.heads, K = c.coeff();
    Loader L{st, ctx};
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
        BlockW &b = m->blocks[i];
        const std::string p = "transformer_blocks." + std::to_string(i) + ".";
        const std::string a1 = p + "attn1.", a2 = p + "attn2.";
        TRY(L.req(a1 + "to_q.weight", {D, D}, b.qkv, LTX_BF16));
        TRY(L.req(a1 + "to_k.weight", {D, D}, b.qkv + D * D, LTX_BF16));
        TRY(L.req(a1 + "to_v.weight", {D, D}, b.qkv + 2 * D * D, LTX_BF16));
        TRY(L.opt(a1 + "to_q.bias", {D}, b.qkv_b, LTX_F32));
        TRY(L.opt(a1 + "to_k.bias", {D}, b.qkv_b + D, LTX_F32));
        TRY(L.opt(a1 + "to_v.bias", {D}, b.qkv_b + 2 * D, LTX_F32));
        TRY(L.req(a1 + "q_norm.weight", {D}, b.qn, LTX_F32));
        TRY(L.req(a1 + "k_norm.weight", {D}, b.kn, LTX_F32));
        TRY(L.req(a1 + "to_out.0.weight", {D, D}, b.o, LTX_BF16));
        TRY(L.opt(a1 + "to_out.0.bias", {D}, b.o_b, LTX_F32));
        TRY(L.req(a2 + "to_q.weight", {D, D}, b.q2, LTX_BF16));
        TRY(L.opt(a2 + "to_q.bias", {D}, b.q2_b, LTX_F32));
        TRY(L.req(a2 + "to_k.weight", {D, Dc}, b.kv2, LTX_BF16));
        TRY(L.req(a2 + "to_v.weight", {D, Dc}, b.kv2 + D * Dc, LTX_BF16));
        TRY(L.opt(a2 + "to_k.bias", {D}, b.kv2_b, LTX_F32));
        TRY(L.opt(a2 + "to_v.bias", {D}, b.kv2_b + D, LTX_F32));
        TRY(L.req(a2 + "q_norm.weight", {D}, b.qn2, LTX_F32));
        TRY(L.req(a2 + "k_norm.weight", {D}, b.kn2, LTX_F32));
        TRY(L.req(a2 + "to_out.0.weight", {D, D}, b.o2, LTX_BF16));
        TRY(L.opt(a2 + "to_out.0.bias", {D}, b.o2_b, LTX_F32));
        if (c.gated) {
            TRY(L.req(a1 + "to_gate_logits.weight", {H, D}, b.g1, LTX_BF16));
            TRY(L.opt(a1 + "to_gate_logits.bias", {H}, b.g1_b, LTX_F32));
            TRY(L.req(a2 + "to_gate_logits.weight", {H, D}, b.g2, LTX_BF16));
            TRY(L.opt(a2 + "to_gate_logits.bias", {H}, b.g2_b, LTX_F32));
        }
        TRY(L.req(p + "ff.net.0.proj.weight", {F, D}, b.ff1, LTX_BF16));
        TRY(L.req(p + "ff.net.2.weight", {D, F}, b.ff2, LTX_BF16));
        if (c.ff_bias) {
            TRY(L.opt(p + "ff.net.0.proj.bias", {F}, b.ff1_b, LTX_F32));
            TRY(L.opt(p + "ff.net.2.bias", {D}, b.ff2_b, LTX_F32));
        }
        TRY(L.req(p + "scale_shift_table", {K, D}, b.sst, LTX_F32));
        if (c.cross_adaln) TRY(L.req(p + "prompt_scale_shift_table", {2, D}, b.pst, LTX_F32));
    }
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "model load");
    return LTX_OK;
}

// ── synthetic FP8 + LoRA checkpoint on the device ────────────────────────────

struct Synth {
    ltx_ctx *ctx;
    uint64_t seed;
    int rank;
    float strength;
    uint64_t sid = 1;
    float *f32 = nullptr;        // [max numel]
    uint8_t *q8 = nullptr;       // [max numel]
    __nv_bfloat16 *la = nullptr, *lb = nullptr;
    float *scale_dev = nullptr;
    unsigned int *work = nullptr;
    // W ~ N(0, 0.02) -> e4m3 with scale amax/448; LoRA A [r, in], B [out, r]
    // bf16 ~ N(0, 0.01), alpha = rank; merged through ltx_dequant_merge.
    int linear(void *dst, int64_t out, int64_t in, int dst_dt) {
        const int64_t n = out * in;
        cudaStream_t st = ctx->stream;
        LTX_CUDA_TRY(ctx, synth_normal_f32(st, ctx->sm_count, f32, n, seed, sid++, 0.f, 0.02f));
        LTX_CUDA_TRY(ctx, synth_quantize_fp8(st, ctx->sm_count, f32, n, q8, scale_dev, work));
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
        return dequant_merge(ctx, st, q8, LTX_F8_E4M3, 1, scale, out, in, &d, nd, dst, dst_dt);
    }
    int vec(float *dst, int64_t n, float mean, float std) {
        LTX_CUDA_TRY(ctx, synth_normal_f32(ctx->stream, ctx->sm_count, dst, n, seed, sid++, mean, std));
        return LTX_OK;
    }
};

static int init_random(ltx_model *m, ltx_ctx *ctx, uint64_t seed, int rank, float strength) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, F = 4 * D, H = c.heads, K = c.coeff();
    const int64_t maxn = std::max<int64_t>({F * D, K * D * D, 2 * D * Dc, 3 * D * D});
    Synth s{ctx, seed, rank, strength};
    // scratch: f32 weight [maxn] | fp8 [maxn] | LoRA A [rank*max_in] | LoRA B [max_out*rank] | scale | amax
    const int64_t max_in = std::max<int64_t>({F, Dc, D, 256, (int64_t)c.in_ch});
    const int64_t max_out = std::max<int64_t>({K * D, F, 3 * D, 2 * D, (int64_t)c.out_ch});
    Arena sz;
    sz.take<float>(maxn);
    sz.take<uint8_t>(maxn);
    sz.take<__nv_bfloat16>((int64_t)rank * max_in);
    sz.take<__nv_bfloat16>(max_out * rank);
    sz.take<float>(1);
    sz.take<unsigned int>(1);
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
    int rc = [&]() -> int {
        TRY(s.linear(m->patch_w, D, c.in_ch, LTX_BF16));
        TRY(s.linear(m->t1_w, D, 256, LTX_F32));
        TRY(s.linear(m->t2_w, D, D, LTX_F32));
        TRY(s.linear(m->lin_w, K * D, D, LTX_F32));
        TRY(s.vec(m->sst_out, 2 * D, 0.f, 0.02f));
        TRY(s.linear(m->out_w, c.out_ch, D, LTX_BF16));
        for (auto &b : m->blocks) {
            TRY(s.linear(b.qkv, 3 * D, D, LTX_BF16));
            TRY(s.linear(b.o, D, D, LTX_BF16));
            TRY(s.linear(b.q2, D, D, LTX_BF16));
            TRY(s.linear(b.kv2, 2 * D, Dc, LTX_BF16));
            TRY(s.linear(b.o2, D, D, LTX_BF16));
            TRY(s.linear(b.ff1, F, D, LTX_BF16));
            TRY(s.linear(b.ff2, D, F, LTX_BF16));
            TRY(s.vec(b.qn, D, 1.f, 0.02f));
            TRY(s.vec(b.kn, D, 1.f, 0.02f));
            TRY(s.vec(b.qn2, D, 1.f, 0.02f));
            TRY(s.vec(b.kn2, D, 1.f, 0.02f));
            TRY(s.vec(b.sst, K * D, 0.f, 0.02f));
            if (b.pst) TRY(s.vec(b.pst, 2 * D, 0.f, 0.02f));
            if (b.g1) {
                TRY(s.linear(b.g1, H, D, LTX_BF16));
                TRY(s.linear(b.g2, H, D, LTX_BF16));
            }
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
    size_t bytes;
};

static Work carve_work(char *base, const DitConfig &c, int64_t rows, int64_t crow, int U, int L) {
    Arena a;
    a.base = base;
    const int64_t D = c.inner(), Dc = c.cross_dim, K = c.coeff();
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
    w.glog = a.take<float>(rows * c.heads);
    w.xn = a.take<__nv_bfloat16>(rows * D);
    w.qkv = a.take<__nv_bfloat16>(rows * 3 * D);
    w.att = a.take<__nv_bfloat16>(rows * D);
    w.q2 = w.qkv;   // cross-attention reuses the self-attention projection buffer
    w.kv2 = a.take<__nv_bfloat16>(crow * 2 * D);
    w.ctxb = a.take<__nv_bfloat16>(crow * Dc);
    w.ffh = a.take<__nv_bfloat16>(rows * 4 * D);
    w.latb = a.take<__nv_bfloat16>(rows * std::max(c.in_ch, 8));
    w.partial = a.take<double>((int64_t)cfg_scratch_bytes() / 8);
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

// The full forward on device buffers.  `ts_host` are the per-token timesteps
// (B*T, host copy) used to build the distinct-timestep index.
static int forward_impl(ltx_model *m, ltx_ctx *ctx, const float *latent, const std::vector<float> &ts_host,
                        const float *positions, const float *context, int B, int T, int S, float *out,
                        const Work *given = nullptr, Work *work_out = nullptr) {
    const DitConfig &c = m->cfg;
    const int64_t D = c.inner(), Dc = c.cross_dim, H = c.heads, d = c.head_dim, K = c.coeff();
    const int64_t rows = (int64_t)B * T, crow = (int64_t)B * S;
    cudaStream_t st = ctx->stream;
    const int sms = ctx->sm_count;
    std::vector<float> uniq;
    std::vector<int> idx;
    const int U = unique_timesteps(ts_host, uniq, idx);
    Work w;
    if (given) {
        w = *given;
    } else {
        Work sizing = carve_work(nullptr, c, rows, crow, U, c.layers);
        TRY(ensure_work(ctx, sizing.bytes));
        w = carve_work(static_cast<char *>(ctx->work), c, rows, crow, U, c.layers);
    }
    if (work_out) *work_out = w;
    {
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

    // patch embedding (model.rs:187): f32 latent -> bf16 -> tensor-core GEMM, f32 out
    CU(f32_to_bf16(st, sms, latent, rows * c.in_ch, w.latb));
    TRY(gemm_bf16(ctx, st, w.latb, c.in_ch, m->patch_w, c.in_ch, (int)rows, (int)D, c.in_ch, LTX_EPI_F32, m->patch_b,
                  w.x, D, nullptr, nullptr, 0));
    // adaLN-single on the distinct timesteps (adaln.rs:130-142), f32 throughout
    CU(sinusoid(st, w.ts_u, U, (float)c.ts_mult, m->sin_freq, w.sinus));
    CU(small_linear(st, w.sinus, U, 256, m->t1_w, m->t1_b, (int)D, false, w.h1));
    CU(small_linear(st, w.h1, U, (int)D, m->t2_w, m->t2_b, (int)D, true, w.emb));
    CU(small_linear(st, w.emb, U, (int)D, m->lin_w, m->lin_b, (int)(K * D), true, w.mod));
    CU(ada_tables(st, sms, m->sst_list, c.layers, (int)K, w.mod, m->sst_out, w.emb, U, (int)D, w.tab, w.otab));
    // RoPE tables (rope.rs:46-167)
    const float mp[3] = {(float)c.max_pos[0], (float)c.max_pos[1], (float)c.max_pos[2]};
    const int width = c.interleaved ? (int)D : (int)(D / 2);
    // The fused Q/K kernel computes RoPE angles in registers for the production
    // shape (D 4096, head dim 128, split RoPE); other shapes use the tables.
    const bool fused_qk = D == 4096 && d == 128 && !c.interleaved;
    if (!fused_qk)
        CU(rope_table(st, sms, positions, B, T, m->rope_freq, m->rope_grid, mp, c.use_mid, c.interleaved, width, w.cos,
                      w.sin));
    if (!c.cross_adaln) CU(f32_to_bf16(st, sms, context, crow * Dc, w.ctxb));

    const float scale = 1.0f / sqrtf((float)d);
    auto attend = [&](const __nv_bfloat16 *q, int64_t ldq, const __nv_bfloat16 *k, int64_t ldk, const __nv_bfloat16 *v,
                      int64_t ldv, int Tk) -> int {
        if (d == 128) return attention_fwd(ctx, st, q, ldq, k, ldk, v, ldv, B, (int)H, T, Tk, scale, w.att, D, true);
        CU(attention_generic(st, q, ldq, k, ldk, v, ldv, B, (int)H, T, Tk, (int)d, scale, w.att, D));
        return LTX_OK;
    };
    for (int l = 0; l < c.layers; ++l) {
        const BlockW &b = m->blocks[l];
        const float *tab = w.tab + (int64_t)l * U * K * D;
        // self-attention: x += attn(mod(rms(x))) * gate_msa
        CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, 1, tab, (int)K, w.idx, 0, w.xn, D));
        // V columns come out as f16: the attention keeps P in f16 for the P.V MMA
        const int vcol = d == 128 ? (int)(2 * D) : (int)(3 * D);
        TRY(gemm_bf16(ctx, st, w.xn, D, b.qkv, D, (int)rows, (int)(3 * D), (int)D, LTX_EPI_BF16, b.qkv_b, w.qkv,
                      3 * D, nullptr, nullptr, 0, vcol));
        if (fused_qk) {
            cudaError_t qe = cudaSuccess;
            qk_norm_rope_fused(st, w.qkv, w.qkv + D, 3 * D, (int)rows, T, (int)D, c.eps, b.qn, b.kn, positions,
                               m->rope_freq, m->rope_grid, mp, c.use_mid, &qe);
            CU(qe);
        } else {
            CU(qk_norm_rope(st, w.qkv, 3 * D, (int)rows, (int)D, (int)H, c.eps, b.qn, w.cos, w.sin, c.interleaved));
            CU(qk_norm_rope(st, w.qkv + D, 3 * D, (int)rows, (int)D, (int)H, c.eps, b.kn, w.cos, w.sin, c.interleaved));
        }
        TRY(attend(w.qkv, 3 * D, w.qkv + D, 3 * D, w.qkv + 2 * D, 3 * D, T));
        if (c.gated) {
            TRY(gemm_bf16(ctx, st, w.xn, D, b.g1, D, (int)rows, (int)H, (int)D, LTX_EPI_F32, b.g1_b, w.glog, H, nullptr,
                          nullptr, 0));
            CU(head_gate(st, sms, w.att, D, w.glog, H, (int)rows, (int)H, (int)d));
        }
        TRY(gemm_bf16(ctx, st, w.att, D, b.o, D, (int)rows, (int)D, (int)D, LTX_EPI_RESID, b.o_b, w.x, D, tab + 2 * D,
                      w.idx, K * D));
        // cross-attention: x += attn(rms(x), ctx)   [flag path: modulated q, gated, modulated ctx]
        if (c.cross_adaln)
            CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, 1, tab, (int)K, w.idx, 6, w.xn, D));
        else
            CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, 0, nullptr, 0, nullptr, 0, w.xn, D));
        TRY(gemm_bf16(ctx, st, w.xn, D, b.q2, D, (int)rows, (int)D, (int)D, LTX_EPI_BF16, b.q2_b, w.q2, D, nullptr,
                      nullptr, 0));
        CU(qk_norm_rope(st, w.q2, D, (int)rows, (int)D, (int)H, c.eps, b.qn2, nullptr, nullptr, false));
        if (c.cross_adaln) CU(ctx_mod(st, sms, context, crow * Dc, (int)Dc, b.pst, w.ctxb));
        TRY(gemm_bf16(ctx, st, w.ctxb, Dc, b.kv2, Dc, (int)crow, (int)(2 * D), (int)Dc, LTX_EPI_BF16, b.kv2_b, w.kv2,
                      2 * D, nullptr, nullptr, 0, d == 128 ? (int)D : (int)(2 * D)));
        CU(qk_norm_rope(st, w.kv2, 2 * D, (int)crow, (int)D, (int)H, c.eps, b.kn2, nullptr, nullptr, false));
        TRY(attend(w.q2, D, w.kv2, 2 * D, w.kv2 + D, 2 * D, S));
        if (c.gated) {
            TRY(gemm_bf16(ctx, st, w.xn, D, b.g2, D, (int)rows, (int)H, (int)D, LTX_EPI_F32, b.g2_b, w.glog, H, nullptr,
                          nullptr, 0));
            CU(head_gate(st, sms, w.att, D, w.glog, H, (int)rows, (int)H, (int)d));
        }
        TRY(gemm_bf16(ctx, st, w.att, D, b.o2, D, (int)rows, (int)D, (int)D, LTX_EPI_RESID, b.o2_b, w.x, D,
                      c.cross_adaln ? tab + 8 * D : nullptr, c.cross_adaln ? w.idx : nullptr, K * D));
        // feed-forward: x += ff(mod(rms(x))) * gate_mlp
        CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, 1, tab, (int)K, w.idx, 3, w.xn, D));
        TRY(gemm_bf16(ctx, st, w.xn, D, b.ff1, D, (int)rows, (int)(4 * D), (int)D, LTX_EPI_GELU_BF16, b.ff1_b, w.ffh,
                      4 * D, nullptr, nullptr, 0));
        TRY(gemm_bf16(ctx, st, w.ffh, 4 * D, b.ff2, 4 * D, (int)rows, (int)D, (int)(4 * D), LTX_EPI_RESID, b.ff2_b, w.x,
                      D, tab + 5 * D, w.idx, K * D));
    }
    // output head: LN(x) * (1 + scale) + shift -> proj_out (model.rs:237-254)
    CU(norm_mod(st, w.x, D, (int)rows, (int)D, c.eps, 2, w.otab, 2, w.idx, 0, w.xn, D));
    TRY(gemm_bf16(ctx, st, w.xn, D, m->out_w, D, (int)rows, c.out_ch, (int)D, LTX_EPI_F32, m->out_b, out, c.out_ch,
                  nullptr, nullptr, 0));
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
    ltx_model *m = nullptr;
    TRY(alloc_model(ctx, cfg, m));
    int rc = load_weights(m, st, ctx);
    if (rc) {
        cudaFree(m->arena);
        delete m;
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
    TRY(alloc_model(ctx, cfg, m));
    int rc = init_random(m, ctx, seed, lora_rank, lora_strength);
    if (rc) {
        cudaFree(m->arena);
        delete m;
        return rc;
    }
    *out = m;
    return LTX_OK;
}

extern "C" void ltx_model_destroy(ltx_model *m) {
    if (!m) return;
    cudaDeviceSynchronize();
    cudaFree(m->arena);
    delete m;
}

extern "C" int64_t ltx_model_weight_bytes(const ltx_model *m) { return m ? (int64_t)m->arena_bytes : 0; }

extern "C" int ltx_model_forward(ltx_model *m, ltx_ctx *ctx, const float *latent_dev, const float *timesteps_dev,
                                 const float *positions_dev, const float *context_dev, int32_t batch, int32_t tokens,
                                 int32_t context_tokens, float *out_dev) {
    if (!m || !ctx || !latent_dev || !timesteps_dev || !positions_dev || !context_dev || !out_dev)
        return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_model_forward: null argument") : LTX_ERR_INVALID_ARG;
    if (batch <= 0 || tokens <= 0 || context_tokens <= 0)
        return fail(ctx, LTX_ERR_SHAPE, "ltx_model_forward: empty batch/tokens/context");
    std::vector<float> ts((size_t)batch * tokens);
    cudaError_t e = cudaMemcpyAsync(ts.data(), timesteps_dev, ts.size() * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "reading timesteps");
    return forward_impl(m, ctx, latent_dev, ts, positions_dev, context_dev, batch, tokens, context_tokens, out_dev);
}

// One Euler step of euler_denoising_loop (loop_.rs:93-149) with GuidedDenoiser::apply
// (guidance.rs:102-166): the cond and uncond passes run as ONE batch-2 forward.
extern "C" int ltx_denoise_step(ltx_model *m, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                                const float *mask_host, const float *mask_dev, const float *positions_dev,
                                const float *ctx_cond_dev, const float *ctx_uncond_dev, int32_t tokens,
                                int32_t context_tokens, float sigma, float sigma_next, float cfg_scale,
                                float rescale_scale) {
    if (!m || !ctx || !latent_dev || !clean_dev || !mask_dev || !positions_dev || !ctx_cond_dev)
        return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_denoise_step: null argument") : LTX_ERR_INVALID_ARG;
    if (!std::isfinite(sigma) || sigma <= 0.f) return fail(ctx, LTX_ERR_SIGMA, "invalid sigma %g", (double)sigma);
    if (!std::isfinite(sigma_next) || sigma_next < 0.f)
        return fail(ctx, LTX_ERR_SIGMA, "invalid next sigma %g", (double)sigma_next);
    const bool use_cfg = std::fabs(cfg_scale - 1.0f) > 1e-5f;   // needs_uncond (guidance.rs:58-60)
    if (use_cfg && !ctx_uncond_dev) return fail(ctx, LTX_ERR_NEGATIVE_CONTEXT, "cfg_scale != 1 needs a negative context");
    const DitConfig &c = m->cfg;
    const int B = use_cfg ? 2 : 1, T = tokens, S = context_tokens, C = c.in_ch;
    if (c.in_ch != c.out_ch) return fail(ctx, LTX_ERR_CONFIG, "denoise step needs in_channels == out_channels");
    const int64_t D = c.inner(), Dc = c.cross_dim;
    cudaStream_t st = ctx->stream;
    // per-token timesteps = mask * sigma (guidance.rs:114), both CFG halves
    std::vector<float> mask_copy;
    if (!mask_host) {
        mask_copy.resize(T);
        CU(cudaMemcpyAsync(mask_copy.data(), mask_dev, (size_t)T * 4, cudaMemcpyDeviceToHost, st));
        CU(cudaStreamSynchronize(st));
        mask_host = mask_copy.data();
    }
    std::vector<float> ts((size_t)B * T);
    for (int b = 0; b < B; ++b)
        for (int t = 0; t < T; ++t) ts[(size_t)b * T + t] = mask_host[t] * sigma;
    // batch-2 inputs live in the step workspace after the forward's own
    const int64_t rows = (int64_t)B * T;
    std::vector<float> uq;
    std::vector<int> ix;
    const int U = unique_timesteps(ts, uq, ix);
    Work sizing = carve_work(nullptr, c, rows, (int64_t)B * S, U, c.layers);
    const size_t extra = (size_t)rows * C * 4 * 2 + (size_t)B * 3 * T * 2 * 4 + (size_t)B * S * Dc * 4 + 4096;
    TRY(ensure_work(ctx, sizing.bytes + extra));
    Work w = carve_work(static_cast<char *>(ctx->work), c, rows, (int64_t)B * S, U, c.layers);
    char *ex = static_cast<char *>(ctx->work) + ((sizing.bytes + 255) & ~size_t(255));
    float *lat2 = reinterpret_cast<float *>(ex);
    float *vel = lat2 + rows * C;
    float *pos2 = vel + rows * C;
    float *ctx2 = pos2 + (int64_t)B * 3 * T * 2;
    for (int b = 0; b < B; ++b) {
        CU(cudaMemcpyAsync(lat2 + (int64_t)b * T * C, latent_dev, (size_t)T * C * 4, cudaMemcpyDeviceToDevice, st));
        CU(cudaMemcpyAsync(pos2 + (int64_t)b * 3 * T * 2, positions_dev, (size_t)3 * T * 2 * 4, cudaMemcpyDeviceToDevice, st));
        CU(cudaMemcpyAsync(ctx2 + (int64_t)b * S * Dc, b == 0 ? ctx_cond_dev : ctx_uncond_dev, (size_t)S * Dc * 4,
                           cudaMemcpyDeviceToDevice, st));
    }
    TRY(forward_impl(m, ctx, lat2, ts, pos2, ctx2, B, T, S, vel, &w));
    // per-token t for the velocity -> x0 adapter: x0 = x - t * v
    TRY(upload(ctx, w.tok_t, ts.data(), (size_t)T * 4));
    CU(cfg_euler(st, ctx->sm_count, latent_dev, vel, use_cfg ? vel + (int64_t)T * C : vel, w.tok_t, mask_dev, clean_dev,
                 T, C, cfg_scale, rescale_scale, use_cfg, w.partial, sigma, sigma_next));
    (void)D;
    return LTX_OK;
}
