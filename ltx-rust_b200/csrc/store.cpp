// ltx_store_*: the ltx-weights WeightStore / LoraFile / KeyMap seam
// (crates/ltx-weights/src/store.rs:124-640, lora.rs:60-209, key_map.rs:90-111,
// 237-273), with every numeric read done on the GPU by ltx_dequant_merge.
#include "store.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <new>

#include "kernels.hpp"

MappedFile::~MappedFile() {
    if (base && base != MAP_FAILED) munmap(base, size);
}

ltx_store::~ltx_store() {
    cudaSetDevice(device);   // cudaFree synchronises the device before it frees
    for (auto &kv : deltas)
        for (auto &d : kv.second) {
            cudaFree(d.a);
            cudaFree(d.b);
        }
    if (staging) cudaFree(staging);
    for (auto *f : files) delete f;
}

namespace ltx {

int dtype_code(const std::string &s) {
    if (s == "F32") return LTX_F32;
    if (s == "F16") return LTX_F16;
    if (s == "BF16") return LTX_BF16;
    if (s == "F8_E4M3") return LTX_F8_E4M3;
    if (s == "F8_E5M2") return LTX_F8_E5M2;
    return -1;
}

static size_t dtype_bytes(const std::string &s) {
    if (s == "F64" || s == "I64" || s == "U64") return 8;
    if (s == "F32" || s == "I32" || s == "U32") return 4;
    if (s == "F16" || s == "BF16" || s == "I16" || s == "U16") return 2;
    return 1;
}

int64_t numel(const std::vector<int64_t> &shape) {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
}

static bool is_fp8(const std::string &dt) { return dt == "F8_E4M3" || dt == "F8_E5M2"; }

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t bits;
    if (e == 31) bits = sign | 0x7F800000u | (m << 13);
    else if (e == 0) {
        float v = std::ldexp((float)m, -24);
        return sign ? -v : v;
    } else bits = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float fp8_to_f32(uint8_t b, bool e4m3) {
    if (e4m3) {
        if ((b & 0x7F) == 0x7F) return NAN;
        const uint32_t e = (b >> 3) & 0xF, m = b & 7;
        float v = e == 0 ? std::ldexp((float)m, -9) : std::ldexp(1.0f + m / 8.0f, (int)e - 7);
        return (b & 0x80) ? -v : v;
    }
    const uint32_t e = (b >> 2) & 0x1F, m = b & 3;
    float v;
    if (e == 31) v = m ? NAN : INFINITY;
    else v = e == 0 ? std::ldexp((float)m, -16) : std::ldexp(1.0f + m / 4.0f, (int)e - 15);
    return (b & 0x80) ? -v : v;
}

bool decode_scalar(const StoreEntry &e, float &out) {
    // decode_scalar_f32 (store.rs:732-735): first element, 1.0 when empty.
    if (e.nbytes == 0) {
        out = 1.0f;
        return true;
    }
    if (e.dtype == "F32" && e.nbytes >= 4) { memcpy(&out, e.data, 4); return true; }
    if (e.dtype == "BF16" && e.nbytes >= 2) {
        uint32_t v = (uint32_t)(e.data[0] | (e.data[1] << 8)) << 16;
        memcpy(&out, &v, 4);
        return true;
    }
    if (e.dtype == "F16" && e.nbytes >= 2) { out = f16_to_f32((uint16_t)(e.data[0] | (e.data[1] << 8))); return true; }
    if (is_fp8(e.dtype)) { out = fp8_to_f32(e.data[0], e.dtype == "F8_E4M3"); return true; }
    return false;
}

static std::string apply_keymap(int keymap, const std::string &key, bool &keep) {
    keep = true;
    if (keymap == 1) {   // KeyMap::transformer (key_map.rs:101-111)
        static const std::string prefix = "model.diffusion_model.";
        if (key.compare(0, prefix.size(), prefix) != 0) {
            keep = false;
            return key;
        }
        std::string out = key;
        size_t pos;
        while ((pos = out.find(prefix)) != std::string::npos) out.erase(pos, prefix.size());
        return out;
    }
    return key;
}

// Parses one safetensors file into (metadata, name -> entry) without renaming.
static int read_safetensors(ltx_ctx *ctx, const char *path, MappedFile *&mf, std::map<std::string, std::string> &meta,
                            std::vector<std::pair<std::string, StoreEntry>> &tensors) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(ctx, LTX_ERR_IO, "cannot open %s", path);
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        close(fd);
        return fail(ctx, LTX_ERR_FORMAT, "%s: too short for safetensors", path);
    }
    mf = new (std::nothrow) MappedFile();
    if (!mf) {
        close(fd);
        return LTX_ERR_OOM;
    }
    mf->size = (size_t)sb.st_size;
    mf->base = mmap(nullptr, mf->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (mf->base == MAP_FAILED) return fail(ctx, LTX_ERR_IO, "mmap %s failed", path);
    const uint8_t *bytes = static_cast<const uint8_t *>(mf->base);
    uint64_t hlen;
    memcpy(&hlen, bytes, 8);
    if (hlen > mf->size - 8) return fail(ctx, LTX_ERR_FORMAT, "%s: header length %llu out of range", path, (unsigned long long)hlen);
    Json hdr;
    if (!parse_json(std::string(reinterpret_cast<const char *>(bytes + 8), hlen), hdr) || hdr.kind != Json::Obj)
        return fail(ctx, LTX_ERR_FORMAT, "%s: bad safetensors header", path);
    const size_t data_start = 8 + hlen;
    for (auto &kv : hdr.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind == Json::Obj)
                for (auto &m : kv.second.obj)
                    if (m.second.kind == Json::Str) meta.emplace(m.first, m.second.str);
            continue;
        }
        const Json *dt = kv.second.get("dtype"), *sh = kv.second.get("shape"), *off = kv.second.get("data_offsets");
        if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr || !off || off->kind != Json::Arr ||
            off->arr.size() != 2)
            return fail(ctx, LTX_ERR_FORMAT, "%s: bad entry %s", path, kv.first.c_str());
        StoreEntry e;
        e.dtype = dt->str;
        for (auto &d : sh->arr) e.shape.push_back((int64_t)d.num);
        const size_t s = (size_t)off->arr[0].num, t = (size_t)off->arr[1].num;
        if (t < s || data_start + t > mf->size)
            return fail(ctx, LTX_ERR_FORMAT, "%s: tensor %s byte range is outside the file", path, kv.first.c_str());
        e.data = bytes + data_start + s;
        e.nbytes = t - s;
        if (e.nbytes != (size_t)numel(e.shape) * dtype_bytes(e.dtype))
            return fail(ctx, LTX_ERR_SHAPE, "invalid tensor data for key %s: header expects %lld bytes, range has %zu",
                        kv.first.c_str(), (long long)(numel(e.shape) * (int64_t)dtype_bytes(e.dtype)), e.nbytes);
        tensors.emplace_back(kv.first, e);
    }
    return LTX_OK;
}

static int ensure_staging(ltx_store *st, size_t bytes) {
    if (st->staging_bytes >= bytes) return LTX_OK;
    cudaStreamSynchronize(st->ctx->stream);
    if (st->staging) cudaFree(st->staging);
    st->staging = nullptr;
    st->staging_bytes = 0;
    size_t want = std::max<size_t>(bytes, 1 << 20);
    if (cudaMalloc(&st->staging, want) != cudaSuccess) return fail(st->ctx, LTX_ERR_OOM, "staging buffer of %zu bytes", want);
    st->staging_bytes = want;
    return LTX_OK;
}

int store_read_device(ltx_store *st, const std::string &key, int dst_dtype, void *dst, int64_t expect_numel) {
    ltx_ctx *ctx = st->ctx;
    auto it = st->entries.find(key);
    if (it == st->entries.end()) return fail(ctx, LTX_ERR_MISSING_KEY, "missing key: \"%s\"", key.c_str());
    const StoreEntry &e = it->second;
    const int dt = dtype_code(e.dtype);
    if (dt < 0) return fail(ctx, LTX_ERR_DTYPE, "unsupported dtype %s for key \"%s\"", e.dtype.c_str(), key.c_str());
    const int64_t n = numel(e.shape);
    if (expect_numel >= 0 && n != expect_numel)
        return fail(ctx, LTX_ERR_SHAPE, "key \"%s\" has %lld elements, expected %lld", key.c_str(), (long long)n,
                    (long long)expect_numel);
    bool has_scale = false;
    float scale = 1.0f;
    if (is_fp8(e.dtype)) {
        auto sk = st->entries.find(key + "_scale");
        if (sk != st->entries.end()) {
            if (!decode_scalar(sk->second, scale))
                return fail(ctx, LTX_ERR_DTYPE, "unsupported dtype for \"%s_scale\"", key.c_str());
            has_scale = true;
        }
    }
    int rc = ensure_staging(st, e.nbytes);
    if (rc) return rc;
    LTX_CUDA_TRY(ctx, cudaMemcpyAsync(st->staging, e.data, e.nbytes, cudaMemcpyHostToDevice, ctx->stream));
    std::vector<ltx_lora_delta> ds;
    int64_t rows, cols;
    auto dit = st->deltas.find(key);
    if (dit != st->deltas.end() && !dit->second.empty()) {
        rows = dit->second[0].out;
        cols = dit->second[0].in;
        if (rows * cols != n) return fail(ctx, LTX_ERR_SHAPE, "LoRA shape mismatch for key \"%s\"", key.c_str());
        for (auto &d : dit->second) ds.push_back(ltx_lora_delta{d.a, d.b, d.rank, d.a_dt, d.b_dt, d.coeff});
        if (ds.size() > LTX_MAX_DELTAS)
            return fail(ctx, LTX_ERR_UNSUPPORTED, "key \"%s\" has %zu LoRA deltas (max %d)", key.c_str(), ds.size(), LTX_MAX_DELTAS);
    } else {
        cols = e.shape.empty() ? 1 : e.shape.back();
        rows = cols ? n / cols : 0;
    }
    return dequant_merge(ctx, ctx->stream, st->staging, dt, has_scale, scale, rows, cols, ds.data(), (int)ds.size(), dst,
                         dst_dtype);
}

}  // namespace ltx

using namespace ltx;

extern "C" int ltx_store_open(ltx_ctx *ctx, const char *const *paths, int32_t n_paths, int32_t keymap,
                              ltx_store **out) {
    if (!ctx || !out || (n_paths > 0 && !paths) || n_paths < 0 || keymap < 0 || keymap > 1)
        return ctx ? fail(ctx, LTX_ERR_INVALID_ARG, "ltx_store_open: bad arguments") : LTX_ERR_INVALID_ARG;
    *out = nullptr;
    ltx_store *st = new (std::nothrow) ltx_store();
    if (!st) return LTX_ERR_OOM;
    st->ctx = ctx;
    st->device = ctx->device;
    for (int i = 0; i < n_paths; ++i) {
        MappedFile *mf = nullptr;
        std::map<std::string, std::string> meta;
        std::vector<std::pair<std::string, StoreEntry>> tensors;
        int rc = read_safetensors(ctx, paths[i], mf, meta, tensors);
        if (mf) st->files.push_back(mf);
        if (rc) {
            delete st;
            return rc;
        }
        for (auto &m : meta) st->metadata.emplace(m.first, m.second);   // first file wins
        for (auto &t : tensors) {
            bool keep;
            std::string renamed = apply_keymap(keymap, t.first, keep);
            if (!keep) continue;
            if (st->entries.count(renamed)) {
                fail(ctx, LTX_ERR_DUPLICATE_KEY, "duplicate key \"%s\" across checkpoint files", renamed.c_str());
                delete st;
                return LTX_ERR_DUPLICATE_KEY;
            }
            st->entries.emplace(renamed, t.second);
        }
    }
    // store.rs:174-187: `{key}_scale` of an FP8 tensor is internal.
    for (auto &kv : st->entries) {
        const std::string &k = kv.first;
        if (k.size() > 6 && k.compare(k.size() - 6, 6, "_scale") == 0) {
            auto base = st->entries.find(k.substr(0, k.size() - 6));
            if (base != st->entries.end() && is_fp8(base->second.dtype)) st->scale_keys.insert(k);
        }
    }
    *out = st;
    return LTX_OK;
}

extern "C" void ltx_store_destroy(ltx_store *st) {
    if (!st) return;
    delete st;
}

extern "C" int ltx_store_contains(const ltx_store *st, const char *key) {
    if (!st || !key) return 0;
    return st->entries.count(key) && !st->scale_keys.count(key);
}

extern "C" int32_t ltx_store_num_keys(const ltx_store *st) {
    if (!st) return 0;
    return (int32_t)(st->entries.size() - st->scale_keys.size());
}

extern "C" const char *ltx_store_key(const ltx_store *st, int32_t index) {
    if (!st || index < 0) return nullptr;
    int32_t i = 0;
    for (auto &kv : st->entries) {
        if (st->scale_keys.count(kv.first)) continue;
        if (i++ == index) return kv.first.c_str();
    }
    return nullptr;
}

extern "C" int ltx_store_shape(ltx_store *st, const char *key, int64_t *dims, int32_t max_dims, int32_t *ndim,
                               int32_t *dtype) {
    if (!st || !key || !ndim) return LTX_ERR_INVALID_ARG;
    auto it = st->entries.find(key);
    if (it == st->entries.end()) return fail(st->ctx, LTX_ERR_MISSING_KEY, "missing key: \"%s\"", key);
    *ndim = (int32_t)it->second.shape.size();
    for (int32_t i = 0; i < *ndim && i < max_dims && dims; ++i) dims[i] = it->second.shape[i];
    if (dtype) *dtype = dtype_code(it->second.dtype);
    return LTX_OK;
}

extern "C" int ltx_store_metadata(const ltx_store *st, const char *key, char *buf, size_t buf_len, size_t *needed) {
    if (!st || !key) return LTX_ERR_INVALID_ARG;
    auto it = st->metadata.find(key);
    if (it == st->metadata.end()) return std::string(key) == "config" ? LTX_ERR_MISSING_CONFIG : LTX_ERR_MISSING_KEY;
    if (needed) *needed = it->second.size() + 1;
    if (buf && buf_len) {
        size_t n = std::min(buf_len - 1, it->second.size());
        memcpy(buf, it->second.data(), n);
        buf[n] = 0;
    }
    return LTX_OK;
}

extern "C" int ltx_store_read(ltx_store *st, const char *key, int32_t dst_dtype, void *dst_dev, size_t dst_bytes) {
    if (!st || !key || !dst_dev) return LTX_ERR_INVALID_ARG;
    auto it = st->entries.find(key);
    if (it == st->entries.end()) return fail(st->ctx, LTX_ERR_MISSING_KEY, "missing key: \"%s\"", key);
    const int64_t n = numel(it->second.shape);
    if (dst_dtype != LTX_F32 && dst_dtype != LTX_BF16)
        return fail(st->ctx, LTX_ERR_DTYPE, "ltx_store_read: output dtype must be F32 or BF16");
    if ((size_t)n * dtype_size(dst_dtype) > dst_bytes)
        return fail(st->ctx, LTX_ERR_SHAPE, "ltx_store_read: %zu-byte buffer for %lld elements", dst_bytes, (long long)n);
    return store_read_device(st, key, dst_dtype, dst_dev, n);
}

// WeightStore::merge_lora (store.rs:542-640) with LoraFile (lora.rs:60-209).
extern "C" int ltx_store_merge_lora(ltx_store *st, const char *lora_path, float strength, int32_t *n_matched,
                                    int32_t *n_unmatched) {
    if (!st || !lora_path) return LTX_ERR_INVALID_ARG;
    ltx_ctx *ctx = st->ctx;
    MappedFile *mf = nullptr;
    std::map<std::string, std::string> meta;
    std::vector<std::pair<std::string, StoreEntry>> tensors;
    int rc = read_safetensors(ctx, lora_path, mf, meta, tensors);
    if (rc) {
        delete mf;
        return rc;
    }
    std::map<std::string, StoreEntry> lora(tensors.begin(), tensors.end());
    static const std::string suffix = ".lora_A.weight";
    std::vector<std::pair<std::string, DeviceDelta>> pending;
    int matched = 0, unmatched = 0;
    auto cleanup = [&]() {
        for (auto &p : pending) {
            cudaFree(p.second.a);
            cudaFree(p.second.b);
        }
        delete mf;
    };
    for (auto &kv : lora) {
        const std::string &key_a = kv.first;
        if (key_a.size() <= suffix.size() || key_a.compare(key_a.size() - suffix.size(), suffix.size(), suffix) != 0)
            continue;
        const std::string prefix = key_a.substr(0, key_a.size() - suffix.size());
        const std::string base_key = prefix + ".weight", key_b = prefix + ".lora_B.weight";
        auto base = st->entries.find(base_key);
        auto kb = lora.find(key_b);
        if (base == st->entries.end() || kb == lora.end()) {
            ++unmatched;
            continue;
        }
        const StoreEntry &ea = kv.second, &eb = kb->second;
        const int adt = dtype_code(ea.dtype), bdt = dtype_code(eb.dtype);
        if (adt < 0 || bdt < 0) {
            cleanup();
            return fail(ctx, LTX_ERR_DTYPE, "unsupported dtype %s for key \"%s\"", (adt < 0 ? ea : eb).dtype.c_str(),
                        (adt < 0 ? key_a : key_b).c_str());
        }
        const int64_t rank_a = ea.shape.empty() ? 0 : ea.shape[0];
        const int64_t rank_b = eb.shape.size() > 1 ? eb.shape[1] : 0;
        if (rank_a != rank_b || rank_a == 0) {
            cleanup();
            return fail(ctx, LTX_ERR_LORA_RANK, "LoRA inner rank mismatch for key \"%s\": A inner %lld, B inner %lld",
                        base_key.c_str(), (long long)rank_a, (long long)rank_b);
        }
        const auto &bs = base->second.shape;
        const int64_t out_f = bs.empty() ? 0 : bs[0], in_f = bs.size() > 1 ? bs[1] : 1;
        const int64_t b_out = eb.shape.empty() ? 0 : eb.shape[0], a_in = ea.shape.size() > 1 ? ea.shape[1] : 0;
        if (b_out != out_f || a_in != in_f) {
            cleanup();
            return fail(ctx, LTX_ERR_SHAPE, "LoRA shape mismatch for key \"%s\"", base_key.c_str());
        }
        // alpha defaults to the rank (store.rs:605-612); coeff = fma(strength, alpha / rank, 0) (:615)
        float alpha = (float)rank_a;
        auto ka = lora.find(prefix + ".alpha");
        if (ka != lora.end()) {
            float v;
            if (decode_scalar(ka->second, v)) alpha = v;
        }
        DeviceDelta d;
        d.rank = (int)rank_a;
        d.a_dt = adt;
        d.b_dt = bdt;
        d.coeff = ltx_lora_coeff(strength, alpha, (int32_t)rank_a);
        d.out = out_f;
        d.in = in_f;
        if (cudaMalloc(&d.a, std::max<size_t>(ea.nbytes, 16)) != cudaSuccess ||
            cudaMalloc(&d.b, std::max<size_t>(eb.nbytes, 16)) != cudaSuccess) {
            cudaFree(d.a);
            cleanup();
            return fail(ctx, LTX_ERR_OOM, "LoRA factor upload");
        }
        cudaMemcpyAsync(d.a, ea.data, ea.nbytes, cudaMemcpyHostToDevice, ctx->stream);
        cudaMemcpyAsync(d.b, eb.data, eb.nbytes, cudaMemcpyHostToDevice, ctx->stream);
        pending.emplace_back(base_key, d);
        ++matched;
    }
    if (matched == 0 && unmatched > 0) {
        cleanup();
        return fail(ctx, LTX_ERR_NO_LORA_MATCHES, "LoRA file did not match any base weight keys");
    }
    cudaStreamSynchronize(ctx->stream);   // the mapped LoRA file is released below
    for (auto &p : pending) st->deltas[p.first].push_back(p.second);
    pending.clear();
    delete mf;
    if (n_matched) *n_matched = matched;
    if (n_unmatched) *n_unmatched = unmatched;
    return LTX_OK;
}
