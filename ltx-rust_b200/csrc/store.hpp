// WeightStore: memory-mapped safetensors with the reference's key renaming,
// FP8 `_scale` handling and factored LoRA deltas, read through the
// dequant+merge kernel into device memory.
#pragma once

#include <map>
#include <set>
#include <string>
#include <vector>

#include "internal.hpp"
#include "json.hpp"

struct MappedFile {
    void *base = nullptr;
    size_t size = 0;
    ~MappedFile();
};

struct StoreEntry {
    std::string dtype;             // safetensors dtype string
    std::vector<int64_t> shape;
    const uint8_t *data = nullptr;  // into a mapped file
    size_t nbytes = 0;
};

struct DeviceDelta {
    void *a = nullptr, *b = nullptr;  // device copies in the stored dtype
    int rank = 0, a_dt = 0, b_dt = 0;
    float coeff = 0.f;
    int64_t out = 0, in = 0;
};

struct ltx_store {
    ltx_ctx *ctx = nullptr;
    int device = 0;            // the context's device; destruction does not touch ctx
    std::vector<MappedFile *> files;
    std::map<std::string, StoreEntry> entries;
    std::set<std::string> scale_keys;
    std::map<std::string, std::string> metadata;
    std::map<std::string, std::vector<DeviceDelta>> deltas;
    void *staging = nullptr;   // device bounce buffer for raw tensor bytes
    size_t staging_bytes = 0;
    ~ltx_store();
};

namespace ltx {

int dtype_code(const std::string &s);   // ltx_dtype or -1
int64_t numel(const std::vector<int64_t> &shape);
// WeightStore::read into device memory (dst_dtype F32 or BF16); checks the element count.
int store_read_device(ltx_store *st, const std::string &key, int dst_dtype, void *dst, int64_t expect_numel);
// Decoded scalar (first element) of a small tensor, for `_scale` and `.alpha`.
bool decode_scalar(const StoreEntry &e, float &out);

}  // namespace ltx
