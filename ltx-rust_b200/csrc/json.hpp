// Minimal JSON reader for safetensors headers and the DiT config
// (objects, arrays, strings with escapes, numbers, true/false/null).
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace ltx {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;   // keeps file order

    const Json *get(const std::string &k) const {
        if (kind != Obj) return nullptr;
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
  public:
    JsonParser(const char *s, size_t n) : p_(s), end_(s + n) {}
    bool parse(Json &out) {
        ws();
        if (!value(out)) return false;
        ws();
        return p_ == end_;
    }

  private:
    const char *p_, *end_;
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool lit(const char *w) {
        size_t n = 0;
        while (w[n]) ++n;
        if ((size_t)(end_ - p_) < n) return false;
        for (size_t i = 0; i < n; ++i)
            if (p_[i] != w[i]) return false;
        p_ += n;
        return true;
    }
    bool string(std::string &s) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c == '\\') {
                if (p_ >= end_) return false;
                char e = *p_++;
                switch (e) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    if (end_ - p_ < 4) return false;
                    unsigned v = (unsigned)strtoul(std::string(p_, 4).c_str(), nullptr, 16);
                    p_ += 4;
                    if (v < 0x80) s += (char)v;
                    else if (v < 0x800) { s += (char)(0xC0 | (v >> 6)); s += (char)(0x80 | (v & 0x3F)); }
                    else { s += (char)(0xE0 | (v >> 12)); s += (char)(0x80 | ((v >> 6) & 0x3F)); s += (char)(0x80 | (v & 0x3F)); }
                    break;
                }
                default: return false;
                }
            } else {
                s += c;
            }
        }
        if (p_ >= end_) return false;
        ++p_;
        return true;
    }
    bool value(Json &v) {
        ws();
        if (p_ >= end_) return false;
        char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = Json::Obj;
            ws();
            if (p_ < end_ && *p_ == '}') { ++p_; return true; }
            while (true) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                Json child;
                if (!value(child)) return false;
                v.obj.emplace_back(std::move(k), std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == '}') { ++p_; return true; }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v.kind = Json::Arr;
            ws();
            if (p_ < end_ && *p_ == ']') { ++p_; return true; }
            while (true) {
                Json child;
                if (!value(child)) return false;
                v.arr.push_back(std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') { ++p_; continue; }
                if (p_ < end_ && *p_ == ']') { ++p_; return true; }
                return false;
            }
        }
        if (c == '"') {
            v.kind = Json::Str;
            return string(v.str);
        }
        if (lit("true")) { v.kind = Json::Bool; v.b = true; return true; }
        if (lit("false")) { v.kind = Json::Bool; v.b = false; return true; }
        if (lit("null")) { v.kind = Json::Null; return true; }
        char *e = nullptr;
        std::string tmp(p_, std::min<size_t>(64, end_ - p_));
        v.num = strtod(tmp.c_str(), &e);
        if (e == tmp.c_str()) return false;
        p_ += (e - tmp.c_str());
        v.kind = Json::Num;
        return true;
    }
};

inline bool parse_json(const std::string &s, Json &out) {
    JsonParser p(s.data(), s.size());
    return p.parse(out);
}

}  // namespace ltx
