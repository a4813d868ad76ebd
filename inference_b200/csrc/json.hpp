// json.hpp -- a small JSON reader for host code (safetensors headers,
// tokenizer.json): objects keep their keys in file order, numbers are
// doubles, strings are UTF-8 (\u escapes, surrogate pairs included, are
// re-encoded).  Nesting is limited to 64 levels.
#pragma once

#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace q3 {

// Code point v as UTF-8.
inline void append_utf8(std::string& out, unsigned v) {
    if (v < 0x80) {
        out += static_cast<char>(v);
    } else if (v < 0x800) {
        out += static_cast<char>(0xC0 | (v >> 6));
        out += static_cast<char>(0x80 | (v & 0x3F));
    } else if (v < 0x10000) {
        out += static_cast<char>(0xE0 | (v >> 12));
        out += static_cast<char>(0x80 | ((v >> 6) & 0x3F));
        out += static_cast<char>(0x80 | (v & 0x3F));
    } else {
        out += static_cast<char>(0xF0 | (v >> 18));
        out += static_cast<char>(0x80 | ((v >> 12) & 0x3F));
        out += static_cast<char>(0x80 | ((v >> 6) & 0x3F));
        out += static_cast<char>(0x80 | (v & 0x3F));
    }
}

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json* get(const std::string& k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct Parser {
    const char* p;
    const char* end;
    std::string err;
    int depth = 0;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    bool hex4(const char* q, unsigned& v) const {
        if (end - q < 4) return false;
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = q[i];
            const int d = c >= '0' && c <= '9' ? c - '0' : c >= 'a' && c <= 'f' ? c - 'a' + 10
                          : c >= 'A' && c <= 'F' ? c - 'A' + 10 : -1;
            if (d < 0) return false;
            v = v * 16 + static_cast<unsigned>(d);
        }
        return true;
    }
    bool string(std::string& out) {
        if (p >= end || *p != '"') return fail("expected a string");
        ++p;
        while (p < end && *p != '"') {
            if (*p == '\\') {
                if (++p >= end) return fail("bad escape");
                switch (*p) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        unsigned v = 0;
                        if (!hex4(p + 1, v)) return fail("bad \\u escape");
                        p += 4;
                        // a UTF-16 surrogate pair spells one code point above U+FFFF
                        if (v >= 0xD800 && v < 0xDC00 && end - p >= 7 && p[1] == '\\' && p[2] == 'u') {
                            unsigned lo = 0;
                            if (hex4(p + 3, lo) && lo >= 0xDC00 && lo < 0xE000) {
                                v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
                                p += 6;
                            }
                        }
                        append_utf8(out, v);
                        break;
                    }
                    default: return fail("bad escape");
                }
                ++p;
            } else {
                out += *p++;
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(Json& v) {
        if (++depth > 64) return fail("nesting too deep");
        ws();
        if (p >= end) return fail("unexpected end");
        bool ok = true;
        if (*p == '{') {
            v.kind = Json::Obj;
            ++p;
            ws();
            if (p < end && *p == '}') {
                ++p;
            } else {
                while (ok) {
                    ws();
                    std::string k;
                    Json c;
                    ok = string(k);
                    ws();
                    if (ok && (p >= end || *p++ != ':')) ok = fail("expected ':'");
                    ok = ok && value(c);
                    if (ok) v.obj.emplace_back(std::move(k), std::move(c));
                    ws();
                    if (ok && p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (ok && (p >= end || *p++ != '}')) ok = fail("expected '}'");
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = Json::Arr;
            ++p;
            ws();
            if (p < end && *p == ']') {
                ++p;
            } else {
                while (ok) {
                    Json c;
                    ok = value(c);
                    if (ok) v.arr.push_back(std::move(c));
                    ws();
                    if (ok && p < end && *p == ',') {
                        ++p;
                        continue;
                    }
                    if (ok && (p >= end || *p++ != ']')) ok = fail("expected ']'");
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = Json::Str;
            ok = string(v.str);
        } else if (end - p >= 4 && !std::strncmp(p, "true", 4)) {
            v.kind = Json::Bool, v.b = true, p += 4;
        } else if (end - p >= 5 && !std::strncmp(p, "false", 5)) {
            v.kind = Json::Bool, p += 5;
        } else if (end - p >= 4 && !std::strncmp(p, "null", 4)) {
            p += 4;
        } else {
            v.kind = Json::Num;
            const char* s = p;
            while (p < end && (std::strchr("+-.eE", *p) || (*p >= '0' && *p <= '9'))) ++p;
            if (p == s) return fail("unexpected character");
            v.num = std::strtod(std::string(s, p).c_str(), nullptr);
        }
        --depth;
        return ok;
    }
};

inline bool parse_json(const char* s, size_t n, Json& out, std::string& err) {
    Parser ps{s, s + n, {}};
    if (!ps.value(out)) {
        err = ps.err;
        return false;
    }
    ps.ws();
    if (ps.p != ps.end) {
        err = "trailing characters";
        return false;
    }
    return true;
}

}  // namespace q3
